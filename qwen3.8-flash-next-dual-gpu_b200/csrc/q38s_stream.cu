// Streaming row sampler for sm_100a: the hot path of every prepare /
// sample-commit / speculative-verification / vocab-shard call.
//
// Work decomposition.  Each virtual row (a batch row, or one target / draft
// row of a speculative verification) is split into `segs` column segments
// (whole 128-column blocks).  A unit is one (row, segment) pair; a persistent
// grid of at most two CTAs per SM walks the units (CTA b takes units b,
// b + G, b + 2G, ...).  Large batches use one segment per row, so every row
// is streamed start to finish by one CTA; small batches split rows so the
// whole GPU pulls HBM.  The last segment of a row to finish (a ticket per
// row, reset by that CTA) merges the segments' candidate lists.  No CTA ever
// waits for another.
//
// Inside a CTA.  Warp 8 is a producer: one lane streams the CTA's tiles
// (16 KB of logits each, plus the matching 1 KB slice of the row's penalty
// bitmap when the row has penalties) through a ring of four shared-memory
// slots with 1-D TMA bulk copies (no multicast), completion on a `full`
// mbarrier per slot.  Warps 0-7 consume: they release a slot on its `empty`
// mbarrier as soon as they have read it, so copies for the next tiles (and
// the next unit) stay in flight while the consumers do per-row serial work.
//
// Per unit the consumers
//   seed    take each thread's largest raw logit of the first tile, evaluate
//           it exactly, and derive theta: the k-th largest of those 256
//           values (a lower bound of the row's k-th largest value) and, for
//           min-p rows, M + ln(min_p) - slack (M = the largest exact value
//           seen, a lower bound of the row maximum);
//   filter  one packed bf16x2 (or f32) maximum over the thread's 32 (16)
//           logits of a tile is compared with theta's raw-logit bound; only
//           hits get the reference's exact penalty / temperature arithmetic
//           (sampling.cc:76-92) and enter a shared-memory buffer as 64-bit
//           rank keys (value desc, token asc).  theta rises with the running
//           maximum (min-p) and by exact compaction of the buffer;
//   finish  exact top-k and min-p cuts of the buffer, a sort, then the
//           reference's softmax / top-p / draw (sampling.cc:105-145) in
//           double precision with its sequential summation order.
// Rows whose candidate sets do not fit (top_k = 0 without min-p, top_k > 256
// without min-p, mass ties) take the CTA's general path: exact keys of every
// column in global scratch, radix selection of the top-k / min-p cut, and
// either an exact gather (kept sets up to 1,024) or a fixed-point
// mass-weighted selection of the top-p cut and the draw.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdlib>

#include "q38s_kernels.cuh"

namespace q38s {
namespace {

constexpr uint32_t kTileBytes = 16384;           // logits per ring slot
constexpr uint32_t kTileBm = 1024;               // bitmap bytes per slot (8,192 columns)
constexpr uint32_t kSlot = kTileBytes + kTileBm;
constexpr uint32_t kRing = 4;                    // ring slots per CTA
constexpr int kCons = 256;                       // consumer threads (warps 0-7)
constexpr int kBlock = kCons + 64;               // + the producer and the evaluator warp
constexpr uint32_t kBuf = 2048;                  // candidate buffer (rank keys)
constexpr uint32_t kQ = 512;                     // raw-candidate queue (entries)
constexpr uint32_t kFinal = kSegCap;             // candidates entering the epilogue
constexpr uint32_t kGather = 1024;               // exact gather of the general path
constexpr uint32_t kArea = 32768;                // candidate / epilogue work area
constexpr double kFix = 8796093022208.0;         // 2^43: fixed-point weight unit

constexpr uint32_t kPosInfKey = 0xff800000u;      // float_key(+inf)
constexpr uint32_t kFOverflow = 1u;
constexpr uint32_t kFInf = 2u;
constexpr uint32_t kFTimeout = 4u;

static_assert(kBuf * 8 + kFinal * 8 + 3 * kFinal * 8 <= kArea, "fast-path area");
static_assert(kQ <= 4 * kFinal, "the queue shares the epilogue's part of the area");

// Optional per-unit trace (build with -DQ38S_TRACE; off in the product
// build): 16 words per unit -- global-timer stamps of the unit's phases, its
// threshold, candidate count, flags and the path that finished it.  The
// buffer is installed with q38s_trace_install().
#ifdef Q38S_TRACE
__device__ unsigned long long* g_trace = nullptr;
__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
#define Q38S_TR(u, slot, val)                                                     \
    do {                                                                          \
        if (g_trace && threadIdx.x == 0 && (u) < 8192)                            \
            g_trace[static_cast<size_t>(u) * 16 + (slot)] =                       \
                static_cast<unsigned long long>(val);                             \
    } while (0)
#define Q38S_TT(u, slot) Q38S_TR(u, slot, gtime())
#else
#define Q38S_TR(u, slot, val) do { } while (0)
#define Q38S_TT(u, slot) do { } while (0)
#endif
static_assert(kGather * 32 <= kArea, "general-path area");

struct __align__(16) Ctl {
    uint64_t full[kRing];
    uint64_t empty[kRing];
    uint32_t abort_flag;   // set by whichever side gave up waiting
    uint32_t prod_done;    // producer left its loop
    uint32_t issued;       // tiles issued by the producer
    uint32_t n_cand;
    uint32_t flags;
    uint32_t mrun;         // the seed's largest exact key
    uint32_t theta_pub;    // the unit's threshold: value keys below it are never kept
    uint32_t fail_g;       // first tile a consumer warp gave up waiting for
    uint32_t q_head;       // queue entries reserved by the consumers (running count)
    uint32_t q_tail;       // queue entries the evaluator has taken (running count)
    uint32_t cons_done;    // consumer warps that finished their units' tiles (running count)
#ifdef Q38S_TRACE
    unsigned long long tr_qwait;  // consumer cycles spent waiting for queue room
#endif
    uint32_t bc_u32[4];
    uint64_t bc_u64[2];
    uint32_t red_u32[kCons / 32];
    uint64_t red_u64[kCons / 32];
    uint32_t hist[256];
    uint64_t hmass[256];
    uint32_t tkey[kCons];
    int32_t e_token;
    int32_t e_status;
    uint32_t e_n;
    uint32_t e_r;
    double e_total;
    double e_draw;
};

// ------------------------------------------------------ consumer barriers
// Named barrier 1 spans exactly the 256 consumer threads; the producer warp
// never takes part.
__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
__device__ __forceinline__ bool cbar_or(bool p) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred q, s;\n setp.ne.u32 q, %1, 0;\n"
        " bar.red.or.pred s, 1, 256, q;\n selp.u32 %0, 1, 0, s;\n}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(p))
        : "memory");
    return r != 0;
}
// Number of consumer threads with p set (a barrier for all of them).
__device__ __forceinline__ uint32_t cbar_count(bool p) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred q;\n setp.ne.u32 q, %1, 0;\n"
        " bar.red.popc.u32 %0, 1, 256, q;\n}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(p))
        : "memory");
    return r;
}
// Named barrier 2 spans the consumers and the evaluator warp (288
// threads): the start and the end of every unit.
__device__ __forceinline__ void ebar() { asm volatile("bar.sync 2, 288;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Block reductions over the consumers.  The leading barrier keeps a
// reduction from overwriting red_* while the previous one is still read.
__device__ uint32_t cmax_u32(uint32_t v, Ctl& c) {
    v = warp_max_u32(v);
    cbar();
    if ((threadIdx.x & 31) == 0) c.red_u32[threadIdx.x >> 5] = v;
    cbar();
    uint32_t r = c.red_u32[0];
    for (int i = 1; i < kCons / 32; ++i) r = max(r, c.red_u32[i]);
    return r;
}
__device__ uint32_t cmin_u32(uint32_t v, Ctl& c) {
    v = warp_min_u32(v);
    cbar();
    if ((threadIdx.x & 31) == 0) c.red_u32[threadIdx.x >> 5] = v;
    cbar();
    uint32_t r = c.red_u32[0];
    for (int i = 1; i < kCons / 32; ++i) r = min(r, c.red_u32[i]);
    return r;
}
__device__ uint32_t cor_u32(uint32_t v, Ctl& c) {
    for (int o = 16; o > 0; o >>= 1) v |= __shfl_xor_sync(0xffffffffu, v, o);
    cbar();
    if ((threadIdx.x & 31) == 0) c.red_u32[threadIdx.x >> 5] = v;
    cbar();
    uint32_t r = 0;
    for (int i = 0; i < kCons / 32; ++i) r |= c.red_u32[i];
    return r;
}
__device__ uint32_t csum_u32(uint32_t v, Ctl& c) {
    v = warp_sum_u32(v);
    cbar();
    if ((threadIdx.x & 31) == 0) c.red_u32[threadIdx.x >> 5] = v;
    cbar();
    uint32_t r = 0;
    for (int i = 0; i < kCons / 32; ++i) r += c.red_u32[i];
    return r;
}
__device__ uint64_t csum_u64(uint64_t v, Ctl& c) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    cbar();
    if ((threadIdx.x & 31) == 0) c.red_u64[threadIdx.x >> 5] = v;
    cbar();
    uint64_t r = 0;
    for (int i = 0; i < kCons / 32; ++i) r += c.red_u64[i];
    return r;
}
// Exclusive prefix sum over the consumers in thread order; *total gets the sum.
__device__ uint32_t cscan_excl(uint32_t v, uint32_t* total, Ctl& c) {
    const uint32_t lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    uint32_t inc = v;
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= static_cast<uint32_t>(o)) inc += y;
    }
    cbar();
    if (lane == 31) c.red_u32[w] = inc;
    cbar();
    uint32_t before = 0, all = 0;
    for (uint32_t i = 0; i < kCons / 32; ++i) {
        const uint32_t x = c.red_u32[i];
        if (i < w) before += x;
        all += x;
    }
    *total = all;
    return before + inc - v;
}

// ------------------------------------------------------------ row context
struct Row {
    uint32_t v;           // virtual row
    uint32_t srow;        // state row
    RowParams p;
    RowState st;          // the state row as of the launch
    uint64_t rng_before;
    uint32_t k_eff;       // 0: no top-k truncation
    bool pen, nonmono, freq, minp;
    const uint32_t* gbm;  // the state row's penalty bitmap
    const uint32_t* counts_row;
    const int32_t* extra; // additional penalty tokens (global token ids)
    uint32_t n_extra;
    double lnmp;          // log(min_p) for min-p rows
};

__device__ __forceinline__ uint32_t state_row(const SampleArgs& a, uint32_t v) {
    return a.vrow_state_const != ~0u ? a.vrow_state_const : v;
}

__device__ void load_row(const SampleArgs& a, uint32_t v, Row& r) {
    r.v = v;
    r.srow = state_row(a, v);
    r.p = a.params[r.srow];
    const uint32_t off = v < a.split ? v : v - a.split;
    r.st = a.state[r.srow];
    r.rng_before = r.st.rng_state + (a.rng_step ? static_cast<uint64_t>(off) * kGamma : 0ull);
    r.pen = (r.p.flags & kFlagPenalties) != 0;
    r.nonmono = (r.p.flags & kFlagNonMonotone) != 0;
    r.freq = (r.p.flags & kFlagFrequency) != 0;
    r.minp = a.mode != kModeShardTopK && r.p.min_p > 0.0f;
    r.lnmp = r.minp ? log(static_cast<double>(r.p.min_p)) : 0.0;
    r.gbm = a.bitmap + static_cast<size_t>(r.srow) * a.bitmap_words;
    r.counts_row = a.counts ? a.counts + static_cast<size_t>(r.srow) * a.vocab : nullptr;
    r.extra = nullptr;
    r.n_extra = 0;
    if (a.extra_mode == 1) {
        r.extra = a.extra_tokens + a.extra_offsets[v];
        r.n_extra = a.extra_offsets[v + 1] - a.extra_offsets[v];
    } else if (a.extra_mode == 2) {
        r.extra = a.extra_tokens;
        r.n_extra = off;
    }
    if (a.mode == kModeShardTopK) r.k_eff = a.k_out >= a.vocab ? 0u : a.k_out;
    else r.k_eff = (r.p.top_k == 0 || r.p.top_k >= a.full_vocab) ? 0u : r.p.top_k;
}

// Occurrences of global token `tok` among this call's additional tokens.
__device__ __forceinline__ uint64_t extra_count(const Row& r, uint32_t tok) {
    uint64_t n = 0;
    for (uint32_t e = 0; e < r.n_extra; ++e) n += static_cast<uint32_t>(r.extra[e]) == tok;
    return n;
}

template <int DT>
__device__ __forceinline__ const unsigned char* row_ptr(const SampleArgs& a, uint32_t v) {
    constexpr uint32_t es = DT == Q38S_DTYPE_BF16 ? 2u : 4u;
    return v < a.split
        ? static_cast<const unsigned char*>(a.logits) + static_cast<size_t>(v) * a.row_stride * es
        : static_cast<const unsigned char*>(a.logits2) +
              static_cast<size_t>(v - a.split) * a.row_stride * es;
}

template <int DT>
__device__ __forceinline__ float load_elem(const unsigned char* base, uint32_t j) {
    if (DT == Q38S_DTYPE_BF16)
        return __uint_as_float(static_cast<uint32_t>(
                                   reinterpret_cast<const uint16_t*>(base)[j]) << 16);
    return reinterpret_cast<const float*>(base)[j];
}

// Element e of a 16-byte vector (e is a compile-time constant after unrolling).
template <int DT>
__device__ __forceinline__ float vec_elem(const uint4& w, int e) {
    if (DT == Q38S_DTYPE_BF16) {
        const uint32_t word = e < 2 ? w.x : e < 4 ? w.y : e < 6 ? w.z : w.w;
        return (e & 1) ? bf16_hi(word) : bf16_lo(word);
    }
    return __uint_as_float(e == 0 ? w.x : e == 1 ? w.y : e == 2 ? w.z : w.w);
}

template <int DT>
__device__ __forceinline__ float vec_max(const uint4& w) {
    if (DT == Q38S_DTYPE_BF16) {
        const __nv_bfloat162 m =
            __hmax2(__hmax2(*reinterpret_cast<const __nv_bfloat162*>(&w.x),
                            *reinterpret_cast<const __nv_bfloat162*>(&w.y)),
                    __hmax2(*reinterpret_cast<const __nv_bfloat162*>(&w.z),
                            *reinterpret_cast<const __nv_bfloat162*>(&w.w)));
        return fmaxf(__low2float(m), __high2float(m));
    }
    return fmaxf(fmaxf(__uint_as_float(w.x), __uint_as_float(w.y)),
                 fmaxf(__uint_as_float(w.z), __uint_as_float(w.w)));
}

// Exact transformed value of a tile element (sampling.cc:76-92): the
// penalised bit comes from the slot's bitmap copy (which carries this
// call's additional tokens), the frequency count from global memory.  One
// out-of-line copy of the IEEE division sequences keeps them out of the
// unrolled streaming loop, so a warp that takes this (rare) path does not
// miss in the instruction cache.
__device__ __noinline__ float exact_value(float x, bool penalized, uint64_t count, RowParams p) {
    return transform(x, penalized, count, p);
}
__device__ __forceinline__ float eval_slot(const Row& r, const uint32_t* bm, float x, uint32_t idx,
                                           uint32_t col, uint32_t tok) {
    bool penalized = false;
    uint64_t count = 1;
    if (r.pen) {
        penalized = (bm[idx >> 5] >> (idx & 31)) & 1u;
        if (penalized && r.freq)
            count = (r.counts_row ? r.counts_row[col] : 0u) + extra_count(r, tok);
    }
    return exact_value(x, penalized, count, r.p);
}

// Lower bound of the smallest value v with exp(v - m) >= min_p, for any
// m' >= m (sampling.cc:112-113 weights; the extension's min-p cut): m +
// ln(min_p) less a slack that covers the rounding of v - m and of exp.
__device__ __forceinline__ uint32_t minp_key(uint32_t mkey, const Row& r) {
    if (mkey <= kNegInfKey) return 0;
    const float m = key_float(mkey);
    if (!isfinite(m)) return 0;
    const double slack = (fabs(static_cast<double>(m)) + fabs(r.lnmp)) * 0x1p-18 + 1e-30;
    return float_key(__double2float_rd(static_cast<double>(m) + r.lnmp - slack));
}

// ---------------------------------------------------------------- selects
// Scan of 256 descending bins by warp 0: first bin at which the running
// count reaches `need`.  Writes bin (or ~0u) and the count above it.
__device__ __forceinline__ void find_bin_desc(const uint32_t* hist, uint32_t need, Ctl& c) {
    if (threadIdx.x < 32) {
        const uint32_t lane = threadIdx.x;
        uint32_t s = 0;
        for (int b = 0; b < 8; ++b) s += hist[255 - 8 * lane - b];
        uint32_t inc = s;
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= static_cast<uint32_t>(o)) inc += y;
        }
        const uint32_t hit = __ballot_sync(0xffffffffu, inc >= need);
        if (lane == 0) c.bc_u32[0] = 0xffffffffu;
        __syncwarp();
        if (hit && lane == static_cast<uint32_t>(__ffs(hit) - 1)) {
            uint32_t acc = inc - s;
            for (int b = 0; b < 8; ++b) {
                const uint32_t bin = 255 - 8 * lane - b;
                acc += hist[bin];
                if (acc >= need) {
                    c.bc_u32[0] = bin;
                    c.bc_u32[1] = acc - hist[bin];
                    break;
                }
            }
        }
    }
}

// Warp-aggregated histogram increment: lanes that share a bin add once, so
// skewed key distributions do not serialise on one shared-memory word.  The
// whole warp calls it; `active` marks the lanes that count.
__device__ __forceinline__ void hist_inc(uint32_t* hist, uint32_t bin, bool active) {
    const uint32_t act = __ballot_sync(0xffffffffu, active);
    if (active) {
        const uint32_t peers = __match_any_sync(act, bin);
        if ((threadIdx.x & 31) == static_cast<uint32_t>(__ffs(peers) - 1))
            atomicAdd(&hist[bin], static_cast<uint32_t>(__popc(peers)));
    }
}
// Same with a fixed-point mass per lane (below 2^44): the lanes of a bin
// add their masses exactly as two 22-bit limbs with warp reductions, and one
// lane per bin updates the shared counters.  The whole warp calls it.
__device__ __forceinline__ void hist_inc_mass(uint32_t* hist, uint64_t* hmass, uint32_t bin,
                                              uint64_t mass, bool active) {
    const uint32_t act = __ballot_sync(0xffffffffu, active);
    if (active) {
        const uint32_t peers = __match_any_sync(act, bin);
        const uint32_t lo = __reduce_add_sync(peers, static_cast<uint32_t>(mass & 0x3fffffu));
        const uint32_t hi = __reduce_add_sync(peers, static_cast<uint32_t>(mass >> 22));
        if ((threadIdx.x & 31) == static_cast<uint32_t>(__ffs(peers) - 1)) {
            atomicAdd(&hist[bin], static_cast<uint32_t>(__popc(peers)));
            atomicAdd(reinterpret_cast<unsigned long long*>(&hmass[bin]),
                      static_cast<unsigned long long>(lo) +
                          (static_cast<unsigned long long>(hi) << 22));
        }
    }
}
// Appends `key` for every lane with `push` set; one atomic per warp.  The
// whole warp calls it.  Returns true when the buffer overflowed.
__device__ __forceinline__ bool warp_push(bool push, uint64_t key, uint64_t* buf, uint32_t cap,
                                          uint32_t* counter) {
    const uint32_t m = __ballot_sync(0xffffffffu, push);
    if (!m) return false;
    const uint32_t lane = threadIdx.x & 31, leader = __ffs(m) - 1;
    uint32_t base = 0;
    if (lane == leader) base = atomicAdd(counter, static_cast<uint32_t>(__popc(m)));
    base = __shfl_sync(0xffffffffu, base, leader);
    const uint32_t pos = base + __popc(m & ((1u << lane) - 1u));
    if (push && pos < cap) buf[pos] = key;
    return base + __popc(m) > cap;
}

// Seed threshold from the consumers' keys (one per thread, 0 = none): the
// largest t on the 2^16 grid with #{keys >= t} >= k, a lower bound of the
// k-th largest key and hence of the row's k-th largest value (0 when k is 0
// or above 256 or fewer than k keys exist); *mx gets the largest key.  The
// search runs bit by bit with every thread voting through a counting
// barrier.
__device__ uint32_t seed_select(uint32_t key, uint32_t k, uint32_t* mx, Ctl& c) {
    *mx = cmax_u32(key, c);
    uint32_t t = 0;
    if (k >= 1 && k <= static_cast<uint32_t>(kCons)) {
#pragma unroll 1
        for (int b = 31; b >= 16; --b) {
            const uint32_t cand = t | (1u << b);
            if (cbar_count(key >= cand) >= k) t = cand;
        }
    }
    return t;
}

// Exact k-th largest value key (upper 32 bits of the rank keys) among
// keys[0..n); n >= k >= 1.
__device__ uint32_t kth_value_key(const uint64_t* keys, uint32_t n, uint32_t k, Ctl& c) {
    uint32_t prefix = 0, mask = 0, need = k;
    for (int level = 0; level < 4; ++level) {
        const int shift = 24 - 8 * level;
        cbar();
        c.hist[threadIdx.x] = 0;
        cbar();
        const uint32_t nr = (n + kCons - 1) / kCons * kCons;
        for (uint32_t i = threadIdx.x; i < nr; i += kCons) {
            const uint32_t vk = i < n ? static_cast<uint32_t>(keys[i] >> 32) : 0u;
            hist_inc(c.hist, (vk >> shift) & 255u, i < n && (vk & mask) == prefix);
        }
        cbar();
        find_bin_desc(c.hist, need, c);
        cbar();
        const uint32_t bin = c.bc_u32[0];
        if (bin == 0xffffffffu) return 0;
        need -= c.bc_u32[1];
        prefix |= bin << shift;
        mask |= 255u << shift;
    }
    return prefix;
}

// Keeps the keys whose value key is >= vk (order not kept); n <= kBuf.
__device__ uint32_t compact_ge(uint64_t* keys, uint32_t n, uint32_t vk, Ctl& c) {
    constexpr uint32_t kPer = kBuf / kCons;
    uint64_t mine[kPer];
    uint32_t cnt = 0;
#pragma unroll
    for (uint32_t u = 0; u < kPer; ++u) {
        const uint32_t i = threadIdx.x + u * kCons;
        mine[u] = i < n ? keys[i] : 0ull;
        cnt += (i < n && static_cast<uint32_t>(mine[u] >> 32) >= vk) ? 1u : 0u;
    }
    uint32_t total;
    uint32_t pos = cscan_excl(cnt, &total, c);  // barriers: every read above is done
#pragma unroll
    for (uint32_t u = 0; u < kPer; ++u) {
        const uint32_t i = threadIdx.x + u * kCons;
        if (i < n && static_cast<uint32_t>(mine[u] >> 32) >= vk) keys[pos++] = mine[u];
    }
    cbar();
    return total;
}

// keys[0..n) (distinct) sorted descending into out[0..n); n <= kGather.
// `out` must have room for the next power of two of n when n > 128.
__device__ void sort_desc(const uint64_t* keys, uint32_t n, uint64_t* out) {
    if (n <= 128) {  // rank by counting
        for (uint32_t i = threadIdx.x; i < n; i += kCons) {
            const uint64_t x = keys[i];
            uint32_t rank = 0;
            for (uint32_t j = 0; j < n; ++j) rank += keys[j] > x;
            out[rank] = x;
        }
        cbar();
        return;
    }
    uint32_t p2 = 1;
    while (p2 < n) p2 <<= 1;
    for (uint32_t i = threadIdx.x; i < p2; i += kCons) out[i] = i < n ? keys[i] : 0ull;
    cbar();
    for (uint32_t size = 2; size <= p2; size <<= 1) {
        for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
            for (uint32_t i = threadIdx.x; i < p2 / 2; i += kCons) {
                const uint32_t lo = 2 * i - (i & (stride - 1));
                const uint32_t hi = lo + stride;
                const bool desc = (lo & size) == 0;
                const uint64_t x = out[lo], y = out[hi];
                if ((x < y) == desc) {
                    out[lo] = y;
                    out[hi] = x;
                }
            }
            cbar();
        }
    }
}

// Exact top-k / min-p cuts of the candidate buffer, then the sorted prefix
// into `sorted`.  Returns the number kept, or ~0u when more than kFinal
// candidates survive the cuts.
__device__ uint32_t finish_buffer(uint64_t* cand, uint32_t n, const Row& r, uint64_t* sorted,
                                  Ctl& c) {
    if (n <= static_cast<uint32_t>(kCons)) {
        // exact sort by rank counting (rank keys are distinct), then the
        // top-k and min-p cuts are prefix lengths
        if (threadIdx.x < n) {
            const uint64_t x = cand[threadIdx.x];
            uint32_t rank = 0;
            for (uint32_t j = 0; j < n; ++j) rank += cand[j] > x;
            sorted[rank] = x;
        }
        cbar();
        uint32_t keep = r.k_eff ? min(n, r.k_eff) : n;
        if (r.minp && keep) {
            const float M = rank_value(sorted[0]);
            if (isfinite(M)) {
                const double floor_w = static_cast<double>(r.p.min_p);
                uint32_t first = keep;
                if (threadIdx.x < keep &&
                    !(exp(static_cast<double>(__fsub_rn(rank_value(sorted[threadIdx.x]), M))) >=
                      floor_w))
                    first = threadIdx.x;
                keep = cmin_u32(first, c);
            }
        }
        return keep;
    }
    uint32_t vk = 0;
    if (r.k_eff && n > r.k_eff) vk = kth_value_key(cand, n, r.k_eff, c);
    if (r.minp && n) {
        // exact min-p against the candidates' maximum (the row maximum, or
        // the segment maximum for a segment's list): keep w >= min_p
        uint32_t mk = 0;
        for (uint32_t i = threadIdx.x; i < n; i += kCons)
            mk = max(mk, static_cast<uint32_t>(cand[i] >> 32));
        mk = cmax_u32(mk, c);
        const float M = key_float(mk);
        if (mk > kNegInfKey && isfinite(M)) {
            const double floor_w = static_cast<double>(r.p.min_p);
            uint32_t lowest = 0xffffffffu;
            for (uint32_t i = threadIdx.x; i < n; i += kCons) {
                const uint32_t k = static_cast<uint32_t>(cand[i] >> 32);
                if (exp(static_cast<double>(__fsub_rn(key_float(k), M))) >= floor_w)
                    lowest = min(lowest, k);
            }
            lowest = cmin_u32(lowest, c);
            if (lowest != 0xffffffffu) vk = max(vk, lowest);
        }
    }
    if (vk) n = compact_ge(cand, n, vk, c);
    if (n > kFinal) return 0xffffffffu;
    sort_desc(cand, n, sorted);
    return r.k_eff ? min(n, r.k_eff) : n;
}

// ------------------------------------------------------ evaluator buffer
// The k-th largest value key among buf[0..n) (n >= k >= 1), rounded down to
// its top 16 bits: the largest t on the 2^16 grid with #{value keys >= t}
// >= k, found bit by bit with warp sums.  The k-th largest of a subset of
// the row is at most the row's k-th largest, so it is a valid threshold.
// One warp.
__device__ __noinline__ uint32_t buf_kth(const uint64_t* buf, uint32_t n, uint32_t k) {
    const uint32_t lane = threadIdx.x & 31;
    uint32_t t = 0;
    if (n <= 512) {  // value keys in registers, 16 per lane
        uint32_t e[16];
#pragma unroll
        for (int m = 0; m < 16; ++m) {
            const uint32_t i = lane + 32u * m;
            e[m] = i < n ? static_cast<uint32_t>(buf[i] >> 32) : 0u;
        }
#pragma unroll 1
        for (int b = 31; b >= 16; --b) {
            const uint32_t cand = t | (1u << b);
            uint32_t cnt = 0;
#pragma unroll
            for (int m = 0; m < 16; ++m) cnt += e[m] >= cand ? 1u : 0u;
            if (__reduce_add_sync(0xffffffffu, cnt) >= k) t = cand;
        }
        return t;
    }
#pragma unroll 1
    for (int b = 31; b >= 16; --b) {
        const uint32_t cand = t | (1u << b);
        uint32_t cnt = 0;
        for (uint32_t i = lane; i < n; i += 32)
            cnt += static_cast<uint32_t>(buf[i] >> 32) >= cand ? 1u : 0u;
        if (__reduce_add_sync(0xffffffffu, cnt) >= k) t = cand;
    }
    return t;
}

// Keeps the entries of buf[0..n) whose value key is >= th, in place (order
// kept); returns their number.  One warp.
__device__ __noinline__ uint32_t buf_compact(uint64_t* buf, uint32_t n, uint32_t th) {
    const uint32_t lane = threadIdx.x & 31;
    uint32_t out = 0;
    for (uint32_t i0 = 0; i0 < n; i0 += 32) {
        const uint32_t i = i0 + lane;
        const uint64_t e = i < n ? buf[i] : 0ull;
        const bool keep = i < n && static_cast<uint32_t>(e >> 32) >= th;
        const uint32_t m = __ballot_sync(0xffffffffu, keep);
        if (keep) buf[out + __popc(m & ((1u << lane) - 1u))] = e;
        out += __popc(m);
    }
    __syncwarp();
    return out;
}

// ---------------------------------------------------------------- epilogue
// Softmax / min-p / top-p / draw over n candidates sorted by rank key, in
// the order of sampling.cc:105-145: w_i = exp((double)(v_i - v_0)) with the
// difference in float, sequential double prefix sums, the quotient-
// accumulating top-p loop (top_p widened from float), total over the
// retained prefix, draw = uniform01(rng_before + gamma) * total, first
// prefix sum above the draw.  min-p keeps the prefix with w_i >= min_p.
// Warp 0 runs it (lane 0 does the sequential sums); results in c.e_*.
__device__ void epilogue(const uint64_t* sorted, uint32_t n, const RowParams& p, bool minp,
                         uint64_t rng_before, double* w, double* S, double* q, Ctl& c) {
    if (threadIdx.x < 32) {
        constexpr unsigned kFull = 0xffffffffu;
        const uint32_t lane = threadIdx.x;
        int32_t status = Q38S_ROW_OK, token = -1;
        uint32_t r = 0;
        double total = 0.0, draw = 0.0;
        if (n == 0 || !isfinite(rank_value(sorted[0]))) {
            status = Q38S_ROW_NO_FINITE;
        } else {
            const float vmax = rank_value(sorted[0]);
            for (uint32_t i = lane; i < n; i += 32)
                w[i] = exp(static_cast<double>(__fsub_rn(rank_value(sorted[i]), vmax)));
            __syncwarp();
            if (minp && p.min_p > 0.0f) {
                const double floor_w = static_cast<double>(p.min_p);
                uint32_t m = n;
                for (uint32_t i0 = 0; i0 < n; i0 += 32) {
                    const uint32_t i = i0 + lane;
                    const uint32_t b = __ballot_sync(kFull, i < n && !(w[i] >= floor_w));
                    if (b) {
                        m = i0 + __ffs(b) - 1;
                        break;
                    }
                }
                n = m;
            }
            if (lane == 0) {
                double acc = 0.0;
                for (uint32_t i = 0; i < n; ++i) {
                    acc += w[i];
                    S[i] = acc;
                }
                total = acc;
            }
            total = __shfl_sync(kFull, total, 0);
            if (!(total > 0.0) || !isfinite(total)) {
                status = Q38S_ROW_NORMALIZATION;
            } else {
                r = n;
                if (p.top_p < 1.0f) {
                    for (uint32_t i = lane; i < n; i += 32) q[i] = w[i] / total;
                    __syncwarp();
                    uint32_t k = 0;
                    if (lane == 0) {
                        const double top_p = static_cast<double>(p.top_p);
                        double cum = 0.0;
                        while (k < n) {
                            cum += q[k];
                            ++k;
                            if (cum >= top_p) break;
                        }
                    }
                    r = __shfl_sync(kFull, k, 0);
                }
                __syncwarp();
                total = S[r - 1];  // the sequential sum over the retained prefix
                draw = uniform01(rng_before + kGamma) * total;
                uint32_t sel = r - 1;
                for (uint32_t i0 = 0; i0 < r; i0 += 32) {
                    const uint32_t i = i0 + lane;
                    const uint32_t b = __ballot_sync(kFull, i < r && draw < S[i]);
                    if (b) {
                        sel = i0 + __ffs(b) - 1;
                        break;
                    }
                }
                token = static_cast<int32_t>(rank_token(sorted[sel]));
            }
        }
        if (lane == 0) {
            c.e_status = status;
            c.e_token = token;
            c.e_n = n;
            c.e_r = r;
            c.e_total = total;
            c.e_draw = draw;
        }
    }
    cbar();
}

// ---------------------------------------------------------------- outputs
__device__ void write_decision(const SampleArgs& a, const Row& r, int32_t token, int32_t status) {
    if (threadIdx.x != 0) return;
    q38s_decision_v1 d;
    d.token = status == Q38S_ROW_OK ? token : -1;
    d.status = status;
    d.rng_before = r.rng_before;
    d.rng_after = r.rng_before + kGamma;
    if (a.decisions) a.decisions[r.v] = d;
    if (a.mode == kModeSampleCommit && status == Q38S_ROW_OK) {
        // commit (sampling.cc:148-156) then commit_token (sampling.cc:163-172)
        // (the state was read at the start of the row; only this row's
        // commit changes it, so it is written without a read)
        RowState s = r.st;
        s.rng_state = d.rng_after;
        s.sampled_tokens += 1;
        const uint32_t col = static_cast<uint32_t>(token) - a.col_begin;
        atomicOr(&a.bitmap[static_cast<size_t>(r.srow) * a.bitmap_words + (col >> 5)],
                 1u << (col & 31));
        if (a.counts) atomicAdd(&a.counts[static_cast<size_t>(r.srow) * a.vocab + col], 1u);
        s.canonical_tokens += 1;
        s.penalty_checksum ^= splitmix64(static_cast<uint64_t>(static_cast<uint32_t>(token)) ^
                                         (s.canonical_tokens * kGamma));
        a.state[r.srow] = s;
    }
}

__device__ void write_distribution(const SampleArgs& a, const Row& r, const uint64_t* sorted,
                                   const double* w, Ctl& c) {
    if (a.dist.capacity == 0) return;
    const uint32_t cap = a.dist.capacity;
    const size_t base = static_cast<size_t>(r.v) * cap;
    const bool ok = c.e_status == Q38S_ROW_OK;
    const uint32_t n = ok ? c.e_n : 0;
    const uint32_t rr = ok ? c.e_r : 0;
    for (uint32_t i = threadIdx.x; i < min(n, cap); i += kCons) {
        if (a.dist.tokens) a.dist.tokens[base + i] = static_cast<int32_t>(rank_token(sorted[i]));
        if (a.dist.values) a.dist.values[base + i] = rank_value(sorted[i]);
        if (a.dist.probs) a.dist.probs[base + i] = i < rr ? w[i] / c.e_total : 0.0;
    }
    if (threadIdx.x == 0) {
        if (a.dist.n_candidates) a.dist.n_candidates[r.v] = n;
        if (a.dist.n_retained) a.dist.n_retained[r.v] = rr;
        if (a.dist.total) a.dist.total[r.v] = c.e_total;
        if (a.dist.draw) a.dist.draw[r.v] = c.e_draw;
    }
}

__device__ void row_error(const SampleArgs& a, const Row& r, int32_t status) {
    if (a.mode == kModeShardTopK) {
        for (uint32_t i = threadIdx.x; i < a.k_out; i += kCons) {
            q38s_candidate cd;
            cd.value = -INFINITY;
            cd.token = -1;
            a.topk_out[static_cast<size_t>(r.v) * a.k_out + i] = cd;
        }
        return;
    }
    write_decision(a, r, -1, status);
    if (a.dist.capacity && threadIdx.x == 0) {
        if (a.dist.n_candidates) a.dist.n_candidates[r.v] = 0;
        if (a.dist.n_retained) a.dist.n_retained[r.v] = 0;
    }
}

// Final outputs of a row from its sorted candidate list.
__device__ void row_output(const SampleArgs& a, const Row& r, const uint64_t* sorted,
                           uint32_t keep, double* w, double* S, double* q, Ctl& c) {
    if (a.mode == kModeShardTopK) {
        for (uint32_t i = threadIdx.x; i < a.k_out; i += kCons) {
            q38s_candidate cd;
            if (i < keep) {
                cd.value = rank_value(sorted[i]);
                cd.token = static_cast<int32_t>(rank_token(sorted[i]));
            } else {
                cd.value = -INFINITY;
                cd.token = -1;
            }
            a.topk_out[static_cast<size_t>(r.v) * a.k_out + i] = cd;
        }
        return;
    }
    epilogue(sorted, keep, r.p, r.minp, r.rng_before, w, S, q, c);
    write_decision(a, r, c.e_token, c.e_status);
    write_distribution(a, r, sorted, w, c);
}

// Speculative verification over all virtual rows' distributions (target
// rows 0..n, draft rows n+1..2n); one thread of the CTA that finished the
// last row.  Leviathan et al. 2023 / Chen et al. 2023 rejection sampling:
// draft i is accepted iff u_i * q_i(d_i) < p_i(d_i) with u_i =
// uniform01(s_i ^ kAcceptDomain), s_i = rng_state + (i + 1) * gamma; the
// first rejection draws from max(0, p_i - q_i) over p_i's sorted support
// with uniform01(s_i); if every draft is accepted the bonus token is the
// reference draw from p_n.  Other CTAs wrote these arrays: L2 loads.
__device__ void mtp_finish(const SampleArgs& a) {
    q38s_mtp_result res;
    const uint32_t n = a.n_draft;
    const uint32_t cap = a.dist.capacity;
    const uint64_t rng0 = __ldcg(reinterpret_cast<const unsigned long long*>(
        &a.state[a.vrow_state_const].rng_state));
    res.rng_before = rng0;
    res.status = Q38S_ROW_OK;
    res.n_tokens = 0;
    res.n_accepted = 0;
    for (uint32_t i = 0; i <= n; ++i) {
        const int32_t t_status = __ldcg(&a.decisions[i].status);
        const int32_t t_token = __ldcg(&a.decisions[i].token);
        const uint64_t s_i = rng0 + (static_cast<uint64_t>(i) + 1) * kGamma;
        if (t_status != Q38S_ROW_OK) {
            res.status = t_status;
            break;
        }
        if (i == n) {  // bonus row: the reference draw from p_n
            res.tokens[res.n_tokens++] = t_token;
            break;
        }
        const int32_t d_status = __ldcg(&a.decisions[n + 1 + i].status);
        if (d_status != Q38S_ROW_OK) {
            res.status = d_status;
            break;
        }
        const uint32_t np = __ldcg(&a.dist.n_retained[i]);
        const uint32_t nq = __ldcg(&a.dist.n_retained[n + 1 + i]);
        if (np > cap || nq > cap || np == 0) {
            res.status = Q38S_ROW_NORMALIZATION;
            break;
        }
        const int32_t* pt = a.dist.tokens + static_cast<size_t>(i) * cap;
        const double* pp = a.dist.probs + static_cast<size_t>(i) * cap;
        const int32_t* qt = a.dist.tokens + static_cast<size_t>(n + 1 + i) * cap;
        const double* qp = a.dist.probs + static_cast<size_t>(n + 1 + i) * cap;
        const int32_t d = a.draft_tokens[i];
        double pd = 0.0, qd = 0.0;
        for (uint32_t j = 0; j < np; ++j)
            if (__ldcg(&pt[j]) == d) pd = __ldcg(&pp[j]);
        for (uint32_t j = 0; j < nq; ++j)
            if (__ldcg(&qt[j]) == d) qd = __ldcg(&qp[j]);
        const double ua = uniform01(s_i ^ kAcceptDomain);
        if (ua * qd < pd) {
            res.tokens[res.n_tokens++] = d;
            ++res.n_accepted;
            continue;
        }
        auto q_of = [&](int32_t tok) {
            double qj = 0.0;
            for (uint32_t m = 0; m < nq; ++m)
                if (__ldcg(&qt[m]) == tok) qj = __ldcg(&qp[m]);
            return qj;
        };
        double rtotal = 0.0;
        for (uint32_t j = 0; j < np; ++j) rtotal += fmax(0.0, __ldcg(&pp[j]) - q_of(__ldcg(&pt[j])));
        int32_t tok = t_token;  // empty residual: the reference draw from p_i
        if (rtotal > 0.0) {
            const double draw = uniform01(s_i) * rtotal;
            double cum = 0.0;
            uint32_t sel = np - 1;
            for (uint32_t j = 0; j < np; ++j) {
                cum += fmax(0.0, __ldcg(&pp[j]) - q_of(__ldcg(&pt[j])));
                if (draw < cum) {
                    sel = j;
                    break;
                }
            }
            tok = __ldcg(&pt[sel]);
        }
        res.tokens[res.n_tokens++] = tok;
        break;
    }
    res.rng_after = res.rng_before + static_cast<uint64_t>(res.n_tokens) * kGamma;
    *a.mtp = res;
}

// A virtual row is complete: the last one runs the speculative verification.
__device__ void row_done(const SampleArgs& a, Ctl& c) {
    if (!a.mtp) return;
    __threadfence();
    cbar();
    if (threadIdx.x == 0) c.bc_u32[2] = atomicAdd(a.ticket, 1u) == a.vrows - 1;
    cbar();
    if (c.bc_u32[2] && threadIdx.x == 0) {
        __threadfence();
        *a.ticket = 0;
        mtp_finish(a);
    }
}

// ------------------------------------------------------------ general path
struct Cut {
    uint32_t M_key;
    float M;
    uint32_t minp_key;
    bool has_cut;
    uint32_t cut_key;
    uint32_t cut_tok;
};

__device__ __forceinline__ bool in_k0(const Cut& g, uint32_t key, uint32_t tok) {
    if (key < g.minp_key) return false;
    if (!g.has_cut) return true;
    return key > g.cut_key || (key == g.cut_key && tok <= g.cut_tok);
}
// Weight of a key relative to the row maximum M, as the mass-weighted
// selection stores it: expf(v - M) in single precision (within a few 2^-24
// relative of the reference's double weights; this path is approximate by
// construction and its draws count as boundary cases).
__device__ __forceinline__ float weight_of(uint32_t key, float M) {
    return expf(__fsub_rn(key_float(key), M));
}
__device__ __forceinline__ uint64_t wfix(float w) {
    return static_cast<uint64_t>(static_cast<double>(w) * kFix + 0.5);
}

// Visits every column j < V of the row's scratch arrays, eight per thread
// per round with the loads issued first (memory-level parallelism for
// L2-resident arrays); f(j, key, weight, valid) runs a warp-uniform number
// of rounds (valid is false past the end), so f may use warp collectives.
// `wts` may be null (weight 0).
template <typename F>
__device__ __forceinline__ void for_keys(const uint32_t* keys, const float* wts, uint32_t V,
                                         F&& f) {
    constexpr uint32_t kStep = 8 * kCons;
    const uint32_t rounds = (V + kStep - 1) / kStep;
    for (uint32_t b = 0; b < rounds; ++b) {
        const uint32_t j0 = b * kStep + threadIdx.x;
        uint32_t kk[8];
        float ww[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t j = j0 + i * kCons;
            kk[i] = j < V ? keys[j] : 0u;
            ww[i] = (wts && j < V) ? wts[j] : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t j = j0 + i * kCons;
            f(j, kk[i], ww[i], j < V);
        }
    }
}

struct Sel {
    bool found;
    uint32_t key;
    uint32_t token;
    uint64_t through;  // count or fixed-point mass up to and including the element
};

// Radix selection over the row's exact keys (global scratch, one per
// column) restricted to K0 (or to key >= minp_key when !restrict_k0): the
// first element in canonical order (value desc, token asc) at which the
// running count (wts == null) or fixed-point mass (wts: the stored weights)
// reaches tau (>= tau, or > tau when strict).
__device__ Sel row_select(const uint32_t* keys, const float* wts, uint32_t V, uint32_t tok0,
                          const Cut& g0, bool restrict_k0, uint64_t tau, bool strict, Ctl& c) {
    const bool weighted = wts != nullptr;
    Cut g = g0;
    if (!restrict_k0) g.has_cut = false;
    uint32_t prefix = 0, mask = 0;
    uint64_t above = 0;
    Sel res{false, 0, 0, 0};
    uint32_t group = 0;
    for (int level = 0; level < 4; ++level) {
        const int shift = 24 - 8 * level;
        cbar();
        c.hist[threadIdx.x] = 0;
        c.hmass[threadIdx.x] = 0;
        cbar();
        for_keys(keys, wts, V, [&](uint32_t j, uint32_t key, float w, bool valid) {
            const bool act = valid && (key & mask) == prefix && in_k0(g, key, tok0 + j);
            const uint32_t d = (key >> shift) & 255u;
            if (weighted) hist_inc_mass(c.hist, c.hmass, d, act ? wfix(w) : 0ull, act);
            else hist_inc(c.hist, d, act);
        });
        cbar();
        if (threadIdx.x == 0) {
            uint64_t acc = above;
            int hit = -1;
            for (int d = 255; d >= 0; --d) {
                if (c.hist[d] == 0) continue;
                const uint64_t nxt = acc + (weighted ? c.hmass[d] : c.hist[d]);
                if (strict ? (nxt > tau) : (nxt >= tau)) {
                    hit = d;
                    break;
                }
                acc = nxt;
            }
            c.bc_u32[0] = static_cast<uint32_t>(hit);
            c.bc_u32[1] = hit >= 0 ? c.hist[hit] : 0u;
            c.bc_u64[0] = acc;
        }
        cbar();
        const int hit = static_cast<int>(c.bc_u32[0]);
        if (hit < 0) return res;
        group = c.bc_u32[1];
        above = c.bc_u64[0];
        prefix |= static_cast<uint32_t>(hit) << shift;
        mask |= 255u << shift;
    }
    // position j inside the tie group {key == prefix} (token order)
    const uint32_t key = prefix;
    uint64_t j, per = 1;
    if (weighted) {
        per = wfix(weight_of(key, g.M));
        if (per == 0) {
            j = 0;
        } else if (strict) {
            j = (tau - above) / per;
        } else {
            const uint64_t need = tau > above ? tau - above : 0;
            j = need == 0 ? 0 : (need + per - 1) / per - 1;
        }
    } else {
        j = tau > above ? tau - above - 1 : 0;
    }
    if (j >= group) j = group - 1;
    // the j-th smallest token of the group: a single member is found in one
    // pass, larger groups by a radix over the token bits
    uint32_t tprefix = 0;
    if (group == 1) {
        cbar();
        for_keys(keys, nullptr, V, [&](uint32_t x, uint32_t k2, float, bool valid) {
            if (valid && k2 == key && in_k0(g, key, tok0 + x)) c.bc_u32[3] = tok0 + x;
        });
        cbar();
        tprefix = c.bc_u32[3];
    } else {
        uint32_t tmask = 0, need = static_cast<uint32_t>(j);
        for (int level = 0; level < 4; ++level) {
            const int shift = 24 - 8 * level;
            cbar();
            c.hist[threadIdx.x] = 0;
            cbar();
            for_keys(keys, nullptr, V, [&](uint32_t x, uint32_t k2, float, bool valid) {
                const uint32_t tok = tok0 + x;
                const bool act =
                    valid && k2 == key && (tok & tmask) == tprefix && in_k0(g, key, tok);
                hist_inc(c.hist, (tok >> shift) & 255u, act);
            });
            cbar();
            if (threadIdx.x == 0) {
                uint32_t left = need, d = 0;
                for (; d < 255; ++d) {
                    if (left < c.hist[d]) break;
                    left -= c.hist[d];
                }
                c.bc_u32[0] = d;
                c.bc_u32[1] = left;
            }
            cbar();
            tprefix |= c.bc_u32[0] << shift;
            tmask |= 255u << shift;
            need = c.bc_u32[1];
        }
    }
    res.found = true;
    res.key = key;
    res.token = tprefix;
    res.through = above + (j + 1) * per;
    return res;
}

template <int DT>
__device__ void general_row(const SampleArgs& a, const Row& r, unsigned char* area, Ctl& c) {
    const uint32_t V = a.vocab;
    const uint32_t tok0 = a.col_begin;
    uint32_t* keys = a.scratch + static_cast<size_t>(r.v) * V;
    float* wts = a.scratch_w + static_cast<size_t>(r.v) * V;
    const unsigned char* row = row_ptr<DT>(a, r.v);
    // this call's penalised columns in shared memory when they fit
    const uint32_t words = (V + 31) / 32;
    const uint32_t* pbm = nullptr;
    if (r.pen && words * 4 <= kArea) {
        uint32_t* sbm = reinterpret_cast<uint32_t*>(area);
        cbar();
        for (uint32_t i = threadIdx.x; i < words; i += kCons) sbm[i] = r.gbm[i];
        cbar();
        for (uint32_t e = threadIdx.x; e < r.n_extra; e += kCons) {
            const uint32_t col = static_cast<uint32_t>(r.extra[e]) - tok0;
            if (col < V) atomicOr(&sbm[col >> 5], 1u << (col & 31));
        }
        cbar();
        pbm = sbm;
    }
    // G0: exact key of every column (eight loads in flight per thread)
    uint32_t kmax = 0;
    constexpr uint32_t kStep = 8 * kCons;
    for (uint32_t b = 0; b < (V + kStep - 1) / kStep; ++b) {
        float xs[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t j = b * kStep + threadIdx.x + i * kCons;
            xs[i] = j < V ? load_elem<DT>(row, j) : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t j = b * kStep + threadIdx.x + i * kCons;
            if (j >= V) break;
            bool penalized = false;
            uint64_t count = 1;
            if (r.pen) {
                if (pbm) {
                    penalized = (pbm[j >> 5] >> (j & 31)) & 1u;
                    if (penalized && r.freq)
                        count = (r.counts_row ? r.counts_row[j] : 0u) + extra_count(r, tok0 + j);
                } else {
                    const uint64_t ex = extra_count(r, tok0 + j);
                    penalized = ((r.gbm[j >> 5] >> (j & 31)) & 1u) || ex;
                    if (penalized && r.freq) count = (r.counts_row ? r.counts_row[j] : 0u) + ex;
                }
            }
            const uint32_t k = float_key(exact_value(xs[i], penalized, count, r.p));
            keys[j] = k;
            kmax = max(kmax, k);
        }
    }
    Q38S_TT(r.v, 6);
    Cut g;
    g.M_key = cmax_u32(kmax, c);  // its barriers also publish keys[] to the CTA
    g.M = key_float(g.M_key);
    g.has_cut = false;
    g.cut_key = 0;
    g.cut_tok = 0;
    g.minp_key = 0;
    if (a.mode != kModeShardTopK && (g.M_key <= kNegInfKey || isinf(g.M))) {
        row_error(a, r, Q38S_ROW_NO_FINITE);
        return;
    }
    // G1: smallest key whose weight reaches min_p
    if (r.minp) {
        if (threadIdx.x == 0) {
            const double floor_w = static_cast<double>(r.p.min_p);
            uint32_t lo = kNegInfKey, hi = g.M_key;  // weight(M) = 1 >= min_p
            while (lo < hi) {
                const uint32_t mid = lo + (hi - lo) / 2;
                const double w = exp(static_cast<double>(__fsub_rn(key_float(mid), g.M)));
                if (w >= floor_w) hi = mid;
                else lo = mid + 1;
            }
            c.bc_u32[3] = hi;
        }
        cbar();
        g.minp_key = c.bc_u32[3];
    }
    // G2: the kept set K0 = top-k of {key >= minp_key}
    uint32_t cnt = 0;
    for_keys(keys, nullptr, V, [&](uint32_t, uint32_t key, float, bool valid) {
        cnt += valid && key >= g.minp_key;
    });
    const uint32_t c_minp = csum_u32(cnt, c);
    const uint32_t n0 = r.k_eff ? min(r.k_eff, c_minp) : c_minp;
    if (n0 < c_minp) {
        const Sel cut = row_select(keys, nullptr, V, tok0, g, false, n0, false, c);
        g.has_cut = true;
        g.cut_key = cut.key;
        g.cut_tok = cut.token;
    }
    Q38S_TT(r.v, 10);
    if (n0 <= kGather) {
        // G3: gather K0, sort, finish exactly
        uint64_t* gk = reinterpret_cast<uint64_t*>(area + kGather * 8);  // unsorted
        uint64_t* lk = reinterpret_cast<uint64_t*>(area);                 // sorted
        cbar();
        if (threadIdx.x == 0) c.bc_u32[2] = 0;
        cbar();
        for_keys(keys, nullptr, V, [&](uint32_t j, uint32_t k, float, bool valid) {
            const bool act = valid && in_k0(g, k, tok0 + j);
            warp_push(act, rank_key(k, tok0 + j), gk, kGather, &c.bc_u32[2]);
        });
        cbar();
        const uint32_t m = min(c.bc_u32[2], kGather);
        sort_desc(gk, m, lk);
        double* w = reinterpret_cast<double*>(area + kGather * 8);
        double* S = reinterpret_cast<double*>(area + kGather * 16);
        double* q = reinterpret_cast<double*>(area + kGather * 24);
        row_output(a, r, lk, m, w, S, q, c);
        return;
    }
    // G4: large kept set: weights once (float), then fixed-point masses
    // (2^-43 units) locate the top-p cut and the draw
    uint64_t part = 0;
    for_keys(keys, nullptr, V, [&](uint32_t j, uint32_t k, float, bool valid) {
        if (!valid) return;
        const bool in = in_k0(g, k, tok0 + j);
        const float w = in ? weight_of(k, g.M) : 0.0f;
        wts[j] = w;
        part += wfix(w);
    });
    const uint64_t Z = csum_u64(part, c);  // its barriers also publish wts[]
    Q38S_TT(r.v, 13);
    int32_t status = Q38S_ROW_OK;
    int32_t token = -1;
    uint64_t Zr = Z;
    Sel cutp{false, 0, 0, 0};
    if (Z == 0) status = Q38S_ROW_NORMALIZATION;
    if (status == Q38S_ROW_OK && r.p.top_p < 1.0f) {
        const uint64_t tau = static_cast<uint64_t>(static_cast<double>(r.p.top_p) *
                                                   static_cast<double>(Z));
        cutp = row_select(keys, wts, V, tok0, g, true, tau, false, c);
        if (cutp.found) Zr = cutp.through;
    }
    Q38S_TT(r.v, 14);
    double draw_d = 0.0;
    if (status == Q38S_ROW_OK) {
        const double u = uniform01(r.rng_before + kGamma);
        const uint64_t draw = static_cast<uint64_t>(u * static_cast<double>(Zr));
        draw_d = static_cast<double>(draw) / kFix;
        const Sel sel = row_select(keys, wts, V, tok0, g, true, draw, true, c);
        if (sel.found) token = static_cast<int32_t>(sel.token);
        else if (cutp.found) token = static_cast<int32_t>(cutp.token);
        else status = Q38S_ROW_NORMALIZATION;
    }
    Q38S_TT(r.v, 15);
    write_decision(a, r, token, status);
    if (a.dist.capacity && threadIdx.x == 0) {
        if (a.dist.n_candidates) a.dist.n_candidates[r.v] = n0;
        if (a.dist.n_retained) a.dist.n_retained[r.v] = 0xffffffffu;
        if (a.dist.total) a.dist.total[r.v] = static_cast<double>(Zr) / kFix;
        if (a.dist.draw) a.dist.draw[r.v] = draw_d;
    }
}

// Completes a row once its candidate list (or failure) is known.
template <int DT>
__device__ void finish_row(const SampleArgs& a, const Row& r, uint32_t flags,
                           const uint64_t* sorted, uint32_t keep, unsigned char* area, Ctl& c) {
    if (flags & kFTimeout) {
        row_error(a, r, Q38S_ROW_TIMEOUT);
    } else if (flags & kFInf) {
        row_error(a, r, Q38S_ROW_NO_FINITE);
    } else if (flags & kFOverflow) {
        general_row<DT>(a, r, area, c);
    } else {
        double* w = reinterpret_cast<double*>(area + (kBuf + kFinal) * 8);
        row_output(a, r, sorted, keep, w, w + kFinal, w + 2 * kFinal, c);
    }
    row_done(a, c);
}

// ------------------------------------------------------------ the kernel
__device__ __forceinline__ void chunk_range(uint32_t vocab, uint32_t S, uint32_t seg, uint32_t& lo,
                                            uint32_t& hi) {
    const uint32_t nblk = (vocab + 127) / 128;
    const uint32_t b0 = static_cast<uint32_t>((static_cast<uint64_t>(nblk) * seg) / S);
    const uint32_t b1 = static_cast<uint32_t>((static_cast<uint64_t>(nblk) * (seg + 1)) / S);
    lo = min(b0 * 128u, vocab);
    hi = min(b1 * 128u, vocab);
}

__device__ bool wait_full(Ctl& c, uint32_t slot, uint32_t phase) {
    if (mbar_try_wait(&c.full[slot], phase)) return true;
    const long long start = clock64();
    while (!mbar_try_wait(&c.full[slot], phase)) {
        if (*reinterpret_cast<volatile uint32_t*>(&c.abort_flag)) return false;
        if (clock64() - start > kWaitLimitCycles) return false;
    }
    return true;
}

// Producer: one lane streams every tile of the CTA's units, in the order
// the consumers read them.
template <int DT>
__device__ void produce(const SampleArgs& a, unsigned char* ring, Ctl& c) {
    constexpr uint32_t es = DT == Q38S_DTYPE_BF16 ? 2u : 4u;
    constexpr uint32_t TC = kTileBytes / es;
    const uint32_t S = a.segs;
    const uint32_t n_units = a.vrows * S;
    uint32_t g = 0;
    for (uint32_t u = blockIdx.x; u < n_units; u += gridDim.x) {
        const uint32_t v = u / S;
        uint32_t c0, c1;
        chunk_range(a.vocab, S, u % S, c0, c1);
        const uint32_t srow = state_row(a, v);
        const bool pen = (a.params[srow].flags & kFlagPenalties) != 0;
        const unsigned char* row = row_ptr<DT>(a, v);
        const uint32_t* bmrow = a.bitmap + static_cast<size_t>(srow) * a.bitmap_words;
        for (uint32_t t0 = c0; t0 < c1; t0 += TC, ++g) {
            const uint32_t slot = g % kRing;
            if (g >= kRing) {
                const long long start = clock64();
                while (!mbar_try_wait(&c.empty[slot], ((g / kRing) - 1) & 1u)) {
                    if (*reinterpret_cast<volatile uint32_t*>(&c.abort_flag) ||
                        clock64() - start > kWaitLimitCycles) {
                        atomicOr(&c.abort_flag, 1u);
                        atomicExch(&c.prod_done, 1u);
                        return;
                    }
                }
            }
            if (*reinterpret_cast<volatile uint32_t*>(&c.abort_flag)) {
                atomicExch(&c.prod_done, 1u);
                return;
            }
            const uint32_t n = min(c1 - t0, TC);
            const uint32_t bytes = n * es;
            const uint32_t bulk = a.use_tma ? (bytes & ~15u) : 0u;
            const uint32_t bmb = pen ? ((n + 127) / 128) * 16 : 0u;
            unsigned char* sl = ring + slot * kSlot;
            mbar_arrive_expect_tx(&c.full[slot], bulk + bmb);
            if (bulk) tma_load_1d(sl, row + static_cast<size_t>(t0) * es, bulk, &c.full[slot]);
            if (bmb) tma_load_1d(sl + kTileBytes, bmrow + t0 / 32, bmb, &c.full[slot]);
            atomicExch(&c.issued, g + 1);
        }
    }
    atomicExch(&c.prod_done, 1u);
}

// Evaluator (warp 9): takes the raw candidates the consumers queue, in
// queue order, 32 per round; gives each its exact value (sampling.cc:76-92)
// and keeps those at or above theta in the unit's candidate buffer as rank
// keys.  theta is the best lower bound known of the smallest value the row
// can keep: the seed's, the k-th largest buffered value and, for min-p
// rows, M + ln(min_p) - slack with M the largest exact value seen.  Every
// rise is published to the consumers, whose filter uses it from their next
// tile on.
//
// The k-th largest buffered value is tracked with a 256-bin histogram of
// value keys laid out from the seed's threshold up to twice the seed's
// maximum (higher keys count in the top bin): after every round the lower
// edge of the highest bin at which the count from the top reaches k is a
// lower bound of the k-th largest buffered value.  Without a seed threshold
// (top_k above 256) a bit search over the buffer refreshes it instead as
// the buffer grows.
//
// Queue protocol: an entry is 1 << 63 | ((column << 1) | penalised) << 32 |
// raw value bits; 0 marks a free slot.  A consumer warp reserves up to 32
// slots at a time on q_head and waits until q_tail leaves room; the
// evaluator takes the contiguous written prefix, clears it and advances
// q_tail.  The oldest reservation always has room (it is at most 32 of kQ
// slots), so every wait ends.
template <int DT>
__device__ void evaluate(const SampleArgs& a, unsigned char* area, Ctl& c) {
    constexpr unsigned kFull = 0xffffffffu;
    const uint32_t lane = threadIdx.x & 31;
    uint64_t* buf = reinterpret_cast<uint64_t*>(area);
    volatile uint64_t* q = reinterpret_cast<volatile uint64_t*>(buf + kBuf);
    uint32_t* hist = c.hist;
    const uint32_t S = a.segs;
    const uint32_t n_units = a.vrows * S;
    uint32_t tail = 0;     // queue entries taken (all units of this CTA)
    uint32_t done_at = 0;  // consumer-warp completions that end the unit
    for (uint32_t u = blockIdx.x; u < n_units; u += gridDim.x) {
        Row r;
        load_row(a, u / S, r);
        done_at += kCons / 32;
        ebar();  // unit start: shared words reset, queue cleared
#pragma unroll
        for (int j = 0; j < 8; ++j) hist[lane * 8 + j] = 0;
        uint32_t theta = 0, pub = 0, mx = 0, n = 0, flags = 0;
        const uint32_t step = r.k_eff ? max(16u, r.k_eff / 4) : 0u;
        uint32_t kth_at = r.k_eff ? r.k_eff + step : 0xffffffffu;
        bool over = false, hist_on = false;
        uint32_t hbase = 0, hshift = 0;
        long long idle0 = clock64();
#ifdef Q38S_TRACE
        uint32_t tr_entries = 0, tr_rounds = 0, tr_kth = 0;
        long long tr_kcyc = 0;
#endif
        while (true) {
            const uint64_t e = q[(tail + lane) % kQ];
            const uint32_t vm = __ballot_sync(kFull, (e >> 63) != 0);
            const uint32_t run = vm == kFull ? 32u : static_cast<uint32_t>(__ffs(~vm) - 1);
            if (run == 0) {
                const uint32_t cd = *reinterpret_cast<volatile uint32_t*>(&c.cons_done);
                if (static_cast<int32_t>(cd - done_at) >= 0) {
                    // every consumer warp has queued its last entry
                    __threadfence_block();
                    const uint32_t head = *reinterpret_cast<volatile uint32_t*>(&c.q_head);
                    if (head == tail || *reinterpret_cast<volatile uint32_t*>(&c.abort_flag)) break;
                }
                if (clock64() - idle0 > 2 * kWaitLimitCycles) {
                    flags |= kFTimeout;
                    if (lane == 0) atomicOr(&c.abort_flag, 1u);
                    break;
                }
                __nanosleep(64);  // leave the issue slots to the consumers
                continue;
            }
            idle0 = clock64();
#ifdef Q38S_TRACE
            tr_entries += run;
            ++tr_rounds;
#endif
            // the seed's bounds (published once per unit by the consumers)
            {
                const uint32_t ts = *reinterpret_cast<volatile uint32_t*>(&c.theta_pub);
                const uint32_t ms = *reinterpret_cast<volatile uint32_t*>(&c.mrun);
                theta = max(theta, ts);
                if (ms > mx) {
                    mx = ms;
                    if (r.minp) theta = max(theta, minp_key(mx, r));
                }
                if (!hist_on && r.k_eff && ts >= 0x10000u) {
                    // bins from the seed threshold up to twice the seed maximum
                    hist_on = true;
                    hbase = ts & 0xffff0000u;
                    const uint32_t range = max(ms, hbase) - hbase;
                    while ((range >> hshift) >= 128u) ++hshift;
                }
            }
            uint32_t k = 0, tok = 0;
            bool inf = false;
            if (lane < run) {
                q[(tail + lane) % kQ] = 0ull;
                if (!over) {
                    const uint32_t col = static_cast<uint32_t>(e >> 33) & 0x3fffffffu;
                    const bool pen = (e >> 32) & 1u;
                    tok = a.col_begin + col;
                    uint64_t count = 1;
                    if (pen && r.freq)
                        count = (r.counts_row ? r.counts_row[col] : 0u) + extra_count(r, tok);
                    const float vx =
                        transform(__uint_as_float(static_cast<uint32_t>(e)), pen, count, r.p);
                    inf = vx == INFINITY;
                    k = float_key(vx);
                }
            }
            tail += run;
            __syncwarp();
            if (lane == 0) {
                __threadfence_block();  // the cleared slots before the new tail
                *reinterpret_cast<volatile uint32_t*>(&c.q_tail) = tail;
            }
            if (over) continue;
            if (__any_sync(kFull, inf)) flags |= kFInf;
            const uint32_t bm = __reduce_max_sync(kFull, k);
            if (bm > mx) {
                mx = bm;
                if (r.minp) theta = max(theta, minp_key(mx, r));
            }
            bool push = lane < run && k >= theta;
            if (n + 32 > kBuf && __any_sync(kFull, push)) {
                // full: compact around the k-th value and theta
                if (r.k_eff && n > r.k_eff) theta = max(theta, buf_kth(buf, n, r.k_eff));
                n = buf_compact(buf, n, theta);
                push = push && k >= theta;
                if (n + 32 > kBuf) {
                    // overflow: the row takes the general path; a threshold
                    // of +inf stops the consumers' queueing
                    over = true;
                    flags |= kFOverflow;
                    if (lane == 0) atomicMax(&c.theta_pub, kPosInfKey);
                    continue;
                }
            }
            const uint32_t pm = __ballot_sync(kFull, push);
            if (push) {
                buf[n + __popc(pm & ((1u << lane) - 1u))] = rank_key(k, tok);
                if (hist_on) atomicAdd(&hist[min((k - hbase) >> hshift, 255u)], 1u);
            }
            n += __popc(pm);
            if (hist_on) {
                if (pm) {
                    __syncwarp();
                    // highest bin at which the count from the top reaches k
                    uint32_t h[8], s8 = 0;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        h[j] = hist[255 - 8 * lane - j];
                        s8 += h[j];
                    }
                    uint32_t inc = s8;
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const uint32_t y = __shfl_up_sync(kFull, inc, o);
                        if (lane >= static_cast<uint32_t>(o)) inc += y;
                    }
                    const uint32_t hit = __ballot_sync(kFull, inc >= r.k_eff);
                    if (hit) {
                        const uint32_t L = __ffs(hit) - 1;
                        uint32_t bin = 0;
                        if (lane == L) {
                            uint32_t acc = inc - s8;
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                acc += h[j];
                                if (acc >= r.k_eff) {
                                    bin = 255 - 8 * lane - j;
                                    break;
                                }
                            }
                        }
                        bin = __shfl_sync(kFull, bin, L);
                        theta = max(theta, hbase + (bin << hshift));
                    }
                }
            } else if (n >= kth_at) {
#ifdef Q38S_TRACE
                const long long tk0 = clock64();
                ++tr_kth;
#endif
                __syncwarp();
                theta = max(theta, buf_kth(buf, n, r.k_eff));
                n = buf_compact(buf, n, theta);
                kth_at = n + step;
#ifdef Q38S_TRACE
                tr_kcyc += clock64() - tk0;
#endif
            }
            if (theta > pub) {
                pub = theta;
                if (lane == 0) atomicMax(&c.theta_pub, theta);
            }
#ifdef Q38S_TRACE
            if (g_trace && lane == 0 && u < 256 && tr_rounds <= 32)
                g_trace[106496 + static_cast<size_t>(u) * 32 + tr_rounds - 1] =
                    ((gtime() & 0xffffffffull) << 32) | theta;
#endif
        }
        tail = *reinterpret_cast<volatile uint32_t*>(&c.q_head);
        // drop what the final threshold excludes
        if (!over && n) n = buf_compact(buf, n, theta);
#ifdef Q38S_TRACE
        if (g_trace && lane == 0 && u < 8192) {
            g_trace[static_cast<size_t>(u) * 16 + 10] = gtime();
            g_trace[static_cast<size_t>(u) * 16 + 14] =
                (static_cast<unsigned long long>(tr_entries) << 32) | tr_rounds;
            g_trace[static_cast<size_t>(u) * 16 + 15] =
                (static_cast<unsigned long long>(tr_kth) << 32) |
                static_cast<unsigned long long>(min(tr_kcyc, 0xffffffffll));
        }
#endif
        if (lane == 0) {
            c.n_cand = over ? 0u : n;
            if (flags) atomicOr(&c.flags, flags);
        }
        __syncwarp();
        ebar();  // unit end: the consumers finish from the buffer
    }
}

template <int DT>
__global__ void __launch_bounds__(kBlock, 2) stream_kernel(const SampleArgs a) {
    extern __shared__ __align__(1024) unsigned char dsm[];
    __shared__ Ctl c;
    constexpr uint32_t es = DT == Q38S_DTYPE_BF16 ? 2u : 4u;
    constexpr uint32_t pv = 16u / es;  // elements per 16-byte vector
    constexpr uint32_t TC = kTileBytes / es;
    constexpr int kU = kTileBytes / 16 / kCons;  // vectors per thread per tile
    constexpr unsigned kFull = 0xffffffffu;
    unsigned char* ring = dsm;
    unsigned char* area = dsm + kRing * kSlot;
    uint64_t* cand = reinterpret_cast<uint64_t*>(area);
    uint64_t* sorted = cand + kBuf;
    const uint32_t tid = threadIdx.x;

    if (tid == 0) {
        for (uint32_t i = 0; i < kRing; ++i) {
            mbar_init(&c.full[i], 1);
            mbar_init(&c.empty[i], kCons / 32);  // one arrival per consumer warp
        }
        c.abort_flag = 0;
        c.prod_done = 0;
        c.issued = 0;
        c.fail_g = 0xffffffffu;
        c.q_head = 0;
        c.q_tail = 0;
        c.cons_done = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (tid >= static_cast<uint32_t>(kCons + 32)) {
        evaluate<DT>(a, area, c);
        return;
    }
    if (tid >= static_cast<uint32_t>(kCons)) {
        if (tid == static_cast<uint32_t>(kCons)) produce<DT>(a, ring, c);
        return;
    }

    // Consumers.  Inside a unit the warps run decoupled: each waits for and
    // releases the slots itself and queues the few elements its filter lets
    // through for the evaluator warp.  Block barriers: the seed (once per
    // unit), rare tile fix-ups, and the start and end of the unit.
    const uint32_t warp = tid >> 5, lane = tid & 31;
    uint64_t* qbuf = cand + kBuf;  // the raw-candidate queue
    const uint32_t S = a.segs;
    const uint32_t n_units = a.vrows * S;
    uint32_t g = 0;     // tiles passed (the producer's order)
    bool stop = false;  // this warp gave up on a copy or a queue slot (warp-uniform)
    for (uint32_t u = blockIdx.x; u < n_units; u += gridDim.x) {
        const uint32_t v = u / S, seg = u % S;
        uint32_t c0, c1;
        chunk_range(a.vocab, S, seg, c0, c1);
        const uint32_t ntiles = (c1 - c0 + TC - 1) / TC;
        Q38S_TT(u, 0);
        Row r;
        load_row(a, v, r);
        Q38S_TT(u, 1);
        if (tid == 0) {
            c.flags = 0;
            c.mrun = 0;
            c.theta_pub = 0;
#ifdef Q38S_TRACE
            c.tr_qwait = 0;
#endif
        }
        // the queue shares the area with the previous unit's epilogue
        for (uint32_t i = tid; i < kQ; i += kCons) qbuf[i] = 0ull;
        ebar();
        uint32_t theta = 0;
        uint32_t rho_theta = 1;  // the threshold rho was derived from (1: none yet)
        float rho = 0.0f;        // raw-logit bound of theta
        bool hopeless = false;
        const unsigned char* src_row = row_ptr<DT>(a, v);
        for (uint32_t t = 0; t < ntiles; ++t, ++g) {
            const uint32_t slot = g % kRing;
            unsigned char* sl = ring + slot * kSlot;
            uint32_t* sbm = reinterpret_cast<uint32_t*>(sl + kTileBytes);
            const uint32_t t0 = c0 + t * TC;
            const uint32_t n = min(c1 - t0, TC);
#ifdef Q38S_TRACE
            const long long tw0 = clock64();
#endif
            bool ok = !stop && wait_full(c, slot, (g / kRing) & 1u);
#ifdef Q38S_TRACE
            const long long tw1 = clock64();
#endif
            ok = __all_sync(kFull, ok);
            if (!ok && !stop) {
                stop = true;
                if (lane == 0) {
                    atomicOr(&c.abort_flag, 1u);
                    atomicMin(&c.fail_g, g);
                }
            }
            // consumer-side writes into the slot: the part the bulk copy
            // cannot move (ragged tail, unaligned rows), -inf padding to a
            // whole vector, this call's additional penalty tokens
            const uint32_t bytes = n * es;
            const uint32_t bulk = a.use_tma ? (bytes & ~15u) : 0u;
            const uint32_t padded = ((n + pv - 1) / pv) * pv;
            const bool fix = bulk < bytes || padded != n;
            const bool mark = r.pen && r.n_extra > 0;
            if (fix || mark) {
                const bool all_ok = !cbar_or(!ok);
                if (all_ok) {
                    const unsigned char* src = src_row + static_cast<size_t>(t0) * es;
                    for (uint32_t b = bulk + tid; b < bytes; b += kCons) sl[b] = src[b];
                    for (uint32_t j = n + tid; j < padded; j += kCons) {
                        if (DT == Q38S_DTYPE_BF16) reinterpret_cast<uint16_t*>(sl)[j] = 0xff80u;
                        else reinterpret_cast<uint32_t*>(sl)[j] = 0xff800000u;
                    }
                    if (mark) {
                        for (uint32_t e = tid; e < r.n_extra; e += kCons) {
                            const uint32_t col = static_cast<uint32_t>(r.extra[e]) - a.col_begin;
                            if (col >= t0 && col < t0 + n)
                                atomicOr(&sbm[(col - t0) >> 5], 1u << ((col - t0) & 31));
                        }
                    }
                }
                fence_async_smem();  // generic writes before the slot's next bulk copy
                cbar();
            }
            // the thread's vectors of this tile
            const uint4* vec = reinterpret_cast<const uint4*>(sl);
            const uint32_t nvec = padded / pv;
            uint4 wv[kU];
#pragma unroll
            for (int q = 0; q < kU; ++q) {
                const uint32_t j = tid + q * kCons;
                wv[q] = (ok && j < nvec)
                            ? vec[j]
                            : (DT == Q38S_DTYPE_BF16
                                   ? make_uint4(0xff80ff80u, 0xff80ff80u, 0xff80ff80u, 0xff80ff80u)
                                   : make_uint4(0xff800000u, 0xff800000u, 0xff800000u,
                                                0xff800000u));
            }
            if (t == 0) {
#ifdef Q38S_TRACE
                const long long ts0 = clock64();
#endif
                // seed (every warp takes part): a lower bound of the exact
                // value of each thread's largest raw logit over the tiles
                // already in the ring (up to four: about a fifth of a row),
                // then the block's k-th / maximum
                float best = -INFINITY;
                int bq = -1;
#pragma unroll
                for (int q = 0; q < kU; ++q) {
                    const float f = vec_max<DT>(wv[q]);
                    if (f > best) {
                        best = f;
                        bq = q;
                    }
                }
                float ahead = -INFINITY;  // the same over the next ring tiles
                if (ok && !r.freq) {
#pragma unroll 1
                    for (uint32_t t2 = 1; t2 < min(ntiles, kRing); ++t2) {
                        const uint32_t g2 = g + t2;
                        const uint32_t n2 = min(c1 - (t0 + t2 * TC), TC);
                        // tiles that need consumer fix-ups are read in their own turn
                        if (!a.use_tma || (n2 * es) % 16 != 0 || n2 % pv != 0) break;
                        if (!wait_full(c, g2 % kRing, (g2 / kRing) & 1u)) break;
                        const uint4* v2 = reinterpret_cast<const uint4*>(ring + (g2 % kRing) * kSlot);
#pragma unroll
                        for (int q = 0; q < kU; ++q) {
                            const uint32_t j = tid + q * kCons;
                            if (j < n2 / pv) ahead = fmaxf(ahead, vec_max<DT>(v2[j]));
                        }
                    }
                }
                if (ahead > best) {
                    best = ahead;
                    bq = 0;
                }
                // Lower bound of the exact value of the thread's largest raw
                // logit, whatever its penalty bit: the smaller of its
                // unpenalised and penalised values (no count is needed without
                // a frequency penalty; those rows find the element instead).
                uint32_t tk = 0;
                if (ok && bq >= 0 && !r.freq) {
                    float lb = exact_value(best, false, 1, r.p);
                    if (r.pen) lb = fminf(lb, exact_value(best, true, 1, r.p));
                    tk = float_key(lb);
                } else if (ok && bq >= 0) {
                    const uint32_t j = tid + bq * kCons;
#pragma unroll 1
                    for (uint32_t e = 0; e < pv; ++e) {
                        const uint32_t idx = j * pv + e;
                        if (idx >= n) break;
                        const float x = load_elem<DT>(sl, idx);
                        if (x == best) {
                            const float vx =
                                eval_slot(r, sbm, x, idx, t0 + idx, a.col_begin + t0 + idx);
                            if (vx == INFINITY) atomicOr(&c.flags, kFInf);
                            tk = float_key(vx);
                            break;
                        }
                    }
                }
#ifdef Q38S_TRACE
                const long long ts1 = clock64();
#endif
                uint32_t m0;
                theta = seed_select(tk, r.k_eff, &m0, c);
#ifdef Q38S_TRACE
                const long long ts2 = clock64();
#endif
                if (r.minp) theta = max(theta, minp_key(m0, r));
#ifdef Q38S_TRACE
                const long long ts3 = clock64();
                if (tid == 0) Q38S_TR(u, 13, ((ts1 - ts0) << 42) | ((ts2 - ts1) << 21) | (ts3 - ts2));
#endif
                if (tid == 0) {
                    atomicMax(&c.mrun, m0);
                    atomicMax(&c.theta_pub, theta);
                }
                hopeless = theta <= kNegInfKey && (c1 - c0) > kBuf;
                Q38S_TT(u, 2);
                Q38S_TR(u, 3, (static_cast<unsigned long long>(theta) << 32) | hopeless);
            } else {
                // the evaluator's threshold
                theta = max(theta, *reinterpret_cast<volatile uint32_t*>(&c.theta_pub));
            }
            if (ok && !hopeless) {
                if (theta != rho_theta) {
                    rho_theta = theta;
                    const float th = theta <= kNegInfKey ? -INFINITY : key_float(theta);
                    rho = raw_bound(th, r.p.temperature);
                }
                // one packed maximum and compare per 16-byte vector: bit q of
                // vhit marks a vector that may hold an element at or above rho
                uint32_t vhit = 0;
                if (DT == Q38S_DTYPE_BF16) {
                    const __nv_bfloat16 rb = __float2bfloat16_rd(rho);
                    const __nv_bfloat162 r2 = __halves2bfloat162(rb, rb);
#pragma unroll
                    for (int q = 0; q < kU; ++q) {
                        const __nv_bfloat162 m =
                            __hmax2(__hmax2(*reinterpret_cast<const __nv_bfloat162*>(&wv[q].x),
                                            *reinterpret_cast<const __nv_bfloat162*>(&wv[q].y)),
                                    __hmax2(*reinterpret_cast<const __nv_bfloat162*>(&wv[q].z),
                                            *reinterpret_cast<const __nv_bfloat162*>(&wv[q].w)));
                        if (!__hblt2(m, r2)) vhit |= 1u << q;
                    }
                } else {
#pragma unroll
                    for (int q = 0; q < kU; ++q)
                        if (!(vec_max<DT>(wv[q]) < rho)) vhit |= 1u << q;
                }
                // Elements of those vectors that may reach theta (raw value at
                // or above rho, or penalised in a row whose penalties can raise
                // a value): bit q * pv + e of look is element e of vector q.
                uint32_t look = 0;
                if (vhit || r.nonmono) {
#pragma unroll
                    for (int q = 0; q < kU; ++q) {
                        const uint32_t j = tid + q * kCons;
                        uint32_t penbits = 0;
                        if (r.nonmono && j < nvec) {
                            const uint32_t e0 = j * pv;
                            penbits = (sbm[e0 >> 5] >> (e0 & 31)) & ((1u << pv) - 1u);
                        }
                        if (((vhit >> q) & 1u) || penbits) {
#pragma unroll
                            for (int e = 0; e < static_cast<int>(pv); ++e) {
                                const float x = vec_elem<DT>(wv[q], e);
                                if ((!(x < rho) || ((penbits >> e) & 1u)) && j * pv + e < n)
                                    look |= 1u << (q * pv + e);
                            }
                        }
                    }
                }
#ifdef Q38S_TRACE
                if (g_trace && u < 256 && t < 20) {
                    const uint32_t nl = __reduce_add_sync(kFull, __popc(look));
                    if (lane == 0)
                        g_trace[65536 + (static_cast<size_t>(u) * 20 + t) * 8 + warp] =
                            (static_cast<unsigned long long>(theta) << 32) | nl;
                    if (lane == 0 && warp == 0)
                        g_trace[114688 + static_cast<size_t>(u) * 20 + t] = gtime();
                }
#endif
                // rare path: the looks go to the evaluator's queue as (raw
                // value, column, penalised bit), at most one per lane and round
                while (__any_sync(kFull, look != 0)) {
                    const uint32_t m = __ballot_sync(kFull, look != 0);
                    uint32_t base = 0, fail = 0;
                    if (lane == 0) {
                        const uint32_t need = __popc(m);
                        base = atomicAdd(&c.q_head, need);
                        const long long w0 = clock64();
                        while (base + need - *reinterpret_cast<volatile uint32_t*>(&c.q_tail) > kQ) {
                            if (*reinterpret_cast<volatile uint32_t*>(&c.abort_flag) ||
                                clock64() - w0 > kWaitLimitCycles) {
                                fail = 1;
                                break;
                            }
                        }
#ifdef Q38S_TRACE
                        atomicAdd(&c.tr_qwait, static_cast<unsigned long long>(clock64() - w0));
#endif
                        __threadfence_block();  // the evaluator's clears before our entries
                    }
                    base = __shfl_sync(kFull, base, 0);
                    if (__shfl_sync(kFull, fail, 0)) {
                        stop = true;
                        if (lane == 0) atomicOr(&c.abort_flag, 1u);
                        break;
                    }
                    if (look) {
                        const uint32_t b = __ffs(look) - 1;
                        look &= look - 1;
                        const uint32_t idx = (tid + (b / pv) * kCons) * pv + (b % pv);
                        const uint32_t pen = r.pen ? (sbm[idx >> 5] >> (idx & 31)) & 1u : 0u;
                        const float x = load_elem<DT>(sl, idx);
                        reinterpret_cast<volatile uint64_t*>(qbuf)[(base + __popc(m & ((1u << lane) - 1u))) % kQ] =
                            (1ull << 63) |
                            (static_cast<uint64_t>(((t0 + idx) << 1) | pen) << 32) |
                            __float_as_uint(x);
                    }
                }
            }
            __syncwarp();
            // release the slot once every lane has read it; a slot whose
            // wait failed is never released (its copy may still land)
#ifdef Q38S_TRACE
            if (g_trace && u < 256 && t < 20 && lane == 0 && warp == 0)
                g_trace[119808 + static_cast<size_t>(u) * 20 + t] =
                    (static_cast<unsigned long long>(tw1 - tw0) << 32) |
                    static_cast<unsigned long long>(clock64() - tw1);
#endif
            if (ok && lane == 0) mbar_arrive(&c.empty[slot]);
        }
        // ---- end of unit: every queued entry is written; the evaluator
        // drains the queue and leaves the candidates in cand[0..n)
        __syncwarp();
        if (lane == 0) {
            __threadfence_block();
            atomicAdd(&c.cons_done, 1u);
        }
        const bool any_stop = cbar_or(stop);
        ebar();
        uint32_t flags = c.flags;
        const uint32_t n = c.n_cand;
        Q38S_TR(u, 6, c.tr_qwait);
        if (any_stop) flags |= kFTimeout;
        if (hopeless) flags |= kFOverflow;
        if (a.mode == kModeShardTopK) flags &= ~kFInf;
        Q38S_TT(u, 4);
        Q38S_TR(u, 5, (static_cast<unsigned long long>(flags) << 32) | n);
        uint32_t keep = 0;
        if (!(flags & (kFTimeout | kFInf | kFOverflow))) {
            keep = finish_buffer(cand, n, r, sorted, c);
            if (keep == 0xffffffffu) flags |= kFOverflow;
        }
        Q38S_TT(u, 7);
        Q38S_TR(u, 11, keep);
        Q38S_TR(u, 12, blockIdx.x);
        if (S == 1) {
            Q38S_TR(u, 8, (flags & kFOverflow) ? 1 : (flags ? 2 : 0));
            finish_row<DT>(a, r, flags, sorted, keep, area, c);
            Q38S_TT(u, 9);
            cbar();
            continue;
        }
        // ---- multi-segment row: park the list, the last segment merges
        {
            const size_t base = static_cast<size_t>(u) * kSegCap;
            const uint32_t len = (flags & (kFTimeout | kFInf | kFOverflow)) ? 0u : keep;
            for (uint32_t i = tid; i < len; i += kCons) a.seg_keys[base + i] = sorted[i];
            if (tid == 0) {
                a.seg_hdr[u * 4 + 0] = len;
                a.seg_hdr[u * 4 + 1] = flags;
            }
            __threadfence();
            cbar();
            if (tid == 0) c.bc_u32[2] = atomicAdd(&a.row_ticket[v], 1u) == S - 1;
            cbar();
            if (!c.bc_u32[2]) {
                Q38S_TR(u, 8, 3);
                Q38S_TT(u, 9);
                continue;
            }
            __threadfence();
            // segment headers in parallel (thread s reads segment s), then
            // every segment's list lands at its prefix offset in cand
            uint32_t my_len = 0, my_flags = 0;
            if (tid < S) {
                my_len = __ldcg(&a.seg_hdr[(v * S + tid) * 4 + 0]);
                my_flags = __ldcg(&a.seg_hdr[(v * S + tid) * 4 + 1]);
            }
            uint32_t rtotal;
            const uint32_t rel_off = cscan_excl(my_len, &rtotal, c);
            uint32_t rflags = cor_u32(my_flags, c);
            if (a.mode == kModeShardTopK) rflags &= ~kFInf;
            uint32_t rkeep = 0;
            if (!(rflags & (kFTimeout | kFInf | kFOverflow)) && rtotal > kBuf) rflags |= kFOverflow;
            if (!(rflags & (kFTimeout | kFInf | kFOverflow))) {
                cbar();
                if (tid < S) {
                    c.hist[tid] = my_len;
                    c.hist[128 + tid] = rel_off;
                }
                cbar();
                // warp w copies segments w, w + 8, ... with lane-strided loads
                for (uint32_t s2 = warp; s2 < S; s2 += kCons / 32) {
                    const uint32_t len2 = c.hist[s2];
                    const uint32_t off2 = c.hist[128 + s2];
                    const uint64_t* src = a.seg_keys + static_cast<size_t>(v * S + s2) * kSegCap;
                    for (uint32_t i = lane; i < len2; i += 32)
                        cand[off2 + i] = __ldcg(reinterpret_cast<const unsigned long long*>(src + i));
                }
                cbar();
                rkeep = finish_buffer(cand, rtotal, r, sorted, c);
                if (rkeep == 0xffffffffu) rflags |= kFOverflow;
            }
            if (tid == 0) a.row_ticket[v] = 0;  // every segment has arrived: reset for the next call
            Q38S_TR(u, 8, 4 + ((rflags & kFOverflow) ? 1 : 0));
            finish_row<DT>(a, r, rflags, sorted, rkeep, area, c);
            Q38S_TT(u, 9);
            cbar();
        }
    }
    const bool aborted = *reinterpret_cast<volatile uint32_t*>(&c.abort_flag) != 0;
    cbar();
    if (aborted || stop) {
        // let the producer stop, then let copies still in flight land before
        // the CTA's shared memory goes away
        if (tid == 0) {
            atomicOr(&c.abort_flag, 1u);
            const long long start = clock64();
            while (!*reinterpret_cast<volatile uint32_t*>(&c.prod_done) &&
                   clock64() - start < kWaitLimitCycles) {
            }
            const uint32_t issued = *reinterpret_cast<volatile uint32_t*>(&c.issued);
            const uint32_t from = min(c.fail_g, g);
            for (uint32_t x = from; x < issued; ++x)
                mbar_wait_bounded(&c.full[x % kRing], (x / kRing) & 1u, kWaitLimitCycles);
        }
        cbar();
    }
}

}  // namespace

size_t stream_smem_bytes() { return kRing * kSlot + kArea; }

#ifdef Q38S_TRACE
}  // namespace q38s
extern "C" int q38s_trace_install(unsigned long long* buf) {
    return static_cast<int>(cudaMemcpyToSymbol(q38s::g_trace, &buf, sizeof(buf)));
}
namespace q38s {
#endif

uint32_t stream_segments(uint32_t vrows, uint32_t vocab, int device) {
    static int sms_cache[64] = {};
    int sms = device >= 0 && device < 64 ? sms_cache[device] : 0;
    if (sms == 0) {
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
        if (sms <= 0) sms = 148;
        if (device >= 0 && device < 64) sms_cache[device] = sms;
    }
    const uint32_t slots = 2u * static_cast<uint32_t>(sms);
    if (vrows == 0 || vrows * 2 >= slots) return 1;
    uint32_t s = slots / vrows;
    const uint32_t nblk = (vocab + 127) / 128;
    const uint32_t by_cols = nblk / 16;  // segments of at least 2,048 columns
    if (s > by_cols) s = by_cols;
    if (s > 64) s = 64;
    while (s > 1 && vrows * s > kMaxSegUnits) --s;
    return s < 1 ? 1 : s;
}

template <int DT>
static int launch_stream_t(const SampleArgs& a, void* stream) {
    auto kern = stream_kernel<DT>;
    const size_t smem = stream_smem_bytes();
    static bool configured[2][64] = {};
    static int sms[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const int slot = DT == Q38S_DTYPE_BF16 ? 0 : 1;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!configured[slot][dev]) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        configured[slot][dev] = true;
    }
    const uint32_t units = a.vrows * a.segs;
    uint32_t cap = 2u * static_cast<uint32_t>(sms[dev]);
#ifdef Q38S_TRACE
    if (const char* gc = getenv("Q38S_TRACE_GRID")) cap = static_cast<uint32_t>(atoi(gc));
#endif
    const uint32_t grid = units < cap ? units : cap;
    kern<<<grid, kBlock, smem, static_cast<cudaStream_t>(stream)>>>(a);
    return cudaGetLastError();
}

int launch_stream(const SampleArgs& a, void* stream) {
    if (a.vrows == 0) return cudaSuccess;
    return a.dtype == Q38S_DTYPE_BF16 ? launch_stream_t<Q38S_DTYPE_BF16>(a, stream)
                                      : launch_stream_t<Q38S_DTYPE_F32>(a, stream);
}

}  // namespace q38s
