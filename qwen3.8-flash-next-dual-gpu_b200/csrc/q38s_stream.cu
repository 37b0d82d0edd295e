// Streaming row sampler for sm_100a: the hot path of every prepare /
// sample-commit / speculative-verification / vocab-shard call.
//
// Work decomposition.  Each virtual row (a batch row, or one target / draft
// row of a speculative verification) is split into `segs` column segments
// (whole 128-column blocks).  A unit is one (row, segment) pair; a persistent
// grid of at most two CTAs per SM walks the units (CTA b takes units b,
// b + G, b + 2G, ...).  Large batches use one segment per row, so every row
// is streamed start to finish by one CTA; small batches split rows so the
// whole GPU pulls HBM.  A split row runs on one thread-block cluster (CTA
// rank = segment): the segments' candidate lists stay in their CTAs' shared
// memory and the leader (rank 0) merges them through distributed shared
// memory.  CTAs of different clusters never wait for one another.
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
//   stream  read every tile once: per thread and tile the largest raw value
//           of its 32 (16) logits, rounded up to bf16 (a bound kept in
//           shared memory), and the thread's largest raw value with its
//           column and penalty bit;
//   theta   the exact values (sampling.cc:76-92) of the 256 threads' largest
//           elements give theta: their k-th largest, a lower bound of the
//           row's k-th largest value, and for min-p rows M + ln(min_p) -
//           slack (M = their largest);
//   gather  the blocks whose bound reaches theta's raw-logit bound are read
//           again (from the ring when the unit is still whole there, else
//           from L2) and their elements at or above theta enter a candidate
//           buffer as 64-bit rank keys (value desc, token asc);
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
constexpr int kBlock = kCons + 32;               // + the producer warp
constexpr uint32_t kBuf = 2048;                  // candidate buffer (rank keys)
constexpr uint32_t kFinal = 1024;                // candidates entering the epilogue
constexpr uint32_t kGather = 1024;               // exact gather of the general path
constexpr uint32_t kArea = 32768;                // candidate / epilogue work area

constexpr uint32_t kHdrKeys = 64;                // value keys per row in the segments' headers

constexpr uint32_t kFOverflow = 1u;
constexpr uint32_t kFInf = 2u;
constexpr uint32_t kFTimeout = 4u;

// Fast-path layout of the area: the candidate buffer (kBuf keys) and, once
// it is sorted, the epilogue's three double arrays (w, S, q) from offset 0;
// the sorted list (kFinal keys) at kSorted; the per-thread tile bounds at
// the tail while a unit streams (dead before the list is sorted).
constexpr uint32_t kSorted = 3 * kFinal * 8;
static_assert(kBuf * 8 <= kSorted && kSorted + kFinal * 8 <= kArea, "fast-path area");

// Optional per-unit trace (build with -DQ38S_TRACE; off in the product
// build): 16 words per unit -- global-timer stamps of the unit's phases, its
// threshold, candidate count, flags and the path that finished it; the SM
// clock at each stamp 131,072 words further.  The buffer is installed with
// q38s_trace_install().
#ifdef Q38S_TRACE
__constant__ unsigned long long* g_trace = nullptr;  // constant: no reload per stamp
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
#define Q38S_TT(u, slot)                                                          \
    do {                                                                          \
        Q38S_TR(u, slot, gtime());                                                \
        if (g_trace && threadIdx.x == 0 && (u) < 8192)                            \
            g_trace[131072 + static_cast<size_t>(u) * 16 + (slot)] =              \
                static_cast<unsigned long long>(clock64());                       \
    } while (0)
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
    uint32_t fail_g;       // first tile a consumer warp gave up waiting for
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
    // rows split over the CTAs of a cluster: the leader (rank 0) collects
    // every segment's list header; each segment waits for the leader to
    // have read its list before it reuses its shared memory
    uint64_t xfull;                 // leader: all headers of the row arrived
    uint64_t xdone;                 // member: the leader has read the list
    uint32_t xh_len[kMaxSegs];      // leader: each list's length, flags, k-th value key
    uint32_t xh_flags[kMaxSegs];
    uint32_t xh_kth[kMaxSegs];
    uint32_t xh_keys[kHdrKeys];     // ... and its first kHdrKeys / S value keys
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
__device__ uint32_t csum_u32(uint32_t v, Ctl& c) {
    v = warp_sum_u32(v);
    cbar();
    if ((threadIdx.x & 31) == 0) c.red_u32[threadIdx.x >> 5] = v;
    cbar();
    uint32_t r = 0;
    for (int i = 0; i < kCons / 32; ++i) r += c.red_u32[i];
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

// Exclusive prefix sum of doubles over the consumers in thread order.
__device__ __forceinline__ double cscan_excl_f64(double v, double* total, Ctl& c) {
    const uint32_t lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    double inc = v;
    for (int o = 1; o < 32; o <<= 1) {
        const double y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= static_cast<uint32_t>(o)) inc += y;
    }
    double excl = __shfl_up_sync(0xffffffffu, inc, 1);
    if (lane == 0) excl = 0.0;
    cbar();
    if (lane == 31) c.red_u64[w] = static_cast<uint64_t>(__double_as_longlong(inc));
    cbar();
    double before = 0.0, all = 0.0;
    for (uint32_t i = 0; i < kCons / 32; ++i) {
        const double x = __longlong_as_double(static_cast<long long>(c.red_u64[i]));
        if (i < w) before += x;
        all += x;
    }
    *total = all;
    return before + excl;
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

__device__ __forceinline__ void load_row(const SampleArgs& a, uint32_t v, Row& r) {
    r.v = v;
    r.srow = state_row(a, v);
    r.p = a.params[r.srow];
    const uint32_t off = v < a.split ? v : v - a.split;
    r.st = a.state[r.srow];
    if (a.rng_from_args) r.st.rng_state = a.rng_state;
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

// Exact transformed value (sampling.cc:76-92), one out-of-line copy of the
// IEEE division sequences for the general path's loop.
__device__ __noinline__ float exact_value(float x, bool penalized, uint64_t count, RowParams p) {
    return transform(x, penalized, count, p);
}

// Exact transformed value of column col given the state row's bitmap word
// holding it (sampling.cc:76-92): the penalised bit, or membership in this
// call's additional tokens; the frequency count from global memory.
__device__ __forceinline__ float exact_pw(const SampleArgs& a, const Row& r, float x, uint32_t col,
                                          uint32_t pw) {
    bool penalized = false;
    uint64_t count = 1;
    if (r.pen) {
        const uint32_t tok = a.col_begin + col;
        const uint64_t ex = r.n_extra ? extra_count(r, tok) : 0u;
        penalized = ((pw >> (col & 31)) & 1u) || ex != 0;
        if (penalized && r.freq) count = (r.counts_row ? r.counts_row[col] : 0u) + ex;
    }
    return exact_value(x, penalized, count, r.p);
}

// Element col of a row, from global memory.
template <int DT>
__device__ __forceinline__ float elem_at(const unsigned char* row, uint32_t col) {
    if (DT == Q38S_DTYPE_BF16)
        return __uint_as_float(static_cast<uint32_t>(
                                   __ldg(reinterpret_cast<const uint16_t*>(row) + col)) << 16);
    return __ldg(reinterpret_cast<const float*>(row) + col);
}

// The 16-byte vector of a row at column col0 (a multiple of its element
// count), from global memory; elements nv and up read as -inf.
template <int DT>
__device__ __forceinline__ uint4 load_vec(const SampleArgs& a, const unsigned char* row,
                                          uint32_t col0, uint32_t nv) {
    constexpr uint32_t es = DT == Q38S_DTYPE_BF16 ? 2u : 4u;
    constexpr uint32_t pv = 16u / es;
    if (a.use_tma && nv == pv)
        return __ldg(reinterpret_cast<const uint4*>(row + static_cast<size_t>(col0) * es));
    uint32_t wd[4];
#pragma unroll
    for (uint32_t i = 0; i < 4; ++i) wd[i] = DT == Q38S_DTYPE_BF16 ? 0xff80ff80u : 0xff800000u;
    for (uint32_t i = 0; i < nv; ++i) {
        const uint32_t bits = __float_as_uint(elem_at<DT>(row, col0 + i));
        if (DT == Q38S_DTYPE_BF16) {
            const uint32_t h = bits >> 16, sh = 16 * (i & 1);
            wd[i >> 1] = (wd[i >> 1] & ~(0xffffu << sh)) | (h << sh);
        } else {
            wd[i] = bits;
        }
    }
    return make_uint4(wd[0], wd[1], wd[2], wd[3]);
}

// Whether a unit streams: its row keeps a top-k of at most 256 or a min-p
// cut (either bounds the candidate set), or the unit is no wider than the
// candidate buffer; and its tile bounds (2 bytes per thread and tile) leave
// room for kFinal candidates in the area.  Other units take the general
// path, which reads the row itself.  The producer and the consumers decide
// alike (tc: columns per tile).
__device__ __forceinline__ bool unit_streams(const SampleArgs& a, uint32_t v, uint32_t cols,
                                             uint32_t tc) {
    if (((cols + tc - 1) / tc) * kCons * 2u + kFinal * 8u > kArea) return false;
    const RowParams& p = a.params[state_row(a, v)];
    const bool minp = a.mode != kModeShardTopK && p.min_p > 0.0f;
    uint32_t k;
    if (a.mode == kModeShardTopK) k = a.k_out >= a.vocab ? 0u : a.k_out;
    else k = (p.top_k == 0 || p.top_k >= a.full_vocab) ? 0u : p.top_k;
    return minp || (k >= 1 && k <= static_cast<uint32_t>(kCons)) || cols <= kBuf;
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
// candidates survive the cuts.  A row's final list (final_list) of at most
// 256 candidates skips the min-p cut here: the epilogue makes the same cut.
__device__ uint32_t finish_buffer(uint64_t* cand, uint32_t n, const Row& r, uint64_t* sorted,
                                  Ctl& c, bool final_list) {
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
        // a row's final list gets its min-p cut in the epilogue
        if (r.minp && keep && !final_list) {
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

// ---------------------------------------------------------------- epilogue
// Softmax / min-p / top-p / draw over n candidates sorted by rank key, in
// the order of sampling.cc:105-145: w_i = exp((double)(v_i - v_0)) with the
// difference in float, double prefix sums S_i of the weights, the top-p cut
// at the first prefix of the quotients w_i / total that reaches top_p (top_p
// widened from float), total over the retained prefix, draw =
// uniform01(rng_before + gamma) * total, the first prefix sum above the
// draw.  min-p keeps the prefix with w_i >= min_p.  The prefix sums are a
// block-wide scan (each thread sums a contiguous run of at most four
// candidates in order, then the runs' totals are scanned): they equal the
// reference's sequential sums to a few units in the last place, so a token
// can differ only where the draw or the top-p target lies within that
// distance of a boundary.  Results in c.e_*.
__device__ void epilogue(const uint64_t* sorted, uint32_t n, const RowParams& p, bool minp,
                         uint64_t rng_before, double* w, double* S, Ctl& c) {
    constexpr uint32_t kRun = kFinal / kCons;  // candidates per thread's run
    static_assert(kFinal % kCons == 0 && kGather <= kFinal, "runs");
    int32_t status = Q38S_ROW_OK, token = -1;
    uint32_t r = 0;
    double total = 0.0, draw = 0.0;
    const bool finite = n != 0 && isfinite(rank_value(sorted[0]));
    if (!finite) {
        status = Q38S_ROW_NO_FINITE;
    } else {
        const float vmax = rank_value(sorted[0]);
        for (uint32_t i = threadIdx.x; i < n; i += kCons)
            w[i] = exp(static_cast<double>(__fsub_rn(rank_value(sorted[i]), vmax)));
        cbar();
        if (minp && p.min_p > 0.0f) {
            const double floor_w = static_cast<double>(p.min_p);
            uint32_t m = n;
            for (uint32_t i = threadIdx.x; i < n; i += kCons)
                if (!(w[i] >= floor_w)) m = min(m, i);
            n = cmin_u32(m, c);
        }
        // inclusive prefix sums of w over runs of kRun consecutive candidates
        const uint32_t i0 = threadIdx.x * kRun;
        double run[kRun];
        double acc = 0.0;
#pragma unroll
        for (uint32_t j = 0; j < kRun; ++j) {
            if (i0 + j < n) acc += w[i0 + j];
            run[j] = acc;
        }
        double all;
        const double off = cscan_excl_f64(acc, &all, c);
#pragma unroll
        for (uint32_t j = 0; j < kRun; ++j)
            if (i0 + j < n) S[i0 + j] = off + run[j];
        cbar();
        total = S[n - 1];
        if (!(total > 0.0) || !isfinite(total)) {
            status = Q38S_ROW_NORMALIZATION;
        } else {
            r = n;
            if (p.top_p < 1.0f) {
                // prefix sums of the quotients, the first reaching top_p
                const double top_p = static_cast<double>(p.top_p);
                double qa = 0.0;
#pragma unroll
                for (uint32_t j = 0; j < kRun; ++j) {
                    if (i0 + j < n) qa += w[i0 + j] / total;
                    run[j] = qa;
                }
                double qall;
                const double qoff = cscan_excl_f64(qa, &qall, c);
                uint32_t hit = n;
#pragma unroll
                for (uint32_t j = 0; j < kRun; ++j)
                    if (i0 + j < n && qoff + run[j] >= top_p) hit = min(hit, i0 + j + 1);
                r = cmin_u32(hit, c);
            }
            total = S[r - 1];  // the sum over the retained prefix
            draw = uniform01(rng_before + kGamma) * total;
            uint32_t sel = r - 1;
            for (uint32_t i = threadIdx.x; i < r; i += kCons)
                if (draw < S[i]) sel = min(sel, i);
            sel = cmin_u32(sel, c);
            token = static_cast<int32_t>(rank_token(sorted[sel]));
        }
    }
    if (threadIdx.x == 0) {
        c.e_status = status;
        c.e_token = token;
        c.e_n = n;
        c.e_r = r;
        c.e_total = total;
        c.e_draw = draw;
    }
    cbar();
}

// ---------------------------------------------------------------- outputs
__device__ __forceinline__ void write_decision(const SampleArgs& a, const Row& r, int32_t token,
                                               int32_t status) {
    if (threadIdx.x != 0) return;
    q38s_decision_v1 d;
    d.token = status == Q38S_ROW_OK ? token : -1;
    d.status = status;
    d.rng_before = r.rng_before;
    d.rng_after = r.rng_before + kGamma;
    if (a.decisions && a.decisions_host) {
        // a host that polls the status sees the other fields first
        volatile q38s_decision_v1* p = a.decisions + r.v;
        p->token = d.token;
        p->rng_before = d.rng_before;
        p->rng_after = d.rng_after;
        __threadfence_system();
        p->status = d.status;
    } else if (a.decisions) {
        a.decisions[r.v] = d;
    }
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

__device__ __forceinline__ void write_distribution(const SampleArgs& a, const Row& r,
                                                   const uint64_t* sorted,
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

__device__ __forceinline__ void row_error(const SampleArgs& a, const Row& r, int32_t status) {
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
__device__ __forceinline__ void row_output(const SampleArgs& a, const Row& r,
                                           const uint64_t* sorted,
                           uint32_t keep, double* w, double* S, Ctl& c) {
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
    epilogue(sorted, keep, r.p, r.minp, r.rng_before, w, S, c);
    Q38S_TT(r.v, 11);
    write_decision(a, r, c.e_token, c.e_status);
    Q38S_TT(r.v, 12);
    write_distribution(a, r, sorted, w, c);
}

// Speculative verification over all virtual rows' distributions (target
// rows 0..n, draft rows n+1..2n), by the whole CTA that finished the last
// row.  Leviathan et al. 2023 / Chen et al. 2023 rejection sampling: draft
// i is accepted iff u_i * q_i(d_i) < p_i(d_i) with u_i = uniform01(s_i ^
// kAcceptDomain), s_i = rng_state + (i + 1) * gamma; the first rejection
// draws from max(0, p_i - q_i) over p_i's sorted support with
// uniform01(s_i); if every draft is accepted the bonus token is the
// reference draw from p_n.  The probability lookups and the per-draft
// verdicts run in parallel (four threads per draft, then one thread per
// draft or support entry); the first draft that is not accepted ends the
// walk; the sequential sums of the residual draw run in one thread, in the
// order written here.  Other CTAs wrote the arrays read here: L2 loads.
__device__ __forceinline__ void mtp_finish(const SampleArgs& a, unsigned char* area, Ctl& c) {
    const uint32_t n = a.n_draft;
    const uint32_t cap = a.dist.capacity;
    const uint32_t tid = threadIdx.x;
    const uint64_t rng0 = __ldcg(reinterpret_cast<const unsigned long long*>(
        &a.state[a.vrow_state_const].rng_state));
    // phase-one layout of the area: result, per-draft p(d), q(d), row
    // headers, verdicts
    q38s_mtp_result* rs = reinterpret_cast<q38s_mtp_result*>(area);
    double* pd = reinterpret_cast<double*>(area + 512);
    double* qd = pd + 64;
    int32_t* hs = reinterpret_cast<int32_t*>(qd + 64);  // row i: t_status, t_token, d_status, np, nq, d
    if (tid <= n) {
        int32_t* h = hs + tid * 6;
        h[0] = __ldcg(&a.decisions[tid].status);
        h[1] = __ldcg(&a.decisions[tid].token);
        if (tid < n) {
            h[2] = __ldcg(&a.decisions[n + 1 + tid].status);
            h[3] = static_cast<int32_t>(__ldcg(&a.dist.n_retained[tid]));
            h[4] = static_cast<int32_t>(__ldcg(&a.dist.n_retained[n + 1 + tid]));
            h[5] = a.draft_tokens[tid];
        }
    }
    if (tid < 64) {
        pd[tid] = 0.0;
        qd[tid] = 0.0;
    }
    cbar();
    // p_i(d_i) and q_i(d_i): draft i = tid % 64, list entries sub, sub + 4, ...
    {
        const uint32_t i = tid & 63u, sub = tid >> 6;
        if (i < n) {
            const int32_t* h = hs + i * 6;
            const uint32_t np = static_cast<uint32_t>(h[3]), nq = static_cast<uint32_t>(h[4]);
            if (h[0] == Q38S_ROW_OK && h[2] == Q38S_ROW_OK && np <= cap && nq <= cap) {
                const int32_t d = h[5];
                const int32_t* pt = a.dist.tokens + static_cast<size_t>(i) * cap;
                const double* pp = a.dist.probs + static_cast<size_t>(i) * cap;
                const int32_t* qt = a.dist.tokens + static_cast<size_t>(n + 1 + i) * cap;
                const double* qp = a.dist.probs + static_cast<size_t>(n + 1 + i) * cap;
#pragma unroll 4
                for (uint32_t j = sub; j < np; j += 4)
                    if (__ldcg(&pt[j]) == d) pd[i] = __ldcg(&pp[j]);
#pragma unroll 4
                for (uint32_t j = sub; j < nq; j += 4)
                    if (__ldcg(&qt[j]) == d) qd[i] = __ldcg(&qp[j]);
            }
        }
    }
    cbar();
    // Each row's verdict, by the thread that loaded it, in the walk's order
    // of checks: 0 draft accepted, 1 draft rejected, 2 the bonus row, 3 a
    // row failed (its status in vs).  The walk stops at the first row whose
    // verdict is not 0.
    uint32_t* vd = reinterpret_cast<uint32_t*>(hs + 65 * 6);
    int32_t* vs = reinterpret_cast<int32_t*>(vd + 65);
    if (tid <= n) {
        const int32_t* h = hs + tid * 6;
        uint32_t v = 0;
        int32_t st = Q38S_ROW_OK;
        if (h[0] != Q38S_ROW_OK) {
            v = 3;
            st = h[0];
        } else if (tid == n) {
            v = 2;
        } else if (h[2] != Q38S_ROW_OK) {
            v = 3;
            st = h[2];
        } else if (static_cast<uint32_t>(h[3]) > cap || static_cast<uint32_t>(h[4]) > cap ||
                   h[3] == 0) {
            v = 3;
            st = Q38S_ROW_NORMALIZATION;
        } else {
            const uint64_t s_i = rng0 + (static_cast<uint64_t>(tid) + 1) * kGamma;
            v = uniform01(s_i ^ kAcceptDomain) * qd[tid] < pd[tid] ? 0u : 1u;
        }
        vd[tid] = v;
        vs[tid] = st;
    }
    cbar();
    if (tid < 32) {
        uint32_t first = n;  // the bonus row's verdict is never 0
        for (uint32_t i0 = 0; i0 <= n; i0 += 32) {
            const uint32_t i = i0 + tid;
            const uint32_t b = __ballot_sync(0xffffffffu, i <= n && vd[i] != 0u);
            if (b) {
                first = i0 + __ffs(b) - 1;
                break;
            }
        }
        if (tid == 0) c.bc_u32[0] = first;
    }
    cbar();
    const uint32_t first = c.bc_u32[0];
    if (tid < first) rs->tokens[tid] = hs[tid * 6 + 5];  // the accepted drafts
    cbar();
    if (tid == 0) {
        rs->rng_before = rng0;
        rs->status = Q38S_ROW_OK;
        rs->n_accepted = first;
        rs->n_tokens = first;
        uint32_t rej = 0xffffffffu;
        if (vd[first] == 3) {
            rs->status = vs[first];
        } else if (vd[first] == 2) {  // bonus row: the reference draw from p_n
            rs->tokens[first] = hs[first * 6 + 1];
            rs->n_tokens = first + 1;
        } else {
            rej = first;
            c.bc_u32[1] = static_cast<uint32_t>(hs[rej * 6 + 3]);
            c.bc_u32[2] = static_cast<uint32_t>(hs[rej * 6 + 4]);
            c.bc_u32[3] = static_cast<uint32_t>(hs[rej * 6 + 1]);
        }
        c.bc_u32[0] = rej;
    }
    cbar();
    const uint32_t rej = c.bc_u32[0];
    if (rej != 0xffffffffu) {
        // residual max(0, p_i - q_i) over p_i's support: the lists in shared
        // memory (the phase-one arrays are dead now), one thread per entry
        const uint32_t np = c.bc_u32[1], nq = c.bc_u32[2];
        const int32_t t_token = static_cast<int32_t>(c.bc_u32[3]);
        int32_t* ptl = reinterpret_cast<int32_t*>(area + 512);
        int32_t* qtl = ptl + kLeaderCap;
        double* ppl = reinterpret_cast<double*>(qtl + kLeaderCap);
        double* qpl = ppl + kLeaderCap;
        const size_t prow = static_cast<size_t>(rej) * cap;
        const size_t qrow = static_cast<size_t>(n + 1 + rej) * cap;
        for (uint32_t j = tid; j < np; j += kCons) {
            ptl[j] = __ldcg(&a.dist.tokens[prow + j]);
            ppl[j] = __ldcg(&a.dist.probs[prow + j]);
        }
        for (uint32_t j = tid; j < nq; j += kCons) {
            qtl[j] = __ldcg(&a.dist.tokens[qrow + j]);
            qpl[j] = __ldcg(&a.dist.probs[qrow + j]);
        }
        cbar();
        for (uint32_t j = tid; j < np; j += kCons) {
            double qj = 0.0;
            const int32_t tok = ptl[j];
            for (uint32_t m = 0; m < nq; ++m)
                if (qtl[m] == tok) qj = qpl[m];
            ppl[j] = fmax(0.0, ppl[j] - qj);  // in place: entry j is this thread's
        }
        cbar();
        if (tid == 0) {
            const uint64_t s_i = rng0 + (static_cast<uint64_t>(rej) + 1) * kGamma;
            double rtotal = 0.0;
            for (uint32_t j = 0; j < np; ++j) rtotal += ppl[j];
            int32_t tok = t_token;  // empty residual: the reference draw from p_i
            if (rtotal > 0.0) {
                const double draw = uniform01(s_i) * rtotal;
                double cum = 0.0;
                uint32_t sel = np - 1;
                for (uint32_t j = 0; j < np; ++j) {
                    cum += ppl[j];
                    if (draw < cum) {
                        sel = j;
                        break;
                    }
                }
                tok = ptl[sel];
            }
            rs->tokens[rs->n_tokens++] = tok;
        }
    }
    if (tid == 0) {
        rs->rng_after = rs->rng_before + static_cast<uint64_t>(rs->n_tokens) * kGamma;
        *a.mtp = *rs;
    }
    cbar();
}

// A virtual row is complete: the last one runs the speculative verification.
__device__ __forceinline__ void row_done(const SampleArgs& a, unsigned char* area, Ctl& c) {
    if (!a.mtp) return;
    cbar();
    // one GPU-scope acquire-release ticket: it publishes this row's outputs
    // (ordered before it by the barrier) and, for the last row, makes every
    // other row's visible
    if (threadIdx.x == 0) {
        c.bc_u32[2] = atom_add_acq_rel_gpu(a.ticket, 1u) == a.vrows - 1;
    }
    cbar();
    if (c.bc_u32[2]) {
        if (threadIdx.x == 0) *a.ticket = 0;
        mtp_finish(a, area, c);
    }
}

// ------------------------------------------------------------ general path
// Rows whose kept set the streaming threshold cannot bound (top_k = 0 or
// top_k > 256 without min-p, or more than kFinal candidates after the cuts).
// One CTA per row:
//   P1  the exact value key (sampling.cc:76-92) of every column into global
//       scratch, and the row maximum M;
//   K0  the candidate set after min-p and top-k (sampling.cc:94-104 plus
//       min-p); a top-k cut is located by count, as below;
//   P2  a histogram of K0 over kGB distance bins: d = fl(M - v) in [0, 64)
//       in steps of 1/32 (d >= 64 and -inf in the last bin).  The
//       reference's weight of an element is exp(fl(v - M)) = exp(-d)
//       (sampling.cc:110-113), so a bin's mass is exp(-b/32) times the sum
//       of its in-bin weights exp(-(d - b/32)), kept in 2^-40 fixed point
//       (exact integer sums, independent of thread order).  Bins in order
//       are the canonical order (value desc); their exclusive prefix counts
//       and masses go to the row's scratch.
//   locate  the first K0 element (canonical order: value desc, token asc) at
//       which the running count, or the running mass, reaches a target: its
//       bin from the prefixes, then key sub-bins of that bin until at most
//       kGL elements remain (gathered, sorted, exact double weights summed
//       in order) or a single key remains (a tie group: the position by
//       arithmetic, the token by a radix over the columns).
// Top-p locates top_p * Z (Z = the mass of K0; the quotient-accumulating
// loop of sampling.cc:119-131 up to rounding); the draw locates
// uniform01(rng + gamma) * Z_r strictly (sampling.cc:133-145), Z_r being the
// mass through the top-p cut.  Masses above the final list are exact to
// about 1e-12 relative; the final list is summed in the reference's order.
constexpr uint32_t kGB = 2048;              // distance bins, 1/32 wide
constexpr double kGUnit = 1099511627776.0;  // 2^40: fixed-point unit of in-bin weights
constexpr uint32_t kGL = kGather;           // largest span gathered and sorted exactly
// scratch words after a row's keys: prefix counts [kGB + 1] (+1 pad), prefix
// masses [kGB + 1] (doubles), then the emission's sub-bin counts, one row of
// kGB per refinement depth
constexpr uint32_t kAuxPm = kGB + 2;
constexpr uint32_t kAuxSub = kAuxPm + 2 * (kGB + 1) + 1;
constexpr uint32_t kEmitDepth = 3;
static_assert(kGB * 12 <= kArea && kGL * 16 + (kGB + 1) * 4 <= kArea, "general-path area");

// A deferred row is shared by a team of general-kernel CTAs when fewer rows
// are deferred than the kernel has CTAs.  Member m takes the column chunk
// [c0, c1) of every pass (32-column aligned), and each pass's reduction (a
// maximum, a count, a histogram, the gathered members of a span) meets in
// the row's team words in global memory: every member adds its CTA's
// partial result with atomics, then the members wait for one another (a
// GPU-scope barrier: an arrival counter and a generation word, bounded by
// the wait limit) and read the total from L2.  The partial results of
// phase q (q team barriers passed) go to slot q % 3; right after barrier q
// the members zero slot (q + 1) % 3, one slice each (it was last read in
// phase q - 1, and is next written in phase q + 1, after barrier q + 1).
// The stream kernel zeroes the barrier words and slots 0 and 1 when it
// defers the row.  A team of one CTA keeps every reduction in shared memory.
constexpr uint32_t kSlotCnt = 0;             // [kGB] counts
constexpr uint32_t kSlotMass = kGB;          // [kGB] 64-bit fixed-point masses
constexpr uint32_t kSlotScal = 3 * kGB;      // [8] scalars: max, ~min, sum, gathered count
constexpr uint32_t kSlotBuf = 3 * kGB + 8;   // [kGL] gathered rank keys
constexpr uint32_t kSlotWords = kSlotBuf + 2 * kGL;
constexpr uint32_t kTeamSync = 8;            // barrier words before slot 0
constexpr uint32_t kTeamOff = 16384;         // team words: after the emission's words
static_assert(kTeamSync + 3 * kSlotWords == kGTeamWords, "team words");
static_assert(kTeamOff + kGTeamWords == kGAuxWords && kSlotWords % 4 == 0, "team layout");
static_assert(kAuxSub + kEmitDepth * kGB <= kTeamOff, "emission words");

// the general kernel's shared memory: the work area, the pass stages, the
// level-1 prefix counts and masses
constexpr uint32_t kPcBytes = ((kGB + 1) * 4 + 15) & ~15u;
constexpr uint32_t kPcPmBytes = kPcBytes + (((kGB + 1) * 8 + 15) & ~15u);

struct GTeam {             // in shared memory, one per CTA
    uint32_t rank, size;   // this CTA's place in the row's team, and its members
    uint32_t* sync;        // [0] arrivals, [1] generation
    uint32_t* slots;       // three accumulation slots
    uint32_t phase;        // team barriers passed
    uint32_t failed;       // a barrier wait ran out: this CTA left the team
};

struct GRow {
    const uint32_t* keys;  // exact key per column (padded to whole 16-byte groups)
    uint4* stage;          // the passes' cp.async slots (kStageBytes of shared memory)
    Ctl* ctl;              // the CTA's control block
    GTeam* t;              // the row's team
    uint32_t c0, c1;       // this CTA's columns
    uint32_t V, tok0;
    float M;               // the row maximum
    uint32_t minp_key;     // smallest key whose weight reaches min_p (0: no min-p)
    bool has_cut;          // top-k cut: the canonical position (cut_key, cut_col)
    uint32_t cut_key, cut_col;
};

__device__ __forceinline__ bool g_in(const GRow g, uint32_t key, uint32_t col) {
    if (key < g.minp_key) return false;
    if (!g.has_cut) return true;
    return key > g.cut_key || (key == g.cut_key && col <= g.cut_col);
}
// Distance d = fl(M - v) (the negated fl(v - M) of the reference) and its bin.
__device__ __forceinline__ uint32_t g_bin(const GRow g, uint32_t key, float& d) {
    d = __fsub_rn(g.M, key_float(key));
    const float s = __fmul_rn(d, 32.0f);
    return s < static_cast<float>(kGB - 1) ? static_cast<uint32_t>(s) : kGB - 1;
}
// exp(-(d - b/32)) in 2^-40 units (0 for d >= 64, where weights are below
// 2^-92 of the maximum's): a Taylor series to the sixth power of r < 1/32
// (truncation below 6e-15).
__device__ __forceinline__ unsigned long long g_tw(float d, uint32_t b) {
    if (!(d < 64.0f)) return 0ull;
    const double r = static_cast<double>(d) - static_cast<double>(b) * 0.03125;
    double t = 1.0 - r * (1.0 / 6.0);
    t = 1.0 - r * 0.2 * t;
    t = 1.0 - r * 0.25 * t;
    t = 1.0 - r * (1.0 / 3.0) * t;
    t = 1.0 - r * 0.5 * t;
    t = 1.0 - r * t;
    return __double2ull_rn(t * kGUnit);
}
// The reference's weight of a key, exp((double)fl(v - M)) (sampling.cc:112).
__device__ __forceinline__ double g_weight(const GRow g, uint32_t key) {
    return exp(static_cast<double>(__fsub_rn(key_float(key), g.M)));
}
__device__ __forceinline__ double g_bin_scale(uint32_t b) {
    return exp(-static_cast<double>(b) * 0.03125);
}
// A 64-bit shared-memory sum kept as two 32-bit words: 32-bit atomics, the
// carry out of the low word added to the high word (exact).
__device__ __forceinline__ void add_u64_split(uint32_t* w, unsigned long long m) {
    const uint32_t lo = static_cast<uint32_t>(m), hi = static_cast<uint32_t>(m >> 32);
    const uint32_t old = atomicAdd(&w[0], lo);
    const uint32_t up = hi + (old + lo < old ? 1u : 0u);
    if (up) atomicAdd(&w[1], up);
}
__device__ __forceinline__ unsigned long long get_u64_split(const uint32_t* w) {
    return static_cast<unsigned long long>(w[0]) | (static_cast<unsigned long long>(w[1]) << 32);
}


// Pipelined passes of the general kernel: every thread streams its own
// 16-byte groups (group r * kCons + tid in round r) through kStages cp.async
// slots of shared memory, kStages - 1 rounds ahead of their use, so 64 KB per
// CTA are in flight without holding registers.  Each thread reads only the
// slots it filled; a slot is refilled after its value was consumed.
constexpr uint32_t kStages = 16;
constexpr uint32_t kStageBytes = kStages * kCons * 16;
static_assert(kStageBytes <= kRing * kSlot, "general-path stages in the ring");

__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)),
                 "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// f(group, 16 bytes, valid) over the nbytes at src (16-byte aligned); a ragged
// last group is zero-filled past its end.  Warp-uniform round count.
template <typename F>
__device__ __forceinline__ void g_pass16(const unsigned char* src, uint64_t nbytes, uint4* stage,
                                         Ctl&, F&& f) {
    const uint32_t n16 = static_cast<uint32_t>((nbytes + 15) / 16);
    const uint32_t rounds = (n16 + kCons - 1) / kCons;
    auto issue = [&](uint32_t r) {
        const uint32_t gi = r * kCons + threadIdx.x;
        if (r < rounds && gi < n16) {
            const uint64_t off = static_cast<uint64_t>(gi) * 16;
            const uint32_t bytes = nbytes - off >= 16 ? 16u : static_cast<uint32_t>(nbytes - off);
            cp_async16(&stage[(r % kStages) * kCons + threadIdx.x], src + off, bytes);
        }
        cp_async_commit();  // one group per round, so the wait counts stay aligned
    };
    for (uint32_t r = 0; r + 1 < kStages; ++r) issue(r);
    for (uint32_t r = 0; r < rounds; ++r) {
        issue(r + kStages - 1);
        cp_async_wait<kStages - 1>();
        const uint32_t gi = r * kCons + threadIdx.x;
        const uint4 v = gi < n16 ? stage[(r % kStages) * kCons + threadIdx.x]
                                 : make_uint4(0u, 0u, 0u, 0u);
        f(gi, v, gi < n16);
    }
    cp_async_wait<0>();
}

// Visits every column of this CTA's chunk with its key; f(col, key, valid)
// runs a warp-uniform number of times.
template <typename F>
__device__ __forceinline__ void g_for_keys(const GRow g, F&& f) {
    g_pass16(reinterpret_cast<const unsigned char*>(g.keys + g.c0),
             static_cast<uint64_t>(g.c1 - g.c0) * 4, g.stage, *g.ctl,
             [&](uint32_t gi, const uint4& kv, bool) {
                 const uint32_t c0 = g.c0 + gi * 4;
                 f(c0, kv.x, c0 < g.c1);
                 f(c0 + 1, kv.y, c0 + 1 < g.c1);
                 f(c0 + 2, kv.z, c0 + 2 < g.c1);
                 f(c0 + 3, kv.w, c0 + 3 < g.c1);
             });
}

// ---- team reductions (no-ops for a team of one)
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// The slot this phase's partial results go to.
__device__ __forceinline__ uint32_t* team_acc(const GTeam& t) {
    return t.slots + (t.phase % 3u) * kSlotWords;
}
// Every member's partial results of the phase are in: the barrier, then the
// zeroing of the slot after next.  The CTA barrier orders every thread's
// partial results before thread 0's acquire-release arrival (release is
// cumulative), and the acquire of the new generation plus the CTA barrier
// after it order the other members' results before this CTA's L2 reads, so
// no separate fence is needed.  Returns the slot that holds the totals,
// or nullptr when this CTA has left the team (its wait ran out now or
// before); a CTA that left neither adds nor waits any more, so the others'
// next wait runs out as well and the row ends with a timeout status.
__device__ __forceinline__ const uint32_t* team_sync(GTeam& t, Ctl& c) {
    const uint32_t* done = team_acc(t);
    cbar();  // the CTA's partial results are issued
    if (threadIdx.x == 0) {
        if (!t.failed) {
            const uint32_t gen = ld_acquire_gpu(t.sync + 1);
            if (atom_add_acq_rel_gpu(t.sync, 1u) + 1u == t.size) {
                t.sync[0] = 0;  // before the release: the next barrier counts from 0
                st_release_gpu(t.sync + 1, gen + 1u);
            } else {
                const long long start = clock64();
                while (ld_acquire_gpu(t.sync + 1) == gen) {
                    if (clock64() - start > kWaitLimitCycles) {
                        t.failed = 1u;
                        break;
                    }
                }
            }
        }
        ++t.phase;
    }
    cbar();
    if (t.failed) return nullptr;
    uint4* z = reinterpret_cast<uint4*>(team_acc(t) + kSlotWords);  // slot (phase + 1) % 3
    if (t.phase % 3u == 2u) z = reinterpret_cast<uint4*>(t.slots);
    constexpr uint32_t n4 = kSlotWords / 4;
    const uint32_t per = (n4 + t.size - 1) / t.size;
    const uint32_t lo = min(n4, t.rank * per), hi = min(n4, lo + per);
    for (uint32_t i = lo + threadIdx.x; i < hi; i += kCons) z[i] = make_uint4(0u, 0u, 0u, 0u);
    return done;
}
// Team-wide maximum (and, with `lo`, minimum) of 32-bit values that the
// CTA has reduced already; a CTA that left the team keeps its own.
__device__ __forceinline__ uint32_t team_max(const GRow g, uint32_t v, uint32_t* lo, Ctl& c) {
    GTeam& t = *g.t;
    if (t.size == 1) return v;
    uint32_t* acc = team_acc(t);
    if (threadIdx.x == 0 && !t.failed) {
        atomicMax(&acc[kSlotScal], v);
        if (lo) atomicMax(&acc[kSlotScal + 1], ~*lo);
    }
    const uint32_t* tot = team_sync(t, c);
    if (!tot) return v;
    if (lo) *lo = ~__ldcg(&tot[kSlotScal + 1]);
    return __ldcg(&tot[kSlotScal]);
}
__device__ __forceinline__ uint32_t team_sum(const GRow g, uint32_t v, Ctl& c) {
    GTeam& t = *g.t;
    if (t.size == 1) return v;
    uint32_t* acc = team_acc(t);
    if (threadIdx.x == 0 && !t.failed) atomicAdd(&acc[kSlotScal + 2], v);
    const uint32_t* tot = team_sync(t, c);
    return tot ? __ldcg(&tot[kSlotScal + 2]) : v;
}
// A shared-memory histogram of nb bins (counts hc, and with hm the split
// 64-bit masses) replaced by the team's total.
__device__ __forceinline__ void team_hist(const GRow g, uint32_t* hc, uint32_t* hm, uint32_t nb,
                                          Ctl& c) {
    GTeam& t = *g.t;
    if (t.size == 1) return;
    uint32_t* acc = team_acc(t);
    cbar();  // the CTA's histogram is complete
    if (!t.failed) {
        for (uint32_t b = threadIdx.x; b < nb; b += kCons) {
            if (hc[b]) atomicAdd(&acc[kSlotCnt + b], hc[b]);
            if (hm) {
                const unsigned long long m = get_u64_split(&hm[2 * b]);
                if (m)
                    atomicAdd(reinterpret_cast<unsigned long long*>(&acc[kSlotMass + 2 * b]), m);
            }
        }
    }
    const uint32_t* tot = team_sync(t, c);
    if (!tot) return;
    for (uint32_t b = threadIdx.x; b < nb; b += kCons) {
        hc[b] = __ldcg(&tot[kSlotCnt + b]);
        if (hm) {
            hm[2 * b] = __ldcg(&tot[kSlotMass + 2 * b]);
            hm[2 * b + 1] = __ldcg(&tot[kSlotMass + 2 * b + 1]);
        }
    }
    cbar();
}
// The rank keys gathered in buf (n of them, n <= kGL in all) replaced by the
// team's; returns their number.  Their order differs between runs: callers
// sort them.
__device__ __forceinline__ uint32_t team_gather(const GRow g, uint64_t* buf, uint32_t n, Ctl& c) {
    GTeam& t = *g.t;
    if (t.size == 1) return n;
    uint32_t* acc = team_acc(t);
    cbar();  // buf is complete (and n read by every thread)
    if (threadIdx.x == 0)
        c.bc_u32[1] = (t.failed || n == 0) ? 0u : atomicAdd(&acc[kSlotScal + 3], n);
    cbar();
    const uint32_t at = c.bc_u32[1];
    uint64_t* gb = reinterpret_cast<uint64_t*>(acc + kSlotBuf);
    if (!t.failed)
        for (uint32_t i = threadIdx.x; i < n; i += kCons)
            if (at + i < kGL) gb[at + i] = buf[i];
    const uint32_t* tot = team_sync(t, c);
    if (!tot) return n;
    const uint32_t m = min(__ldcg(&tot[kSlotScal + 3]), kGL);
    const uint64_t* src = reinterpret_cast<const uint64_t*>(tot + kSlotBuf);
    for (uint32_t i = threadIdx.x; i < m; i += kCons) buf[i] = __ldcg(&src[i]);
    cbar();
    return m;
}

// P1: the exact key (sampling.cc:76-92) of every column of [c0, c1) into
// keys (16-byte stores); the logits arrive through the pipelined pass when
// rows are 16-byte aligned.  Returns the CTA's largest key.
template <int DT>
__device__ __forceinline__ uint32_t g_keys(const SampleArgs& a, const Row& r, const unsigned char* row,
                                           const uint32_t* pbm, uint32_t* keys, uint32_t V,
                                           uint32_t c0, uint32_t c1, uint4* stage, Ctl& c) {
    constexpr uint32_t es = DT == Q38S_DTYPE_BF16 ? 2u : 4u;
    constexpr uint32_t pv = 16u / es;
    uint32_t kmax = 0;
    // the reciprocal of the temperature, correctly rounded, for the division
    // of unpenalised logits (temperatures in [2^-30, 2^30])
    const float rcp_t = __frcp_rn(r.p.temperature);
    const bool rcp_ok = r.p.temperature >= 0x1p-30f && r.p.temperature <= 0x1p30f;
    auto group = [&](uint32_t q, const uint4& w) {
        const uint32_t col0 = q * pv;
        uint32_t pw = 0;  // penalised bits of the 32-column word holding the group
        if (r.pen) pw = pbm ? pbm[col0 >> 5] : r.gbm[col0 >> 5];
        uint32_t k[pv];
#pragma unroll
        for (uint32_t e = 0; e < pv; ++e) {
            const uint32_t col = col0 + e;
            bool pen = false;
            uint64_t count = 1;
            if (r.pen && col < V) {
                const uint64_t ex = (!pbm && r.n_extra) ? extra_count(r, a.col_begin + col) : 0u;
                pen = ((pw >> (col & 31)) & 1u) || ex != 0;
                if (pen && r.freq)
                    count = (r.counts_row ? r.counts_row[col] : 0u) +
                            (pbm ? extra_count(r, a.col_begin + col) : ex);
            }
            float x = vec_elem<DT>(w, static_cast<int>(e));
            float v;
            const float ax = fabsf(x);
            if (!pen && ax <= 0x1p60f && (ax >= 0x1p-60f || ax == 0.0f)) {
                // x / T by the reciprocal and one Markstein correction step
                // (exact in this range for the temperature range checked below)
                const float q0 = __fmul_rn(x, rcp_t);
                v = __fmaf_rn(__fmaf_rn(-q0, r.p.temperature, x), rcp_t, q0);
                if (!rcp_ok) v = __fdiv_rn(x, r.p.temperature);
            } else {
                v = transform(x, pen, count, r.p);
            }
            k[e] = col < V ? float_key(v) : 0u;
            kmax = max(kmax, k[e]);
        }
        if (col0 + pv <= V) {
            uint4* dst = reinterpret_cast<uint4*>(keys + col0);
            dst[0] = make_uint4(k[0], k[1], k[2], k[3]);
            if (pv == 8)
                dst[1] = make_uint4(k[pv == 8 ? 4 : 0], k[pv == 8 ? 5 : 0], k[pv == 8 ? 6 : 0],
                                    k[pv == 8 ? 7 : 0]);
        } else {
#pragma unroll
            for (uint32_t e = 0; e < pv; ++e)
                if (col0 + e < V) keys[col0 + e] = k[e];
        }
    };
    const uint32_t q0 = c0 / pv;  // c0 is a multiple of 32
    if (a.use_tma) {
        g_pass16(row + static_cast<size_t>(c0) * es, static_cast<uint64_t>(c1 - c0) * es, stage, c,
                 [&](uint32_t q, const uint4& w, bool valid) {
                     if (valid) group(q0 + q, w);
                 });
    } else {
        const uint32_t nvec = (c1 + pv - 1) / pv;
        for (uint32_t q = q0 + threadIdx.x; q < nvec; q += kCons)
            group(q, load_vec<DT>(a, row, q * pv, min(pv, V - q * pv)));
    }
    return cmax_u32(kmax, c);  // its barriers also publish keys[] to the CTA
}

// P2: histogram of K0 over the distance bins, then each bin's exclusive
// prefix count (pc) and, when weighted, mass (pm); pc[kGB] / pm[kGB] hold
// the totals.  Returns |K0|; *Z gets its mass.
__device__ __forceinline__ uint32_t g_level1(const GRow g, bool weighted, unsigned char* area, uint32_t* pc,
                             double* pm, double* Z, Ctl& c) {
    uint32_t* hc = reinterpret_cast<uint32_t*>(area);
    uint32_t* hm = reinterpret_cast<uint32_t*>(area + kGB * 4);  // kGB split 64-bit sums
    cbar();
    for (uint32_t i = threadIdx.x; i < kGB; i += kCons) {
        hc[i] = 0;
        hm[2 * i] = 0;
        hm[2 * i + 1] = 0;
    }
    cbar();
    g_for_keys(g, [&](uint32_t col, uint32_t key, bool valid) {
        if (!valid || !g_in(g, key, col)) return;
        float d;
        const uint32_t b = g_bin(g, key, d);
        atomicAdd(&hc[b], 1u);
        if (weighted) add_u64_split(&hm[2 * b], g_tw(d, b));
    });
    cbar();
    team_hist(g, hc, weighted ? hm : nullptr, kGB, c);
    constexpr uint32_t kPer = kGB / kCons;
    uint32_t lc[kPer], sc = 0;
    double lm[kPer], sm = 0.0;
#pragma unroll
    for (uint32_t j = 0; j < kPer; ++j) {
        const uint32_t b = threadIdx.x * kPer + j;
        lc[j] = hc[b];
        const unsigned long long mb = weighted ? get_u64_split(&hm[2 * b]) : 0ull;
        lm[j] = mb ? g_bin_scale(b) * (static_cast<double>(mb) / kGUnit) : 0.0;
        sc += lc[j];
        sm += lm[j];
    }
    uint32_t tc;
    uint32_t rc = cscan_excl(sc, &tc, c);
    double tm = 0.0, rm = 0.0;
    if (weighted) rm = cscan_excl_f64(sm, &tm, c);
#pragma unroll
    for (uint32_t j = 0; j < kPer; ++j) {
        const uint32_t b = threadIdx.x * kPer + j;
        pc[b] = rc;
        rc += lc[j];
        if (weighted) {
            pm[b] = rm;
            rm += lm[j];
        }
    }
    if (threadIdx.x == kCons - 1) {
        pc[kGB] = tc;
        if (weighted) pm[kGB] = tm;
    }
    cbar();
    *Z = tm;
    return tc;
}

struct GLoc {
    bool found;
    uint32_t key, col;  // the element
    uint32_t idx;       // its canonical position in K0
    double through;     // the mass (or count) of K0 through it
};

struct GSpan {          // the K0 members with distance bin b1 and key in [lo, hi]
    uint32_t b1, lo, hi;
    uint32_t above_cnt;  // K0 elements before the span
    double above_mass;
    uint32_t n;          // K0 elements in the span
};

__device__ __forceinline__ bool g_member(const GRow g, const GSpan s, uint32_t key,
                                         uint32_t col) {
    if (key < s.lo || key > s.hi || !g_in(g, key, col)) return false;
    float d;
    return g_bin(g, key, d) == s.b1;
}

// Smallest and largest key of the span's members.
__device__ __forceinline__ void g_minmax(const GRow g, GSpan& s, Ctl& c) {
    uint32_t lo = 0xffffffffu, hi = 0;
    g_for_keys(g, [&](uint32_t col, uint32_t key, bool valid) {
        if (valid && g_member(g, s, key, col)) {
            lo = min(lo, key);
            hi = max(hi, key);
        }
    });
    lo = cmin_u32(lo, c);
    hi = cmax_u32(hi, c);
    s.hi = team_max(g, hi, &lo, c);
    s.lo = lo;
}

// The span's members as rank keys, sorted descending into `sorted`
// (gathered in `buf`); returns their number (at most kGL).
__device__ __forceinline__ uint32_t g_gather_sorted(const GRow g, const GSpan s, uint32_t blo, uint32_t bhi,
                                    uint64_t* buf, uint64_t* sorted, Ctl& c) {
    cbar();
    if (threadIdx.x == 0) c.bc_u32[2] = 0;
    cbar();
    g_for_keys(g, [&](uint32_t col, uint32_t key, bool valid) {
        bool in = valid && key >= s.lo && key <= s.hi && g_in(g, key, col);
        if (in) {
            float d;
            const uint32_t b = g_bin(g, key, d);
            in = b >= blo && b <= bhi;
        }
        warp_push(in, rank_key(key, g.tok0 + col), buf, kGL, &c.bc_u32[2]);
    });
    cbar();
    const uint32_t n = team_gather(g, buf, min(c.bc_u32[2], kGL), c);
    sort_desc(buf, n, sorted);
    return n;
}

// The first of n members lk[0..n) (sorted, canonical order) at which the
// mass, summed from `above` with exact weights in canonical order, reaches
// tau (> tau when strict); the last member when none does.  Each thread sums
// a run of four consecutive members, then the runs' sums are scanned.  The
// member's index goes to c.bc_u32[0] and the mass through it to c.bc_u64[0].
__device__ __forceinline__ void g_scan_mass(const GRow g, const uint64_t* lk, uint32_t n,
                                            double above, double tau, bool strict, Ctl& c) {
    constexpr uint32_t kRun = kGL / kCons;
    const uint32_t i0 = threadIdx.x * kRun;
    double run[kRun];
    double acc = 0.0;
#pragma unroll
    for (uint32_t j = 0; j < kRun; ++j) {
        if (i0 + j < n) acc += g_weight(g, static_cast<uint32_t>(lk[i0 + j] >> 32));
        run[j] = acc;
    }
    double all;
    const double off = above + cscan_excl_f64(acc, &all, c);
    uint32_t hit = 0xffffffffu;
#pragma unroll
    for (uint32_t j = 0; j < kRun; ++j) {
        const double S = off + run[j];
        if (i0 + j < n && (strict ? (S > tau) : (S >= tau))) hit = min(hit, i0 + j);
    }
    hit = cmin_u32(hit, c);
    const uint32_t sel = hit == 0xffffffffu ? n - 1 : hit;
#pragma unroll
    for (uint32_t j = 0; j < kRun; ++j) {
        if (i0 + j == sel) {
            c.bc_u32[0] = sel;
            c.bc_u64[0] = static_cast<uint64_t>(__double_as_longlong(off + run[j]));
        }
    }
}

// The located element inside a span of at most kGL members: exact weights
// summed in canonical order from the mass above the span.
__device__ __forceinline__ GLoc g_final(const GRow g, const GSpan s, bool mass, double tau, bool strict,
                        unsigned char* area, Ctl& c) {
    uint64_t* buf = reinterpret_cast<uint64_t*>(area);
    uint64_t* lk = reinterpret_cast<uint64_t*>(area + kGL * 8);
    const uint32_t n = g_gather_sorted(g, s, s.b1, s.b1, buf, lk, c);
    GLoc res{false, 0, 0, 0, 0.0};
    if (n == 0) return res;
    if (!mass) {
        if (threadIdx.x == 0) {
            const double pos = tau - static_cast<double>(s.above_cnt) - 1.0;
            const uint32_t sel = pos <= 0.0 ? 0u : min(n - 1, static_cast<uint32_t>(pos));
            c.bc_u32[0] = sel;
            c.bc_u64[0] = static_cast<uint64_t>(
                __double_as_longlong(static_cast<double>(s.above_cnt + sel + 1)));
        }
    } else {
        g_scan_mass(g, lk, n, s.above_mass, tau, strict, c);
    }
    cbar();
    const uint32_t sel = c.bc_u32[0];
    res.found = true;
    res.key = static_cast<uint32_t>(lk[sel] >> 32);
    res.col = rank_token(lk[sel]) - g.tok0;
    res.idx = s.above_cnt + sel;
    res.through = __longlong_as_double(static_cast<long long>(c.bc_u64[0]));
    cbar();
    return res;
}

// The j-th smallest column among the K0 members holding `key`: a radix over
// the column bits, 11 then 9 bits (columns < 2^20).
__device__ __forceinline__ uint32_t g_tie_col(const GRow g, uint32_t key, uint32_t j, unsigned char* area,
                              Ctl& c) {
    uint32_t* h = reinterpret_cast<uint32_t*>(area);
    uint32_t prefix = 0, need = j;
    for (int level = 0; level < 2; ++level) {
        const uint32_t nb = level == 0 ? 2048u : 512u;
        cbar();
        for (uint32_t i = threadIdx.x; i < nb; i += kCons) h[i] = 0;
        cbar();
        g_for_keys(g, [&](uint32_t col, uint32_t k, bool valid) {
            if (valid && k == key && g_in(g, k, col) && (level == 0 || (col >> 9) == prefix))
                atomicAdd(&h[level == 0 ? (col >> 9) : (col & 511u)], 1u);
        });
        cbar();
        team_hist(g, h, nullptr, nb, c);
        if (threadIdx.x == 0) {
            uint32_t left = need, d = 0;
            for (; d < nb - 1; ++d) {
                if (left < h[d]) break;
                left -= h[d];
            }
            c.bc_u32[0] = d;
            c.bc_u32[1] = left;
        }
        cbar();
        if (level == 0) prefix = c.bc_u32[0];
        else prefix = (prefix << 9) | c.bc_u32[0];
        need = c.bc_u32[1];
    }
    return prefix;
}

// The located element in a tie group (a span holding one key).
__device__ __forceinline__ GLoc g_tie(const GRow g, const GSpan s, bool mass, double tau, bool strict,
                      unsigned char* area, Ctl& c) {
    const uint32_t key = s.lo;
    const double w = g_weight(g, key);
    double j;
    if (!mass) j = tau - static_cast<double>(s.above_cnt) - 1.0;
    else if (!(w > 0.0)) j = static_cast<double>(s.n) - 1.0;
    else if (strict) j = floor((tau - s.above_mass) / w);
    else j = ceil((tau - s.above_mass) / w) - 1.0;
    const uint32_t jj = j <= 0.0 ? 0u : (j >= static_cast<double>(s.n - 1) ? s.n - 1
                                                                          : static_cast<uint32_t>(j));
    GLoc res;
    res.found = true;
    res.key = key;
    res.col = g_tie_col(g, key, jj, area, c);
    res.idx = s.above_cnt + jj;
    res.through = mass ? s.above_mass + static_cast<double>(jj + 1) * w
                       : static_cast<double>(s.above_cnt + jj + 1);
    return res;
}

// The level-1 bin in which the running count (mass false: tau an integer
// count) or mass first reaches tau (>= tau, or > tau when strict): the first
// non-empty bin whose prefix through it reaches tau, else (rounding: the
// target lies past the last bin) the last non-empty bin; 0xffffffff when K0
// is empty.
__device__ __forceinline__ uint32_t g_bin_of(const uint32_t* pc, const double* pm, bool mass,
                                             double tau, bool strict, Ctl& c) {
    constexpr uint32_t kPer = kGB / kCons;
    uint32_t first = 0xffffffffu;
#pragma unroll
    for (uint32_t j = 0; j < kPer; ++j) {
        const uint32_t b = threadIdx.x * kPer + j;
        const bool hit = mass ? (strict ? pm[b + 1] > tau : pm[b + 1] >= tau)
                              : static_cast<double>(pc[b + 1]) >= tau;
        if (hit && first == 0xffffffffu && pc[b + 1] > pc[b]) first = b;
    }
    first = cmin_u32(first, c);
    if (first == 0xffffffffu) {
        uint32_t last = 0;
        for (uint32_t j = 0; j < kPer; ++j) {
            const uint32_t b = threadIdx.x * kPer + j;
            if (pc[b + 1] > pc[b]) last = b + 1;
        }
        last = cmax_u32(last, c);
        first = last == 0 ? 0xffffffffu : last - 1;
    }
    return first;
}

// First K0 element at which the running count (mass false: tau an integer
// count) or mass reaches tau (>= tau, or > tau when strict).
__device__ __forceinline__ GLoc g_locate(const GRow g, const uint32_t* pc, const double* pm, bool mass,
                         double tau, bool strict, unsigned char* area, Ctl& c) {
    constexpr uint32_t kPer = kGB / kCons;
    const uint32_t first = g_bin_of(pc, pm, mass, tau, strict, c);
    if (first == 0xffffffffu) return GLoc{false, 0, 0, 0, 0.0};
    GSpan s;
    s.b1 = first;
    s.lo = 0;
    s.hi = 0xffffffffu;
    s.above_cnt = pc[first];
    s.above_mass = mass ? pm[first] : 0.0;
    s.n = pc[first + 1] - s.above_cnt;
    const double scale = g_bin_scale(first);
    bool bounded = false;
    for (int level = 0; level < 6; ++level) {
        if (s.n <= kGL) return g_final(g, s, mass, tau, strict, area, c);
        if (!bounded) {
            g_minmax(g, s, c);
            bounded = true;
        }
        if (s.lo == s.hi) return g_tie(g, s, mass, tau, strict, area, c);
        // key sub-bins of the span, highest keys first
        const uint32_t span = s.hi - s.lo;
        const int sh = span > kGB - 1 ? (32 - __clz(span)) - 11 : 0;
        const uint32_t top = span >> sh;
        uint32_t* hc = reinterpret_cast<uint32_t*>(area);
        uint32_t* hm = reinterpret_cast<uint32_t*>(area + kGB * 4);  // split 64-bit sums
        cbar();
        for (uint32_t i = threadIdx.x; i < kGB; i += kCons) {
            hc[i] = 0;
            hm[2 * i] = 0;
            hm[2 * i + 1] = 0;
        }
        cbar();
        g_for_keys(g, [&](uint32_t col, uint32_t key, bool valid) {
            if (!valid || !g_member(g, s, key, col)) return;
            const uint32_t sb = top - ((key - s.lo) >> sh);
            atomicAdd(&hc[sb], 1u);
            if (mass) {
                float d;
                g_bin(g, key, d);
                add_u64_split(&hm[2 * sb], g_tw(d, s.b1));
            }
        });
        cbar();
        team_hist(g, hc, mass ? hm : nullptr, kGB, c);
        uint32_t lc[kPer], sc = 0;
        double lm[kPer], sm = 0.0;
#pragma unroll
        for (uint32_t j = 0; j < kPer; ++j) {
            const uint32_t b = threadIdx.x * kPer + j;
            lc[j] = hc[b];
            lm[j] = mass ? scale * (static_cast<double>(get_u64_split(&hm[2 * b])) / kGUnit) : 0.0;
            sc += lc[j];
            sm += lm[j];
        }
        uint32_t tc;
        const uint32_t rc0 = cscan_excl(sc, &tc, c);
        double tm = 0.0, rm0 = 0.0;
        if (mass) rm0 = cscan_excl_f64(sm, &tm, c);
        uint32_t hit = 0xffffffffu, last = 0;
        {
            uint32_t rc = rc0;
            double rm = rm0;
#pragma unroll
            for (uint32_t j = 0; j < kPer; ++j) {
                const uint32_t b = threadIdx.x * kPer + j;
                if (lc[j]) {
                    last = b + 1;
                    const bool h = mass ? (strict ? s.above_mass + rm + lm[j] > tau
                                                  : s.above_mass + rm + lm[j] >= tau)
                                        : static_cast<double>(s.above_cnt + rc + lc[j]) >= tau;
                    if (h && hit == 0xffffffffu) hit = b;
                }
                rc += lc[j];
                rm += lm[j];
            }
        }
        const uint32_t fh = cmin_u32(hit, c);
        const uint32_t fl = cmax_u32(last, c);
        const uint32_t sb = fh != 0xffffffffu ? fh : fl - 1;  // rounding: the last non-empty
        // the owner of sub-bin sb publishes the count and mass before it
        if (threadIdx.x == sb / kPer) {
            uint32_t rc = rc0;
            double rm = rm0;
            uint32_t own = 0;
#pragma unroll
            for (uint32_t j = 0; j < kPer; ++j) {
                if (j < sb % kPer) {
                    rc += lc[j];
                    rm += lm[j];
                } else if (j == sb % kPer) {
                    own = lc[j];
                }
            }
            c.bc_u32[0] = rc;
            c.bc_u64[0] = static_cast<uint64_t>(__double_as_longlong(rm));
            c.bc_u32[1] = own;
        }
        cbar();
        const uint32_t lo2 = s.lo + ((top - sb) << sh);
        const uint32_t hi2 = sh ? min(s.hi, lo2 + ((1u << sh) - 1u)) : lo2;
        s.above_cnt += c.bc_u32[0];
        if (mass) s.above_mass += __longlong_as_double(static_cast<long long>(c.bc_u64[0]));
        s.n = c.bc_u32[1];
        s.lo = lo2;
        s.hi = hi2;
        cbar();
    }
    return g_final(g, s, mass, tau, strict, area, c);
}

// ---- distribution output of a general row: K0's first n_emit members in
// canonical order with their values, and w_i / Z_r for the first r_cnt.
struct GOut {
    int32_t* tokens;  // the distribution arrays (any may be null)
    float* values;
    double* probs;
    size_t base;      // row offset in the distribution arrays
    uint32_t n_emit;
    uint32_t r_cnt;
    double Zr;
};

__device__ __forceinline__ void g_write_list(const GRow g, const GOut o, const uint64_t* lk,
                             uint32_t n, uint32_t pos) {
    for (uint32_t i = threadIdx.x; i < n; i += kCons) {
        const uint32_t p = pos + i;
        if (p >= o.n_emit) break;
        const uint32_t key = static_cast<uint32_t>(lk[i] >> 32);
        if (o.tokens) o.tokens[o.base + p] = static_cast<int32_t>(rank_token(lk[i]));
        if (o.values) o.values[o.base + p] = key_float(key);
        if (o.probs) o.probs[o.base + p] = p < o.r_cnt ? g_weight(g, key) / o.Zr : 0.0;
    }
    cbar();
}

// The K0 members holding `key` in column order (a tie group), at pos: each
// round of the pass covers 4 * kCons consecutive columns in thread order.
__device__ __forceinline__ void g_write_tie(const GRow g, const GOut o, uint32_t key, uint32_t pos,
                                            Ctl& c) {
    const float val = key_float(key);
    const double w = g_weight(g, key);
    g_pass16(reinterpret_cast<const unsigned char*>(g.keys), static_cast<uint64_t>(g.V) * 4, g.stage,
             c, [&](uint32_t gi, const uint4& kv, bool) {
                 const uint32_t kk[4] = {kv.x, kv.y, kv.z, kv.w};
                 uint32_t flags = 0;
#pragma unroll
                 for (uint32_t e = 0; e < 4; ++e) {
                     const uint32_t col = gi * 4 + e;
                     if (col < g.V && kk[e] == key && g_in(g, key, col)) flags |= 1u << e;
                 }
                 uint32_t tot;
                 uint32_t off = cscan_excl(__popc(flags), &tot, c);
                 while (flags) {
                     const uint32_t e = __ffs(flags) - 1;
                     flags &= flags - 1;
                     const uint32_t p = pos + off++;
                     if (p < o.n_emit) {
                         if (o.tokens) o.tokens[o.base + p] = static_cast<int32_t>(g.tok0 + gi * 4 + e);
                         if (o.values) o.values[o.base + p] = val;
                         if (o.probs) o.probs[o.base + p] = p < o.r_cnt ? w / o.Zr : 0.0;
                     }
                 }
                 pos += tot;
             });
    cbar();
}

// Counts of the key sub-bins of a span (highest keys first) into h.
__device__ __forceinline__ void g_subcount(const GRow g, const GSpan s, int sh, uint32_t top, uint32_t* h) {
    cbar();
    for (uint32_t i = threadIdx.x; i < kGB; i += kCons) h[i] = 0;
    cbar();
    g_for_keys(g, [&](uint32_t col, uint32_t key, bool valid) {
        if (valid && g_member(g, s, key, col)) atomicAdd(&h[top - ((key - s.lo) >> sh)], 1u);
    });
    cbar();
}

// A distance bin of more than kGL members: its key sub-bins depth first
// (sub-bin counts of the open levels in scratch, the current one in shared
// memory), groups of consecutive small sub-bins gathered and sorted, single
// keys written as tie groups.
__device__ __forceinline__ void g_emit_big(const GRow g, const GOut o, GSpan root,
                           uint32_t pos, uint32_t* subh, unsigned char* area, Ctl& c) {
    uint64_t* buf = reinterpret_cast<uint64_t*>(area);
    uint64_t* lk = reinterpret_cast<uint64_t*>(area + kGL * 8);
    uint32_t* hs = reinterpret_cast<uint32_t*>(area + kArea - kGB * 4);
    struct Frame {
        uint32_t lo, hi, top, sb, pos;
        int sh;
    };
    Frame st[kEmitDepth];
    int d = 0;
    auto open = [&](int depth, uint32_t lo, uint32_t hi, uint32_t p) {
        Frame& f = st[depth];
        f.lo = lo;
        f.hi = hi;
        const uint32_t span = hi - lo;
        f.sh = span > kGB - 1 ? (32 - __clz(span)) - 11 : 0;
        f.top = span >> f.sh;
        f.sb = 0;
        f.pos = p;
        GSpan s = root;
        s.lo = lo;
        s.hi = hi;
        g_subcount(g, s, f.sh, f.top, hs);
        for (uint32_t i = threadIdx.x; i < kGB; i += kCons) subh[depth * kGB + i] = hs[i];
        cbar();
    };
    if (root.lo == root.hi) {
        g_write_tie(g, o, root.lo, pos, c);
        return;
    }
    open(0, root.lo, root.hi, pos);
    while (d >= 0) {
        Frame& f = st[d];
        bool descended = false;
        while (f.sb <= f.top && f.pos < o.n_emit) {
            const uint32_t cnt = hs[f.sb];
            if (cnt == 0) {
                ++f.sb;
                continue;
            }
            const uint32_t lo2 = f.lo + ((f.top - f.sb) << f.sh);
            const uint32_t hi2 = f.sh ? min(f.hi, lo2 + ((1u << f.sh) - 1u)) : lo2;
            if (cnt > kGL) {
                if (lo2 == hi2 || d + 1 >= static_cast<int>(kEmitDepth)) {
                    g_write_tie(g, o, lo2, f.pos, c);
                    f.pos += cnt;
                    ++f.sb;
                    continue;
                }
                const uint32_t p = f.pos;
                f.pos += cnt;
                ++f.sb;
                open(d + 1, lo2, hi2, p);
                ++d;
                descended = true;
                break;
            }
            // consecutive sub-bins holding at most kGL members in all
            uint32_t e = f.sb + 1, tot = cnt;
            while (e <= f.top && tot + hs[e] <= kGL) tot += hs[e++];
            GSpan s = root;
            s.lo = f.lo + ((f.top - (e - 1)) << f.sh);
            s.hi = hi2;
            const uint32_t n = g_gather_sorted(g, s, root.b1, root.b1, buf, lk, c);
            g_write_list(g, o, lk, n, f.pos);
            f.pos += n;
            f.sb = e;
        }
        if (descended) continue;
        --d;
        if (d >= 0) {  // back to the parent's sub-bin counts
            cbar();
            for (uint32_t i = threadIdx.x; i < kGB; i += kCons) hs[i] = __ldcg(&subh[d * kGB + i]);
            cbar();
        }
    }
}

__device__ __forceinline__ void g_emit(const GRow g, const GOut o, const uint32_t* pc, uint32_t* subh,
                       unsigned char* area, Ctl& c) {
    uint64_t* buf = reinterpret_cast<uint64_t*>(area);
    uint64_t* lk = reinterpret_cast<uint64_t*>(area + kGL * 8);
    uint32_t* bcnt = reinterpret_cast<uint32_t*>(area + kGL * 16);  // level-1 counts
    cbar();
    for (uint32_t b = threadIdx.x; b < kGB; b += kCons) bcnt[b] = pc[b + 1] - pc[b];
    cbar();
    uint32_t pos = 0, b = 0;
    while (b < kGB && pos < o.n_emit) {
        const uint32_t cnt = bcnt[b];
        if (cnt == 0) {
            ++b;
            continue;
        }
        GSpan s;
        s.b1 = b;
        s.lo = 0;
        s.hi = 0xffffffffu;
        s.above_cnt = pos;
        s.above_mass = 0.0;
        s.n = cnt;
        if (cnt > kGL) {
            g_minmax(g, s, c);
            g_emit_big(g, o, s, pos, subh, area, c);
            // the level-1 counts live beside the sub-bin counts: reload them
            cbar();
            for (uint32_t i = threadIdx.x; i < kGB; i += kCons) bcnt[i] = pc[i + 1] - pc[i];
            cbar();
            pos += cnt;
            ++b;
            continue;
        }
        uint32_t e = b + 1, tot = cnt;
        while (e < kGB && tot + bcnt[e] <= kGL) tot += bcnt[e++];
        const uint32_t n = g_gather_sorted(g, s, b, e - 1, buf, lk, c);
        g_write_list(g, o, lk, n, pos);
        pos += n;
        b = e;
    }
}

// One deferred row by this CTA's part of its team; the leader (rank 0)
// writes every output.  pcpm: shared memory for the level-1 prefix counts
// (kGB + 1) and masses (kGB + 1 doubles).
template <int DT>
__device__ __forceinline__ void general_row(const SampleArgs& a, const Row& r, unsigned char* area,
                                            uint4* stage, unsigned char* pcpm, GTeam& t, Ctl& c) {
    const uint32_t V = a.vocab;
    const uint32_t tok0 = a.col_begin;
    const bool lead = t.rank == 0;
    uint32_t* keys = a.scratch + static_cast<size_t>(r.v) * a.scratch_stride;
    uint32_t* aux = keys + ((V + 3u) & ~3u);
    uint32_t* subh = aux + kAuxSub;
    uint32_t* pc = reinterpret_cast<uint32_t*>(pcpm);
    double* pm = reinterpret_cast<double*>(pcpm + kPcBytes);
    const unsigned char* row = row_ptr<DT>(a, r.v);
    // this CTA's columns: 32-aligned chunks, one per member
    const uint32_t chunk = ((V + t.size - 1) / t.size + 31u) & ~31u;
    const uint32_t c0 = min(V, t.rank * chunk), c1 = min(V, c0 + chunk);
    // this call's penalised columns (bitmap plus additional tokens) in
    // shared memory when they fit
    const uint32_t words = (V + 31) / 32;
    const uint32_t* pbm = nullptr;
    if (r.pen && words * 4 <= kArea) {
        uint32_t* sbm = reinterpret_cast<uint32_t*>(area);
        cbar();
        for (uint32_t i = c0 / 32 + threadIdx.x; i < (c1 + 31) / 32; i += kCons) sbm[i] = r.gbm[i];
        cbar();
        for (uint32_t e = threadIdx.x; e < r.n_extra; e += kCons) {
            const uint32_t col = static_cast<uint32_t>(r.extra[e]) - tok0;
            if (col >= c0 && col < c1) atomicOr(&sbm[col >> 5], 1u << (col & 31));
        }
        cbar();
        pbm = sbm;
    }
    GRow g;
    g.keys = keys;
    g.stage = stage;
    g.ctl = &c;
    g.t = &t;
    g.c0 = c0;
    g.c1 = c1;
    g.V = V;
    g.tok0 = tok0;
    const uint32_t M_key =
        team_max(g, g_keys<DT>(a, r, row, pbm, keys, V, c0, c1, g.stage, c), nullptr, c);
    Q38S_TT(r.v, 6);
    g.M = key_float(M_key);
    g.minp_key = 0;
    g.has_cut = false;
    g.cut_key = 0;
    g.cut_col = 0;
    auto fail = [&](int32_t status) {
        if (lead) row_error(a, r, t.failed ? Q38S_ROW_TIMEOUT : status);
    };
    if (a.mode != kModeShardTopK && (M_key <= kNegInfKey || isinf(g.M))) {
        fail(Q38S_ROW_NO_FINITE);
        return;
    }
    // smallest key whose weight reaches min_p
    if (r.minp && M_key > kNegInfKey && !isinf(g.M)) {
        if (threadIdx.x == 0) {
            const double floor_w = static_cast<double>(r.p.min_p);
            uint32_t lo = kNegInfKey, hi = M_key;  // weight(M) = 1 >= min_p
            while (lo < hi) {
                const uint32_t mid = lo + (hi - lo) / 2;
                if (g_weight(g, mid) >= floor_w) hi = mid;
                else lo = mid + 1;
            }
            c.bc_u32[3] = hi;
        }
        cbar();
        g.minp_key = c.bc_u32[3];
    }
    // |K0| and the top-k cut
    uint32_t n0 = V;
    if (r.minp || r.k_eff) {
        uint32_t cnt = 0;
        g_for_keys(g, [&](uint32_t, uint32_t key, bool valid) {
            cnt += valid && key >= g.minp_key;
        });
        n0 = team_sum(g, csum_u32(cnt, c), c);
        if (r.k_eff && r.k_eff < n0) {
            double unused;
            g_level1(g, false, area, pc, pm, &unused, c);
            const GLoc cut = g_locate(g, pc, pm, false, static_cast<double>(r.k_eff), false, area, c);
            g.has_cut = true;
            g.cut_key = cut.key;
            g.cut_col = cut.col;
            n0 = r.k_eff;
        }
    }
    Q38S_TT(r.v, 10);
    if (n0 <= kGL) {
        // gather K0, sort, and the exact epilogue of the fast path
        uint64_t* buf = reinterpret_cast<uint64_t*>(area);
        uint64_t* lk = reinterpret_cast<uint64_t*>(area + kGL * 8);
        GSpan s;
        s.b1 = 0;
        s.lo = 0;
        s.hi = 0xffffffffu;
        const uint32_t m = g_gather_sorted(g, s, 0, kGB - 1, buf, lk, c);
        if (!lead) return;
        if (t.failed) {
            fail(Q38S_ROW_TIMEOUT);
            return;
        }
        double* w = reinterpret_cast<double*>(area);  // over the dead gather buffer
        double* S = reinterpret_cast<double*>(area + kGL * 16);
        row_output(a, r, lk, m, w, S, c);
        return;
    }
    if (a.mode == kModeShardTopK) {  // candidate lists hold at most kLeaderCap
        fail(Q38S_ROW_NORMALIZATION);
        return;
    }
    double Z = 0.0;
    g_level1(g, true, area, pc, pm, &Z, c);
    Q38S_TT(r.v, 13);
    if (!(Z > 0.0) || !isfinite(Z)) {
        fail(Q38S_ROW_NORMALIZATION);
        return;
    }
    uint32_t r_cnt = n0;
    double Zr = Z;
    GLoc cut{false, 0, 0, 0, 0.0};
    if (r.p.top_p < 1.0f) {
        cut = g_locate(g, pc, pm, true, static_cast<double>(r.p.top_p) * Z, false, area, c);
        if (cut.found) {
            r_cnt = cut.idx + 1;
            Zr = cut.through;
        }
    }
    Q38S_TT(r.v, 14);
    const double draw = uniform01(r.rng_before + kGamma) * Zr;
    GLoc sel = g_locate(g, pc, pm, true, draw, true, area, c);
    if (!sel.found || sel.idx >= r_cnt) {
        // no prefix sum exceeds the draw (rounding): the last retained element
        // (sampling.cc:137-144)
        sel = cut.found ? cut
                        : g_locate(g, pc, pm, false, static_cast<double>(r_cnt), false, area, c);
    }
    Q38S_TT(r.v, 15);
    if (!lead) return;
    if (!sel.found || t.failed) {
        fail(Q38S_ROW_NORMALIZATION);
        return;
    }
    write_decision(a, r, static_cast<int32_t>(tok0 + sel.col), Q38S_ROW_OK);
    if (a.dist.capacity) {
        if (threadIdx.x == 0) {
            if (a.dist.n_candidates) a.dist.n_candidates[r.v] = n0;
            if (a.dist.n_retained) a.dist.n_retained[r.v] = r_cnt;
            if (a.dist.total) a.dist.total[r.v] = Zr;
            if (a.dist.draw) a.dist.draw[r.v] = draw;
        }
        if (a.dist.tokens || a.dist.values || a.dist.probs) {
            // the leader alone, over the whole row (every member's keys are
            // visible after the team's barriers)
            cbar();
            if (threadIdx.x == 0) t.size = 1;
            cbar();
            g.c0 = 0;
            g.c1 = V;
            GOut o;
            o.tokens = a.dist.tokens;
            o.values = a.dist.values;
            o.probs = a.dist.probs;
            o.base = static_cast<size_t>(r.v) * a.dist.capacity;
            o.n_emit = min(n0, a.dist.capacity);
            o.r_cnt = r_cnt;
            o.Zr = Zr;
            g_emit(g, o, pc, subh, area, c);
        }
    }
}

// Completes a row once its candidate list (or failure) is known.
template <int DT>
__device__ __forceinline__ void finish_row(const SampleArgs& a, const Row& r, uint32_t flags,
                                           const uint64_t* sorted, uint32_t keep,
                                           unsigned char* area, Ctl& c) {
    if (flags & kFTimeout) {
        row_error(a, r, Q38S_ROW_TIMEOUT);
    } else if (flags & kFInf) {
        row_error(a, r, Q38S_ROW_NO_FINITE);
    } else if (flags & kFOverflow) {
        // the general path runs in general_kernel, launched behind this one
        // (or by the caller, told through the row's status); the row's team
        // words start from zero
        uint4* tw = reinterpret_cast<uint4*>(a.scratch + static_cast<size_t>(r.v) * a.scratch_stride +
                                             ((a.vocab + 3u) & ~3u) + kTeamOff);
        for (uint32_t i = threadIdx.x; i < (kTeamSync + 2 * kSlotWords) / 4; i += kCons)
            tw[i] = make_uint4(0u, 0u, 0u, 0u);
        cbar();
        if (threadIdx.x == 0) a.deferred[r.v] = 1u;
        if (a.host_general) write_decision(a, r, -1, kRowDeferred);
        return;
    } else {
        double* w = reinterpret_cast<double*>(area);  // over the dead candidate buffer
        row_output(a, r, sorted, keep, w, w + kFinal, c);
    }
    row_done(a, area, c);
}

// ------------------------------------------------------------ general kernel
// The rows the stream kernel deferred (deferred[v] != 0; the stream kernel
// writes every row's flag), launched right behind the stream kernel as its
// programmatic dependent: it may be scheduled early and waits
// (griddepcontrol.wait) until the stream kernel has completed.  Every CTA
// reads all flags.  With D deferred rows and G CTAs: D >= G, CTA i takes the
// deferred rows of rank i, i + G, ... alone; D < G, the CTAs form D teams of
// G / D (team j takes the deferred row of rank j; CTAs past D * (G / D) have
// nothing to do).  With no deferred row every CTA returns at once.  The
// stream kernel stays free of the general path's code.
template <int DT>
__global__ void __launch_bounds__(kCons, 1) general_kernel(const SampleArgs a) {
    extern __shared__ __align__(1024) unsigned char gsm[];
    __shared__ Ctl c;
    __shared__ Row rs;
    __shared__ GTeam gt;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    unsigned char* area = gsm;
    uint4* stage = reinterpret_cast<uint4*>(gsm + kArea);
    unsigned char* pcpm = gsm + kArea + kStageBytes;
    // D: the deferred rows
    uint32_t D = 0;
    for (uint32_t base = 0; base < a.vrows; base += kCons) {
        const uint32_t v = base + threadIdx.x;
        D += csum_u32(v < a.vrows && __ldcg(&a.deferred[v]) != 0 ? 1u : 0u, c);
    }
    if (D == 0) return;
    const uint32_t G = gridDim.x;
    const uint32_t T = D >= G ? 1u : G / D;     // team size
    const uint32_t team = blockIdx.x / T;       // D >= G: the CTA's first rank
    if (team >= D) return;
    // the deferred rows in rank order, chunk by chunk; this CTA takes ranks
    // team, team + G, ... (T == 1) or rank team alone (T > 1)
    __shared__ uint32_t taken_rows[kCons];
    uint32_t seen = 0;
    for (uint32_t base = 0; base < a.vrows; base += kCons) {
        const uint32_t v = base + threadIdx.x;
        const uint32_t mine = v < a.vrows && __ldcg(&a.deferred[v]) != 0 ? 1u : 0u;
        uint32_t n;
        const uint32_t pos = seen + cscan_excl(mine, &n, c);
        // the first rank this CTA takes at or after `seen`
        uint32_t first = 0xffffffffu;
        if (team >= seen) first = team;
        else if (T == 1) first = team + ((seen - team + G - 1) / G) * G;
        uint32_t taken = 0;
        if (first < seen + n) taken = T == 1 ? (seen + n - 1 - first) / G + 1 : 1u;
        if (mine && pos >= first && pos < seen + n) {
            if (T == 1 && (pos - first) % G == 0) taken_rows[(pos - first) / G] = v;
            if (T > 1 && pos == first) taken_rows[0] = v;
        }
        cbar();
        for (uint32_t i = 0; i < taken; ++i) {
            const uint32_t vr = taken_rows[i];
            cbar();
            if (threadIdx.x == 0) {
                load_row(a, vr, rs);
                gt.rank = T == 1 ? 0u : blockIdx.x % T;
                gt.size = T;
                uint32_t* aux = a.scratch + static_cast<size_t>(vr) * a.scratch_stride +
                                ((a.vocab + 3u) & ~3u);
                gt.sync = aux + kTeamOff;
                gt.slots = aux + kTeamOff + kTeamSync;
                gt.phase = 0;
                gt.failed = 0;
            }
            cbar();
            general_row<DT>(a, rs, area, stage, pcpm, gt, c);
            if (gt.rank == 0) row_done(a, area, c);
            cbar();
        }
        seen += n;
        cbar();  // taken_rows is rewritten by the next chunk
    }
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

__device__ bool wait_full(const SampleArgs& a, Ctl& c, uint32_t slot, uint32_t phase) {
    if (mbar_try_wait(&c.full[slot], phase)) return true;
    // the limit (a test may shorten the first CTA's) is read only when waiting
    const long long limit =
        (a.test_withhold && blockIdx.x == 0) ? a.test_wait_cycles : kWaitLimitCycles;
    const long long start = clock64();
    while (!mbar_try_wait(&c.full[slot], phase)) {
        if (*reinterpret_cast<volatile uint32_t*>(&c.abort_flag)) return false;
        if (clock64() - start > limit) return false;
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
    if (a.test_withhold && blockIdx.x == 0) {  // failure injection: no copy at all
        atomicExch(&c.prod_done, 1u);
        return;
    }
    uint32_t g = 0;
    for (uint32_t u = blockIdx.x; u < n_units; u += gridDim.x) {
        const uint32_t v = u / S;
        uint32_t c0, c1;
        chunk_range(a.vocab, S, u % S, c0, c1);
        if (!unit_streams(a, v, c1 - c0, TC)) continue;
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
            // the tile's slice of the penalty bitmap rides along (the stream
            // reads the penalty bit of each thread's largest element)
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

template <int DT>
__global__ void __launch_bounds__(kBlock, 2) stream_kernel(const SampleArgs a) {
    extern __shared__ __align__(1024) unsigned char dsm[];
    __shared__ Ctl c;
    __shared__ Row rs;
    // the general kernel behind this one may be scheduled now, onto SMs this
    // grid leaves free; it waits for this grid's completion before it reads
    // anything this grid writes
    if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    constexpr uint32_t es = DT == Q38S_DTYPE_BF16 ? 2u : 4u;
    constexpr uint32_t pv = 16u / es;  // elements per 16-byte vector
    constexpr uint32_t TC = kTileBytes / es;
    constexpr int kU = kTileBytes / 16 / kCons;  // vectors per thread per tile
    constexpr unsigned kFull = 0xffffffffu;
    unsigned char* ring = dsm;
    unsigned char* area = dsm + kRing * kSlot;
    uint64_t* cand = reinterpret_cast<uint64_t*>(area);
    uint64_t* sorted = reinterpret_cast<uint64_t*>(area + kSorted);
    const uint32_t tid = threadIdx.x;

    if (tid == 0) {
        for (uint32_t i = 0; i < kRing; ++i) {
            mbar_init(&c.full[i], 1);
            mbar_init(&c.empty[i], kCons / 32);  // one arrival per consumer warp
        }
        mbar_init(&c.xfull, kHdrKeys / a.segs * a.segs);  // one per header key of a row
        mbar_init(&c.xdone, 1);       // the leader's
        c.abort_flag = 0;
        c.prod_done = 0;
        c.issued = 0;
        c.fail_g = 0xffffffffu;
        fence_mbar_init();
    }
    __syncthreads();
    // a row split into segments runs on one cluster: no CTA arrives on a
    // peer's barriers before the peer has initialised them
    if (a.segs > 1) cluster_sync_all();
    if (tid >= static_cast<uint32_t>(kCons)) {
        if (tid == static_cast<uint32_t>(kCons)) produce<DT>(a, ring, c);
        return;
    }

    // Consumers.  Per unit:
    //   stream   every tile of the unit, keeping per thread and tile the
    //            largest raw value of the thread's four vectors (an upper
    //            bound, in the area's tail) and the thread's largest raw
    //            value with its tile;
    //   theta    the exact values of the 256 threads' largest elements
    //            (distinct elements) give theta: their k-th largest, and
    //            for min-p rows M + ln(min_p) - slack with M their largest;
    //   gather   the thread's tiles whose bound reaches theta's raw bound are
    //            read again from global memory (L2 holds them: the unit has
    //            just streamed through) and their elements at or above
    //            theta join the candidate buffer.
    // The warps stream decoupled; block barriers come once per unit.
    const uint32_t warp = tid >> 5, lane = tid & 31;
    const uint32_t S = a.segs;
    const uint32_t n_units = a.vrows * S;
    uint32_t g = 0;     // tiles passed (the producer's order)
    uint32_t xrow = 0;  // multi-segment rows passed (the cluster barriers' parity)
    bool stop = false;  // this warp gave up on a copy (warp-uniform)
    (void)warp;
    for (uint32_t u = blockIdx.x; u < n_units; u += gridDim.x) {
        const uint32_t v = u / S, seg = u % S;
        uint32_t c0, c1;
        chunk_range(a.vocab, S, seg, c0, c1);
        const uint32_t ntiles = (c1 - c0 + TC - 1) / TC;
        Q38S_TT(u, 0);
        // one copy of the row context per CTA, in shared memory: it is
        // needed in the row's tail, and registers are scarce in the stream
        // loop (every consumer finished the previous unit at its last barrier)
        if (tid == 0) {
            load_row(a, v, rs);
            if (seg == 0) a.deferred[v] = 0u;  // set again if the row is deferred
        }
        cbar();
        const Row& r = rs;
        Q38S_TT(u, 1);
        const bool streams = unit_streams(a, v, c1 - c0, TC);
        const unsigned char* src_row = row_ptr<DT>(a, v);
        // per-thread tile bounds in the area's tail; candidates in its head
        uint16_t* bkey = reinterpret_cast<uint16_t*>(area + kArea) - ntiles * kCons;
        const uint32_t cap = min(kBuf, (kArea - ntiles * kCons * 2u) / 8u);
        if (tid == 0) {
            c.flags = 0;
            c.n_cand = 0;
#ifdef Q38S_TRACE
            c.bc_u32[3] = 0;
#endif
        }
        float tmax = -INFINITY;  // the thread's largest raw value ...
        uint32_t tcol = 0;       // ... the first column holding it
        uint32_t tpen = 0;       // ... and that column's bit of the state row's bitmap
        bool tnan = false;       // some block of the thread has only NaN maxima
        for (uint32_t t = 0; streams && t < ntiles; ++t, ++g) {
            const uint32_t slot = g % kRing;
            unsigned char* sl = ring + slot * kSlot;
            const uint32_t t0 = c0 + t * TC;
            const uint32_t n = min(c1 - t0, TC);
#ifdef Q38S_TRACE
            const long long tw0 = clock64();
#endif
            bool ok = !stop && wait_full(a, c, slot, (g / kRing) & 1u);
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
            // cannot move (ragged tail, unaligned rows) and -inf padding to
            // a whole vector
            const uint32_t bytes = n * es;
            const uint32_t bulk = a.use_tma ? (bytes & ~15u) : 0u;
            const uint32_t padded = ((n + pv - 1) / pv) * pv;
            if (bulk < bytes || padded != n) {
                const bool all_ok = !cbar_or(!ok);
                if (all_ok) {
                    const unsigned char* src = src_row + static_cast<size_t>(t0) * es;
                    for (uint32_t b = bulk + tid; b < bytes; b += kCons) sl[b] = src[b];
                    for (uint32_t j = n + tid; j < padded; j += kCons) {
                        if (DT == Q38S_DTYPE_BF16) reinterpret_cast<uint16_t*>(sl)[j] = 0xff80u;
                        else reinterpret_cast<uint32_t*>(sl)[j] = 0xff800000u;
                    }
                }
                fence_async_smem();  // generic writes before the slot's next bulk copy
                cbar();
            }
            // the largest raw value of the thread's vectors of this tile
            const uint4* vec = reinterpret_cast<const uint4*>(sl);
            const uint32_t nvec = padded / pv;
            float bm = -INFINITY;
            if (ok) {
                if (DT == Q38S_DTYPE_BF16) {
                    __nv_bfloat162 m2 = __float2bfloat162_rn(-INFINITY);
#pragma unroll
                    for (int q = 0; q < kU; ++q) {
                        const uint32_t j = tid + q * kCons;
                        if (j < nvec) {
                            const uint4 w = vec[j];
                            m2 = __hmax2(m2, __hmax2(__hmax2(*reinterpret_cast<const __nv_bfloat162*>(&w.x),
                                                             *reinterpret_cast<const __nv_bfloat162*>(&w.y)),
                                                     __hmax2(*reinterpret_cast<const __nv_bfloat162*>(&w.z),
                                                             *reinterpret_cast<const __nv_bfloat162*>(&w.w))));
                        }
                    }
                    bm = fmaxf(__low2float(m2), __high2float(m2));
                } else {
#pragma unroll
                    for (int q = 0; q < kU; ++q) {
                        const uint32_t j = tid + q * kCons;
                        if (j < nvec) bm = fmaxf(bm, vec_max<DT>(vec[j]));
                    }
                }
            }
            // bf16 rounded up: an upper bound of every element of the block
            bkey[t * kCons + tid] = __bfloat16_as_ushort(__float2bfloat16_ru(bm));
            if (bm > tmax) {
                // a new largest value: its first element (vector, then lane
                // of the vector) and penalty bit, from the slot
                tmax = bm;
                const uint32_t* sbm = reinterpret_cast<const uint32_t*>(sl + kTileBytes);
                uint32_t jm = 0xffffffffu;
#pragma unroll
                for (int q = kU - 1; q >= 0; --q) {
                    const uint32_t j = tid + q * kCons;
                    if (j < nvec && vec_max<DT>(vec[j]) == bm) jm = j;
                }
                if (jm != 0xffffffffu) {
                    const uint4 w = vec[jm];
                    uint32_t e = 0;
#pragma unroll
                    for (int i = static_cast<int>(pv) - 1; i >= 0; --i)
                        if (vec_elem<DT>(w, i) == bm) e = static_cast<uint32_t>(i);
                    const uint32_t idx = jm * pv + e;
                    tcol = t0 + idx;
                    tpen = r.pen ? (sbm[idx >> 5] >> (idx & 31)) & 1u : 0u;
                }
            }
            tnan |= bm != bm;
#ifdef Q38S_TRACE
            if (g_trace && u < 256 && t < 20 && lane == 0 && warp == 0)
                g_trace[119808 + static_cast<size_t>(u) * 20 + t] =
                    (static_cast<unsigned long long>(tw1 - tw0) << 32) |
                    static_cast<unsigned long long>(clock64() - tw1);
#endif
            // release the slot once every lane has read it; a slot whose
            // wait failed is never released (its copy may still land)
            __syncwarp();
            if (ok && lane == 0) mbar_arrive(&c.empty[slot]);
        }
        // ---- the exact value of the thread's largest element (one element
        // per thread keeps the k-th largest key a lower bound of the row's)
        uint32_t tk = 0;
        if (streams && !stop && tmax > -INFINITY) {
            const float vx = exact_pw(a, r, tmax, tcol, tpen << (tcol & 31));
            if (vx == INFINITY) atomicOr(&c.flags, kFInf);
            tk = float_key(vx);
        }
        c.tkey[tid] = tk;
        Q38S_TT(u, 15);
        const bool any_stop = cbar_or(stop);  // also publishes the keys
        Q38S_TT(u, 2);
        uint32_t theta = 0;
        bool overflow = !streams;
        if (streams && !any_stop) {
            // ---- theta: the k-th largest and the largest of the 256 keys
            // (warp 0)
            if (warp == 0) {
                uint32_t kk[kCons / 32], mx = 0, mn = 0xffffffffu, nz = 0;
#pragma unroll
                for (int i = 0; i < kCons / 32; ++i) {
                    kk[i] = c.tkey[lane + 32 * i];
                    mx = max(mx, kk[i]);
                    if (kk[i]) {
                        mn = min(mn, kk[i]);
                        ++nz;
                    }
                }
                mx = __reduce_max_sync(kFull, mx);
                mn = __reduce_min_sync(kFull, mn);
                nz = __reduce_add_sync(kFull, nz);
                uint32_t tt = 0;
                if (r.k_eff >= 1 && r.k_eff <= nz) {
                    // the k-th largest key lies in [mn, mx]: the bits above
                    // the highest one where those differ are fixed
                    const uint32_t diff = (mx ^ mn) & 0xffff0000u;
                    const int top = diff ? 31 - __clz(diff) : 15;
                    tt = top == 31 ? 0u : (mx & ~((2u << top) - 1u)) & 0xffff0000u;
#pragma unroll 1
                    for (int b = top; b >= 16; --b) {
                        const uint32_t cand = tt | (1u << b);
                        uint32_t cnt = 0;
#pragma unroll
                        for (int i = 0; i < kCons / 32; ++i) cnt += kk[i] >= cand ? 1u : 0u;
                        if (__reduce_add_sync(kFull, cnt) >= r.k_eff) tt = cand;
                    }
                }
                if (lane == 0) {
                    c.bc_u32[0] = tt;
                    c.bc_u32[1] = mx;
                }
            }
            cbar();
            theta = c.bc_u32[0];
            const uint32_t m0 = c.bc_u32[1];
            if (r.minp) theta = max(theta, minp_key(m0, r));
            Q38S_TR(u, 3, theta);
            Q38S_TT(u, 6);
            overflow = theta <= kNegInfKey && (c1 - c0) > cap;
        }
        if (streams && !any_stop && !overflow) {
            // ---- gather: every element whose exact value may reach theta
            const float rho = raw_bound(theta <= kNegInfKey ? -INFINITY : key_float(theta),
                                        r.p.temperature);
            auto consider = [&](float x, uint32_t col, uint32_t pw) {
                const float vx = exact_pw(a, r, x, col, pw);
                const uint32_t k = float_key(vx);
                if (vx == INFINITY) atomicOr(&c.flags, kFInf);
                if (k >= theta) {
                    const uint32_t at = atomicAdd(&c.n_cand, 1u);
                    if (at < cap) cand[at] = rank_key(k, a.col_begin + col);
                }
            };
            // the thread's tiles whose bound reaches rho (a NaN bound counts)
            // (no bound of a thread exceeds its largest value rounded up)
            uint64_t hm = 0;
            if (tnan || !(__bfloat162float(__float2bfloat16_ru(tmax)) < rho)) {
#pragma unroll 4
                for (uint32_t t = 0; t < ntiles; ++t) {
                    const float bound = __bfloat162float(__ushort_as_bfloat16(bkey[t * kCons + tid]));
                    if (!(bound < rho)) hm |= 1ull << t;
                }
            }
#ifdef Q38S_TRACE
            atomicAdd(&c.bc_u32[3], __popcll(hm));
            Q38S_TT(u, 10);
#endif
            // one list of (tile, thread) blocks for the whole CTA, so that no
            // thread reads more than its share (the bounds' space is free
            // once every thread has read its own)
            uint32_t n_hit;
            uint32_t hoff = cscan_excl(__popcll(hm), &n_hit, c);
            uint16_t* hlist = bkey;
            while (hm) {
                const uint32_t t = __ffsll(static_cast<long long>(hm)) - 1;
                hm &= hm - 1;
                hlist[hoff++] = static_cast<uint16_t>(t * kCons + tid);
            }
            cbar();
            // the CTA's last unit of at most kRing tiles is still whole in
            // the ring (tile t in slot (g - ntiles + t) % kRing, padded to
            // whole vectors with -inf, its bitmap slice behind it): read it
            // there instead of from L2
            const bool resident = ntiles <= kRing && u + gridDim.x >= n_units;
            // the vectors of hit block hidx (a thread's block of a tile)
            auto load_block = [&](uint32_t hidx, uint4 (&w)[kU]) {
                const uint32_t t = hlist[hidx] / kCons, thr = hlist[hidx] % kCons;
                const uint32_t t0 = c0 + t * TC;
                const uint32_t n = min(c1 - t0, TC);
                const unsigned char* sl = ring + ((g - ntiles + t) % kRing) * kSlot;
#pragma unroll
                for (int q = 0; q < kU; ++q) {  // every load in flight at once
                    const uint32_t e0 = (thr + q * kCons) * pv;
                    const uint32_t nv = e0 < n ? min(pv, n - e0) : 0u;
                    if (resident)
                        w[q] = nv ? *reinterpret_cast<const uint4*>(sl + e0 * es)
                                  : make_uint4(0u, 0u, 0u, 0u);
                    else
                        w[q] = nv ? load_vec<DT>(a, src_row, t0 + e0, nv)
                                  : make_uint4(0u, 0u, 0u, 0u);
                }
            };
            // its elements that reach rho join the candidates (the penalty
            // word of a candidate's vector is read only for candidates)
            auto scan_block = [&](uint32_t hidx, const uint4 (&w)[kU]) {
                const uint32_t t = hlist[hidx] / kCons, thr = hlist[hidx] % kCons;
                const uint32_t t0 = c0 + t * TC;
                const uint32_t n = min(c1 - t0, TC);
                uint32_t cm = 0;  // bit q * pv + e: element e of vector q reaches rho
#pragma unroll
                for (int q = 0; q < kU; ++q) {
                    const uint32_t e0 = (thr + q * kCons) * pv;
#pragma unroll
                    for (uint32_t e = 0; e < pv; ++e) {
                        const float x = vec_elem<DT>(w[q], static_cast<int>(e));
                        if (e0 + e < n && !(x < rho)) cm |= 1u << (q * pv + e);
                    }
                }
                while (cm) {
                    const uint32_t b = __ffs(cm) - 1;
                    cm &= cm - 1;
                    const uint32_t qv = b / pv, ev = b % pv;
                    uint4 wq = w[0];
#pragma unroll
                    for (int q = 1; q < kU; ++q)
                        if (qv == static_cast<uint32_t>(q)) wq = w[q];
                    float x = 0.0f;
#pragma unroll
                    for (uint32_t e = 0; e < pv; ++e)
                        if (ev == e) x = vec_elem<DT>(wq, static_cast<int>(e));
                    const uint32_t e0 = (thr + qv * kCons) * pv;
                    uint32_t pq = 0;
                    if (r.pen) {
                        pq = resident ? reinterpret_cast<const uint32_t*>(
                                            ring + ((g - ntiles + t) % kRing) * kSlot +
                                            kTileBytes)[e0 >> 5]
                                      : __ldg(&r.gbm[(t0 + e0) >> 5]);
                    }
                    consider(x, t0 + e0 + ev, pq);
                }
            };
            // two blocks per round, both blocks' loads in flight before either
            // is scanned (the re-reads come from L2 or HBM while other CTAs
            // still stream: their latency dominates this loop)
#pragma unroll 1
            for (uint32_t hi = tid; hi < n_hit; hi += 2 * kCons) {
                // a buffer that has overflowed sends the row to the general
                // path: stop gathering
                if (*reinterpret_cast<volatile uint32_t*>(&c.n_cand) > cap) break;
                const bool two = hi + kCons < n_hit;
                uint4 w0[kU], w1[kU];
                load_block(hi, w0);
                if (two) load_block(hi + kCons, w1);
                scan_block(hi, w0);
                if (two) scan_block(hi + kCons, w1);
            }
            if (r.nonmono) {
                // penalties can raise a value: every penalised element below
                // rho as well (the state row's bitmap, then this call's
                // additional tokens that the bitmap does not hold, once each)
                for (uint32_t wd = c0 / 32 + tid; wd * 32 < c1; wd += kCons) {
                    uint32_t bits = r.gbm[wd];
                    while (bits) {
                        const uint32_t col = wd * 32 + __ffs(bits) - 1;
                        bits &= bits - 1;
                        if (col < c0 || col >= c1) continue;
                        const float x = elem_at<DT>(src_row, col);
                        if (x < rho) consider(x, col, r.gbm[wd]);
                    }
                }
                for (uint32_t e = tid; e < r.n_extra; e += kCons) {
                    const uint32_t col = static_cast<uint32_t>(r.extra[e]) - a.col_begin;
                    if (col < c0 || col >= c1) continue;
                    if ((r.gbm[col >> 5] >> (col & 31)) & 1u) continue;
                    bool first = true;
                    for (uint32_t e2 = 0; e2 < e && first; ++e2) first = r.extra[e2] != r.extra[e];
                    if (!first) continue;
                    const float x = elem_at<DT>(src_row, col);
                    if (x < rho) consider(x, col, 0u);
                }
            }
        }
        cbar();
        Q38S_TR(u, 14, c.bc_u32[3]);
        uint32_t flags = c.flags;
        uint32_t n = c.n_cand;
        if (n > cap) overflow = true;
        if (overflow) n = 0;
        if (any_stop) flags |= kFTimeout;
        if (overflow) flags |= kFOverflow;
        if (a.mode == kModeShardTopK) flags &= ~kFInf;
        Q38S_TT(u, 4);
        Q38S_TR(u, 5, (static_cast<unsigned long long>(flags) << 32) | n);
        uint32_t keep = 0;
        if (!(flags & (kFTimeout | kFInf | kFOverflow))) {
            keep = finish_buffer(cand, n, r, sorted, c, S == 1);
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
        // ---- multi-segment row: the S CTAs of a cluster hold its segments
        // (cluster rank = segment).  Each keeps its sorted list in its own
        // shared memory and hands the list's header to the leader (rank 0)
        // through distributed shared memory; the leader reads the entries
        // that can still qualify straight from the segments' shared memory,
        // then lets each segment go on.
        {
            const uint32_t len = (flags & (kFTimeout | kFInf | kFOverflow)) ? 0u : keep;
            const uint32_t par = xrow & 1u;
            ++xrow;
            cbar();  // the list is complete
            // lane j < m of warp 0 writes key j of the header (lane 0 also
            // its length, flags and k-th key), then arrives on the leader's
            // barrier itself: the leader waits for S * m arrivals
            const uint32_t m = kHdrKeys / S;  // 64 / kMaxSegs .. 32
            if (tid < m) {
                if (tid == 0) {
                    const uint32_t kth = (r.k_eff && len >= r.k_eff)
                        ? static_cast<uint32_t>(sorted[r.k_eff - 1] >> 32) : 0u;
                    st_cluster_u32(cluster_addr(&c.xh_len[seg], 0), len);
                    st_cluster_u32(cluster_addr(&c.xh_flags[seg], 0), flags);
                    st_cluster_u32(cluster_addr(&c.xh_kth[seg], 0), kth);
                }
                st_cluster_u32(cluster_addr(&c.xh_keys[seg * m + tid], 0),
                               tid < len ? static_cast<uint32_t>(sorted[tid] >> 32) : 0u);
                // the list (every thread's writes, ordered by the barrier
                // above) and this lane's header words before its arrival
                fence_acq_rel_cluster();
                mbar_arrive_cluster(cluster_addr(&c.xfull, 0));
            }
            if (seg != 0) {
                // the list stays put until the leader has read it (a wait
                // that runs out leaves the row to the leader's status)
                if (tid == 0) mbar_wait_cluster_bounded(&c.xdone, par, kWaitLimitCycles);
                cbar();
                Q38S_TR(u, 8, 3);
                Q38S_TT(u, 9);
                continue;
            }
            if (tid == 0) c.bc_u32[2] = mbar_wait_cluster_bounded(&c.xfull, par, kWaitLimitCycles);
            if (tid == 0) c.n_cand = 0;
            cbar();
            Q38S_TT(u, 13);
            uint32_t rflags = c.bc_u32[2] ? 0u : kFTimeout;
            uint32_t mkth = 0, mtop = 0;
            for (uint32_t s2 = 0; s2 < S; ++s2) {
                rflags |= c.xh_flags[s2];
                mkth = max(mkth, c.xh_kth[s2]);
                if (c.xh_len[s2]) mtop = max(mtop, c.xh_keys[s2 * m]);
            }
            // The lists are sorted: the row's k-th largest value is at least
            // every segment's k-th and the k-th largest of the segments'
            // first m entries (distinct entries of the row); its largest
            // value is the largest first entry.  Only entries at or above
            // the better bound (and the min-p bound) are merged.
            if (r.k_eff && r.k_eff <= S * m) {
                // key x is the k-th largest when fewer than k keys exceed it
                // and at least k reach it (every thread of warps 0-1 ranks one)
                if (tid == 0) c.bc_u32[0] = 0;
                cbar();
                if (tid < S * m) {
                    const uint32_t x = c.xh_keys[tid];
                    uint32_t gt = 0, ge = 0;
#pragma unroll 8
                    for (uint32_t j = 0; j < S * m; ++j) {
                        const uint32_t y = c.xh_keys[j];
                        gt += y > x ? 1u : 0u;
                        ge += y >= x ? 1u : 0u;
                    }
                    if (x && gt < r.k_eff && ge >= r.k_eff) c.bc_u32[0] = x;  // equal writers
                }
                cbar();
                mkth = max(mkth, c.bc_u32[0]);
            }
            Q38S_TT(u, 15);
            if (a.mode == kModeShardTopK) rflags &= ~kFInf;
            uint32_t rkeep = 0;
            bool over = false;
            if (!(rflags & (kFTimeout | kFInf | kFOverflow))) {
                uint32_t th = mkth;
                if (r.minp) th = max(th, minp_key(mtop, r));
                // warp w reads the lists of segments w, w + 8, ... down to
                // the first entry below th
                for (uint32_t s2 = warp; s2 < S; s2 += kCons / 32) {
                    const uint32_t ls = c.xh_len[s2];
                    const uint32_t src = cluster_addr(sorted, s2);
                    for (uint32_t i0 = 0; i0 < ls; i0 += 32) {
                        const uint32_t i = i0 + lane;
                        const uint64_t e = i < ls ? ld_cluster_u64(src + 8u * i) : 0ull;
                        const bool in = i < ls && static_cast<uint32_t>(e >> 32) >= th;
                        over |= warp_push(in, e, cand, kBuf, &c.n_cand);
                        if (__ballot_sync(kFull, i < ls && !in)) break;
                    }
                }
            }
            over = cbar_or(over);  // also: every read of the segments' lists is done
            if (tid > 0 && tid < S) mbar_arrive_cluster(cluster_addr(&c.xdone, tid));
            Q38S_TT(u, 6);
            if (!(rflags & (kFTimeout | kFInf | kFOverflow))) {
                const uint32_t nm = min(c.n_cand, kBuf);
                if (over) rflags |= kFOverflow;  // more than the buffer holds
                if (!(rflags & kFOverflow)) {
                    rkeep = finish_buffer(cand, nm, r, sorted, c, true);
                    if (rkeep == 0xffffffffu) rflags |= kFOverflow;
                }
                Q38S_TR(u, 14, nm);
            }
            Q38S_TT(u, 10);
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
    if (s > kMaxSegs) s = kMaxSegs;
    return s < 1 ? 1 : s;
}

static uint32_t g_fault_withhold = 0;
static long long g_fault_wait = 0;

void set_stream_fault(uint32_t withhold, long long wait_cycles) {
    g_fault_withhold = withhold;
    g_fault_wait = wait_cycles;
}

// The general kernel behind every stream kernel, as its programmatic
// dependent (the launch overlaps the stream kernel).
template <int DT>
static cudaError_t launch_general(const SampleArgs& a, void* stream, int sms,
                                  uint32_t stream_grid) {
    static bool configured[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    constexpr uint32_t smem = kArea + kStageBytes + kPcPmBytes;
    if (!configured[dev]) {
        e = cudaFuncSetAttribute(general_kernel<DT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    // one CTA per SM (its registers admit no second, nor a stream CTA beside
    // it): every CTA of a team is resident once the stream kernel has left
    // the SMs.  (A grid of only the SMs a small stream grid leaves free made
    // batch-1 no faster and split 16 deferred rows into teams of one.)
    (void)stream_grid;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<uint32_t>(sms));
    cfg.blockDim = dim3(kCons);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, general_kernel<DT>, a);
}

template <int DT>
static int launch_stream_t(const SampleArgs& a_in, void* stream) {
    SampleArgs a = a_in;
    a.test_withhold = g_fault_withhold;
    a.test_wait_cycles = g_fault_wait;
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
        if (kMaxSegs > 8) {  // clusters beyond the portable size
            e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
            if (e != cudaSuccess) return e;
        }
        e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        configured[slot][dev] = true;
    }
    const uint32_t units = a.vrows * a.segs;
    uint32_t cap = 2u * static_cast<uint32_t>(sms[dev]);
#ifdef Q38S_TRACE
    if (const char* gc = getenv("Q38S_TRACE_GRID")) cap = static_cast<uint32_t>(atoi(gc));
#endif
    cap -= cap % a.segs;  // whole clusters (units is a multiple of segs)
    const uint32_t grid = units < cap ? units : cap;
    if (a.segs == 1) {
        kern<<<grid, kBlock, smem, static_cast<cudaStream_t>(stream)>>>(a);
        e = cudaGetLastError();
        return (e != cudaSuccess || a.host_general) ? e
                                                     : launch_general<DT>(a, stream, sms[dev], grid);
    }
    // one cluster of segs CTAs per row: CTA rank = segment
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kBlock);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = a.segs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, a);
    return (e != cudaSuccess || a.host_general) ? e
                                                 : launch_general<DT>(a, stream, sms[dev], grid);
}

int launch_general_only(const SampleArgs& a, void* stream) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    return a.dtype == Q38S_DTYPE_BF16 ? launch_general<Q38S_DTYPE_BF16>(a, stream, sms, 0)
                                      : launch_general<Q38S_DTYPE_F32>(a, stream, sms, 0);
}

int launch_stream(const SampleArgs& a, void* stream) {
    if (a.vrows == 0) return cudaSuccess;
    return a.dtype == Q38S_DTYPE_BF16 ? launch_stream_t<Q38S_DTYPE_BF16>(a, stream)
                                      : launch_stream_t<Q38S_DTYPE_F32>(a, stream);
}

}  // namespace q38s
