// Row-sampling kernels for sm_100a.
//
// One thread-block cluster of S CTAs (S = 8 at V = 151,936) samples one row.
// CTA c owns a contiguous chunk of the row's columns (whole 128-column
// blocks), pulls it into shared memory with 1-D TMA bulk copies (no
// multicast) together with its slice of the row's penalty bitmap, and
//
//   pass 1  takes the per-thread maximum raw logit (bf16x2 / f32x4 maxima),
//           evaluates those 256 elements exactly and derives a threshold
//           theta: the k-th largest of them (a lower bound of the row's k-th
//           largest value) and, for min-p, M_lb + ln(min_p) (M_lb a lower
//           bound of the row maximum).  The CTAs combine theirs over DSMEM.
//   pass 2  streams the chunk again from shared memory; a vector whose raw
//           maximum is below the raw bound of theta is skipped with one
//           packed compare; the rare survivors get the reference's exact
//           penalty/temperature arithmetic (sampling.cc:76-92) and enter a
//           candidate buffer as 64-bit rank keys (value desc, token asc).
//   merge   each CTA sorts its candidates; the leader CTA gathers the lists
//           through DSMEM, merges them by rank, and runs the reference's
//           softmax / min-p / top-p / draw (sampling.cc:105-145) in double
//           precision with the reference's sequential summation order.
//
// Rows whose candidate sets do not fit (top_k = 0 with no or tiny min_p,
// heavy ties, top_k > 128) take the cluster-wide general path: exact keys
// for every column go to a global scratch array, 8-bit radix histograms over
// the cluster select the top-k cut, and either the kept set is gathered and
// finished exactly, or (kept sets above 1,024 tokens) the top-p cut and the
// draw are located by mass-weighted radix selection with 2^-44 fixed-point
// masses.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include "q38s_kernels.cuh"

namespace cg = cooperative_groups;

namespace q38s {

namespace {

constexpr uint32_t kFlagOverflow = 1u;
constexpr uint32_t kFlagInf = 2u;
constexpr uint32_t kFlagTimeout = 4u;
constexpr double kFix = 17592186044416.0;  // 2^44

struct __align__(16) Ctl {
    uint64_t bar[kPieces + 1];
    uint32_t n_cand;
    uint32_t flags;
    uint32_t theta_key;
    uint32_t max_key;
    uint32_t pub_theta;     // leader: max over the cluster
    uint32_t pub_max;       // leader: max over the cluster
    uint32_t list_len;
    uint32_t g_count;       // leader: general-path gather count
    uint64_t list_top;
    uint64_t g_sum;         // general path: partial sums
    uint32_t g_u32;
    uint32_t sel_token;     // leader: selected token of a tie group
    uint32_t bcast_u32[4];
    uint64_t bcast_u64[4];
    uint32_t red_u32[kThreads / 32];
    uint64_t red_u64[kThreads / 32];
    uint32_t tkey[kThreads];
    // epilogue results
    int32_t e_token;
    int32_t e_status;
    uint32_t e_n;
    uint32_t e_r;
    uint32_t e_sel;
    double e_total;
    double e_draw;
};

__device__ __forceinline__ uint32_t block_max_u32(uint32_t v, Ctl& c) {
    v = warp_max_u32(v);
    const int w = threadIdx.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) c.red_u32[w] = v;
    __syncthreads();
    uint32_t r = 0;
    for (int i = 0; i < kThreads / 32; ++i) r = max(r, c.red_u32[i]);
    __syncthreads();
    return r;
}
__device__ __forceinline__ uint32_t block_min_u32(uint32_t v, Ctl& c) {
    v = warp_min_u32(v);
    const int w = threadIdx.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) c.red_u32[w] = v;
    __syncthreads();
    uint32_t r = 0xffffffffu;
    for (int i = 0; i < kThreads / 32; ++i) r = min(r, c.red_u32[i]);
    __syncthreads();
    return r;
}
__device__ __forceinline__ uint32_t block_sum_u32(uint32_t v, Ctl& c) {
    v = warp_sum_u32(v);
    const int w = threadIdx.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) c.red_u32[w] = v;
    __syncthreads();
    uint32_t r = 0;
    for (int i = 0; i < kThreads / 32; ++i) r += c.red_u32[i];
    __syncthreads();
    return r;
}
__device__ __forceinline__ uint64_t block_sum_u64(uint64_t v, Ctl& c) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) c.red_u64[w] = v;
    __syncthreads();
    uint64_t r = 0;
    for (int i = 0; i < kThreads / 32; ++i) r += c.red_u64[i];
    __syncthreads();
    return r;
}

// Sorts keys[0..n) in descending order; n is a power of two; whole block.
__device__ void bitonic_desc(uint64_t* keys, uint32_t n) {
    for (uint32_t size = 2; size <= n; size <<= 1) {
        for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
            for (uint32_t i = threadIdx.x; i < n / 2; i += blockDim.x) {
                const uint32_t lo = 2 * i - (i & (stride - 1));
                const uint32_t hi = lo + stride;
                const bool desc = (lo & size) == 0;
                const uint64_t a = keys[lo], b = keys[hi];
                if ((a < b) == desc) {
                    keys[lo] = b;
                    keys[hi] = a;
                }
            }
            __syncthreads();
        }
    }
}

__device__ __forceinline__ uint32_t pow2_at_least(uint32_t n) {
    uint32_t p = 1;
    while (p < n) p <<= 1;
    return p;
}

// Column partition: 128-column blocks spread over S CTAs.
__device__ __forceinline__ void chunk_range(uint32_t vocab, int S, int rank, uint32_t& lo,
                                            uint32_t& hi) {
    const uint32_t nblk = (vocab + 127) / 128;
    const uint32_t b0 = static_cast<uint32_t>((static_cast<uint64_t>(nblk) * rank) / S);
    const uint32_t b1 = static_cast<uint32_t>((static_cast<uint64_t>(nblk) * (rank + 1)) / S);
    lo = min(b0 * 128u, vocab);
    hi = min(b1 * 128u, vocab);
}

// Softmax / min-p / top-p / draw over `n` candidates sorted by rank key,
// exactly in the order of sampling.cc:105-145: weights exp((double)(v_i -
// v_0)), sequential double prefix sums, the quotient-accumulating top-p
// loop, draw = uniform01(rng_before + gamma) * total, first prefix sum above
// the draw.  min-p (extension) keeps the prefix with w_i >= min_p.  The
// whole block calls it; results land in c.e_*.
__device__ void epilogue(const uint64_t* sorted, uint32_t n, const RowParams& p, bool minp,
                         uint64_t rng_before, double* w, double* S, double* q, Ctl& c) {
    const int tid = threadIdx.x;
    if (tid == 0) {
        c.e_status = Q38S_ROW_OK;
        c.e_token = -1;
        c.e_n = n;
        c.e_r = 0;
        c.e_sel = 0;
        c.e_total = 0.0;
        c.e_draw = 0.0;
    }
    __syncthreads();
    if (n == 0 || !isfinite(rank_value(sorted[0]))) {
        if (tid == 0) c.e_status = Q38S_ROW_NO_FINITE;
        __syncthreads();
        return;
    }
    const float vmax = rank_value(sorted[0]);
    for (uint32_t i = tid; i < n; i += blockDim.x)
        w[i] = exp(static_cast<double>(__fsub_rn(rank_value(sorted[i]), vmax)));
    __syncthreads();
    if (minp && p.min_p > 0.0f) {
        const double floor_w = static_cast<double>(p.min_p);
        uint32_t m = n;
        for (uint32_t i = tid; i < n; i += blockDim.x)
            if (w[i] < floor_w) m = min(m, i);
        n = block_min_u32(m, c);
    }
    if (tid == 0) {
        double acc = 0.0;
        for (uint32_t i = 0; i < n; ++i) {
            acc += w[i];
            S[i] = acc;
        }
        c.e_n = n;
        c.e_total = acc;
        if (!(acc > 0.0) || !isfinite(acc)) c.e_status = Q38S_ROW_NORMALIZATION;
    }
    __syncthreads();
    if (c.e_status != Q38S_ROW_OK) return;
    const double total = c.e_total;
    uint32_t r = n;
    if (p.top_p < 1.0f) {
        for (uint32_t i = tid; i < n; i += blockDim.x) q[i] = w[i] / total;
        __syncthreads();
        if (tid == 0) {
            const double top_p = static_cast<double>(p.top_p);
            double cum = 0.0;
            uint32_t k = 0;
            while (k < n) {
                cum += q[k];
                ++k;
                if (cum >= top_p) break;
            }
            c.e_r = k;
            c.e_total = S[k - 1];
        }
        __syncthreads();
        r = c.e_r;
    } else if (tid == 0) {
        c.e_r = n;
    }
    __syncthreads();
    const double total_r = c.e_total;
    const double draw = uniform01(rng_before + kGamma) * total_r;
    uint32_t sel = r - 1;
    for (uint32_t i = tid; i < r; i += blockDim.x)
        if (draw < S[i]) sel = min(sel, i);
    sel = block_min_u32(sel, c);
    if (tid == 0) {
        c.e_sel = sel;
        c.e_draw = draw;
        c.e_token = static_cast<int32_t>(rank_token(sorted[sel]));
    }
    __syncthreads();
}

struct RowCtx {
    uint32_t v;          // virtual row
    uint32_t srow;       // state row
    RowParams p;
    RowState st;
    uint64_t rng_before;
    uint32_t lo, hi, n;  // chunk
    const uint32_t* bm;  // smem bitmap slice (or null)
    const uint32_t* counts_row;
    const int32_t* extra;
    uint32_t n_extra;
    uint32_t k_eff;      // 0 = no top-k truncation
    bool pen, nonmono, freq;
};

__device__ __forceinline__ float eval_exact(const RowCtx& r, float x, uint32_t j,
                                            uint32_t col_begin) {
    bool penalized = false;
    uint64_t count = 1;
    if (r.pen) {
        penalized = (r.bm[j >> 5] >> (j & 31)) & 1u;
        if (penalized && r.freq) {
            const uint32_t col = r.lo + j;
            count = r.counts_row ? r.counts_row[col] : 0u;
            for (uint32_t e = 0; e < r.n_extra; ++e)
                count += (static_cast<uint32_t>(r.extra[e]) == col) ? 1u : 0u;
        }
    }
    (void)col_begin;
    return transform(x, penalized, count, r.p);
}

template <int DT>
__device__ __forceinline__ float load_elem(const unsigned char* chunk, uint32_t j) {
    if (DT == Q38S_DTYPE_BF16)
        return __uint_as_float(static_cast<uint32_t>(
                                   reinterpret_cast<const uint16_t*>(chunk)[j])
                               << 16);
    return reinterpret_cast<const float*>(chunk)[j];
}

// Per-virtual-row outputs once the token (or error) is known.  Leader CTA,
// whole block.
__device__ void write_decision(const SampleArgs& a, const RowCtx& r, int32_t token,
                               int32_t status) {
    if (threadIdx.x != 0) return;
    q38s_decision_v1 d;
    d.token = status == Q38S_ROW_OK ? token : -1;
    d.status = status;
    d.rng_before = r.rng_before;
    d.rng_after = r.rng_before + kGamma;
    if (a.decisions) a.decisions[r.v] = d;
    if (a.mode == kModeSampleCommit && status == Q38S_ROW_OK) {
        // commit (sampling.cc:148-156) then commit_token (sampling.cc:163-172)
        RowState& s = a.state[r.srow];
        s.rng_state = d.rng_after;
        s.sampled_tokens += 1;
        const uint32_t col = static_cast<uint32_t>(token) - a.col_begin;
        atomicOr(&a.bitmap[static_cast<size_t>(r.srow) * a.bitmap_words + (col >> 5)],
                 1u << (col & 31));
        if (a.counts) atomicAdd(&a.counts[static_cast<size_t>(r.srow) * a.vocab + col], 1u);
        s.canonical_tokens += 1;
        s.penalty_checksum ^=
            splitmix64(static_cast<uint64_t>(static_cast<uint32_t>(token)) ^
                       (s.canonical_tokens * kGamma));
    }
}

__device__ void write_distribution(const SampleArgs& a, const RowCtx& r,
                                   const uint64_t* sorted, const double* w, Ctl& c) {
    if (a.dist.capacity == 0) return;
    const uint32_t cap = a.dist.capacity;
    const size_t base = static_cast<size_t>(r.v) * cap;
    const uint32_t n = c.e_status == Q38S_ROW_OK ? c.e_n : 0;
    const uint32_t rr = c.e_status == Q38S_ROW_OK ? c.e_r : 0;
    for (uint32_t i = threadIdx.x; i < min(n, cap); i += blockDim.x) {
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

// Speculative verification over the distributions of all virtual rows
// (target rows 0..n, draft rows n+1..2n).  One thread; runs in the CTA that
// finished last.
__device__ void mtp_finish(const SampleArgs& a) {
    q38s_mtp_result res;
    const uint32_t n = a.n_draft;
    const uint32_t cap = a.dist.capacity;
    const RowState st = a.state[a.vrow_state_const];
    res.rng_before = st.rng_state;
    res.status = Q38S_ROW_OK;
    res.n_tokens = 0;
    res.n_accepted = 0;
    for (uint32_t i = 0; i <= n; ++i) {
        const q38s_decision_v1 dt = a.decisions[i];
        const uint64_t s_i = st.rng_state + (static_cast<uint64_t>(i) + 1) * kGamma;
        if (dt.status != Q38S_ROW_OK) {
            res.status = dt.status;
            break;
        }
        if (i == n) {  // bonus row: the reference draw from p_n
            res.tokens[res.n_tokens++] = dt.token;
            break;
        }
        const q38s_decision_v1 dd = a.decisions[n + 1 + i];
        if (dd.status != Q38S_ROW_OK) {
            res.status = dd.status;
            break;
        }
        const uint32_t np = a.dist.n_retained[i];
        const uint32_t nq = a.dist.n_retained[n + 1 + i];
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
            if (pt[j] == d) pd = pp[j];
        for (uint32_t j = 0; j < nq; ++j)
            if (qt[j] == d) qd = qp[j];
        const double ua = uniform01(s_i ^ kAcceptDomain);
        if (ua * qd < pd) {
            res.tokens[res.n_tokens++] = d;
            ++res.n_accepted;
            continue;
        }
        // rejected: residual max(0, p - q) over p's sorted support
        double rtotal = 0.0;
        for (uint32_t j = 0; j < np; ++j) {
            double qj = 0.0;
            for (uint32_t m = 0; m < nq; ++m)
                if (qt[m] == pt[j]) qj = qp[m];
            rtotal += fmax(0.0, pp[j] - qj);
        }
        int32_t tok = dt.token;  // empty residual: reference draw from p_i
        if (rtotal > 0.0) {
            const double draw = uniform01(s_i) * rtotal;
            double cum = 0.0;
            uint32_t sel = np - 1;
            for (uint32_t j = 0; j < np; ++j) {
                double qj = 0.0;
                for (uint32_t m = 0; m < nq; ++m)
                    if (qt[m] == pt[j]) qj = qp[m];
                cum += fmax(0.0, pp[j] - qj);
                if (draw < cum) {
                    sel = j;
                    break;
                }
            }
            tok = pt[sel];
        }
        res.tokens[res.n_tokens++] = tok;
        break;
    }
    res.rng_after = res.rng_before + static_cast<uint64_t>(res.n_tokens) * kGamma;
    *a.mtp = res;
}

// Leader-side completion of a row from a sorted candidate list.
__device__ void finish_row(const SampleArgs& a, const RowCtx& r, uint64_t* sorted,
                           uint32_t n, unsigned char* area, Ctl& c) {
    if (a.mode == kModeShardTopK) {
        const uint32_t k = a.k_out;
        for (uint32_t i = threadIdx.x; i < k; i += blockDim.x) {
            q38s_candidate cd;
            if (i < n) {
                cd.value = rank_value(sorted[i]);
                cd.token = static_cast<int32_t>(rank_token(sorted[i]));
            } else {
                cd.value = -INFINITY;
                cd.token = -1;
            }
            a.topk_out[static_cast<size_t>(r.v) * k + i] = cd;
        }
        return;
    }
    double* w = reinterpret_cast<double*>(area + kLeaderCap * 8);
    double* S = reinterpret_cast<double*>(area + kLeaderCap * 16);
    double* q = reinterpret_cast<double*>(area + kLeaderCap * 24);
    epilogue(sorted, n, r.p, true, r.rng_before, w, S, q, c);
    write_decision(a, r, c.e_token, c.e_status);
    write_distribution(a, r, sorted, w, c);
}

// ------------------------------------------------------- general path
struct GenState {
    uint32_t M_key;
    float M;
    uint32_t minp_key;
    bool has_cut;
    uint32_t cut_key;
    uint32_t cut_tok;
};

__device__ __forceinline__ bool in_k0(const GenState& g, uint32_t key, uint32_t tok) {
    if (key < g.minp_key) return false;
    if (!g.has_cut) return true;
    return key > g.cut_key || (key == g.cut_key && tok <= g.cut_tok);
}
__device__ __forceinline__ uint64_t wfix(const GenState& g, uint32_t key) {
    const double w = exp(static_cast<double>(__fsub_rn(key_float(key), g.M)));
    return static_cast<uint64_t>(w * kFix + 0.5);
}

struct SelResult {
    bool found;
    uint32_t key;
    uint32_t token;
    uint64_t through;  // count or fixed-point mass through the element
};

// Cluster-collective radix selection over the chunk keys in `keys`
// (global scratch) restricted to K0 (or to {key >= minp_key} when
// `restrict_k0` is false).  Finds the first element in canonical order at
// which the running count (weighted = false) or fixed-point mass
// (weighted = true) reaches `tau` (>= tau, or > tau when `strict`).
__device__ SelResult cluster_select(cg::cluster_group& cluster, const uint32_t* keys,
                                    uint32_t n, uint32_t tok0, const GenState& g,
                                    bool restrict_k0, bool weighted, uint64_t tau,
                                    bool strict, unsigned char* area, Ctl& c) {
    const int S = static_cast<int>(cluster.num_blocks());
    const int me = static_cast<int>(cluster.block_rank());
    uint64_t* hmass = reinterpret_cast<uint64_t*>(area);
    uint32_t* hcnt = reinterpret_cast<uint32_t*>(area + kHistBins * 8);
    uint64_t* tmass = reinterpret_cast<uint64_t*>(area + kHistBins * 12);
    uint32_t* tcnt = reinterpret_cast<uint32_t*>(area + kHistBins * 20);
    GenState gs = g;
    if (!restrict_k0) gs.has_cut = false;
    uint32_t prefix = 0, mask = 0;
    uint64_t above = 0;  // count or mass above the current bin range
    SelResult res{false, 0, 0, 0};
    uint32_t last_digit = 0;
    for (int level = 0; level < 4; ++level) {
        const int shift = 24 - 8 * level;
        for (int i = threadIdx.x; i < kHistBins; i += blockDim.x) {
            hmass[i] = 0;
            hcnt[i] = 0;
        }
        __syncthreads();
        for (uint32_t j = threadIdx.x; j < n; j += blockDim.x) {
            const uint32_t key = keys[j];
            if ((key & mask) != prefix || !in_k0(gs, key, tok0 + j)) continue;
            const uint32_t d = (key >> shift) & 255u;
            atomicAdd(&hcnt[d], 1u);
            if (weighted) atomicAdd(reinterpret_cast<unsigned long long*>(&hmass[d]),
                                    static_cast<unsigned long long>(wfix(gs, key)));
        }
        __syncthreads();
        cluster.sync();
        for (int d = threadIdx.x; d < kHistBins; d += blockDim.x) {
            uint64_t m = 0;
            uint32_t k = 0;
            for (int s = 0; s < S; ++s) {
                const uint64_t* rm = cluster.map_shared_rank(hmass, s);
                const uint32_t* rc = cluster.map_shared_rank(hcnt, s);
                m += rm[d];
                k += rc[d];
            }
            tmass[d] = m;
            tcnt[d] = k;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            uint64_t acc = above;
            int hit = -1;
            for (int d = kHistBins - 1; d >= 0; --d) {
                const uint64_t add = weighted ? tmass[d] : tcnt[d];
                if (tcnt[d] == 0) continue;
                const uint64_t nxt = acc + add;
                if (strict ? (nxt > tau) : (nxt >= tau)) {
                    hit = d;
                    break;
                }
                acc = nxt;
            }
            c.bcast_u32[0] = static_cast<uint32_t>(hit);
            c.bcast_u64[0] = acc;
        }
        __syncthreads();
        const int hit = static_cast<int>(c.bcast_u32[0]);
        if (hit < 0) {
            cluster.sync();  // peers finished reading this level's histograms
            return res;
        }
        above = c.bcast_u64[0];
        prefix |= static_cast<uint32_t>(hit) << shift;
        mask |= 255u << shift;
        last_digit = static_cast<uint32_t>(hit);
        if (level < 3) cluster.sync();  // before the histograms are cleared
    }
    // Tie group: every element with key == prefix inside K0, in token order.
    const uint32_t key = prefix;
    const uint32_t group = tcnt[last_digit];
    uint64_t j;  // position inside the group
    uint64_t per = 1;
    if (weighted) {
        per = wfix(gs, key);
        if (per == 0) {
            j = 0;
        } else if (strict) {
            j = (tau - above) / per;  // smallest j: above + (j+1) per > tau
        } else {
            const uint64_t need = tau > above ? tau - above : 0;
            j = need == 0 ? 0 : (need + per - 1) / per - 1;
        }
    } else {
        j = tau > above ? tau - above - 1 : 0;
    }
    if (j >= group) j = group - 1;
    // Owner CTA by prefix over ranks of the per-CTA counts of this digit.
    uint32_t before = 0;
    int owner = S - 1;
    for (int s = 0; s < S; ++s) {
        const uint32_t cs = cluster.map_shared_rank(hcnt, s)[last_digit];
        if (j < before + cs) {
            owner = s;
            break;
        }
        before += cs;
    }
    if (me == owner) {
        // ordered scan: thread t owns columns [t*per_t, (t+1)*per_t)
        const uint32_t per_t = (n + blockDim.x - 1) / blockDim.x;
        const uint32_t b = threadIdx.x * per_t;
        const uint32_t e = min(n, b + per_t);
        uint32_t mine = 0;
        for (uint32_t x = b; x < e; ++x)
            mine += (keys[x] == key && in_k0(gs, key, tok0 + x)) ? 1u : 0u;
        c.tkey[threadIdx.x] = mine;
        __syncthreads();
        if (threadIdx.x == 0) {
            uint32_t acc = 0;
            for (int t = 0; t < kThreads; ++t) {
                const uint32_t m = c.tkey[t];
                c.tkey[t] = acc;
                acc += m;
            }
        }
        __syncthreads();
        const uint32_t want = static_cast<uint32_t>(j) - before;
        uint32_t seen = c.tkey[threadIdx.x];
        if (want >= seen && want < seen + mine) {
            for (uint32_t x = b; x < e; ++x) {
                if (keys[x] == key && in_k0(gs, key, tok0 + x)) {
                    if (seen == want) {
                        *cluster.map_shared_rank(&c.sel_token, 0) = tok0 + x;
                        break;
                    }
                    ++seen;
                }
            }
        }
    }
    cluster.sync();
    res.found = true;
    res.key = key;
    res.token = *cluster.map_shared_rank(&c.sel_token, 0);
    res.through = above + (j + 1) * per;
    cluster.sync();
    return res;
}

template <int DT>
__device__ void general_path(const SampleArgs& a, cg::cluster_group& cluster, RowCtx& r,
                             unsigned char* chunk, unsigned char* area, Ctl& c) {
    const int S = static_cast<int>(cluster.num_blocks());
    const int me = static_cast<int>(cluster.block_rank());
    const uint32_t tok0 = a.col_begin + r.lo;
    uint32_t* keys = a.scratch + static_cast<size_t>(r.v) * a.vocab + r.lo;
    // G0: exact keys of every column of the chunk.
    uint32_t kmax = 0;
    for (uint32_t j = threadIdx.x; j < r.n; j += blockDim.x) {
        const float x = load_elem<DT>(chunk, j);
        const uint32_t k = float_key(eval_exact(r, x, j, a.col_begin));
        keys[j] = k;
        kmax = max(kmax, k);
    }
    kmax = block_max_u32(kmax, c);
    if (threadIdx.x == 0) c.g_u32 = kmax;
    __syncthreads();
    cluster.sync();
    GenState g;
    g.M_key = 0;
    for (int s = 0; s < S; ++s) g.M_key = max(g.M_key, *cluster.map_shared_rank(&c.g_u32, s));
    g.M = key_float(g.M_key);
    g.has_cut = false;
    g.cut_key = 0;
    g.cut_tok = 0;
    g.minp_key = 0;
    cluster.sync();  // everyone read g_u32
    const bool leader = me == 0;
    if (g.M_key <= kNegInfKey || isinf(g.M)) {
        if (leader) write_decision(a, r, -1, Q38S_ROW_NO_FINITE);
        if (leader && a.dist.capacity) {
            if (threadIdx.x == 0) {
                if (a.dist.n_candidates) a.dist.n_candidates[r.v] = 0;
                if (a.dist.n_retained) a.dist.n_retained[r.v] = 0;
            }
        }
        return;
    }
    // G1: min-p key threshold (smallest key whose weight reaches min_p).
    const bool use_minp = a.mode != kModeShardTopK && r.p.min_p > 0.0f;
    if (use_minp) {
        if (threadIdx.x == 0) {
            const double floor_w = static_cast<double>(r.p.min_p);
            uint32_t lo = kNegInfKey, hi = g.M_key;  // weight(hi) = 1 >= min_p
            while (lo < hi) {
                const uint32_t mid = lo + (hi - lo) / 2;
                const double w = exp(static_cast<double>(__fsub_rn(key_float(mid), g.M)));
                if (w >= floor_w) hi = mid; else lo = mid + 1;
            }
            c.bcast_u32[1] = hi;
        }
        __syncthreads();
        g.minp_key = c.bcast_u32[1];
    }
    uint32_t cnt = 0;
    for (uint32_t j = threadIdx.x; j < r.n; j += blockDim.x) cnt += keys[j] >= g.minp_key;
    cnt = block_sum_u32(cnt, c);
    if (threadIdx.x == 0) c.g_u32 = cnt;
    __syncthreads();
    cluster.sync();
    uint32_t c_minp = 0;
    for (int s = 0; s < S; ++s) c_minp += *cluster.map_shared_rank(&c.g_u32, s);
    cluster.sync();
    const uint32_t n0 = r.k_eff ? min(r.k_eff, c_minp) : c_minp;
    if (n0 < c_minp) {
        const SelResult cut = cluster_select(cluster, keys, r.n, tok0, g, false, false, n0,
                                             false, area, c);
        g.has_cut = true;
        g.cut_key = cut.key;
        g.cut_tok = cut.token;
    }
    if (n0 <= kLeaderCap) {
        // G2: gather K0 into the leader and finish exactly.
        uint64_t* lkeys = reinterpret_cast<uint64_t*>(area);
        uint64_t* rkeys = cluster.map_shared_rank(lkeys, 0);
        uint32_t* rcount = cluster.map_shared_rank(&c.g_count, 0);
        for (uint32_t j = threadIdx.x; j < r.n; j += blockDim.x) {
            const uint32_t k = keys[j];
            if (!in_k0(g, k, tok0 + j)) continue;
            const uint32_t pos = atomicAdd(rcount, 1u);
            if (pos < kLeaderCap) rkeys[pos] = rank_key(k, tok0 + j);
        }
        __syncthreads();
        cluster.sync();
        if (!leader) return;
        const uint32_t m = min(c.g_count, static_cast<uint32_t>(kLeaderCap));
        const uint32_t p2 = pow2_at_least(m);
        for (uint32_t i = m + threadIdx.x; i < p2; i += blockDim.x) lkeys[i] = 0;
        __syncthreads();
        bitonic_desc(lkeys, p2);
        finish_row(a, r, lkeys, m, area, c);
        return;
    }
    // G3: large kept set; fixed-point masses.
    uint64_t part = 0;
    for (uint32_t j = threadIdx.x; j < r.n; j += blockDim.x) {
        const uint32_t k = keys[j];
        if (in_k0(g, k, tok0 + j)) part += wfix(g, k);
    }
    part = block_sum_u64(part, c);
    if (threadIdx.x == 0) c.g_sum = part;
    __syncthreads();
    cluster.sync();
    uint64_t Z = 0;
    for (int s = 0; s < S; ++s) Z += *cluster.map_shared_rank(&c.g_sum, s);
    cluster.sync();
    int32_t status = Q38S_ROW_OK;
    int32_t token = -1;
    uint64_t Zr = Z;
    SelResult cutp{false, 0, 0, 0};
    if (Z == 0) status = Q38S_ROW_NORMALIZATION;
    if (status == Q38S_ROW_OK && r.p.top_p < 1.0f) {
        const uint64_t tau = static_cast<uint64_t>(static_cast<double>(r.p.top_p) *
                                                   static_cast<double>(Z));
        cutp = cluster_select(cluster, keys, r.n, tok0, g, true, true, tau, false, area, c);
        if (cutp.found) Zr = cutp.through;
    }
    double draw_d = 0.0;
    if (status == Q38S_ROW_OK) {
        const double u = uniform01(r.rng_before + kGamma);
        const uint64_t draw = static_cast<uint64_t>(u * static_cast<double>(Zr));
        draw_d = static_cast<double>(draw) / kFix;
        const SelResult sel =
            cluster_select(cluster, keys, r.n, tok0, g, true, true, draw, true, area, c);
        if (sel.found) token = static_cast<int32_t>(sel.token);
        else if (cutp.found) token = static_cast<int32_t>(cutp.token);
        else status = Q38S_ROW_NORMALIZATION;
    }
    if (leader) {
        write_decision(a, r, token, status);
        if (a.dist.capacity && threadIdx.x == 0) {
            if (a.dist.n_candidates) a.dist.n_candidates[r.v] = n0;
            if (a.dist.n_retained) a.dist.n_retained[r.v] = 0xffffffffu;
            if (a.dist.total) a.dist.total[r.v] = static_cast<double>(Zr) / kFix;
            if (a.dist.draw) a.dist.draw[r.v] = draw_d;
        }
    }
}

template <int DT>
__global__ void __launch_bounds__(kThreads, 4)
    sample_rows_kernel(const SampleArgs a) {
    extern __shared__ __align__(128) unsigned char dsm[];
    __shared__ Ctl c;
    cg::cluster_group cluster = cg::this_cluster();
    const int S = static_cast<int>(cluster.num_blocks());
    const int me = static_cast<int>(cluster.block_rank());
    const int tid = threadIdx.x;
    constexpr uint32_t es = DT == Q38S_DTYPE_BF16 ? 2u : 4u;
    constexpr uint32_t per_vec = 16u / es;

    RowCtx r;
    r.v = blockIdx.y;
    r.srow = a.vrow_state_const != ~0u ? a.vrow_state_const : r.v;
    r.p = a.params[r.srow];
    r.st = a.state[r.srow];
    const uint32_t off = r.v < a.split ? r.v : r.v - a.split;
    r.rng_before = r.st.rng_state + (a.rng_step ? static_cast<uint64_t>(off) * kGamma : 0ull);
    chunk_range(a.vocab, S, me, r.lo, r.hi);
    r.n = r.hi - r.lo;
    r.pen = (r.p.flags & kFlagPenalties) != 0;
    r.nonmono = (r.p.flags & kFlagNonMonotone) != 0;
    r.freq = (r.p.flags & kFlagFrequency) != 0;
    r.counts_row = a.counts ? a.counts + static_cast<size_t>(r.srow) * a.vocab : nullptr;
    r.extra = nullptr;
    r.n_extra = 0;
    if (a.extra_mode == 1) {
        r.extra = a.extra_tokens + a.extra_offsets[r.v];
        r.n_extra = a.extra_offsets[r.v + 1] - a.extra_offsets[r.v];
    } else if (a.extra_mode == 2) {
        r.extra = a.extra_tokens;
        r.n_extra = off;
    }
    if (a.mode == kModeShardTopK) r.k_eff = a.k_out >= a.vocab ? 0u : a.k_out;
    else r.k_eff = (r.p.top_k == 0 || r.p.top_k >= a.full_vocab) ? 0u : r.p.top_k;

    // ---- shared memory carve-up
    const uint32_t nblk = (a.vocab + 127) / 128;
    const uint32_t chunk_cap = ((nblk + S - 1) / S) * 128;  // columns
    size_t area_bytes = static_cast<size_t>(chunk_cap) * es + 16;
    if (area_bytes < static_cast<size_t>(kLeaderCap) * 32) area_bytes = kLeaderCap * 32;
    area_bytes = (area_bytes + 127) & ~static_cast<size_t>(127);
    unsigned char* area = dsm;
    unsigned char* chunk = dsm;
    uint32_t* bm = reinterpret_cast<uint32_t*>(dsm + area_bytes);
    const size_t bm_bytes = ((chunk_cap / 32) * 4 + 15) & ~static_cast<size_t>(15);
    uint64_t* cand = reinterpret_cast<uint64_t*>(dsm + area_bytes + bm_bytes);
    r.bm = bm;

    // ---- phase 0: barriers, copies
    const char* row_ptr = r.v < a.split
        ? static_cast<const char*>(a.logits) + static_cast<size_t>(r.v) * a.row_stride * es
        : static_cast<const char*>(a.logits2) + static_cast<size_t>(off) * a.row_stride * es;
    const char* src = row_ptr + static_cast<size_t>(r.lo) * es;
    const uint32_t bytes = r.n * es;
    const uint32_t bulk = a.use_tma ? (bytes & ~15u) : 0u;
    const uint32_t* bm_src = a.bitmap + static_cast<size_t>(r.srow) * a.bitmap_words + r.lo / 32;
    const uint32_t bm_copy = ((((r.n + 31) / 32) * 4) + 15) & ~15u;
    if (tid == 0) {
        for (int i = 0; i < kPieces + 1; ++i) mbar_init(&c.bar[i], 1);
        c.n_cand = 0;
        c.flags = 0;
        c.theta_key = 0;
        c.max_key = 0;
        c.pub_theta = 0;
        c.pub_max = 0;
        c.list_len = 0;
        c.list_top = 0;
        c.g_count = 0;
        c.sel_token = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        // pieces of the chunk, 16-byte granular
        const uint32_t units = bulk / 16;
        for (int q = 0; q < kPieces; ++q) {
            const uint32_t u0 = units * q / kPieces, u1 = units * (q + 1) / kPieces;
            const uint32_t pb = (u1 - u0) * 16;
            mbar_arrive_expect_tx(&c.bar[q], pb);
            if (pb) tma_load_1d(chunk + u0 * 16, src + u0 * 16, pb, &c.bar[q]);
        }
        const uint32_t bmb = (r.pen && r.n > 0) ? bm_copy : 0u;
        mbar_arrive_expect_tx(&c.bar[kPieces], bmb);
        if (bmb) tma_load_1d(bm, bm_src, bmb, &c.bar[kPieces]);
    }
    // ragged tail (or everything without TMA) with plain loads, then -inf pad
    for (uint32_t b = bulk + tid; b < bytes; b += kThreads) chunk[b] = src[b];
    const uint32_t padded = ((r.n + per_vec - 1) / per_vec) * per_vec;
    for (uint32_t j = r.n + tid; j < padded; j += kThreads) {
        if (DT == Q38S_DTYPE_BF16) reinterpret_cast<uint16_t*>(chunk)[j] = 0xff80u;
        else reinterpret_cast<uint32_t*>(chunk)[j] = 0xff800000u;
    }
    cluster.sync();  // [S1] peers initialised (DSMEM below)

    bool ok = true;
    if (r.pen) {
        ok &= mbar_wait_bounded(&c.bar[kPieces], 0, kWaitLimitCycles);
        // additional penalty tokens of this call mark the private bitmap copy
        for (uint32_t e = tid; e < r.n_extra; e += kThreads) {
            const uint32_t col = static_cast<uint32_t>(r.extra[e]);
            if (col >= r.lo && col < r.hi)
                atomicOr(&bm[(col - r.lo) >> 5], 1u << ((col - r.lo) & 31));
        }
        __syncthreads();
    }

    // ---- pass 1: per-thread maximum raw logit
    const uint32_t nvec = padded / per_vec;
    const uint32_t units = bulk / 16;  // vectors covered by TMA pieces
    float best = -INFINITY;
    int bestvec = -1;
    for (int q = 0; q <= kPieces; ++q) {
        uint32_t v0, v1;
        if (q < kPieces) {
            v0 = units * q / kPieces;
            v1 = units * (q + 1) / kPieces;
            ok &= mbar_wait_bounded(&c.bar[q], 0, kWaitLimitCycles);
        } else {
            v0 = units;
            v1 = nvec;
        }
        for (uint32_t j = v0 + tid; j < v1; j += kThreads) {
            const uint4 w4 = reinterpret_cast<const uint4*>(chunk)[j];
            float f;
            if (DT == Q38S_DTYPE_BF16) {
                const __nv_bfloat162 a0 = *reinterpret_cast<const __nv_bfloat162*>(&w4.x);
                const __nv_bfloat162 a1 = *reinterpret_cast<const __nv_bfloat162*>(&w4.y);
                const __nv_bfloat162 a2 = *reinterpret_cast<const __nv_bfloat162*>(&w4.z);
                const __nv_bfloat162 a3 = *reinterpret_cast<const __nv_bfloat162*>(&w4.w);
                const __nv_bfloat162 m = __hmax2(__hmax2(a0, a1), __hmax2(a2, a3));
                f = fmaxf(__low2float(m), __high2float(m));
            } else {
                f = fmaxf(fmaxf(__uint_as_float(w4.x), __uint_as_float(w4.y)),
                          fmaxf(__uint_as_float(w4.z), __uint_as_float(w4.w)));
            }
            if (f > best) {
                best = f;
                bestvec = static_cast<int>(j);
            }
        }
    }
    const bool timed_out = __syncthreads_or(!ok);
    uint32_t tk = 0;
    if (bestvec >= 0) {
        for (uint32_t e = 0; e < per_vec; ++e) {
            const uint32_t j = static_cast<uint32_t>(bestvec) * per_vec + e;
            if (j < r.n && load_elem<DT>(chunk, j) == best) {
                const float vx = eval_exact(r, best, j, a.col_begin);
                if (vx == INFINITY) atomicOr(&c.flags, kFlagInf);
                tk = float_key(vx);
                break;
            }
        }
    }
    c.tkey[tid] = tk;
    __syncthreads();
    if (r.k_eff > 0 && r.k_eff <= static_cast<uint32_t>(kThreads) && tk != 0) {
        uint32_t rank = 0;
        for (int j = 0; j < kThreads; ++j) {
            const uint32_t o = c.tkey[j];
            rank += (o > tk) || (o == tk && j < tid);
        }
        if (rank == r.k_eff - 1) c.theta_key = tk;
    }
    const uint32_t local_max = block_max_u32(tk, c);
    if (tid == 0) {
        atomicMax(cluster.map_shared_rank(&c.pub_theta, 0), c.theta_key);
        atomicMax(cluster.map_shared_rank(&c.pub_max, 0), local_max);
        if (timed_out) atomicOr(&c.flags, kFlagTimeout);
    }
    cluster.sync();  // [S2]
    uint32_t theta_key = *cluster.map_shared_rank(&c.pub_theta, 0);
    const uint32_t mlb_key = *cluster.map_shared_rank(&c.pub_max, 0);
    if (a.mode != kModeShardTopK && r.p.min_p > 0.0f && mlb_key > kNegInfKey) {
        const float mlb = key_float(mlb_key);
        if (isfinite(mlb)) {
            const double lnmp = log(static_cast<double>(r.p.min_p));
            const double slack = (fabs(static_cast<double>(mlb)) + fabs(lnmp)) * 0x1p-18 + 1e-30;
            const float th = __double2float_rd(static_cast<double>(mlb) + lnmp - slack);
            theta_key = max(theta_key, float_key(th));
        }
    }
    const float theta = theta_key <= kNegInfKey ? -INFINITY : key_float(theta_key);

    // ---- pass 2: filter
    const bool hopeless = theta_key <= kNegInfKey && r.n > static_cast<uint32_t>(kCap);
    if (hopeless) {
        if (tid == 0) atomicOr(&c.flags, kFlagOverflow);
    } else {
        const float rho = raw_bound(theta, r.p.temperature);
        const uint32_t tok0 = a.col_begin + r.lo;
        const __nv_bfloat16 rb = __float2bfloat16_rd(rho);
        const __nv_bfloat162 rho2 = __halves2bfloat162(rb, rb);
        for (uint32_t j = tid; j < nvec; j += kThreads) {
            const uint4 w4 = reinterpret_cast<const uint4*>(chunk)[j];
            bool any;
            if (DT == Q38S_DTYPE_BF16) {
                const __nv_bfloat162 a0 = *reinterpret_cast<const __nv_bfloat162*>(&w4.x);
                const __nv_bfloat162 a1 = *reinterpret_cast<const __nv_bfloat162*>(&w4.y);
                const __nv_bfloat162 a2 = *reinterpret_cast<const __nv_bfloat162*>(&w4.z);
                const __nv_bfloat162 a3 = *reinterpret_cast<const __nv_bfloat162*>(&w4.w);
                const __nv_bfloat162 m = __hmax2(__hmax2(a0, a1), __hmax2(a2, a3));
                any = !__hblt2(m, rho2);
            } else {
                const float f = fmaxf(fmaxf(__uint_as_float(w4.x), __uint_as_float(w4.y)),
                                      fmaxf(__uint_as_float(w4.z), __uint_as_float(w4.w)));
                any = !(f < rho);
            }
            uint32_t penbits = 0;
            if (r.nonmono) {
                const uint32_t e0 = j * per_vec;
                penbits = (bm[e0 >> 5] >> (e0 & 31)) & ((1u << per_vec) - 1u);
            }
            if (!any && !penbits) continue;
            for (uint32_t e = 0; e < per_vec; ++e) {
                const uint32_t idx = j * per_vec + e;
                if (idx >= r.n) break;
                const float x = load_elem<DT>(chunk, idx);
                if ((x < rho) && !((penbits >> e) & 1u)) continue;
                const float vx = eval_exact(r, x, idx, a.col_begin);
                if (vx == INFINITY) atomicOr(&c.flags, kFlagInf);
                const uint32_t k = float_key(vx);
                if (k >= theta_key) {
                    const uint32_t pos = atomicAdd(&c.n_cand, 1u);
                    if (pos < static_cast<uint32_t>(kCap)) cand[pos] = rank_key(k, tok0 + idx);
                }
            }
        }
    }
    __syncthreads();
    uint32_t n_c = c.n_cand;
    if (n_c > static_cast<uint32_t>(kCap)) {
        if (tid == 0) atomicOr(&c.flags, kFlagOverflow);
        n_c = kCap;
    }
    __syncthreads();
    const bool overflow = (c.flags & kFlagOverflow) != 0;
    if (!overflow && n_c > 1) {
        const uint32_t p2 = pow2_at_least(n_c);
        for (uint32_t i = n_c + tid; i < p2; i += kThreads) cand[i] = 0;
        __syncthreads();
        bitonic_desc(cand, p2);
    }
    if (tid == 0) {
        c.list_len = overflow ? 0 : (r.k_eff ? min(n_c, r.k_eff) : n_c);
        c.list_top = n_c ? cand[0] : 0;
    }
    __syncthreads();
    cluster.sync();  // [S3]
    uint32_t total = 0, flags = 0;
    uint32_t lens[kMaxCluster];
    for (int s = 0; s < S; ++s) {
        const Ctl* rc = cluster.map_shared_rank(&c, s);
        lens[s] = rc->list_len;
        total += lens[s];
        flags |= rc->flags;
    }
    const bool leader = me == 0;
    if (flags & (kFlagTimeout | kFlagInf)) {
        cluster.sync();  // [S4]
        if (leader) {
            const int32_t st = (flags & kFlagTimeout) ? Q38S_ROW_TIMEOUT : Q38S_ROW_NO_FINITE;
            write_decision(a, r, -1, st);
            if (a.dist.capacity && tid == 0) {
                if (a.dist.n_candidates) a.dist.n_candidates[r.v] = 0;
                if (a.dist.n_retained) a.dist.n_retained[r.v] = 0;
            }
        }
    } else if ((flags & kFlagOverflow) || total > static_cast<uint32_t>(kLeaderCap)) {
        general_path<DT>(a, cluster, r, chunk, area, c);
        cluster.sync();
    } else {
        // fast path: gather the sorted lists into the leader
        uint64_t* lkeys = reinterpret_cast<uint64_t*>(area);          // concatenated
        uint64_t* merged = reinterpret_cast<uint64_t*>(area) + kLeaderCap;  // reused as q
        if (leader) {
            uint32_t offs = 0;
            for (int s = 0; s < S; ++s) {
                const uint64_t* rc = cluster.map_shared_rank(cand, s);
                for (uint32_t i = tid; i < lens[s]; i += kThreads) lkeys[offs + i] = rc[i];
                offs += lens[s];
            }
        }
        __syncthreads();
        cluster.sync();  // [S4] peers may exit
        if (leader) {
            const uint32_t keep = r.k_eff ? min(total, r.k_eff) : total;
            uint32_t starts[kMaxCluster];
            uint32_t acc = 0;
            for (int s = 0; s < S; ++s) {
                starts[s] = acc;
                acc += lens[s];
            }
            for (uint32_t i = tid; i < total; i += kThreads) {
                int s = 0;
                while (s + 1 < S && i >= starts[s + 1]) ++s;
                const uint64_t x = lkeys[i];
                uint32_t rank = i - starts[s];
                for (int t = 0; t < S; ++t) {
                    if (t == s) continue;
                    // entries of list t greater than x (list sorted desc)
                    uint32_t lo = 0, hi = lens[t];
                    const uint64_t* L = lkeys + starts[t];
                    while (lo < hi) {
                        const uint32_t mid = (lo + hi) >> 1;
                        if (L[mid] > x) lo = mid + 1; else hi = mid;
                    }
                    rank += lo;
                }
                if (rank < keep) merged[rank] = x;
            }
            __syncthreads();
            // move merged to the front so the epilogue arrays do not alias it
            for (uint32_t i = tid; i < keep; i += kThreads) lkeys[i] = merged[i];
            __syncthreads();
            finish_row(a, r, lkeys, keep, area, c);
        }
    }
    // speculative verification: the last virtual row to finish runs it
    if (a.mtp && leader) {
        __shared__ uint32_t last;
        __threadfence();
        __syncthreads();
        if (tid == 0) last = atomicAdd(a.ticket, 1u) == a.vrows - 1;
        __syncthreads();
        if (last) {
            __threadfence();
            if (tid == 0) {
                mtp_finish(a);
                *a.ticket = 0;
            }
        }
    }
    if (timed_out) {
        // let any copy still in flight land before the CTA's memory goes away
        for (int q = 0; q <= kPieces; ++q) mbar_wait_bounded(&c.bar[q], 0, kWaitLimitCycles);
    }
}

// --------------------------------------------------- commit kernels
// commit_tokens for each row (sampling.cc:158-172).  Block per row; the
// checksum terms depend only on (position, token) and XOR commutes, so the
// tokens are processed in parallel.  Tokens after the first invalid one are
// not applied, as the reference's loop throws at the invalid token.
__global__ void commit_tokens_kernel(RowState* state, uint32_t* bitmap, uint32_t bitmap_words,
                                     uint32_t* counts, uint32_t vocab, uint32_t col_begin,
                                     const int32_t* tokens, const uint32_t* offsets,
                                     int32_t* status) {
    __shared__ uint32_t first_bad;
    __shared__ uint64_t xr[kThreads / 32];
    const uint32_t row = blockIdx.x;
    const uint32_t b = offsets[row], e = offsets[row + 1];
    if (threadIdx.x == 0) first_bad = e - b;
    __syncthreads();
    for (uint32_t i = b + threadIdx.x; i < e; i += blockDim.x) {
        const int32_t t = tokens[i];
        const int64_t col = static_cast<int64_t>(t) - col_begin;
        if (t < 0 || col < 0 || col >= vocab) atomicMin(&first_bad, i - b);
    }
    __syncthreads();
    const uint32_t n = first_bad;
    const uint64_t c0 = state[row].canonical_tokens;
    uint64_t x = 0;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const uint32_t t = static_cast<uint32_t>(tokens[b + i]);
        const uint32_t col = t - col_begin;
        atomicOr(&bitmap[static_cast<size_t>(row) * bitmap_words + (col >> 5)], 1u << (col & 31));
        if (counts) atomicAdd(&counts[static_cast<size_t>(row) * vocab + col], 1u);
        x ^= splitmix64(static_cast<uint64_t>(t) ^ ((c0 + i + 1) * kGamma));
    }
    for (int o = 16; o > 0; o >>= 1) x ^= __shfl_xor_sync(0xffffffffu, x, o);
    if ((threadIdx.x & 31) == 0) xr[threadIdx.x >> 5] = x;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint64_t all = 0;
        for (int i = 0; i < kThreads / 32; ++i) all ^= xr[i];
        state[row].canonical_tokens = c0 + n;
        state[row].penalty_checksum ^= all;
        if (status) status[row] = n < e - b ? Q38S_ROW_BAD_TOKEN : Q38S_ROW_OK;
    }
}

// commit (sampling.cc:148-156) per row.
__global__ void commit_kernel(RowState* state, uint32_t rows, uint32_t vocab_limit,
                              q38s_decision_v1* d) {
    const uint32_t row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= rows) return;
    q38s_decision_v1 x = d[row];
    RowState& s = state[row];
    if (x.token < 0 || static_cast<uint32_t>(x.token) >= vocab_limit ||
        x.rng_before != s.rng_state || x.rng_after != x.rng_before + kGamma) {
        d[row].status = Q38S_ROW_STATE_MISMATCH;
        return;
    }
    s.rng_state = x.rng_after;
    s.sampled_tokens += 1;
}

__global__ void reset_states_kernel(RowState* state, const uint64_t* seeds, uint32_t rows) {
    const uint32_t row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= rows) return;
    state[row] = RowState{seeds[row], 0, 0, 0};
}

// ------------------------------------------------ vocab-shard merge
// One CTA per row: candidates of all shards -> global top-k (canonical
// order) -> min-p / top-p / draw.
__global__ void __launch_bounds__(kThreads) shard_merge_kernel(
    const RowParams* params, const RowState* state, const q38s_candidate* gathered,
    uint32_t rows, uint32_t n_shards, uint32_t k_local, q38s_decision_v1* decisions) {
    extern __shared__ __align__(16) unsigned char sm[];
    __shared__ Ctl c;
    const uint32_t row = blockIdx.x;
    const uint32_t total = n_shards * k_local;
    const uint32_t p2 = pow2_at_least(total);
    uint64_t* keys = reinterpret_cast<uint64_t*>(sm);
    double* w = reinterpret_cast<double*>(sm + static_cast<size_t>(p2) * 8);
    double* S = w + p2;
    double* q = S + p2;
    for (uint32_t i = threadIdx.x; i < p2; i += blockDim.x) {
        uint64_t k = 0;
        if (i < total) {
            const uint32_t s = i / k_local, j = i % k_local;
            const q38s_candidate cd =
                gathered[(static_cast<size_t>(s) * rows + row) * k_local + j];
            if (cd.token >= 0) k = rank_key(float_key(cd.value), static_cast<uint32_t>(cd.token));
        }
        keys[i] = k;
    }
    __syncthreads();
    bitonic_desc(keys, p2);
    uint32_t valid = 0;
    for (uint32_t i = threadIdx.x; i < total; i += blockDim.x) valid += keys[i] != 0;
    valid = block_sum_u32(valid, c);
    const RowParams p = params[row];
    const uint32_t keep = (p.top_k && p.top_k < valid) ? p.top_k : valid;
    const uint64_t rb = state[row].rng_state;
    epilogue(keys, keep, p, true, rb, w, S, q, c);
    if (threadIdx.x == 0) {
        q38s_decision_v1 d;
        d.token = c.e_status == Q38S_ROW_OK ? c.e_token : -1;
        d.status = c.e_status;
        d.rng_before = rb;
        d.rng_after = rb + kGamma;
        decisions[row] = d;
    }
}

// --------------------------------------------------------- argmax
// Greedy selection (replaces argmax_bf16_kernel, q38_kernels.cu:320-356):
// largest value above -3.402823466e38, lowest index among equals, -1 when
// none.  One cluster of 8 CTAs x 512 threads; DSMEM reduction.
__global__ void __launch_bounds__(512) argmax_bf16_kernel(const uint16_t* logits,
                                                          uint32_t count, int32_t* out) {
    __shared__ unsigned long long red[16];
    __shared__ unsigned long long best_cta;
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t S = cluster.num_blocks();
    const uint32_t me = cluster.block_rank();
    const uint32_t per = (count + S - 1) / S;
    const uint32_t lo = min(count, per * me), hi = min(count, lo + per);
    unsigned long long best = 0;
    for (uint32_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const float v = __uint_as_float(static_cast<uint32_t>(logits[i]) << 16);
        if (v > -3.402823466e+38f) {
            const unsigned long long k = rank_key(float_key(v), i);
            best = k > best ? k : best;
        }
    }
    best = warp_max_u64(best);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long b = 0;
        for (int i = 0; i < static_cast<int>(blockDim.x / 32); ++i) b = red[i] > b ? red[i] : b;
        best_cta = b;
    }
    cluster.sync();
    if (me == 0 && threadIdx.x == 0) {
        unsigned long long b = 0;
        for (uint32_t s = 0; s < S; ++s) {
            const unsigned long long o = *cluster.map_shared_rank(&best_cta, s);
            b = o > b ? o : b;
        }
        *out = b == 0 ? -1 : static_cast<int32_t>(rank_token(b));
    }
    cluster.sync();
}

}  // namespace

// ------------------------------------------------------------ launchers
int sample_cluster_size(uint32_t vocab) {
    const uint32_t nblk = (vocab + 127) / 128;
    return nblk >= 64 ? kMaxCluster : (nblk >= 8 ? 4 : 1);
}

size_t sample_smem_bytes(uint32_t vocab, int dtype, int cluster) {
    const uint32_t es = dtype == Q38S_DTYPE_BF16 ? 2u : 4u;
    const uint32_t nblk = (vocab + 127) / 128;
    const uint32_t chunk_cap = ((nblk + cluster - 1) / cluster) * 128;
    size_t area = static_cast<size_t>(chunk_cap) * es + 16;
    if (area < static_cast<size_t>(kLeaderCap) * 32) area = kLeaderCap * 32;
    area = (area + 127) & ~static_cast<size_t>(127);
    const size_t bm = ((chunk_cap / 32) * 4 + 15) & ~static_cast<size_t>(15);
    return area + bm + static_cast<size_t>(kCap) * 8;
}

template <int DT>
static int launch_sample_t(const SampleArgs& a, void* stream) {
    const int S = sample_cluster_size(a.vocab);
    const size_t smem = sample_smem_bytes(a.vocab, DT, S);
    auto kern = sample_rows_kernel<DT>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S, a.vrows, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = S;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, a);
    return e;
}

int launch_sample(const SampleArgs& a, void* stream) {
    if (a.vrows == 0) return cudaSuccess;
    return a.dtype == Q38S_DTYPE_BF16 ? launch_sample_t<Q38S_DTYPE_BF16>(a, stream)
                                      : launch_sample_t<Q38S_DTYPE_F32>(a, stream);
}

int launch_commit_tokens(RowState* state, uint32_t* bitmap, uint32_t bitmap_words,
                         uint32_t* counts, uint32_t vocab, uint32_t col_begin, uint32_t rows,
                         const int32_t* tokens, const uint32_t* offsets, int32_t* status,
                         void* stream) {
    if (rows == 0) return cudaSuccess;
    commit_tokens_kernel<<<rows, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        state, bitmap, bitmap_words, counts, vocab, col_begin, tokens, offsets, status);
    return cudaGetLastError();
}

int launch_commit(RowState* state, uint32_t rows, uint32_t vocab,
                  q38s_decision_v1* decisions, void* stream) {
    if (rows == 0) return cudaSuccess;
    commit_kernel<<<(rows + 127) / 128, 128, 0, static_cast<cudaStream_t>(stream)>>>(
        state, rows, vocab, decisions);
    return cudaGetLastError();
}

int launch_reset_states(RowState* state, const uint64_t* seeds, uint32_t rows, void* stream) {
    if (rows == 0) return cudaSuccess;
    reset_states_kernel<<<(rows + 127) / 128, 128, 0, static_cast<cudaStream_t>(stream)>>>(
        state, seeds, rows);
    return cudaGetLastError();
}

int launch_shard_merge(const RowParams* params, const RowState* state, uint32_t rows,
                       const q38s_candidate* gathered, uint32_t n_shards, uint32_t k_local,
                       q38s_decision_v1* decisions, void* stream) {
    if (rows == 0) return cudaSuccess;
    uint32_t p2 = 1;
    while (p2 < n_shards * k_local) p2 <<= 1;
    const size_t smem = static_cast<size_t>(p2) * 32;
    cudaError_t e = cudaFuncSetAttribute(shard_merge_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    shard_merge_kernel<<<rows, kThreads, smem, static_cast<cudaStream_t>(stream)>>>(
        params, state, gathered, rows, n_shards, k_local, decisions);
    return cudaGetLastError();
}

int launch_argmax_bf16(const uint16_t* logits, uint32_t count, int32_t* out, void* stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(8, 1, 1);
    cfg.blockDim = dim3(512, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 8;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, argmax_bf16_kernel, logits, count, out);
}

}  // namespace q38s
