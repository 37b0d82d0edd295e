// Small kernels beside the streaming sampler (q38s_stream.cu): history
// commits (sampling.cc:158-172), decision commits (sampling.cc:148-156),
// state resets, the vocab-shard merge (the union of every shard's top-k
// list, then the reference epilogue) and greedy argmax
// (q38_kernels.cu:320-356).
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include "q38s_kernels.cuh"

namespace cg = cooperative_groups;

namespace q38s {

namespace {

// Shared words of the shard-merge kernel: block reductions and the
// epilogue's results.
struct __align__(16) Ctl {
    uint32_t red_u32[kThreads / 32];
    // epilogue results
    int32_t e_token;
    int32_t e_status;
    uint32_t e_n;
    uint32_t e_r;
    uint32_t e_sel;
    double e_total;
    double e_draw;
};

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
// Column partition: 128-column blocks spread over S CTAs.

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

constexpr uint32_t kMaxShards = 64;  // column shards one merge takes

// ------------------------------------------------ vocab-shard merge
// One CTA per row.  Each shard's list arrives sorted in canonical order
// (value desc, token asc) with its invalid entries (token -1) at the end, and
// tokens are distinct across shards, so an entry's position in the merged
// order is its index in its own list plus, for every other shard, the number
// of that shard's entries that rank above it (a binary search).  Entries
// whose position is below the row's top-k are written to their place; no
// sort is needed.  Then min-p / top-p / the draw (the stream kernel's
// epilogue) over that prefix.
__global__ void __launch_bounds__(kThreads) shard_merge_kernel(
    const RowParams* params, const RowState* state, const q38s_candidate* gathered,
    uint32_t rows, uint32_t n_shards, uint32_t k_local, q38s_decision_v1* decisions) {
    extern __shared__ __align__(16) unsigned char sm[];
    __shared__ Ctl c;
    __shared__ uint32_t len[kMaxShards];
    const uint32_t row = blockIdx.x;
    const uint32_t total = n_shards * k_local;
    uint64_t* keys = reinterpret_cast<uint64_t*>(sm);         // [total], by shard
    uint64_t* out = keys + total;                             // [k_local]: the merged prefix
    double* w = reinterpret_cast<double*>(out + k_local);
    double* S = w + k_local;
    double* q = S + k_local;
    if (threadIdx.x < n_shards) len[threadIdx.x] = 0;
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < total; i += blockDim.x) {
        const uint32_t s = i / k_local, j = i % k_local;
        const q38s_candidate cd = gathered[(static_cast<size_t>(s) * rows + row) * k_local + j];
        const bool ok = cd.token >= 0;
        keys[i] = ok ? rank_key(float_key(cd.value), static_cast<uint32_t>(cd.token)) : 0ull;
        if (ok) atomicMax(&len[s], j + 1);  // valid entries form a prefix of the list
    }
    __syncthreads();
    uint32_t valid = 0;
    for (uint32_t s = 0; s < n_shards; ++s) valid += len[s];
    const RowParams p = params[row];
    const uint32_t keep = (p.top_k && p.top_k < valid) ? p.top_k : valid;
    for (uint32_t i = threadIdx.x; i < total; i += blockDim.x) {
        const uint32_t s = i / k_local, j = i % k_local;
        if (j >= len[s]) continue;
        const uint64_t x = keys[i];
        uint32_t pos = j;
        for (uint32_t s2 = 0; s2 < n_shards && pos < keep; ++s2) {
            if (s2 == s) continue;
            const uint64_t* l = keys + static_cast<size_t>(s2) * k_local;
            uint32_t lo = 0, hi = len[s2];  // entries of l above x: the first index below x
            while (lo < hi) {
                const uint32_t mid = (lo + hi) >> 1;
                if (l[mid] > x) lo = mid + 1;
                else hi = mid;
            }
            pos += lo;
        }
        if (pos < keep) out[pos] = x;
    }
    __syncthreads();
    const uint64_t rb = state[row].rng_state;
    epilogue(out, keep, p, true, rb, w, S, q, c);
    if (threadIdx.x == 0) {
        q38s_decision_v1 d;
        d.token = c.e_status == Q38S_ROW_OK ? c.e_token : -1;
        d.status = c.e_status;
        d.rng_before = rb;
        d.rng_after = rb + kGamma;
        decisions[row] = d;
    }
}

// ------------------------------------------------------ MoE router
// Router top-k (replaces the reference's cuda_topk_router_bf16,
// q38_kernels.cu:667-687, kernels :358-480), one warp per token, the token's
// logits in shared memory.  The top_k experts come from top_k rounds of a
// warp-wide maximum of 64-bit keys (a selected key is cleared):
//   by_logit  (512 experts, normalised; the reference's decode path): key
//             (logit desc, expert asc); numerator expf(logit - largest);
//   otherwise (the reference's general path): key (expf(x - max) desc,
//             expert asc), max = fmaxf over the token's logits.
// The denominators are the reference's sequential fp32 sums: over the ranks
// (normalised) or over all experts in expert order; weight = numerator /
// denominator.
__global__ void __launch_bounds__(kThreads) topk_router_kernel(
    const uint16_t* logits, int32_t* expert_ids, float* expert_weights, uint32_t tokens,
    uint32_t experts, uint32_t top_k, int normalize, int by_logit) {
    extern __shared__ __align__(16) unsigned char sm[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t token = blockIdx.x * (kThreads / 32) + warp;
    if (token >= tokens) return;
    float* x = reinterpret_cast<float*>(sm) + static_cast<size_t>(warp) * experts;
    float* p = x + static_cast<size_t>(kThreads / 32) * experts;  // expf(x - max), general path
    const uint16_t* row = logits + static_cast<size_t>(token) * experts;
    float mx = -3.402823466e+38f;
    for (uint32_t e = lane; e < experts; e += 32) {
        const float v = __uint_as_float(static_cast<uint32_t>(row[e]) << 16);
        x[e] = v;
        mx = fmaxf(mx, v);
    }
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (!by_logit)
        for (uint32_t e = lane; e < experts; e += 32) p[e] = expf(x[e] - mx);
    __syncwarp();
    __shared__ float num[kThreads / 32][32];
    __shared__ int32_t ids[kThreads / 32][32];
    float top_logit = 0.0f;
    for (uint32_t rank = 0; rank < top_k; ++rank) {
        uint64_t best = 0;
        for (uint32_t e = lane; e < experts; e += 32) {
            const float f = by_logit ? x[e] : p[e];
            const uint64_t key = (static_cast<uint64_t>(float_key(f)) << 32) | (0xffffffffu - e);
            if (f == f && key > best) best = key;  // a selected entry holds NaN
        }
        best = warp_max_u64(best);
        if (best == 0) {  // nothing left that is a number: the reference's empty slot
            if (lane == 0) {
                ids[warp][rank] = -1;
                num[warp][rank] = -3.402823466e+38f;
            }
            __syncwarp();
            continue;
        }
        const uint32_t e = rank_token(best);
        if (lane == 0) {
            ids[warp][rank] = static_cast<int32_t>(e);
            num[warp][rank] = by_logit ? x[e] : p[e];
        }
        __syncwarp();
        if (lane == (e & 31)) {  // the owner of expert e takes it out
            if (by_logit) x[e] = __uint_as_float(0x7fffffffu);
            else p[e] = __uint_as_float(0x7fffffffu);
        }
        __syncwarp();
    }
    if (lane == 0) {
        if (by_logit) {
            top_logit = num[warp][0];
            for (uint32_t r = 0; r < top_k; ++r) num[warp][r] = expf(num[warp][r] - top_logit);
        }
        float den = 0.0f;
        if (normalize) {
            for (uint32_t r = 0; r < top_k; ++r) den += num[warp][r];
        } else {
            // the sum over all experts in expert order (selected entries were
            // cleared: recompute them)
            for (uint32_t e = 0; e < experts; ++e)
                den += expf(__uint_as_float(static_cast<uint32_t>(row[e]) << 16) - mx);
        }
        for (uint32_t r = 0; r < top_k; ++r) {
            const size_t o = static_cast<size_t>(token) * top_k + r;
            expert_ids[o] = ids[warp][r];
            expert_weights[o] = num[warp][r] / den;
        }
    }
}

// --------------------------------------------------------- argmax
// Greedy selection (replaces argmax_bf16_kernel, q38_kernels.cu:320-356):
// largest value above -3.402823466e38, lowest index among equals, -1 when
// none.  One cluster of 8 CTAs x 512 threads: the row in 16-byte vectors
// (four per thread in flight at once; scalar head and tail around them when
// the row is not 16-byte aligned), 64-bit rank keys (value key, inverted
// index) reduced by warp, CTA and DSMEM.
__device__ __forceinline__ void argmax_take(unsigned long long& best, uint32_t bits, uint32_t i) {
    const float v = __uint_as_float(bits << 16);
    if (v > -3.402823466e+38f) {
        const unsigned long long k = rank_key(float_key(v), i);
        best = k > best ? k : best;
    }
}
__global__ void __launch_bounds__(512) argmax_bf16_kernel(const uint16_t* logits,
                                                          uint32_t count, int32_t* out) {
    __shared__ unsigned long long red[16];
    __shared__ unsigned long long best_cta;
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t nt = cluster.num_blocks() * blockDim.x;
    const uint32_t me = cluster.block_rank();
    const uint32_t gt = me * blockDim.x + threadIdx.x;
    const uint32_t mis = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(logits) & 15u) / 2u;
    const uint32_t head = min(count, (8u - mis) & 7u);
    const uint32_t nvec = (count - head) / 8u;
    const uint4* vec = reinterpret_cast<const uint4*>(logits + head);
    unsigned long long best = 0;
    for (uint32_t i = gt; i < head; i += nt) argmax_take(best, logits[i], i);
    for (uint32_t base = 0; base < nvec; base += 4u * nt) {
        uint4 w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t j = base + k * nt + gt;
            w[k] = j < nvec ? __ldg(&vec[j]) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t j = base + k * nt + gt;
            if (j < nvec) {
                const uint32_t i0 = head + j * 8u;
                const uint32_t q[4] = {w[k].x, w[k].y, w[k].z, w[k].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    argmax_take(best, q[e] & 0xffffu, i0 + 2 * e);
                    argmax_take(best, q[e] >> 16, i0 + 2 * e + 1);
                }
            }
        }
    }
    for (uint32_t i = head + nvec * 8u + gt; i < count; i += nt) argmax_take(best, logits[i], i);
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
        for (uint32_t s = 0; s < cluster.num_blocks(); ++s) {
            const unsigned long long o = *cluster.map_shared_rank(&best_cta, s);
            b = o > b ? o : b;
        }
        *out = b == 0 ? -1 : static_cast<int32_t>(rank_token(b));
    }
    cluster.sync();
}

}  // namespace

// ------------------------------------------------------------ launchers
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
    if (n_shards > kMaxShards) return cudaErrorInvalidValue;
    const size_t smem = static_cast<size_t>(n_shards) * k_local * 8 + static_cast<size_t>(k_local) * 32;
    static size_t configured[64] = {};  // largest shared-memory size set, per device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (smem > 48 * 1024 && smem > configured[dev]) {
        e = cudaFuncSetAttribute(shard_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        configured[dev] = smem;
    }
    shard_merge_kernel<<<rows, kThreads, smem, static_cast<cudaStream_t>(stream)>>>(
        params, state, gathered, rows, n_shards, k_local, decisions);
    return cudaGetLastError();
}

int launch_topk_router(const uint16_t* logits, int32_t* expert_ids, float* expert_weights,
                       uint32_t tokens, uint32_t experts, uint32_t top_k, int normalize,
                       int by_logit, void* stream) {
    constexpr uint32_t kWarps = kThreads / 32;
    const size_t smem = static_cast<size_t>(2) * kWarps * experts * sizeof(float);
    static size_t configured[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (smem > 48 * 1024 && smem > configured[dev]) {
        e = cudaFuncSetAttribute(topk_router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        configured[dev] = smem;
    }
    topk_router_kernel<<<(tokens + kWarps - 1) / kWarps, kThreads, smem,
                         static_cast<cudaStream_t>(stream)>>>(
        logits, expert_ids, expert_weights, tokens, experts, top_k, normalize, by_logit);
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
