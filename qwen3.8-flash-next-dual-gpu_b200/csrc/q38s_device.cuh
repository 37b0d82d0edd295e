// Device-side building blocks of the sampler kernels (sm_100a).
//
//  * TMA bulk copies (cp.async.bulk, 1-D, no multicast) with mbarrier
//    completion and bounded waits,
//  * the reference's RNG (src/sampling.cc:22-36) and penalty/temperature
//    transform (sampling.cc:75-92) with the same IEEE float operations,
//  * order-preserving 32-bit keys and the 64-bit canonical rank key
//    (value desc, token asc).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace q38s {

constexpr uint64_t kGamma = 0x9e3779b97f4a7c15ull;
constexpr uint64_t kAcceptDomain = 0xd6e8feb86659fd93ull;

// ---------------------------------------------------------------- RNG
// splitmix64 / next_state / uniform01: sampling.cc:22-36.
__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t v) {
    v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
    v = (v ^ (v >> 27)) * 0x94d049bb133111ebull;
    return v ^ (v >> 31);
}
__host__ __device__ __forceinline__ double uniform01(uint64_t state) {
    return static_cast<double>(splitmix64(state) >> 11) *
           (1.0 / 9007199254740992.0);
}

// -------------------------------------------------------- order keys
// Order-preserving key of a float: larger float -> larger key.  -0.0 is
// folded onto +0.0 first (the reference's comparator treats them as equal).
__device__ __forceinline__ uint32_t float_key(float v) {
    const uint32_t b = __float_as_uint(__fadd_rn(v, 0.0f));
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
    const uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return __uint_as_float(b);
}
// Canonical rank key: sorting descending orders by (value desc, token asc).
__device__ __forceinline__ uint64_t rank_key(uint32_t vkey, uint32_t token) {
    return (static_cast<uint64_t>(vkey) << 32) | (0xffffffffu - token);
}
__device__ __forceinline__ uint32_t rank_token(uint64_t rk) {
    return 0xffffffffu - static_cast<uint32_t>(rk);
}
__device__ __forceinline__ float rank_value(uint64_t rk) {
    return key_float(static_cast<uint32_t>(rk >> 32));
}
constexpr uint32_t kNegInfKey = 0x007fffffu;  // float_key(-inf)

// ------------------------------------------------- penalty/temperature
// Per-row sampling parameters as the kernels consume them.
struct RowParams {
    uint32_t top_k;
    float top_p;
    float min_p;
    float temperature;
    float repetition_penalty;
    float frequency_penalty;
    float presence_penalty;
    uint32_t flags;
};
constexpr uint32_t kFlagPenalties = 1u;     // rep != 1 || presence != 0 || frequency != 0
constexpr uint32_t kFlagNonMonotone = 2u;   // presence < 0 || frequency < 0
constexpr uint32_t kFlagFrequency = 4u;     // frequency != 0 (needs counts)

// Stage A of sampling.cc:76-92 for one token.  `penalized` is count != 0,
// `count` the committed + additional count (used only for frequency).
// Every operation is an explicitly rounded IEEE op, so no FMA contraction
// can change a result relative to the reference.
__device__ __forceinline__ float transform(float x, bool penalized,
                                           uint64_t count,
                                           const RowParams& p) {
    if (!isfinite(x)) x = -INFINITY;
    if (penalized) {
        if (p.repetition_penalty != 1.0f)
            x = x > 0.0f ? __fdiv_rn(x, p.repetition_penalty)
                         : __fmul_rn(x, p.repetition_penalty);
        x = __fsub_rn(x, p.presence_penalty);
        x = __fsub_rn(x, __fmul_rn(p.frequency_penalty,
                                   __ull2float_rn(count)));
    }
    return __fdiv_rn(x, p.temperature);
}

// A raw-logit bound rho with:  transform(x) >= theta  =>  x >= rho, for
// rows whose penalties can only lower a logit (rep >= 1, presence >= 0,
// frequency >= 0).  Derivation: transform(x) <= fl(x / T); fl(x/T) >= theta
// implies x >= theta*T*(1 - 2^-24); the margin below covers the rounding of
// theta*T and subnormal/zero thresholds.
__device__ __forceinline__ float raw_bound(float theta, float temperature) {
    if (!(theta > -INFINITY)) return -INFINITY;
    if (isinf(theta)) return theta;  // +inf: only +inf results qualify
    const float t = __fmul_rn(theta, temperature);
    const float margin = fabsf(t) * 0x1p-20f + 0x1p-126f;
    return __fsub_rn(t, margin);
}

// ------------------------------------------------------------- bf16
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// ------------------------------------------------------- TMA / mbarrier
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(count)
                 : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                     smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}
// 1-D bulk copy global -> this CTA's shared memory, completion counted on
// `bar`.  dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void tma_load_1d(void* dst, const void* src, uint32_t bytes,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}
// atomicAdd with acquire-release semantics at GPU scope; returns the old value.
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}" : "=r"(ok) : "r"(smem_addr(bar)), "r"(phase) : "memory");
    return ok != 0;
}
// Bounded wait: gives up after `limit` clock cycles.  Returns true on
// completion.  Callers turn a timeout into a row status instead of hanging.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t phase,
                                                  long long limit) {
    const long long start = clock64();
    while (!mbar_try_wait(bar, phase)) {
        if (clock64() - start > limit) return false;
    }
    return true;
}
// ~2 s at 1.9 GHz: far beyond any legitimate copy of a few tens of KB.
constexpr long long kWaitLimitCycles = 4000000000ll;

// ------------------------------------------- thread-block cluster (DSMEM)
// The address of the same shared-memory location in CTA `rank` of this
// CTA's cluster (its own rank included), for the shared::cluster forms.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(p)), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_cluster_u32(uint32_t addr, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_cluster_u64(uint32_t addr) {
    uint64_t v;
    asm volatile("ld.shared::cluster.u64 %0, [%1];" : "=l"(v) : "r"(addr) : "memory");
    return v;
}
// Orders this thread's earlier accesses (and those it has synchronised
// with) before its later ones for every thread of the cluster.
__device__ __forceinline__ void fence_acq_rel_cluster() {
    asm volatile("fence.acq_rel.cluster;" ::: "memory");
}
// One arrival, release at cluster scope, on an mbarrier given by its
// cluster address (another CTA's, or this CTA's own).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar)
                 : "memory");
}
// Bounded wait, acquire at cluster scope, on one of this CTA's mbarriers
// that other CTAs of the cluster arrive on.  Returns true on completion.
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t* bar, uint32_t phase,
                                                          long long limit) {
    const long long start = clock64();
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n"
            " mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
            " selp.u32 %0, 1, 0, p;\n}" : "=r"(ok) : "r"(smem_addr(bar)), "r"(phase) : "memory");
        if (ok) return true;
        if (clock64() - start > limit) return false;
    }
}
// Every thread of every CTA of the cluster (the whole block calls it).
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ------------------------------------------------------------ warp utils
__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
    for (int o = 16; o > 0; o >>= 1) {
        const uint64_t w = __shfl_xor_sync(0xffffffffu, v, o);
        v = w > v ? w : v;
    }
    return v;
}
__device__ __forceinline__ uint32_t warp_max_u32(uint32_t v) {
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ uint32_t warp_sum_u32(uint32_t v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ uint32_t warp_min_u32(uint32_t v) {
    for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  // namespace q38s
