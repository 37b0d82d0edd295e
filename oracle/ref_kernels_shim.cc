// C entry points over the reference's own device kernels (TEST AND BENCH
// INFRASTRUCTURE ONLY): cuda/q38_kernels.cu of the reference, compiled
// unmodified for sm_100a by oracle/Makefile into _ref/libq38ref_kernels.so.
//   q38ref_argmax_bf16        cuda_argmax_bf16 (q38_kernels.cu:656-665,
//                             kernel :320-356)
//   q38ref_topk_router_bf16   cuda_topk_router_bf16 (q38_kernels.cu:667-687,
//                             kernels :358-480)
// Both return 0, or 1 when the reference throws (message in err).
#include "q38/cuda_kernels.h"

#include <cstdint>
#include <cstring>
#include <exception>

namespace {
void put(char* err, std::size_t n, const char* msg) {
    if (err && n) {
        std::strncpy(err, msg, n - 1);
        err[n - 1] = 0;
    }
}
}  // namespace

extern "C" int q38ref_argmax_bf16(const std::uint16_t* logits, std::uint32_t count,
                                  std::int32_t* output, void* stream, int device, char* err,
                                  std::size_t err_n) {
    try {
        q38::cuda_argmax_bf16(logits, count, output, stream, device);
        return 0;
    } catch (const std::exception& e) {
        put(err, err_n, e.what());
        return 1;
    }
}

extern "C" int q38ref_topk_router_bf16(const std::uint16_t* logits, std::int32_t* expert_ids,
                                       float* expert_weights, std::uint32_t tokens,
                                       std::uint32_t experts, std::uint32_t top_k,
                                       int normalize_top_k, void* stream, int device, char* err,
                                       std::size_t err_n) {
    try {
        q38::cuda_topk_router_bf16(logits, expert_ids, expert_weights, tokens, experts, top_k,
                                   normalize_top_k != 0, stream, device);
        return 0;
    } catch (const std::exception& e) {
        put(err, err_n, e.what());
        return 1;
    }
}
