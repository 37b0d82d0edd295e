// Device-logits decode loop (TEST INFRASTRUCTURE ONLY): the caller side of
// the executor integration in which the stage-1 logits never leave the GPU.
//
// The reference copies the LM head's logits to the host and synchronises
// the stream before every sampled step (cuda_backend.cu:2765-2779), then
// samples on the host (executor.cc:450-469).  Here the logits of each step
// are written into device memory by a kernel (standing for the LM head's
// workspace.logits, cuda_backend.cu:957) and handed to
// TransactionalSampler::prepare_device on the same stream: no D2H copy of
// the logits and no synchronisation before sampling; only the 24-byte
// decision comes back.  The step sequence is the executor's sampled decode
// (executor.cc:672-687 decode_one): the first sample after an appended
// chunk takes the chunk as additional penalty tokens (executor.cc:455-459),
// then commit(decision) (executor.cc:537-540) and commit_token of the
// published token (executor.cc:684).
//
// Logits follow the reference mock backend (mock_backend.cc:197-204): -8
// everywhere, +8 at the predicted next token, +7.5 at the one after it, the
// prediction being mix(previous token ^ position * 0x9e3779b97f4a7c15) mod V
// (mock_backend.cc:81-86; mix is the splitmix64 output function), at the
// Qwen3.8 vocabulary of 248,320.
//
// One source, two arms:
//   dev_q38s  (nvcc, -DQ38S_DEVICE_ARM) this repository's sampler on device
//             logits;
//   dev_ref   (g++) the reference's CPU sampler (src/sampling.cc) on the
//             same logits built on the host.
// Identical output lines mean the device path is a drop-in.  A final
// "timing" line (not compared) gives the mean step time of each arm: for
// dev_q38s prepare_device + commit + commit_token on resident logits; for
// dev_ref the same on host logits, to which the reference adds the 485 KiB
// D2H copy and stream synchronisation.
#include "q38/sampling.h"

#include <chrono>
#include <cinttypes>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <stdexcept>
#include <vector>

#ifdef Q38S_DEVICE_ARM
#include <cuda_runtime.h>
#endif

namespace {

constexpr std::uint32_t kVocab = 248320;

std::uint64_t mix(std::uint64_t v) {
    v ^= v >> 30u;
    v *= UINT64_C(0xbf58476d1ce4e5b9);
    v ^= v >> 27u;
    v *= UINT64_C(0x94d049bb133111eb);
    return v ^ (v >> 31u);
}

std::int32_t predict(std::int32_t token, std::uint64_t position) {
    return static_cast<std::int32_t>(
        mix(static_cast<std::uint32_t>(token) ^ (position * UINT64_C(0x9e3779b97f4a7c15))) %
        kVocab);
}

constexpr std::uint16_t kMinus8 = 0xc100;  // bf16 -8.0
constexpr std::uint16_t kPlus8 = 0x4100;   // bf16 8.0
constexpr std::uint16_t kPlus75 = 0x40f0;  // bf16 7.5

#ifdef Q38S_DEVICE_ARM
__global__ void mock_logits_kernel(std::uint16_t* out, std::uint32_t n, std::int32_t next) {
    const std::uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const std::uint32_t hot = static_cast<std::uint32_t>(next);
    out[i] = i == hot ? kPlus8 : (i == (hot + 1u) % n ? kPlus75 : kMinus8);
}
#endif

q38::SamplingConfigV1 config(std::uint32_t top_k, float top_p, float temperature, float rep,
                             float freq, float presence, std::uint64_t seed) {
    q38::SamplingConfigV1 c;
    c.mode = q38::SamplingModeV1::kTopKTopP;
    c.top_k = top_k;
    c.top_p = top_p;
    c.temperature = temperature;
    c.repetition_penalty = rep;
    c.frequency_penalty = freq;
    c.presence_penalty = presence;
    c.seed = seed;
    return c;
}

void print_step(const char* name, int step, std::int32_t token, const q38::SamplerStateV1& s) {
    std::printf("{\"session\":\"%s\",\"step\":%d,\"token\":%d,\"rng_state\":%" PRIu64
                ",\"sampled\":%" PRIu64 ",\"canonical\":%" PRIu64 ",\"checksum\":%" PRIu64 "}\n",
                name, step, token, s.rng_state, s.sampled_tokens, s.canonical_tokens,
                s.penalty_checksum);
}

struct Logits {
#ifdef Q38S_DEVICE_ARM
    std::uint16_t* dev = nullptr;
    cudaStream_t stream = nullptr;
    Logits() {
        if (cudaMalloc(&dev, sizeof(std::uint16_t) * kVocab) != cudaSuccess ||
            cudaStreamCreate(&stream) != cudaSuccess)
            throw std::runtime_error("device buffers");
    }
    ~Logits() {
        cudaFree(dev);
        cudaStreamDestroy(stream);
    }
    q38::SamplerDecisionV1 sample(q38::TransactionalSampler& s, std::int32_t next,
                                  const std::vector<std::int32_t>& extra) {
        mock_logits_kernel<<<(kVocab + 255) / 256, 256, 0, stream>>>(dev, kVocab, next);
        return s.prepare_device(dev, q38::DType::kBFloat16, kVocab, extra, stream);
    }
#else
    std::vector<std::uint16_t> host = std::vector<std::uint16_t>(kVocab, kMinus8);
    std::int32_t last = -1;
    q38::SamplerDecisionV1 sample(q38::TransactionalSampler& s, std::int32_t next,
                                  const std::vector<std::int32_t>& extra) {
        if (last >= 0) {
            host[static_cast<std::uint32_t>(last)] = kMinus8;
            host[(static_cast<std::uint32_t>(last) + 1u) % kVocab] = kMinus8;
        }
        host[static_cast<std::uint32_t>(next)] = kPlus8;
        host[(static_cast<std::uint32_t>(next) + 1u) % kVocab] = kPlus75;
        last = next;
        return s.prepare(host, extra);
    }
#endif
};

double session(Logits& lg, const char* name, const q38::SamplingConfigV1& cfg, int steps) {
    q38::TransactionalSampler s(kVocab, cfg);
    // an appended prompt chunk: its tokens are the first sample's extra
    // penalty tokens, then join the history (executor.cc:455-459, :643)
    const std::vector<std::int32_t> prompt{11, 12, 13, 12, 240000};
    std::uint64_t position = prompt.size();
    std::int32_t prev = prompt.back();
    auto d = lg.sample(s, predict(prev, position), prompt);
    s.commit(d);
    s.commit_tokens(prompt);
    s.commit_token(d.token);
    print_step(name, 0, d.token, s.state());
    prev = d.token;
    const auto t0 = std::chrono::steady_clock::now();
    for (int i = 1; i <= steps; ++i) {
        ++position;
        d = lg.sample(s, predict(prev, position), {});
        s.commit(d);
        s.commit_token(d.token);
        print_step(name, i, d.token, s.state());
        prev = d.token;
    }
    const auto dt = std::chrono::duration<double, std::micro>(
                        std::chrono::steady_clock::now() - t0).count();
    return dt / steps;
}

}  // namespace

int main(int argc, char** argv) {
    const int steps = argc > 1 ? std::atoi(argv[1]) : 120;
    try {
        Logits lg;
        const double a = session(lg, "fixture", config(3, 0.9f, 0.8f, 1.1f, 0.2f, 0.1f, 170), steps);
        // top_k = 0: the whole vocabulary is the candidate set (the GPU
        // sampler's general path)
        const double b = session(lg, "topk0", config(0, 0.95f, 1.0f, 1.0f, 0.0f, 0.0f, 2024), steps);
        const double c = session(lg, "penalties", config(20, 1.0f, 0.6f, 1.2f, 0.3f, 0.5f, 77), steps);
        std::printf("{\"op\":\"timing\",\"us_per_step\":{\"fixture\":%.2f,\"topk0\":%.2f,"
                    "\"penalties\":%.2f}}\n", a, b, c);
    } catch (const std::exception& e) {
        std::printf("{\"error\":\"%s\"}\n", e.what());
        return 2;
    }
    return 0;
}
