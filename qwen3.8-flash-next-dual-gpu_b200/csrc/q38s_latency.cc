// Batch-1 decode latency as a native caller sees it: the wall time of
// q38::TransactionalSampler::prepare_device per step, with commit() and
// commit_token() between steps, the way the reference executor drives its
// sampler (executor.cc:455 prepare, :538 commit of the decision, :663
// commit_token of the emitted token).  The benchmark's configuration 2
// calls it through ctypes; it is a measurement harness over the public C++
// API, not part of the engine (lib/libq38s_latency.so, linked against
// lib/libq38s.so).
#include <chrono>
#include <cstddef>
#include <cstdint>
#include <exception>
#include <vector>

#include "q38/sampling.h"

// pool: pool_rows bf16 rows of `vocabulary` logits on the current device;
// step i samples row i % pool_rows.  lat_us receives `steps` latencies (the
// `warmup` steps before them are not recorded).  Returns 0, or non-zero
// when an argument is null or the sampler threw.
extern "C" int q38s_latency_batch1(uint32_t vocabulary, const void* config_v1,
                                   const int32_t* history, size_t n_history,
                                   const uint16_t* pool, uint32_t pool_rows, uint32_t warmup,
                                   uint32_t steps, double* lat_us) {
    if (!config_v1 || !pool || !lat_us || pool_rows == 0) return 1;
    try {
        q38::TransactionalSampler s(vocabulary,
                                    *static_cast<const q38::SamplingConfigV1*>(config_v1));
        if (n_history) s.commit_tokens(std::vector<int32_t>(history, history + n_history));
        for (uint32_t i = 0; i < warmup + steps; ++i) {
            const uint16_t* row = pool + static_cast<size_t>(i % pool_rows) * vocabulary;
            const auto t0 = std::chrono::steady_clock::now();
            const q38::SamplerDecisionV1 d =
                s.prepare_device(row, q38::DType::kBFloat16, vocabulary);
            const auto t1 = std::chrono::steady_clock::now();
            s.commit(d);
            s.commit_token(d.token);
            if (i >= warmup)
                lat_us[i - warmup] = std::chrono::duration<double, std::micro>(t1 - t0).count();
        }
    } catch (const std::exception&) {
        return 2;
    }
    return 0;
}
