// Executor harness (TEST INFRASTRUCTURE ONLY): drives the reference runtime's
// own DualStageExecutor with its mock stage backends (src/executor.cc,
// src/mock_backend.cc and their dependencies, compiled unmodified from the
// reference sources by oracle/Makefile) through a fixed script of sampled
// decode steps, and prints one JSON object per step.
//
// The same file is linked twice:
//   exec_ref   against the reference's include/q38/sampling.h and
//              src/sampling.cc (the original CPU sampler);
//   exec_q38s  against this repository's include/q38/sampling.h and
//              lib/libq38s.so (the GPU sampler as a drop-in).
// Their outputs must be identical: the executor calls the sampler exactly as
// it does in production (executor.cc:450-469 prepare, :537-540 commit, :643 /
// :663 / :684 / :734 commit_token(s), :767 reset), and the mock logits
// (mock_backend.cc:197-204: -8 everywhere, +8 at the predicted token, +7.5 at
// the next one) put no tied values inside any retained set of the script's
// configurations, so the reference's libstdc++ tie order cannot show.
//
// Part 1 repeats the operations of the reference's only sampler test,
// test_transactional_sampling (tests/test_runtime.cc:1088-1137): retry
// determinism of prepare, commit, commit_tokens, and the executor counters
// through append / seed_decode / decode_one / speculative_step.  Part 2 runs
// longer decode sessions under three sampling configurations, with a reset.
#include "q38/executor.h"
#include "q38/mock_backend.h"
#include "q38/sampling.h"

#include <cinttypes>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

namespace {

std::uint16_t bf16_rne(float value) {
    std::uint32_t bits = 0;
    std::memcpy(&bits, &value, sizeof(bits));
    return static_cast<std::uint16_t>((bits + 0x7fffu + ((bits >> 16u) & 1u)) >> 16u);
}

void print_state(const char* op, const q38::SamplerStateV1& s,
                 const std::vector<std::int32_t>& tokens, const q38::ExecutorStatsV1* stats) {
    std::printf("{\"op\":\"%s\",\"rng_state\":%" PRIu64 ",\"sampled\":%" PRIu64
                ",\"canonical\":%" PRIu64 ",\"checksum\":%" PRIu64 ",\"tokens\":[",
                op, s.rng_state, s.sampled_tokens, s.canonical_tokens, s.penalty_checksum);
    for (std::size_t i = 0; i < tokens.size(); ++i)
        std::printf("%s%d", i ? "," : "", tokens[i]);
    std::printf("]");
    if (stats)
        std::printf(",\"sampled_stat\":%" PRIu64 ",\"spec_txn\":%" PRIu64 ",\"drafted\":%" PRIu64,
                    stats->sampled_tokens, stats->speculative_transactions,
                    stats->drafted_tokens);
    std::printf("}\n");
}

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

int part_sampler() {
    // the fixture of tests/test_runtime.cc:1088-1103
    const auto cfg = config(3, 0.9f, 0.8f, 1.1f, 0.2f, 0.1f, 170);
    q38::TransactionalSampler sampler(4, cfg);
    const std::vector<std::uint16_t> logits{bf16_rne(0.0f), bf16_rne(1.0f), bf16_rne(2.0f),
                                            bf16_rne(3.0f)};
    const auto first = sampler.prepare(logits, {3, 3});
    const auto retry = sampler.prepare(logits, {3, 3});
    if (first.token != retry.token || first.rng_before != retry.rng_before ||
        first.rng_after != retry.rng_after) {
        std::printf("{\"error\":\"prepare is not retry-deterministic\"}\n");
        return 1;
    }
    print_state("fixture_prepare", sampler.state(), {first.token}, nullptr);
    sampler.commit(first);
    print_state("fixture_commit", sampler.state(), {}, nullptr);
    sampler.commit_tokens({1, 2, 2});
    print_state("fixture_commit_tokens", sampler.state(), {}, nullptr);
    try {
        sampler.commit(first);  // the state has moved on: a logic_error
        std::printf("{\"error\":\"stale decision accepted\"}\n");
        return 1;
    } catch (const std::logic_error& e) {
        std::printf("{\"op\":\"stale_commit\",\"error\":\"%s\"}\n", e.what());
    }
    return 0;
}

void part_executor(const char* name, const q38::SamplingConfigV1& cfg, int decode_steps,
                   bool with_reset) {
    q38::ExecutorOptions options;
    options.vocab_size = 100;
    options.context_limit = 256;
    options.append_chunk_tokens = 2;
    options.sampling = cfg;
    auto ex = q38::make_mock_executor(options);
    std::string op = std::string(name) + ":append";
    ex->append({1, 2, 3, 4, 5});
    auto stats = ex->stats();
    print_state(op.c_str(), ex->sampler_state(), {}, &stats);
    op = std::string(name) + ":seed_decode";
    const auto seeded = ex->seed_decode();
    stats = ex->stats();
    print_state(op.c_str(), ex->sampler_state(), {seeded}, &stats);
    for (int i = 0; i < decode_steps; ++i) {
        const auto r = ex->decode_one();
        stats = ex->stats();
        op = std::string(name) + ":decode_one";
        print_state(op.c_str(), ex->sampler_state(), r.published_tokens, &stats);
        if (i % 7 == 3) {
            // sampled mode: the executor falls back to target-only decode
            // (executor.cc:696-699), one sampled token per step
            const auto s = ex->speculative_step(4);
            stats = ex->stats();
            op = std::string(name) + ":speculative_step";
            print_state(op.c_str(), ex->sampler_state(), s.published_tokens, &stats);
        }
    }
    if (with_reset) {
        ex->reset_session();
        stats = ex->stats();
        op = std::string(name) + ":reset";
        print_state(op.c_str(), ex->sampler_state(), {}, &stats);
        ex->append({7, 8, 9});
        const auto s2 = ex->seed_decode();
        stats = ex->stats();
        op = std::string(name) + ":seed_after_reset";
        print_state(op.c_str(), ex->sampler_state(), {s2}, &stats);
        for (int i = 0; i < 5; ++i) {
            const auto r = ex->decode_one();
            stats = ex->stats();
            op = std::string(name) + ":decode_after_reset";
            print_state(op.c_str(), ex->sampler_state(), r.published_tokens, &stats);
        }
    }
}

}  // namespace

int main() {
    try {
        if (part_sampler()) return 1;
        // the fixture's configuration inside the executor (test_runtime.cc:1118-1136)
        part_executor("fixture", config(3, 0.9f, 0.8f, 1.1f, 0.2f, 0.1f, 170), 20, true);
        // top_k = 0 (a full sort in the reference) with a top-p cut
        part_executor("topk0", config(0, 0.95f, 1.3f, 1.0f, 0.0f, 0.0f, 2024), 40, false);
        // strong penalties: a sampled token drops below the runner-up
        part_executor("penalties", config(20, 1.0f, 0.6f, 1.2f, 0.3f, 0.5f, 77), 60, true);
    } catch (const std::exception& e) {
        std::printf("{\"error\":\"%s\"}\n", e.what());
        return 2;
    }
    return 0;
}
