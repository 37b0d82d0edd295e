// q38::TransactionalSampler over the q38s C ABI.
//
// Each method forwards to the matching q38s_sampler_* entry point and turns
// its status code back into the exception class the reference throws
// (src/sampling.cc:44, :47, :55, :63, :65, :71, :106, :117, :153, :166),
// with the reference's message text.
#include "q38/sampling.h"

#include <cuda_runtime.h>

#include <cstring>
#include <stdexcept>
#include <string>
#include <utility>

#include "q38s.h"

namespace q38 {

static_assert(sizeof(q38s_sampling_config_v1) == sizeof(SamplingConfigV1),
              "C ABI config layout differs from SamplingConfigV1");
static_assert(sizeof(q38s_sampler_state_v1) == sizeof(SamplerStateV1),
              "C ABI state layout differs from SamplerStateV1");

namespace {

[[noreturn]] void raise(int code, const std::string& msg) {
    switch (code) {
        case Q38S_INVALID_ARGUMENT: throw std::invalid_argument(msg);
        case Q38S_LOGIC_ERROR: throw std::logic_error(msg);
        default: throw std::runtime_error(msg);
    }
}

inline void check(int code) {
    if (code != Q38S_OK) raise(code, q38s_last_error());
}

// The message of a failed call, taken before any later call (the state
// read-back after a commit) can replace it.
inline std::string error_text(int code) {
    return code != Q38S_OK ? std::string(q38s_last_error()) : std::string();
}
inline void check(int code, const std::string& msg) {
    if (code != Q38S_OK) raise(code, msg);
}

SamplerDecisionV1 to_decision(const q38s_decision_v1& d) {
    SamplerDecisionV1 r;
    r.token = d.token;
    r.rng_before = d.rng_before;
    r.rng_after = d.rng_after;
    return r;
}

}  // namespace

TransactionalSampler::TransactionalSampler(std::uint32_t vocabulary,
                                           SamplingConfigV1 config)
    : vocabulary_(vocabulary), config_(config) {
    q38s_sampling_config_v1 c;
    std::memcpy(static_cast<void*>(&c), static_cast<const void*>(&config), sizeof(c));
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) device = 0;
    check(q38s_sampler_create(device, vocabulary, &c, &engine_));
    sync_state();
}

TransactionalSampler::~TransactionalSampler() { q38s_sampler_destroy(engine_); }

TransactionalSampler::TransactionalSampler(TransactionalSampler&& o) noexcept
    : vocabulary_(o.vocabulary_), config_(o.config_), state_(o.state_),
      engine_(std::exchange(o.engine_, nullptr)) {}

TransactionalSampler& TransactionalSampler::operator=(TransactionalSampler&& o) noexcept {
    if (this != &o) {
        q38s_sampler_destroy(engine_);
        vocabulary_ = o.vocabulary_;
        config_ = o.config_;
        state_ = o.state_;
        engine_ = std::exchange(o.engine_, nullptr);
    }
    return *this;
}

void TransactionalSampler::sync_state() {
    q38s_sampler_state_v1 s;
    check(q38s_sampler_state(engine_, &s));
    state_.magic = s.magic;
    state_.version = s.version;
    state_.header_bytes = s.header_bytes;
    state_.rng_state = s.rng_state;
    state_.sampled_tokens = s.sampled_tokens;
    state_.canonical_tokens = s.canonical_tokens;
    state_.penalty_checksum = s.penalty_checksum;
}

SamplerDecisionV1 TransactionalSampler::prepare(
    const std::vector<std::uint16_t>& logits_bf16,
    const std::vector<std::int32_t>& additional_penalty_tokens) const {
    q38s_decision_v1 d;
    check(q38s_sampler_prepare(engine_, logits_bf16.data(), logits_bf16.size(),
                               additional_penalty_tokens.data(),
                               additional_penalty_tokens.size(), &d));
    return to_decision(d);
}

SamplerDecisionV1 TransactionalSampler::prepare_device(
    const void* logits, DType dtype, std::size_t count,
    const std::vector<std::int32_t>& additional_penalty_tokens, void* stream) const {
    q38s_decision_v1 d;
    check(q38s_sampler_prepare_device(engine_, logits, static_cast<std::uint16_t>(dtype),
                                      count, additional_penalty_tokens.data(),
                                      additional_penalty_tokens.size(), &d, stream));
    return to_decision(d);
}

void TransactionalSampler::commit(const SamplerDecisionV1& decision) {
    q38s_decision_v1 d;
    d.token = decision.token;
    d.status = 0;
    d.rng_before = decision.rng_before;
    d.rng_after = decision.rng_after;
    const int rc = q38s_sampler_commit(engine_, &d);
    const std::string msg = error_text(rc);
    sync_state();
    check(rc, msg);
}

void TransactionalSampler::commit_tokens(const std::vector<std::int32_t>& tokens) {
    const int rc = q38s_sampler_commit_tokens(engine_, tokens.data(), tokens.size());
    const std::string msg = error_text(rc);
    sync_state();
    check(rc, msg);
}

void TransactionalSampler::commit_token(std::int32_t token) {
    const int rc = q38s_sampler_commit_tokens(engine_, &token, 1);
    const std::string msg = error_text(rc);
    sync_state();
    check(rc, msg);
}

void TransactionalSampler::reset() {
    const int rc = q38s_sampler_reset(engine_);
    const std::string msg = error_text(rc);
    sync_state();
    check(rc, msg);
}

}  // namespace q38
