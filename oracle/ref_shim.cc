// C-ABI shim around the UNMODIFIED reference sampler (src/sampling.cc of the
// reference runtime), compiled together with it into oracle/_ref/libq38ref.so.
//
// TEST INFRASTRUCTURE ONLY.  This file is the checker side of the parity
// tests and the CPU-baseline arm of bench.py.  Nothing in the product links
// or loads it.
//
// The shim adds no arithmetic.  Every entry point forwards to
// q38::TransactionalSampler (include/q38/sampling.h:52-75) and turns its
// exceptions into status codes:
//   0 ok, 1 std::invalid_argument, 2 std::logic_error, 3 std::runtime_error,
//   9 any other exception.
#include "q38/sampling.h"

#include <cstdint>
#include <cstring>
#include <exception>
#include <stdexcept>
#include <thread>
#include <vector>

namespace {

int classify(const std::exception_ptr& ep, char* err, std::size_t errlen) {
    int code = 9;
    const char* what = "unknown exception";
    try {
        std::rethrow_exception(ep);
    } catch (const std::invalid_argument& e) {
        code = 1;
        what = e.what();
        if (err && errlen) std::strncpy(err, what, errlen - 1), err[errlen - 1] = 0;
        return code;
    } catch (const std::logic_error& e) {
        code = 2;
        what = e.what();
        if (err && errlen) std::strncpy(err, what, errlen - 1), err[errlen - 1] = 0;
        return code;
    } catch (const std::runtime_error& e) {
        code = 3;
        what = e.what();
        if (err && errlen) std::strncpy(err, what, errlen - 1), err[errlen - 1] = 0;
        return code;
    } catch (const std::exception& e) {
        what = e.what();
    } catch (...) {
    }
    if (err && errlen) std::strncpy(err, what, errlen - 1), err[errlen - 1] = 0;
    return code;
}

q38::SamplingConfigV1 load_config(const void* bytes40) {
    q38::SamplingConfigV1 c;
    std::memcpy(&c, bytes40, sizeof(c));
    return c;
}

}  // namespace

extern "C" {

// Constructs a sampler (sampling.cc:40-57).  Returns 0 and a handle, or an
// error code with the exception text copied into err.
int q38ref_create(std::uint32_t vocabulary, const void* config40, void** out,
                  char* err, std::size_t errlen) {
    *out = nullptr;
    try {
        *out = new q38::TransactionalSampler(vocabulary, load_config(config40));
        return 0;
    } catch (...) {
        return classify(std::current_exception(), err, errlen);
    }
}

void q38ref_destroy(void* h) { delete static_cast<q38::TransactionalSampler*>(h); }

// prepare() (sampling.cc:59-146): const, returns the decision.
int q38ref_prepare(const void* h, const std::uint16_t* logits, std::size_t n,
                   const std::int32_t* extra, std::size_t n_extra,
                   std::int32_t* token, std::uint64_t* rng_before,
                   std::uint64_t* rng_after, char* err, std::size_t errlen) {
    try {
        const auto* s = static_cast<const q38::TransactionalSampler*>(h);
        std::vector<std::uint16_t> l(logits, logits + n);
        std::vector<std::int32_t> e(extra, extra + n_extra);
        const auto d = s->prepare(l, e);
        *token = d.token;
        *rng_before = d.rng_before;
        *rng_after = d.rng_after;
        return 0;
    } catch (...) {
        return classify(std::current_exception(), err, errlen);
    }
}

int q38ref_commit(void* h, std::int32_t token, std::uint64_t rng_before,
                  std::uint64_t rng_after, char* err, std::size_t errlen) {
    try {
        q38::SamplerDecisionV1 d{token, rng_before, rng_after};
        static_cast<q38::TransactionalSampler*>(h)->commit(d);
        return 0;
    } catch (...) {
        return classify(std::current_exception(), err, errlen);
    }
}

int q38ref_commit_tokens(void* h, const std::int32_t* tokens, std::size_t n,
                         char* err, std::size_t errlen) {
    try {
        std::vector<std::int32_t> t(tokens, tokens + n);
        static_cast<q38::TransactionalSampler*>(h)->commit_tokens(t);
        return 0;
    } catch (...) {
        return classify(std::current_exception(), err, errlen);
    }
}

void q38ref_state(const void* h, void* state40) {
    const auto& s = static_cast<const q38::TransactionalSampler*>(h)->state();
    std::memcpy(state40, &s, sizeof(s));
}

void q38ref_config(const void* h, void* config40) {
    const auto& c = static_cast<const q38::TransactionalSampler*>(h)->config();
    std::memcpy(config40, &c, sizeof(c));
}

void q38ref_reset(void* h) { static_cast<q38::TransactionalSampler*>(h)->reset(); }

std::uint32_t q38ref_sizeof_config() { return sizeof(q38::SamplingConfigV1); }
std::uint32_t q38ref_sizeof_state() { return sizeof(q38::SamplerStateV1); }

// Batched CPU baseline: calls prepare() on `rows` independent samplers
// (handles[r] for row r) over row-major bf16 logits, spreading rows over
// `threads` std::threads.  Status per row goes to status[r].  This is how a
// host that owns one TransactionalSampler per session would serve a batch.
void q38ref_prepare_rows(void* const* handles, std::uint32_t rows,
                         const std::uint16_t* logits, std::size_t vocab,
                         std::int32_t* tokens, std::int32_t* status,
                         int threads) {
    if (threads < 1) threads = 1;
    auto work = [&](std::uint32_t begin, std::uint32_t end) {
        std::vector<std::uint16_t> l(vocab);
        const std::vector<std::int32_t> none;
        for (std::uint32_t r = begin; r < end; ++r) {
            std::memcpy(l.data(), logits + static_cast<std::size_t>(r) * vocab,
                        vocab * sizeof(std::uint16_t));
            try {
                const auto* s =
                    static_cast<const q38::TransactionalSampler*>(handles[r]);
                tokens[r] = s->prepare(l, none).token;
                status[r] = 0;
            } catch (...) {
                tokens[r] = -1;
                status[r] = classify(std::current_exception(), nullptr, 0);
            }
        }
    };
    std::vector<std::thread> pool;
    const std::uint32_t per = (rows + threads - 1) / threads;
    for (int t = 0; t < threads; ++t) {
        const std::uint32_t b = t * per;
        const std::uint32_t e = b + per < rows ? b + per : rows;
        if (b >= e) break;
        pool.emplace_back(work, b, e);
    }
    for (auto& th : pool) th.join();
}

}  // extern "C"
