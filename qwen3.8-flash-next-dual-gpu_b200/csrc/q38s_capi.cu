// Host implementation of the q38s C ABI (include/q38s.h).
//
// Validation and error text follow src/sampling.cc of the reference
// (constructor :43-55, prepare :62-71, commit :149-153, commit_token
// :164-165, device failures :105-117).  No exception leaves this file.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "q38s.h"
#include "q38s_kernels.cuh"

using namespace q38s;

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}
int ok() {
    g_last_error.clear();
    return Q38S_OK;
}
int cuda_fail(cudaError_t e, const char* what) {
    return fail(e == cudaErrorMemoryAllocation ? Q38S_OUT_OF_MEMORY : Q38S_CUDA_ERROR,
                std::string(what) + ": " + cudaGetErrorString(e));
}
#define Q38S_CUDA(expr, what)                       \
    do {                                            \
        cudaError_t e_ = (expr);                    \
        if (e_ != cudaSuccess) return cuda_fail(e_, what); \
    } while (0)

constexpr const char* kMsgDims = "invalid sampler dimensions/version";
constexpr const char* kMsgMode = "unsupported sampling mode";
constexpr const char* kMsgParams = "invalid sampling parameters";
constexpr const char* kMsgGreedy = "greedy sampler does not consume RNG";
constexpr const char* kMsgSize = "sampler logits size differs from vocabulary";
constexpr const char* kMsgPenaltyToken = "penalty token is outside vocabulary";
constexpr const char* kMsgNoFinite = "sampler has no finite candidate logits";
constexpr const char* kMsgNorm = "sampler probability normalization failed";
constexpr const char* kMsgMismatch = "sampler decision does not match committed state";
constexpr const char* kMsgCommitted = "committed penalty token is invalid";
constexpr uint32_t kStateMagic = 0x53383351u;  // fourcc('Q','3','8','S')

// sampling.cc:43-55 (plus min_p in [0, 1] for V2).
int validate_config(uint32_t vocab, uint32_t version_expected,
                    const q38s_sampling_config_v2& c) {
    if (vocab == 0 || c.version != version_expected) return fail(Q38S_INVALID_ARGUMENT, kMsgDims);
    if (c.mode != Q38S_MODE_GREEDY && c.mode != Q38S_MODE_TOP_K_TOP_P)
        return fail(Q38S_INVALID_ARGUMENT, kMsgMode);
    if (!(c.temperature > 0.0f) || !std::isfinite(c.temperature) || !(c.top_p > 0.0f) ||
        c.top_p > 1.0f || !std::isfinite(c.top_p) || c.top_k > vocab ||
        c.repetition_penalty < 1.0f || !std::isfinite(c.repetition_penalty) ||
        !std::isfinite(c.frequency_penalty) || !std::isfinite(c.presence_penalty) ||
        !(c.min_p >= 0.0f) || c.min_p > 1.0f)
        return fail(Q38S_INVALID_ARGUMENT, kMsgParams);
    return Q38S_OK;
}

q38s_sampling_config_v2 from_v1(const q38s_sampling_config_v1& c) {
    q38s_sampling_config_v2 v;
    v.mode = c.mode;
    v.version = c.version;
    v.top_k = c.top_k;
    v.top_p = c.top_p;
    v.temperature = c.temperature;
    v.repetition_penalty = c.repetition_penalty;
    v.frequency_penalty = c.frequency_penalty;
    v.presence_penalty = c.presence_penalty;
    v.min_p = 0.0f;
    v.seed = c.seed;
    return v;
}

RowParams to_params(const q38s_sampling_config_v2& c) {
    RowParams p;
    p.top_k = c.top_k;
    p.top_p = c.top_p;
    p.min_p = c.min_p;
    p.temperature = c.temperature;
    p.repetition_penalty = c.repetition_penalty;
    p.frequency_penalty = c.frequency_penalty;
    p.presence_penalty = c.presence_penalty;
    p.flags = 0;
    if (c.repetition_penalty != 1.0f || c.presence_penalty != 0.0f ||
        c.frequency_penalty != 0.0f)
        p.flags |= kFlagPenalties;
    if (c.presence_penalty < 0.0f || c.frequency_penalty < 0.0f) p.flags |= kFlagNonMonotone;
    if (c.frequency_penalty != 0.0f) p.flags |= kFlagFrequency;
    return p;
}

class DeviceGuard {
public:
    explicit DeviceGuard(int device) {
        cudaGetDevice(&prev_);
        if (prev_ != device) cudaSetDevice(device);
        restore_ = prev_ != device;
    }
    ~DeviceGuard() {
        if (restore_) cudaSetDevice(prev_);
    }

private:
    int prev_ = 0;
    bool restore_ = false;
};

}  // namespace

// ------------------------------------------------------------------ batch
struct q38s_batch {
    int device = 0;
    uint32_t vocab = 0;       // columns owned
    uint32_t full_vocab = 0;  // LM head width
    uint32_t col_begin = 0;
    uint32_t rows = 0;
    std::vector<q38s_sampling_config_v2> configs;
    bool any_greedy = false;
    bool any_frequency = false;
    RowParams* d_params = nullptr;
    RowState* d_state = nullptr;
    uint64_t* d_seeds = nullptr;
    uint32_t* d_bitmap = nullptr;
    uint32_t bitmap_words = 0;
    uint32_t* d_counts = nullptr;
    uint32_t* d_scratch = nullptr;
    uint32_t scratch_rows = 0;
    uint32_t* d_gen = nullptr;  // per row: deferred to the general kernel
    // speculative verification workspace
    uint32_t* d_mtp_scratch = nullptr;
    uint32_t* d_mtp_gen = nullptr;
    int32_t* d_mtp_tokens = nullptr;
    double* d_mtp_probs = nullptr;
    uint32_t* d_mtp_nret = nullptr;
    uint32_t* d_mtp_ncand = nullptr;
    q38s_decision_v1* d_mtp_dec = nullptr;
    uint32_t* d_ticket = nullptr;
};

namespace {

constexpr uint32_t kMtpRows = 2 * 64 + 1;

void free_batch(q38s_batch* b) {
    if (!b) return;
    DeviceGuard g(b->device);
    cudaFree(b->d_params);
    cudaFree(b->d_state);
    cudaFree(b->d_seeds);
    cudaFree(b->d_bitmap);
    cudaFree(b->d_counts);
    cudaFree(b->d_scratch);
    cudaFree(b->d_gen);
    cudaFree(b->d_mtp_scratch);
    cudaFree(b->d_mtp_gen);
    cudaFree(b->d_mtp_tokens);
    cudaFree(b->d_mtp_probs);
    cudaFree(b->d_mtp_nret);
    cudaFree(b->d_mtp_ncand);
    cudaFree(b->d_mtp_dec);
    cudaFree(b->d_ticket);
    delete b;
}

int create_batch(int device, uint32_t full_vocab, uint32_t col_begin, uint32_t columns,
                 uint32_t rows, const q38s_sampling_config_v2* configs, uint32_t version,
                 q38s_batch** out) {
    if (!out) return fail(Q38S_INVALID_ARGUMENT, "null output handle");
    *out = nullptr;
    if (rows == 0 || !configs) return fail(Q38S_INVALID_ARGUMENT, kMsgDims);
    if (columns == 0 || static_cast<uint64_t>(col_begin) + columns > full_vocab)
        return fail(Q38S_INVALID_ARGUMENT, kMsgDims);
    // the general path's fixed-point masses (2^43 per token) sum without
    // overflow up to 2^20 columns
    if (columns > kMaxGeneralVocab)
        return fail(Q38S_INVALID_ARGUMENT, "more than 1,048,576 columns per batch");
    for (uint32_t r = 0; r < rows; ++r) {
        const int rc = validate_config(full_vocab, version, configs[r]);
        if (rc) return rc;
    }
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
        return fail(Q38S_CUDA_ERROR, "no such CUDA device");
    auto* b = new (std::nothrow) q38s_batch();
    if (!b) return fail(Q38S_OUT_OF_MEMORY, "host allocation failed");
    b->device = device;
    b->vocab = columns;
    b->full_vocab = full_vocab;
    b->col_begin = col_begin;
    b->rows = rows;
    b->configs.assign(configs, configs + rows);
    std::vector<RowParams> params(rows);
    std::vector<uint64_t> seeds(rows);
    for (uint32_t r = 0; r < rows; ++r) {
        params[r] = to_params(configs[r]);
        seeds[r] = configs[r].seed;
        b->any_greedy |= configs[r].mode == Q38S_MODE_GREEDY;
        b->any_frequency |= configs[r].frequency_penalty != 0.0f;
    }
    DeviceGuard g(device);
    b->bitmap_words = ((columns + 127) / 128) * 4;
    cudaError_t e = cudaSuccess;
    auto alloc = [&](void** p, size_t bytes) {
        if (e == cudaSuccess) e = cudaMalloc(p, bytes);
    };
    alloc(reinterpret_cast<void**>(&b->d_params), sizeof(RowParams) * rows);
    alloc(reinterpret_cast<void**>(&b->d_state), sizeof(RowState) * rows);
    alloc(reinterpret_cast<void**>(&b->d_seeds), sizeof(uint64_t) * rows);
    alloc(reinterpret_cast<void**>(&b->d_bitmap),
          sizeof(uint32_t) * static_cast<size_t>(b->bitmap_words) * rows);
    if (b->any_frequency)
        alloc(reinterpret_cast<void**>(&b->d_counts),
              sizeof(uint32_t) * static_cast<size_t>(columns) * rows);
    alloc(reinterpret_cast<void**>(&b->d_scratch),
          sizeof(uint32_t) * scratch_stride(columns) * rows);  // general-path keys, sums
    alloc(reinterpret_cast<void**>(&b->d_gen), sizeof(uint32_t) * static_cast<size_t>(rows));
    if (e == cudaSuccess) e = cudaMemset(b->d_gen, 0, sizeof(uint32_t) * rows);
    b->scratch_rows = rows;
    if (e == cudaSuccess)
        e = cudaMemcpy(b->d_params, params.data(), sizeof(RowParams) * rows,
                       cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy(b->d_seeds, seeds.data(), sizeof(uint64_t) * rows,
                       cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemset(b->d_bitmap, 0,
                       sizeof(uint32_t) * static_cast<size_t>(b->bitmap_words) * rows);
    if (e == cudaSuccess && b->d_counts)
        e = cudaMemset(b->d_counts, 0, sizeof(uint32_t) * static_cast<size_t>(columns) * rows);
    if (e == cudaSuccess) e = static_cast<cudaError_t>(launch_reset_states(b->d_state, b->d_seeds, rows, nullptr));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        free_batch(b);
        return cuda_fail(e, "batch allocation");
    }
    *out = b;
    return ok();
}

int check_logits_args(const q38s_batch* b, const void* logits, uint16_t dtype,
                      uint64_t row_stride) {
    if (!b) return fail(Q38S_INVALID_ARGUMENT, "null batch");
    if (!logits) return fail(Q38S_INVALID_ARGUMENT, "null logits");
    if (dtype != Q38S_DTYPE_BF16 && dtype != Q38S_DTYPE_F32)
        return fail(Q38S_INVALID_ARGUMENT, "logits dtype must be bf16 or f32");
    if (row_stride < b->vocab) return fail(Q38S_INVALID_ARGUMENT, kMsgSize);
    return Q38S_OK;
}

SampleArgs base_args(const q38s_batch* b, const void* logits, uint16_t dtype,
                     uint64_t row_stride) {
    SampleArgs a;
    std::memset(&a, 0, sizeof(a));
    const uint32_t es = dtype == Q38S_DTYPE_BF16 ? 2u : 4u;
    a.logits = logits;
    a.logits2 = logits;
    a.split = b->rows;
    a.row_stride = row_stride;
    a.dtype = dtype;
    a.use_tma = (reinterpret_cast<uintptr_t>(logits) % 16 == 0) && ((row_stride * es) % 16 == 0);
    a.vocab = b->vocab;
    a.full_vocab = b->full_vocab;
    a.col_begin = b->col_begin;
    a.vrows = b->rows;
    a.mode = kModePrepare;
    a.params = b->d_params;
    a.state = b->d_state;
    a.bitmap = b->d_bitmap;
    a.bitmap_words = b->bitmap_words;
    a.counts = b->d_counts;
    a.vrow_state_const = ~0u;
    a.scratch = b->d_scratch;
    a.scratch_stride = scratch_stride(b->vocab);
    a.deferred = b->d_gen;
    return a;
}

// Every row-sampling call goes through the streaming sampler; the number
// of column segments per row follows from the number of virtual rows.
int launch_checked(SampleArgs a, void* stream, const char* what, int device) {
    a.segs = stream_segments(a.vrows, a.vocab, device);
    const int e = launch_stream(a, stream);
    if (e != cudaSuccess) return cuda_fail(static_cast<cudaError_t>(e), what);
    return ok();
}

}  // namespace

extern "C" {

const char* q38s_last_error(void) { return g_last_error.c_str(); }
const char* q38s_version(void) { return "q38s 0.1 sm_100a"; }

int q38s_batch_create(int device, uint32_t vocabulary, uint32_t rows,
                      const q38s_sampling_config_v2* configs, q38s_batch** out) {
    return create_batch(device, vocabulary, 0, vocabulary, rows, configs, 2, out);
}

int q38s_batch_create_shard(int device, uint32_t vocabulary, uint32_t col_begin,
                            uint32_t columns, uint32_t rows,
                            const q38s_sampling_config_v2* configs, q38s_batch** out) {
    return create_batch(device, vocabulary, col_begin, columns, rows, configs, 2, out);
}

void q38s_batch_destroy(q38s_batch* batch) { free_batch(batch); }

uint32_t q38s_batch_rows(const q38s_batch* batch) { return batch ? batch->rows : 0; }

int q38s_batch_reset(q38s_batch* b, void* stream) {
    if (!b) return fail(Q38S_INVALID_ARGUMENT, "null batch");
    DeviceGuard g(b->device);
    auto s = static_cast<cudaStream_t>(stream);
    Q38S_CUDA(cudaMemsetAsync(b->d_bitmap, 0,
                              sizeof(uint32_t) * static_cast<size_t>(b->bitmap_words) * b->rows, s),
              "reset bitmap");
    if (b->d_counts)
        Q38S_CUDA(cudaMemsetAsync(b->d_counts, 0,
                                  sizeof(uint32_t) * static_cast<size_t>(b->vocab) * b->rows, s),
                  "reset counts");
    Q38S_CUDA(static_cast<cudaError_t>(launch_reset_states(b->d_state, b->d_seeds, b->rows, stream)),
              "reset states");
    return ok();
}

int q38s_batch_states(const q38s_batch* b, q38s_sampler_state_v1* out, void* stream) {
    if (!b || !out) return fail(Q38S_INVALID_ARGUMENT, "null argument");
    DeviceGuard g(b->device);
    std::vector<RowState> st(b->rows);
    Q38S_CUDA(cudaMemcpyAsync(st.data(), b->d_state, sizeof(RowState) * b->rows,
                              cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream)),
              "read states");
    Q38S_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "read states");
    for (uint32_t r = 0; r < b->rows; ++r) {
        out[r].magic = kStateMagic;
        out[r].version = 1;
        out[r].header_bytes = sizeof(q38s_sampler_state_v1);
        out[r].rng_state = st[r].rng_state;
        out[r].sampled_tokens = st[r].sampled_tokens;
        out[r].canonical_tokens = st[r].canonical_tokens;
        out[r].penalty_checksum = st[r].penalty_checksum;
    }
    return ok();
}

int q38s_batch_commit_tokens(q38s_batch* b, const int32_t* tokens, const uint32_t* offsets,
                             int32_t* status, void* stream) {
    if (!b || !offsets) return fail(Q38S_INVALID_ARGUMENT, "null argument");
    DeviceGuard g(b->device);
    const int e = launch_commit_tokens(b->d_state, b->d_bitmap, b->bitmap_words, b->d_counts,
                                       b->vocab, b->col_begin, b->rows, tokens, offsets,
                                       status, stream);
    if (e != cudaSuccess) return cuda_fail(static_cast<cudaError_t>(e), "commit_tokens");
    return ok();
}

int q38s_batch_prepare(const q38s_batch* b, const void* logits, uint16_t dtype,
                       uint64_t row_stride, const q38s_penalty_extra* extra,
                       q38s_decision_v1* decisions, const q38s_distribution* dist,
                       void* stream) {
    int rc = check_logits_args(b, logits, dtype, row_stride);
    if (rc) return rc;
    if (b->any_greedy) return fail(Q38S_LOGIC_ERROR, kMsgGreedy);
    if (!decisions) return fail(Q38S_INVALID_ARGUMENT, "null decisions");
    DeviceGuard g(b->device);
    SampleArgs a = base_args(b, logits, dtype, row_stride);
    a.decisions = decisions;
    if (extra && extra->offsets) {
        a.extra_mode = 1;
        a.extra_tokens = extra->tokens;
        a.extra_offsets = extra->offsets;
    }
    if (dist) {
        a.dist = *dist;
        a.mode = kModeDistribution;
    }
    return launch_checked(a, stream, "prepare", b->device);
}

int q38s_batch_sample_commit(q38s_batch* b, const void* logits, uint16_t dtype,
                             uint64_t row_stride, q38s_decision_v1* decisions, void* stream) {
    int rc = check_logits_args(b, logits, dtype, row_stride);
    if (rc) return rc;
    if (b->any_greedy) return fail(Q38S_LOGIC_ERROR, kMsgGreedy);
    DeviceGuard g(b->device);
    SampleArgs a = base_args(b, logits, dtype, row_stride);
    a.decisions = decisions;
    a.mode = kModeSampleCommit;
    return launch_checked(a, stream, "sample_commit", b->device);
}

int q38s_batch_commit(q38s_batch* b, q38s_decision_v1* decisions, void* stream) {
    if (!b || !decisions) return fail(Q38S_INVALID_ARGUMENT, "null argument");
    if (b->any_greedy) return fail(Q38S_LOGIC_ERROR, kMsgMismatch);
    DeviceGuard g(b->device);
    const int e = launch_commit(b->d_state, b->rows, b->full_vocab, decisions, stream);
    if (e != cudaSuccess) return cuda_fail(static_cast<cudaError_t>(e), "commit");
    return ok();
}

int q38s_mtp_verify(const q38s_batch* bc, uint32_t row, const void* target, const void* draft,
                    uint16_t dtype, uint64_t row_stride, const int32_t* draft_tokens,
                    uint32_t n_draft, q38s_mtp_result* result, void* stream) {
    auto* b = const_cast<q38s_batch*>(bc);
    int rc = check_logits_args(b, target, dtype, row_stride);
    if (rc) return rc;
    if (!draft || !result || (n_draft && !draft_tokens))
        return fail(Q38S_INVALID_ARGUMENT, "null argument");
    if (row >= b->rows) return fail(Q38S_INVALID_ARGUMENT, "row outside the batch");
    if (n_draft > 64) return fail(Q38S_INVALID_ARGUMENT, "MTP draft width exceeds 64");
    if (b->col_begin != 0 || b->vocab != b->full_vocab)
        return fail(Q38S_INVALID_ARGUMENT, "speculative verification needs a full-vocabulary batch");
    const auto& cfg = b->configs[row];
    if (cfg.mode == Q38S_MODE_GREEDY) return fail(Q38S_LOGIC_ERROR, kMsgGreedy);
    if (cfg.top_k == 0 || cfg.top_k > static_cast<uint32_t>(kLeaderCap))
        return fail(Q38S_INVALID_ARGUMENT,
                    "speculative verification needs 0 < top_k <= 1024");
    DeviceGuard g(b->device);
    if (!b->d_mtp_scratch) {
        cudaError_t e = cudaMalloc(&b->d_mtp_scratch,  // general-path keys, sums
                                   sizeof(uint32_t) * scratch_stride(b->vocab) * kMtpRows);
        if (e == cudaSuccess)
            e = cudaMalloc(&b->d_mtp_tokens, sizeof(int32_t) * kLeaderCap * kMtpRows);
        if (e == cudaSuccess)
            e = cudaMalloc(&b->d_mtp_probs, sizeof(double) * kLeaderCap * kMtpRows);
        if (e == cudaSuccess) e = cudaMalloc(&b->d_mtp_nret, sizeof(uint32_t) * kMtpRows);
        if (e == cudaSuccess) e = cudaMalloc(&b->d_mtp_ncand, sizeof(uint32_t) * kMtpRows);
        if (e == cudaSuccess) e = cudaMalloc(&b->d_mtp_dec, sizeof(q38s_decision_v1) * kMtpRows);
        if (e == cudaSuccess) e = cudaMalloc(&b->d_ticket, sizeof(uint32_t));
        if (e == cudaSuccess) e = cudaMalloc(&b->d_mtp_gen, sizeof(uint32_t) * kMtpRows);
        if (e == cudaSuccess) e = cudaMemset(b->d_mtp_gen, 0, sizeof(uint32_t) * kMtpRows);
        if (e == cudaSuccess) e = cudaMemset(b->d_ticket, 0, sizeof(uint32_t));
        if (e != cudaSuccess) return cuda_fail(e, "speculative workspace");
    }
    SampleArgs a = base_args(b, target, dtype, row_stride);
    a.logits2 = draft;
    a.split = n_draft + 1;
    a.vrows = 2 * n_draft + 1;
    a.vrow_state_const = row;
    a.rng_step = 1;
    a.extra_mode = n_draft ? 2 : 0;
    a.extra_tokens = draft_tokens;
    a.mode = kModeDistribution;
    a.decisions = b->d_mtp_dec;
    a.dist.capacity = kLeaderCap;
    a.dist.tokens = b->d_mtp_tokens;
    a.dist.probs = b->d_mtp_probs;
    a.dist.n_retained = b->d_mtp_nret;
    a.dist.n_candidates = b->d_mtp_ncand;
    a.scratch = b->d_mtp_scratch;
    a.scratch_stride = scratch_stride(b->vocab);
    a.deferred = b->d_mtp_gen;
    a.mtp = result;
    a.n_draft = n_draft;
    a.draft_tokens = draft_tokens;
    a.ticket = b->d_ticket;
    if (!(reinterpret_cast<uintptr_t>(draft) % 16 == 0)) a.use_tma = 0;
    return launch_checked(a, stream, "mtp_verify", b->device);
}

int q38s_shard_topk(const q38s_batch* b, const void* logits, uint16_t dtype,
                    uint64_t row_stride, uint32_t k_local, q38s_candidate* out, void* stream) {
    int rc = check_logits_args(b, logits, dtype, row_stride);
    if (rc) return rc;
    if (!out || k_local == 0 || k_local > static_cast<uint32_t>(kLeaderCap))
        return fail(Q38S_INVALID_ARGUMENT, "k_local must be in [1, 1024]");
    DeviceGuard g(b->device);
    SampleArgs a = base_args(b, logits, dtype, row_stride);
    a.mode = kModeShardTopK;
    a.topk_out = out;
    a.k_out = k_local;
    return launch_checked(a, stream, "shard_topk", b->device);
}

int q38s_shard_merge_sample(const q38s_batch* b, const q38s_candidate* gathered,
                            uint32_t n_shards, uint32_t k_local, q38s_decision_v1* decisions,
                            void* stream) {
    if (!b || !gathered || !decisions) return fail(Q38S_INVALID_ARGUMENT, "null argument");
    if (n_shards == 0 || k_local == 0 || static_cast<uint64_t>(n_shards) * k_local > 4096)
        return fail(Q38S_INVALID_ARGUMENT, "n_shards * k_local must be in [1, 4096]");
    if (n_shards > 64) return fail(Q38S_INVALID_ARGUMENT, "at most 64 column shards");
    if (b->any_greedy) return fail(Q38S_LOGIC_ERROR, kMsgGreedy);
    for (uint32_t r = 0; r < b->rows; ++r)
        if (b->configs[r].top_k == 0 || b->configs[r].top_k > k_local)
            return fail(Q38S_INVALID_ARGUMENT,
                        "vocab-sharded sampling needs 0 < top_k <= k_local on every row");
    DeviceGuard g(b->device);
    const int e = launch_shard_merge(b->d_params, b->d_state, b->rows, gathered, n_shards,
                                     k_local, decisions, stream);
    if (e != cudaSuccess) return cuda_fail(static_cast<cudaError_t>(e), "shard_merge_sample");
    return ok();
}

int q38s_topk_router_bf16(const uint16_t* logits, int32_t* expert_ids, float* expert_weights,
                          uint32_t tokens, uint32_t experts, uint32_t top_k,
                          int normalize_top_k, void* stream, int device) {
    // q38_kernels.cu:671-673: the reference's argument checks and message
    if (!logits || !expert_ids || !expert_weights || tokens == 0 || experts == 0 ||
        top_k == 0 || top_k > experts || top_k > 32)
        return fail(Q38S_INVALID_ARGUMENT, "invalid top-k router buffers");
    if (experts > 3072)
        return fail(Q38S_INVALID_ARGUMENT, "router experts above 3,072 per token");
    if (device < 0) return fail(Q38S_INVALID_ARGUMENT, "invalid CUDA kernel launch context");
    // the reference's dispatch (q38_kernels.cu:34-42, :674): its 512-expert
    // decode path orders by logit, unless Q38_CUDA_DECODE_TOPK disables it
    static const bool decode_path = [] {
        const char* v = std::getenv("Q38_CUDA_DECODE_TOPK");
        return !v || (std::strcmp(v, "scalar") != 0 && std::strcmp(v, "0") != 0 &&
                      std::strcmp(v, "false") != 0);
    }();
    const int by_logit = (experts == 512 && normalize_top_k && decode_path) ? 1 : 0;
    DeviceGuard g(device);
    const int e = launch_topk_router(logits, expert_ids, expert_weights, tokens, experts, top_k,
                                     normalize_top_k ? 1 : 0, by_logit, stream);
    if (e != cudaSuccess) return cuda_fail(static_cast<cudaError_t>(e), "topk_router_bf16");
    return ok();
}

int q38s_argmax_bf16(const uint16_t* logits, uint32_t count, int32_t* output, void* stream,
                     int device) {
    if (!logits || !output || count == 0)
        return fail(Q38S_INVALID_ARGUMENT, "invalid BF16 argmax buffers");
    DeviceGuard g(device);
    const int e = launch_argmax_bf16(logits, count, output, stream);
    if (e != cudaSuccess) return cuda_fail(static_cast<cudaError_t>(e), "argmax_bf16");
    return ok();
}

}  // extern "C"

// --------------------------------------------------------- single session
struct q38s_sampler {
    q38s_batch* batch = nullptr;
    q38s_sampling_config_v1 config{};  // as passed (V1 view)
    q38s_sampling_config_v2 config2{};
    q38s_sampler_state_v1 state{};     // host mirror (authoritative)
    cudaStream_t stream = nullptr;
    void* d_logits = nullptr;          // staging for host logits (bf16)
    // token staging (commit_tokens, additional penalty tokens): {0, n}
    // then the n tokens, uploaded with one copy from a pinned mirror
    uint32_t* d_stage = nullptr;
    uint32_t* h_stage = nullptr;             // pinned
    uint32_t token_cap = 0;
    uint32_t* d_offsets = nullptr;           // d_stage
    int32_t* d_tokens = nullptr;             // d_stage + 2
    uint32_t* h_offsets = nullptr;           // h_stage
    int32_t* h_tokens = nullptr;             // h_stage + 2
    cudaEvent_t staged = nullptr;            // the last upload out of h_stage
    bool staged_pending = false;             // ... may not have run yet
    q38s_decision_v1* d_decision = nullptr;  // device view of h_decision
    q38s_decision_v1* h_decision = nullptr;  // pinned, mapped: the kernel writes it directly
};

namespace {

void free_sampler(q38s_sampler* s) {
    if (!s) return;
    if (s->batch) {
        DeviceGuard g(s->batch->device);
        if (s->stream) cudaStreamSynchronize(s->stream);
        cudaFree(s->d_logits);
        cudaFree(s->d_stage);
        cudaFreeHost(s->h_decision);
        cudaFreeHost(s->h_stage);
        if (s->staged) cudaEventDestroy(s->staged);
        if (s->stream) cudaStreamDestroy(s->stream);
        free_batch(s->batch);
    }
    delete s;
}

int ensure_tokens(q38s_sampler* s, size_t n) {
    if (n <= s->token_cap) return Q38S_OK;
    uint32_t cap = std::max<uint32_t>(1024, s->token_cap);
    while (cap < n) cap *= 2;
    // queued work may still read the old buffers
    if (s->stream) Q38S_CUDA(cudaStreamSynchronize(s->stream), "token staging");
    s->staged_pending = false;
    cudaFree(s->d_stage);
    cudaFreeHost(s->h_stage);
    s->d_stage = s->h_stage = s->d_offsets = s->h_offsets = nullptr;
    s->d_tokens = s->h_tokens = nullptr;
    s->token_cap = 0;
    Q38S_CUDA(cudaMalloc(&s->d_stage, sizeof(uint32_t) * (2 + static_cast<size_t>(cap))),
              "token staging");
    Q38S_CUDA(cudaMallocHost(&s->h_stage, sizeof(uint32_t) * (2 + static_cast<size_t>(cap))),
              "token staging");
    s->d_offsets = s->d_stage;
    s->h_offsets = s->h_stage;
    s->d_tokens = reinterpret_cast<int32_t*>(s->d_stage + 2);
    s->h_tokens = reinterpret_cast<int32_t*>(s->h_stage + 2);
    s->token_cap = cap;
    return Q38S_OK;
}

int sampler_create(int device, uint32_t vocabulary, const q38s_sampling_config_v1& v1,
                   const q38s_sampling_config_v2& v2, uint32_t version, q38s_sampler** out) {
    if (!out) return fail(Q38S_INVALID_ARGUMENT, "null output handle");
    *out = nullptr;
    const int vrc = validate_config(vocabulary, version, v2);
    if (vrc) return vrc;
    auto* s = new (std::nothrow) q38s_sampler();
    if (!s) return fail(Q38S_OUT_OF_MEMORY, "host allocation failed");
    int rc = create_batch(device, vocabulary, 0, vocabulary, 1, &v2, version, &s->batch);
    if (rc) {
        delete s;
        return rc;
    }
    s->config = v1;
    s->config2 = v2;
    s->state.magic = kStateMagic;
    s->state.version = 1;
    s->state.header_bytes = sizeof(q38s_sampler_state_v1);
    s->state.rng_state = v2.seed;
    DeviceGuard g(device);
    cudaError_t e = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&s->d_logits, sizeof(uint16_t) * static_cast<size_t>(vocabulary));
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->staged, cudaEventDisableTiming);
    if (e == cudaSuccess)
        e = cudaHostAlloc(reinterpret_cast<void**>(&s->h_decision), sizeof(q38s_decision_v1),
                          cudaHostAllocMapped);
    if (e == cudaSuccess)
        e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&s->d_decision), s->h_decision, 0);
    if (e != cudaSuccess) {
        free_sampler(s);
        return cuda_fail(e, "sampler allocation");
    }
    rc = ensure_tokens(s, 1024);
    if (rc) {
        free_sampler(s);
        return rc;
    }
    *out = s;
    return ok();
}

// Uploads {0, n} and n tokens into d_stage on s->stream, one copy.  The
// pinned mirror is rewritten only after the previous upload out of it ran.
int stage_tokens(q38s_sampler* s, const int32_t* tokens, size_t n) {
    int rc = ensure_tokens(s, n);
    if (rc) return rc;
    if (s->staged_pending) {
        Q38S_CUDA(cudaEventSynchronize(s->staged), "token upload");
        s->staged_pending = false;
    }
    s->h_offsets[0] = 0;
    s->h_offsets[1] = static_cast<uint32_t>(n);
    if (n) std::memcpy(s->h_tokens, tokens, sizeof(int32_t) * n);
    Q38S_CUDA(cudaMemcpyAsync(s->d_stage, s->h_stage, sizeof(uint32_t) * (2 + n),
                              cudaMemcpyHostToDevice, s->stream),
              "token upload");
    Q38S_CUDA(cudaEventRecord(s->staged, s->stream), "token upload");
    s->staged_pending = true;
    return Q38S_OK;
}

// Status of a decision the kernel has not written yet (no Q38S_ROW_* value).
constexpr int32_t kStatusPending = INT32_MIN;

int prepare_common(const q38s_sampler* cs, const void* d_logits, uint16_t dtype, size_t count,
                   const int32_t* extra, size_t n_extra, q38s_decision_v1* out,
                   cudaStream_t stream, bool host_logits, const void* h_logits) {
    auto* s = const_cast<q38s_sampler*>(cs);
    if (!s || !out) return fail(Q38S_INVALID_ARGUMENT, "null argument");
    // sampling.cc:62-71, in the reference's order
    if (s->config2.mode == Q38S_MODE_GREEDY) return fail(Q38S_LOGIC_ERROR, kMsgGreedy);
    if (count != s->batch->vocab) return fail(Q38S_INVALID_ARGUMENT, kMsgSize);
    for (size_t i = 0; i < n_extra; ++i)
        if (extra[i] < 0 || static_cast<uint32_t>(extra[i]) >= s->batch->vocab)
            return fail(Q38S_INVALID_ARGUMENT, kMsgPenaltyToken);
    DeviceGuard g(s->batch->device);
    if (stream && stream != s->stream) {
        // order the sampler's own stream after the caller's work
        cudaEvent_t ev;
        Q38S_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "event");
        cudaEventRecord(ev, stream);
        cudaStreamWaitEvent(s->stream, ev, 0);
        cudaEventDestroy(ev);
    }
    if (host_logits)
        Q38S_CUDA(cudaMemcpyAsync(s->d_logits, h_logits, sizeof(uint16_t) * count,
                                  cudaMemcpyHostToDevice, s->stream),
                  "logits upload");
    int rc = n_extra ? stage_tokens(s, extra, n_extra) : Q38S_OK;  // nothing to upload without
    if (rc) return rc;
    SampleArgs a = base_args(s->batch, host_logits ? s->d_logits : d_logits, dtype, count);
    // The kernel writes the decision into mapped host memory, status last;
    // the host waits for the status to change (bounded), so a call costs no
    // read-back copy and no stream synchronisation on the common path.
    a.decisions = s->d_decision;
    a.decisions_host = 1;
    a.host_general = 1;   // the general kernel only for a deferred row (below)
    a.rng_from_args = 1;  // the committed state lives on the host
    a.rng_state = s->state.rng_state;
    if (n_extra) {
        a.extra_mode = 1;
        a.extra_tokens = s->d_tokens;
        a.extra_offsets = s->d_offsets;
    }
    volatile q38s_decision_v1* hd = s->h_decision;
    hd->status = kStatusPending;
    rc = launch_checked(a, s->stream, "prepare", s->batch->device);
    if (rc) return rc;
    auto wait_decision = [&]() -> int {
        const auto t_start = std::chrono::steady_clock::now();
        for (uint32_t spin = 1; hd->status == kStatusPending; ++spin) {
            if ((spin & 1023u) == 0 &&
                std::chrono::steady_clock::now() - t_start > std::chrono::milliseconds(200))
                break;  // long or failed: the stream reports it
        }
        if (hd->status == kStatusPending) Q38S_CUDA(cudaStreamSynchronize(s->stream), "prepare");
        return Q38S_OK;
    };
    rc = wait_decision();
    if (rc) return rc;
    if (hd->status == kRowDeferred) {
        // the row needs the general path: its kernel, then the decision
        hd->status = kStatusPending;
        const int e = launch_general_only(a, s->stream);
        if (e != cudaSuccess) return cuda_fail(static_cast<cudaError_t>(e), "prepare");
        rc = wait_decision();
        if (rc) return rc;
    }
    q38s_decision_v1 d;
    d.token = hd->token;
    d.status = hd->status;
    d.rng_before = hd->rng_before;
    d.rng_after = hd->rng_after;
    switch (d.status) {
        case Q38S_ROW_OK: break;
        case Q38S_ROW_NO_FINITE: return fail(Q38S_RUNTIME_ERROR, kMsgNoFinite);
        case Q38S_ROW_NORMALIZATION: return fail(Q38S_RUNTIME_ERROR, kMsgNorm);
        case Q38S_ROW_TIMEOUT: return fail(Q38S_TIMEOUT, "device copy wait timed out");
        default: return fail(Q38S_RUNTIME_ERROR, "device sampler failed");
    }
    *out = d;
    out->status = 0;
    return ok();
}

}  // namespace

extern "C" {

int q38s_sampler_create(int device, uint32_t vocabulary, const q38s_sampling_config_v1* config,
                        q38s_sampler** out) {
    if (!config) return fail(Q38S_INVALID_ARGUMENT, "null config");
    return sampler_create(device, vocabulary, *config, from_v1(*config), 1, out);
}

int q38s_sampler_create_v2(int device, uint32_t vocabulary,
                           const q38s_sampling_config_v2* config, q38s_sampler** out) {
    if (!config) return fail(Q38S_INVALID_ARGUMENT, "null config");
    q38s_sampling_config_v1 v1;
    std::memset(&v1, 0, sizeof(v1));
    v1.mode = config->mode;
    v1.version = 1;
    v1.top_k = config->top_k;
    v1.top_p = config->top_p;
    v1.temperature = config->temperature;
    v1.repetition_penalty = config->repetition_penalty;
    v1.frequency_penalty = config->frequency_penalty;
    v1.presence_penalty = config->presence_penalty;
    v1.seed = config->seed;
    return sampler_create(device, vocabulary, v1, *config, 2, out);
}

void q38s_sampler_destroy(q38s_sampler* sampler) { free_sampler(sampler); }

int q38s_sampler_prepare(const q38s_sampler* s, const uint16_t* logits, size_t count,
                         const int32_t* extra, size_t n_extra, q38s_decision_v1* out) {
    if (!s) return fail(Q38S_INVALID_ARGUMENT, "null sampler");
    if (s->config2.mode != Q38S_MODE_GREEDY && count == s->batch->vocab && !logits)
        return fail(Q38S_INVALID_ARGUMENT, "null logits");
    return prepare_common(s, nullptr, Q38S_DTYPE_BF16, count, extra, n_extra, out, nullptr,
                          true, logits);
}

int q38s_sampler_prepare_device(const q38s_sampler* s, const void* logits, uint16_t dtype,
                                size_t count, const int32_t* extra, size_t n_extra,
                                q38s_decision_v1* out, void* stream) {
    if (!s) return fail(Q38S_INVALID_ARGUMENT, "null sampler");
    if (dtype != Q38S_DTYPE_BF16 && dtype != Q38S_DTYPE_F32)
        return fail(Q38S_INVALID_ARGUMENT, "logits dtype must be bf16 or f32");
    if (s->config2.mode != Q38S_MODE_GREEDY && count == s->batch->vocab && !logits)
        return fail(Q38S_INVALID_ARGUMENT, "null logits");
    return prepare_common(s, logits, dtype, count, extra, n_extra, out,
                          static_cast<cudaStream_t>(stream), false, nullptr);
}

int q38s_sampler_commit(q38s_sampler* s, const q38s_decision_v1* d) {
    if (!s || !d) return fail(Q38S_INVALID_ARGUMENT, "null argument");
    // sampling.cc:149-153
    if (s->config2.mode == Q38S_MODE_GREEDY || d->token < 0 ||
        static_cast<uint32_t>(d->token) >= s->batch->vocab ||
        d->rng_before != s->state.rng_state || d->rng_after != d->rng_before + kGamma)
        return fail(Q38S_LOGIC_ERROR, kMsgMismatch);
    // host only: prepare passes the committed rng state to the kernel
    s->state.rng_state = d->rng_after;
    ++s->state.sampled_tokens;
    return ok();
}

int q38s_sampler_commit_tokens(q38s_sampler* s, const int32_t* tokens, size_t count) {
    if (!s || (count && !tokens)) return fail(Q38S_INVALID_ARGUMENT, "null argument");
    // sampling.cc:158-172: tokens before the first invalid one are committed
    size_t valid = 0;
    while (valid < count && tokens[valid] >= 0 &&
           static_cast<uint32_t>(tokens[valid]) < s->batch->vocab)
        ++valid;
    if (valid) {
        DeviceGuard g(s->batch->device);
        int rc = stage_tokens(s, tokens, valid);
        if (rc) return rc;
        const int e = launch_commit_tokens(s->batch->d_state, s->batch->d_bitmap,
                                           s->batch->bitmap_words, s->batch->d_counts,
                                           s->batch->vocab, 0, 1, s->d_tokens, s->d_offsets,
                                           nullptr, s->stream);
        if (e != cudaSuccess) return cuda_fail(static_cast<cudaError_t>(e), "commit_tokens");
        // no synchronisation: later calls are ordered after it on s->stream
        for (size_t i = 0; i < valid; ++i) {
            ++s->state.canonical_tokens;
            s->state.penalty_checksum ^=
                splitmix64(static_cast<uint64_t>(static_cast<uint32_t>(tokens[i])) ^
                           (s->state.canonical_tokens * kGamma));
        }
    }
    if (valid < count) return fail(Q38S_INVALID_ARGUMENT, kMsgCommitted);
    return ok();
}

int q38s_sampler_reset(q38s_sampler* s) {
    if (!s) return fail(Q38S_INVALID_ARGUMENT, "null sampler");
    const int rc = q38s_batch_reset(s->batch, s->stream);
    if (rc) return rc;
    DeviceGuard g(s->batch->device);
    Q38S_CUDA(cudaStreamSynchronize(s->stream), "reset");
    s->state = q38s_sampler_state_v1{};
    s->state.magic = kStateMagic;
    s->state.version = 1;
    s->state.header_bytes = sizeof(q38s_sampler_state_v1);
    s->state.rng_state = s->config2.seed;
    return ok();
}

int q38s_sampler_state(const q38s_sampler* s, q38s_sampler_state_v1* out) {
    if (!s || !out) return fail(Q38S_INVALID_ARGUMENT, "null argument");
    *out = s->state;
    return ok();
}

int q38s_sampler_config(const q38s_sampler* s, q38s_sampling_config_v1* out) {
    if (!s || !out) return fail(Q38S_INVALID_ARGUMENT, "null argument");
    *out = s->config;
    return ok();
}

int q38s_testing_set_fault(uint32_t withhold_copies, uint64_t wait_cycles) {
    if (withhold_copies && (wait_cycles == 0 || wait_cycles > 4000000000ull))
        return fail(Q38S_INVALID_ARGUMENT, "fault wait must be 1 to 4e9 cycles");
    set_stream_fault(withhold_copies ? 1u : 0u, static_cast<long long>(wait_cycles));
    return ok();
}

}  // extern "C"

// ------------------------------------------------------ no-allocation entry
// q38s_prepare_noalloc: every working buffer of the sampling kernel lives in
// one statically sized device array (one copy per GPU that loads the
// library), so the call allocates nothing.  Host code only ever passes the
// array's device address, resolved once per device with
// cudaGetSymbolAddress; the array's name in host code is not an address.
namespace {

constexpr uint32_t kNoAllocRows = 4;
constexpr uint32_t kNoAllocVocab = 262144;
constexpr uint32_t kNoAllocBitmapWords = ((kNoAllocVocab + 127) / 128) * 4;

struct NoAllocLayout {  // byte offsets into the static array
    static constexpr size_t params = 0;
    static constexpr size_t state = params + 256;
    static constexpr size_t gen = state + 256;     // deferred-row flags
    static constexpr size_t bitmap = gen + 256;    // cleared per call
    static constexpr size_t scratch =  // general-path keys and sums, per row
        bitmap + sizeof(uint32_t) * static_cast<size_t>(kNoAllocBitmapWords) * kNoAllocRows;
    static constexpr size_t end =
        scratch + sizeof(uint32_t) * ((static_cast<size_t>(kNoAllocVocab) + 3u) / 4u * 4u +
                                      kGAuxWords) * kNoAllocRows;
};
static_assert(sizeof(RowParams) * kNoAllocRows <= 256, "params slot");
static_assert(sizeof(RowState) * kNoAllocRows <= 256, "state slot");
static_assert(sizeof(uint32_t) * kNoAllocRows <= 256, "deferred-row slot");
static_assert(NoAllocLayout::end % 256 == 0, "layout");

static __device__ __align__(256) unsigned char g_noalloc_scratch[NoAllocLayout::end];

std::mutex g_noalloc_mu;
unsigned char* g_noalloc_ptr[64] = {};  // device address per device ordinal

// The rows of one call, handed to the device as kernel arguments: nothing is
// read from host memory after the launch returns.
struct NoAllocRows {
    RowParams params[kNoAllocRows];
    RowState states[kNoAllocRows];
};

// Writes the call's parameters and states into the array and clears the
// rows' penalty bitmaps (calls share the array; a fresh sampler has no
// history).  Ordered before the sampling kernel on the caller's stream.
__global__ void noalloc_stage_kernel(NoAllocRows in, uint32_t rows, uint32_t bitmap_words,
                                     unsigned char* base) {
    const uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
    if (tid < rows) {
        reinterpret_cast<RowParams*>(base + NoAllocLayout::params)[tid] = in.params[tid];
        reinterpret_cast<RowState*>(base + NoAllocLayout::state)[tid] = in.states[tid];
    }
    if (tid < kNoAllocRows)  // no row deferred to the general path
        reinterpret_cast<uint32_t*>(base + NoAllocLayout::gen)[tid] = 0u;
    uint32_t* bm = reinterpret_cast<uint32_t*>(base + NoAllocLayout::bitmap);
    const uint32_t n = rows * bitmap_words;
    for (uint32_t i = tid; i < n; i += gridDim.x * blockDim.x) bm[i] = 0u;
}

// Once per device, with that device current: the array's device address.
// (cudaGetSymbolAddress may load this library's device code on first use.)
int noalloc_setup(int device, unsigned char** out) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (device < 0 || device >= 64) return fail(Q38S_CUDA_ERROR, "device ordinal out of range");
    if (!g_noalloc_ptr[device]) {
        void* p = nullptr;
        Q38S_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch), "no-alloc scratch address");
        g_noalloc_ptr[device] = static_cast<unsigned char*>(p);
    }
    *out = g_noalloc_ptr[device];
    return Q38S_OK;
}

}  // namespace

extern "C" int q38s_prepare_noalloc(const void* logits, uint16_t dtype, uint32_t vocabulary,
                                    uint32_t rows, uint64_t row_stride,
                                    const q38s_sampling_config_v2* configs,
                                    const uint64_t* rng_states, q38s_decision_v1* decisions,
                                    void* stream) {
    if (!logits || !configs || !decisions) return fail(Q38S_INVALID_ARGUMENT, "null argument");
    if (rows == 0 || rows > kNoAllocRows)
        return fail(Q38S_INVALID_ARGUMENT,
                    "q38s_prepare_noalloc takes 1 to 4 rows (its working memory is static)");
    if (vocabulary == 0 || vocabulary > kNoAllocVocab)
        return fail(Q38S_INVALID_ARGUMENT,
                    "q38s_prepare_noalloc takes a vocabulary of at most 262,144 tokens");
    if (dtype != Q38S_DTYPE_BF16 && dtype != Q38S_DTYPE_F32)
        return fail(Q38S_INVALID_ARGUMENT, "logits dtype must be bf16 or f32");
    if (row_stride < vocabulary) return fail(Q38S_INVALID_ARGUMENT, kMsgSize);
    NoAllocRows in;
    std::memset(&in, 0, sizeof(in));
    for (uint32_t r = 0; r < rows; ++r) {
        const int rc = validate_config(vocabulary, 2, configs[r]);
        if (rc) return rc;
        if (configs[r].mode == Q38S_MODE_GREEDY) return fail(Q38S_LOGIC_ERROR, kMsgGreedy);
        in.params[r] = to_params(configs[r]);
        in.states[r] = RowState{rng_states ? rng_states[r] : configs[r].seed, 0, 0, 0};
    }
    int device = 0;
    Q38S_CUDA(cudaGetDevice(&device), "current device");
    unsigned char* base = nullptr;
    int rc = noalloc_setup(device, &base);
    if (rc) return rc;
    auto s = static_cast<cudaStream_t>(stream);
    const uint32_t bitmap_words = ((vocabulary + 127) / 128) * 4;
    noalloc_stage_kernel<<<8, 256, 0, s>>>(in, rows, bitmap_words, base);
    Q38S_CUDA(cudaGetLastError(), "no-alloc staging");
    const uint32_t es = dtype == Q38S_DTYPE_BF16 ? 2u : 4u;
    SampleArgs a;
    std::memset(&a, 0, sizeof(a));
    a.logits = logits;
    a.logits2 = logits;
    a.split = rows;
    a.row_stride = row_stride;
    a.dtype = dtype;
    a.use_tma = (reinterpret_cast<uintptr_t>(logits) % 16 == 0) && ((row_stride * es) % 16 == 0);
    a.vocab = vocabulary;
    a.full_vocab = vocabulary;
    a.col_begin = 0;
    a.vrows = rows;
    a.mode = kModePrepare;
    a.params = reinterpret_cast<const RowParams*>(base + NoAllocLayout::params);
    a.state = reinterpret_cast<RowState*>(base + NoAllocLayout::state);
    a.bitmap = reinterpret_cast<uint32_t*>(base + NoAllocLayout::bitmap);
    a.bitmap_words = bitmap_words;
    a.counts = nullptr;  // no history: every count is zero
    a.vrow_state_const = ~0u;
    a.decisions = decisions;
    a.scratch = reinterpret_cast<uint32_t*>(base + NoAllocLayout::scratch);
    a.scratch_stride = scratch_stride(vocabulary);
    a.deferred = reinterpret_cast<uint32_t*>(base + NoAllocLayout::gen);
    a.segs = stream_segments(rows, vocabulary, device);
    const int e = launch_stream(a, stream);
    if (e != cudaSuccess) return cuda_fail(static_cast<cudaError_t>(e), "prepare_noalloc");
    return ok();
}
