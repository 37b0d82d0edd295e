// Kernel-side data structures shared by the kernels and the host ABI.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "q38s.h"
#include "q38s_device.cuh"

namespace q38s {

constexpr int kThreads = 256;        // threads per CTA of the small kernels
constexpr int kLeaderCap = 1024;     // candidates of a distribution / shard list
constexpr uint32_t kMaxGeneralVocab = 1u << 20;  // column radix of the general path
constexpr uint32_t kGTeamWords = 24608;          // a deferred row's team words (barrier, slots)
constexpr uint32_t kGAuxWords = 16384 + kGTeamWords;  // general-path words after a row's keys

// 32-bit words of general-path scratch per virtual row (16-byte aligned rows).
__host__ __device__ inline uint64_t scratch_stride(uint32_t vocab) {
    return ((static_cast<uint64_t>(vocab) + 3u) & ~3ull) + kGAuxWords;
}

// Per-row mutable sampler state: SamplerStateV1 (sampling.h:31-39) minus
// its constant header words.
struct RowState {
    uint64_t rng_state;
    uint64_t sampled_tokens;
    uint64_t canonical_tokens;
    uint64_t penalty_checksum;
};

enum Mode : int {
    kModePrepare = 0,       // decisions only
    kModeSampleCommit = 1,  // decisions + commit + commit_token
    kModeShardTopK = 2,     // emit the local top-k candidate list
    kModeDistribution = 3,  // decisions + per-row distribution (+ MTP)
};

// Arguments of the row-sampling kernel.  A "virtual row" is one unit of
// work: normally one batch row; for speculative verification one target or
// draft row of a single session.
struct SampleArgs {
    // virtual row v < split reads logits + v * row_stride elements,
    // v >= split reads logits2 + (v - split) * row_stride.
    const void* logits;
    const void* logits2;
    uint32_t split;
    uint64_t row_stride;
    int dtype;            // Q38S_DTYPE_*
    int use_tma;          // rows are 16-byte aligned
    uint32_t vocab;       // columns of this batch (shard width or full vocab)
    uint32_t full_vocab;  // vocabulary of the whole LM head
    uint32_t col_begin;   // global token id of column 0
    uint32_t vrows;
    int mode;
    // per state row
    const RowParams* params;
    RowState* state;
    uint32_t* bitmap;     // state row r: bitmap + r * bitmap_words
    uint32_t bitmap_words;
    uint32_t* counts;     // state row r: counts + r * vocab (or null)
    // virtual row -> state row: vrow_state_const if != ~0u, else identity
    uint32_t vrow_state_const;
    // the draw of virtual row v uses rng_state + (1 + rng_offset(v)) * gamma,
    // rng_offset(v) = rng_step ? (v < split ? v : v - split) : 0
    int rng_step;
    // rng_from_args: the rng_state of every state row is rng_state below,
    // not the state array's (the one-session sampler keeps its committed
    // state on the host, so a commit needs no device update)
    int rng_from_args;
    uint64_t rng_state;
    // additional penalty tokens: 0 none; 1 CSR (extra_offsets); 2 prefix of
    // extra_tokens of length (v < split ? v : v - split)
    int extra_mode;
    const int32_t* extra_tokens;
    const uint32_t* extra_offsets;
    // outputs
    q38s_decision_v1* decisions;
    int decisions_host;   // decisions is mapped host memory: status is written last
    q38s_distribution dist;
    q38s_candidate* topk_out;  // kModeShardTopK: vrows * k_out entries
    uint32_t k_out;
    // general-path scratch, scratch_stride 32-bit words per virtual row:
    // the exact key of every column (padded to a multiple of 4 words), then
    // kGAuxWords of histograms and, for a row shared by several CTAs, its
    // team words
    uint32_t* scratch;
    uint64_t scratch_stride;
    // deferred[v] != 0: virtual row v takes the general path (general
    // kernel); zero between launches (vrows words)
    uint32_t* deferred;
    // host_general: the caller launches the general kernel itself, only when
    // a row reports kRowDeferred (the one-session sampler, which waits for
    // its decision anyway); otherwise it runs behind every stream kernel
    int host_general;
    // speculative verification, run by the last row to finish
    q38s_mtp_result* mtp;
    uint32_t n_draft;
    const int32_t* draft_tokens;
    uint32_t* ticket;
    // streaming sampler (q38s_stream.cu): each virtual row is split into
    // `segs` column segments; with segs > 1 the kernel runs as clusters of
    // segs CTAs, one cluster per row, and the segments' lists are merged
    // in the cluster's shared memory
    uint32_t segs;
    // failure injection for the tests of the bounded waits (0 in normal
    // use): with test_withhold set, the producer of CTA 0 issues no copy and
    // that CTA's consumers give up on a tile after test_wait_cycles, so the
    // wait runs out on a barrier nothing completes, with no copy in flight
    uint32_t test_withhold;
    long long test_wait_cycles;
};

// Most segments per row: one cluster per split row (8 is the portable
// cluster size; above it the kernel allows non-portable sizes).
constexpr uint32_t kMaxSegs = 8;

// Decision status of a row handed to the general kernel when the caller
// launches that kernel itself (host_general); never returned to users.
constexpr int32_t kRowDeferred = 100;

// Launchers (q38s_stream.cu, q38s_sample.cu).  All return a cudaError_t as int.
int launch_stream(const SampleArgs& a, void* stream);   // streaming sampler
int launch_general_only(const SampleArgs& a, void* stream);  // the deferred rows of a launch
// Failure injection applied to every later stream-kernel launch of the
// process (tests only; withhold 0 turns it off).
void set_stream_fault(uint32_t withhold, long long wait_cycles);
uint32_t stream_segments(uint32_t vrows, uint32_t vocab, int device);
int launch_commit_tokens(RowState* state, uint32_t* bitmap, uint32_t bitmap_words,
                         uint32_t* counts, uint32_t vocab, uint32_t col_begin,
                         uint32_t rows, const int32_t* tokens, const uint32_t* offsets,
                         int32_t* status, void* stream);
int launch_commit(RowState* state, uint32_t rows, uint32_t vocab,
                  q38s_decision_v1* decisions, void* stream);
int launch_reset_states(RowState* state, const uint64_t* seeds, uint32_t rows,
                        void* stream);
int launch_shard_merge(const RowParams* params, const RowState* state, uint32_t rows,
                       const q38s_candidate* gathered, uint32_t n_shards,
                       uint32_t k_local, q38s_decision_v1* decisions, void* stream);
int launch_argmax_bf16(const uint16_t* logits, uint32_t count, int32_t* out,
                       void* stream);
int launch_topk_router(const uint16_t* logits, int32_t* expert_ids, float* expert_weights,
                       uint32_t tokens, uint32_t experts, uint32_t top_k, int normalize,
                       int by_logit, void* stream);

}  // namespace q38s
