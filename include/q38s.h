/*
 * q38s -- C ABI of the B200 token-sampling engine.
 *
 * This is the drop-in boundary for the reference runtime's sampler
 * (src/sampling.cc + include/q38/sampling.h of the reference).  Every entry
 * point takes plain pointers and sizes, returns a status code and never lets
 * a C++ exception cross the ABI.  Status codes map one to one onto the
 * exception classes the reference throws (sampling.cc:43-71, 105-117,
 * 148-166); q38s_last_error() returns the reference's message text for the
 * calling thread's last failure.
 *
 * Two families of calls:
 *   q38s_sampler_*  one session, host or device logits: the exact semantics
 *                   of q38::TransactionalSampler (sampling.h:52-75).  The C++
 *                   class in include/q38/sampling.h is a thin wrapper over it.
 *   q38s_batch_*    many sessions ("rows") resident on one GPU, device
 *                   logits, per-row parameters (SamplingConfigV2 adds min_p),
 *                   per-row status words, no host synchronisation.
 * plus speculative (MTP) verification, vocab-sharded sampling and greedy
 * argmax.
 *
 * Threading: like the reference (executor.cc:455, :538) a sampler or batch
 * is not thread-safe; one host thread drives it.  Calls on a batch are
 * ordered on the CUDA stream passed in (NULL = the legacy default stream).
 */
#ifndef Q38S_H
#define Q38S_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (return value of every entry point) ------------------ */
#define Q38S_OK 0
#define Q38S_INVALID_ARGUMENT 1 /* std::invalid_argument in the reference */
#define Q38S_LOGIC_ERROR 2      /* std::logic_error                       */
#define Q38S_RUNTIME_ERROR 3    /* std::runtime_error                     */
#define Q38S_CUDA_ERROR 4       /* CUDA runtime failure                   */
#define Q38S_OUT_OF_MEMORY 5
#define Q38S_TIMEOUT 6          /* a bounded device wait ran out          */

/* ---- per-row status words written by the kernels ----------------------- */
#define Q38S_ROW_OK 0
#define Q38S_ROW_NO_FINITE 1     /* "sampler has no finite candidate logits"  (sampling.cc:105-106) */
#define Q38S_ROW_NORMALIZATION 2 /* "sampler probability normalization failed" (sampling.cc:116-117) */
#define Q38S_ROW_STATE_MISMATCH 3 /* "sampler decision does not match committed state" (sampling.cc:149-153) */
#define Q38S_ROW_TIMEOUT 4       /* bounded wait for a TMA copy ran out */
#define Q38S_ROW_BAD_TOKEN 5     /* committed token outside the vocabulary (sampling.cc:164-165) */

/* ---- logits element types: q38::DType (contracts.h:19-26) -------------- */
#define Q38S_DTYPE_BF16 1
#define Q38S_DTYPE_F32 2

/* ---- modes: q38::SamplingModeV1 (sampling.h:14-17) ---------------------- */
#define Q38S_MODE_GREEDY 0
#define Q38S_MODE_TOP_K_TOP_P 1

/* SamplingConfigV1 (sampling.h:19-29), 40 bytes, identical layout. */
typedef struct q38s_sampling_config_v1 {
    uint16_t mode;
    uint16_t version; /* must be 1 */
    uint32_t top_k;   /* 0 = off */
    float top_p;
    float temperature;
    float repetition_penalty;
    float frequency_penalty;
    float presence_penalty;
    uint32_t reserved_; /* padding of the reference struct */
    uint64_t seed;
} q38s_sampling_config_v1;

/* SamplingConfigV2: V1 plus min_p in V1's padding word; version must be 2.
 * min_p in [0, 1]; 0 disables it and reduces exactly to V1. */
typedef struct q38s_sampling_config_v2 {
    uint16_t mode;
    uint16_t version; /* must be 2 */
    uint32_t top_k;
    float top_p;
    float temperature;
    float repetition_penalty;
    float frequency_penalty;
    float presence_penalty;
    float min_p;
    uint64_t seed;
} q38s_sampling_config_v2;

/* SamplerStateV1 (sampling.h:31-39), 40 bytes, identical layout. */
typedef struct q38s_sampler_state_v1 {
    uint32_t magic; /* fourcc('Q','3','8','S') */
    uint16_t version;
    uint16_t header_bytes;
    uint64_t rng_state;
    uint64_t sampled_tokens;
    uint64_t canonical_tokens;
    uint64_t penalty_checksum;
} q38s_sampler_state_v1;

/* SamplerDecisionV1 (sampling.h:41-45), 24 bytes, identical layout; the
 * reference's padding word carries the row status (Q38S_ROW_*). */
typedef struct q38s_decision_v1 {
    int32_t token;
    int32_t status;
    uint64_t rng_before;
    uint64_t rng_after;
} q38s_decision_v1;

/* One (value, token) pair of a top-k candidate list. */
typedef struct q38s_candidate {
    float value; /* logit after penalties and temperature */
    int32_t token;
} q38s_candidate;

/* Optional per-row distribution output of q38s_batch_prepare (device
 * arrays, `rows * capacity` entries each; any pointer may be NULL).
 * Row r receives its sorted candidates after top-k and min-p (tokens,
 * values), the probabilities w_i / total over the retained top-p prefix,
 * the candidate and retained counts and the totals of sampling.cc:110-134. */
typedef struct q38s_distribution {
    uint32_t capacity;
    int32_t* tokens;
    float* values;
    double* probs;
    uint32_t* n_candidates;
    uint32_t* n_retained;
    double* total;
    double* draw;
} q38s_distribution;

/* Additional penalty tokens of one prepare call (sampling.cc:67-73), per
 * row, on the device: row r uses tokens[offsets[r] .. offsets[r+1]).
 * Duplicates count once per occurrence, as in the reference. */
typedef struct q38s_penalty_extra {
    const int32_t* tokens;
    const uint32_t* offsets; /* rows + 1 entries */
} q38s_penalty_extra;

typedef struct q38s_sampler q38s_sampler;
typedef struct q38s_batch q38s_batch;

/* ------------------------------------------------------------------------
 * Library
 * ---------------------------------------------------------------------- */
/* Message of the calling thread's last failing call ("" if none). */
const char* q38s_last_error(void);
/* Build identification ("q38s <version> sm_100a"). */
const char* q38s_version(void);

/* ------------------------------------------------------------------------
 * Single session: q38::TransactionalSampler (sampling.h:52-75)
 * ---------------------------------------------------------------------- */
/* Replaces TransactionalSampler::TransactionalSampler (sampling.cc:40-57).
 * Validates exactly as the reference (Q38S_INVALID_ARGUMENT with its
 * messages), allocates the device penalty state on `device`. */
int q38s_sampler_create(int device, uint32_t vocabulary,
                        const q38s_sampling_config_v1* config,
                        q38s_sampler** out);
/* Same with a V2 config (min_p). */
int q38s_sampler_create_v2(int device, uint32_t vocabulary,
                           const q38s_sampling_config_v2* config,
                           q38s_sampler** out);
void q38s_sampler_destroy(q38s_sampler* sampler);

/* Replaces TransactionalSampler::prepare (sampling.cc:59-146) for HOST bf16
 * logits (StageOutput::logits_bf16, backend.h:143): copies them to the GPU,
 * samples, returns the decision.  const: no state changes. */
int q38s_sampler_prepare(const q38s_sampler* sampler,
                         const uint16_t* logits_bf16, size_t count,
                         const int32_t* additional_penalty_tokens,
                         size_t n_additional, q38s_decision_v1* out);
/* prepare() on logits already on the device (the producer's
 * workspace.logits, cuda_backend.cu:957), bf16 or fp32.  Only the decision
 * (24 bytes) crosses PCIe. */
int q38s_sampler_prepare_device(const q38s_sampler* sampler,
                                const void* logits, uint16_t dtype,
                                size_t count,
                                const int32_t* additional_penalty_tokens,
                                size_t n_additional, q38s_decision_v1* out,
                                void* stream);
/* Replaces TransactionalSampler::commit (sampling.cc:148-156). */
int q38s_sampler_commit(q38s_sampler* sampler, const q38s_decision_v1* d);
/* Replaces commit_tokens / commit_token (sampling.cc:158-172). */
int q38s_sampler_commit_tokens(q38s_sampler* sampler, const int32_t* tokens,
                               size_t count);
/* Replaces reset (sampling.cc:174-178). */
int q38s_sampler_reset(q38s_sampler* sampler);
/* state() / config() accessors (sampling.h:60-61). */
int q38s_sampler_state(const q38s_sampler* sampler,
                       q38s_sampler_state_v1* out);
int q38s_sampler_config(const q38s_sampler* sampler,
                        q38s_sampling_config_v1* out);

/* ------------------------------------------------------------------------
 * Batch: one TransactionalSampler per row, all rows on one GPU.
 * ---------------------------------------------------------------------- */
/* `rows` samplers over `vocabulary` tokens (sampling.cc:40-57 per row). */
int q38s_batch_create(int device, uint32_t vocabulary, uint32_t rows,
                      const q38s_sampling_config_v2* configs,
                      q38s_batch** out);
/* A batch that owns the contiguous vocabulary columns [col_begin,
 * col_begin + columns) of a `vocabulary`-wide LM head (vocab-parallel
 * sampling).  Penalty state covers only the owned columns. */
int q38s_batch_create_shard(int device, uint32_t vocabulary,
                            uint32_t col_begin, uint32_t columns,
                            uint32_t rows,
                            const q38s_sampling_config_v2* configs,
                            q38s_batch** out);
void q38s_batch_destroy(q38s_batch* batch);
uint32_t q38s_batch_rows(const q38s_batch* batch);

/* reset() of every row (sampling.cc:174-178). */
int q38s_batch_reset(q38s_batch* batch, void* stream);
/* Copies the rows' SamplerStateV1 to host memory (synchronises stream). */
int q38s_batch_states(const q38s_batch* batch, q38s_sampler_state_v1* out,
                      void* stream);
/* commit_tokens() per row (sampling.cc:158-172): row r appends device
 * tokens[offsets[r] .. offsets[r+1]).  Tokens outside the vocabulary (or the
 * shard's columns, for a shard batch) set that row's status to
 * Q38S_ROW_BAD_TOKEN in `status` (may be NULL) and are skipped. */
int q38s_batch_commit_tokens(q38s_batch* batch, const int32_t* tokens,
                             const uint32_t* offsets, int32_t* status,
                             void* stream);
/* prepare() for every row (sampling.cc:59-146) over device logits (row r at
 * logits + r * row_stride elements).  Writes decisions[r] (token, status,
 * rng pair); mutates nothing.  `extra` and `dist` may be NULL. */
int q38s_batch_prepare(const q38s_batch* batch, const void* logits,
                       uint16_t dtype, uint64_t row_stride,
                       const q38s_penalty_extra* extra,
                       q38s_decision_v1* decisions,
                       const q38s_distribution* dist, void* stream);
/* commit() for every row (sampling.cc:148-156).  A decision that does not
 * match the row's state sets decisions[r].status = Q38S_ROW_STATE_MISMATCH
 * and leaves the row unchanged. */
int q38s_batch_commit(q38s_batch* batch, q38s_decision_v1* decisions,
                      void* stream);
/* One decode step for every row: prepare, then commit the decision and the
 * sampled token (the sequence of DualStageExecutor::decode_one,
 * executor.cc:672-687, sampler calls at :455-459, :538, :684) in one launch. */
int q38s_batch_sample_commit(q38s_batch* batch, const void* logits,
                             uint16_t dtype, uint64_t row_stride,
                             q38s_decision_v1* decisions, void* stream);

/* ------------------------------------------------------------------------
 * Speculative (MTP) verification -- the entry DualStageExecutor::
 * speculative_step would call instead of its sampled-mode fallback
 * (executor.cc:696-699); draft width <= 64 (backend.h:17).
 * ---------------------------------------------------------------------- */
typedef struct q38s_mtp_result {
    int32_t tokens[65];   /* accepted drafts, then one sampled token */
    uint32_t n_tokens;    /* n_accepted + 1 */
    uint32_t n_accepted;
    int32_t status;       /* Q38S_ROW_* */
    uint64_t rng_before;
    uint64_t rng_after;   /* rng_before + n_tokens * 0x9e3779b97f4a7c15 */
} q38s_mtp_result;

/* Verifies n_draft draft tokens of batch row `row` against n_draft + 1
 * target rows (target + i * row_stride) and n_draft draft rows.  Target
 * and draft row i are transformed with the row's parameters and penalty
 * state plus draft_tokens[0..i) as additional penalty tokens.  Draft i is
 * accepted iff u_i * q_i(d_i) < p_i(d_i) with u_i = uniform01(s_i ^
 * 0xd6e8feb86659fd93), s_i = rng_state + (i + 1) * gamma; on the first
 * rejection the token is drawn from max(0, p_i - q_i) with uniform01(s_i);
 * if all are accepted the bonus token is the reference draw from
 * p_n_draft.  Writes *result on the device; mutates nothing (commit with
 * q38s_batch_commit_tokens and the returned rng_after). */
int q38s_mtp_verify(const q38s_batch* batch, uint32_t row,
                    const void* target, const void* draft, uint16_t dtype,
                    uint64_t row_stride, const int32_t* draft_tokens,
                    uint32_t n_draft, q38s_mtp_result* result,
                    void* stream);

/* ------------------------------------------------------------------------
 * Vocab-parallel sampling (no reference counterpart; the reference runs its
 * LM head whole on one GPU, cuda_backend.cu:1665-1669).
 * ---------------------------------------------------------------------- */
/* Local top-`k_local` candidates of every row over this shard's columns,
 * after the row's penalties and temperature, canonical order (value desc,
 * token asc), global token ids: out[r * k_local + j]. */
int q38s_shard_topk(const q38s_batch* shard, const void* logits,
                    uint16_t dtype, uint64_t row_stride, uint32_t k_local,
                    q38s_candidate* out, void* stream);
/* Merges n_shards gathered candidate lists (gathered[(s * rows + r) *
 * k_local + j], shards in column order) into each row's global top-k, then
 * min-p, top-p and the seeded draw with the row's parameters (rows must
 * have 0 < top_k <= k_local).  Writes decisions[r]; mutates nothing. */
int q38s_shard_merge_sample(const q38s_batch* shard,
                            const q38s_candidate* gathered,
                            uint32_t n_shards, uint32_t k_local,
                            q38s_decision_v1* decisions, void* stream);

/* ------------------------------------------------------------------------
 * Greedy: replaces cuda_argmax_bf16 (cuda/q38_kernels.cu:656-665,
 * kernel :320-356): index of the largest bf16 value, lowest index on ties,
 * NaN never selected.
 * ---------------------------------------------------------------------- */
int q38s_argmax_bf16(const uint16_t* logits, uint32_t count, int32_t* output,
                     void* stream, int device);

/* ------------------------------------------------------------------------
 * MoE router top-k: replaces cuda_topk_router_bf16 (cuda/q38_kernels.cu:
 * 667-687, kernels :358-480) with the same arguments, checks and results.
 * For each of `tokens` rows of `experts` bf16 logits (row-major, device):
 * the top_k experts (top_k <= 32) and their weights, expert_ids[t * top_k +
 * r] / expert_weights[t * top_k + r].  With 512 experts and normalisation
 * (the reference's decode path, unless Q38_CUDA_DECODE_TOPK is "scalar",
 * "0" or "false") experts are ordered by logit, lowest expert first on ties,
 * and weight_r = expf(logit_r - logit_0) / sum of those over the ranks;
 * otherwise by p = expf(logit - max) (lowest expert first on equal p) and
 * weight_r = p_r / (normalize_top_k ? sum of the top_k p : sum of every p),
 * the sums sequential in fp32 in the reference's order.  At most 3,072
 * experts per token (the reference takes any count). */
int q38s_topk_router_bf16(const uint16_t* logits, int32_t* expert_ids,
                          float* expert_weights, uint32_t tokens,
                          uint32_t experts, uint32_t top_k,
                          int normalize_top_k, void* stream, int device);

/* ------------------------------------------------------------------------
 * Failure injection, for tests of the bounded device waits only.  No
 * counterpart in the reference (its sampler runs on the host and has no
 * device waits).
 *
 * With withhold_copies != 0, every later sampling launch of this process
 * has its first CTA issue no logit copy, and that CTA's consumers give up
 * waiting for a tile after wait_cycles SM clock cycles: the wait runs out on
 * a barrier nothing completes, with no copy in flight.  The rows of that CTA
 * report Q38S_ROW_TIMEOUT (a one-session prepare returns Q38S_TIMEOUT); the
 * others are sampled normally.  withhold_copies = 0 restores normal
 * operation.  Not thread-safe; never set in production. */
int q38s_testing_set_fault(uint32_t withhold_copies, uint64_t wait_cycles);

/* ------------------------------------------------------------------------
 * Sampling without device allocation.  No counterpart in the reference.
 *
 * For callers that must not allocate GPU memory themselves or through this
 * library: code that runs inside a memory pool or arena it does not own, a
 * plug-in loaded into a host process that forbids cudaMalloc after start-up,
 * or a real-time loop in which an allocation (and the device-wide
 * synchronisation it can cause) is not allowed.  Every working buffer lives
 * in one fixed, statically sized device array inside this library
 * (4,982,016 bytes on every GPU that loads it, held until the process
 * exits); the caller passes only inputs and outputs.
 *
 * prepare() (sampling.cc:59-146 plus min_p) for `rows` rows of device logits
 * (row r at logits + r * row_stride elements, bf16 or f32) as freshly
 * constructed samplers: no committed penalty history and no additional
 * penalty tokens, so repetition / presence / frequency penalties have
 * nothing to act on.  configs: host array of `rows` V2 configs (validated
 * as q38s_batch_create does).  rng_states: host array of each row's
 * SamplerStateV1::rng_state before the draw, or NULL for each config's
 * seed.  decisions: device array of `rows` entries.  The result equals
 * q38s_batch_prepare on a new batch with the same configs and states.
 * Limits: 1 <= rows <= 4, vocabulary <= 262,144; larger sizes are rejected
 * with Q38S_INVALID_ARGUMENT.  Host arrays are read before the call
 * returns (the rows reach the device as kernel arguments).  The first call
 * on a device looks up the static array's device address
 * (cudaGetSymbolAddress, which may load this library's device code and
 * synchronise): make that first call before any stream capture.  Every
 * call shares the array and leaves its contents behind (each call rewrites
 * the rows' parameters and clears their penalty bitmaps first), so calls
 * whose work overlaps on the GPU (other streams, other host threads) race;
 * order them on one stream. */
int q38s_prepare_noalloc(const void* logits, uint16_t dtype, uint32_t vocabulary,
                         uint32_t rows, uint64_t row_stride,
                         const q38s_sampling_config_v2* configs,
                         const uint64_t* rng_states, q38s_decision_v1* decisions,
                         void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* Q38S_H */
