/*
 * sixi_smp.h - C ABI of the B200 logits-to-token path (sampler chain, grammar-mask application,
 * speculative verifier) of the Sixi-ASI engine.
 *
 * Every entry point is `extern "C"`, takes plain pointers and sizes, and returns an int32 status
 * whose values are the engine's `sixi_asi::ErrorCode` integers (include/sixi_asi/common.hpp:40-66
 * in the engine). Device-side failures of a single row (NaN/Inf logits, all-masked row, bad
 * draft id) are reported per row in `out_status` and never trap the GPU.
 *
 * Unless stated otherwise all array arguments are DEVICE pointers, every call is asynchronous on
 * the caller's CUDA stream (`stream` is a `cudaStream_t` passed as `void*`, NULL = legacy default
 * stream) and performs no host synchronisation. The handle owns device workspace only; it is not
 * thread-safe (one handle per host thread or external serialisation), matching the engine, where
 * device access is serialised by the batch leader (src/core/core_execution.cpp:1398-1530).
 */
#ifndef SIXI_SMP_H
#define SIXI_SMP_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SIXI_SMP_ABI_VERSION 1

#if defined(__GNUC__)
#define SIXI_SMP_API __attribute__((visibility("default")))
#else
#define SIXI_SMP_API
#endif

/* Status codes: the engine's ErrorCode values (include/sixi_asi/common.hpp:40-66). */
enum {
    SIXI_OK = 0,
    SIXI_INVALID_ARGUMENT = 1,
    SIXI_OUT_OF_BOUNDS = 2,
    SIXI_OUT_OF_MEMORY_VRAM = 11,
    SIXI_NUMERIC_NAN_OR_INF = 16,
    SIXI_BACKEND_ERROR = 23,
    SIXI_UNSUPPORTED_HARDWARE = 24
};

/* Logits element type. */
enum { SIXI_SMP_F32 = 0, SIXI_SMP_BF16 = 1 };

/* ExecutionMode (include/sixi_asi/common.hpp:133-136): penalties apply only in Adaptive. */
enum { SIXI_SMP_STRICT_REPLAY = 0, SIXI_SMP_ADAPTIVE = 1 };

/* sixi_smp_params.flags */
enum {
    SIXI_SMP_ROW_MASKED = 1u /* apply this row's grammar bitmask (mask_words row) */
};

/*
 * Per-row (sampler) or per-stream (verifier) sampling parameters. Mirrors
 * sixi_asi::core::SamplingParams (include/sixi_asi/core_execution.hpp:136-144); `min_p` and
 * `frequency_penalty` are extensions that are identity at 0 (they do not exist in the engine).
 * Uniform draws, when not supplied by the caller, come from Philox4x32-10 with
 * key = seed and counter = {slot, 0, lo32(counter + step), hi32(counter + step)}.
 */
typedef struct sixi_smp_params {
    float temperature;        /* <= 0: greedy argmax, lowest id wins ties, consumes no uniform */
    int32_t top_k;            /* <= 0 or >= allowed vocab: no top-k truncation */
    float top_p;              /* truncation applied when 0 < top_p < 1 (crossing token kept) */
    float min_p;              /* extension: keep prob >= min_p * max prob; 0 = off */
    float repetition_penalty; /* 1 = off; v<0 ? v*rep : v/rep once per unique history id */
    float presence_penalty;   /* 0 = off; subtracted once per unique history id */
    float frequency_penalty;  /* extension: subtracted once per history occurrence; 0 = off */
    uint32_t mode;            /* SIXI_SMP_STRICT_REPLAY or SIXI_SMP_ADAPTIVE */
    uint32_t flags;           /* SIXI_SMP_ROW_MASKED */
    uint32_t reserved;
    uint64_t seed;            /* Philox key */
    uint64_t counter;         /* Philox counter base (e.g. the request's decode step) */
} sixi_smp_params;

/* A batch of logits rows in device memory: row r starts at data + r * row_stride elements. */
typedef struct sixi_smp_rows {
    const void* data;
    uint32_t dtype;       /* SIXI_SMP_F32 or SIXI_SMP_BF16 */
    uint32_t n_rows;
    uint64_t row_stride;  /* in elements, >= vocab */
} sixi_smp_rows;

typedef struct sixi_smp sixi_smp; /* opaque handle */

/* Creates a handle bound to `device` for rows of `vocab` entries. Replaces the construction of the
 * engine's sampler state; the engine's DeterministicSampler is stateless
 * (include/sixi_asi/core_execution.hpp:146-183), so the handle holds only device workspace for
 * up to `max_rows` rows per call and the launch configuration. */
SIXI_SMP_API int32_t sixi_smp_create(int32_t device, uint32_t max_rows, uint32_t vocab, sixi_smp** out);
SIXI_SMP_API int32_t sixi_smp_destroy(sixi_smp* h);
SIXI_SMP_API uint32_t sixi_smp_vocab(const sixi_smp* h);
SIXI_SMP_API uint32_t sixi_smp_mask_words(const sixi_smp* h); /* ceil(vocab / 32) */
SIXI_SMP_API const char* sixi_smp_status_string(int32_t status);

/*
 * Fused sampler over a batch of rows: grammar mask -> NaN/Inf check -> penalties -> greedy argmax
 * or top-k -> temperature softmax -> top-p -> min-p -> draw. One token per row.
 * Replaces DeterministicSampler::sample_token / compute_sampling_candidates /
 * sample_from_candidates (src/core/core_execution.cpp:449-619).
 *   params      [n_rows]
 *   mask_words  [n_rows][sixi_smp_mask_words(h)] or NULL; bit (i % 32) of word (i / 32) set =
 *               token i allowed; used by rows whose params.flags has SIXI_SMP_ROW_MASKED
 *   hist_tokens/hist_offsets: CSR token history, row r = hist_tokens[hist_offsets[r] ..
 *               hist_offsets[r+1]); hist_tokens may be NULL (no history)
 *   uniforms    [n_rows] in [0,1) or NULL (Philox slot 0); greedy rows consume none
 *   out_tokens  [n_rows] (-1 on error), out_status [n_rows]
 */
SIXI_SMP_API int32_t sixi_smp_sample(sixi_smp* h, const sixi_smp_rows* rows, const sixi_smp_params* params,
                        const uint32_t* mask_words, const int32_t* hist_tokens,
                        const int64_t* hist_offsets, const double* uniforms, uint64_t step,
                        int32_t* out_tokens, int32_t* out_status, void* stream);

/*
 * sixi_smp_sample over rows picked out of a batch (no counterpart in the engine): row j of `rows`
 * is sampled with the parameters, mask, history and uniform of batch row row_map[j], and its token
 * and status go to out_tokens[row_map[j]] and out_status[row_map[j]]; the other slots are left as
 * they are. row_map: device memory, rows->n_rows distinct batch-row indices; params, mask_words,
 * hist_*, uniforms and the outputs are the whole batch's arrays. The vocab-sharded mode's second
 * round samples its rebuilt rows this way, without building subset arrays.
 */
SIXI_SMP_API int32_t sixi_smp_sample_indexed(sixi_smp* h, const sixi_smp_rows* rows, const uint32_t* row_map,
                                            const sixi_smp_params* params, const uint32_t* mask_words,
                                            const int32_t* hist_tokens, const int64_t* hist_offsets,
                                            const double* uniforms, uint64_t step, int32_t* out_tokens,
                                            int32_t* out_status, void* stream);

/*
 * Row gather on the device (no counterpart in the engine): dst row j = the first `width` elements
 * of src row row_index[j], rows of src's dtype, dst rows dst_stride elements apart; n <= 65,535.
 * Packs the rows of a batch that a second exchange round needs.
 */
SIXI_SMP_API int32_t sixi_smp_gather_rows(sixi_smp* h, const sixi_smp_rows* src, const int32_t* row_index,
                                         uint32_t n, uint32_t width, void* dst, uint64_t dst_stride, void* stream);

/*
 * Same as sixi_smp_sample with HOST inputs and outputs: copies the logits (pinned host memory
 * recommended), params, masks, histories and uniforms to handle-owned device staging, samples, and
 * copies tokens and statuses back, then synchronises `stream`. This is the engine-facing call
 * shape of DeterministicSampler::sample_token (src/core/core_execution.cpp:603-619), which takes
 * host logits. The staging buffers grow on demand: the first call with a larger batch allocates.
 */
SIXI_SMP_API int32_t sixi_smp_sample_host(sixi_smp* h, const void* host_logits, uint32_t dtype,
                             uint32_t n_rows, uint64_t row_stride,
                             const sixi_smp_params* host_params, const uint32_t* host_mask_words,
                             const int32_t* host_hist_tokens, const int64_t* host_hist_offsets,
                             const double* host_uniforms, uint64_t step, int32_t* host_out_tokens,
                             int32_t* host_out_status, void* stream);

/*
 * sixi_smp_sample_host without the final synchronisation, for pipelines over independent batches
 * (no counterpart in the engine, whose sampler call returns the token). Two device staging slots
 * alternate between calls: a call copies its inputs into its slot on the handle's own copy stream,
 * after the kernel of the call that last used that slot has finished, and its kernel on `stream`
 * waits for that copy; so call i + 1's host->device copy overlaps call i's kernel. Tokens and
 * statuses are copied back on `stream`. The caller keeps the host inputs unchanged and alive, and
 * reads the outputs only after synchronising `stream` (or an event recorded on it after the call).
 * Host buffers must be pinned for the copies to be asynchronous. Calls on one handle must come from
 * one thread at a time. A call that needs larger staging than its slot has waits for that slot and
 * reallocates it.
 */
SIXI_SMP_API int32_t sixi_smp_sample_host_async(sixi_smp* h, const void* host_logits, uint32_t dtype,
                                               uint32_t n_rows, uint64_t row_stride,
                                               const sixi_smp_params* host_params,
                                               const uint32_t* host_mask_words, const int32_t* host_hist_tokens,
                                               const int64_t* host_hist_offsets, const double* host_uniforms,
                                               uint64_t step, int32_t* host_out_tokens, int32_t* host_out_status,
                                               void* stream);

/*
 * Greedy argmax per row on the raw (optionally masked) logits, lowest id on ties; a NaN at index 0
 * yields 0 and other NaNs never win, exactly as DeterministicSampler::sample_greedy_argmax
 * (src/core/core_execution.cpp:394-407). Replaces the llama.cpp greedy sampler hook
 * (set_gpu_greedy_sampling_enabled / forward_sequence_greedy_argmax,
 * src/core/core_execution.cpp:3067-3104, 3847-3923). `mask_words`, when not NULL, masks every row.
 */
SIXI_SMP_API int32_t sixi_smp_greedy_argmax(sixi_smp* h, const sixi_smp_rows* rows, const uint32_t* mask_words,
                               int32_t* out_tokens, int32_t* out_status, void* stream);

/*
 * Diagnostic / parity: the sorted candidate list (logit desc, id asc) that a row's draw uses, i.e.
 * compute_sampling_candidates (src/core/core_execution.cpp:449-584). Writes the first
 * min(max_out, n) candidates of each row into out_ids/out_probs [n_rows][max_out] and the full
 * candidate count n into out_count. max_out <= 256.
 */
SIXI_SMP_API int32_t sixi_smp_candidates(sixi_smp* h, const sixi_smp_rows* rows, const sixi_smp_params* params,
                            const uint32_t* mask_words, const int32_t* hist_tokens,
                            const int64_t* hist_offsets, uint32_t max_out, int32_t* out_ids,
                            double* out_probs, int32_t* out_count, int32_t* out_status,
                            void* stream);

/*
 * Speculative verification of n_streams streams with k drafted tokens each.
 *   target      n_streams * (k + 1) rows; row s*(k+1)+i is the target distribution that verifies
 *               draft i (i < k); row s*(k+1)+k draws the bonus token on full acceptance.
 *   draft_probs [n_streams][k][row_stride] fp32 dense draft distributions q, or NULL for one-hot
 *               drafts. Dense q follows SpeculativeDecoder::step's verification with draft
 *               probabilities (src/speculative/speculative.cpp:801-916): accept with
 *               min(1, p/q), residual max(0, p - q) drawn in vocab-id order. NULL follows the
 *               fast path (src/speculative/speculative.cpp:589-692): accept with p, residual =
 *               candidates without the draft, drawn in candidate order.
 *   drafts      [n_streams][k]; n_drafts [n_streams] or NULL (= k for every stream)
 *   params      [n_streams]; temperature <= 0 selects greedy match (argmax of raw logits)
 *   mask_words  [n_streams * (k + 1)][mask words] or NULL; used by streams with
 *               SIXI_SMP_ROW_MASKED
 *   hist_*      CSR per-stream base history (the context; for one-hot drafts include the anchor).
 *               Row i is penalised with base + drafts[0..i-1]; the bonus row with base only for
 *               dense q (speculative.cpp:908-915) and base + all drafts for one-hot.
 *   uniforms    [n_streams][k + 1] or NULL (Philox slots 0..k). The uniforms are consumed in
 *               order exactly like the engine's DeterministicRng: one per examined draft, then one
 *               for the residual or bonus draw; out_uniforms_used reports how many.
 *   outputs     out_accepted [S], out_tokens [S][k+1] (committed tokens, -1 padded),
 *               out_n_tokens [S], out_first_reject [S] (-1 on full accept),
 *               out_uniforms_used [S], out_status [S]
 */
SIXI_SMP_API int32_t sixi_smp_verify(sixi_smp* h, const sixi_smp_rows* target, const float* draft_probs,
                        const int32_t* drafts, const int32_t* n_drafts, uint32_t n_streams,
                        uint32_t k, const sixi_smp_params* params, const uint32_t* mask_words,
                        const int32_t* hist_tokens, const int64_t* hist_offsets,
                        const double* uniforms, uint64_t step, int32_t* out_accepted,
                        int32_t* out_tokens, int32_t* out_n_tokens, int32_t* out_first_reject,
                        int32_t* out_uniforms_used, int32_t* out_status, void* stream);

/*
 * Full-vocabulary softmax of each row: DeterministicSampler::compute_full_distribution
 * (src/core/core_execution.cpp:409-447), the producer of dense draft distributions
 * (src/speculative/speculative.cpp:279-280). temperatures [n_rows] (device); out_probs
 * [n_rows][out_stride] fp32 (out_stride >= vocab). temperature <= 0 writes a one-hot row at the raw
 * argmax (sample_greedy_argmax); otherwise float(exp(x / T - max) / sum) with fp64 terms, and all
 * zeros when the row holds a NaN or +inf, as the engine leaves it.
 */
SIXI_SMP_API int32_t sixi_smp_full_distribution(sixi_smp* h, const sixi_smp_rows* rows, const float* temperatures,
                                   float* out_probs, uint64_t out_stride, void* stream);

/*
 * sixi_smp_verify with dense q given as the draft model's logits: q of draft row r is
 * compute_full_distribution(draft_logits row r, draft_temperatures[r]) (src/speculative/
 * speculative.cpp:279-280 builds it so; src/core/core_execution.cpp:409-447), and verification
 * follows speculative.cpp:801-916 as in sixi_smp_verify with that q. q is never stored: a
 * statistics pass keeps each draft row's maximum and fp64 sum, and the verifier evaluates q with
 * the same operations where it reads it (the drafted id; the residual on rejection). Results equal
 * sixi_smp_full_distribution followed by sixi_smp_verify on the same rows. draft_logits: S*k rows
 * (fp32 or bf16, row_stride >= vocab); draft_temperatures: [S*k] (device). Other arguments and
 * outputs as sixi_smp_verify. S*k must not exceed the handle's max_rows.
 */
SIXI_SMP_API int32_t sixi_smp_verify_draft_logits(sixi_smp* h, const sixi_smp_rows* target,
                                                  const sixi_smp_rows* draft_logits,
                                                  const float* draft_temperatures, const int32_t* drafts,
                                                  const int32_t* n_drafts, uint32_t n_streams, uint32_t k,
                                                  const sixi_smp_params* params, const uint32_t* mask_words,
                                                  const int32_t* hist_tokens, const int64_t* hist_offsets,
                                                  const double* uniforms, uint64_t step, int32_t* out_accepted,
                                                  int32_t* out_tokens, int32_t* out_n_tokens,
                                                  int32_t* out_first_reject, int32_t* out_uniforms_used,
                                                  int32_t* out_status, void* stream);

/*
 * sixi_smp_verify without a handle and without any allocation (no counterpart in the engine).
 * For callers that may not allocate device memory at all - for instance a serving loop whose
 * device memory is owned by an external allocator, or one that must not call into the CUDA
 * allocator (cudaMalloc / cudaFree synchronize the device) - and therefore cannot create a
 * handle. Same arguments, semantics and outputs as sixi_smp_verify, with the vocabulary and the
 * device given directly; it runs on `device` (made current for the call).
 *   - The per-row workspace is a static device array of SIXI_SMP_STATIC_VERIFY_ROWS rows (16 bytes
 *     each, 64 KB): n_streams * (k + 1) larger than that returns SIXI_OUT_OF_BOUNDS.
 *   - Nothing in it has to start at zero: every row's slot is written before it is read.
 *   - The first call on each device resolves the workspace address (cudaGetSymbolAddress) and
 *     sets the kernels' shared-memory limits; make that first call before any stream capture
 *     begins on that device.
 *   - All calls on one device share the workspace: calls that overlap in time (on different
 *     streams, or from different threads) race and must be serialized by the caller.
 */
#define SIXI_SMP_STATIC_VERIFY_ROWS 4096u
SIXI_SMP_API int32_t sixi_smp_verify_static(int32_t device, uint32_t vocab, const sixi_smp_rows* target,
                               const float* draft_probs, const int32_t* drafts, const int32_t* n_drafts,
                               uint32_t n_streams, uint32_t k, const sixi_smp_params* params,
                               const uint32_t* mask_words, const int32_t* hist_tokens,
                               const int64_t* hist_offsets, const double* uniforms, uint64_t step,
                               int32_t* out_accepted, int32_t* out_tokens, int32_t* out_n_tokens,
                               int32_t* out_first_reject, int32_t* out_uniforms_used, int32_t* out_status,
                               void* stream);

/*
 * Vocab-sharded mode (logits produced vocab-parallel; no counterpart in the engine, which runs on
 * one device). The handle is created for the full vocabulary.
 * Stage 1 on every rank: for each row of this rank's slice [vocab_offset, vocab_offset +
 * shard_vocab) (shard_rows: n_rows rows of shard_vocab <= row_stride logits; shard_vocab <=
 * 97,000), apply mask and penalties as sixi_smp_sample does and emit the slice's best `top_n`
 * (1..64) candidates (adjusted logit, global id; sorted logit desc, id asc; padded with -inf / -1),
 * the slice max, the sum of exp((x - max) / T) over the slice (fp32 terms ~1e-7 relative, fp64
 * sum) and the allowed count.
 *   params      [n_rows] (the same records on every rank)
 *   mask_words  full-vocabulary masks [n_rows][ceil(full_vocab/32)]; the slice reads its bit range
 *   hist_*      CSR histories of global ids (the same on every rank)
 *   out_cand    [n_rows][top_n] of {float logit; int32 id} (8 bytes each)
 *   out_stats   [n_rows] of {float max; int32 n_allowed; double sum_exp; int32 status; int32 pad}
 * Stage 2, after an all-gather of both arrays over the ranks (rank-major: [n_shards][n_rows][top_n]
 * and [n_shards][n_rows]), runs identically on every rank: it merges the shards of each row and
 * draws the token as sixi_smp_sample would on the full row (uniforms [n_rows] or NULL for Philox
 * slot 0). Exact whenever top_k <= top_n. Otherwise the merged list is known down to the worst
 * listed candidate of any shard whose list was truncated; a row whose top-k, top-p, min-p or draw
 * decision falls beyond that point reports SIXI_OUT_OF_BOUNDS (n_shards <= 16,
 * n_shards * top_n <= 1024).
 */
SIXI_SMP_API int32_t sixi_smp_shard_candidates(sixi_smp* h, const sixi_smp_rows* shard_rows,
                                  uint32_t vocab_offset, uint32_t shard_vocab, uint32_t full_vocab,
                                  const sixi_smp_params* params, const uint32_t* mask_words,
                                  const int32_t* hist_tokens, const int64_t* hist_offsets,
                                  uint32_t top_n, void* out_cand, void* out_stats, void* stream);
SIXI_SMP_API int32_t sixi_smp_merge_shards(sixi_smp* h, uint32_t n_rows, uint32_t n_shards, uint32_t top_n,
                              const void* gathered_cand, const void* gathered_stats,
                              const sixi_smp_params* params, const double* uniforms, uint64_t step,
                              int32_t* out_tokens, int32_t* out_status, void* stream);

/*
 * NaN / Inf inspection and policy of logits rows, in place: inspect_and_apply_numeric_policy
 * (src/core/numeric.cpp:628-699; NumericPolicy and NumericHealthReport,
 * include/sixi_asi/numeric.hpp:126-140), batched over device rows. The engine applies it to a row's
 * logits before sampling (src/core/core_execution.cpp:2127-2135, src/server/server.cpp:2351-2366).
 * For each of n_rows rows of vocab fp32 logits (rows + r * row_stride; 4-byte aligned):
 *   - counts NaNs and infinities and finds the first index holding either (-1 when none);
 *   - SIXI_SMP_NUMERIC_FAIL leaves the row unchanged; a row with any NaN or Inf reports
 *     healthy = 0, request_corrupted = state_invalidated = 1, emergency_clamped = 0 and status
 *     SIXI_NUMERIC_NAN_OR_INF;
 *   - SIXI_SMP_NUMERIC_CLAMP writes NaN -> +0, +-Inf -> +-|clamp_abs_max| and, when
 *     |clamp_abs_max| > 0, finite values beyond it -> +-|clamp_abs_max|; a row with any NaN or Inf
 *     reports healthy = 0, and emergency_clamped = 1 when it was bad or a finite value was clamped;
 *     status SIXI_OK.
 * out_reports [n_rows] is device memory. Asynchronous on `stream`; the return value covers the
 * arguments and the launch only.
 */
#define SIXI_SMP_NUMERIC_FAIL 0u  /* NumericPolicy::FailAndInvalidate */
#define SIXI_SMP_NUMERIC_CLAMP 1u /* NumericPolicy::EmergencyClampAndReport */
typedef struct sixi_smp_numeric_report {
    uint8_t healthy;
    uint8_t request_corrupted;
    uint8_t state_invalidated;
    uint8_t emergency_clamped;
    int32_t status;          /* SIXI_OK or SIXI_NUMERIC_NAN_OR_INF */
    uint64_t nan_count;
    uint64_t inf_count;
    int64_t first_bad_index; /* -1 when every value is finite */
} sixi_smp_numeric_report;   /* 32 bytes */
SIXI_SMP_API int32_t sixi_smp_numeric_policy(sixi_smp* h, float* rows, uint32_t n_rows, uint64_t row_stride,
                                             uint32_t policy, float clamp_abs_max,
                                             sixi_smp_numeric_report* out_reports, void* stream);

/*
 * Suffix n-gram drafting for a batch of streams on the device: SuffixDrafter::propose and
 * SuffixDrafter::propose_anchored (src/speculative/speculative.cpp:24-176;
 * include/sixi_asi/speculative.hpp:33-54), the engine's first drafter in SpeculativeDecoder
 * (speculative.cpp:329, 340-360). Histories are CSR like the penalty histories: stream s owns
 * hist_tokens[hist_offsets[s] .. hist_offsets[s + 1]) (device memory).
 *   anchors == NULL: propose - the most recent, longest match (at most 16 tokens, at least
 *     min_match_len) of the history's suffix within its last max_window_tokens tokens;
 *   anchors != NULL: propose_anchored - the same with anchors[s] as the pattern's last token.
 * The k drafts continue the history after the match, repeating the continuation when it is
 * shorter than k. out_drafts [n_streams][k] (-1 for a stream without a proposal); out_match_len
 * [n_streams]: the engine's match_len, 0 when the engine returns no proposal. The drafts are
 * one-hot (sixi_smp_verify with draft_probs = NULL). min_match_len <= 64, k <= 4096.
 */
SIXI_SMP_API int32_t sixi_smp_suffix_draft(sixi_smp* h, const int32_t* hist_tokens, const int64_t* hist_offsets,
                                           uint32_t n_streams, uint32_t min_match_len, uint32_t max_window_tokens,
                                           const int32_t* anchors, uint32_t k, int32_t* out_drafts,
                                           int32_t* out_match_len, void* stream);

/* Philox4x32-10 uniform used when `uniforms` is NULL (host copy of the device function). */
SIXI_SMP_API double sixi_smp_philox_uniform(uint64_t seed, uint64_t counter, uint32_t slot);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* SIXI_SMP_H */
