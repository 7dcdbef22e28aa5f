/*
 * sixi_oracle.h - TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the Sixi-ASI engine's logits-to-token path, used as the parity checker of the
 * B200 kernels (tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg only). Nothing in
 * the product library links or calls it. Two implementations export these symbols:
 *   - liboracle.so  (sixi_oracle.c): a plain-C restatement ("port");
 *   - _ref/libsixiref.so (ref_shim.cpp): the engine's own DeterministicSampler code compiled from
 *     its sources, wrapped with the same signatures ("reference").
 * Parity of the port is pinned against the reference build and against the golden vectors in
 * tests/golden/ that the reference build produced.
 *
 * Conventions are those of include/sixi_smp.h (status codes, params, mask layout, CSR history),
 * with HOST pointers everywhere.
 */
#ifndef SIXI_ORACLE_H
#define SIXI_ORACLE_H

#include <stdint.h>
#include "../include/sixi_smp.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Returned by the reference shim for inputs the engine cannot express (min_p / frequency). */
#define ORC_UNSUPPORTED (-2)

/* Which implementation this library is: 0 = port, 1 = reference build. */
int32_t orc_kind(void);

/* Philox4x32-10 (Salmon et al., SC'11), and the 53-bit uniform built from its first two words. */
void orc_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]);
double orc_philox_uniform(uint64_t seed, uint64_t counter, uint32_t slot);

/* DeterministicSampler::sample_greedy_argmax on fp32 logits (core_execution.cpp:394-407). */
int32_t orc_greedy_argmax(const float* logits, uint64_t vocab);

/* Greedy argmax of one row with optional mask (argmax of the compacted allowed logits).
 * Returns the status (OK, INVALID_ARGUMENT when nothing is allowed, NUMERIC_NAN_OR_INF when an
 * allowed logit is not finite - the token is still produced as the engine would). */
int32_t orc_greedy_row(const void* row, uint32_t dtype, uint64_t vocab, const uint32_t* mask,
                       int32_t* out_token);

/* compute_sampling_candidates (core_execution.cpp:449-584) of one row, with the grammar mask
 * applied by compaction. Writes up to `cap` candidates (sorted) and the full count. */
int32_t orc_candidates(const void* row, uint32_t dtype, uint64_t vocab, const sixi_smp_params* p,
                       const int32_t* hist, uint64_t n_hist, const uint32_t* mask, uint64_t cap,
                       int32_t* out_ids, double* out_probs, uint64_t* out_n);

/* sample_token (core_execution.cpp:603-619) of one row with a supplied uniform `u`. */
int32_t orc_sample(const void* row, uint32_t dtype, uint64_t vocab, const sixi_smp_params* p,
                   const int32_t* hist, uint64_t n_hist, const uint32_t* mask, double u,
                   int32_t* out_token);

/* Batch of rows, same layout as sixi_smp_sample (host memory). `uniforms` NULL = Philox slot 0.
 * Rows are spread over `n_threads` threads (<= 0: all hardware threads). */
int32_t orc_sample_batch(const void* logits, uint32_t dtype, uint32_t n_rows, uint64_t row_stride,
                         uint64_t vocab, const sixi_smp_params* params, const uint32_t* masks,
                         const int32_t* hist_tokens, const int64_t* hist_offsets,
                         const double* uniforms, uint64_t step, int32_t* out_tokens,
                         int32_t* out_status, int32_t n_threads);

/* compute_full_distribution (core_execution.cpp:409-447) of one row: temperature <= 0 gives a
 * one-hot at the raw argmax; otherwise float(exp(x/T - max) / sum) with fp64 terms. */
void orc_full_distribution(const void* row, uint32_t dtype, uint64_t vocab, float temperature, float* out);

/* SuffixDrafter::propose (use_anchor = 0) or ::propose_anchored (use_anchor = 1, anchor) with
 * SuffixDrafter(min_match_len, max_window_tokens) (speculative.cpp:24-176) on one history of n
 * tokens. Returns the proposal's match_len, 0 when there is none; writes k drafts (-1 when none). */
int32_t orc_suffix_draft(const int32_t* hist, uint64_t n, uint32_t min_match_len, uint32_t max_window_tokens,
                         int32_t use_anchor, int32_t anchor, uint32_t k, int32_t* out_drafts);

/* inspect_and_apply_numeric_policy (numeric.cpp:628-699) on one fp32 row, in place. Returns the
 * engine's status (SIXI_NUMERIC_NAN_OR_INF for a bad row under SIXI_SMP_NUMERIC_FAIL) and fills
 * `out` in the layout of sixi_smp_numeric_report (whose status field repeats the return value). */
int32_t orc_numeric_policy(float* data, int64_t n, uint32_t policy, float clamp_abs_max,
                           sixi_smp_numeric_report* out);

/* Speculative verification, same layout and semantics as sixi_smp_verify (host memory). */
int32_t orc_verify(const void* target, uint32_t dtype, uint64_t row_stride, uint64_t vocab,
                   const float* draft_probs, const int32_t* drafts, const int32_t* n_drafts,
                   uint32_t n_streams, uint32_t k, const sixi_smp_params* params,
                   const uint32_t* masks, const int32_t* hist_tokens, const int64_t* hist_offsets,
                   const double* uniforms, uint64_t step, int32_t* out_accepted,
                   int32_t* out_tokens, int32_t* out_n_tokens, int32_t* out_first_reject,
                   int32_t* out_uniforms_used, int32_t* out_status, int32_t n_threads);

#ifdef __cplusplus
}
#endif

#endif
