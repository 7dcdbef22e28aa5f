// smp_kernels.cuh - launch interface of the row-engine kernels (host side, internal).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/sixi_smp.h"

namespace sixi_b200 {

enum KernelMode : int {
    kModeSample = 0,      // one token per row (sixi_smp_sample)
    kModeCandidates = 1,  // sorted candidate list per row (sixi_smp_candidates)
    kModeGreedy = 2,      // raw argmax per row (sixi_smp_greedy_argmax)
    kModeVerify = 3,      // per target row verification partials (sixi_smp_verify)
};

// One row of the verifier's per-row workspace (global scratch written by the row kernel and read
// by the per-stream finalize kernel).
struct VerifyRowResult {
    int32_t status;
    int32_t accept;  // draft rows: 1 if the draft token was accepted
    int32_t token;   // greedy: argmax; stochastic draft row: residual draw; bonus row: bonus
    int32_t pad;
};

// Statistics of one draft row's full distribution (DeterministicSampler::compute_full_distribution,
// src/core/core_execution.cpp:409-447): q_i = float(exp(x_i * inv_t - maxs) / sum) (mode 0), one-hot
// at `amax` (mode 1: temperature <= 0), or all zero (mode 2: a NaN or +inf logit, no finite
// maximum, or a sum that is not positive). Written by dist_kernel's statistics pass, read by the
// verifier, so that q is evaluated where it is needed instead of being stored.
struct DraftStat {
    double inv_t;
    double maxs;
    double sum;
    int32_t amax;
    int32_t mode;
};
static_assert(sizeof(DraftStat) == 32, "DraftStat layout");

struct RowArgs {
    const void* data;
    uint64_t row_stride;  // elements
    uint32_t dtype;
    uint32_t vocab;
    uint32_t n_rows;
    uint32_t chunk;  // elements per CTA, multiple of 8
    uint32_t use_tma;
    uint32_t mask_words;
    const sixi_smp_params* params;
    const uint32_t* mask;
    const int32_t* hist;
    const int64_t* hist_off;
    const double* uniforms;
    uint64_t step;
    // sample mode: row j of `data` is sampled as row row_map[j] (its parameters, mask, history,
    // uniform and output slots); nullptr = the identity
    const uint32_t* row_map;
    // verify
    const float* q;            // dense draft probabilities [S*k][row_stride], or
    const void* qlog;          // draft logits [S*k][qlog_stride] (dtype qlog_dtype) with their
    const DraftStat* qstat;    //   distribution statistics [S*k]: q evaluated on demand
    uint64_t qlog_stride;
    uint32_t qlog_dtype;
    const int32_t* drafts;
    const int32_t* n_drafts;
    uint32_t k;
    VerifyRowResult* ws;
    // outputs
    int32_t* out_tok;
    int32_t* out_status;
    uint32_t max_out;
    int32_t* out_ids;
    double* out_probs;
    int32_t* out_count;
};

// Launch configuration chosen by the host for a vocabulary size.
struct LaunchPlan {
    uint32_t cluster;  // CTAs per row
    uint32_t chunk;    // elements per CTA (multiple of 8)
    size_t smem;       // dynamic shared memory bytes
};

// Launch plan for a vocabulary and batch: the smallest cluster whose chunk fits shared memory,
// widened (up to 8 CTAs) while the batch leaves more than half of the device's `sms` SMs idle
// (sms = 0: no widening; the plan then only validates the vocabulary) and, when `device` >= 0 and
// prepare_plans has run for it, while every cluster of the wider size is still resident at once
// (clusters are placed whole within a GPC, so fewer of them fit than the SM count suggests).
bool plan_rows(uint32_t vocab, uint32_t n_rows, uint32_t sms, LaunchPlan* plan, int device = -1);
// Records, for `device` and the plans of `vocab`, how many clusters of each size the device holds
// at once (cudaOccupancyMaxActiveClusters), for plan_rows. Call with `device` current, after
// prepare_kernels, before any stream capture.
cudaError_t prepare_plans(int device, uint32_t vocab);
// Clusters of `cluster` CTAs with `smem` bytes of dynamic shared memory each that the current
// device holds at once, for the row engine's launch shape (defined with the sample-mode instance).
cudaError_t query_max_clusters(uint32_t cluster, size_t smem, int* n_clusters);
// Streaming multiprocessors of `device` (queried once per device; 0 when the query fails).
uint32_t device_sm_count(int device);
cudaError_t launch_rows(int mode, const RowArgs& a, const LaunchPlan& plan, cudaStream_t stream);
cudaError_t launch_verify_finalize(const RowArgs& a, uint32_t n_streams, int32_t* out_accepted,
                                   int32_t* out_tokens, int32_t* out_n_tokens,
                                   int32_t* out_first_reject, int32_t* out_uniforms_used,
                                   int32_t* out_status, cudaStream_t stream);
// Sets the row engine's launch attributes (shared-memory opt-in, non-portable cluster sizes) for
// every (mode, dtype) instance on the current device, `device`, so that no later launch issues an
// attribute call (launches may then run inside a stream capture).
cudaError_t prepare_kernels(int device);
template <int MODE, int DT>
cudaError_t prepare_mode_dt(int device);

// ---- NaN / Inf policy (smp_numeric.cu) -------------------------------------------------------
cudaError_t launch_numeric_policy(float* data, uint32_t n_rows, uint64_t row_stride, uint32_t vocab, uint32_t policy,
                                  float limit, sixi_smp_numeric_report* out, cudaStream_t stream);

// ---- suffix n-gram drafting (smp_suffix.cu) --------------------------------------------------
cudaError_t launch_suffix_draft(const int32_t* hist, const int64_t* off, uint32_t n_streams, uint32_t min_match,
                                uint32_t window, const int32_t* anchors, uint32_t k, int32_t* out_drafts,
                                int32_t* out_match, cudaStream_t stream);

// ---- vocab-sharded mode (smp_shard.cu) ---------------------------------------------------------
struct ShardCand {  // one candidate of a shard (8 bytes, the layout of include/sixi_smp.h)
    float logit;    // adjusted logit (mask, penalties applied)
    int32_t id;     // global token id, -1 for padding
};
struct ShardStats {  // per-row summary of a shard (24 bytes)
    float max;       // largest adjusted allowed logit (-inf when none)
    int32_t n_allowed;
    double sum_exp;  // sum over allowed ids of exp((x - max) / T) (0 for greedy rows)
    int32_t status;
    int32_t pad;
};
static_assert(sizeof(ShardCand) == 8 && sizeof(ShardStats) == 24, "shard record layouts");

constexpr uint32_t kMaxShards = 16;
constexpr uint32_t kMaxShardTopN = 64;
constexpr size_t kMaxShardSmem = 227 * 1024;

struct ShardArgs {
    const void* data;
    uint64_t row_stride;  // elements
    uint32_t dtype;
    uint32_t shard_vocab;
    uint32_t vocab_offset;
    uint32_t full_vocab;
    uint32_t mask_words;  // words per full-vocabulary mask row
    uint32_t n_rows;
    uint32_t top_n;
    const sixi_smp_params* params;
    const uint32_t* mask;
    const int32_t* hist;
    const int64_t* hist_off;
    ShardCand* out_cand;
    ShardStats* out_stats;
};
struct MergeArgs {
    uint32_t n_rows, n_shards, top_n;
    const ShardCand* cand;    // [n_shards][n_rows][top_n]
    const ShardStats* stats;  // [n_shards][n_rows]
    const sixi_smp_params* params;
    const double* uniforms;
    uint64_t step;
    int32_t* out_tok;
    int32_t* out_status;
};
size_t shard_smem_bytes(uint32_t shard_vocab);

// ---- full-vocabulary softmax rows (smp_dist.cu) -------------------------------------------------
struct DistArgs {
    const void* data;
    uint64_t row_stride;  // elements
    uint32_t dtype;
    uint32_t vocab;
    uint32_t n_rows;
    uint32_t chunk;       // elements per CTA of a row's cluster
    const float* temperatures;
    float* out;           // the distribution rows, or nullptr with `stats` (statistics only)
    uint64_t out_stride;  // elements
    DraftStat* stats;     // per-row statistics (nullable)
};
cudaError_t launch_full_distribution(const DistArgs& a, const LaunchPlan& plan, cudaStream_t stream);
cudaError_t prepare_full_distribution(int device);  // its launch attributes, once per device
cudaError_t launch_shard_candidates(const ShardArgs& a, cudaStream_t stream);
cudaError_t launch_merge_shards(const MergeArgs& a, cudaStream_t stream);
cudaError_t launch_gather_rows(const void* src, uint64_t src_stride, uint32_t esz, const int32_t* index, uint32_t n,
                               uint32_t width, void* dst, uint64_t dst_stride, cudaStream_t stream);

}  // namespace sixi_b200
