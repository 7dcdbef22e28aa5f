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
    // verify
    const float* q;
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
// widened (up to 8 CTAs) while the batch leaves SMs idle.
bool plan_rows(uint32_t vocab, uint32_t n_rows, LaunchPlan* plan);
cudaError_t launch_rows(int mode, const RowArgs& a, const LaunchPlan& plan, cudaStream_t stream);
cudaError_t launch_verify_finalize(const RowArgs& a, uint32_t n_streams, int32_t* out_accepted,
                                   int32_t* out_tokens, int32_t* out_n_tokens,
                                   int32_t* out_first_reject, int32_t* out_uniforms_used,
                                   int32_t* out_status, cudaStream_t stream);
cudaError_t prepare_kernels(int device);

}  // namespace sixi_b200
