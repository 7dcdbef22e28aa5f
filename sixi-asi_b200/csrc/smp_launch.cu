// smp_launch.cu - host-side launch planning and dispatch of the row-engine kernels.
#include "smp_row.cuh"

namespace sixi_b200 {

int pick_ept(uint32_t chunk) {
    const uint32_t per = (chunk + kNT - 1) / kNT;
    if (per <= 8) return 8;
    if (per <= 16) return 16;
    if (per <= 80) return 80;
    if (per <= 128) return 128;
    return 0;
}

bool plan_for_vocab(uint32_t vocab, LaunchPlan* plan) {
    if (vocab == 0) return false;
    uint32_t chunk = (vocab + kC - 1) / kC;
    chunk = (chunk + 7u) / 8u * 8u;
    const int ept = pick_ept(chunk);
    if (ept == 0) return false;
    plan->ept = ept;
    plan->chunk = chunk;
    plan->smem = make_layout(chunk).total;
    return plan->smem <= static_cast<size_t>(kMaxSmem);
}

template <int MODE>
static cudaError_t launch_dt(const RowArgs& a, const LaunchPlan& plan, cudaStream_t stream) {
    return a.dtype == SIXI_SMP_BF16 ? launch_mode_dt<MODE, SIXI_SMP_BF16>(a, plan, stream)
                                    : launch_mode_dt<MODE, SIXI_SMP_F32>(a, plan, stream);
}

cudaError_t launch_rows(int mode, const RowArgs& a, const LaunchPlan& plan, cudaStream_t stream) {
    if (a.n_rows == 0) return cudaSuccess;
    switch (mode) {
        case kModeSample: return launch_dt<kModeSample>(a, plan, stream);
        case kModeCandidates: return launch_dt<kModeCandidates>(a, plan, stream);
        case kModeGreedy: return launch_dt<kModeGreedy>(a, plan, stream);
        case kModeVerify: return launch_dt<kModeVerify>(a, plan, stream);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_verify_finalize(const RowArgs& a, uint32_t n_streams, int32_t* out_accepted,
                                   int32_t* out_tokens, int32_t* out_n_tokens,
                                   int32_t* out_first_reject, int32_t* out_uniforms_used,
                                   int32_t* out_status, cudaStream_t stream) {
    if (n_streams == 0) return cudaSuccess;
    const uint32_t nb = (n_streams + 127) / 128;
    verify_finalize_kernel<<<nb, 128, 0, stream>>>(a, n_streams, out_accepted, out_tokens,
                                                   out_n_tokens, out_first_reject,
                                                   out_uniforms_used, out_status);
    return cudaGetLastError();
}

cudaError_t prepare_kernels(int device) {
    (void)device;
    return cudaSuccess;
}

}  // namespace sixi_b200
