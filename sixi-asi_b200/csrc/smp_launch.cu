// smp_launch.cu - host-side launch planning and dispatch of the row-engine kernels.
#include <atomic>

#include "smp_row.cuh"

namespace sixi_b200 {

static uint32_t chunk_for(uint32_t vocab, uint32_t c) {
    uint32_t chunk = (vocab + c - 1) / c;
    return (chunk + 7u) / 8u * 8u;
}

uint32_t device_sm_count(int device) {
    static std::atomic<uint32_t> cache[64];
    if (device < 0 || device >= 64) return 0;
    uint32_t n = cache[device].load(std::memory_order_relaxed);
    if (n != 0) return n;
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0) return 0;
    cache[device].store(static_cast<uint32_t>(v), std::memory_order_relaxed);
    return static_cast<uint32_t>(v);
}

// Resident-cluster counts per device and cluster size (1, 2, 4, 8, 16), each packed as
// (shared-memory bytes << 32) | clusters; 0 = not queried. plan_rows uses an entry only when its
// shared-memory size is the plan's (the count depends on it).
static std::atomic<uint64_t> g_max_clusters[64][5];

static int cluster_slot(uint32_t c) { return c == 1 ? 0 : c == 2 ? 1 : c == 4 ? 2 : c == 8 ? 3 : c == 16 ? 4 : -1; }

static uint32_t resident_clusters(int device, uint32_t c, size_t smem) {
    const int s = cluster_slot(c);
    if (device < 0 || device >= 64 || s < 0) return 0;
    const uint64_t v = g_max_clusters[device][s].load(std::memory_order_relaxed);
    return (v >> 32) == smem ? static_cast<uint32_t>(v & 0xFFFFFFFFu) : 0u;
}

cudaError_t prepare_plans(int device, uint32_t vocab) {
    if (device < 0 || device >= 64 || vocab == 0) return cudaErrorInvalidValue;
    for (uint32_t c = 1; c <= 16; c *= 2) {
        if (chunk_for(vocab, c) > kMaxChunk) continue;
        const size_t smem = make_layout(chunk_for(vocab, c), c).total;
        if (smem > static_cast<size_t>(kMaxSmem)) continue;
        int n = 0;
        const cudaError_t e = query_max_clusters(c, smem, &n);
        if (e != cudaSuccess) return e;
        g_max_clusters[device][cluster_slot(c)].store((static_cast<uint64_t>(smem) << 32) | static_cast<uint32_t>(n),
                                                      std::memory_order_relaxed);
    }
    return cudaSuccess;
}

bool plan_rows(uint32_t vocab, uint32_t n_rows, uint32_t sms, LaunchPlan* plan, int device) {
    if (vocab == 0) return false;
    uint32_t c = 1;
    while (c <= 16 && chunk_for(vocab, c) > kMaxChunk) c *= 2;
    if (c > 16) return false;
    // widen the cluster (up to 8 CTAs) while the batch would leave more than half of the SMs idle;
    // 16-CTA clusters for a lone row measured slower (18.1 against 16.4 us per config-1 step). A
    // wider cluster must also leave every row resident at once: at 8 CTAs a B200 holds 16
    // clusters, so 17 list rows took 32.7 us per step (two waves) against 24.8 us at 4 CTAs.
    while (c < 8 && n_rows > 0 && static_cast<uint64_t>(n_rows) * c * 2 <= sms && chunk_for(vocab, 2 * c) >= 2048) {
        const uint32_t held = resident_clusters(device, 2 * c, make_layout(chunk_for(vocab, 2 * c), 2 * c).total);
        if (held != 0 && n_rows > held) break;
        c *= 2;
    }
    plan->cluster = c;
    plan->chunk = chunk_for(vocab, c);
    plan->smem = make_layout(plan->chunk, c).total;
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
    cudaError_t e = prepare_mode_dt<kModeSample, SIXI_SMP_F32>(device);
    if (e == cudaSuccess) e = prepare_mode_dt<kModeSample, SIXI_SMP_BF16>(device);
    if (e == cudaSuccess) e = prepare_mode_dt<kModeCandidates, SIXI_SMP_F32>(device);
    if (e == cudaSuccess) e = prepare_mode_dt<kModeCandidates, SIXI_SMP_BF16>(device);
    if (e == cudaSuccess) e = prepare_mode_dt<kModeGreedy, SIXI_SMP_F32>(device);
    if (e == cudaSuccess) e = prepare_mode_dt<kModeGreedy, SIXI_SMP_BF16>(device);
    if (e == cudaSuccess) e = prepare_mode_dt<kModeVerify, SIXI_SMP_F32>(device);
    if (e == cudaSuccess) e = prepare_mode_dt<kModeVerify, SIXI_SMP_BF16>(device);
    if (e == cudaSuccess) e = prepare_full_distribution(device);
    return e;
}

}  // namespace sixi_b200
