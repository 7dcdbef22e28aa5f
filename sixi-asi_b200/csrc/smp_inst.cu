// smp_inst.cu - one (mode, dtype) family of row-engine kernel instances. The build compiles
// this file once per pair with -DSIXI_INST_MODE=<mode> -DSIXI_INST_DT=<dtype>, in parallel.
#include <atomic>

#include "smp_row.cuh"

#ifndef SIXI_INST_MODE
#error "SIXI_INST_MODE must be defined"
#endif
#ifndef SIXI_INST_DT
#error "SIXI_INST_DT must be defined"
#endif

namespace sixi_b200 {

// The shared-memory opt-in and non-portable cluster sizes of this instance, set once per device
// (prepare_kernels sets them for every instance up front, so that later launches issue no
// attribute call: they may be inside a stream capture).
static std::atomic<uint64_t> g_ready{0};

static cudaError_t prepare_this(int dev) {
    auto kfn = row_kernel<SIXI_INST_DT, SIXI_INST_MODE>;
    const uint64_t bit = 1ull << (dev & 63);
    if (g_ready.load(std::memory_order_acquire) & bit) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kfn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    g_ready.fetch_or(bit, std::memory_order_acq_rel);
    return cudaSuccess;
}

static cudaError_t launch_one(const RowArgs& a, const LaunchPlan& plan, cudaStream_t stream) {
    auto kfn = row_kernel<SIXI_INST_DT, SIXI_INST_MODE>;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    e = prepare_this(dev);
    if (e != cudaSuccess) return e;
    if (plan.smem > static_cast<size_t>(kMaxSmem)) return cudaErrorInvalidValue;
    // one CTA per (row, cluster rank): refuse grids beyond the 2^31 - 1 CTAs of gridDim.x
    const uint64_t ctas = static_cast<uint64_t>(a.n_rows) * plan.cluster;
    if (ctas == 0) return cudaSuccess;
    if (ctas > 0x7FFFFFFFull) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<uint32_t>(ctas), 1, 1);
    cfg.blockDim = dim3(kNT, 1, 1);
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = plan.cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kfn, a);
}

template <>
cudaError_t launch_mode_dt<SIXI_INST_MODE, SIXI_INST_DT>(const RowArgs& a, const LaunchPlan& plan,
                                                         cudaStream_t stream) {
    return launch_one(a, plan, stream);
}

template <>
cudaError_t prepare_mode_dt<SIXI_INST_MODE, SIXI_INST_DT>(int device) {
    return prepare_this(device);
}

#if SIXI_INST_MODE == 0 && SIXI_INST_DT == 0
cudaError_t query_max_clusters(uint32_t cluster, size_t smem, int* n_clusters) {
    auto kfn = row_kernel<SIXI_INST_DT, SIXI_INST_MODE>;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = prepare_this(dev);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cluster, 1, 1);
    cfg.blockDim = dim3(kNT, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaOccupancyMaxActiveClusters(n_clusters, kfn, &cfg);
}
#endif

}  // namespace sixi_b200
