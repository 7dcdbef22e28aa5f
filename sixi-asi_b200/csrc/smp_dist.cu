// smp_dist.cu - full-vocabulary softmax rows (sixi_smp_full_distribution), the producer of dense
// draft distributions: DeterministicSampler::compute_full_distribution
// (src/core/core_execution.cpp:409-447) per row, with one cluster of CTAs per row. With `stats` and
// no `out` only the row's maximum and sum are kept (DraftStat), from which the verifier evaluates
// the same q values where it reads them (sixi_smp_verify_draft_logits).
//
//   temperature <= 0  a one-hot row at the raw argmax (strict >, so the lowest id wins ties, a NaN
//                     at index 0 wins and other NaNs never do; sample_greedy_argmax)
//   otherwise         float(exp(x / T - max) / sum) with fp64 terms: max over x * (1 / T) (NaN
//                     ignored); a NaN or +inf logit makes the sum NaN and the engine leaves every
//                     probability 0, as here. The per-element operations are the engine's (a
//                     multiply, then a subtract, no contraction); the sum runs in parallel, so it
//                     differs from the engine's sequential sum only by fp64 rounding.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cfloat>
#include <cstdint>

#include "../../include/sixi_smp.h"
#include "smp_device.cuh"
#include "smp_kernels.cuh"

namespace cg = cooperative_groups;

namespace sixi_b200 {
namespace {

constexpr int kDT = 256;
constexpr int kDW = kDT / 32;
constexpr int kDMaxC = 16;
constexpr uint32_t kDChunk = 12288;     // preferred largest chunk per CTA (48 KB of fp32)
constexpr uint32_t kDMaxChunk = 37984;  // hard limit: 16 CTAs cover the row engine's widest vocabulary
constexpr uint32_t kDWaitIters = 1u << 24;  // bound of the bulk-copy wait

struct DistShared {
    uint64_t mbar;                   // completion of the chunk's bulk copy
    double mx[kDMaxC];               // per-CTA scaled maxima (pushed by every CTA)
    double sm[kDMaxC];               // per-CTA partial sums
    unsigned int bad[kDMaxC];        // per-CTA NaN / +inf flags
    unsigned long long best[kDMaxC]; // per-CTA argmax composites (greedy rows)
    double redd[kDW];
    unsigned long long red[kDW];
    unsigned int redu[kDW];
};

__device__ __forceinline__ float dist_logit(const DistArgs& a, const uint8_t* row, uint32_t e) {
    if (a.dtype == SIXI_SMP_BF16)
        return __uint_as_float(static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(row)[e]) << 16);
    return reinterpret_cast<const float*>(row)[e];
}

__global__ void __launch_bounds__(kDT, 4) dist_kernel(const DistArgs a) {
    __shared__ DistShared sh;
    extern __shared__ __align__(16) uint8_t xs[];  // the chunk's raw elements (fp32 or bf16)
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t C = cluster.num_blocks();
    const uint32_t crank = cluster.block_rank();
    const uint32_t row = blockIdx.x / C;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const uint8_t* rowp = static_cast<const uint8_t*>(a.data) +
                          static_cast<size_t>(row) * a.row_stride * (a.dtype == SIXI_SMP_BF16 ? 2 : 4);
    float* out = a.out != nullptr ? a.out + static_cast<size_t>(row) * a.out_stride : nullptr;
    const uint32_t c0 = crank * a.chunk;
    const uint32_t c1 = c0 + a.chunk < a.vocab ? c0 + a.chunk : a.vocab;
    const float T = a.temperatures[row];
    if (T <= 0.0f) {
        // raw argmax: the composite (key, id) with NaN excluded; a NaN at index 0 is the answer
        unsigned long long best = 0ull;
        for (uint32_t e = c0 + tid; e < c1; e += kDT) {
            const float x = dist_logit(a, rowp, e);
            if (x != x) continue;
            const unsigned long long c = comp_of(fkey(x), e);
            best = c > best ? c : best;
        }
        best = warp_max_u64(best);
        if (lane == 0) sh.red[w] = best;
        __syncthreads();
        if (tid == 0) {
            unsigned long long b = 0ull;
            for (int i = 0; i < kDW; ++i) b = sh.red[i] > b ? sh.red[i] : b;
            for (uint32_t q = 0; q < C; ++q) cluster.map_shared_rank(&sh, q)->best[crank] = b;
        }
        cluster.sync();
        unsigned long long b = 0ull;
        for (uint32_t q = 0; q < C; ++q) b = sh.best[q] > b ? sh.best[q] : b;
        const float x0 = dist_logit(a, rowp, 0);
        const uint32_t win = (x0 != x0 || b == 0ull) ? 0u : comp_id(b);
        if (a.stats != nullptr && crank == 0 && tid == 0)
            a.stats[row] = DraftStat{0.0, 0.0, 0.0, static_cast<int32_t>(win), 1};
        if (a.out != nullptr)
            for (uint32_t e = c0 + tid; e < c1; e += kDT) out[e] = e == win ? 1.0f : 0.0f;
        return;
    }
    const double inv_temp = 1.0 / static_cast<double>(T);
    // 1. the chunk staged in shared memory by one bulk copy (phases 2 and 3 read it there; the
    // unaligned head or ragged tail with plain loads), its scaled maximum (NaN ignored) and its
    // non-finite flag
    const uint32_t n = c1 > c0 ? c1 - c0 : 0u;
    const uint32_t esz = a.dtype == SIXI_SMP_BF16 ? 2u : 4u;
    const uint8_t* src = rowp + static_cast<size_t>(c0) * esz;
    const uint32_t nbulk = (reinterpret_cast<uintptr_t>(src) & 15u) == 0u ? (n * esz) / 16u * 16u / esz : 0u;
    if (tid == 0) {
        mbar_init(&sh.mbar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0 && nbulk > 0u) {
        mbar_arrive_expect_tx(&sh.mbar, nbulk * esz);
        for (uint32_t off = 0; off < nbulk * esz; off += 32768u) {
            const uint32_t nb = nbulk * esz - off < 32768u ? nbulk * esz - off : 32768u;
            bulk_g2s(xs + off, src + off, nb, &sh.mbar);
        }
    }
    uint32_t first = nbulk;  // elements still to load with plain loads
    if (nbulk > 0u && !mbar_wait(&sh.mbar, 0, kDWaitIters)) first = 0u;  // not expected: reload all
    for (uint32_t e = first + tid; e < n; e += kDT) {
        if (esz == 2u) {
            reinterpret_cast<uint16_t*>(xs)[e] = reinterpret_cast<const uint16_t*>(src)[e];
        } else {
            reinterpret_cast<float*>(xs)[e] = reinterpret_cast<const float*>(src)[e];
        }
    }
    __syncthreads();
    auto xs_at = [&](uint32_t e) -> float {
        if (esz == 2u) return __uint_as_float(static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(xs)[e]) << 16);
        return reinterpret_cast<const float*>(xs)[e];
    };
    double mx = -INFINITY;
    unsigned int bad = 0u;
    for (uint32_t e = tid; e < n; e += kDT) {
        const float x = xs_at(e);
        bad |= (x != x || x == INFINITY) ? 1u : 0u;
        const double sc = __dmul_rn(static_cast<double>(x), inv_temp);
        mx = sc > mx ? sc : mx;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const double t = __shfl_xor_sync(0xFFFFFFFFu, mx, o);
        mx = t > mx ? t : mx;
        bad |= __shfl_xor_sync(0xFFFFFFFFu, bad, o);
    }
    if (lane == 0) {
        sh.redd[w] = mx;
        sh.redu[w] = bad;
    }
    __syncthreads();
    if (tid == 0) {
        double m = -INFINITY;
        unsigned int bd = 0u;
        for (int i = 0; i < kDW; ++i) {
            m = sh.redd[i] > m ? sh.redd[i] : m;
            bd |= sh.redu[i];
        }
        for (uint32_t q = 0; q < C; ++q) {
            DistShared* d = cluster.map_shared_rank(&sh, q);
            d->mx[crank] = m;
            d->bad[crank] = bd;
        }
    }
    cluster.sync();
    double max_scaled = -INFINITY;
    unsigned int any_bad = 0u;
    for (uint32_t q = 0; q < C; ++q) {
        max_scaled = sh.mx[q] > max_scaled ? sh.mx[q] : max_scaled;
        any_bad |= sh.bad[q];
    }
    // every x * inv_temp - max is NaN when the row holds a NaN or +inf, or is all -inf: zeros
    const bool zero = any_bad != 0u || max_scaled == -INFINITY;
    // 2. the partial sums of exp(x * inv_temp - max), in the same element order as before staging
    double s = 0.0;
    if (!zero) {
        // four independent exponentials per step, added in element order (the sum is the same as
        // with one element per step)
        auto term = [&](uint32_t e) {
            return exp(__dsub_rn(__dmul_rn(static_cast<double>(xs_at(e)), inv_temp), max_scaled));
        };
        uint32_t e = tid;
        for (; e + 3u * kDT < n; e += 4u * kDT) {
            const double t0 = term(e), t1 = term(e + kDT), t2 = term(e + 2u * kDT), t3 = term(e + 3u * kDT);
            s += t0;
            s += t1;
            s += t2;
            s += t3;
        }
        for (; e < n; e += kDT) s += term(e);
    }
    s = warp_sum_f64(s);
    if (lane == 0) sh.redd[w] = s;
    __syncthreads();
    if (tid == 0) {
        double t = 0.0;
        for (int i = 0; i < kDW; ++i) t += sh.redd[i];
        for (uint32_t q = 0; q < C; ++q) cluster.map_shared_rank(&sh, q)->sm[crank] = t;
    }
    cluster.sync();
    double sum = 0.0;
    for (uint32_t q = 0; q < C; ++q) sum += sh.sm[q];
    if (a.stats != nullptr && crank == 0 && tid == 0)
        a.stats[row] = DraftStat{inv_temp, max_scaled, sum, 0, (zero || !(sum > 0.0)) ? 2 : 0};
    if (a.out == nullptr) return;
    // 3. the probabilities
    if (zero || !(sum > 0.0)) {
        for (uint32_t e = c0 + tid; e < c1; e += kDT) out[e] = 0.0f;
        return;
    }
    for (uint32_t e = tid; e < n; e += kDT) {
        const double ex = exp(__dsub_rn(__dmul_rn(static_cast<double>(xs_at(e)), inv_temp), max_scaled));
        out[c0 + e] = static_cast<float>(ex / sum);
    }
}

}  // namespace

// The distribution's own launch shape: clusters wide enough (up to 16 CTAs) that a CTA's chunk takes
// at most 48 KB of shared memory, so that four CTAs (256 threads each) share an SM and one CTA's
// bulk copy and cluster barriers overlap another's fp64 arithmetic. The row engine's plan is not
// used.
static std::atomic<uint64_t> g_dist_ready{0};  // attributes set once per device

cudaError_t prepare_full_distribution(int dev) {
    const uint64_t bit = 1ull << (dev & 63);
    if (g_dist_ready.load(std::memory_order_acquire) & bit) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(dist_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(dist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(4u * kDMaxChunk));
    if (e != cudaSuccess) return e;
    g_dist_ready.fetch_or(bit, std::memory_order_acq_rel);
    return cudaSuccess;
}

cudaError_t launch_full_distribution(const DistArgs& args, const LaunchPlan& plan, cudaStream_t stream) {
    (void)plan;
    int dev = 0;
    cudaError_t pe = cudaGetDevice(&dev);
    if (pe == cudaSuccess) pe = prepare_full_distribution(dev);
    if (pe != cudaSuccess) return pe;
    uint32_t c = 1;
    while (c < static_cast<uint32_t>(kDMaxC) && (args.vocab + c - 1) / c > kDChunk) c *= 2;
    DistArgs a = args;
    a.chunk = ((args.vocab + c - 1) / c + 7u) / 8u * 8u;  // 16-byte aligned chunk starts
    if (a.chunk > kDMaxChunk) return cudaErrorInvalidValue;
    // one CTA per (row, cluster rank): refuse grids beyond the 2^31 - 1 CTAs of gridDim.x
    const uint64_t ctas = static_cast<uint64_t>(a.n_rows) * c;
    if (ctas == 0) return cudaSuccess;
    if (ctas > 0x7FFFFFFFull) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<uint32_t>(ctas));
    cfg.blockDim = dim3(kDT);
    cfg.dynamicSmemBytes = 4u * a.chunk;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = c;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, dist_kernel, a);
}

}  // namespace sixi_b200
