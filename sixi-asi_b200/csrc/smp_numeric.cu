// smp_numeric.cu - NaN / Inf inspection and policy of logits rows (sixi_smp_numeric_policy).
//
// Restates inspect_and_apply_numeric_policy (src/core/numeric.cpp:628-699) for a batch of device
// rows. The pass is one read of every logit (and, under the clamp policy, a write of the 16-byte
// vectors that change), so it is bound by HBM bandwidth: each row is split over a cluster of up to
// 8 CTAs. A CTA whose chunk is 16-byte aligned and fits kNumStageMax bytes has it brought into
// shared memory by bulk copies issued at once (one memory round trip for the whole chunk, two CTAs
// per SM); otherwise every thread keeps ten 16-byte loads in flight. The per-CTA counts meet in
// CTA 0's shared memory (distributed shared memory), which writes the row's report. No scratch
// memory and no atomics in global memory are used, so one launch does the whole batch.
#include <atomic>

#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/sixi_smp.h"
#include "smp_device.cuh"
#include "smp_kernels.cuh"

namespace cg = cooperative_groups;

namespace sixi_b200 {
namespace {

constexpr int kNumNT = 256;      // threads per CTA (two CTAs per SM: a 32-row batch is resident at once)
constexpr int kNumUnroll = 10;   // 16-byte loads in flight per thread
constexpr uint32_t kNumMaxCpr = 8;
constexpr uint32_t kNumPerCta = 8192;  // elements per CTA that justify another CTA of the cluster
constexpr uint32_t kNumFillCtas = 2u * 148u;  // CTAs that fill a B200 (two per SM)
constexpr uint32_t kNumStageMax = 96u * 1024u;  // largest chunk staged in shared memory (bytes)
constexpr uint32_t kNumPiece = 32768u;          // bytes per bulk copy
constexpr uint32_t kNumWaitIters = 1u << 24;    // bound of the staging wait (never expected to run out)

struct NumPart {
    uint32_t nan, inf, first, clamped;
};

struct NumAcc {
    uint32_t nan = 0, inf = 0, first = 0xFFFFFFFFu, clamped = 0;
};

// One value (numeric.cpp:642-671): returns true when the value was rewritten.
__device__ __forceinline__ bool inspect_one(float& v, uint32_t idx, bool clamp, float limit, NumAcc& a) {
    const uint32_t b = __float_as_uint(v);
    if ((b & 0x7F800000u) == 0x7F800000u) {  // NaN or infinity
        const bool is_nan = (b & 0x007FFFFFu) != 0u;
        a.nan += is_nan ? 1u : 0u;
        a.inf += is_nan ? 0u : 1u;
        a.first = idx < a.first ? idx : a.first;
        if (clamp) {
            v = is_nan ? 0.0f : ((b >> 31) ? -limit : limit);
            return true;
        }
        return false;
    }
    if (clamp && limit > 0.0f) {
        if (v > limit) {
            v = limit;
            a.clamped = 1u;
            return true;
        }
        if (v < -limit) {
            v = -limit;
            a.clamped = 1u;
            return true;
        }
    }
    return false;
}

__global__ void __launch_bounds__(kNumNT, 2) numeric_kernel(float* __restrict__ data, uint64_t row_stride, uint32_t vocab,
                                                         uint32_t cpr, uint32_t per, uint32_t vec, uint32_t staged,
                                                         uint32_t clamp, float limit,
                                                         sixi_smp_numeric_report* __restrict__ out) {
    __shared__ NumPart parts[kNumMaxCpr];
    __shared__ NumPart red[kNumNT / 32];
    __shared__ __align__(8) uint64_t bar;
    extern __shared__ __align__(16) float4 stg[];
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t crank = cluster.block_rank();
    const uint64_t row = blockIdx.x / cpr;
    const int tid = threadIdx.x;
    const bool cl = clamp != 0u;
    float* x = data + row * row_stride;
    // this CTA's elements [b0, b1); per is a multiple of 4, so vector chunks stay aligned
    const uint32_t b0 = min(vocab, crank * per);
    const uint32_t b1 = min(vocab, b0 + per);
    NumAcc a;
    uint32_t tail0 = b0;
    if (staged) {
        // the chunk's whole 16-byte vectors by bulk copies, then the vectors from shared memory
        const uint32_t nv = (b1 - b0) >> 2;
        const uint32_t bytes = 16u * nv;
        if (tid == 0) {
            mbar_init(&bar, 1);
            fence_mbar_init();
            if (bytes > 0u) {
                mbar_arrive_expect_tx(&bar, bytes);
                for (uint32_t off = 0; off < bytes; off += kNumPiece) {
                    const uint32_t nb = bytes - off < kNumPiece ? bytes - off : kNumPiece;
                    bulk_g2s(reinterpret_cast<uint8_t*>(stg) + off, reinterpret_cast<const uint8_t*>(x + b0) + off,
                             nb, &bar);
                }
            }
        }
        __syncthreads();
        // on an expired wait (never expected) the vectors are read from global memory instead, and
        // the copies are waited for again before the CTA may exit
        const bool ok = bytes == 0u || mbar_wait(&bar, 0, kNumWaitIters);
        float4* x4 = reinterpret_cast<float4*>(x + b0);
        for (uint32_t j = tid; j < nv; j += kNumNT) {
            float4 v = ok ? stg[j] : x4[j];
            const uint32_t e = b0 + 4u * j;
            bool ch = inspect_one(v.x, e, cl, limit, a);
            ch |= inspect_one(v.y, e + 1u, cl, limit, a);
            ch |= inspect_one(v.z, e + 2u, cl, limit, a);
            ch |= inspect_one(v.w, e + 3u, cl, limit, a);
            if (ch) x4[j] = v;
        }
        if (!ok) mbar_wait(&bar, 0, kNumWaitIters);
        tail0 = b0 + 4u * nv;
    } else if (vec) {
        const uint32_t nv = (b1 - b0) >> 2;
        float4* x4 = reinterpret_cast<float4*>(x + b0);
        for (uint32_t i = tid; i < nv; i += kNumNT * kNumUnroll) {
            float4 v[kNumUnroll];
#pragma unroll
            for (int u = 0; u < kNumUnroll; ++u) {
                const uint32_t j = i + u * kNumNT;
                if (j < nv) v[u] = x4[j];
            }
#pragma unroll
            for (int u = 0; u < kNumUnroll; ++u) {
                const uint32_t j = i + u * kNumNT;
                if (j >= nv) continue;
                const uint32_t e = b0 + 4u * j;
                bool ch = inspect_one(v[u].x, e, cl, limit, a);
                ch |= inspect_one(v[u].y, e + 1u, cl, limit, a);
                ch |= inspect_one(v[u].z, e + 2u, cl, limit, a);
                ch |= inspect_one(v[u].w, e + 3u, cl, limit, a);
                if (ch) x4[j] = v[u];
            }
        }
        tail0 = b0 + 4u * nv;
    }
    for (uint32_t e = tail0 + tid; e < b1; e += kNumNT) {
        float v = x[e];
        if (inspect_one(v, e, cl, limit, a)) x[e] = v;
    }
    // block reduction, then CTA 0 of the cluster combines the CTAs in rank order
    const int w = tid >> 5, lane = tid & 31;
    const uint32_t wn = __reduce_add_sync(0xFFFFFFFFu, a.nan);
    const uint32_t wi = __reduce_add_sync(0xFFFFFFFFu, a.inf);
    const uint32_t wf = __reduce_min_sync(0xFFFFFFFFu, a.first);
    const uint32_t wc = __reduce_or_sync(0xFFFFFFFFu, a.clamped);
    if (lane == 0) red[w] = NumPart{wn, wi, wf, wc};
    __syncthreads();
    if (tid == 0) {
        NumPart p{0u, 0u, 0xFFFFFFFFu, 0u};
#pragma unroll
        for (int q = 0; q < kNumNT / 32; ++q) {
            p.nan += red[q].nan;
            p.inf += red[q].inf;
            p.first = red[q].first < p.first ? red[q].first : p.first;
            p.clamped |= red[q].clamped;
        }
        cluster.map_shared_rank(parts, 0)[crank] = p;
    }
    cluster.sync();
    if (crank == 0 && tid == 0) {
        unsigned long long n_nan = 0ull, n_inf = 0ull;
        uint32_t first = 0xFFFFFFFFu, clamped = 0u;
        for (uint32_t q = 0; q < cpr; ++q) {
            n_nan += parts[q].nan;
            n_inf += parts[q].inf;
            first = parts[q].first < first ? parts[q].first : first;
            clamped |= parts[q].clamped;
        }
        sixi_smp_numeric_report r;
        const bool bad = (n_nan + n_inf) > 0ull;
        r.healthy = bad ? 0u : 1u;
        r.request_corrupted = (bad && !cl) ? 1u : 0u;
        r.state_invalidated = (bad && !cl) ? 1u : 0u;
        r.emergency_clamped = cl ? ((bad || clamped) ? 1u : 0u) : 0u;
        r.status = (bad && !cl) ? SIXI_NUMERIC_NAN_OR_INF : SIXI_OK;
        r.nan_count = n_nan;
        r.inf_count = n_inf;
        r.first_bad_index = first == 0xFFFFFFFFu ? -1ll : static_cast<long long>(first);
        out[row] = r;
    }
}

}  // namespace

cudaError_t launch_numeric_policy(float* data, uint32_t n_rows, uint64_t row_stride, uint32_t vocab, uint32_t policy,
                                  float limit, sixi_smp_numeric_report* out, cudaStream_t stream) {
    if (n_rows == 0) return cudaSuccess;
    // CTAs per row: one per kNumPerCta elements, at most kNumMaxCpr, so that a row's chunks fit the
    // staged path. A batch of at least half a GPU's worth of CTAs in rows takes just enough CTAs per
    // row to fill the GPU (one per row from kNumFillCtas rows): there, clusters of 8 measured slower
    // (202 against 153 us at 1,024 rows, 55 against 44 us at 256 rows), while below it the staged
    // 8-CTA split is the faster one (16 against 20 us at 64 rows).
    uint32_t cpr = (vocab + kNumPerCta - 1) / kNumPerCta;
    cpr = cpr < 1u ? 1u : (cpr > kNumMaxCpr ? kNumMaxCpr : cpr);
    if (n_rows >= kNumFillCtas / 2) {
        const uint32_t want = (kNumFillCtas + n_rows - 1) / n_rows;
        cpr = cpr < want ? cpr : want;
    }
    if (static_cast<uint64_t>(n_rows) * cpr > 0x7FFFFFFFull) return cudaErrorInvalidValue;  // grid limit
    const uint32_t per = (((vocab + cpr - 1) / cpr) + 3u) & ~3u;
    const uint32_t vec = ((reinterpret_cast<uintptr_t>(data) & 15u) == 0 && (row_stride & 3u) == 0) ? 1u : 0u;
    const uint32_t staged = (vec && 4u * per <= kNumStageMax) ? 1u : 0u;
    // the shared-memory opt-in is set once per device, so later calls issue no attribute call
    static std::atomic<uint64_t> ready{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = 1ull << (dev & 63);
    if (!(ready.load(std::memory_order_acquire) & bit)) {
        e = cudaFuncSetAttribute(numeric_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kNumStageMax));
        if (e != cudaSuccess) return e;
        ready.fetch_or(bit, std::memory_order_acq_rel);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_rows * cpr, 1, 1);
    cfg.blockDim = dim3(kNumNT, 1, 1);
    cfg.dynamicSmemBytes = staged ? 4u * per : 0u;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cpr;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, numeric_kernel, data, row_stride, vocab, cpr, per, vec, staged,
                              policy == SIXI_SMP_NUMERIC_CLAMP ? 1u : 0u, limit, out);
}

}  // namespace sixi_b200
