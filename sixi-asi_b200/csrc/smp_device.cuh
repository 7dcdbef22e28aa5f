// smp_device.cuh - device building blocks of the B200 logits-to-token kernels (sm_100a).
//
// Ordering, keys and weights:
//   * Every logit is held as a 32-bit monotone key (fkey): larger key = larger logit, -0 and +0
//     share a key, masked / out-of-range entries are key 0. The engine's candidate order
//     "logit desc, id asc" (src/core/core_execution.cpp:521-527) is the order of the 64-bit
//     composite (key << 32) | (0xFFFFFFFF - id), larger = better, unique per row.
//   * The probability mass of a candidate, for the selections that run over the whole vocabulary
//     (top_k = 0 or large k), is an unsigned 64-bit fixed-point weight
//     w ~ round(exp((x - max) / T) * 2^43) (see weight_of). Integer sums are exact and
//     order-independent, so
//     every CTA of a cluster derives identical cumulative masses and the selection is
//     deterministic. The exponent is computed with hi/lo-split constants so that the only
//     rounding is one fp32 rounding of the exponent and the ex2 approximation (relative error
//     ~1e-7 per weight); weights below 2^-44 of the maximum round to 0 and are never drawn.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace sixi_b200 {

constexpr uint32_t kPhiloxM0 = 0xD2511F53u;
constexpr uint32_t kPhiloxM1 = 0xCD9E8D57u;
constexpr uint32_t kPhiloxW0 = 0x9E3779B9u;
constexpr uint32_t kPhiloxW1 = 0xBB67AE85u;

// Philox4x32-10 (Salmon et al., SC'11).
__host__ __device__ inline void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint64_t p0 = static_cast<uint64_t>(kPhiloxM0) * c[0];
        const uint64_t p1 = static_cast<uint64_t>(kPhiloxM1) * c[2];
        const uint32_t n0 = static_cast<uint32_t>(p1 >> 32) ^ c[1] ^ k0;
        const uint32_t n2 = static_cast<uint32_t>(p0 >> 32) ^ c[3] ^ k1;
        c[1] = static_cast<uint32_t>(p1);
        c[3] = static_cast<uint32_t>(p0);
        c[0] = n0;
        c[2] = n2;
        k0 += kPhiloxW0;
        k1 += kPhiloxW1;
    }
}

// 53-bit uniform in [0,1) from Philox(key = seed, counter = {slot, 0, lo(ctr), hi(ctr)}), built
// like DeterministicRng::next_uniform01 (src/core/core_execution.cpp:55-61).
__host__ __device__ inline double philox_uniform(uint64_t seed, uint64_t ctr, uint32_t slot) {
    uint32_t c[4] = {slot, 0u, static_cast<uint32_t>(ctr), static_cast<uint32_t>(ctr >> 32)};
    philox4x32_10(c, static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
    const uint64_t v = (static_cast<uint64_t>(c[0]) << 32) | c[1];
    return static_cast<double>(v >> 11) * (1.0 / 9007199254740992.0);
}

// ---------------------------------------------------------------------------------------------
// keys

__device__ __forceinline__ uint32_t fkey(float f) {
    uint32_t b = __float_as_uint(f);
    if (b == 0x80000000u) b = 0u;  // -0 -> +0 (they compare equal)
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float kval(uint32_t k) {
    // (k & 0x80000000) ? (k & 0x7FFFFFFF) : ~k, as one shift and one three-input logic operation
    const uint32_t s = static_cast<uint32_t>(static_cast<int32_t>(k) >> 31);
    return __uint_as_float(k ^ (0x80000000u | ~s));
}

__device__ __forceinline__ uint64_t comp_of(uint32_t key, uint32_t id) {
    return (static_cast<uint64_t>(key) << 32) | (0xFFFFFFFFu - id);
}
__device__ __forceinline__ uint32_t comp_id(uint64_t c) {
    return 0xFFFFFFFFu - static_cast<uint32_t>(c);
}
__device__ __forceinline__ uint32_t comp_key(uint64_t c) { return static_cast<uint32_t>(c >> 32); }

// ---------------------------------------------------------------------------------------------
// fixed-point weights (see header comment)

constexpr double kWeightScale = 8796093022208.0;  // 2^43
constexpr int kABins = 2048;                      // exp-domain histogram bins per row

struct WeightCtx {
    float s_hi, s_lo;    // log2(e)/T split in two floats
    float c_hi, c_lo;    // -max*log2(e)/T split
    float bin_scale;     // bins per unit of -log2(weight) (>0)
};

__host__ __device__ inline void make_weight_ctx(float temperature, float max_logit, float range_log2,
                                                WeightCtx& w) {
    const double s = 1.4426950408889634 / static_cast<double>(temperature);
    const double c = -static_cast<double>(max_logit) * s;
    w.s_hi = static_cast<float>(s);
    w.s_lo = static_cast<float>(s - static_cast<double>(w.s_hi));
    w.c_hi = static_cast<float>(c);
    w.c_lo = static_cast<float>(c - static_cast<double>(w.c_hi));
    double r = range_log2;
    if (!(r > 1e-6)) r = 1e-6;
    if (r > 46.0) r = 46.0;  // below 2^-44 every weight is 0
    w.bin_scale = static_cast<float>((kABins - 1) / r);
}

// log2 of the relative weight (<= 0 for every candidate).
__device__ __forceinline__ float neg_log2w(float x, const WeightCtx& w) {
    return __fmaf_rn(x, w.s_hi, w.c_hi) + __fmaf_rn(x, w.s_lo, w.c_lo);
}

__device__ __forceinline__ float fast_ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Fixed-point weight round(2^t * 2^43) of t = neg_log2w(x) <= 0 (the scaling by 2^43 is exact, the
// conversion rounds to nearest; 0 below 2^-44).
__device__ __forceinline__ uint64_t weight_of(float x, const WeightCtx& w) {
    const float t = fminf(neg_log2w(x, w), 0.0f);
    return __float2ull_rn(fast_ex2(t) * 8796093022208.0f);  // in [0, 2^43]
}

// histogram bin of a candidate (0 = most likely); monotone non-increasing in x
__device__ __forceinline__ int abin_of(float x, const WeightCtx& w) {
    const float t = -neg_log2w(x, w);  // >= 0 (up to rounding)
    const float b = t * w.bin_scale;
    int ib = (b > 0.0f) ? static_cast<int>(b) : 0;
    return ib < kABins - 1 ? ib : kABins - 1;
}

// ---------------------------------------------------------------------------------------------
// 64x64 -> high 64 and uniform scaling of an integer mass: floor(u * total), u in [0,1)
__device__ __forceinline__ uint64_t scale_mass(double u, uint64_t total) {
    // u = m * 2^-53 (exactly for Philox draws; truncated otherwise)
    double um = u * 9007199254740992.0;
    if (!(um >= 0.0)) um = 0.0;
    uint64_t m = static_cast<uint64_t>(um);
    if (m > (1ull << 53) - 1) m = (1ull << 53) - 1;
    const uint64_t hi = __umul64hi(m, total);
    const uint64_t lo = m * total;
    return (hi << 11) | (lo >> 53);
}

// ceil(p * total) for a probability p in (0,1)
__device__ __forceinline__ uint64_t ceil_mass(float p, uint64_t total) {
    // p * 2^48 is an integer for float p >= 2^-24
    const uint64_t pm = static_cast<uint64_t>(static_cast<double>(p) * 281474976710656.0);
    const uint64_t hi = __umul64hi(pm, total);
    const uint64_t lo = pm * total;
    const uint64_t q = (hi << 16) | (lo >> 48);
    return q + ((lo & ((1ull << 48) - 1)) != 0 ? 1 : 0);
}

// ---------------------------------------------------------------------------------------------
// exact 64-bit sums in shared memory from native 32-bit atomics
//
// A 64-bit shared-memory atomicAdd is not a single native operation on sm_100 and slows down
// sharply when threads hit the same address; 32-bit adds are native. A split counter keeps the
// low and high words in separate arrays: the low word wraps, and the one thread whose add wraps
// it carries one into the high word, so (hi << 32) | lo is the exact sum in any order.

__device__ __forceinline__ void smem_add_split(uint32_t* lo, uint32_t* hi, unsigned long long w) {
    const uint32_t l = static_cast<uint32_t>(w);
    const uint32_t old = atomicAdd(lo, l);
    const uint32_t h = static_cast<uint32_t>(w >> 32) + ((old + l < old) ? 1u : 0u);
    if (h != 0u) atomicAdd(hi, h);
}
__device__ __forceinline__ unsigned long long join_split(uint32_t lo, uint32_t hi) {
    return (static_cast<unsigned long long>(hi) << 32) | lo;
}

// ---------------------------------------------------------------------------------------------
// warp / block primitives

__device__ __forceinline__ unsigned long long warp_sum_u64(unsigned long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}
__device__ __forceinline__ uint32_t warp_sum_u32(uint32_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}
__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}
__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xFFFFFFFFu, v, o);
        v = t > v ? t : v;
    }
    return v;
}
__device__ __forceinline__ unsigned long long warp_min_u64(unsigned long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xFFFFFFFFu, v, o);
        v = t < v ? t : v;
    }
    return v;
}
// inclusive scans within a warp
__device__ __forceinline__ uint32_t warp_incl_u32(uint32_t v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, v, o);
        if (lane >= o) v += t;
    }
    return v;
}
__device__ __forceinline__ unsigned long long warp_incl_u64(unsigned long long v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long t = __shfl_up_sync(0xFFFFFFFFu, v, o);
        if (lane >= o) v += t;
    }
    return v;
}
__device__ __forceinline__ double warp_incl_f64(double v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double t = __shfl_up_sync(0xFFFFFFFFu, v, o);
        if (lane >= o) v += t;
    }
    return v;
}

// Block-wide reductions; `red` is shared scratch of >= NT/32 entries of 8 bytes. Contains
// __syncthreads: every thread of the block must call.
template <int NT>
__device__ __forceinline__ unsigned long long block_sum_u64(unsigned long long v, unsigned long long* red) {
    v = warp_sum_u64(v);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    unsigned long long s = 0;
#pragma unroll
    for (int i = 0; i < NT / 32; ++i) s += red[i];
    return s;
}
template <int NT>
__device__ __forceinline__ unsigned long long block_max_u64(unsigned long long v, unsigned long long* red) {
    v = warp_max_u64(v);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    unsigned long long s = 0;
#pragma unroll
    for (int i = 0; i < NT / 32; ++i) s = red[i] > s ? red[i] : s;
    return s;
}
template <int NT>
__device__ __forceinline__ unsigned long long block_min_u64(unsigned long long v, unsigned long long* red) {
    v = warp_min_u64(v);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    unsigned long long s = ~0ull;
#pragma unroll
    for (int i = 0; i < NT / 32; ++i) s = red[i] < s ? red[i] : s;
    return s;
}
// exclusive prefix over threads (in thread order) of u32 values; returns the block total in *tot
template <int NT>
__device__ __forceinline__ uint32_t block_excl_u32(uint32_t v, uint32_t* red, uint32_t* tot) {
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t inc = warp_incl_u32(v);
    __syncthreads();
    if (lane == 31) red[w] = inc;
    __syncthreads();
    uint32_t before = 0, all = 0;
#pragma unroll
    for (int i = 0; i < NT / 32; ++i) {
        const uint32_t t = red[i];
        before += (i < w) ? t : 0u;
        all += t;
    }
    *tot = all;
    return before + inc - v;
}

// ---------------------------------------------------------------------------------------------
// TMA bulk copies (cp.async.bulk, no tensor map) and mbarriers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile(
        "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
        "r"(bytes)
        : "memory");
}

// Bounded wait on phase `parity`; returns false if the bound ran out (never expected: the copies
// read local HBM and complete in microseconds).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t max_iter) {
    const uint32_t a = smem_u32(bar);
    for (uint32_t i = 0; i < max_iter; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

// global -> shared bulk copy completing on `bar` (dst, src 16-byte aligned; bytes % 16 == 0)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// L2 policy for data read exactly once (a batch of logits): evicted first, so that streaming it
// through L2 does not displace data that is read again (in an engine, the model's own working set).
// At config 2 it measured neutral for the sampler itself.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// bulk_g2s with an L2 cache policy (from l2_evict_first_policy)
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

}  // namespace sixi_b200
