// smp_suffix.cu - suffix n-gram drafting for a batch of streams (sixi_smp_suffix_draft).
//
// Restates SuffixDrafter::propose and ::propose_anchored (src/speculative/speculative.cpp:24-176)
// with one CTA per stream. The engine scans candidate positions from the most recent backwards and
// keeps a new best only when its match is strictly longer, so the result is the longest match and,
// among equal lengths, the most recent position: here every thread scores a share of the positions
// and a block-wide maximum of (length << 32 | position) picks the same one. The window (plus the 16
// tokens an anchored match may reach below it) is staged in shared memory when it fits.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "../../include/sixi_smp.h"
#include "smp_kernels.cuh"

namespace sixi_b200 {
namespace {

constexpr int kSdNT = 1024;
constexpr uint32_t kSdMaxPattern = 16;             // speculative.cpp:39, 132
constexpr uint32_t kSdStageMax = 96u * 1024u;      // bytes of history staged in shared memory

struct SdHist {  // the stream's history, staged (base = s0) or in global memory (base = 0)
    const int32_t* p;
    uint64_t base;
    __device__ __forceinline__ int32_t operator[](uint64_t i) const { return p[i - base]; }
};

__device__ __forceinline__ unsigned long long block_max(unsigned long long v, unsigned long long* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xFFFFFFFFu, v, o);
        v = t > v ? t : v;
    }
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    unsigned long long m = 0ull;
#pragma unroll
    for (int q = 0; q < kSdNT / 32; ++q) m = red[q] > m ? red[q] : m;
    return m;
}

__global__ void __launch_bounds__(kSdNT) suffix_kernel(const int32_t* __restrict__ hist, const int64_t* __restrict__ off,
                                                       uint32_t min_match, uint32_t window, const int32_t* anchors,
                                                       uint32_t k, uint32_t stage_cap, int32_t* __restrict__ out_drafts,
                                                       int32_t* __restrict__ out_match) {
    extern __shared__ int32_t sh[];
    __shared__ unsigned long long red[kSdNT / 32];
    const uint32_t s = blockIdx.x;
    const int tid = threadIdx.x;
    const int64_t h0 = off[s];
    const uint64_t n = static_cast<uint64_t>(off[s + 1] - h0);
    const int32_t* g = hist + h0;
    const bool anchored = anchors != nullptr;
    const int32_t anchor = anchored ? anchors[s] : 0;
    const uint64_t ws = n > window ? n - window : 0;
    // staging: [s0, n) with s0 up to 16 below the window (an anchored match may reach there)
    const uint64_t s0 = ws > kSdMaxPattern ? ws - kSdMaxPattern : 0;
    const bool staged = n - s0 <= stage_cap;
    if (staged) {
        for (uint64_t i = s0 + tid; i < n; i += kSdNT) sh[i - s0] = g[i];
        __syncthreads();
    }
    const SdHist H{staged ? sh : g, staged ? s0 : 0};

    uint32_t best_len = 0;
    uint64_t cont = 0;
    bool ok = false;
    if (!anchored) {
        // propose (speculative.cpp:28-113)
        if (k != 0 && min_match != 0 && n > min_match) {
            const uint64_t maxp = n - 1 < kSdMaxPattern ? n - 1 : kSdMaxPattern;
            unsigned long long cand = 0ull;
            if (n - min_match - 1 >= ws) {
                for (uint64_t pos = ws + tid; pos <= n - min_match - 1; pos += kSdNT) {
                    const uint64_t L = maxp < n - 1 - pos ? maxp : n - 1 - pos;
                    uint64_t m = 0;
                    while (m < L && H[pos + L - 1 - m] == H[n - 1 - m]) ++m;
                    if (m >= min_match) {
                        const unsigned long long c = (static_cast<unsigned long long>(m) << 32) | pos;
                        cand = c > cand ? c : cand;
                    }
                }
            }
            cand = block_max(cand, red);
            if (cand != 0ull) {
                best_len = static_cast<uint32_t>(cand >> 32);
                const uint64_t pos = cand & 0xFFFFFFFFull;
                cont = pos + (maxp < n - 1 - pos ? maxp : n - 1 - pos);
            }
            // exact tail matches, longest first (speculative.cpp:66-90): one pass over the positions
            // tests every length (the first token of each tail is held in a register), then the
            // longest length with a match takes its most recent position
            if (best_len < min_match && maxp >= min_match) {
                int32_t first[kSdMaxPattern + 1];
                uint32_t hit[kSdMaxPattern + 1];  // per length: position + 1 of the most recent match
#pragma unroll
                for (uint32_t len = 1; len <= kSdMaxPattern; ++len) {
                    first[len] = len <= maxp ? H[n - len] : 0;
                    hit[len] = 0u;
                }
                for (uint64_t pos = ws + tid; pos + min_match < n; pos += kSdNT) {
                    const int32_t h0 = H[pos];
#pragma unroll
                    for (uint32_t len = 1; len <= kSdMaxPattern; ++len) {
                        if (len < min_match || len > maxp || pos + len >= n || h0 != first[len]) continue;
                        uint64_t i = 1;
                        while (i < len && H[pos + i] == H[n - len + i]) ++i;
                        if (i == len) hit[len] = static_cast<uint32_t>(pos + 1);  // positions rise per thread
                    }
                }
                __shared__ uint32_t hred[kSdNT / 32][kSdMaxPattern + 1];
                const int w = tid >> 5, lane = tid & 31;
#pragma unroll
                for (uint32_t len = 1; len <= kSdMaxPattern; ++len) {
                    const uint32_t m = __reduce_max_sync(0xFFFFFFFFu, hit[len]);
                    if (lane == 0) hred[w][len] = m;
                }
                __syncthreads();
                for (uint64_t len = maxp; len >= min_match; --len) {
                    uint32_t m = 0u;
                    for (int q = 0; q < kSdNT / 32; ++q) m = hred[q][len] > m ? hred[q][len] : m;
                    if (m != 0u) {
                        best_len = static_cast<uint32_t>(len);
                        cont = (m - 1) + len;
                        break;
                    }
                    if (len == min_match) break;
                }
            }
            ok = best_len >= min_match && cont < n;
        }
    } else {
        // propose_anchored (speculative.cpp:115-176)
        if (k != 0 && n >= 2) {
            const uint64_t min_total = (min_match + 1u) > 2u ? min_match + 1u : 2u;
            const uint64_t max_total = n < kSdMaxPattern ? n : kSdMaxPattern;
            unsigned long long cand = 0ull;
            for (uint64_t pos = ws + tid; pos <= n - 1; pos += kSdNT) {
                if (H[pos] != anchor || pos + 1 >= n) continue;
                uint64_t m = 1;
                const uint64_t max_here = max_total < pos + 1 ? max_total : pos + 1;
                while (m < max_here && H[pos - m] == H[n - m]) ++m;
                if (m >= min_total) {
                    const unsigned long long c = (static_cast<unsigned long long>(m) << 32) | pos;
                    cand = c > cand ? c : cand;
                }
            }
            cand = block_max(cand, red);
            if (cand != 0ull) {
                best_len = static_cast<uint32_t>(cand >> 32);
                cont = (cand & 0xFFFFFFFFull) + 1;
            }
            ok = cand != 0ull && best_len >= min_total && cont < n;
        }
    }
    if (tid == 0) out_match[s] = ok ? static_cast<int32_t>(best_len) : 0;
    const uint64_t span = n - cont;
    for (uint32_t i = tid; i < k; i += kSdNT) out_drafts[static_cast<uint64_t>(s) * k + i] = ok ? H[cont + (i % span)] : -1;
}

}  // namespace

cudaError_t launch_suffix_draft(const int32_t* hist, const int64_t* off, uint32_t n_streams, uint32_t min_match,
                                uint32_t window, const int32_t* anchors, uint32_t k, int32_t* out_drafts,
                                int32_t* out_match, cudaStream_t stream) {
    if (n_streams == 0) return cudaSuccess;
    if (n_streams > 0x7FFFFFFFu) return cudaErrorInvalidValue;  // grid limit
    // the staged span is at most window + 16 tokens (and the history itself)
    const uint64_t span = static_cast<uint64_t>(window) + kSdMaxPattern;
    const uint32_t cap_tokens = kSdStageMax / 4u;
    const uint32_t stage_cap = span <= cap_tokens ? static_cast<uint32_t>(span) : 0u;
    static std::atomic<uint64_t> ready{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = 1ull << (dev & 63);
    if (!(ready.load(std::memory_order_acquire) & bit)) {
        e = cudaFuncSetAttribute(suffix_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kSdStageMax));
        if (e != cudaSuccess) return e;
        ready.fetch_or(bit, std::memory_order_acq_rel);
    }
    suffix_kernel<<<n_streams, kSdNT, 4u * stage_cap, stream>>>(hist, off, min_match, window, anchors, k, stage_cap,
                                                                 out_drafts, out_match);
    return cudaGetLastError();
}

}  // namespace sixi_b200
