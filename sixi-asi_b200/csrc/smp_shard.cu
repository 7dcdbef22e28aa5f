// smp_shard.cu - vocab-sharded mode: per-shard candidates (stage 1) and the merge (stage 2) behind
// sixi_smp_shard_candidates / sixi_smp_merge_shards (include/sixi_smp.h).
//
// Stage 1 runs on every rank over its slice [vocab_offset, vocab_offset + shard_vocab) of each
// row: mask, NaN/Inf check and penalties exactly as the single-device path (the engine's rules,
// src/core/core_execution.cpp:459-492, plus the per-occurrence frequency extension), then the
// shard's best top_n candidates (adjusted logit desc, id asc), the shard maximum, the sum of
// exp((x - max) / T) over the shard and the allowed count. Stage 2 runs identically on every rank
// after an all-gather of stage 1's outputs: it merges the shard lists by rank and reproduces the
// engine's selection (core_execution.cpp:507-601: top-k, fp64 softmax, top-p with the crossing
// token kept, renormalisation, CDF draw; min-p as in the single-device path) on the merged list.
// The merged list is exact down to the worst listed entry of any shard whose list was truncated
// (the certified prefix); a row whose top-k, top-p, min-p or draw decision falls beyond it reports
// SIXI_OUT_OF_BOUNDS. With top_k <= top_n every row is exact.
#include <cuda_runtime.h>

#include <atomic>
#include <cfloat>
#include <cstdint>

#include "../../include/sixi_smp.h"
#include "smp_device.cuh"
#include "smp_kernels.cuh"

namespace sixi_b200 {
namespace {

constexpr int kSh = 512;                 // threads of the shard and merge blocks
constexpr int kShW = kSh / 32;
constexpr uint32_t kCollectCap = 4096;   // candidates collected per row before ranking
constexpr uint32_t kMaxMerge = 1024;     // n_shards * top_n handled by one merge block
constexpr int kUnroll = 8;               // global loads in flight per thread in stage 1's loops

struct ShardShared {
    unsigned long long red[kShW];
    double redd[kShW];
    uint32_t red32[kShW];
    unsigned long long bc[4];
    uint32_t fill;
    uint32_t flags;
};

__device__ __forceinline__ bool bit_allowed(const uint32_t* mask, uint32_t gid) {
    return mask == nullptr || ((mask[gid >> 5] >> (gid & 31)) & 1u);
}

__device__ __forceinline__ float shard_logit(const ShardArgs& a, const uint8_t* row, uint32_t e) {
    if (a.dtype == SIXI_SMP_BF16)
        return __uint_as_float(static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(row)[e]) << 16);
    return reinterpret_cast<const float*>(row)[e];
}

// The engine's unique-token penalty, then the frequency penalty once per occurrence (identical
// fp32 operations, in the same order as the single-device path).
__device__ __forceinline__ float penalize_count(float v, const sixi_smp_params& p, uint32_t count) {
    if (p.repetition_penalty != 1.0f && p.repetition_penalty > 0.0f)
        v = (v < 0.0f) ? __fmul_rn(v, p.repetition_penalty) : __fdiv_rn(v, p.repetition_penalty);
    v = __fsub_rn(v, p.presence_penalty);
    if (p.frequency_penalty != 0.0f)
        for (uint32_t i = 0; i < count; ++i) v = __fsub_rn(v, p.frequency_penalty);
    return v;
}

__device__ __forceinline__ unsigned long long blk_max(unsigned long long v, ShardShared* sh) {
    v = warp_max_u64(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sh->red[threadIdx.x >> 5] = v;
    __syncthreads();
    unsigned long long m = 0ull;
#pragma unroll
    for (int i = 0; i < kShW; ++i) m = sh->red[i] > m ? sh->red[i] : m;
    return m;
}
__device__ __forceinline__ uint32_t blk_sum32(uint32_t v, ShardShared* sh) {
    v = warp_sum_u32(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sh->red32[threadIdx.x >> 5] = v;
    __syncthreads();
    uint32_t s = 0u;
#pragma unroll
    for (int i = 0; i < kShW; ++i) s += sh->red32[i];
    return s;
}
__device__ __forceinline__ double blk_sumd(double v, ShardShared* sh) {
    v = warp_sum_f64(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sh->redd[threadIdx.x >> 5] = v;
    __syncthreads();
    double s = 0.0;
#pragma unroll
    for (int i = 0; i < kShW; ++i) s += sh->redd[i];
    return s;
}

// ------------------------------------------------------------------------------------------ stage 1
// One block per row. Shared memory: per-id history counts of the slice (16 bits each), the
// collected candidates and the per-thread maxima.
__global__ void __launch_bounds__(kSh, 1) shard_kernel(const ShardArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    ShardShared* sh = reinterpret_cast<ShardShared*>(smem);
    uint32_t* cnt = reinterpret_cast<uint32_t*>(smem + ((sizeof(ShardShared) + 15) / 16) * 16);
    const uint32_t cnt_words = (a.shard_vocab + 1u) / 2u;
    unsigned long long* list = reinterpret_cast<unsigned long long*>(cnt + ((cnt_words + 3u) / 4u) * 4u);
    unsigned long long* tmax = list + kCollectCap;
    const int tid = threadIdx.x;
    const uint32_t row = blockIdx.x;
    const sixi_smp_params P = a.params[row];
    const uint8_t* rowp = static_cast<const uint8_t*>(a.data) +
                          static_cast<size_t>(row) * a.row_stride * (a.dtype == SIXI_SMP_BF16 ? 2 : 4);
    const uint32_t* mask = (a.mask != nullptr && (P.flags & SIXI_SMP_ROW_MASKED))
                               ? a.mask + static_cast<size_t>(row) * a.mask_words
                               : nullptr;
    int64_t h0 = 0, h1 = 0;
    if (a.hist != nullptr) {
        h0 = a.hist_off[row];
        h1 = a.hist_off[row + 1];
    }
    const bool pen = P.mode != SIXI_SMP_STRICT_REPLAY && h1 > h0 &&
                     (P.repetition_penalty != 1.0f || P.presence_penalty != 0.0f || P.frequency_penalty != 0.0f);
    if (tid == 0) {
        sh->fill = 0u;
        sh->flags = 0u;
    }
    for (uint32_t i = tid; i < cnt_words; i += kSh) cnt[i] = 0u;
    __syncthreads();
    if (pen) {
        if (P.frequency_penalty != 0.0f && h1 - h0 > 65535) {
            if (tid == 0) sh->flags |= 2u;  // a count could pass 16 bits
        }
        for (int64_t j0 = h0 + tid; j0 < h1; j0 += kUnroll * kSh) {  // kUnroll loads in flight
            int32_t t8[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int64_t j = j0 + static_cast<int64_t>(u) * kSh;
                t8[u] = j < h1 ? a.hist[j] : -1;
            }
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int32_t t = t8[u];
                if (t < static_cast<int32_t>(a.vocab_offset) ||
                    t >= static_cast<int32_t>(a.vocab_offset + a.shard_vocab) ||
                    !bit_allowed(mask, static_cast<uint32_t>(t)))
                    continue;
                const uint32_t e = static_cast<uint32_t>(t) - a.vocab_offset;
                atomicAdd(&cnt[e >> 1], 1u << (16u * (e & 1u)));
            }
        }
    }
    __syncthreads();
    auto adjusted = [&](uint32_t e, float raw) -> float {
        if (!pen) return raw;
        const uint32_t c = (cnt[e >> 1] >> (16u * (e & 1u))) & 0xFFFFu;
        return c ? penalize_count(raw, P, c) : raw;
    };
    // pass 1: checks, allowed count, per-thread maxima of the composite (key, id)
    uint32_t n_al = 0u;
    unsigned long long best = 0ull;
    bool bad = false;
    for (uint32_t e0 = tid; e0 < a.shard_vocab; e0 += kUnroll * kSh) {  // kUnroll loads in flight
        float x8[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const uint32_t e = e0 + u * kSh;
            x8[u] = e < a.shard_vocab ? shard_logit(a, rowp, e) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const uint32_t e = e0 + u * kSh;
            const uint32_t gid = a.vocab_offset + e;
            if (e >= a.shard_vocab || !bit_allowed(mask, gid)) continue;
            const float raw = x8[u];
            bad |= !isfinite(raw);
            ++n_al;
            const unsigned long long c = comp_of(fkey(adjusted(e, raw)), gid);
            best = c > best ? c : best;
        }
    }
    tmax[tid] = best;
    const uint32_t n_allowed = blk_sum32(n_al, sh);
    if (bad) atomicOr(&sh->flags, 1u);
    const unsigned long long gbest = blk_max(best, sh);
    int32_t status = SIXI_OK;
    if (sh->flags & 1u) status = SIXI_NUMERIC_NAN_OR_INF;
    else if (sh->flags & 2u) status = SIXI_OUT_OF_BOUNDS;
    const uint32_t top_n = a.top_n;
    ShardCand* outc = a.out_cand + static_cast<size_t>(row) * top_n;
    if (status != SIXI_OK || n_allowed == 0u) {
        for (uint32_t i = tid; i < top_n; i += kSh) outc[i] = ShardCand{-INFINITY, -1};
        if (tid == 0) a.out_stats[row] = ShardStats{-INFINITY, static_cast<int32_t>(n_allowed), 0.0, status, 0};
        return;
    }
    // threshold: the top_n-th largest per-thread maximum bounds the shard's top_n from below
    unsigned long long theta = 1ull;
    {
        uint32_t nz = blk_sum32(best != 0ull ? 1u : 0u, sh);
        if (nz >= top_n) {
            uint32_t r = 0u;
            for (int j = 0; j < kSh; ++j) r += tmax[j] > best ? 1u : 0u;
            if (best != 0ull && r == top_n - 1u) sh->bc[0] = best;
            __syncthreads();
            theta = sh->bc[0];
        }
    }
    // pass 2: collect the candidates >= theta; the sum of exp((x - max) / T) over the shard
    const float xmax = kval(comp_key(gbest));
    const bool sampled = P.temperature > 0.0f;
    WeightCtx wc{};
    if (sampled) make_weight_ctx(P.temperature, xmax, 46.0f, wc);
    double se = 0.0;
    for (uint32_t e0 = tid; e0 < a.shard_vocab; e0 += kUnroll * kSh) {  // kUnroll loads in flight
        float x8[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const uint32_t e = e0 + u * kSh;
            x8[u] = e < a.shard_vocab ? shard_logit(a, rowp, e) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const uint32_t e = e0 + u * kSh;
            const uint32_t gid = a.vocab_offset + e;
            if (e >= a.shard_vocab || !bit_allowed(mask, gid)) continue;
            const float x = adjusted(e, x8[u]);
            const unsigned long long c = comp_of(fkey(x), gid);
            if (c >= theta) {
                const uint32_t slot = atomicAdd(&sh->fill, 1u);
                if (slot < kCollectCap) list[slot] = c;
            }
            if (sampled) se += static_cast<double>(fast_ex2(fminf(neg_log2w(x, wc), 0.0f)));
        }
    }
    const double sum_exp = sampled ? blk_sumd(se, sh) : 0.0;
    uint32_t n_col = sh->fill;
    if (n_col > kCollectCap) {
        // Heavily tied rows overflow the collection: find the exact top_n-th composite by an
        // 8-bit radix select over the slice (8 more passes), then collect exactly top_n.
        unsigned long long prefix = 0ull, pmask = 0ull;
        uint32_t need = top_n;
        uint32_t* dh = reinterpret_cast<uint32_t*>(tmax);  // 256 counters (tmax is free now)
        for (int shift = 56; shift >= 0; shift -= 8) {
            __syncthreads();
            for (int i = tid; i < 256; i += kSh) dh[i] = 0u;
            __syncthreads();
            for (uint32_t e = tid; e < a.shard_vocab; e += kSh) {
                const uint32_t gid = a.vocab_offset + e;
                if (!bit_allowed(mask, gid)) continue;
                const unsigned long long c = comp_of(fkey(adjusted(e, shard_logit(a, rowp, e))), gid);
                if ((c & pmask) == prefix) atomicAdd(&dh[(c >> shift) & 255u], 1u);
            }
            __syncthreads();
            if (tid == 0) {
                uint32_t acc = 0u;
                int d = 255;
                for (; d > 0; --d) {
                    if (acc + dh[d] >= need) break;
                    acc += dh[d];
                }
                sh->bc[1] = static_cast<unsigned long long>(d);
                sh->bc[2] = acc;
            }
            __syncthreads();
            prefix |= sh->bc[1] << shift;
            pmask |= 255ull << shift;
            need -= static_cast<uint32_t>(sh->bc[2]);
        }
        theta = prefix;  // the exact top_n-th composite
        __syncthreads();
        if (tid == 0) sh->fill = 0u;
        __syncthreads();
        for (uint32_t e = tid; e < a.shard_vocab; e += kSh) {
            const uint32_t gid = a.vocab_offset + e;
            if (!bit_allowed(mask, gid)) continue;
            const unsigned long long c = comp_of(fkey(adjusted(e, shard_logit(a, rowp, e))), gid);
            if (c >= theta) list[atomicAdd(&sh->fill, 1u)] = c;  // exactly top_n entries
        }
        __syncthreads();
        n_col = sh->fill;
    }
    // rank the collected candidates (unique composites) and write the best top_n
    for (uint32_t i = tid; i < n_col; i += kSh) {
        const unsigned long long c = list[i];
        uint32_t r = 0u;
        for (uint32_t j = 0; j < n_col; ++j) r += list[j] > c ? 1u : 0u;
        if (r < top_n) outc[r] = ShardCand{kval(comp_key(c)), static_cast<int32_t>(comp_id(c))};
    }
    for (uint32_t i = n_col + tid; i < top_n; i += kSh) outc[i] = ShardCand{-INFINITY, -1};
    if (tid == 0) a.out_stats[row] = ShardStats{xmax, static_cast<int32_t>(n_allowed), sum_exp, SIXI_OK, 0};
}

// ------------------------------------------------------------------------------------------ stage 2
__device__ __forceinline__ double warp_incl_f64(double v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double t = __shfl_up_sync(0xFFFFFFFFu, v, o);
        if (lane >= o) v += t;
    }
    return v;
}

// Over merged candidates [0, n) (sorted), warp 0 finds the first index whose running sum of
// f(i) reaches `target` (>= comparison); returns n when none does. *total receives the sum over
// [0, n). Called by all 32 lanes of warp 0.
template <class F>
__device__ int warp_first_cum_ge(int n, double target, F f, double* total) {
    const int lane = threadIdx.x & 31;
    double base = 0.0;
    int found = n;
    for (int c0 = 0; c0 < n; c0 += 32) {
        const int i = c0 + lane;
        const double v = i < n ? f(i) : 0.0;
        const double cum = base + warp_incl_f64(v);
        const unsigned ball = __ballot_sync(0xFFFFFFFFu, i < n && cum >= target);
        if (found == n && ball != 0u) found = c0 + __ffs(ball) - 1;
        base = __shfl_sync(0xFFFFFFFFu, cum, 31);
    }
    *total = base;
    return found;
}
// the same with a strict comparison (u < cdf, the engine's draw)
template <class F>
__device__ int warp_first_cum_gt(int n, double u, F f) {
    const int lane = threadIdx.x & 31;
    double base = 0.0;
    for (int c0 = 0; c0 < n; c0 += 32) {
        const int i = c0 + lane;
        const double v = i < n ? f(i) : 0.0;
        const double cum = base + warp_incl_f64(v);
        const unsigned ball = __ballot_sync(0xFFFFFFFFu, i < n && u < cum);
        if (ball != 0u) return c0 + __ffs(ball) - 1;
        base = __shfl_sync(0xFFFFFFFFu, cum, 31);
    }
    return n;
}

__global__ void __launch_bounds__(kSh, 1) merge_kernel(const MergeArgs a) {
    __shared__ ShardStats st[kMaxShards];
    __shared__ unsigned long long L[kMaxMerge];   // shard lists (composites), shard-major
    __shared__ unsigned long long M[kMaxMerge];   // merged, descending
    const int tid = threadIdx.x;
    const uint32_t row = blockIdx.x;
    const uint32_t S = a.n_shards, n = a.top_n, tot = S * n;
    if (tid < static_cast<int>(S)) st[tid] = a.stats[static_cast<size_t>(tid) * a.n_rows + row];
    for (uint32_t i = tid; i < tot; i += kSh) {
        const uint32_t s = i / n, j = i % n;
        const ShardCand c = a.cand[(static_cast<size_t>(s) * a.n_rows + row) * n + j];
        L[i] = c.id >= 0 ? comp_of(fkey(c.logit), static_cast<uint32_t>(c.id)) : 0ull;
        M[i] = 0ull;
    }
    __syncthreads();
    int32_t status = SIXI_OK;
    uint64_t n_allowed = 0;
    for (uint32_t s = 0; s < S; ++s) {
        if (status == SIXI_OK && st[s].status != SIXI_OK) status = st[s].status;
        n_allowed += static_cast<uint64_t>(st[s].n_allowed > 0 ? st[s].n_allowed : 0);
    }
    if (status == SIXI_OK && n_allowed == 0) status = SIXI_INVALID_ARGUMENT;
    if (status != SIXI_OK) {
        if (tid == 0) {
            a.out_tok[row] = -1;
            a.out_status[row] = status;
        }
        return;
    }
    // merge by rank: position in its own list + entries of the other lists that are larger
    uint32_t total_listed = 0;
    for (uint32_t s = 0; s < S; ++s)
        total_listed += static_cast<uint32_t>(st[s].n_allowed) < n ? static_cast<uint32_t>(st[s].n_allowed) : n;
    for (uint32_t i = tid; i < tot; i += kSh) {
        const unsigned long long c = L[i];
        if (c == 0ull) continue;
        const uint32_t s = i / n;
        uint32_t r = i % n;
        for (uint32_t o = 0; o < S; ++o) {
            if (o == s) continue;
            const unsigned long long* lo = L + o * n;
            uint32_t a0 = 0, b0 = n;  // count of entries > c (lists are descending, zero-padded)
            while (a0 < b0) {
                const uint32_t m = (a0 + b0) >> 1;
                if (lo[m] > c) a0 = m + 1;
                else b0 = m;
            }
            r += a0;
        }
        M[r] = c;
    }
    __syncthreads();
    // certified prefix: entries at or above the worst listed entry of every truncated shard
    unsigned long long wcut = 0ull;
    for (uint32_t s = 0; s < S; ++s)
        if (static_cast<uint32_t>(st[s].n_allowed) > n && L[s * n + n - 1] > wcut) wcut = L[s * n + n - 1];
    if (tid < 32) {
        const sixi_smp_params P = a.params[row];
        int cc = static_cast<int>(total_listed);
        if (wcut != 0ull) {
            int lo = 0, hi = static_cast<int>(total_listed);  // number of entries >= wcut
            while (lo < hi) {
                const int m = (lo + hi) >> 1;
                if (M[m] >= wcut) lo = m + 1;
                else hi = m;
            }
            cc = lo;
        }
        int32_t tok = -1, rst = SIXI_OK;
        if (P.temperature <= 0.0f) {
            tok = static_cast<int32_t>(comp_id(M[0]));
        } else {
            const double u = a.uniforms != nullptr ? a.uniforms[row]
                                                   : philox_uniform(P.seed, P.counter + a.step, 0u);
            const uint64_t k = (P.top_k > 0 && static_cast<uint64_t>(P.top_k) < n_allowed)
                                   ? static_cast<uint64_t>(P.top_k)
                                   : n_allowed;
            const double inv_temp = 1.0 / static_cast<double>(P.temperature);
            const double max_scaled = static_cast<double>(kval(comp_key(M[0]))) * inv_temp;
            auto ex = [&](int i) { return exp(static_cast<double>(kval(comp_key(M[i]))) * inv_temp - max_scaled); };
            double z = 0.0;
            int avail;  // candidates whose probabilities are known exactly
            if (k <= static_cast<uint64_t>(cc)) {
                avail = static_cast<int>(k);
                warp_first_cum_ge(avail, 2.0, ex, &z);  // sum over the k candidates
            } else if (k == n_allowed) {
                avail = cc;
                for (uint32_t s = 0; s < S; ++s)  // the whole slice's mass, rescaled to the row max
                    if (st[s].n_allowed > 0)
                        z += st[s].sum_exp * exp(static_cast<double>(st[s].max) * inv_temp - max_scaled);
            } else {
                avail = -1;
                rst = SIXI_OUT_OF_BOUNDS;  // top_k > top_n on a truncated merge
            }
            if (avail >= 0) {
                const bool all_known = k <= static_cast<uint64_t>(cc);
                int keep = all_known ? avail : -1;  // -1: kept set reaches past the known prefix
                double kept = 1.0;                   // mass of the kept set in units of p
                auto pr = [&](int i) { return ex(i) / z; };
                if (P.top_p > 0.0f && P.top_p < 1.0f) {
                    double t;
                    const int f = warp_first_cum_ge(avail, static_cast<double>(P.top_p), pr, &t);
                    if (f < avail) {
                        keep = f + 1;
                    } else if (!all_known) {
                        rst = SIXI_OUT_OF_BOUNDS;
                    }
                    if (keep >= 0 && keep < static_cast<int>(k)) warp_first_cum_ge(keep, 2.0, pr, &kept);
                }
                if (rst == SIXI_OK && P.min_p > 0.0f) {
                    const double thr = static_cast<double>(P.min_p) * (pr(0) / kept);
                    const int lim = keep >= 0 ? keep : avail;
                    int cut = lim;
                    for (int c0 = 1; c0 < lim; c0 += 32) {
                        const int i = c0 + (tid & 31);
                        const unsigned ball = __ballot_sync(0xFFFFFFFFu, i < lim && pr(i) / kept < thr);
                        if (ball != 0u) {
                            cut = c0 + __ffs(ball) - 1;
                            break;
                        }
                    }
                    if (cut < lim) {
                        keep = cut;
                        double nk;
                        warp_first_cum_ge(keep, 2.0, pr, &nk);
                        kept = nk;
                    } else if (keep < 0) {
                        rst = SIXI_OUT_OF_BOUNDS;
                    }
                }
                if (rst == SIXI_OK) {
                    const int lim = keep >= 0 ? keep : avail;
                    const int f = warp_first_cum_gt(lim, u, [&](int i) { return pr(i) / kept; });
                    if (f < lim) tok = static_cast<int32_t>(comp_id(M[f]));
                    else if (keep >= 0) tok = static_cast<int32_t>(comp_id(M[keep - 1]));  // last kept
                    else rst = SIXI_OUT_OF_BOUNDS;
                }
            }
        }
        if (tid == 0) {
            a.out_tok[row] = rst == SIXI_OK ? tok : -1;
            a.out_status[row] = rst;
        }
    }
}

}  // namespace

size_t shard_smem_bytes(uint32_t shard_vocab) {
    const size_t head = ((sizeof(ShardShared) + 15) / 16) * 16;
    const size_t cnt_words = (shard_vocab + 1u) / 2u;
    return head + ((cnt_words + 3u) / 4u) * 4u * 4u + (kCollectCap + kSh) * 8u;
}

cudaError_t launch_shard_candidates(const ShardArgs& a, cudaStream_t stream) {
    const size_t smem = shard_smem_bytes(a.shard_vocab);
    static std::atomic<uint64_t> ready{0};  // attribute set once per device (the maximum)
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(ready.load(std::memory_order_acquire) & bit)) {
        cudaError_t e = cudaFuncSetAttribute(shard_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kMaxShardSmem));
        if (e != cudaSuccess) return e;
        ready.fetch_or(bit, std::memory_order_acq_rel);
    }
    shard_kernel<<<a.n_rows, kSh, smem, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_merge_shards(const MergeArgs& a, cudaStream_t stream) {
    merge_kernel<<<a.n_rows, kSh, 0, stream>>>(a);
    return cudaGetLastError();
}

namespace {

// dst row j = the first `width` elements of src row index[j] (element size 2 or 4 bytes);
// blockIdx.y picks the row, the x blocks stride over its elements
template <typename T>
__global__ void gather_rows_kernel(const T* __restrict__ src, uint64_t src_stride, const int32_t* __restrict__ index,
                                   uint32_t width, T* __restrict__ dst, uint64_t dst_stride) {
    const uint32_t j = blockIdx.y;
    const T* s = src + static_cast<uint64_t>(index[j]) * src_stride;
    T* d = dst + static_cast<uint64_t>(j) * dst_stride;
    for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < width; e += gridDim.x * blockDim.x) d[e] = s[e];
}

}  // namespace

cudaError_t launch_gather_rows(const void* src, uint64_t src_stride, uint32_t esz, const int32_t* index, uint32_t n,
                               uint32_t width, void* dst, uint64_t dst_stride, cudaStream_t stream) {
    if (n == 0 || width == 0) return cudaSuccess;
    if (n > 65535u) return cudaErrorInvalidValue;  // one grid row per gathered row
    const dim3 grid((width + 1023u) / 1024u < 32u ? (width + 1023u) / 1024u : 32u, n);
    if (esz == 2)
        gather_rows_kernel<uint16_t><<<grid, 256, 0, stream>>>(static_cast<const uint16_t*>(src), src_stride, index,
                                                                width, static_cast<uint16_t*>(dst), dst_stride);
    else
        gather_rows_kernel<uint32_t><<<grid, 256, 0, stream>>>(static_cast<const uint32_t*>(src), src_stride, index,
                                                                width, static_cast<uint32_t*>(dst), dst_stride);
    return cudaGetLastError();
}

}  // namespace sixi_b200
