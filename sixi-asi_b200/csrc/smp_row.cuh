#pragma once
// smp_row.cuh - the B200 (sm_100a) row engine behind sixi_smp_sample / _candidates /
// _greedy_argmax / _verify.
//
// One cluster of C CTAs (C = 1..16, chosen per vocabulary and batch) owns one logits row. CTA c
// bulk-copies (TMA, cp.async.bulk) its contiguous chunk of the row from HBM into shared memory in
// kStages pipelined stages and converts each stage in place into 32-bit monotone keys while the
// next stages are still in flight, applying the grammar mask, the NaN/Inf check and the
// repetition/presence penalties on the way. From then on every step (argmax, top-k, softmax mass,
// top-p / min-p crossing, the draw, the verifier's accept test and residual) runs over the
// shared-memory-resident keys with compact loops, block reductions and DSMEM exchanges inside the
// cluster. HBM is read exactly once per row: the path is bandwidth-bound and uses no tensor cores.
//
// Reference semantics (Sixi-ASI engine):
//   DeterministicSampler::sample_greedy_argmax        src/core/core_execution.cpp:394-407
//   DeterministicSampler::compute_sampling_candidates  src/core/core_execution.cpp:449-584
//   DeterministicSampler::sample_from_candidates       src/core/core_execution.cpp:586-601
//   DeterministicSampler::sample_token                 src/core/core_execution.cpp:603-619
//   SpeculativeDecoder::step verification              src/speculative/speculative.cpp:589-692, 801-916
//
// Two selection paths:
//   * list path (k <= kKS candidates): before the first cluster barrier each CTA selects its
//     local top-k superset (a histogram of per-thread maxima bounds it), rank-sorts it and pushes
//     the best k into CTA 0's shared memory. CTA 0 merges the sorted lists and reproduces the
//     engine's fp64 softmax over the k candidates, top-p, renormalisation and CDF draw (same
//     per-element operations; sums are parallel, so they differ only by fp64 rounding).
//   * mass path (top_k = 0 or k > kKS): an exp-domain histogram of fixed-point weights is reduced
//     over the cluster, then the crossing bin of each selection (k boundary, top-p, draw,
//     residual) is gathered into every CTA and resolved exactly by a radix select over the unique
//     (key, id) composites; bins too full to gather are refined by key digits across the cluster.
//     Integer masses make every CTA reach identical decisions.
//
// Cluster barriers: every cluster.sync() sits at the top level of the kernel, and whether a CTA
// reaches the next one depends only on data every CTA of the cluster holds identically (the
// exchanged row statistics, the assembled histograms, gathered sets and pushed partial results),
// so all CTAs of a cluster take the same barriers. The only waits the kernel spins on (the
// mbarriers of its own bulk copies) are bounded and report SIXI_BACKEND_ERROR on expiry.
#include <cooperative_groups.h>

#include <cfloat>
#include <climits>

#include "smp_device.cuh"
#include "smp_kernels.cuh"

namespace cg = cooperative_groups;

namespace sixi_b200 {

constexpr int kNT = 512;        // threads per CTA
constexpr int kNW = kNT / 32;   // warps per CTA
constexpr int kCMax = 16;       // largest cluster
constexpr int kKS = 256;        // max candidates of the list path
constexpr int kLCap = 1536;     // local candidate superset capacity
constexpr int kGCap = 1536;     // gathered-bin capacity
constexpr int kTB = 2048;       // bins of the per-thread-maximum histogram
constexpr int kStages = 4;      // bulk-copy pipeline stages per chunk
constexpr int kVecMax = 5;      // 16-byte vectors per thread per stage (bound, see plan)
constexpr int kMaxRounds = 48;  // bound on the mass path's exchange rounds (normally 2-5)
constexpr uint32_t kSmallSelect = kNT;  // selections over at most this many entries rank directly
constexpr uint32_t kWaitIters = 1u << 24;
constexpr uint32_t kNoList = 0xFFFFFFFFu;
constexpr int kMaxSmem = 227 * 1024;       // per-block opt-in limit of sm_100
constexpr uint32_t kMaxChunk = 37984;      // keys per CTA (148,352 bytes)

static_assert(kKS <= kNT, "list path assumes one candidate per thread");
static_assert((kMaxChunk * 4 / 16 + kStages * kNT - 1) / (kStages * kNT) <= kVecMax, "stage vectors");

// ---------------------------------------------------------------------------------------------
// shared memory layout

struct RowStat {
    unsigned long long best;  // max composite (key, id) over valid entries; 0 if none
    unsigned int min_key;     // min key over valid entries
    unsigned int n_allowed;   // allowed in-range entries
    unsigned int first;       // first allowed id (0xFFFFFFFF if none)
    unsigned int flags;       // bit 0: allowed entry NaN/Inf; bit 1: copy wait expired;
                              // bit 2: the first allowed entry is NaN (raw-argmax modes)
    unsigned int dkey;        // key of the draft token when it lies in this chunk
    unsigned int dhas;        // 1 when the draft token lies in this chunk
};

struct ClusterShared {  // written by remote CTAs of the cluster
    RowStat xs[kCMax];
    unsigned long long z[kCMax];     // partial weight sums
    unsigned long long wmin[kCMax];  // partial min-p prefix weight
    unsigned long long cnt[kCMax];   // partial counts
    unsigned long long mm[kCMax];    // refine: (min key << 32) | max key of the bin's entries
    unsigned long long rcnt[kCMax];  // refine: tie counts
    double rsum[kCMax];              // dense residual partial sums
    double psum[kCMax];              // dense fallback (p_target) partial sums
    unsigned long long rsel;         // refine: composite of the crossing tie (from its owner)
    unsigned int lcnt[kCMax];        // list path: list lengths pushed to CTA 0
    unsigned int gseg[2][kCMax];     // gather buffers: entries each source CTA wrote (may
                                     // exceed the segment, which signals an overfull bin)
    int result;                      // token sent to CTA 0 by the dense-residual owner
    int pad;
};

struct LocalShared {
    unsigned long long red[kNW * 8];
    unsigned int red32[kNW];
    unsigned long long bc[16];  // broadcast scalars
    double bcd[kNW];
    unsigned long long cge[32];  // mass path: CG at the end of each 64-bin chunk
    unsigned int lcount;        // local list fill counter
    unsigned int gfill[2];      // this CTA's fill of its segment in each gather buffer
    unsigned int pad;
    uint64_t mbar[kStages];
    sixi_smp_params prm;        // the row's parameters (read once from global memory)
};

struct Layout {
    uint32_t off_ls, off_dyn;
    // relative to off_dyn
    uint32_t off_k, off_x, off_y, off_z, off_r, off_f;
    uint32_t seg;  // histogram bins reduced by each CTA
    uint32_t dyn_bytes, total;
};

__host__ __device__ inline uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }
__host__ __device__ inline uint32_t umax(uint32_t a, uint32_t b) { return a > b ? a : b; }

// Regions (lifetimes):
//   K  keys (staging area of the bulk copies, then the keys of the chunk; live throughout)
//   X  list path: MA, CTA 0's merge area (remote writes before CS1, read in phase B);
//      mass path: the local weight histograms HB/HA/HLO (remote reads between CS2 and CS3), then
//      CG/CGC
//   Y  phase A: history bitmap + mask words (until P0 ends), then the local list LL;
//      mass path: the local counts HC (k-bound rows, remote reads between CS2 and CS3), then the
//      two gather buffers
//   Z  phase A: per-thread-maximum histogram; later the block-select digit histograms BH/BW
//   R  reduced histogram segment (remote reads right after CS3), then the refine rounds
//      double-buffered digit histograms (remote reads, first written two rounds after CS3)
//   F  FL/FP/FQ: CTA 0's sorted candidates, probabilities and scratch
__host__ __device__ inline Layout make_layout(uint32_t chunk, uint32_t C) {
    Layout L{};
    uint32_t o = align_up(static_cast<uint32_t>(sizeof(ClusterShared)), 16);
    L.off_ls = o;
    o = align_up(o + static_cast<uint32_t>(sizeof(LocalShared)), 16);
    L.off_dyn = align_up(o, 128);
    L.seg = kABins / C;
    uint32_t w = 0;
    L.off_k = w;
    w += align_up(4u * chunk, 128);
    L.off_x = w;
    w += align_up(umax(8u * C * kKS, 12u * kABins), 128);
    L.off_y = w;
    const uint32_t bitwords = 4u * (chunk / 32u + 2u) + 4u * (chunk / 32u + 4u);
    w += align_up(umax(umax(8u * kLCap, 16u * kGCap), bitwords), 128);
    L.off_z = w;
    w += align_up(umax(4u * kTB, 4u * 256u + 8u * 256u), 128);
    L.off_r = w;
    w += align_up(umax(12u * L.seg, 6144u), 128);
    L.off_f = w;
    w += 3u * 8u * kKS;
    L.dyn_bytes = w;
    L.total = L.off_dyn + w;
    return L;
}

// ---------------------------------------------------------------------------------------------
// per-row context

struct RowCtx {
    const sixi_smp_params* p;
    const uint8_t* row;
    const uint32_t* mask;   // full-row mask words or nullptr
    const int32_t* hist;
    int64_t nh;
    const int32_t* extra;   // verify: drafts appended to the history
    int32_t n_extra;
    int32_t active;         // row has work
    int32_t vrole;          // verify: 0 draft row, 1 bonus row
    int32_t draft;          // verify draft token (draft rows), else -1
    int32_t pen;            // penalties apply
    int32_t greedy;         // temperature <= 0 (or the raw-argmax entry)
    uint32_t stream;
    uint32_t vidx;          // verify: position i within the stream
    uint32_t orow;          // row of the parameter, mask, history, uniform and output arrays
    double u_draw;          // uniform of the draw (sample/bonus) or of the residual (draft row)
    double u_accept;        // verify draft row: accept uniform
};

__device__ __forceinline__ double row_uniform(const RowArgs& a, const sixi_smp_params* p,
                                              uint64_t base, uint32_t slot) {
    if (a.uniforms != nullptr) return a.uniforms[base + slot];
    return philox_uniform(p->seed, p->counter + a.step, slot);
}

template <int MODE>
__device__ RowCtx make_row_ctx(const RowArgs& a, uint32_t row) {
    RowCtx r{};
    const size_t esz = a.dtype == SIXI_SMP_BF16 ? 2 : 4;
    r.row = static_cast<const uint8_t*>(a.data) + static_cast<size_t>(row) * a.row_stride * esz;
    r.active = 1;
    r.draft = -1;
    r.extra = nullptr;
    r.n_extra = 0;
    r.hist = nullptr;
    r.nh = 0;
    if (MODE == kModeVerify) {
        const uint32_t kp1 = a.k + 1;
        const uint32_t s = row / kp1, i = row % kp1;
        r.stream = s;
        r.vidx = i;
        r.p = &a.params[s];
        const int32_t nd = a.n_drafts ? a.n_drafts[s] : static_cast<int32_t>(a.k);
        if (nd < 0 || nd > static_cast<int32_t>(a.k) || static_cast<int32_t>(i) > nd) r.active = 0;
        r.vrole = (static_cast<int32_t>(i) == nd) ? 1 : 0;
        const int32_t* d = a.drafts + static_cast<size_t>(s) * a.k;
        if (r.active && r.vrole == 0) r.draft = d[i];
        r.greedy = r.p->temperature <= 0.0f;
        // history: base + drafts[0..i) (draft rows); bonus: base (dense q) or base + all drafts
        r.extra = d;
        r.n_extra = r.vrole == 0 ? static_cast<int32_t>(i) : ((a.q || a.qlog) ? 0 : (nd > 0 ? nd : 0));
        if (a.hist && a.hist_off) {
            r.hist = a.hist + a.hist_off[s];
            r.nh = a.hist_off[s + 1] - a.hist_off[s];
        }
        const uint64_t ubase = static_cast<uint64_t>(s) * kp1;
        if (r.active && !r.greedy) {
            if (r.vrole == 0) {
                r.u_accept = row_uniform(a, r.p, ubase, i);
                r.u_draw = row_uniform(a, r.p, ubase, i + 1);
            } else {
                r.u_draw = row_uniform(a, r.p, ubase, static_cast<uint32_t>(nd));
            }
        }
    } else {
        const uint32_t orow = (MODE == kModeSample && a.row_map != nullptr) ? a.row_map[row] : row;
        r.orow = orow;
        // the raw-argmax entry passes one default record for all rows
        r.p = (MODE == kModeGreedy) ? a.params : &a.params[orow];
        r.greedy = (MODE == kModeGreedy) ? 1 : (r.p->temperature <= 0.0f);
        if (a.hist && a.hist_off && MODE != kModeGreedy) {
            r.hist = a.hist + a.hist_off[orow];
            r.nh = a.hist_off[orow + 1] - a.hist_off[orow];
        }
        if (MODE == kModeSample && !r.greedy) r.u_draw = row_uniform(a, r.p, orow, 0);
    }
    if (MODE == kModeVerify) r.orow = row;
    if (a.mask != nullptr && (MODE == kModeGreedy || (r.p->flags & SIXI_SMP_ROW_MASKED))) {
        r.mask = a.mask + static_cast<size_t>(r.orow) * a.mask_words;
    } else {
        r.mask = nullptr;
    }
    const bool raw_argmax = (MODE == kModeGreedy) || (MODE == kModeVerify && r.greedy);
    r.pen = !raw_argmax && r.p->mode != SIXI_SMP_STRICT_REPLAY && (r.nh + r.n_extra) > 0 &&
            (r.p->repetition_penalty != 1.0f || r.p->presence_penalty != 0.0f ||
             r.p->frequency_penalty != 0.0f);
    return r;
}

__device__ __forceinline__ int32_t hist_at(const RowCtx& r, int64_t j) {
    return j < r.nh ? r.hist[j] : r.extra[j - r.nh];
}

// repetition / presence penalty of one logit (core_execution.cpp:482-488), IEEE fp32 operations
__device__ __forceinline__ float penalize(float v, const sixi_smp_params* p) {
    const float rep = p->repetition_penalty;
    if (rep != 1.0f && rep > 0.0f) v = (v < 0.0f) ? __fmul_rn(v, rep) : __fdiv_rn(v, rep);
    return __fsub_rn(v, p->presence_penalty);
}

// block-wide helpers (all threads call) -------------------------------------------------------

__device__ __forceinline__ double block_sum_f64(double v, LocalShared* ls) {
    v = warp_sum_f64(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) ls->bcd[threadIdx.x >> 5] = v;
    __syncthreads();
    double s = 0.0;
#pragma unroll
    for (int w = 0; w < kNW; ++w) s += ls->bcd[w];
    __syncthreads();
    return s;
}

// inclusive prefix over threads (thread order); returns the block total in *tot
__device__ __forceinline__ double block_incl_f64(double v, LocalShared* ls, double* tot) {
    const double inc = warp_incl_f64(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 31) ls->bcd[threadIdx.x >> 5] = inc;
    __syncthreads();
    double before = 0.0, all = 0.0;
#pragma unroll
    for (int w = 0; w < kNW; ++w) {
        const double t = ls->bcd[w];
        before += (w < static_cast<int>(threadIdx.x >> 5)) ? t : 0.0;
        all += t;
    }
    __syncthreads();
    *tot = all;
    return before + inc;
}

__device__ __forceinline__ unsigned long long block_min_bc(unsigned long long v, LocalShared* ls) {
    return block_min_u64<kNT>(v, ls->red);
}

// warp-aggregated reservation of `n` slots (per lane) in a counter; returns the lane's first slot
__device__ __forceinline__ uint32_t warp_reserve(uint32_t n, unsigned int* counter) {
    const int lane = threadIdx.x & 31;
    const uint32_t incl = warp_incl_u32(n);
    const uint32_t total = __shfl_sync(0xFFFFFFFFu, incl, 31);
    uint32_t base = 0;
    if (lane == 31 && total > 0) base = atomicAdd(counter, total);
    base = __shfl_sync(0xFFFFFFFFu, base, 31);
    return base + incl - n;
}

// ---------------------------------------------------------------------------------------------
// The selection below for at most 32 entries in total (block-wide call, one warp works): lane i
// takes the i-th entry, ranks come from 32 shuffles, the entries are put in order through a
// shared scratch and one warp prefix sum finds the crossing; a single barrier publishes the
// result. Same contract as block_select.
__device__ __forceinline__ unsigned long long block_select_tiny(const unsigned long long* g, const unsigned int* cnt,
                                                               uint32_t C, uint32_t seg,
                                                               unsigned long long target, const WeightCtx wc,
                                                               bool weighted, unsigned long long lowb,
                                                               unsigned long long excl, LocalShared* ls,
                                                               unsigned long long* cum_through) {
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        uint32_t t = static_cast<uint32_t>(lane), q = 0;
        for (; q < C; ++q) {
            if (t < cnt[q]) break;
            t -= cnt[q];
        }
        unsigned long long e = 0ull;
        if (q < C) {
            e = g[q * seg + t];
            if (e < lowb || e == excl) e = 0ull;  // 0 sorts below every entry and weighs nothing
        }
        const unsigned long long w = e ? (weighted ? weight_of(kval(comp_key(e)), wc) : 1ull) : 0ull;
        // rank among the first `n` lanes (the others hold 0 and weigh nothing): the entries get
        // distinct ranks below n; zeros may share ranks, which only ever write zeros
        uint32_t n = 0;
        for (uint32_t qq = 0; qq < C; ++qq) n += cnt[qq];
        uint32_t rank = 0;
        for (uint32_t j = 0; j < n; ++j) {
            const unsigned long long o = __shfl_sync(0xFFFFFFFFu, e, static_cast<int>(j));
            rank += (o > e || (o == e && static_cast<int>(j) < lane)) ? 1u : 0u;
        }
        unsigned long long* S = ls->red;  // 64 of its words; the other warps wait at the barrier
        S[lane] = 0ull;
        S[32 + lane] = 0ull;
        __syncwarp();
        if (rank < 32u) {
            S[rank] = e;
            S[32 + rank] = w;
        }
        __syncwarp();
        const unsigned long long es = S[lane], ws = S[32 + lane];
        const unsigned long long cum = warp_incl_u64(ws);
        const unsigned ball = __ballot_sync(0xFFFFFFFFu, ws > 0ull && cum >= target && cum - ws < target);
        const int src = ball ? __ffs(ball) - 1 : 0;
        const unsigned long long se = __shfl_sync(0xFFFFFFFFu, es, src);
        const unsigned long long sc = __shfl_sync(0xFFFFFFFFu, cum, src);
        __syncwarp();
        if (lane == 0) {
            ls->bc[3] = ball ? se : 0ull;
            ls->bc[4] = sc;
        }
    }
    __syncthreads();
    const unsigned long long sel = ls->bc[3];
    *cum_through = sel ? ls->bc[4] : 0ull;
    __syncthreads();  // ls->red and ls->bc are free again
    return sel;
}

// ---------------------------------------------------------------------------------------------
// The selection below for at most kNT entries in total (block-wide, all threads call): one entry
// per thread, compacted; its rank is the number of larger entries (a broadcast scan of the list);
// the entries are scattered into descending order and one block prefix sum of their weights finds
// the crossing. `hz` is 8 KB of scratch. Same contract as block_select.
__device__ __forceinline__ unsigned long long block_select_small(const unsigned long long* g, const unsigned int* cnt,
                                                                uint32_t C, uint32_t seg,
                                                                unsigned long long target, const WeightCtx wc,
                                                                bool weighted, unsigned long long lowb,
                                                                unsigned long long excl, uint32_t* hz,
                                                                LocalShared* ls, unsigned long long* cum_through) {
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    unsigned long long* L = reinterpret_cast<unsigned long long*>(hz);  // entries, then in order
    unsigned long long* W = L + kNT;                                    // their weights
    unsigned long long e = 0ull;
    bool valid = false;
    {
        uint32_t t = static_cast<uint32_t>(tid), q = 0;
        for (; q < C; ++q) {
            if (t < cnt[q]) break;
            t -= cnt[q];
        }
        if (q < C) {
            e = g[q * seg + t];
            valid = e >= lowb && e != excl;
        }
    }
    uint32_t n = 0;
    const uint32_t pos = block_excl_u32<kNT>(valid ? 1u : 0u, ls->red32, &n);
    const unsigned long long we = valid ? (weighted ? weight_of(kval(comp_key(e)), wc) : 1ull) : 0ull;
    if (valid) L[pos] = e;
    if (tid == 0) ls->bc[3] = 0ull;
    if (valid && (pos & 1u) == 0u && pos + 1u == n) L[n] = 0ull;  // pad the list to an even length
    __syncthreads();
    // Entries are unique: rank = number of larger entries. `tpe` threads share one entry, each
    // scanning every tpe-th pair of the list (two composites per load; the group's loads are
    // contiguous), and add their counts.
    const uint32_t tpe = n <= kNT / 8 ? 8u : (n <= kNT / 4 ? 4u : (n <= kNT / 2 ? 2u : 1u));
    uint32_t rank = 0;
    {
        const uint32_t me = static_cast<uint32_t>(tid) / tpe, part = static_cast<uint32_t>(tid) % tpe;
        const unsigned long long c = me < n ? L[me] : ~0ull;
        const uint32_t half = (n + 1u) / 2u;  // pairs
        uint32_t r = 0;
        const ulonglong2* L2 = reinterpret_cast<const ulonglong2*>(L);
        uint32_t j = part;
        for (; j + 3u * tpe < half; j += 4u * tpe) {  // four loads in flight
            const ulonglong2 v0 = L2[j], v1 = L2[j + tpe], v2 = L2[j + 2u * tpe], v3 = L2[j + 3u * tpe];
            r += (v0.x > c ? 1u : 0u) + (v0.y > c ? 1u : 0u) + (v1.x > c ? 1u : 0u) + (v1.y > c ? 1u : 0u) +
                 (v2.x > c ? 1u : 0u) + (v2.y > c ? 1u : 0u) + (v3.x > c ? 1u : 0u) + (v3.y > c ? 1u : 0u);
        }
        for (; j < half; j += tpe) {
            const ulonglong2 v = L2[j];
            r += (v.x > c ? 1u : 0u) + (v.y > c ? 1u : 0u);
        }
        for (uint32_t o = 1; o < tpe; o <<= 1) r += __shfl_xor_sync(0xFFFFFFFFu, r, o);
        // the rank of entry `me` sits in every thread of its group; hand it to the entry's owner
        // W is free until the scatter (the weights stay in registers): it carries the ranks
        if (part == 0u && me < n) reinterpret_cast<uint32_t*>(W)[me] = r;
    }
    __syncthreads();
    if (valid) rank = reinterpret_cast<const uint32_t*>(W)[pos];
    __syncthreads();
    if (valid) {
        L[rank] = e;
        W[rank] = we;
    }
    __syncthreads();
    const unsigned long long ws = (static_cast<uint32_t>(tid) < n) ? W[tid] : 0ull;
    const unsigned long long inc = warp_incl_u64(ws);
    if (lane == 31) ls->red[w] = inc;
    __syncthreads();
    unsigned long long cum = inc;
#pragma unroll
    for (int i = 0; i < kNW; ++i) cum += (i < w) ? ls->red[i] : 0ull;
    if (static_cast<uint32_t>(tid) < n && ws > 0ull && cum >= target && cum - ws < target) {
        ls->bc[3] = L[tid];  // the one entry whose prefix first reaches the target
        ls->bc[4] = cum;
    }
    __syncthreads();
    const unsigned long long sel = ls->bc[3];
    *cum_through = sel ? ls->bc[4] : 0ull;
    __syncthreads();  // ls->red and ls->bc are free again
    return sel;
}

// ---------------------------------------------------------------------------------------------
// Exact selection over a shared-memory array of unique composites (block-wide, all threads call).
// Considers entries c with c >= lowb and c != excl. Finds the first entry in descending order at
// which the running sum (count, or weight when `weighted`) reaches `target` (>= 1) and returns
// it; *cum_through receives the running sum through it. Returns 0 when the target is not reached.
// The entries are held in C segments of `seg` slots: segment q holds cnt[q] entries.
// Radix select over 8-bit digits below the entries' common prefix. `hz` is 2 x 1024 words of
// scratch: per level a digit histogram of counts and of weights in three 16/16/32-bit parts (at
// most 1536 entries, so no part can wrap), double-buffered so that a level needs two barriers.
__device__ __forceinline__ unsigned long long block_select(const unsigned long long* g, const unsigned int* cnt,
                                                  uint32_t C, uint32_t seg,
                                                  unsigned long long target, const WeightCtx wc, bool weighted,
                                                  unsigned long long lowb, unsigned long long excl,
                                                  uint32_t* hz, LocalShared* ls, unsigned long long* cum_through) {
    const int tid = threadIdx.x;
    {
        uint32_t total = 0;
        for (uint32_t q = 0; q < C; ++q) total += cnt[q];
        if (total <= 4u) {
            // a handful of entries: every thread evaluates them (the same broadcast reads), so no
            // exchange and no barrier is needed. Each entry is inserted into four registers kept in
            // descending order (no indexed array: that would live in local memory, whose L1 misses
            // cost an L2 round trip each here).
            unsigned long long e4[4] = {0ull, 0ull, 0ull, 0ull};
            for (uint32_t q = 0; q < C; ++q) {
                for (uint32_t i = 0; i < cnt[q]; ++i) {
                    unsigned long long e = g[q * seg + i];
                    e = (e >= lowb && e != excl) ? e : 0ull;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {  // insertion: e4 stays sorted, e carries the smaller
                        const unsigned long long hi = e4[j] > e ? e4[j] : e;
                        e = e4[j] > e ? e : e4[j];
                        e4[j] = hi;
                    }
                }
            }
            unsigned long long cum = 0ull, sel = 0ull, through = 0ull;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const unsigned long long w =
                    e4[i] ? (weighted ? weight_of(kval(comp_key(e4[i])), wc) : 1ull) : 0ull;
                cum += w;
                if (sel == 0ull && w > 0ull && cum >= target) {
                    sel = e4[i];
                    through = cum;
                }
            }
            *cum_through = through;
            return sel;
        }
        if (total <= 32u)
            return block_select_tiny(g, cnt, C, seg, target, wc, weighted, lowb, excl, ls, cum_through);
        if (total <= kSmallSelect)
            return block_select_small(g, cnt, C, seg, target, wc, weighted, lowb, excl, hz, ls, cum_through);
    }
    for (int i = tid; i < 1024; i += kNT) hz[i] = 0u;  // level-0 buffer
    unsigned long long andv = ~0ull, orv = 0ull;
    uint32_t cnt_l = 0;
    for (uint32_t q = 0; q < C; ++q) {
        const unsigned long long* gq = g + q * seg;
        for (uint32_t i = tid; i < cnt[q]; i += kNT) {
            const unsigned long long c = gq[i];
            if (c < lowb || c == excl) continue;
            andv &= c;
            orv |= c;
            ++cnt_l;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        andv &= __shfl_xor_sync(0xFFFFFFFFu, andv, o);
        orv |= __shfl_xor_sync(0xFFFFFFFFu, orv, o);
    }
    cnt_l = warp_sum_u32(cnt_l);
    __syncthreads();  // earlier readers of ls->red are done
    if ((tid & 31) == 0) {
        ls->red[tid >> 5] = andv;
        ls->red[kNW + (tid >> 5)] = orv;
        ls->red[2 * kNW + (tid >> 5)] = cnt_l;
    }
    __syncthreads();
    andv = ~0ull;
    orv = 0ull;
    unsigned long long ncons = 0;
#pragma unroll
    for (int w = 0; w < kNW; ++w) {
        andv &= ls->red[w];
        orv |= ls->red[kNW + w];
        ncons += ls->red[2 * kNW + w];
    }
    __syncthreads();  // ls->red is free again
    *cum_through = 0;
    if (ncons == 0) return 0ull;
    if (ncons == 1) {
        const unsigned long long w = weighted ? weight_of(kval(comp_key(andv)), wc) : 1ull;
        if (w >= target && w > 0) {
            *cum_through = w;
            return andv;
        }
        return 0ull;
    }
    const unsigned long long diff = andv ^ orv;  // non-zero: entries are unique
    int top = 63 - __clzll(static_cast<long long>(diff));
    unsigned long long pmask = (top == 63) ? 0ull : ~((2ull << top) - 1ull);
    unsigned long long prefix = andv & pmask;
    unsigned long long base = 0;
#pragma unroll 1
    for (int level = 0; level < 9 && top >= 0; ++level) {
        const int buf = level & 1;
        uint32_t* bh = hz + buf * 1024;  // counts, then weight parts c, b, a
        uint32_t* nxt = hz + (buf ^ 1) * 1024;
        const int shift = top - 7 > 0 ? top - 7 : 0;
        const int width = top - shift + 1;
        const unsigned int nd = 1u << width;
        for (int i = tid; i < 1024; i += kNT) nxt[i] = 0u;  // read last in the previous level
        for (uint32_t q = 0; q < C; ++q) {
            const unsigned long long* gq = g + q * seg;
            for (uint32_t i = tid; i < cnt[q]; i += kNT) {
                const unsigned long long c = gq[i];
                if (c < lowb || c == excl || (c & pmask) != prefix) continue;
                const unsigned int d = static_cast<unsigned int>(c >> shift) & (nd - 1u);
                atomicAdd(&bh[d], 1u);
                if (weighted) {
                    const unsigned long long w = weight_of(kval(comp_key(c)), wc);
                    const uint32_t wc0 = static_cast<uint32_t>(w) & 0xFFFFu;
                    const uint32_t wb = static_cast<uint32_t>(w >> 16) & 0xFFFFu;
                    const uint32_t wa = static_cast<uint32_t>(w >> 32);
                    if (wc0 != 0u) atomicAdd(&bh[256 + d], wc0);
                    if (wb != 0u) atomicAdd(&bh[512 + d], wb);
                    if (wa != 0u) atomicAdd(&bh[768 + d], wa);
                }
            }
        }
        __syncthreads();
        unsigned long long* bco = ls->bc + (buf ? 5 : 0);  // double-buffered broadcast slots
        if (tid < 32) {
            unsigned long long part[8];
            unsigned long long lsum = 0;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const int d = 255 - (tid * 8 + q);
                unsigned long long v = 0;
                if (d < static_cast<int>(nd)) {
                    v = weighted ? (static_cast<unsigned long long>(bh[768 + d]) << 32) +
                                 (static_cast<unsigned long long>(bh[512 + d]) << 16) + bh[256 + d]
                           : static_cast<unsigned long long>(bh[d]);
                }
                part[q] = v;
                lsum += v;
            }
            const unsigned long long incl = warp_incl_u64(lsum);
            unsigned long long run = base + incl - lsum;
            int found = -1;
            unsigned long long above = 0;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                if (found < 0 && part[q] > 0 && run + part[q] >= target) {
                    found = 255 - (tid * 8 + q);
                    above = run;
                }
                run += part[q];
            }
            const unsigned int ball = __ballot_sync(0xFFFFFFFFu, found >= 0);
            if (ball) {
                const int src = __ffs(ball) - 1;
                const int fd = __shfl_sync(0xFFFFFFFFu, found, src);
                const unsigned long long ab = __shfl_sync(0xFFFFFFFFu, above, src);
                if (tid == 0) {
                    bco[0] = static_cast<unsigned long long>(fd);
                    bco[1] = ab;
                    bco[2] = bh[fd];
                }
            } else if (tid == 0) {
                bco[0] = ~0ull;
            }
        }
        __syncthreads();
        const unsigned long long fd = bco[0];
        if (fd == ~0ull) return 0ull;
        base = bco[1];
        const unsigned long long dcnt = bco[2];  // entries with the chosen digit
        prefix |= fd << shift;
        pmask |= (static_cast<unsigned long long>(nd) - 1ull) << shift;
        if (dcnt == 1ull || shift == 0) {
            for (uint32_t q = 0; q < C; ++q) {
                const unsigned long long* gq = g + q * seg;
                for (uint32_t i = tid; i < cnt[q]; i += kNT) {
                    const unsigned long long c = gq[i];
                    if (c < lowb || c == excl || (c & pmask) != prefix) continue;
                    ls->bc[3] = c;
                }
            }
            __syncthreads();
            const unsigned long long c = ls->bc[3];
            const unsigned long long w = weighted ? weight_of(kval(comp_key(c)), wc) : 1ull;
            *cum_through = base + w;
            return c;
        }
        top = shift - 1;
    }
    return 0ull;
}

// ---------------------------------------------------------------------------------------------
// warp-level scans over kKS candidates held kPL per lane (candidate order = lane-major)

constexpr int kPL = kKS / 32;

// first candidate index whose inclusive cumulative is >= t (0xFFFFFFFF if none below n)
__device__ __forceinline__ uint32_t lane_first_cum_ge(const double (&v)[kPL], double t, uint32_t n, int lane) {
    double run = 0.0;
#pragma unroll
    for (int j = 0; j < kPL; ++j) run += v[j];
    double acc = warp_incl_f64(run) - run;
    uint32_t mine = 0xFFFFFFFFu;
#pragma unroll
    for (int j = 0; j < kPL; ++j) {
        acc += v[j];
        const uint32_t idx = lane * kPL + j;
        if (mine == 0xFFFFFFFFu && idx < n && acc >= t) mine = idx;
    }
    return __reduce_min_sync(0xFFFFFFFFu, mine);
}

// first candidate index whose inclusive cumulative is > u (the CDF draw `u < cdf`)
__device__ __forceinline__ uint32_t lane_first_cum_gt(const double (&v)[kPL], double u, uint32_t n, int lane) {
    double run = 0.0;
#pragma unroll
    for (int j = 0; j < kPL; ++j) run += v[j];
    double acc = warp_incl_f64(run) - run;
    uint32_t mine = 0xFFFFFFFFu;
#pragma unroll
    for (int j = 0; j < kPL; ++j) {
        acc += v[j];
        const uint32_t idx = lane * kPL + j;
        if (mine == 0xFFFFFFFFu && idx < n && u < acc) mine = idx;
    }
    return __reduce_min_sync(0xFFFFFFFFu, mine);
}

// renormalise the first `keep` candidates to sum 1
__device__ __forceinline__ void lane_renorm(double (&v)[kPL], uint32_t keep, int lane) {
    double s = 0.0;
#pragma unroll
    for (int j = 0; j < kPL; ++j) s += (lane * kPL + j < keep) ? v[j] : 0.0;
    const double r = warp_sum_f64(s);
    if (r > 0.0) {
#pragma unroll
        for (int j = 0; j < kPL; ++j) v[j] /= r;
    }
}

// ---------------------------------------------------------------------------------------------
// mass-path state machine

enum Stage : int {
    kStKBound = 0,  // find the k-th candidate (count select)
    kStTopP = 1,    // top-p crossing (weight select)
    kStKept = 2,    // min-p, then the verifier's accept test
    kStDraw = 3,    // the draw (weight select)
    kStResid = 4,   // one-hot residual draw without the draft (weight select)
    kStDSum = 5,    // dense residual: partial sums pushed
    kStDWait = 6,   // dense residual: CTA 0 reads the token
    kStCount = 7,   // candidates: kept count partials pushed
    kStDone = 8
};

struct GatherReq {  // the bins a round gathers: bin bA, and bins bBlo..bBhi (bBlo < 0: none)
    int bA, bufA, bBlo, bBhi, bufB;
    unsigned long long lowb;
};

constexpr int kPreBins = 4;  // bin ranges this narrow are gathered ahead of time for the draw; wider
                             // ones when their key count is bounded by the gather segment

struct LState {
    int stage;
    int pending_bin;  // bin of the pending selection (-1 none)
    int pending_kind; // 0 none, 1 gather, 2 exchange, 3 refine, 4 resolve a prefetched bin now
    int pre_lo, pre_hi;  // bins gathered ahead of time for the draw (pre_lo < 0: none), and their
    int pre_buf;         // buffer
    unsigned long long tabs;  // the draw's target as a cumulative mass from the top
    unsigned long long target;
    unsigned long long zk, zkept, kbound, xcross, excl, wexcl;
    int32_t result;
    int32_t err;
};

// Key-digit refinement of a selection whose bin holds more entries than a gather buffer (heavy
// ties, e.g. integer-valued logits): 8-bit digit histograms are combined across the cluster until
// the key is resolved, then the crossing tie is found in vocabulary-id order by its owner CTA.
struct Refine {
    int active;
    int phase;  // 0 key range exchanged, 1 digit histograms exchanged, 2 tie counts, 3 tie found
    int bin;
    int cmode;  // count (k boundary) or weight selection
    unsigned long long t;  // target within the bin
    unsigned long long lowb, excl;
    uint32_t prefix, pmask;
    int top, shift, width;
    unsigned long long above_c, above_w, tie_w;
    int buf;
};

// ---------------------------------------------------------------------------------------------

// Draft probabilities of one draft row as the verifier reads them: stored (dense q) or evaluated
// from the draft logits and their DraftStat with the engine's operations
// (compute_full_distribution, src/core/core_execution.cpp:409-447): a multiply, a subtract, exp,
// one division by the fp64 sum, rounded to float.
struct QView {
    const float* q;
    const uint8_t* lg;
    uint32_t dt;
    double inv_t, maxs, sum;
    int32_t amax, mode;
};

__device__ __forceinline__ QView q_view(const RowArgs& a, size_t qr) {
    QView v{};
    if (a.q != nullptr) {
        v.q = a.q + qr * a.row_stride;
        return v;
    }
    const DraftStat st = a.qstat[qr];
    v.lg = static_cast<const uint8_t*>(a.qlog) + qr * a.qlog_stride * (a.qlog_dtype == SIXI_SMP_BF16 ? 2u : 4u);
    v.dt = a.qlog_dtype;
    v.inv_t = st.inv_t;
    v.maxs = st.maxs;
    v.sum = st.sum;
    v.amax = st.amax;
    v.mode = st.mode;
    return v;
}

__device__ __forceinline__ float q_of(const QView& v, uint32_t i) {
    if (v.q != nullptr) return v.q[i];
    if (v.mode == 2) return 0.0f;
    if (v.mode == 1) return i == static_cast<uint32_t>(v.amax) ? 1.0f : 0.0f;
    const float x = v.dt == SIXI_SMP_BF16
                        ? __uint_as_float(static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(v.lg)[i]) << 16)
                        : reinterpret_cast<const float*>(v.lg)[i];
    return static_cast<float>(exp(__dsub_rn(__dmul_rn(static_cast<double>(x), v.inv_t), v.maxs)) / v.sum);
}

// The mass-path histogram pass (block-wide): fixed-point weights of the keys K[0, 4 * nq) in three
// 32-bit parts, w = a * 2^32 + b * 2^16 + c (a < 2^12, b, c < 2^16): with at most 2^16 keys per
// CTA none of the part sums can wrap, so the adds are fire-and-forget. Returns this thread's
// share of the min-p prefix mass (keys >= x_minp) when use_minp. Kept out of line so that the
// loop is scheduled with the whole register budget. The pass is bound by integer issue, so the
// per-key integer work is kept minimal: the adds are reductions predicated once per key (valid, and
// a non-zero low word; a zero part adds nothing), and the b, a and c parts lie at fixed offsets from
// one address (HA = HB + kABins, HLO = HB + 2 kABins); the counts (k-bound rows only) have their
// own array HC.
// (Measured at config 2, 38K keys per CTA: each integer operation added per key costs about
// 0.6 us per pass; three fewer per key took the pass from 11.2-12.2 us to 8.9-10.8 us.)
static __device__ __noinline__ unsigned long long mass_histogram(const uint32_t* K, int nq, const WeightCtx wc,
                                                          float x_minp, bool use_minp, bool need_counts,
                                                          uint32_t* HB, uint32_t* HC) {
    static_assert(kABins * 4 == 8192, "part offsets below");
    const int tid = threadIdx.x;
    const uint32_t hi_base = smem_u32(HB), hc_base = smem_u32(HC);
    unsigned long long wp = 0ull;
    const int nq8 = (nq + 1) >> 1;
    const int it8 = (nq8 + kNT - 1) / kNT;
#pragma unroll 1
    for (int m = 0; m < it8; ++m) {  // 8 keys per iteration: independent chains
        const int q = tid + m * kNT;
        if (q >= nq8) break;
        // groups q and q + nq8: a warp's 16-byte loads are contiguous (no bank conflicts)
        const uint4 va = reinterpret_cast<const uint4*>(K)[q];
        const uint4 vb = (q + nq8 < nq) ? reinterpret_cast<const uint4*>(K)[q + nq8] : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t k8[8] = {va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w};
        uint32_t am8[8], ah8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t k = k8[i];
            const float x = kval(k);
            const unsigned long long w = weight_of(x, wc);  // meaningless for k == 0 (never added)
            const uint32_t b = static_cast<uint32_t>(abin_of(x, wc));
            const uint32_t ahi = hi_base + 4u * b;
            const bool valid = k != 0u;
            am8[i] = valid ? static_cast<uint32_t>(w >> 32) : 0u;
            ah8[i] = ahi;
            // The low parts are added when the key is valid and its low word is non-zero. Keys of
            // zero weight (far below the maximum, all in the last bin) must add nothing: at low
            // temperatures they are most of the row, and adds to one address serialise.
            asm volatile(
                "{\n\t.reg .pred pk;\n\t"
                "setp.ne.u32 pk, %0, 0;\n\t"
                "setp.ne.and.u32 pk, %2, 0, pk;\n\t"
                "@pk red.shared.add.u32 [%1+16384], %3;\n\t"
                "@pk red.shared.add.u32 [%1], %4;\n\t}" ::"r"(valid ? 1u : 0u),
                "r"(ahi), "r"(static_cast<uint32_t>(w)), "r"(static_cast<uint32_t>(w) & 0xFFFFu),
                "r"(static_cast<uint32_t>(w) >> 16)
                : "memory");
            if (need_counts) {
                asm volatile(
                    "{\n\t.reg .pred pk;\n\t"
                    "setp.ne.u32 pk, %0, 0;\n\t"
                    "@pk red.shared.add.u32 [%1], 1;\n\t}" ::"r"(valid ? 1u : 0u),
                    "r"(hc_base + 4u * b)
                    : "memory");
            }
            if (use_minp) wp += (valid && x >= x_minp) ? w : 0ull;
        }
        // The high parts are non-zero only for keys within 2^-11 of the row's largest weight, so
        // in nearly every warp all eight are zero: one vote skips their reductions.
        const uint32_t any_hi = am8[0] | am8[1] | am8[2] | am8[3] | am8[4] | am8[5] | am8[6] | am8[7];
        if (__any_sync(__activemask(), any_hi != 0u)) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                asm volatile(
                    "{\n\t.reg .pred p;\n\t"
                    "setp.ne.u32 p, %1, 0;\n\t"
                    "@p red.shared.add.u32 [%0+8192], %1;\n\t}" ::"r"(ah8[i]),
                    "r"(am8[i])
                    : "memory");
            }
        }
    }
    return wp;
}

// The list path's collect pass (block-wide): appends every key >= kthr of K[0, 4 * nq) as a
// (key, id) composite to LL (unordered; slots past kLCap are counted in *lcount but not written).
// Eight keys per iteration (two 16-byte loads, contiguous across the warp), slots reserved per
// warp only where a lane holds a match; kept out of line so that the loop is scheduled with the
// whole register budget. Keys past the chunk are 0, below every threshold (kthr >= 1).
static __device__ __noinline__ void collect_scan(const uint32_t* K, int nq, uint32_t c0, uint32_t kthr,
                                                 unsigned long long* LL, unsigned int* lcount) {
    const int tid = threadIdx.x;
    const int nq8 = (nq + 1) >> 1;
    const int it8 = (nq8 + kNT - 1) / kNT;
#pragma unroll 1
    for (int m = 0; m < it8; ++m) {  // warp-uniform trip count
        const int q = tid + m * kNT;
        // key i of the iteration is element 4 q + i (i < 4) or 4 (q + nq8) + i - 4
        uint4 va = make_uint4(0u, 0u, 0u, 0u), vb = make_uint4(0u, 0u, 0u, 0u);
        if (q < nq8) va = reinterpret_cast<const uint4*>(K)[q];
        if (q < nq8 && q + nq8 < nq) vb = reinterpret_cast<const uint4*>(K)[q + nq8];
        const uint32_t k8[8] = {va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w};
        uint32_t mk = 0u;
#pragma unroll
        for (int i = 0; i < 8; ++i) mk |= (k8[i] >= kthr) ? (1u << i) : 0u;
        if (__ballot_sync(0xFFFFFFFFu, mk != 0u) == 0u) continue;
        uint32_t slot = warp_reserve(static_cast<uint32_t>(__popc(mk)), lcount);
        while (mk != 0u) {
            const int i = __ffs(mk) - 1;
            mk &= mk - 1u;
            const int e = i < 4 ? 4 * q + i : 4 * (q + nq8) + i - 4;
            if (slot < static_cast<uint32_t>(kLCap)) LL[slot] = comp_of(K[e], c0 + static_cast<uint32_t>(e));
            ++slot;
        }
    }
}

// The gather pass's scan (block-wide): pushes this CTA's keys of interval A (k - kloA < wA) and of
// interval B as (key, id) composites >= lowb (lowb != 0: k-bound rows) into its segment of gather
// buffers gA / gB in every CTA of the cluster; gfill[0..1] count them (above gseg: overfull). One
// pass of 8 keys per iteration: per key only the interval tests (touch: one test against the
// union); a warp reserves slots (local counter) only on the rare iterations where one of its lanes
// holds a match, so the remote traffic is plain stores. Keys past the chunk read as 0, which no
// interval contains. Kept out of line so that the loop is scheduled with the whole register budget
// (inline, amid the round loop's live state, it measured 0.6 us slower per config-2 step).
static __device__ __noinline__ void gather_scan(const uint32_t* K, int nq, uint32_t c0, uint32_t kloA, uint32_t wA,
                                                uint32_t kloB, uint32_t wB, bool touch, uint32_t kloU, uint32_t wU,
                                                unsigned long long lowb, unsigned long long* gA,
                                                unsigned long long* gB, uint32_t gseg, uint32_t C,
                                                unsigned int* gfill) {
    cg::cluster_group cluster = cg::this_cluster();
    const int tid = threadIdx.x;
    const bool use_lowb = lowb != 0ull;
    const int nq8 = (nq + 1) >> 1;
    const int it8 = (nq8 + kNT - 1) / kNT;
#pragma unroll 1
    for (int m = 0; m < it8; ++m) {  // warp-uniform trip count
        const int q = tid + m * kNT;
        // groups q and q + nq8 (contiguous 16-byte loads across the warp); key i of the
        // iteration is element 4 q + i (i < 4) or 4 (q + nq8) + i - 4
        uint4 va = make_uint4(0u, 0u, 0u, 0u), vb = make_uint4(0u, 0u, 0u, 0u);
        if (q < nq8) va = reinterpret_cast<const uint4*>(K)[q];
        if (q < nq8 && q + nq8 < nq) vb = reinterpret_cast<const uint4*>(K)[q + nq8];
        const uint32_t k8[8] = {va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w};
        bool hit = false;
        if (touch) {
#pragma unroll
            for (int i = 0; i < 8; ++i) hit |= k8[i] - kloU < wU;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) hit |= (k8[i] - kloA < wA) | (k8[i] - kloB < wB);
        }
        if (__ballot_sync(0xFFFFFFFFu, hit) == 0u) continue;
        uint32_t mA = 0u, mB = 0u;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            mA |= (k8[i] - kloA < wA) ? (1u << i) : 0u;
            mB |= (k8[i] - kloB < wB) ? (1u << i) : 0u;
        }
        if (__ballot_sync(0xFFFFFFFFu, (mA | mB) != 0u) == 0u) continue;
        if (use_lowb) {  // k-bound rows: drop entries below the composite bound
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int e = i < 4 ? 4 * q + i : 4 * (q + nq8) + i - 4;
                if (comp_of(k8[i], c0 + static_cast<uint32_t>(e)) < lowb) {
                    mA &= ~(1u << i);
                    mB &= ~(1u << i);
                }
            }
        }
        uint32_t pA = warp_reserve(static_cast<uint32_t>(__popc(mA)), &gfill[0]);
        uint32_t pB = warp_reserve(static_cast<uint32_t>(__popc(mB)), &gfill[1]);
        uint32_t mk = mA | mB;
        while (mk != 0u) {
            const int i = __ffs(mk) - 1;
            mk &= mk - 1u;
            const int e = i < 4 ? 4 * q + i : 4 * (q + nq8) + i - 4;
            const unsigned long long cp = comp_of(K[e], c0 + static_cast<uint32_t>(e));
            if ((mA >> i) & 1u) {
                if (pA < gseg) {
#pragma unroll 1
                    for (uint32_t dst = 0; dst < C; ++dst) cluster.map_shared_rank(gA, dst)[pA] = cp;
                }
                ++pA;
            }
            if ((mB >> i) & 1u) {
                if (pB < gseg) {
#pragma unroll 1
                    for (uint32_t dst = 0; dst < C; ++dst) cluster.map_shared_rank(gB, dst)[pB] = cp;
                }
                ++pB;
            }
        }
    }
}

template <int DT, int MODE>
__global__ void __launch_bounds__(kNT, 1) row_kernel(const RowArgs a) {
    constexpr int ESZ = (DT == SIXI_SMP_BF16) ? 2 : 4;
    constexpr int EPV = 16 / ESZ;  // input elements per 16-byte vector

    extern __shared__ __align__(128) uint8_t smem[];
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t C = cluster.num_blocks();
    const uint32_t crank = cluster.block_rank();
    const uint32_t row = blockIdx.x / C;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const Layout lay = make_layout(a.chunk, C);

    ClusterShared* cs = reinterpret_cast<ClusterShared*>(smem);
    LocalShared* ls = reinterpret_cast<LocalShared*>(smem + lay.off_ls);
    uint8_t* dyn = smem + lay.off_dyn;
    uint32_t* K = reinterpret_cast<uint32_t*>(dyn + lay.off_k);
    float* KF = reinterpret_cast<float*>(dyn + lay.off_k);
    // X
    unsigned long long* MA = reinterpret_cast<unsigned long long*>(dyn + lay.off_x);
    uint32_t* HB = reinterpret_cast<uint32_t*>(dyn + lay.off_x);  // weight sums, bits 16..31 parts
    uint32_t* HA = HB + kABins;                                      // bits 32.. parts
    uint32_t* HLO = HB + 2 * kABins;                                 // bits 0..15 parts
    unsigned long long* CG = reinterpret_cast<unsigned long long*>(dyn + lay.off_x);  // HB/HA are dead
                                                                                      // once reduced
    uint32_t* CGC = HB + 2 * kABins;  // HLO is dead once reduced
    // Y
    uint32_t* hb = reinterpret_cast<uint32_t*>(dyn + lay.off_y);
    uint32_t* mw = hb + (a.chunk / 32u + 2u);
    unsigned long long* LL = reinterpret_cast<unsigned long long*>(dyn + lay.off_y);
    unsigned long long* G0 = reinterpret_cast<unsigned long long*>(dyn + lay.off_y);
    unsigned long long* G1 = G0 + kGCap;
    uint32_t* HC = reinterpret_cast<uint32_t*>(dyn + lay.off_y);   // counts (k-bound rows)
    // Z
    uint32_t* H32 = reinterpret_cast<uint32_t*>(dyn + lay.off_z);
    uint32_t* BH = reinterpret_cast<uint32_t*>(dyn + lay.off_z);
    unsigned long long* BW = reinterpret_cast<unsigned long long*>(dyn + lay.off_z + 1024u);
    // R
    unsigned long long* R = reinterpret_cast<unsigned long long*>(dyn + lay.off_r);
    uint32_t* RC = reinterpret_cast<uint32_t*>(dyn + lay.off_r + 8u * lay.seg);
    // F
    unsigned long long* FL = reinterpret_cast<unsigned long long*>(dyn + lay.off_f);
    double* FP = reinterpret_cast<double*>(dyn + lay.off_f + 8u * kKS);
    double* FQ = reinterpret_cast<double*>(dyn + lay.off_f + 16u * kKS);

    const int32_t c0 = static_cast<int32_t>(crank * a.chunk);
    int32_t len_load = static_cast<int32_t>(a.vocab) - c0;
    if (len_load < 0) len_load = 0;
    if (len_load > static_cast<int32_t>(a.chunk)) len_load = static_cast<int32_t>(a.chunk);
    const uint8_t* gchunk = static_cast<const uint8_t*>(a.data) +
                            (static_cast<size_t>(row) * a.row_stride + static_cast<size_t>(c0)) * ESZ;

    // ======================================================================== phase A
    // The bulk copies go out first (they need only the row address); the parameters, mask words
    // and history are read while they are in flight.
    const int32_t tma_bytes = a.use_tma ? (len_load * ESZ) / 16 * 16 : 0;
    const int32_t len_t = tma_bytes / ESZ;
    const int32_t nvec = tma_bytes / 16;
    uint8_t* stg = (DT == SIXI_SMP_BF16) ? dyn + lay.off_k + 2u * a.chunk : dyn + lay.off_k;
    auto stage_vec = [&](int s) { return static_cast<int32_t>((static_cast<int64_t>(nvec) * s) / kStages); };
    if (tid == 0) {
#pragma unroll
        for (int s = 0; s < kStages; ++s) mbar_init(&ls->mbar[s], 1);
        fence_mbar_init();
        const uint64_t pol = l2_evict_first_policy();  // the row is read once
        for (int s = 0; s < kStages; ++s) {
            const int32_t b0 = stage_vec(s) * 16, b1 = stage_vec(s + 1) * 16;
            if (b1 <= b0) continue;
            mbar_arrive_expect_tx(&ls->mbar[s], static_cast<uint32_t>(b1 - b0));
            for (int32_t off = b0; off < b1; off += 32768) {
                const int32_t nb = (b1 - off) < 32768 ? (b1 - off) : 32768;
                bulk_g2s_hint(stg + off, gchunk + off, static_cast<uint32_t>(nb), &ls->mbar[s], pol);
            }
        }
        for (int q = 0; q < kCMax; ++q) {
            cs->gseg[0][q] = 0;
            cs->gseg[1][q] = 0;
        }
        cs->result = -1;
        cs->rsel = 0ull;
        ls->bc[15] = 0;
        ls->lcount = 0;
    }

    const RowCtx rc = make_row_ctx<MODE>(a, row);
    // The parameters are read from a shared copy: through the global pointer every use after a
    // barrier or a shared-memory store would be a fresh global load (an L2 round trip, as the L1
    // is mostly carved out for shared memory).
    if (tid < static_cast<int>(sizeof(sixi_smp_params) / 4))
        reinterpret_cast<uint32_t*>(&ls->prm)[tid] = reinterpret_cast<const uint32_t*>(rc.p)[tid];
    const sixi_smp_params* P = &ls->prm;
    const int32_t len = rc.active ? len_load : 0;
    const int nq = (len + 3) >> 2;  // 4-key groups of this chunk
    const int nq_iter = (nq + kNT - 1) / kNT;

    const int nbw = static_cast<int>(a.chunk / 32u + 2u);
    for (int i = tid; i < nbw; i += kNT) hb[i] = 0u;
    const uint32_t wbase = static_cast<uint32_t>(c0) >> 5;
    const int nmw = static_cast<int>(a.chunk / 32u + 4u);
    if (rc.mask != nullptr) {
        for (int i = tid; i < nmw; i += kNT) {
            const uint32_t w = wbase + static_cast<uint32_t>(i);
            mw[i] = w < a.mask_words ? rc.mask[w] : 0u;
        }
    }
    __syncthreads();
    auto allowed = [&](int32_t gid) -> bool {
        if (rc.mask == nullptr) return true;
        return (mw[(static_cast<uint32_t>(gid) >> 5) - wbase] >> (gid & 31)) & 1u;
    };
    const int64_t nht = rc.nh + rc.n_extra;
    const bool pen_smem = rc.pen && P->frequency_penalty != 0.0f;
    // unique history ids of this chunk -> bitmap (overlaps the bulk copy; 4 loads in flight)
    if (rc.pen && len > 0) {
        for (int64_t j0 = tid; j0 < nht; j0 += 4 * kNT) {
            int32_t t4[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int64_t j = j0 + u * kNT;
                t4[u] = j < nht ? hist_at(rc, j) : -1;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int32_t t = t4[u];
                if (t < c0 || t >= c0 + len || !allowed(t)) continue;
                const int32_t e = t - c0;
                atomicOr(&hb[e >> 5], 1u << (e & 31));
            }
        }
    }
    // allowed count and first allowed id of this chunk (from the mask words, not per element)
    uint32_t t_cnt = 0, t_first = 0xFFFFFFFFu;
    if (rc.mask == nullptr) {
        if (tid == 0 && len > 0) {
            t_cnt = static_cast<uint32_t>(len);
            t_first = static_cast<uint32_t>(c0);
        }
    } else {
        const int32_t w_lo = 0, w_hi = (len > 0) ? static_cast<int32_t>(((c0 + len - 1) >> 5) - wbase) : -1;
        for (int32_t i = w_lo + tid; i <= w_hi; i += kNT) {
            uint32_t w = mw[i];
            const int32_t g0 = static_cast<int32_t>((wbase + i) << 5);
            if (g0 < c0) w &= ~0u << (c0 - g0);
            if (g0 + 32 > c0 + len) w &= (c0 + len - g0) >= 32 ? ~0u : ((1u << (c0 + len - g0)) - 1u);
            t_cnt += __popc(w);
            if (w && t_first == 0xFFFFFFFFu) t_first = static_cast<uint32_t>(g0 + __ffs(w) - 1);
        }
    }
    __syncthreads();

    auto load_global = [&](int32_t e) -> float {
        if (DT == SIXI_SMP_BF16) {
            const uint16_t b = reinterpret_cast<const uint16_t*>(gchunk)[e];
            return __uint_as_float(static_cast<uint32_t>(b) << 16);
        }
        return reinterpret_cast<const float*>(gchunk)[e];
    };
    // P0: staged input -> keys, in place. Per entry: mask bit, |bits| for the NaN/Inf check,
    // -0 -> +0, monotone key, running max (first occurrence) and min. Entries in the penalty
    // bitmap are excluded from the running statistics here and fixed up sparsely afterwards.
    // (Straight-line code with register accumulators: no lambda captures of mutable state.)
    constexpr bool kRaw = (MODE == kModeGreedy) || (MODE == kModeVerify);
    const bool has_mask = rc.mask != nullptr;
    const bool use_pbits = rc.pen && !pen_smem;
    // t_mn1 tracks (smallest valid key) - 1 as an unsigned minimum, with invalid keys (0) wrapping
    // to the neutral 0xFFFFFFFF: two integer operations per entry instead of three (P0 is bound
    // by integer issue); t_mn is derived from it once P0 is done.
    uint32_t t_mk = 0u, t_mi = 0u, t_mn = 0xFFFFFFFFu, t_mn1 = 0xFFFFFFFFu, t_amax = 0u;
    bool t_bad = false;  // an allowed raw logit is NaN or infinite (modes that do not track t_amax)
    // Entries of inactive rows are never allowed (MBIT is 0 for them). AMAX: track the largest
    // |bits| (raw-argmax modes, whose NaN keys are 0, and the frequency path); elsewhere a
    // non-finite raw logit shows up in the key extremes (see t_bad).
    const uint32_t act = len > 0 ? 0xFFFFFFFFu : 0u;
#define SIXI_ADMIT(E, XV, MBIT, PBIT, KOUT, AMAX)                                             \
    {                                                                                        \
        float x_ = (XV);                                                                     \
        const bool ok_ = (MBIT);                                                             \
        if (AMAX) {                                                                          \
            const uint32_t raw_ = __float_as_uint(x_) & 0x7FFFFFFFu;                         \
            t_amax = (ok_ && raw_ > t_amax) ? raw_ : t_amax;                                 \
        }                                                                                    \
        x_ = __fadd_rn(x_, 0.0f);                                                            \
        const uint32_t b_ = __float_as_uint(x_);                                             \
        uint32_t k_ = b_ ^ (static_cast<uint32_t>(static_cast<int32_t>(b_) >> 31) | 0x80000000u); \
        if (kRaw && x_ != x_) k_ = 0u;                                                       \
        k_ = ok_ ? k_ : 0u;                                                                  \
        const uint32_t ks_ = (PBIT) ? 0u : k_;                                               \
        if (ks_ > t_mk) {                                                                    \
            t_mk = ks_;                                                                      \
            t_mi = static_cast<uint32_t>(E);                                                 \
        }                                                                                    \
        t_mn1 = min(t_mn1, ks_ - 1u);                                                        \
        (KOUT) = k_;                                                                         \
    }
    if (!pen_smem) {
        for (int s = 0; s < kStages; ++s) {
            const int32_t v0 = stage_vec(s), v1 = stage_vec(s + 1);
            if (v1 > v0) {
                if (!mbar_wait(&ls->mbar[s], 0, kWaitIters)) ls->bc[15] = 1;
            }
            if (DT == SIXI_SMP_BF16) {
                // keys overwrite the bf16 sources in place: read the whole stage first
                uint4 raw4[kVecMax];
#pragma unroll
                for (int m = 0; m < kVecMax; ++m) {
                    const int32_t v = v0 + tid + m * kNT;
                    if (v < v1) raw4[m] = *reinterpret_cast<const uint4*>(stg + 16u * v);
                }
                __syncthreads();
                // mb: the mask bits of the eight entries (all set for an active row without a mask,
                // a case written out on its own so that no mask bit is tested)
                auto admit8 = [&](const int32_t v, const uint4 r, const uint32_t mb, const bool plain) {
                    const int32_t e0 = v * 8;
                    const uint32_t pb = use_pbits ? (hb[e0 >> 5] >> (e0 & 31)) & 0xFFu : 0u;
                    const uint32_t w4[4] = {r.x, r.y, r.z, r.w};
                    uint32_t k8[8];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        SIXI_ADMIT(e0 + 2 * i, __uint_as_float(w4[i] << 16), plain ? 1u : (mb >> (2 * i)) & 1u,
                                   (pb >> (2 * i)) & 1u, k8[2 * i], kRaw);
                        SIXI_ADMIT(e0 + 2 * i + 1, __uint_as_float(w4[i] & 0xFFFF0000u),
                                   plain ? 1u : (mb >> (2 * i + 1)) & 1u, (pb >> (2 * i + 1)) & 1u, k8[2 * i + 1], kRaw);
                    }
                    *reinterpret_cast<uint4*>(K + e0) = make_uint4(k8[0], k8[1], k8[2], k8[3]);
                    *reinterpret_cast<uint4*>(K + e0 + 4) = make_uint4(k8[4], k8[5], k8[6], k8[7]);
                };
                if (!has_mask && len > 0) {
#pragma unroll
                    for (int m = 0; m < kVecMax; ++m) {
                        const int32_t v = v0 + tid + m * kNT;
                        if (v < v1) admit8(v, raw4[m], 0xFFu, true);
                    }
                } else {
#pragma unroll
                    for (int m = 0; m < kVecMax; ++m) {
                        const int32_t v = v0 + tid + m * kNT;
                        if (v < v1) {
                            const uint32_t g = static_cast<uint32_t>(c0 + v * 8);
                            admit8(v, raw4[m], (has_mask ? (mw[(g >> 5) - wbase] >> (g & 31)) & 0xFFu : 0xFFu) & act, false);
                        }
                    }
                }
                __syncthreads();
            } else if (!has_mask && len > 0) {
                // every entry allowed (no mask, active row): no mask bits to test
#pragma unroll
                for (int m = 0; m < kVecMax; ++m) {
                    const int32_t v = v0 + tid + m * kNT;
                    if (v < v1) {
                        const float4 f = *reinterpret_cast<const float4*>(stg + 16u * v);
                        const int32_t e0 = v * 4;
                        const uint32_t pb = use_pbits ? (hb[e0 >> 5] >> (e0 & 31)) & 0xFu : 0u;
                        uint32_t k0, k1, k2, k3;
                        SIXI_ADMIT(e0 + 0, f.x, 1u, pb & 1u, k0, kRaw);
                        SIXI_ADMIT(e0 + 1, f.y, 1u, (pb >> 1) & 1u, k1, kRaw);
                        SIXI_ADMIT(e0 + 2, f.z, 1u, (pb >> 2) & 1u, k2, kRaw);
                        SIXI_ADMIT(e0 + 3, f.w, 1u, (pb >> 3) & 1u, k3, kRaw);
                        *reinterpret_cast<uint4*>(K + e0) = make_uint4(k0, k1, k2, k3);
                    }
                }
            } else {
#pragma unroll
                for (int m = 0; m < kVecMax; ++m) {
                    const int32_t v = v0 + tid + m * kNT;
                    if (v < v1) {
                        const float4 f = *reinterpret_cast<const float4*>(stg + 16u * v);
                        const int32_t e0 = v * 4;
                        const uint32_t g = static_cast<uint32_t>(c0 + e0);
                        const uint32_t mb = (has_mask ? (mw[(g >> 5) - wbase] >> (g & 31)) & 0xFu : 0xFu) & act;
                        const uint32_t pb = use_pbits ? (hb[e0 >> 5] >> (e0 & 31)) & 0xFu : 0u;
                        uint32_t k0, k1, k2, k3;
                        SIXI_ADMIT(e0 + 0, f.x, mb & 1u, pb & 1u, k0, kRaw);
                        SIXI_ADMIT(e0 + 1, f.y, (mb >> 1) & 1u, (pb >> 1) & 1u, k1, kRaw);
                        SIXI_ADMIT(e0 + 2, f.z, (mb >> 2) & 1u, (pb >> 2) & 1u, k2, kRaw);
                        SIXI_ADMIT(e0 + 3, f.w, (mb >> 3) & 1u, (pb >> 3) & 1u, k3, kRaw);
                        *reinterpret_cast<uint4*>(K + e0) = make_uint4(k0, k1, k2, k3);
                    }
                }
            }
        }
        for (int32_t e = len_t + tid; e < len; e += kNT) {  // ragged tail: plain loads
            float x;
            if (DT == SIXI_SMP_BF16) {
                x = __uint_as_float(static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(gchunk)[e]) << 16);
            } else {
                x = reinterpret_cast<const float*>(gchunk)[e];
            }
            const uint32_t mb = allowed(c0 + e) ? 1u : 0u;
            const uint32_t pb = use_pbits ? (hb[e >> 5] >> (e & 31)) & 1u : 0u;
            uint32_t k;
            SIXI_ADMIT(e, x, mb, pb, k, kRaw);
            K[e] = k;
        }
        t_mn = (t_mn1 == 0xFFFFFFFFu) ? 0xFFFFFFFFu : t_mn1 + 1u;
        // raw non-finite values of the entries seen so far (penalised entries are checked below,
        // on their raw keys, before a penalty could overflow them)
        if (!kRaw) t_bad = t_mk >= 0xFF800000u || t_mn <= 0x007FFFFFu;
        if (use_pbits) {
            // sparse penalty fix-up: each set bit of the history bitmap is one unique allowed id of
            // this chunk (no second pass over the history in global memory)
            __syncthreads();
            const float rep = P->repetition_penalty, pres = P->presence_penalty;
            const int nbits = (len + 31) >> 5;
            for (int wi = tid; wi < nbits; wi += kNT) {
                uint32_t bits = hb[wi];
                while (bits != 0u) {
                    const int e = (wi << 5) + __ffs(bits) - 1;
                    bits &= bits - 1u;
                    if (!kRaw && (K[e] >= 0xFF800000u || K[e] <= 0x007FFFFFu)) t_bad = true;
                    float v = kval(K[e]);
                    if (rep != 1.0f && rep > 0.0f) v = (v < 0.0f) ? __fmul_rn(v, rep) : __fdiv_rn(v, rep);
                    v = __fsub_rn(v, pres);
                    v = __fadd_rn(v, 0.0f);
                    const uint32_t b = __float_as_uint(v);
                    uint32_t k = b ^ (static_cast<uint32_t>(static_cast<int32_t>(b) >> 31) | 0x80000000u);
                    K[e] = k;
                    if (k > t_mk || (k == t_mk && static_cast<uint32_t>(e) < t_mi)) {
                        t_mk = k;
                        t_mi = static_cast<uint32_t>(e);
                    }
                    t_mn = (k != 0u && k < t_mn) ? k : t_mn;
                }
            }
        }
    } else {
        // frequency-penalty rows: fp32 values first, then the per-unique penalty, then the
        // per-occurrence frequency penalty (identical addends, so the order of the atomic updates
        // does not change the result), then keys
        for (int s = 0; s < kStages; ++s) {
            const int32_t v0 = stage_vec(s), v1 = stage_vec(s + 1);
            if (v1 > v0) {
                if (!mbar_wait(&ls->mbar[s], 0, kWaitIters)) ls->bc[15] = 1;
            }
            if (DT == SIXI_SMP_BF16) {
                uint4 raw4[kVecMax];
#pragma unroll
                for (int m = 0; m < kVecMax; ++m) {
                    const int32_t v = v0 + tid + m * kNT;
                    if (v < v1) raw4[m] = *reinterpret_cast<const uint4*>(stg + 16u * v);
                }
                __syncthreads();
#pragma unroll
                for (int m = 0; m < kVecMax; ++m) {
                    const int32_t v = v0 + tid + m * kNT;
                    if (v < v1) {
                        const uint32_t w4[4] = {raw4[m].x, raw4[m].y, raw4[m].z, raw4[m].w};
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            KF[v * 8 + 2 * i] = __uint_as_float(w4[i] << 16);
                            KF[v * 8 + 2 * i + 1] = __uint_as_float(w4[i] & 0xFFFF0000u);
                        }
                    }
                }
                __syncthreads();
            }
        }
        for (int32_t e = len_t + tid; e < len; e += kNT) KF[e] = load_global(e);
        __syncthreads();
        for (int64_t j = tid; j < nht; j += kNT) {
            const int32_t t = hist_at(rc, j);
            if (t < c0 || t >= c0 + len || !allowed(t)) continue;
            const int32_t e = t - c0;
            const uint32_t bit = 1u << (e & 31);
            const uint32_t old = atomicAnd(&hb[e >> 5], ~bit);
            if (old & bit) KF[e] = penalize(KF[e], P);
        }
        __syncthreads();
        for (int64_t j = tid; j < nht; j += kNT) {
            const int32_t t = hist_at(rc, j);
            if (t < c0 || t >= c0 + len || !allowed(t)) continue;
            atomicAdd(&KF[t - c0], -P->frequency_penalty);
        }
        __syncthreads();
        for (int32_t e = tid; e < len; e += kNT) {
            uint32_t k;
            SIXI_ADMIT(e, KF[e], allowed(c0 + e) ? 1u : 0u, 0u, k, true);
            K[e] = k;
        }
        t_mn = (t_mn1 == 0xFFFFFFFFu) ? 0xFFFFFFFFu : t_mn1 + 1u;
    }
#undef SIXI_ADMIT
    // keys past the chunk end (up to a multiple of 4) are invalid
    if (tid < 4 && len + tid < nq * 4) K[len + tid] = 0u;
    __syncthreads();

    // block reduction of the row statistics; the result is pushed to every CTA of the cluster
    unsigned long long l_best;
    uint32_t l_n;
    {
        const int w = tid >> 5;
        const uint32_t wmk = __reduce_max_sync(0xFFFFFFFFu, t_mk);
        const uint32_t wmi = __reduce_min_sync(0xFFFFFFFFu, (t_mk == wmk && wmk != 0u) ? t_mi : 0xFFFFFFFFu);
        const uint32_t wmn = __reduce_min_sync(0xFFFFFFFFu, t_mn);
        const uint32_t wam = __reduce_max_sync(0xFFFFFFFFu, t_amax);
        const uint32_t wcn = __reduce_add_sync(0xFFFFFFFFu, t_cnt);
        const uint32_t wfi = __reduce_min_sync(0xFFFFFFFFu, t_first);
        const uint32_t wbad = __reduce_or_sync(0xFFFFFFFFu, t_bad ? 1u : 0u);
        if (lane == 0) {
            ls->red[w * 8 + 0] = (static_cast<unsigned long long>(wmk) << 32) | wmi;
            ls->red[w * 8 + 1] = wmn;
            ls->red[w * 8 + 2] = wam;
            ls->red[w * 8 + 3] = wcn;
            ls->red[w * 8 + 4] = wfi;
            ls->red[w * 8 + 5] = wbad;
        }
        __syncthreads();
        uint32_t mk = 0u, mi = 0xFFFFFFFFu, mn = 0xFFFFFFFFu, am = 0u, cn = 0u, fi = 0xFFFFFFFFu, bd = 0u;
#pragma unroll
        for (int q = 0; q < kNW; ++q) {
            const uint32_t k = static_cast<uint32_t>(ls->red[q * 8 + 0] >> 32);
            const uint32_t i = static_cast<uint32_t>(ls->red[q * 8 + 0]);
            if (k > mk || (k == mk && i < mi)) {
                mk = k;
                mi = i;
            }
            mn = static_cast<uint32_t>(ls->red[q * 8 + 1]) < mn ? static_cast<uint32_t>(ls->red[q * 8 + 1]) : mn;
            am = static_cast<uint32_t>(ls->red[q * 8 + 2]) > am ? static_cast<uint32_t>(ls->red[q * 8 + 2]) : am;
            cn += static_cast<uint32_t>(ls->red[q * 8 + 3]);
            fi = static_cast<uint32_t>(ls->red[q * 8 + 4]) < fi ? static_cast<uint32_t>(ls->red[q * 8 + 4]) : fi;
            bd |= static_cast<uint32_t>(ls->red[q * 8 + 5]);
        }
        RowStat st;
        st.best = (mk != 0u) ? comp_of(mk, static_cast<uint32_t>(c0) + mi) : 0ull;
        st.min_key = mn;
        st.n_allowed = cn;
        st.first = fi;
        st.flags = (am >= 0x7F800000u || bd != 0u ? 1u : 0u) | (ls->bc[15] ? 2u : 0u);
        if (kRaw && fi != 0xFFFFFFFFu && K[fi - static_cast<uint32_t>(c0)] == 0u) st.flags |= 4u;
        st.dhas = (rc.draft >= c0 && rc.draft < c0 + len) ? 1u : 0u;
        st.dkey = st.dhas ? K[rc.draft - c0] : 0u;
        l_best = st.best;
        l_n = cn;
        if (tid < static_cast<int>(C)) cluster.map_shared_rank(cs, tid)->xs[crank] = st;
        __syncthreads();  // also: the history bitmap / mask words (region Y) are dead from here
    }

    // list-path local selection (before the first cluster barrier). A row takes the list path
    // when its k is at most kKS: either 1 <= top_k <= kKS, or it has at most kKS allowed entries
    // (then every chunk has at most kKS and pushes all of them). The candidates entry also pushes
    // its best min(max_out, kKS) for rows on the mass path.
    {
        const bool stoch = !rc.greedy && rc.active && MODE != kModeGreedy;
        const int32_t tk = P->top_k;
        uint32_t ksel = 0;
        bool push = false;
        if (stoch) {
            if (tk >= 1 && tk <= kKS) {
                ksel = static_cast<uint32_t>(tk);
                push = true;
            } else if (l_n <= static_cast<uint32_t>(kKS)) {
                ksel = l_n;
                push = true;
            } else if (MODE == kModeCandidates) {
                ksel = a.max_out < static_cast<uint32_t>(kKS) ? a.max_out : static_cast<uint32_t>(kKS);
                push = true;
            }
        }
        const uint32_t kl = ksel < l_n ? ksel : l_n;
        if (push && kl > 0) {
            // Key threshold from the per-thread maxima: the bin (exp domain, relative to the local
            // max) where their cumulative count reaches kl; every key >= the smallest of those
            // maxima is a candidate, which is a superset of the local top-kl.
            const float lmax = kval(comp_key(l_best));
            const float bscale = static_cast<float>(
                (kTB - 1) / (46.0 * 0.6931471805599453 * static_cast<double>(P->temperature)));
            auto xbin = [&](uint32_t key) -> int {
                const float d = (lmax - kval(key)) * bscale;
                int b = d > 0.0f ? static_cast<int>(d) : 0;
                return b < kTB - 1 ? b : kTB - 1;
            };
            for (int i = tid; i < kTB; i += kNT) H32[i] = 0u;
            __syncthreads();
            if (t_mk != 0u) atomicAdd(&H32[xbin(t_mk)], 1u);
            __syncthreads();
            constexpr int PER = kTB / kNT;
            const int b0 = tid * PER;
            uint32_t s8 = 0;
#pragma unroll
            for (int q = 0; q < PER; ++q) s8 += H32[b0 + q];
            uint32_t tot = 0;
            const uint32_t ex = block_excl_u32<kNT>(s8, ls->red32, &tot);
            if (tid == 0) ls->bc[4] = kTB - 1;
            __syncthreads();
            if (ex < kl && ex + s8 >= kl) {
                uint32_t run = ex;
                for (int q = 0; q < PER; ++q) {
                    run += H32[b0 + q];
                    if (run >= kl) {
                        ls->bc[4] = static_cast<unsigned long long>(b0 + q);
                        break;
                    }
                }
            }
            __syncthreads();
            const int b1 = static_cast<int>(ls->bc[4]);
            // fewer than kl threads hold a valid entry: every valid entry is a candidate
            const uint32_t kthr = (tot < kl) ? 1u : static_cast<uint32_t>(
                block_min_bc((t_mk != 0u && xbin(t_mk) <= b1) ? t_mk : 0xFFFFFFFFull, ls));
            // collect the superset into LL (unordered)
            collect_scan(K, nq, static_cast<uint32_t>(c0), kthr, LL, &ls->lcount);
            __syncthreads();
            uint32_t ncand = ls->lcount;
            if (ncand > static_cast<uint32_t>(kLCap)) {
                // too many: exact kl-th largest composite by a radix select over the keys
                uint32_t prefix = 0, pmask = 0, above = 0;
                for (int shift = 24; shift >= 0; shift -= 8) {
                    for (int i = tid; i < 256; i += kNT) BH[i] = 0u;
                    __syncthreads();
                    for (int e = tid; e < len; e += kNT) {
                        const uint32_t k = K[e];
                        if (k == 0u || (k & pmask) != prefix) continue;
                        atomicAdd(&BH[(k >> shift) & 255u], 1u);
                    }
                    __syncthreads();
                    if (tid == 0) {
                        uint32_t run = above;
                        int dsel = 0;
                        for (int d = 255; d >= 0; --d) {
                            if (BH[d] > 0 && run + BH[d] >= kl) {
                                dsel = d;
                                break;
                            }
                            run += BH[d];
                        }
                        ls->bc[5] = static_cast<unsigned long long>(dsel);
                        ls->bc[6] = run;
                    }
                    __syncthreads();
                    prefix |= static_cast<uint32_t>(ls->bc[5]) << shift;
                    pmask |= 255u << shift;
                    above = static_cast<uint32_t>(ls->bc[6]);
                    __syncthreads();
                }
                // entries with key == prefix are ties: the (kl - above)-th lowest id closes the set
                const uint32_t need = kl - above;
                uint32_t taken = 0;
                for (int m = 0; m < nq_iter; ++m) {
                    const int q = tid + m * kNT;
                    uint32_t t = 0;
                    if (q < nq) {
#pragma unroll
                        for (int i = 0; i < 4; ++i) t += (K[4 * q + i] == prefix) ? 1u : 0u;
                    }
                    uint32_t tot2 = 0;
                    const uint32_t ex2 = block_excl_u32<kNT>(t, ls->red32, &tot2);
                    uint32_t run = taken + ex2;
                    if (q < nq) {
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            if (K[4 * q + i] != prefix) continue;
                            ++run;
                            if (run == need) ls->bc[7] = comp_of(prefix, static_cast<uint32_t>(c0 + 4 * q + i));
                        }
                    }
                    taken += tot2;
                }
                __syncthreads();
                const unsigned long long thr = ls->bc[7];
                if (tid == 0) ls->lcount = 0;
                __syncthreads();
                for (int m = 0; m < nq_iter; ++m) {
                    const int q = tid + m * kNT;
                    uint4 v = make_uint4(0u, 0u, 0u, 0u);
                    if (q < nq) v = reinterpret_cast<const uint4*>(K)[q];
                    const uint32_t k4[4] = {v.x, v.y, v.z, v.w};
                    uint32_t c = 0;
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        c += (k4[i] != 0u && comp_of(k4[i], static_cast<uint32_t>(c0 + 4 * q + i)) >= thr) ? 1u : 0u;
                    uint32_t slot = warp_reserve(c, &ls->lcount);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const unsigned long long cp = comp_of(k4[i], static_cast<uint32_t>(c0 + 4 * q + i));
                        if (k4[i] != 0u && cp >= thr) LL[slot++] = cp;
                    }
                }
                __syncthreads();
                ncand = ls->lcount;
            }
            // rank sort; the best kl go to CTA 0's merge area at their rank
            unsigned long long* ma0 = cluster.map_shared_rank(MA, 0);
            for (uint32_t i = tid; i < ncand; i += kNT) {
                const unsigned long long v = LL[i];
                uint32_t rank = 0;
                for (uint32_t j2 = 0; j2 < ncand; ++j2) rank += (LL[j2] > v) ? 1u : 0u;
                if (rank < kl) ma0[crank * kKS + rank] = v;
            }
        }
        if (tid == 0) cluster.map_shared_rank(cs, 0)->lcnt[crank] = push ? kl : kNoList;
        __syncthreads();
    }

    cluster.sync();  // ======================================================== CS1

    // ======================================================================== phase B
    unsigned long long best = 0ull;
    uint32_t first = 0xFFFFFFFFu, first_nan = 0u, dkey = 0u, dhas = 0u;
    uint32_t min_key = 0xFFFFFFFFu, n_allowed = 0, bad = 0;
    for (uint32_t q = 0; q < C; ++q) {
        const RowStat& s = cs->xs[q];
        best = s.best > best ? s.best : best;
        if (s.first < first) {
            first = s.first;
            first_nan = (s.flags >> 2) & 1u;
        }
        if (s.dhas) {
            dhas = 1u;
            dkey = s.dkey;
        }
        min_key = s.min_key < min_key ? s.min_key : min_key;
        n_allowed += s.n_allowed;
        bad |= s.flags & 3u;
    }
    const bool raw_argmax = (MODE == kModeGreedy) || (MODE == kModeVerify && rc.greedy);
    int32_t status = SIXI_OK;
    int path = 0;  // 0 nothing more, 1 list, 2 mass
    uint32_t k_eff = 0;
    if (!rc.active) {
        status = SIXI_OK;
    } else if (bad & 2u) {
        status = SIXI_BACKEND_ERROR;
    } else if (n_allowed == 0) {
        status = SIXI_INVALID_ARGUMENT;
    } else if ((bad & 1u) && !raw_argmax) {
        status = SIXI_NUMERIC_NAN_OR_INF;
    } else if (!rc.greedy) {
        const int32_t tk = P->top_k;
        k_eff = (tk > 0 && static_cast<uint32_t>(tk) < n_allowed) ? static_cast<uint32_t>(tk) : n_allowed;
        path = (k_eff <= static_cast<uint32_t>(kKS)) ? 1 : 2;
    }
    int32_t res_status = status;
    int32_t res_token = -1;
    int32_t res_accept = 0;
    if (rc.active && status == SIXI_OK && rc.greedy) {
        res_token = (raw_argmax && (first_nan || best == 0ull)) ? static_cast<int32_t>(first)
                                                              : static_cast<int32_t>(comp_id(best));
        if (raw_argmax && (bad & 1u)) res_status = SIXI_NUMERIC_NAN_OR_INF;
    }

    const double invT = 1.0 / static_cast<double>(P->temperature);
    const float M = kval(comp_key(best));
    const double maxs = static_cast<double>(M) * invT;
    const bool dvalid = dhas != 0u && dkey != 0u;
    const float xd = dvalid ? kval(dkey) : 0.0f;
    const unsigned long long dcomp = dvalid ? comp_of(dkey, static_cast<uint32_t>(rc.draft)) : 0ull;

    // merge of the pushed lists at CTA 0 into FL (sorted). Used by the list path and by the
    // candidates entry on the mass path.
    uint32_t fl_n = 0;
    const bool want_lists = crank == 0 && (path == 1 || (path == 2 && MODE == kModeCandidates));
    if (want_lists) {
        uint32_t total = 0;
        bool ok = true;
        for (uint32_t q = 0; q < C; ++q) {
            if (cs->lcnt[q] == kNoList) ok = false;
            else total += cs->lcnt[q];
        }
        fl_n = (path == 1) ? k_eff : (total < a.max_out ? total : a.max_out);
        if (fl_n > static_cast<uint32_t>(kKS)) fl_n = kKS;
        if (!ok || total < fl_n) {
            res_status = SIXI_BACKEND_ERROR;
            path = (path == 1) ? 0 : path;
            fl_n = 0;
        }
        // merge: rank of every pushed entry = its position + entries greater in the other lists
        // entries list-minor (x -> list x % C, position x / C): for k <= kNT / C every thread
        // merges at most one entry, instead of one entry of every list in turn
        for (uint32_t x = tid; fl_n > 0 && x < C * kKS; x += kNT) {
            const uint32_t q = x % C, pidx = x / C;
            if (pidx >= fl_n) break;  // its rank is at least pidx: never among the first fl_n
            if (pidx >= cs->lcnt[q]) continue;
            const unsigned long long v = MA[q * kKS + pidx];
            uint32_t rank = pidx;
            for (uint32_t o = 0; o < C; ++o) {
                if (o == q) continue;
                uint32_t lo = 0, hi = cs->lcnt[o];
                const unsigned long long* lp = MA + o * kKS;
                while (lo < hi) {
                    const uint32_t mid = (lo + hi) >> 1;
                    if (lp[mid] > v) lo = mid + 1;
                    else hi = mid;
                }
                rank += lo;
            }
            if (rank < fl_n) FL[rank] = v;
        }
        __syncthreads();
    }
    // list path: CTA 0 (the other CTAs of such rows are finished). Softmax terms by all threads;
    // sums and the top-p decision by warp 0 with 8 candidates per lane (candidate order =
    // lane-major); each division by a sum by its own thread (an fp64 division is a long dependent
    // sequence: eight in a row per lane would dominate the phase).
    const bool use_top_p = P->top_p > 0.0f && P->top_p < 1.0f;
    if (crank == 0 && path == 1) {
        const uint32_t n = fl_n;
        // fp64 softmax terms over the k candidates (core_execution.cpp:538-549)
        if (static_cast<uint32_t>(tid) < n) FP[tid] = exp(static_cast<double>(kval(comp_key(FL[tid]))) * invT - maxs);
        __syncthreads();
        if (tid < 32) {
            double lsum = 0.0;
#pragma unroll
            for (int j = 0; j < kPL; ++j) {
                const uint32_t idx = lane * kPL + j;
                lsum += idx < n ? FP[idx] : 0.0;
            }
            const double sum_exp = warp_sum_f64(lsum);
            if (lane == 0) ls->bc[8] = static_cast<unsigned long long>(__double_as_longlong(sum_exp));
        }
        __syncthreads();
        const double sum_exp = __longlong_as_double(static_cast<long long>(ls->bc[8]));
        if (sum_exp > 0.0 && static_cast<uint32_t>(tid) < n) FP[tid] /= sum_exp;
        __syncthreads();
        if (use_top_p) {
            // top-p: keep through the first index with cumulative >= top_p, renormalise
            // (core_execution.cpp:551-575)
            if (tid < 32) {
                double pr[kPL];
#pragma unroll
                for (int j = 0; j < kPL; ++j) {
                    const uint32_t idx = lane * kPL + j;
                    pr[j] = idx < n ? FP[idx] : 0.0;
                }
                const uint32_t f = lane_first_cum_ge(pr, static_cast<double>(P->top_p), n, lane);
                const uint32_t keep = (f == 0xFFFFFFFFu) ? n : f + 1u;
                double ks = 0.0;
#pragma unroll
                for (int j = 0; j < kPL; ++j) ks += (lane * kPL + j < keep) ? pr[j] : 0.0;
                const double r = warp_sum_f64(ks);
                if (lane == 0) {
                    ls->bc[8] = static_cast<unsigned long long>(__double_as_longlong(r));
                    ls->bc[9] = keep;
                }
            }
            __syncthreads();
            const uint32_t keep = static_cast<uint32_t>(ls->bc[9]);
            const double r = __longlong_as_double(static_cast<long long>(ls->bc[8]));
            if (keep < n && r > 0.0 && static_cast<uint32_t>(tid) < n) FP[tid] /= r;
            __syncthreads();
        }
    }
    if (crank == 0 && path == 1 && tid < 32) {
        const uint32_t n = fl_n;
        double pr[kPL];
#pragma unroll
        for (int j = 0; j < kPL; ++j) {
            const uint32_t idx = lane * kPL + j;
            pr[j] = idx < n ? FP[idx] : 0.0;
        }
        uint32_t keep = use_top_p ? static_cast<uint32_t>(ls->bc[9]) : n;
        if (P->min_p > 0.0f) {
            // min-p extension: keep prob >= min_p * max prob, renormalise
            const double thr = static_cast<double>(P->min_p) * __shfl_sync(0xFFFFFFFFu, pr[0], 0);
            uint32_t mine = 0xFFFFFFFFu;
#pragma unroll
            for (int j = kPL - 1; j >= 0; --j) {
                const uint32_t idx = lane * kPL + j;
                if (idx >= 1 && idx < keep && pr[j] < thr) mine = idx;
            }
            const uint32_t f = __reduce_min_sync(0xFFFFFFFFu, mine);
            if (f != 0xFFFFFFFFu && f < keep) {
                keep = f;
                lane_renorm(pr, keep, lane);
            }
        }
#pragma unroll
        for (int j = 0; j < kPL; ++j) {
            if (lane * kPL + j >= keep) pr[j] = 0.0;
            FP[lane * kPL + j] = pr[j];
        }
        __syncwarp();
        if (MODE == kModeSample || (MODE == kModeVerify && rc.vrole == 1)) {
            // CDF draw in candidate order (core_execution.cpp:586-601)
            const uint32_t f = lane_first_cum_gt(pr, rc.u_draw, keep, lane);
            res_token = static_cast<int32_t>(comp_id(FL[f == 0xFFFFFFFFu ? keep - 1u : f]));
        } else if (MODE == kModeCandidates) {
#pragma unroll
            for (int j = 0; j < kPL; ++j) {
                const uint32_t idx = lane * kPL + j;
                if (idx < keep && idx < a.max_out) {
                    a.out_ids[static_cast<size_t>(row) * a.max_out + idx] = static_cast<int32_t>(comp_id(FL[idx]));
                    a.out_probs[static_cast<size_t>(row) * a.max_out + idx] = pr[j];
                }
            }
            if (lane == 0) a.out_count[row] = static_cast<int32_t>(keep);
        } else if (MODE == kModeVerify) {
            const int32_t d = rc.draft;
            uint32_t mine = 0xFFFFFFFFu;
#pragma unroll
            for (int j = kPL - 1; j >= 0; --j) {
                const uint32_t idx = lane * kPL + j;
                if (idx < keep && static_cast<int32_t>(comp_id(FL[idx])) == d) mine = idx;
            }
            const uint32_t dpos = __reduce_min_sync(0xFFFFFFFFu, mine);
            const double pd = (dpos == 0xFFFFFFFFu) ? 0.0 : FP[dpos];
            const bool in_range = d >= 0 && static_cast<uint32_t>(d) < a.vocab;
            if (a.q != nullptr || a.qlog != nullptr) {
                // dense draft probabilities (speculative.cpp:823-903)
                const QView qv = q_view(a, static_cast<size_t>(rc.stream) * a.k + rc.vidx);
                const float p_d = static_cast<float>(pd);
                const float q_d = in_range ? q_of(qv, static_cast<uint32_t>(d)) : 1.0f;
                const double accept_prob = (q_d <= 0.0f) ? (p_d > 0.0f ? 1.0 : 0.0)
                    : fmin(1.0, static_cast<double>(p_d) / fmax(1e-12, static_cast<double>(q_d)));
                res_accept = rc.u_accept < accept_prob ? 1 : 0;
                if (!res_accept) {
                    // residual max(0, p - q) is non-zero only on the kept candidates: walk them in
                    // vocabulary-id order (rank of each id among the kept ids)
                    double res[kPL];
                    double rs = 0.0;
#pragma unroll
                    for (int j = 0; j < kPL; ++j) {
                        const uint32_t idx = lane * kPL + j;
                        res[j] = 0.0;
                        if (idx < keep) {
                            const uint32_t id = comp_id(FL[idx]);
                            res[j] = fmax(0.0, static_cast<double>(static_cast<float>(pr[j])) - static_cast<double>(q_of(qv, id)));
                        }
                        rs += res[j];
                    }
                    const double res_sum = warp_sum_f64(rs);
#pragma unroll
                    for (int j = 0; j < kPL; ++j) {
                        const uint32_t idx = lane * kPL + j;
                        if (idx < keep) {
                            const uint32_t id = comp_id(FL[idx]);
                            uint32_t r = 0;
                            for (uint32_t o = 0; o < keep; ++o) r += comp_id(FL[o]) < id ? 1u : 0u;
                            FQ[r] = res_sum > 1e-12 ? res[j] / res_sum : static_cast<double>(static_cast<float>(pr[j]));
                            BH[r] = id;
                        }
                    }
                    __syncwarp();
                    double v[kPL];
#pragma unroll
                    for (int j = 0; j < kPL; ++j) v[j] = (lane * kPL + j < keep) ? FQ[lane * kPL + j] : 0.0;
                    const uint32_t f = lane_first_cum_gt(v, rc.u_draw, keep, lane);
                    res_token = (f == 0xFFFFFFFFu) ? static_cast<int32_t>(a.vocab - 1) : static_cast<int32_t>(BH[f]);
                }
            } else {
                // one-hot drafts (speculative.cpp:638-681): residual = the kept candidates without
                // the draft, renormalised, drawn in candidate order
                res_accept = rc.u_accept < pd ? 1 : 0;
                if (!res_accept) {
                    double v[kPL];
                    double rs = 0.0;
#pragma unroll
                    for (int j = 0; j < kPL; ++j) {
                        v[j] = (lane * kPL + j == dpos) ? 0.0 : pr[j];
                        rs += v[j];
                    }
                    const double res_sum = warp_sum_f64(rs);
                    const uint32_t m = keep - (dpos != 0xFFFFFFFFu ? 1u : 0u);
                    if (m > 0 && res_sum > 0.0) {
#pragma unroll
                        for (int j = 0; j < kPL; ++j) v[j] /= res_sum;
                        const uint32_t last = (dpos == keep - 1u) ? keep - 2u : keep - 1u;
                        const uint32_t f = lane_first_cum_gt(v, rc.u_draw, keep, lane);
                        res_token = static_cast<int32_t>(comp_id(FL[f == 0xFFFFFFFFu ? last : f]));
                    } else {
                        const uint32_t f = lane_first_cum_gt(pr, rc.u_draw, keep, lane);
                        res_token = static_cast<int32_t>(comp_id(FL[f == 0xFFFFFFFFu ? keep - 1u : f]));
                    }
                }
            }
        }
    }

    // ======================================================================== outputs
    auto write_outputs = [&]() {
        if (crank != 0 || tid != 0) return;
        if (MODE == kModeVerify) {
            VerifyRowResult r;
            r.status = rc.active ? res_status : SIXI_OK;
            r.accept = res_accept;
            r.token = res_token;
            r.pad = 0;
            a.ws[row] = r;
        } else if (MODE == kModeCandidates) {
            a.out_status[row] = res_status;
            if (res_status != SIXI_OK) a.out_count[row] = 0;
            if (res_status == SIXI_OK && rc.greedy) {
                a.out_count[row] = 1;
                if (a.max_out > 0) {
                    a.out_ids[static_cast<size_t>(row) * a.max_out] = res_token;
                    a.out_probs[static_cast<size_t>(row) * a.max_out] = 1.0;
                }
            }
        } else {
            const bool ok = res_status == SIXI_OK || (MODE == kModeGreedy && res_status == SIXI_NUMERIC_NAN_OR_INF);
            a.out_tok[rc.orow] = ok ? res_token : -1;
            a.out_status[rc.orow] = res_status;
        }
    };

    // Rows without a mass-path selection are finished: on them no CTA touches another CTA's shared
    // memory after CS1, and `path` is computed from the same exchanged statistics in every CTA of
    // the cluster, so all CTAs of the cluster leave here together.
    if (path != 2) {
        write_outputs();
        return;
    }

    // ======================================================================== mass path
    WeightCtx wc{};
    unsigned long long Z = 0ull, Wmin = 0ull;
    float x_minp = -FLT_MAX;
    const bool need_counts = k_eff < n_allowed;
    // bins are uniform in t = log2 of the relative weight (the same t the weight is built from)
    auto xbin_g = [&](uint32_t key) -> int { return abin_of(kval(key), wc); };
    {
        const float m = kval(min_key);
        const double range_log2 = (static_cast<double>(M) - static_cast<double>(m)) * 1.4426950408889634 /
                                  static_cast<double>(P->temperature);
        make_weight_ctx(P->temperature, M, static_cast<float>(range_log2), wc);  // caps it at 46
        if (P->min_p > 0.0f) {
            x_minp = static_cast<float>(static_cast<double>(M) +
                                        static_cast<double>(P->temperature) * log(static_cast<double>(P->min_p)));
        }
        // Weight sums in three 32-bit parts (see mass_histogram), in region X. The counts use region
        // Y, which no CTA writes to before the third cluster barrier.
        for (int i = tid; i < kABins; i += kNT) {
            HB[i] = 0u;
            HA[i] = 0u;
            HC[i] = 0u;
            HLO[i] = 0u;
        }
        __syncthreads();
        // min-p prefix mass (only when min-p is set); the row mass Z is read off the assembled
        // cumulative histogram instead of being summed separately
        const bool use_minp = P->min_p > 0.0f;
        unsigned long long wp = mass_histogram(K, nq, wc, x_minp, use_minp, need_counts, HB, HC);
        if (use_minp) {
            wp = block_sum_u64<kNT>(wp, ls->red);
            if (tid < static_cast<int>(C)) cluster.map_shared_rank(cs, tid)->wmin[crank] = wp;
        }
    }

    cluster.sync();  // ======================================================== CS2

    // reduce histogram segment `crank` over all CTAs of the cluster (the loads of the C sources
    // are independent, so the unrolled loop keeps several remote round trips in flight)
    for (uint32_t i = tid; i < lay.seg; i += kNT) {
        const uint32_t j = crank * lay.seg + i;
        unsigned long long s = 0ull;
        uint32_t sc = 0;
#pragma unroll 4
        for (uint32_t q = 0; q < C; ++q) {
            s += (static_cast<unsigned long long>(cluster.map_shared_rank(HA, q)[j]) << 32) +
                 (static_cast<unsigned long long>(cluster.map_shared_rank(HB, q)[j]) << 16) +
                 cluster.map_shared_rank(HLO, q)[j];
            if (need_counts) sc += cluster.map_shared_rank(HC, q)[j];
        }
        R[i] = s;
        RC[i] = sc;
    }
    if (P->min_p > 0.0f) {
        for (uint32_t q = 0; q < C; ++q) Wmin += cs->wmin[q];
    }

    cluster.sync();  // ======================================================== CS3

    // Smallest valid key whose bin is <= bb (kmax + 1 when there is none); the bin is non-increasing
    // in the key. The boundary is estimated from the inverse of the bin function and then stepped
    // to the exact key where xbin_g changes, so the interval matches the histogram exactly.
    const uint32_t kmax = comp_key(best);
    const double inv_tscale = static_cast<double>(P->temperature) /
                              (1.4426950408889634 * static_cast<double>(wc.bin_scale));
    auto first_key_bin_le = [&](int bb) -> unsigned long long {
        if (bb < 0 || xbin_g(kmax) > bb) return static_cast<unsigned long long>(kmax) + 1ull;
        if (xbin_g(min_key) <= bb) return min_key;
        // now bin(min_key) > bb >= bin(kmax): the answer lies in (min_key, kmax]
        uint32_t k = fkey(static_cast<float>(static_cast<double>(M) - static_cast<double>(bb + 1) * inv_tscale));
        k = k <= min_key ? min_key + 1u : (k > kmax ? kmax : k);
#pragma unroll 1
        for (int it = 0; it < 64; ++it) {
            if (xbin_g(k) > bb) {
                ++k;  // k <= kmax here since bin(kmax) <= bb
            } else if (xbin_g(k - 1u) <= bb) {
                --k;  // k - 1 > min_key here since bin(min_key) > bb
            } else {
                return k;
            }
        }
        uint32_t lo = min_key + 1u, hi = kmax;  // far from the estimate: bisect
        while (lo < hi) {
            const uint32_t mid = lo + ((hi - lo) >> 1);
            if (xbin_g(mid) <= bb) hi = mid;
            else lo = mid + 1u;
        }
        return lo;
    };
    // The same boundary found by a whole warp: 32 consecutive keys tested per round in a window
    // that starts at the estimate and moves by 32 keys until it holds the change of bin (the bin
    // is monotone in the key, so the ballot is a run of zeros then ones); bisection after that.
    auto first_key_bin_le_warp = [&](int bb) -> unsigned long long {
        if (bb < 0 || xbin_g(kmax) > bb) return static_cast<unsigned long long>(kmax) + 1ull;
        if (xbin_g(min_key) <= bb) return min_key;
        // the answer lies in [lo, hi]: bin(lo - 1) > bb >= bin(hi)
        const uint32_t lo = min_key + 1u, hi = kmax;
        uint32_t k = fkey(static_cast<float>(static_cast<double>(M) - static_cast<double>(bb + 1) * inv_tscale));
        k = k < lo ? lo : (k > hi ? hi : k);
        uint32_t start = k - lo >= 16u ? k - 16u : lo;
#pragma unroll 1
        for (int it = 0; it < 32; ++it) {
            const uint32_t kj = start + static_cast<uint32_t>(lane);
            const bool le = kj >= hi || kj < start || xbin_g(kj) <= bb;  // past hi (or wrapped): true
            const unsigned bal = __ballot_sync(0xFFFFFFFFu, le);
            if (bal == 0u) {
                start += 32u;  // the answer is above the window, so start + 32 <= answer <= hi
            } else if (bal & 1u) {
                if (start == lo) return lo;
                start = start - lo > 31u ? start - 31u : lo;  // the new window ends at the old start
            } else {
                return start + static_cast<uint32_t>(__ffs(bal) - 1);
            }
        }
        return first_key_bin_le(bb);
    };
    // First bin with CG >= t (the last bin when there is none), by every warp: a ballot over the
    // ends of the 32 chunks of 64 bins (a contiguous copy), then over the chunk's two halves. CG is
    // non-decreasing.
    static_assert(kABins == 2048, "two-level search over 32 x 64 bins");
    auto bin_of_target = [&](unsigned long long t) -> int {
        const unsigned b1 = __ballot_sync(0xFFFFFFFFu, ls->cge[lane] >= t);  // chunk ends, contiguous
        if (b1 == 0u) return kABins - 1;
        const int base = (__ffs(b1) - 1) * 64;
        const unsigned lo = __ballot_sync(0xFFFFFFFFu, CG[base + lane] >= t);
        if (lo != 0u) return base + __ffs(lo) - 1;
        const unsigned hi = __ballot_sync(0xFFFFFFFFu, CG[base + 32 + lane] >= t);  // non-zero: CG[base + 63] >= t
        return base + 32 + __ffs(hi) - 1;
    };
    // Pushes my entries of bin bA (and of bins bBlo..bBhi when bBlo >= 0) whose composite is >= lowb
    // into my segment of gather buffer bufA (bufB) in every CTA of the cluster, then publishes how many I
    // have (a count above the segment size marks the bin overfull). Slots come from a local
    // counter, so the remote traffic is plain stores.
    const uint32_t gseg = static_cast<uint32_t>(kGCap) / C;
    // True when bins lo..hi provably hold at most gseg keys, so that gathering them cannot overflow
    // any CTA's segment. Every key of bin b weighs at least 2^(43 - (b + 1) / bin_scale), less the
    // errors of the exponential and of the rounding (far below the 0.1 % margin while that weight
    // is at least 1,024), so the bins' mass bounds their count.
    auto bins_fit = [&](int lo, int hi) -> bool {
        const double wmin = exp2(43.0 - static_cast<double>(hi + 1) / static_cast<double>(wc.bin_scale));
        if (!(wmin >= 1024.0)) return false;
        const double mass = static_cast<double>(CG[hi] - (lo > 0 ? CG[lo - 1] : 0ull));
        return mass <= 0.999 * wmin * static_cast<double>(gseg);
    };
    auto gather = [&](int bA, int bufA, int bBlo, int bBhi, int bufB, unsigned long long lowb) {
        // key intervals: bin bA, and bins bBlo..bBhi (empty when bBlo < 0); the four boundaries are
        // computed at once by warps 0-3
        if (tid < 128) {
            const int w = tid >> 5;
            const int bb = w == 0 ? bA : (w == 1 ? bA - 1 : (w == 2 ? bBhi : bBlo - 1));
            const unsigned long long kb = (w < 2 || bBlo >= 0) ? first_key_bin_le_warp(bb) : 0ull;
            if (lane == 0) ls->bc[4 + w] = kb;
        }
        if (tid == 0) {
            ls->gfill[0] = 0u;
            ls->gfill[1] = 0u;
        }
        __syncthreads();
        const uint32_t kloA = static_cast<uint32_t>(ls->bc[4]);
        const unsigned long long khiA1 = ls->bc[5];  // one past bin bA
        const uint32_t kloB = bBlo >= 0 ? static_cast<uint32_t>(ls->bc[6]) : 1u;
        const unsigned long long khiB1 = bBlo >= 0 ? ls->bc[7] : 0ull;
        unsigned long long* gA = (bufA ? G1 : G0) + crank * gseg;
        unsigned long long* gB = (bufB ? G1 : G0) + crank * gseg;
        // Membership is one unsigned subtract-compare per interval; the composite lower bound is
        // tested only when it is set (k-bound rows). These loops are bound by the integer pipe.
        const uint32_t wA = static_cast<uint32_t>(khiA1 - kloA);
        const uint32_t wB = bBlo >= 0 ? static_cast<uint32_t>(khiB1 - kloB) : 0u;  // empty set B
        // When the two sets touch (or B is empty), one test per key against their union screens
        // the keys; when they are apart, the screen is the pair of exact tests (a screen over the
        // gap would admit its keys and run the per-hit path for nothing).
        const bool touch = wB == 0u || (static_cast<unsigned long long>(kloB) <= khiA1 &&
                                        static_cast<unsigned long long>(kloA) <= khiB1);
        const uint32_t kloU = (wB != 0u && kloB < kloA) ? kloB : kloA;
        const unsigned long long khiU1 = (wB != 0u && khiB1 > khiA1) ? khiB1 : khiA1;
        const uint32_t wU = static_cast<uint32_t>(khiU1 - kloU);
        gather_scan(K, nq, static_cast<uint32_t>(c0), kloA, wA, kloB, wB, touch, kloU, wU, lowb, gA, gB, gseg, C,
                    ls->gfill);
        __syncthreads();
        const uint32_t tot = ls->gfill[0] | (ls->gfill[1] << 16);
        if (tid < static_cast<int>(C)) {  // publish my counts (above gseg: the bin is overfull)
            ClusterShared* d = cluster.map_shared_rank(cs, tid);
            d->gseg[bufA][crank] = tot & 0xFFFFu;
            if (bBlo >= 0) d->gseg[bufB][crank] = tot >> 16;
        }
    };

    // every CTA assembles the same global cumulative histograms (CG/CGC overwrite H/HC). Each
    // thread owns 4 consecutive bins and moves them with 16-byte accesses (4-byte or 8-byte ones at
    // a 16- or 32-byte thread stride would conflict on the shared-memory banks).
    {
        constexpr int PER = kABins / kNT;
        static_assert(PER == 4, "16-byte accesses of 4 bins");
        unsigned long long v[PER];
        uint32_t vc[PER];
        unsigned long long s = 0ull;
        uint32_t sc = 0;
        {
            const uint32_t i0 = tid * PER;  // the PER bins lie in one segment (seg % PER == 0)
            const ulonglong2* rs = reinterpret_cast<const ulonglong2*>(cluster.map_shared_rank(R, i0 / lay.seg) +
                                                                        i0 % lay.seg);
            const ulonglong2 v01 = rs[0], v23 = rs[1];
            v[0] = v01.x;
            v[1] = v01.y;
            v[2] = v23.x;
            v[3] = v23.y;
            uint4 c4 = make_uint4(0u, 0u, 0u, 0u);
            if (need_counts)
                c4 = *reinterpret_cast<const uint4*>(cluster.map_shared_rank(RC, i0 / lay.seg) + i0 % lay.seg);
            vc[0] = c4.x;
            vc[1] = c4.y;
            vc[2] = c4.z;
            vc[3] = c4.w;
#pragma unroll
            for (int q = 0; q < PER; ++q) {
                s += v[q];
                sc += vc[q];
            }
        }
        const unsigned long long inc = warp_incl_u64(s);
        const uint32_t incc = warp_incl_u32(sc);
        if (lane == 31) {
            ls->red[tid >> 5] = inc;
            ls->red[kNW + (tid >> 5)] = incc;
        }
        __syncthreads();
        unsigned long long before = 0ull, beforec = 0ull;
#pragma unroll
        for (int w = 0; w < kNW; ++w) {  // independent loads, predicated adds
            const unsigned long long t = ls->red[w], tc = ls->red[kNW + w];
            before += (w < (tid >> 5)) ? t : 0ull;
            beforec += (w < (tid >> 5)) ? tc : 0ull;
        }
        unsigned long long run = before + inc - s;
        uint32_t runc = static_cast<uint32_t>(beforec) + incc - sc;
        unsigned long long p[PER];
        uint32_t pc[PER];
#pragma unroll
        for (int q = 0; q < PER; ++q) {
            run += v[q];
            runc += vc[q];
            p[q] = run;
            pc[q] = runc;
        }
        ulonglong2* cg2 = reinterpret_cast<ulonglong2*>(CG + tid * PER);
        cg2[0] = make_ulonglong2(p[0], p[1]);
        cg2[1] = make_ulonglong2(p[2], p[3]);
        *reinterpret_cast<uint4*>(CGC + tid * PER) = make_uint4(pc[0], pc[1], pc[2], pc[3]);
        if ((tid & 15) == 15) ls->cge[tid >> 4] = p[3];  // CG[64 w + 63]: the ends of the 64-bin chunks
        __syncthreads();
    }

    // The state below is advanced identically in every CTA of the cluster: every decision reads
    // only cluster-uniform data (exchanged statistics, the assembled histograms, gathered sets,
    // pushed partial results), so the loop's early exit is uniform within the cluster.
    Z = CG[kABins - 1];  // every positive weight lies in some bin
    // rows whose kept set is followed directly by a draw (sampled rows, the verifier's bonus rows)
    const bool draw_follows = (MODE == kModeSample) || (MODE == kModeVerify && rc.vrole == 1);
    LState st{};
    st.stage = need_counts ? kStKBound : kStTopP;
    st.pending_bin = -1;
    st.pending_kind = 0;
    st.pre_lo = -1;
    st.pre_hi = -1;
    st.pre_buf = 0;
    st.tabs = 0ull;
    st.result = -1;
    st.err = 0;
    st.zk = Z;
    st.zkept = Z;
    st.kbound = 0ull;
    st.xcross = 0ull;
    st.excl = 0ull;
    st.wexcl = 0ull;
    Refine rf{};
    // refine digit histograms (double-buffered) in region R: the reduced segments there are last
    // read remotely in the assembly above, at least one barrier before the first refine level
    // (computed from the buffer index rather than held in a pointer array, which an indexed access
    // would place in local memory)
    auto RH = [&](int buf) -> uint32_t* { return reinterpret_cast<uint32_t*>(R) + 256 * buf; };
    auto RW = [&](int buf) -> uint32_t* { return reinterpret_cast<uint32_t*>(R + 256) + 512 * buf; };  // split

    auto rf_match = [&](int e, uint32_t k) -> bool {
        if (k == 0u || (k & rf.pmask) != rf.prefix || xbin_g(k) != rf.bin) return false;
        const unsigned long long cp = comp_of(k, static_cast<uint32_t>(c0 + e));
        return cp >= rf.lowb && cp != rf.excl;
    };
    auto rf_build = [&](int buf) {  // local digit histogram of the refine level
        for (int i = tid; i < 256; i += kNT) {
            RH(buf)[i] = 0u;
            RW(buf)[i] = 0u;
            RW(buf)[256 + i] = 0u;
        }
        __syncthreads();
        for (int e = tid; e < len; e += kNT) {
            const uint32_t k = K[e];
            if (!rf_match(e, k)) continue;
            const uint32_t d = (k >> rf.shift) & ((1u << rf.width) - 1u);
            atomicAdd(&RH(buf)[d], 1u);
            smem_add_split(&RW(buf)[d], &RW(buf)[256 + d], weight_of(kval(k), wc));
        }
        __syncthreads();
    };
    auto rf_level = [&](int top) {
        rf.top = top;
        rf.shift = top - 7 > 0 ? top - 7 : 0;
        rf.width = top - rf.shift + 1;
    };

#pragma unroll 1
    for (int round = 0; round < kMaxRounds; ++round) {
        if (st.stage == kStDone || st.err) break;
        const int cur = round & 1;
        const int prev = cur ^ 1;
        bool read_buf = false;  // a gather buffer was read in this round
        // Whether this round touched another CTA's shared memory (or let another CTA touch mine).
        // The first round always counts: the histogram assembly before it read the peers' segments.
        bool remote = round == 0;
        // a second pass runs only when the draw bin was gathered ahead of time (pending_kind 4)
#pragma unroll 1
        for (int pass = 0; pass < 3; ++pass) {
        bool have_sel = false;
        unsigned long long sel = 0ull, cum_sel = 0ull, wthrough = 0ull;
        const int sel_bin = st.pending_bin;
        // ------------------------------------------------ resolve what the previous round started
        if (st.pending_kind == 1 || st.pending_kind == 4) {
            const int gbuf = (st.pending_kind == 4) ? st.pre_buf : prev;
            if (st.pending_kind == 4) st.pre_lo = -1;
            const unsigned int* gcn = cs->gseg[gbuf];
            bool over = false;
            for (uint32_t q = 0; q < C; ++q) over |= gcn[q] > gseg;
            if (over && st.pending_kind == 4) {  // refine the draw's own bin
                const int b = st.pending_bin;
                st.target = st.tabs - (b > 0 ? CG[b - 1] : 0ull);
            }
            const unsigned long long lowb = (st.stage == kStKBound) ? 0ull : st.kbound;
            const unsigned long long ex = (st.stage == kStResid) ? st.excl : 0ull;
            const bool cmode = (st.stage == kStKBound);
            read_buf = true;
            if (over) {
                // the bin is too full to gather: refine it by key digits across the cluster
                rf.active = 1;
                rf.phase = 0;
                rf.bin = st.pending_bin;
                rf.cmode = cmode ? 1 : 0;
                rf.t = st.target;
                rf.lowb = lowb;
                rf.excl = ex;
                rf.prefix = 0u;
                rf.pmask = 0u;
                rf.above_c = 0ull;
                rf.above_w = 0ull;
                rf.buf = 0;
                uint32_t lo = 0xFFFFFFFFu, hi = 0u;
                for (int e = tid; e < len; e += kNT) {
                    const uint32_t k = K[e];
                    if (!rf_match(e, k)) continue;
                    lo = k < lo ? k : lo;
                    hi = k > hi ? k : hi;
                }
                const unsigned long long l2 = block_min_u64<kNT>(lo, ls->red);
                const unsigned long long h2 = block_max_u64<kNT>(hi, ls->red);
                if (tid < static_cast<int>(C)) cluster.map_shared_rank(cs, tid)->mm[crank] = (l2 << 32) | h2;
                st.pending_kind = 3;
                remote = true;
            } else {
                const unsigned long long* gp = gbuf ? G1 : G0;
                sel = block_select(gp, gcn, C, gseg, st.target, wc, !cmode, lowb, ex, BH, ls, &cum_sel);
                if (sel == 0ull) {
                    st.err = 2;
                } else {
                    have_sel = true;
                    if (cmode) {
                        unsigned long long wpart = 0ull;
                        for (uint32_t q = 0; q < C; ++q) {
                            for (uint32_t i = tid; i < gcn[q]; i += kNT) {
                                const unsigned long long c = gp[q * gseg + i];
                                if (c >= sel) wpart += weight_of(kval(comp_key(c)), wc);
                            }
                        }
                        wthrough = block_sum_u64<kNT>(wpart, ls->red);
                    }
                }
                st.pending_kind = 0;
            }
            __syncthreads();
        } else if (st.pending_kind == 3) {
            remote = true;
            if (rf.phase == 0) {
                uint32_t klo = 0xFFFFFFFFu, khi = 0u;
                for (uint32_t q = 0; q < C; ++q) {
                    const unsigned long long v = cs->mm[q];
                    const uint32_t l = static_cast<uint32_t>(v >> 32), h = static_cast<uint32_t>(v);
                    klo = l < klo ? l : klo;
                    khi = h > khi ? h : khi;
                }
                if (klo > khi) {
                    st.err = 6;
                } else if (klo == khi) {
                    rf.prefix = klo;
                    rf.pmask = 0xFFFFFFFFu;
                    rf.phase = 2;
                } else {
                    const int top = 31 - __clz(static_cast<int>(klo ^ khi));
                    rf.pmask = (top == 31) ? 0u : ~((2u << top) - 1u);
                    rf.prefix = klo & rf.pmask;
                    rf_level(top);
                    rf.phase = 1;
                }
            } else if (rf.phase == 1) {
                // combine the digit histograms of all CTAs, choose the digit of the crossing
                if (tid < 256) {
                    unsigned long long sc = 0ull, sw = 0ull;
                    for (uint32_t q = 0; q < C; ++q) {
                        sc += cluster.map_shared_rank(RH(rf.buf), q)[tid];
                        const uint32_t* rw = cluster.map_shared_rank(RW(rf.buf), q);
                        sw += join_split(rw[tid], rw[256 + tid]);
                    }
                    BH[tid] = static_cast<uint32_t>(sc);
                    BW[tid] = sw;
                }
                __syncthreads();
                if (tid < 32) {
                    const unsigned int nd = 1u << rf.width;
                    unsigned long long pc[8], pw[8];
                    unsigned long long lsum = 0, lc = 0, lw = 0;
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const int dd = 255 - (tid * 8 + q);
                        pc[q] = dd < static_cast<int>(nd) ? BH[dd] : 0ull;
                        pw[q] = dd < static_cast<int>(nd) ? BW[dd] : 0ull;
                        lsum += rf.cmode ? pc[q] : pw[q];
                        lc += pc[q];
                        lw += pw[q];
                    }
                    const unsigned long long incl = warp_incl_u64(lsum);
                    const unsigned long long inclc = warp_incl_u64(lc);
                    const unsigned long long inclw = warp_incl_u64(lw);
                    unsigned long long run = (rf.cmode ? rf.above_c : rf.above_w) + incl - lsum;
                    unsigned long long runc = rf.above_c + inclc - lc, runw = rf.above_w + inclw - lw;
                    int found = -1;
                    unsigned long long fc = 0, fw = 0;
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const unsigned long long part = rf.cmode ? pc[q] : pw[q];
                        if (found < 0 && part > 0 && run + part >= rf.t) {
                            found = 255 - (tid * 8 + q);
                            fc = runc;
                            fw = runw;
                        }
                        run += part;
                        runc += pc[q];
                        runw += pw[q];
                    }
                    const unsigned ball = __ballot_sync(0xFFFFFFFFu, found >= 0);
                    if (ball) {
                        const int src = __ffs(ball) - 1;
                        const int fd = __shfl_sync(0xFFFFFFFFu, found, src);
                        const unsigned long long a1 = __shfl_sync(0xFFFFFFFFu, fc, src);
                        const unsigned long long a2 = __shfl_sync(0xFFFFFFFFu, fw, src);
                        if (tid == 0) {
                            ls->bc[10] = static_cast<unsigned long long>(fd);
                            ls->bc[11] = a1;
                            ls->bc[12] = a2;
                        }
                    } else if (tid == 0) {
                        ls->bc[10] = ~0ull;
                    }
                }
                __syncthreads();
                const unsigned long long fd = ls->bc[10];
                if (fd == ~0ull) {
                    st.err = 7;
                } else {
                    rf.above_c = ls->bc[11];
                    rf.above_w = ls->bc[12];
                    rf.prefix |= static_cast<uint32_t>(fd) << rf.shift;
                    rf.pmask |= ((1u << rf.width) - 1u) << rf.shift;
                    if (rf.shift == 0) {
                        rf.phase = 2;
                    } else {
                        rf_level(rf.shift - 1);
                        rf.buf ^= 1;
                    }
                }
                __syncthreads();
            } else if (rf.phase == 2) {
                // ties of the resolved key: find the owner CTA of the crossing entry (id order)
                // w: the selection unit of one tie (1 when counting); wk: its weight, for the mass
                const unsigned long long wk = weight_of(kval(rf.prefix), wc);
                const unsigned long long w = rf.cmode ? 1ull : wk;
                const unsigned long long done_sel = rf.cmode ? rf.above_c : rf.above_w;
                if (w == 0ull || rf.t <= done_sel) {
                    st.err = 8;
                } else {
                    const unsigned long long idx = (rf.t - done_sel + w - 1ull) / w - 1ull;
                    unsigned long long before = 0ull;
                    int owner = -1;
                    for (uint32_t q = 0; q < C; ++q) {
                        const unsigned long long c = cs->rcnt[q];
                        if (idx < before + c) {
                            owner = static_cast<int>(q);
                            break;
                        }
                        before += c;
                    }
                    if (owner < 0) {
                        st.err = 9;
                    } else {
                        rf.above_c += idx;  // entries before the crossing tie
                        rf.above_w += idx * wk;
                        rf.tie_w = wk;
                        if (owner == static_cast<int>(crank)) {
                            const unsigned long long li = idx - before;
                            unsigned long long taken = 0ull;
                            if (tid == 0) ls->bc[13] = 0ull;
                            for (int m = 0; m < nq_iter; ++m) {
                                const int q = tid + m * kNT;
                                uint32_t t = 0;
                                if (q < nq) {
#pragma unroll
                                    for (int i = 0; i < 4; ++i) t += rf_match(4 * q + i, K[4 * q + i]) ? 1u : 0u;
                                }
                                uint32_t tot = 0;
                                const uint32_t ex2 = block_excl_u32<kNT>(t, ls->red32, &tot);
                                unsigned long long r2 = taken + ex2;
                                if (q < nq) {
#pragma unroll
                                    for (int i = 0; i < 4; ++i) {
                                        if (!rf_match(4 * q + i, K[4 * q + i])) continue;
                                        if (r2 == li) ls->bc[13] = comp_of(K[4 * q + i], static_cast<uint32_t>(c0 + 4 * q + i));
                                        ++r2;
                                    }
                                }
                                taken += tot;
                            }
                            __syncthreads();
                            if (tid < static_cast<int>(C)) cluster.map_shared_rank(cs, tid)->rsel = ls->bc[13];
                        }
                        rf.phase = 3;
                    }
                }
            } else {  // phase 3: the owner's composite has arrived
                sel = cs->rsel;
                if (sel == 0ull) {
                    st.err = 10;
                } else {
                    have_sel = true;
                    cum_sel = rf.cmode ? rf.above_c + 1ull : rf.above_w + rf.tie_w;
                    wthrough = rf.above_w + rf.tie_w;
                }
                rf.active = 0;
                st.pending_kind = 0;
            }
            // issue this round's refine exchange
            if (rf.active && !st.err) {
                if (rf.phase == 1) {
                    rf_build(rf.buf);
                } else if (rf.phase == 2) {
                    uint32_t c = 0;
                    for (int e = tid; e < len; e += kNT) c += rf_match(e, K[e]) ? 1u : 0u;
                    const unsigned long long tc = block_sum_u64<kNT>(c, ls->red);
                    if (tid < static_cast<int>(C)) cluster.map_shared_rank(cs, tid)->rcnt[crank] = tc;
                }
            }
        } else if (st.pending_kind == 2) {
            remote = true;
            if (st.stage == kStDSum) {
                // dense residual: totals, then the owner CTA of the crossing finds the token
                double rs = 0.0, ps = 0.0;
                for (uint32_t q = 0; q < C; ++q) {
                    rs += cs->rsum[q];
                    ps += cs->psum[q];
                }
                const bool use_res = rs > 1e-12;
                const double target = rc.u_draw * (use_res ? rs : 1.0);
                int owner = -1;
                double before = 0.0;
                for (uint32_t q = 0; q < C; ++q) {
                    const double v = use_res ? cs->rsum[q] : cs->psum[q];
                    if (before + v > target && v > 0.0) {
                        owner = static_cast<int>(q);
                        break;
                    }
                    before += v;
                }
                if (owner < 0) {
                    st.result = static_cast<int32_t>(a.vocab - 1);
                    st.stage = kStDone;
                    st.pending_kind = 0;
                } else {
                    if (owner == static_cast<int>(crank)) {
                        // ordered scan of my entries in vocabulary-id order
                        const QView qv = q_view(a, static_cast<size_t>(rc.stream) * a.k + rc.vidx);
                        const double zk_d = static_cast<double>(st.zkept);
                        double run = before;
                        unsigned long long found = ~0ull;
                        for (int m = 0; m < nq_iter && found == ~0ull; ++m) {
                            const int q = tid + m * kNT;
                            double vals[4];
                            double s = 0.0;
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const int e = 4 * q + i;
                                double v = 0.0;
                                if (q < nq && e < len) {
                                    const uint32_t k = K[e];
                                    if (k != 0u) {
                                        const unsigned long long cp = comp_of(k, static_cast<uint32_t>(c0 + e));
                                        const float x = kval(k);
                                        if (cp >= st.xcross && cp >= st.kbound && x >= x_minp) {
                                            const float pf = static_cast<float>(static_cast<double>(weight_of(x, wc)) / zk_d);
                                            v = use_res ? fmax(0.0, static_cast<double>(pf) - static_cast<double>(q_of(qv, static_cast<uint32_t>(c0 + e))))
                                                        : static_cast<double>(pf);
                                        }
                                    }
                                }
                                vals[i] = v;
                                s += v;
                            }
                            double tot2 = 0.0;
                            const double incl = block_incl_f64(s, ls, &tot2);
                            double acc = run + incl - s;
                            unsigned long long cand = ~0ull;
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                acc += vals[i];
                                if (cand == ~0ull && vals[i] > 0.0 && acc > target)
                                    cand = static_cast<unsigned long long>(c0 + 4 * q + i);
                            }
                            found = block_min_bc(cand, ls);
                            run += tot2;
                        }
                        if (tid == 0) {
                            cluster.map_shared_rank(cs, 0)->result =
                                found != ~0ull ? static_cast<int>(found) : static_cast<int>(a.vocab - 1);
                        }
                    }
                    st.stage = kStDWait;
                    st.pending_kind = 2;
                }
            } else if (st.stage == kStDWait) {
                st.result = cs->result;  // meaningful in CTA 0, which writes the outputs
                st.stage = kStDone;
                st.pending_kind = 0;
            } else if (st.stage == kStCount) {
                unsigned long long nk = 0ull;
                for (uint32_t q = 0; q < C; ++q) nk += cs->cnt[q];
                st.result = static_cast<int32_t>(nk);
                st.stage = kStDone;
                st.pending_kind = 0;
            }
        }
        // ------------------------------------------------ apply a resolved selection
        if (have_sel) {
            const unsigned long long above_w = sel_bin > 0 ? CG[sel_bin - 1] : 0ull;
            if (st.stage == kStKBound) {
                st.kbound = sel;
                st.zk = above_w + wthrough;
                st.zkept = st.zk;
                st.stage = kStTopP;
            } else if (st.stage == kStTopP) {
                st.xcross = sel;
                st.zkept = above_w + cum_sel;
                st.stage = kStKept;
            } else {  // draw or residual
                st.result = static_cast<int32_t>(comp_id(sel));
                st.stage = kStDone;
            }
            st.pending_bin = -1;
        }
        // ------------------------------------------------ advance stages and issue the next exchange
        GatherReq gq{-1, 0, -1, -1, 0, 0ull};
        while (!st.err && st.stage != kStDone && st.pending_kind == 0) {
            if (st.stage == kStKBound) {
                const unsigned long long t = k_eff;
                int lo = 0, hi = kABins - 1;
                while (lo < hi) {
                    const int mid = (lo + hi) >> 1;
                    if (CGC[mid] >= t) hi = mid;
                    else lo = mid + 1;
                }
                st.target = t - (lo > 0 ? CGC[lo - 1] : 0u);
                st.pending_bin = lo;
                st.pending_kind = 1;
                gq = GatherReq{lo, cur, -1, -1, 0, 0ull};
            } else if (st.stage == kStTopP) {
                if (P->top_p > 0.0f && P->top_p < 1.0f) {
                    unsigned long long t1 = ceil_mass(P->top_p, st.zk);
                    if (t1 < 1ull) t1 = 1ull;
                    const int b = bin_of_target(t1);
                    st.target = t1 - (b > 0 ? CG[b - 1] : 0ull);
                    st.pending_bin = b;
                    st.pending_kind = 1;
                    // The kept mass will lie in [CG[b-1] + 1, CG[b]] (min-p can only lower it), so the
                    // draw lands in bins blo..bhi. When that range is narrow it is gathered now as
                    // well, into the other buffer (free: nothing was read from it in this round).
                    int blo = -1, bhi = -1;
                    if (draw_follows && !read_buf) {
                        unsigned long long zlo = (b > 0 ? CG[b - 1] : 0ull) + 1ull, zhi = CG[b];
                        if (P->min_p > 0.0f) {
                            zlo = zlo < Wmin ? zlo : Wmin;
                            zhi = zhi < Wmin ? zhi : Wmin;
                        }
                        if (zlo > 0ull) {
                            blo = bin_of_target(scale_mass(rc.u_draw, zlo) + 1ull);
                            bhi = bin_of_target(scale_mass(rc.u_draw, zhi) + 1ull);
                            if (bhi - blo >= kPreBins && !bins_fit(blo, bhi)) blo = bhi = -1;
                        }
                    }
                    if (blo >= 0 && !(blo == b && bhi == b)) {
                        gq = GatherReq{b, cur, blo, bhi, prev, st.kbound};
                        st.pre_buf = prev;
                    } else {
                        gq = GatherReq{b, cur, -1, -1, 0, st.kbound};
                        st.pre_buf = cur;  // the draw bin is the top-p bin
                    }
                    st.pre_lo = blo;
                    st.pre_hi = bhi;
                } else {
                    st.zkept = st.zk;
                    st.stage = kStKept;
                }
            } else if (st.stage == kStKept) {
                if (P->min_p > 0.0f && Wmin < st.zkept) st.zkept = Wmin;
                if (MODE == kModeCandidates) {
                    uint32_t c = 0;
                    for (int e = tid; e < len; e += kNT) {
                        const uint32_t k = K[e];
                        if (k == 0u) continue;
                        const unsigned long long cp = comp_of(k, static_cast<uint32_t>(c0 + e));
                        if (cp >= st.xcross && cp >= st.kbound && kval(k) >= x_minp) ++c;
                    }
                    const unsigned long long tc = block_sum_u64<kNT>(c, ls->red);
                    if (tid < static_cast<int>(C)) cluster.map_shared_rank(cs, tid)->cnt[crank] = tc;
                    st.stage = kStCount;
                    remote = true;
                    st.pending_kind = 2;
                } else if (MODE == kModeVerify && rc.vrole == 0) {
                    const bool kept = dvalid && dcomp >= st.xcross && dcomp >= st.kbound && xd >= x_minp;
                    double pd = 0.0;
                    if (kept) {
                        const double ed = exp(static_cast<double>(xd) * invT - maxs);
                        pd = ed / (static_cast<double>(st.zkept) / kWeightScale);
                    }
                    const bool in_range = rc.draft >= 0 && static_cast<uint32_t>(rc.draft) < a.vocab;
                    if (a.q != nullptr || a.qlog != nullptr) {
                        const QView qv = q_view(a, static_cast<size_t>(rc.stream) * a.k + rc.vidx);
                        const float p_d = static_cast<float>(pd);
                        const float q_d = in_range ? q_of(qv, static_cast<uint32_t>(rc.draft)) : 1.0f;
                        const double accept_prob = (q_d <= 0.0f) ? (p_d > 0.0f ? 1.0 : 0.0)
                            : fmin(1.0, static_cast<double>(p_d) / fmax(1e-12, static_cast<double>(q_d)));
                        res_accept = rc.u_accept < accept_prob ? 1 : 0;
                        if (res_accept) {
                            st.stage = kStDone;
                        } else {
                            // partial sums of the residual and of p_target over this chunk
                            const double zk_d = static_cast<double>(st.zkept);
                            double rsum = 0.0, psum = 0.0;
                            for (int e = tid; e < len; e += kNT) {
                                const uint32_t k = K[e];
                                if (k == 0u) continue;
                                const unsigned long long cp = comp_of(k, static_cast<uint32_t>(c0 + e));
                                const float x = kval(k);
                                if (!(cp >= st.xcross && cp >= st.kbound && x >= x_minp)) continue;
                                const float pf = static_cast<float>(static_cast<double>(weight_of(x, wc)) / zk_d);
                                rsum += fmax(0.0, static_cast<double>(pf) - static_cast<double>(q_of(qv, static_cast<uint32_t>(c0 + e))));
                                psum += static_cast<double>(pf);
                            }
                            rsum = block_sum_f64(rsum, ls);
                            psum = block_sum_f64(psum, ls);
                            if (tid < static_cast<int>(C)) {
                                ClusterShared* dst = cluster.map_shared_rank(cs, tid);
                                dst->rsum[crank] = rsum;
                                dst->psum[crank] = psum;
                            }
                            st.stage = kStDSum;
                            remote = true;
                            st.pending_kind = 2;
                        }
                    } else {
                        res_accept = rc.u_accept < pd ? 1 : 0;
                        if (res_accept) {
                            st.stage = kStDone;
                        } else {
                            const unsigned long long wd = kept ? weight_of(xd, wc) : 0ull;
                            const unsigned long long zr = st.zkept - wd;
                            if (zr > 0ull) {
                                st.excl = kept ? dcomp : 0ull;
                                st.wexcl = wd;
                                const unsigned long long t = scale_mass(rc.u_draw, zr) + 1ull;
                                const int bd = kept ? xbin_g(dkey) : kABins;
                                int lo = 0, hi = kABins - 1;
                                while (lo < hi) {
                                    const int mid = (lo + hi) >> 1;
                                    const unsigned long long cgm = CG[mid] - (mid >= bd ? wd : 0ull);
                                    if (cgm >= t) hi = mid;
                                    else lo = mid + 1;
                                }
                                const unsigned long long ab = lo > 0 ? CG[lo - 1] - ((lo - 1) >= bd ? wd : 0ull) : 0ull;
                                st.target = t - ab;
                                st.stage = kStResid;
                                st.pending_bin = lo;
                                st.pending_kind = 1;
                                gq = GatherReq{lo, cur, -1, -1, 0, st.kbound};
                            } else {
                                st.stage = kStDraw;  // residual empty: draw from the kept set
                            }
                        }
                    }
                } else {
                    st.stage = kStDraw;
                }
            } else if (st.stage == kStDraw) {
                const unsigned long long t = scale_mass(rc.u_draw, st.zkept) + 1ull;
                const int b = bin_of_target(t);
                st.target = t - (b > 0 ? CG[b - 1] : 0ull);
                st.pending_bin = b;
                st.tabs = t;
                if (st.pre_lo >= 0 && b >= st.pre_lo && b <= st.pre_hi) {
                    // gathered with the top-p bin: select over the whole prefetched range now
                    st.target = t - (st.pre_lo > 0 ? CG[st.pre_lo - 1] : 0ull);
                    st.pending_kind = 4;
                } else if (read_buf && st.pre_lo >= 0) {
                    // unreachable when the prediction holds; the prefetch buffer may still be read
                    // by this round's resolution, so the gather waits for the next round
                    st.pre_lo = -1;
                    st.pending_kind = 5;
                } else {
                    st.pre_lo = -1;
                    st.pending_kind = 1;
                    gq = GatherReq{b, cur, -1, -1, 0, st.kbound};
                }
            } else {
                st.err = 4;
            }
        }
        if (gq.bA >= 0) {
            gather(gq.bA, gq.bufA, gq.bBlo, gq.bBhi, gq.bufB, gq.lowb);  // the one gather site
            remote = true;
        }
        if (st.pending_kind != 4) break;
        }  // pass
        // A round that ends the row and neither read nor wrote a peer's shared memory needs no
        // barrier: no CTA of the cluster touches another's memory again. The condition is
        // cluster-uniform (the state advances identically in every CTA).
        if ((st.stage == kStDone || st.err) && !remote) break;
        cluster.sync();  // ============================================ one barrier per round
        if (st.pending_kind == 5) {  // deferred draw gather (see kStDraw)
            st.pending_kind = 0;
            st.stage = kStDraw;
        }
    }
    if (st.stage != kStDone && !st.err) st.err = 5;

    if (st.err) {
        res_status = SIXI_BACKEND_ERROR;
        res_token = -1;
    } else if (MODE == kModeSample || (MODE == kModeVerify && (rc.vrole == 1 || !res_accept))) {
        res_token = st.result;
    } else if (MODE == kModeCandidates && crank == 0) {
        // the best fl_n merged candidates that are kept, with their probabilities
        const uint32_t nkept = static_cast<uint32_t>(st.result);
        const uint32_t nout = fl_n < nkept ? fl_n : nkept;
        const double zk_d = static_cast<double>(st.zkept) / kWeightScale;
        if (static_cast<uint32_t>(tid) < nout) {
            const unsigned long long c = FL[tid];
            const double e = exp(static_cast<double>(kval(comp_key(c))) * invT - maxs);
            a.out_ids[static_cast<size_t>(row) * a.max_out + tid] = static_cast<int32_t>(comp_id(c));
            a.out_probs[static_cast<size_t>(row) * a.max_out + tid] = e / zk_d;
        }
        if (tid == 0) a.out_count[row] = static_cast<int32_t>(nkept);
    }
    write_outputs();
}

// ---------------------------------------------------------------------------------------------
// per-stream verification finalize: first rejected draft, committed tokens, uniforms used
// (speculative.cpp:801-916 / 630-692 decision order)

inline __global__ void verify_finalize_kernel(const RowArgs a, uint32_t n_streams, int32_t* out_accepted,
                                              int32_t* out_tokens, int32_t* out_n_tokens,
                                              int32_t* out_first_reject, int32_t* out_uniforms_used,
                                              int32_t* out_status) {
    const uint32_t s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= n_streams) return;
    const uint32_t kp1 = a.k + 1;
    const int32_t nd = a.n_drafts ? a.n_drafts[s] : static_cast<int32_t>(a.k);
    int32_t* out = out_tokens + static_cast<size_t>(s) * kp1;
    for (uint32_t i = 0; i < kp1; ++i) out[i] = -1;
    if (nd < 0 || nd > static_cast<int32_t>(a.k)) {
        out_accepted[s] = 0;
        out_n_tokens[s] = 0;
        out_first_reject[s] = -1;
        out_uniforms_used[s] = 0;
        out_status[s] = SIXI_INVALID_ARGUMENT;
        return;
    }
    const VerifyRowResult* w = a.ws + static_cast<size_t>(s) * kp1;
    const int32_t* d = a.drafts + static_cast<size_t>(s) * a.k;
    const bool greedy = a.params[s].temperature <= 0.0f;
    int32_t status = SIXI_OK, acc = 0, n = 0, first_reject = -1, used = 0;
    for (int32_t i = 0; i <= nd; ++i) {
        const VerifyRowResult r = w[i];
        if (r.status != SIXI_OK) {
            if (greedy && r.status == SIXI_NUMERIC_NAN_OR_INF) {
                if (status == SIXI_OK) status = r.status;
            } else {
                status = r.status;
                break;
            }
        }
        if (i == nd) {  // bonus
            out[n++] = r.token;
            if (!greedy) ++used;
            break;
        }
        if (greedy) {
            if (r.token == d[i]) {
                out[n++] = d[i];
                ++acc;
            } else {
                out[n++] = r.token;
                first_reject = i;
                break;
            }
        } else {
            ++used;
            if (r.accept) {
                out[n++] = d[i];
                ++acc;
            } else {
                out[n++] = r.token;
                ++used;
                first_reject = i;
                break;
            }
        }
    }
    if (status != SIXI_OK && status != SIXI_NUMERIC_NAN_OR_INF) {
        for (uint32_t i = 0; i < kp1; ++i) out[i] = -1;
        n = 0;
        acc = 0;
        first_reject = -1;
    }
    out_accepted[s] = acc;
    out_n_tokens[s] = n;
    out_first_reject[s] = first_reject;
    out_uniforms_used[s] = used;
    out_status[s] = status;
}

// ---------------------------------------------------------------------------------------------
// launch of one (mode, dtype) kernel; defined in smp_inst.cu, compiled once per pair

template <int MODE, int DT>
cudaError_t launch_mode_dt(const RowArgs& a, const LaunchPlan& plan, cudaStream_t stream);

#define SIXI_DECL_INST(M, D) \
    template <>              \
    cudaError_t launch_mode_dt<M, D>(const RowArgs& a, const LaunchPlan& plan, cudaStream_t stream);
SIXI_DECL_INST(kModeSample, SIXI_SMP_F32)
SIXI_DECL_INST(kModeSample, SIXI_SMP_BF16)
SIXI_DECL_INST(kModeCandidates, SIXI_SMP_F32)
SIXI_DECL_INST(kModeCandidates, SIXI_SMP_BF16)
SIXI_DECL_INST(kModeGreedy, SIXI_SMP_F32)
SIXI_DECL_INST(kModeGreedy, SIXI_SMP_BF16)
SIXI_DECL_INST(kModeVerify, SIXI_SMP_F32)
SIXI_DECL_INST(kModeVerify, SIXI_SMP_BF16)
#undef SIXI_DECL_INST

}  // namespace sixi_b200
