#pragma once
// smp_row.cuh - the B200 (sm_100a) row engine behind sixi_smp_sample / _candidates /
// _greedy_argmax / _verify.
//
// One cluster of kC CTAs owns one logits row. CTA c bulk-copies (TMA, cp.async.bulk) its
// contiguous chunk of the row from HBM into shared memory once, converts it to 32-bit monotone
// keys held in registers while applying the grammar mask, the NaN/Inf check and the
// repetition/presence penalties, and from then on every step (argmax, top-k, softmax mass,
// top-p / min-p crossing, the draw, the verifier's accept test and residual) runs on the
// register-resident row with block reductions and DSMEM exchanges inside the cluster. HBM is read
// exactly once per row: the path is bandwidth-bound and uses no tensor cores.
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
//     (key, id) composites. Integer masses make every CTA reach identical decisions.
//
// Cluster barriers: every cluster.sync() sits at the top level of the kernel, and whether a CTA
// reaches the next one depends only on data every CTA of the cluster holds identically (the
// exchanged row statistics, the assembled histograms, gathered sets and pushed partial results),
// so all CTAs of a cluster take the same barriers. The only wait the kernel spins on (the
// mbarrier of its own bulk copy) is bounded and reports SIXI_BACKEND_ERROR on expiry.
#include <cooperative_groups.h>

#include <cfloat>
#include <climits>

#include "smp_device.cuh"
#include "smp_kernels.cuh"

namespace cg = cooperative_groups;

namespace sixi_b200 {

constexpr int kC = 8;          // CTAs per row (cluster size)
constexpr int kNT = 256;       // threads per CTA
constexpr int kNW = kNT / 32;  // warps per CTA
constexpr int kKS = 256;       // max candidates of the list path
constexpr int kLCap = 1024;    // local candidate superset capacity
constexpr int kGCap = 1024;    // gathered-bin capacity
constexpr int kSeg = kABins / kC;
constexpr int kMaxRounds = 48; // bound on the mass path's exchange rounds (normally 2-5)
constexpr uint32_t kWaitIters = 1u << 24;
constexpr uint32_t kNoList = 0xFFFFFFFFu;
constexpr int kMaxSmem = 227 * 1024;  // per-block opt-in limit of sm_100

static_assert(kNT == 256 && kNW == 8, "block primitives assume 8 warps");
static_assert(kKS <= kNT, "list path assumes one candidate per thread");

// ---------------------------------------------------------------------------------------------
// shared memory layout

struct RowStat {
    unsigned long long best;   // max composite (key, id) over valid entries; 0 if none
    unsigned long long first;  // (first allowed id << 1) | raw-NaN flag; ~0 if none
    unsigned long long dkey;   // (1 << 32) | key of the draft token if it lies in this chunk
    unsigned int min_key;      // min key over valid entries
    unsigned int n_allowed;    // allowed in-range entries
    unsigned int bad;          // bit 0: an allowed entry was NaN/Inf; bit 1: copy wait expired
    unsigned int pad;
};

struct ClusterShared {  // written by remote CTAs of the cluster
    RowStat xs[kC];
    unsigned long long z[kC];     // partial weight sums
    unsigned long long wmin[kC];  // partial min-p prefix weight
    unsigned long long segw[kC];  // reduced segment weight totals (unused beyond checks)
    unsigned long long cnt[kC];   // partial counts
    double rsum[kC];              // dense residual partial sums
    double psum[kC];              // dense fallback (p_target) partial sums
    unsigned long long mm[kC];    // refine: (min key << 32) | max key of the bin's entries
    unsigned long long rcnt[kC];  // refine: tie counts
    unsigned long long rsel;      // refine: composite of the crossing tie (from its owner)
    unsigned int lcnt[kC];        // list path: list lengths pushed to CTA 0
    unsigned int gcnt[2];         // gather buffer counters
    int result;                   // token sent to CTA 0 by the dense-residual owner
    int pad;
};

struct LocalShared {
    unsigned long long red[kNW * 8];
    unsigned int red32[kNW];
    unsigned long long bc[16];  // broadcast scalars
    double bcd[kNW];
    uint64_t mbar[1];
};

struct Layout {
    uint32_t off_ls, off_hb, off_mw, off_dyn;
    // work area (relative to off_dyn)
    uint32_t off_h, off_hc, off_r, off_rc, off_cg, off_cgc, off_g0, off_g1, off_bh, off_bw;
    uint32_t off_ll, off_ma, off_fl, off_fp, off_fq;
    uint32_t dyn_bytes, total;
};

__host__ __device__ inline uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline Layout make_layout(uint32_t chunk) {
    Layout L{};
    uint32_t o = align_up(static_cast<uint32_t>(sizeof(ClusterShared)), 16);
    L.off_ls = o;
    o = align_up(o + static_cast<uint32_t>(sizeof(LocalShared)), 16);
    L.off_hb = o;
    o = align_up(o + 4u * (chunk / 32u + 2u), 16);
    L.off_mw = o;
    o = align_up(o + 4u * (chunk / 32u + 4u), 128);
    L.off_dyn = o;
    // Work area. Lifetimes: the thread-maximum histogram (u32) aliases H and the local list LL
    // aliases CG (both die before the first cluster barrier); the list-path merge area MA aliases
    // the two gather buffers (MA dies before the first gather).
    uint32_t w = 0;
    L.off_h = w;   w += 8u * kABins;
    L.off_hc = w;  w += 4u * kABins;
    L.off_r = w;   w += 8u * kSeg;
    L.off_rc = w;  w += 4u * kSeg;
    L.off_cg = w;  w += 8u * kABins;
    L.off_cgc = w; w += 4u * kABins;
    L.off_ll = L.off_cg;
    L.off_g0 = w;  w += 8u * kGCap;
    L.off_g1 = w;  w += 8u * kGCap;
    L.off_ma = L.off_g0;
    L.off_bh = w;  w += 4u * 256u;
    L.off_bw = w;  w += 8u * 256u;
    L.off_fl = w;  w += 8u * kKS;
    L.off_fp = w;  w += 8u * kKS;
    L.off_fq = w;  w += 8u * kKS;
    const uint32_t stg = 4u * chunk;
    L.dyn_bytes = w > stg ? w : stg;
    L.total = L.off_dyn + L.dyn_bytes;
    return L;
}
static_assert(8 * kC * kKS <= 2 * 8 * kGCap, "MA must fit in the gather buffers");
static_assert(8 * kLCap <= 8 * kABins, "LL must fit in CG");

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
        r.n_extra = r.vrole == 0 ? static_cast<int32_t>(i) : (a.q ? 0 : (nd > 0 ? nd : 0));
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
        // the raw-argmax entry passes one default record for all rows
        r.p = (MODE == kModeGreedy) ? a.params : &a.params[row];
        r.greedy = (MODE == kModeGreedy) ? 1 : (r.p->temperature <= 0.0f);
        if (a.hist && a.hist_off && MODE != kModeGreedy) {
            r.hist = a.hist + a.hist_off[row];
            r.nh = a.hist_off[row + 1] - a.hist_off[row];
        }
        if (MODE == kModeSample && !r.greedy) r.u_draw = row_uniform(a, r.p, row, 0);
    }
    if (a.mask != nullptr && (MODE == kModeGreedy || (r.p->flags & SIXI_SMP_ROW_MASKED))) {
        r.mask = a.mask + static_cast<size_t>(row) * a.mask_words;
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

template <int SW>
__device__ __forceinline__ int elem_of(int j, int i) {
    return SW * (static_cast<int>(threadIdx.x) + kNT * j) + i;
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

// smallest value over the block of v (u64), all threads get it
__device__ __forceinline__ unsigned long long block_min_bc(unsigned long long v, LocalShared* ls) {
    return block_min_u64<kNT>(v, ls->red);
}

// ---------------------------------------------------------------------------------------------
// Exact selection over a shared-memory array of unique composites (block-wide, all threads call).
// Considers entries c with c >= lowb and c != excl. Finds the first entry in descending order at
// which the running sum (count, or weight when wc != nullptr) reaches `target` (>= 1) and returns
// it; *cum_through receives the running sum through it. Returns 0 when the target is not reached.
inline __device__ unsigned long long block_select(const unsigned long long* g, uint32_t n,
                                           unsigned long long target, const WeightCtx* wc,
                                           unsigned long long lowb, unsigned long long excl,
                                           uint32_t* bh, unsigned long long* bw, LocalShared* ls,
                                           unsigned long long* cum_through) {
    const int tid = threadIdx.x;
    unsigned long long andv = ~0ull, orv = 0ull;
    uint32_t cnt_l = 0;
    for (uint32_t i = tid; i < n; i += kNT) {
        const unsigned long long c = g[i];
        if (c < lowb || c == excl) continue;
        andv &= c;
        orv |= c;
        ++cnt_l;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        andv &= __shfl_xor_sync(0xFFFFFFFFu, andv, o);
        orv |= __shfl_xor_sync(0xFFFFFFFFu, orv, o);
    }
    cnt_l = warp_sum_u32(cnt_l);
    __syncthreads();
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
    __syncthreads();
    *cum_through = 0;
    if (ncons == 0) return 0ull;
    if (ncons == 1) {
        const unsigned long long w = wc ? weight_of(kval(comp_key(andv)), *wc) : 1ull;
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
    for (int level = 0; level < 9 && top >= 0; ++level) {
        const int shift = top - 7 > 0 ? top - 7 : 0;
        const int width = top - shift + 1;
        const unsigned int nd = 1u << width;
        for (int i = tid; i < 256; i += kNT) {
            bh[i] = 0;
            bw[i] = 0;
        }
        __syncthreads();
        for (uint32_t i = tid; i < n; i += kNT) {
            const unsigned long long c = g[i];
            if (c < lowb || c == excl || (c & pmask) != prefix) continue;
            const unsigned int d = static_cast<unsigned int>(c >> shift) & (nd - 1u);
            atomicAdd(&bh[d], 1u);
            if (wc) atomicAdd(&bw[d], weight_of(kval(comp_key(c)), *wc));
        }
        __syncthreads();
        if (tid < 32) {
            unsigned long long part[8];
            unsigned long long lsum = 0;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const int d = 255 - (tid * 8 + q);
                unsigned long long v = 0;
                if (d < static_cast<int>(nd)) v = wc ? bw[d] : static_cast<unsigned long long>(bh[d]);
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
                    ls->bc[0] = static_cast<unsigned long long>(fd);
                    ls->bc[1] = ab;
                    ls->bc[2] = bh[fd];
                }
            } else if (tid == 0) {
                ls->bc[0] = ~0ull;
            }
        }
        __syncthreads();
        const unsigned long long fd = ls->bc[0];
        if (fd == ~0ull) {
            __syncthreads();
            return 0ull;
        }
        base = ls->bc[1];
        const unsigned long long cnt = ls->bc[2];
        prefix |= fd << shift;
        pmask |= (static_cast<unsigned long long>(nd) - 1ull) << shift;
        __syncthreads();
        if (cnt == 1ull || shift == 0) {
            for (uint32_t i = tid; i < n; i += kNT) {
                const unsigned long long c = g[i];
                if (c < lowb || c == excl || (c & pmask) != prefix) continue;
                ls->bc[3] = c;
            }
            __syncthreads();
            const unsigned long long c = ls->bc[3];
            __syncthreads();
            const unsigned long long w = wc ? weight_of(kval(comp_key(c)), *wc) : 1ull;
            *cum_through = base + w;
            return c;
        }
        top = shift - 1;
    }
    return 0ull;
}

// ---------------------------------------------------------------------------------------------
// mass-path state machine stages
enum Stage : int {
    kStKBound = 0,   // find the k-th candidate (count select)
    kStTopP = 1,     // top-p crossing (weight select)
    kStKept = 2,     // min-p, then the verifier's accept test
    kStDraw = 3,     // the draw (weight select)
    kStResid = 4,    // one-hot residual draw without the draft (weight select)
    kStDSum = 5,     // dense residual: partial sums pushed
    kStDFind = 6,    // dense residual: owner CTA finds the token, sends it to CTA 0
    kStDWait = 7,    // dense residual: CTA 0 reads the token
    kStCount = 8,    // candidates: kept count partials pushed
    kStDone = 9
};

struct LState {
    int stage;
    int pending_bin;  // bin gathered this round (-1 none)
    int pending_kind; // 0 none, 1 gather, 2 exchange, 3 refine
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

template <int EPT, int DT, int MODE>
__global__ void __launch_bounds__(kNT, (EPT <= 80) ? 2 : 1) row_kernel(const RowArgs a) {
    constexpr int SW = (DT == SIXI_SMP_BF16) ? 8 : 4;
    constexpr int NV = EPT / SW;
    constexpr int ESZ = (DT == SIXI_SMP_BF16) ? 2 : 4;
    static_assert(EPT % 8 == 0, "EPT must be a multiple of 8");

    extern __shared__ __align__(128) uint8_t smem[];
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t crank = cluster.block_rank();
    const uint32_t row = blockIdx.x / kC;
    const int tid = threadIdx.x;
    const Layout lay = make_layout(a.chunk);

    ClusterShared* cs = reinterpret_cast<ClusterShared*>(smem);
    LocalShared* ls = reinterpret_cast<LocalShared*>(smem + lay.off_ls);
    uint32_t* hb = reinterpret_cast<uint32_t*>(smem + lay.off_hb);
    uint32_t* mw = reinterpret_cast<uint32_t*>(smem + lay.off_mw);
    uint8_t* dyn = smem + lay.off_dyn;
    float* stg = reinterpret_cast<float*>(dyn);
    unsigned long long* H = reinterpret_cast<unsigned long long*>(dyn + lay.off_h);
    uint32_t* H32 = reinterpret_cast<uint32_t*>(dyn + lay.off_h);
    uint32_t* HC = reinterpret_cast<uint32_t*>(dyn + lay.off_hc);
    unsigned long long* R = reinterpret_cast<unsigned long long*>(dyn + lay.off_r);
    uint32_t* RC = reinterpret_cast<uint32_t*>(dyn + lay.off_rc);
    unsigned long long* CG = reinterpret_cast<unsigned long long*>(dyn + lay.off_cg);
    uint32_t* CGC = reinterpret_cast<uint32_t*>(dyn + lay.off_cgc);
    unsigned long long* LL = reinterpret_cast<unsigned long long*>(dyn + lay.off_ll);
    unsigned long long* G0 = reinterpret_cast<unsigned long long*>(dyn + lay.off_g0);
    unsigned long long* G1 = reinterpret_cast<unsigned long long*>(dyn + lay.off_g1);
    uint32_t* BH = reinterpret_cast<uint32_t*>(dyn + lay.off_bh);
    unsigned long long* BW = reinterpret_cast<unsigned long long*>(dyn + lay.off_bw);
    unsigned long long* MA = reinterpret_cast<unsigned long long*>(dyn + lay.off_ma);
    unsigned long long* FL = reinterpret_cast<unsigned long long*>(dyn + lay.off_fl);
    double* FP = reinterpret_cast<double*>(dyn + lay.off_fp);
    double* FQ = reinterpret_cast<double*>(dyn + lay.off_fq);

    const RowCtx rc = make_row_ctx<MODE>(a, row);
    const sixi_smp_params* P = rc.p;
    const int32_t c0 = static_cast<int32_t>(crank * a.chunk);
    int32_t len = static_cast<int32_t>(a.vocab) - c0;
    if (len < 0) len = 0;
    if (len > static_cast<int32_t>(a.chunk)) len = static_cast<int32_t>(a.chunk);
    if (!rc.active) len = 0;
    const uint8_t* gchunk = rc.row + static_cast<size_t>(c0) * ESZ;

    // ======================================================================== phase A
    // bulk copy of the chunk (fp32 at the start of the staging area, bf16 in its upper half)
    const int32_t tma_bytes = a.use_tma ? (len * ESZ) / 16 * 16 : 0;
    const int32_t len_t = tma_bytes / ESZ;
    uint8_t* stg_dst = (DT == SIXI_SMP_BF16) ? dyn + 2u * a.chunk : dyn;
    if (tid == 0) {
        mbar_init(&ls->mbar[0], 1);
        fence_mbar_init();
        if (tma_bytes > 0) {
            mbar_arrive_expect_tx(&ls->mbar[0], static_cast<uint32_t>(tma_bytes));
            for (int32_t off = 0; off < tma_bytes; off += 32768) {
                const int32_t nb = (tma_bytes - off) < 32768 ? (tma_bytes - off) : 32768;
                bulk_g2s(stg_dst + off, gchunk + off, static_cast<uint32_t>(nb), &ls->mbar[0]);
            }
        }
        cs->gcnt[0] = 0;
        cs->gcnt[1] = 0;
        cs->result = -1;
        ls->bc[15] = 0;
    }
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
    // unique history ids of this chunk -> bitmap (overlaps the bulk copy)
    if (rc.pen && len > 0) {
        for (int64_t j = tid; j < nht; j += kNT) {
            const int32_t t = hist_at(rc, j);
            if (t < c0 || t >= c0 + len || !allowed(t)) continue;
            const int32_t e = t - c0;
            atomicOr(&hb[e >> 5], 1u << (e & 31));
        }
    }
    if (tma_bytes > 0) {
        if (!mbar_wait(&ls->mbar[0], 0, kWaitIters)) ls->bc[15] = 1;
    }
    __syncthreads();
    if (pen_smem && len > 0) {
        // frequency-penalty rows: materialise the chunk as fp32 in shared memory, apply the
        // per-unique penalty, then the per-occurrence frequency penalty (identical addends, so the
        // order of the atomic updates does not change the result)
        if (DT == SIXI_SMP_BF16) {
            const uint16_t* src = reinterpret_cast<const uint16_t*>(dyn + 2u * a.chunk);
            for (int32_t t0 = 0; t0 < len; t0 += kNT * 8) {
                float v[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int32_t e = t0 + tid * 8 + i;
                    uint16_t b = 0;
                    if (e < len_t) b = src[e];
                    else if (e < len) b = reinterpret_cast<const uint16_t*>(gchunk)[e];
                    v[i] = __uint_as_float(static_cast<uint32_t>(b) << 16);
                }
                __syncthreads();
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int32_t e = t0 + tid * 8 + i;
                    if (e < len) stg[e] = v[i];
                }
                __syncthreads();
            }
        } else {
            for (int32_t e = len_t + tid; e < len; e += kNT) stg[e] = reinterpret_cast<const float*>(gchunk)[e];
            __syncthreads();
        }
        for (int64_t j = tid; j < nht; j += kNT) {
            const int32_t t = hist_at(rc, j);
            if (t < c0 || t >= c0 + len || !allowed(t)) continue;
            const int32_t e = t - c0;
            const uint32_t bit = 1u << (e & 31);
            const uint32_t old = atomicAnd(&hb[e >> 5], ~bit);
            if (old & bit) stg[e] = penalize(stg[e], P);
        }
        __syncthreads();
        for (int64_t j = tid; j < nht; j += kNT) {
            const int32_t t = hist_at(rc, j);
            if (t < c0 || t >= c0 + len || !allowed(t)) continue;
            atomicAdd(&stg[t - c0], -P->frequency_penalty);
        }
        __syncthreads();
    }

    // P0: shared / global -> register keys, with mask, NaN/Inf check and penalties
    uint32_t keys[EPT];
    unsigned long long t_best = 0ull, t_first = ~0ull, t_dkey = 0ull;
    uint32_t t_min = 0xFFFFFFFFu, t_n = 0u, t_bad = 0u;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const int e0 = SW * (tid + kNT * j);
        float xv[SW];
        if (pen_smem) {
#pragma unroll
            for (int i = 0; i < SW; ++i) xv[i] = (e0 + i < len) ? stg[e0 + i] : 0.0f;
        } else if (e0 + SW <= len_t) {
            if (DT == SIXI_SMP_BF16) {
                const uint4 v = *reinterpret_cast<const uint4*>(dyn + 2u * a.chunk + 2u * e0);
                const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    xv[2 * i] = __uint_as_float(w4[i] << 16);
                    xv[2 * i + 1] = __uint_as_float(w4[i] & 0xFFFF0000u);
                }
            } else {
                const float4 v = *reinterpret_cast<const float4*>(stg + e0);
                xv[0] = v.x;
                xv[1] = v.y;
                xv[2] = v.z;
                xv[3] = v.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < SW; ++i) {
                const int e = e0 + i;
                float x = 0.0f;
                if (e < len) {
                    if (DT == SIXI_SMP_BF16) {
                        const uint16_t b = reinterpret_cast<const uint16_t*>(gchunk)[e];
                        x = __uint_as_float(static_cast<uint32_t>(b) << 16);
                    } else {
                        x = reinterpret_cast<const float*>(gchunk)[e];
                    }
                }
                xv[i] = x;
            }
        }
        uint32_t mbits = (1u << SW) - 1u;
        if (rc.mask != nullptr && e0 < len) {
            const uint32_t g = static_cast<uint32_t>(c0 + e0);
            mbits = (mw[(g >> 5) - wbase] >> (g & 31)) & ((1u << SW) - 1u);
        }
        uint32_t pbits = 0;
        if (rc.pen && !pen_smem && e0 < len) pbits = (hb[e0 >> 5] >> (e0 & 31)) & ((1u << SW) - 1u);
#pragma unroll
        for (int i = 0; i < SW; ++i) {
            const int e = e0 + i;
            const bool ok = (e < len) && ((mbits >> i) & 1u);
            float x = xv[i];
            uint32_t k = 0u;
            if (ok) {
                const bool nan = isnan(x);
                if (!isfinite(x)) t_bad = 1u;
                const unsigned long long f = (static_cast<unsigned long long>(c0 + e) << 1) | (nan ? 1ull : 0ull);
                t_first = f < t_first ? f : t_first;
                ++t_n;
                if ((pbits >> i) & 1u) x = penalize(x, P);
                if (!isnan(x)) {
                    k = fkey(x);
                    const unsigned long long cp = comp_of(k, static_cast<uint32_t>(c0 + e));
                    t_best = cp > t_best ? cp : t_best;
                    t_min = k < t_min ? k : t_min;
                }
            }
            if (e < len && c0 + e == rc.draft) t_dkey = (1ull << 32) | k;
            keys[j * SW + i] = k;
        }
    }
    // block reduction of the row statistics; the result is pushed to every CTA of the cluster
    unsigned long long l_best;
    uint32_t l_n;
    {
        const unsigned long long v0 = warp_max_u64(t_best), v1 = warp_min_u64(t_first),
                                 v2 = warp_max_u64(t_dkey), v3 = warp_min_u64(t_min);
        const uint32_t v4 = warp_sum_u32(t_n);
        const uint32_t v5 = __reduce_or_sync(0xFFFFFFFFu, t_bad);
        const int w = tid >> 5;
        if ((tid & 31) == 0) {
            ls->red[w * 8 + 0] = v0;
            ls->red[w * 8 + 1] = v1;
            ls->red[w * 8 + 2] = v2;
            ls->red[w * 8 + 3] = v3;
            ls->red[w * 8 + 4] = v4;
            ls->red[w * 8 + 5] = v5;
        }
        __syncthreads();
        RowStat st;
        st.best = 0ull;
        st.first = ~0ull;
        st.dkey = 0ull;
        unsigned long long mn = ~0ull;
        uint32_t n = 0, bad = 0;
#pragma unroll
        for (int q = 0; q < kNW; ++q) {
            st.best = ls->red[q * 8 + 0] > st.best ? ls->red[q * 8 + 0] : st.best;
            st.first = ls->red[q * 8 + 1] < st.first ? ls->red[q * 8 + 1] : st.first;
            st.dkey = ls->red[q * 8 + 2] > st.dkey ? ls->red[q * 8 + 2] : st.dkey;
            mn = ls->red[q * 8 + 3] < mn ? ls->red[q * 8 + 3] : mn;
            n += static_cast<uint32_t>(ls->red[q * 8 + 4]);
            bad |= static_cast<uint32_t>(ls->red[q * 8 + 5]);
        }
        st.min_key = static_cast<uint32_t>(mn);
        st.n_allowed = n;
        st.bad = bad | (ls->bc[15] ? 2u : 0u);
        st.pad = 0;
        l_best = st.best;
        l_n = n;
        if (tid < kC) cluster.map_shared_rank(cs, tid)->xs[crank] = st;
        __syncthreads();
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
            // histogram of the per-thread maxima over exp-domain bins relative to the local max
            const float lmax = kval(comp_key(l_best));
            const float bscale = static_cast<float>(
                (kABins - 1) / (46.0 * 0.6931471805599453 * static_cast<double>(P->temperature)));
            auto xbin = [&](uint32_t key) -> int {
                const float d = (lmax - kval(key)) * bscale;
                int b = d > 0.0f ? static_cast<int>(d) : 0;
                return b < kABins - 1 ? b : kABins - 1;
            };
            unsigned long long tmax = 0ull;
#pragma unroll
            for (int q = 0; q < EPT; ++q) {
                if (keys[q] == 0u) continue;
                const unsigned long long cp = comp_of(keys[q], static_cast<uint32_t>(c0 + elem_of<SW>(q / SW, q % SW)));
                tmax = cp > tmax ? cp : tmax;
            }
            for (int i = tid; i < kABins; i += kNT) H32[i] = 0u;
            __syncthreads();
            if (tmax != 0ull) atomicAdd(&H32[xbin(comp_key(tmax))], 1u);
            __syncthreads();
            // b1 = first bin where the cumulative count of per-thread maxima reaches kl; then at
            // least kl entries lie in bins <= b1
            constexpr int PER = kABins / kNT;
            const int b0 = tid * PER;
            uint32_t s8 = 0;
#pragma unroll
            for (int q = 0; q < PER; ++q) s8 += H32[b0 + q];
            uint32_t tot = 0;
            const uint32_t ex = block_excl_u32<kNT>(s8, ls->red32, &tot);
            if (tid == 0) ls->bc[4] = kABins - 1;
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
            uint32_t mine = 0;
#pragma unroll
            for (int q = 0; q < EPT; ++q)
                if (keys[q] != 0u && xbin(keys[q]) <= b1) ++mine;
            uint32_t ncand = 0;
            uint32_t off = block_excl_u32<kNT>(mine, ls->red32, &ncand);
            unsigned long long thr = 0ull;
            if (ncand > static_cast<uint32_t>(kLCap)) {
                // too many: exact kl-th largest composite by a radix select over the registers
                uint32_t prefix = 0, pmask = 0, above = 0;
                for (int shift = 24; shift >= 0; shift -= 8) {
                    for (int i = tid; i < 256; i += kNT) BH[i] = 0u;
                    __syncthreads();
#pragma unroll
                    for (int q = 0; q < EPT; ++q) {
                        const uint32_t k = keys[q];
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
                for (int j = 0; j < NV; ++j) {
                    uint32_t t = 0;
#pragma unroll
                    for (int i = 0; i < SW; ++i) t += (keys[j * SW + i] == prefix) ? 1u : 0u;
                    uint32_t tot2 = 0;
                    const uint32_t ex2 = block_excl_u32<kNT>(t, ls->red32, &tot2);
                    uint32_t run = taken + ex2;
#pragma unroll
                    for (int i = 0; i < SW; ++i) {
                        if (keys[j * SW + i] != prefix) continue;
                        ++run;
                        if (run == need) ls->bc[7] = comp_of(prefix, static_cast<uint32_t>(c0 + elem_of<SW>(j, i)));
                    }
                    taken += tot2;
                }
                __syncthreads();
                thr = ls->bc[7];
                mine = 0;
#pragma unroll
                for (int q = 0; q < EPT; ++q) {
                    if (keys[q] == 0u) continue;
                    if (comp_of(keys[q], static_cast<uint32_t>(c0 + elem_of<SW>(q / SW, q % SW))) >= thr) ++mine;
                }
                off = block_excl_u32<kNT>(mine, ls->red32, &ncand);
            }
#pragma unroll
            for (int q = 0; q < EPT; ++q) {
                if (keys[q] == 0u) continue;
                const unsigned long long cp = comp_of(keys[q], static_cast<uint32_t>(c0 + elem_of<SW>(q / SW, q % SW)));
                const bool take = thr ? (cp >= thr) : (xbin(keys[q]) <= b1);
                if (take) LL[off++] = cp;
            }
            __syncthreads();
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
    unsigned long long best = 0ull, first = ~0ull, dkey = 0ull;
    uint32_t min_key = 0xFFFFFFFFu, n_allowed = 0, bad = 0;
#pragma unroll
    for (int q = 0; q < kC; ++q) {
        const RowStat& s = cs->xs[q];
        best = s.best > best ? s.best : best;
        first = s.first < first ? s.first : first;
        dkey = s.dkey > dkey ? s.dkey : dkey;
        min_key = s.min_key < min_key ? s.min_key : min_key;
        n_allowed += s.n_allowed;
        bad |= s.bad;
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
        const bool first_nan = (first != ~0ull) && (first & 1ull);
        res_token = (raw_argmax && (first_nan || best == 0ull)) ? static_cast<int32_t>(first >> 1)
                                                              : static_cast<int32_t>(comp_id(best));
        if (raw_argmax && (bad & 1u)) res_status = SIXI_NUMERIC_NAN_OR_INF;
    }

    const double invT = 1.0 / static_cast<double>(P->temperature);
    const float M = kval(comp_key(best));
    const double maxs = static_cast<double>(M) * invT;
    const bool dvalid = (dkey >> 32) != 0ull && static_cast<uint32_t>(dkey) != 0u;
    const float xd = dvalid ? kval(static_cast<uint32_t>(dkey)) : 0.0f;
    const unsigned long long dcomp = dvalid ? comp_of(static_cast<uint32_t>(dkey), static_cast<uint32_t>(rc.draft)) : 0ull;

    // merge of the pushed lists at CTA 0 into FL (sorted). Used by the list path and by the
    // candidates entry on the mass path.
    uint32_t fl_n = 0;
    const bool want_lists = crank == 0 && (path == 1 || (path == 2 && MODE == kModeCandidates));
    if (want_lists) {
        uint32_t total = 0;
        bool ok = true;
#pragma unroll
        for (int q = 0; q < kC; ++q) {
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
        for (int q = 0; q < kC && fl_n > 0; ++q) {
            const uint32_t nq = cs->lcnt[q];
            for (uint32_t pidx = tid; pidx < nq; pidx += kNT) {
                const unsigned long long v = MA[q * kKS + pidx];
                uint32_t rank = pidx;
#pragma unroll
                for (int o = 0; o < kC; ++o) {
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
        }
        __syncthreads();
    }
    // CTA-uniform for CTA 0 only; other CTAs skip the list path entirely
    if (crank == 0 && path == 1) {
        // fp64 softmax over the k candidates (core_execution.cpp:538-549)
        const uint32_t n = fl_n;
        const bool act = static_cast<uint32_t>(tid) < n;
        double e = 0.0;
        if (act) e = exp(static_cast<double>(kval(comp_key(FL[tid]))) * invT - maxs);
        const double sum_exp = block_sum_f64(e, ls);
        double prob = (sum_exp > 0.0) ? e / sum_exp : e;
        // top-p: keep through the first index with cumulative >= top_p (core_execution.cpp:551-575)
        uint32_t keep = n;
        double tot = 0.0;
        if (P->top_p > 0.0f && P->top_p < 1.0f) {
            const double cum = block_incl_f64(act ? prob : 0.0, ls, &tot);
            const bool hit = act && cum >= static_cast<double>(P->top_p);
            const unsigned long long first_hit = block_min_bc(hit ? static_cast<unsigned long long>(tid) : ~0ull, ls);
            keep = (first_hit == ~0ull) ? n : static_cast<uint32_t>(first_hit) + 1u;
            if (keep < n) {
                const double renorm = block_sum_f64(static_cast<uint32_t>(tid) < keep ? prob : 0.0, ls);
                if (renorm > 0.0) prob = prob / renorm;
            }
        }
        // min-p extension: keep prob >= min_p * max prob, renormalise
        if (P->min_p > 0.0f) {
            if (tid == 0) ls->bcd[0] = prob;
            __syncthreads();
            const double thr = static_cast<double>(P->min_p) * ls->bcd[0];
            __syncthreads();
            const bool drop = static_cast<uint32_t>(tid) < keep && prob < thr;
            const unsigned long long fd = block_min_bc(drop ? static_cast<unsigned long long>(tid) : ~0ull, ls);
            if (fd != ~0ull && fd >= 1ull && static_cast<uint32_t>(fd) < keep) {
                keep = static_cast<uint32_t>(fd);
                const double renorm = block_sum_f64(static_cast<uint32_t>(tid) < keep ? prob : 0.0, ls);
                if (renorm > 0.0) prob = prob / renorm;
            }
        }
        if (tid < kKS) FP[tid] = static_cast<uint32_t>(tid) < keep ? prob : 0.0;
        __syncthreads();
        // CDF draw in candidate order over FL/`pr` (core_execution.cpp:586-601)
        auto draw_list = [&](double u, const double* pr, const unsigned long long* ids, uint32_t nk) -> int32_t {
            double t2 = 0.0;
            const double v = static_cast<uint32_t>(tid) < nk ? pr[tid] : 0.0;
            const double cdf = block_incl_f64(v, ls, &t2);
            const bool hit = static_cast<uint32_t>(tid) < nk && u < cdf;
            const unsigned long long j = block_min_bc(hit ? static_cast<unsigned long long>(tid) : ~0ull, ls);
            const uint32_t jj = (j == ~0ull) ? nk - 1u : static_cast<uint32_t>(j);
            return static_cast<int32_t>(comp_id(ids[jj]));
        };
        if (MODE == kModeSample || (MODE == kModeVerify && rc.vrole == 1)) {
            res_token = draw_list(rc.u_draw, FP, FL, keep);
        } else if (MODE == kModeCandidates) {
            if (static_cast<uint32_t>(tid) < keep && static_cast<uint32_t>(tid) < a.max_out) {
                a.out_ids[static_cast<size_t>(row) * a.max_out + tid] = static_cast<int32_t>(comp_id(FL[tid]));
                a.out_probs[static_cast<size_t>(row) * a.max_out + tid] = FP[tid];
            }
            if (tid == 0) a.out_count[row] = static_cast<int32_t>(keep);
        } else if (MODE == kModeVerify) {
            const int32_t d = rc.draft;
            const bool kact = static_cast<uint32_t>(tid) < keep;
            const bool isd = kact && static_cast<int32_t>(comp_id(FL[tid])) == d;
            const unsigned long long dpos = block_min_bc(isd ? static_cast<unsigned long long>(tid) : ~0ull, ls);
            const double pd = (dpos == ~0ull) ? 0.0 : FP[dpos];
            const bool in_range = d >= 0 && static_cast<uint32_t>(d) < a.vocab;
            if (a.q != nullptr) {
                // dense draft probabilities (speculative.cpp:823-903)
                const float* qrow = a.q + (static_cast<size_t>(rc.stream) * a.k + rc.vidx) * a.row_stride;
                const float p_d = static_cast<float>(pd);
                const float q_d = in_range ? qrow[d] : 1.0f;
                const double accept_prob = (q_d <= 0.0f) ? (p_d > 0.0f ? 1.0 : 0.0)
                    : fmin(1.0, static_cast<double>(p_d) / fmax(1e-12, static_cast<double>(q_d)));
                res_accept = rc.u_accept < accept_prob ? 1 : 0;
                if (!res_accept) {
                    // residual max(0, p - q) is non-zero only on the kept candidates; walk them in
                    // vocabulary-id order
                    const uint32_t myid = kact ? comp_id(FL[tid]) : 0xFFFFFFFFu;
                    const float pf = kact ? static_cast<float>(FP[tid]) : 0.0f;
                    const double res = kact ? fmax(0.0, static_cast<double>(pf) - static_cast<double>(qrow[myid])) : 0.0;
                    uint32_t idr = 0;
                    if (kact) {
                        for (uint32_t j = 0; j < keep; ++j) idr += (comp_id(FL[j]) < myid) ? 1u : 0u;
                    }
                    const double res_sum = block_sum_f64(res, ls);
                    if (kact) {
                        FQ[idr] = (res_sum > 1e-12) ? res / res_sum : static_cast<double>(pf);
                        BH[idr] = myid;
                    }
                    __syncthreads();
                    double t3 = 0.0;
                    const double v = kact ? FQ[tid] : 0.0;
                    const double cdf = block_incl_f64(v, ls, &t3);
                    const bool hit = kact && rc.u_draw < cdf;
                    const unsigned long long j = block_min_bc(hit ? static_cast<unsigned long long>(tid) : ~0ull, ls);
                    res_token = (j == ~0ull) ? static_cast<int32_t>(a.vocab - 1) : static_cast<int32_t>(BH[j]);
                }
            } else {
                // one-hot drafts (speculative.cpp:638-681)
                res_accept = rc.u_accept < pd ? 1 : 0;
                if (!res_accept) {
                    const bool has_d = dpos != ~0ull;
                    const double res_sum = block_sum_f64((kact && !isd) ? FP[tid] : 0.0, ls);
                    const uint32_t m = keep - (has_d ? 1u : 0u);
                    if (m > 0 && res_sum > 0.0) {
                        const uint32_t pos = static_cast<uint32_t>(tid) - ((has_d && static_cast<unsigned long long>(tid) > dpos) ? 1u : 0u);
                        const double pv = (kact && !isd) ? FP[tid] / res_sum : 0.0;
                        const unsigned long long fv = (kact && !isd) ? FL[tid] : 0ull;
                        __syncthreads();
                        if (kact && !isd) {
                            FQ[pos] = pv;
                            LL[pos] = fv;
                        }
                        __syncthreads();
                        res_token = draw_list(rc.u_draw, FQ, LL, m);
                    } else {
                        res_token = draw_list(rc.u_draw, FP, FL, keep);
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
            a.out_tok[row] = ok ? res_token : -1;
            a.out_status[row] = res_status;
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
    {
        const float m = kval(min_key);
        double range = static_cast<double>(M) - static_cast<double>(m);
        const double cap = 46.0 * 0.6931471805599453 * static_cast<double>(P->temperature);
        if (range > cap) range = cap;
        make_weight_ctx(P->temperature, M, 46.0f, wc);
        wc.bin_scale = static_cast<float>((kABins - 1) / (range > 1e-30 ? range : 1e-30));
        if (P->min_p > 0.0f) {
            x_minp = static_cast<float>(static_cast<double>(M) +
                                        static_cast<double>(P->temperature) * log(static_cast<double>(P->min_p)));
        }
        for (int i = tid; i < kABins; i += kNT) {
            H[i] = 0ull;
            HC[i] = 0u;
        }
        __syncthreads();
        unsigned long long zp = 0ull, wp = 0ull;
#pragma unroll
        for (int q = 0; q < EPT; ++q) {
            const uint32_t k = keys[q];
            if (k == 0u) continue;
            const float x = kval(k);
            const unsigned long long w = weight_of(x, wc);
            zp += w;
            if (x >= x_minp) wp += w;
            if (w || need_counts) {
                const float dd = (M - x) * wc.bin_scale;
                int b = dd > 0.0f ? static_cast<int>(dd) : 0;
                b = b < kABins - 1 ? b : kABins - 1;
                if (w) atomicAdd(&H[b], w);
                if (need_counts) atomicAdd(&HC[b], 1u);
            }
        }
        zp = block_sum_u64<kNT>(zp, ls->red);
        wp = block_sum_u64<kNT>(wp, ls->red);
        if (tid < kC) {
            ClusterShared* dst = cluster.map_shared_rank(cs, tid);
            dst->z[crank] = zp;
            dst->wmin[crank] = wp;
        }
    }

    cluster.sync();  // ======================================================== CS2

    // reduce histogram segment `crank` over all CTAs of the cluster
    for (int i = tid; i < kSeg; i += kNT) {
        unsigned long long s = 0ull;
        uint32_t sc = 0;
#pragma unroll
        for (int q = 0; q < kC; ++q) {
            s += cluster.map_shared_rank(H, q)[crank * kSeg + i];
            if (need_counts) sc += cluster.map_shared_rank(HC, q)[crank * kSeg + i];
        }
        R[i] = s;
        RC[i] = sc;
    }
#pragma unroll
    for (int q = 0; q < kC; ++q) {
        Z += cs->z[q];
        Wmin += cs->wmin[q];
    }

    cluster.sync();  // ======================================================== CS3

    auto xbin_g = [&](uint32_t key) -> int {
        const float dd = (M - kval(key)) * wc.bin_scale;
        int b = dd > 0.0f ? static_cast<int>(dd) : 0;
        return b < kABins - 1 ? b : kABins - 1;
    };
    auto comp_at = [&](int q) -> unsigned long long {
        return comp_of(keys[q], static_cast<uint32_t>(c0 + elem_of<SW>(q / SW, q % SW)));
    };
    auto bin_of_target = [&](unsigned long long t) -> int {  // first bin with CG >= t
        int lo = 0, hi = kABins - 1;
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (CG[mid] >= t) hi = mid;
            else lo = mid + 1;
        }
        return lo;
    };
    // push my entries of bin b (composite >= lowb) into gather buffer gbuf of every CTA
    auto gather = [&](int b, int gbuf, unsigned long long lowb) {
        unsigned long long* gb = gbuf ? G1 : G0;
        const int lane = tid & 31;
#pragma unroll
        for (int q = 0; q < EPT; ++q) {
            const uint32_t k = keys[q];
            const unsigned long long cp = comp_at(q);
            const bool mine = k != 0u && xbin_g(k) == b && cp >= lowb;
            const unsigned ball = __ballot_sync(0xFFFFFFFFu, mine);
            if (ball == 0u) continue;
            const int leader = __ffs(ball) - 1;
            const uint32_t cnt = __popc(ball);
            const uint32_t rk = __popc(ball & ((1u << lane) - 1u));
#pragma unroll 1
            for (int dst = 0; dst < kC; ++dst) {
                uint32_t basei = 0;
                if (lane == leader) basei = atomicAdd(&cluster.map_shared_rank(cs, dst)->gcnt[gbuf], cnt);
                basei = __shfl_sync(0xFFFFFFFFu, basei, leader);
                if (mine && basei + rk < static_cast<uint32_t>(kGCap)) cluster.map_shared_rank(gb, dst)[basei + rk] = cp;
            }
        }
    };

    // every CTA assembles the same global cumulative histograms
    for (int i = tid; i < kABins; i += kNT) {
        CG[i] = cluster.map_shared_rank(R, i / kSeg)[i % kSeg];
        CGC[i] = need_counts ? cluster.map_shared_rank(RC, i / kSeg)[i % kSeg] : 0u;
    }
    __syncthreads();
    {
        constexpr int PER = kABins / kNT;
        unsigned long long v[PER];
        uint32_t vc[PER];
        unsigned long long s = 0ull;
        uint32_t sc = 0;
#pragma unroll
        for (int q = 0; q < PER; ++q) {
            v[q] = CG[tid * PER + q];
            vc[q] = CGC[tid * PER + q];
            s += v[q];
            sc += vc[q];
        }
        const unsigned long long inc = warp_incl_u64(s);
        const uint32_t incc = warp_incl_u32(sc);
        if ((tid & 31) == 31) {
            ls->red[tid >> 5] = inc;
            ls->red[kNW + (tid >> 5)] = incc;
        }
        __syncthreads();
        unsigned long long before = 0ull, beforec = 0ull;
        for (int w = 0; w < (tid >> 5); ++w) {
            before += ls->red[w];
            beforec += ls->red[kNW + w];
        }
        unsigned long long run = before + inc - s;
        uint32_t runc = static_cast<uint32_t>(beforec) + incc - sc;
#pragma unroll
        for (int q = 0; q < PER; ++q) {
            run += v[q];
            runc += vc[q];
            CG[tid * PER + q] = run;
            CGC[tid * PER + q] = runc;
        }
        __syncthreads();
    }

    // The state below is advanced identically in every CTA of the cluster: every decision reads
    // only cluster-uniform data (exchanged statistics, the assembled histograms, gathered sets,
    // pushed partial results), so the loop's early exit is uniform within the cluster.
    LState st{};
    st.stage = need_counts ? kStKBound : kStTopP;
    st.pending_bin = -1;
    st.pending_kind = 0;
    st.result = -1;
    st.err = 0;
    st.zk = Z;
    st.zkept = Z;
    st.kbound = 0ull;
    st.xcross = 0ull;
    st.excl = 0ull;
    st.wexcl = 0ull;
    Refine rf{};
    uint32_t* RH[2] = {reinterpret_cast<uint32_t*>(dyn + lay.off_h),
                       reinterpret_cast<uint32_t*>(dyn + lay.off_h) + 256};
    unsigned long long* RW[2] = {reinterpret_cast<unsigned long long*>(dyn + lay.off_h + 2048u),
                                 reinterpret_cast<unsigned long long*>(dyn + lay.off_h + 2048u) + 256};

    // entries of the selection `rf` describes (bin, lower bound, exclusion, key prefix)
    auto rf_match = [&](int q) -> bool {
        const uint32_t k = keys[q];
        if (k == 0u || (k & rf.pmask) != rf.prefix || xbin_g(k) != rf.bin) return false;
        const unsigned long long cp = comp_at(q);
        return cp >= rf.lowb && cp != rf.excl;
    };
    auto rf_build = [&](int buf) {  // local digit histogram of the refine level
        for (int i = tid; i < 256; i += kNT) {
            RH[buf][i] = 0u;
            RW[buf][i] = 0ull;
        }
        __syncthreads();
#pragma unroll
        for (int q = 0; q < EPT; ++q) {
            if (!rf_match(q)) continue;
            const uint32_t d = (keys[q] >> rf.shift) & ((1u << rf.width) - 1u);
            atomicAdd(&RH[buf][d], 1u);
            atomicAdd(&RW[buf][d], static_cast<unsigned long long>(weight_of(kval(keys[q]), wc)));
        }
        __syncthreads();
    };
    auto rf_level = [&](int top) {
        rf.top = top;
        rf.shift = top - 7 > 0 ? top - 7 : 0;
        rf.width = top - rf.shift + 1;
    };

    const double zero_d = 0.0;
    (void)zero_d;

#pragma unroll 1
    for (int round = 0; round < kMaxRounds; ++round) {
        if (st.stage == kStDone || st.err) break;
        const int cur = round & 1;
        const int prev = cur ^ 1;
        bool have_sel = false;
        unsigned long long sel = 0ull, cum_sel = 0ull, wthrough = 0ull;
        int sel_bin = st.pending_bin;
        // ------------------------------------------------ resolve what the previous round started
        if (st.pending_kind == 1) {
            const uint32_t n = cs->gcnt[prev];
            const unsigned long long lowb = (st.stage == kStKBound) ? 0ull : st.kbound;
            const unsigned long long ex = (st.stage == kStResid) ? st.excl : 0ull;
            const bool cmode = (st.stage == kStKBound);
            if (n > static_cast<uint32_t>(kGCap)) {
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
#pragma unroll
                for (int q = 0; q < EPT; ++q) {
                    if (!rf_match(q)) continue;
                    lo = keys[q] < lo ? keys[q] : lo;
                    hi = keys[q] > hi ? keys[q] : hi;
                }
                const unsigned long long l2 = block_min_u64<kNT>(lo, ls->red);
                const unsigned long long h2 = block_max_u64<kNT>(hi, ls->red);
                if (tid < kC) cluster.map_shared_rank(cs, tid)->mm[crank] = (l2 << 32) | h2;
                st.pending_kind = 3;
            } else {
                const unsigned long long* gp = prev ? G1 : G0;
                sel = block_select(gp, n, st.target, cmode ? nullptr : &wc, lowb, ex, BH, BW, ls, &cum_sel);
                if (sel == 0ull) {
                    st.err = 2;
                } else {
                    have_sel = true;
                    if (cmode) {
                        unsigned long long wpart = 0ull;
                        for (uint32_t i = tid; i < n; i += kNT) {
                            const unsigned long long c = gp[i];
                            if (c >= sel) wpart += weight_of(kval(comp_key(c)), wc);
                        }
                        wthrough = block_sum_u64<kNT>(wpart, ls->red);
                    }
                }
                st.pending_kind = 0;
            }
            __syncthreads();
            if (tid == 0) cs->gcnt[prev] = 0u;  // refilled two rounds later, after a barrier
        } else if (st.pending_kind == 3) {
            if (rf.phase == 0) {
                uint32_t klo = 0xFFFFFFFFu, khi = 0u;
#pragma unroll
                for (int q = 0; q < kC; ++q) {
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
                const int d = tid;  // kNT == 256 digits
                unsigned long long sc = 0ull, sw = 0ull;
#pragma unroll
                for (int q = 0; q < kC; ++q) {
                    sc += cluster.map_shared_rank(RH[rf.buf], q)[d];
                    sw += cluster.map_shared_rank(RW[rf.buf], q)[d];
                }
                BH[d] = static_cast<uint32_t>(sc);
                BW[d] = sw;
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
                const unsigned long long w = rf.cmode ? 1ull : weight_of(kval(rf.prefix), wc);
                const unsigned long long done_sel = rf.cmode ? rf.above_c : rf.above_w;
                if (w == 0ull || rf.t <= done_sel) {
                    st.err = 8;
                } else {
                    const unsigned long long idx = (rf.t - done_sel + w - 1ull) / w - 1ull;
                    unsigned long long before = 0ull;
                    int owner = -1;
                    for (int q = 0; q < kC; ++q) {
                        const unsigned long long c = cs->rcnt[q];
                        if (owner < 0 && idx < before + c) {
                            owner = q;
                            break;
                        }
                        before += c;
                    }
                    if (owner < 0) {
                        st.err = 9;
                    } else {
                        rf.above_c += idx;  // count before the crossing tie (excl.)
                        rf.above_w += idx * w;
                        rf.tie_w = w;
                        if (owner == static_cast<int>(crank)) {
                            const unsigned long long li = idx - before;
                            unsigned long long taken = 0ull;
                            if (tid == 0) ls->bc[13] = 0ull;
                            for (int j = 0; j < NV; ++j) {
                                uint32_t t = 0;
#pragma unroll
                                for (int i = 0; i < SW; ++i) t += rf_match(j * SW + i) ? 1u : 0u;
                                uint32_t tot = 0;
                                const uint32_t ex2 = block_excl_u32<kNT>(t, ls->red32, &tot);
                                unsigned long long r2 = taken + ex2;
#pragma unroll
                                for (int i = 0; i < SW; ++i) {
                                    if (!rf_match(j * SW + i)) continue;
                                    if (r2 == li) ls->bc[13] = comp_at(j * SW + i);
                                    ++r2;
                                }
                                taken += tot;
                            }
                            __syncthreads();
                            if (tid < kC) cluster.map_shared_rank(cs, tid)->rsel = ls->bc[13];
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
#pragma unroll
                    for (int q = 0; q < EPT; ++q) c += rf_match(q) ? 1u : 0u;
                    const unsigned long long tc = block_sum_u64<kNT>(c, ls->red);
                    if (tid < kC) cluster.map_shared_rank(cs, tid)->rcnt[crank] = tc;
                }
            }
        } else if (st.pending_kind == 2) {
            if (st.stage == kStDSum) {
                // dense residual: totals, then the owner CTA of the crossing finds the token
                double rs = 0.0, ps = 0.0;
#pragma unroll
                for (int q = 0; q < kC; ++q) {
                    rs += cs->rsum[q];
                    ps += cs->psum[q];
                }
                const bool use_res = rs > 1e-12;
                const double target = rc.u_draw * (use_res ? rs : 1.0);
                int owner = -1;
                double before = 0.0;
                for (int q = 0; q < kC; ++q) {
                    const double v = use_res ? cs->rsum[q] : cs->psum[q];
                    if (owner < 0 && before + v > target && v > 0.0) {
                        owner = q;
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
                        // ordered scan of my entries in vocabulary-id order (slot-major)
                        const float* qrow = a.q + (static_cast<size_t>(rc.stream) * a.k + rc.vidx) * a.row_stride + c0;
                        const double zk_d = static_cast<double>(st.zkept);
                        double run = before;
                        unsigned long long found = ~0ull;
                        for (int j = 0; j < NV && found == ~0ull; ++j) {
                            double vals[SW];
                            double s = 0.0;
#pragma unroll
                            for (int i = 0; i < SW; ++i) {
                                const int q = j * SW + i;
                                const uint32_t k = keys[q];
                                double v = 0.0;
                                if (k != 0u) {
                                    const unsigned long long cp = comp_at(q);
                                    const float x = kval(k);
                                    if (cp >= st.xcross && cp >= st.kbound && x >= x_minp) {
                                        const float pf = static_cast<float>(static_cast<double>(weight_of(x, wc)) / zk_d);
                                        v = use_res ? fmax(0.0, static_cast<double>(pf) - static_cast<double>(qrow[elem_of<SW>(j, i)]))
                                                    : static_cast<double>(pf);
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
                            for (int i = 0; i < SW; ++i) {
                                acc += vals[i];
                                if (cand == ~0ull && vals[i] > 0.0 && acc > target)
                                    cand = static_cast<unsigned long long>(c0 + elem_of<SW>(j, i));
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
#pragma unroll
                for (int q = 0; q < kC; ++q) nk += cs->cnt[q];
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
                gather(lo, cur, 0ull);
            } else if (st.stage == kStTopP) {
                if (P->top_p > 0.0f && P->top_p < 1.0f) {
                    unsigned long long t1 = ceil_mass(P->top_p, st.zk);
                    if (t1 < 1ull) t1 = 1ull;
                    const int b = bin_of_target(t1);
                    st.target = t1 - (b > 0 ? CG[b - 1] : 0ull);
                    st.pending_bin = b;
                    st.pending_kind = 1;
                    gather(b, cur, st.kbound);
                } else {
                    st.zkept = st.zk;
                    st.stage = kStKept;
                }
            } else if (st.stage == kStKept) {
                if (P->min_p > 0.0f && Wmin < st.zkept) st.zkept = Wmin;
                if (MODE == kModeCandidates) {
                    uint32_t c = 0;
#pragma unroll
                    for (int q = 0; q < EPT; ++q) {
                        const uint32_t k = keys[q];
                        if (k == 0u) continue;
                        const unsigned long long cp = comp_at(q);
                        if (cp >= st.xcross && cp >= st.kbound && kval(k) >= x_minp) ++c;
                    }
                    const unsigned long long tc = block_sum_u64<kNT>(c, ls->red);
                    if (tid < kC) cluster.map_shared_rank(cs, tid)->cnt[crank] = tc;
                    st.stage = kStCount;
                    st.pending_kind = 2;
                } else if (MODE == kModeVerify && rc.vrole == 0) {
                    const bool kept = dvalid && dcomp >= st.xcross && dcomp >= st.kbound && xd >= x_minp;
                    double pd = 0.0;
                    if (kept) {
                        const double ed = exp(static_cast<double>(xd) * invT - maxs);
                        pd = ed / (static_cast<double>(st.zkept) / kWeightScale);
                    }
                    const bool in_range = rc.draft >= 0 && static_cast<uint32_t>(rc.draft) < a.vocab;
                    if (a.q != nullptr) {
                        const float* qrow = a.q + (static_cast<size_t>(rc.stream) * a.k + rc.vidx) * a.row_stride;
                        const float p_d = static_cast<float>(pd);
                        const float q_d = in_range ? qrow[rc.draft] : 1.0f;
                        const double accept_prob = (q_d <= 0.0f) ? (p_d > 0.0f ? 1.0 : 0.0)
                            : fmin(1.0, static_cast<double>(p_d) / fmax(1e-12, static_cast<double>(q_d)));
                        res_accept = rc.u_accept < accept_prob ? 1 : 0;
                        if (res_accept) {
                            st.stage = kStDone;
                        } else {
                            // partial sums of the residual and of p_target over this chunk
                            const float* qrow_c = qrow + c0;
                            const double zk_d = static_cast<double>(st.zkept);
                            double rsum = 0.0, psum = 0.0;
#pragma unroll
                            for (int q = 0; q < EPT; ++q) {
                                const uint32_t k = keys[q];
                                if (k == 0u) continue;
                                const unsigned long long cp = comp_at(q);
                                const float x = kval(k);
                                if (!(cp >= st.xcross && cp >= st.kbound && x >= x_minp)) continue;
                                const float pf = static_cast<float>(static_cast<double>(weight_of(x, wc)) / zk_d);
                                rsum += fmax(0.0, static_cast<double>(pf) -
                                                      static_cast<double>(qrow_c[elem_of<SW>(q / SW, q % SW)]));
                                psum += static_cast<double>(pf);
                            }
                            rsum = block_sum_f64(rsum, ls);
                            psum = block_sum_f64(psum, ls);
                            if (tid < kC) {
                                ClusterShared* dst = cluster.map_shared_rank(cs, tid);
                                dst->rsum[crank] = rsum;
                                dst->psum[crank] = psum;
                            }
                            st.stage = kStDSum;
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
                                const int bd = kept ? xbin_g(static_cast<uint32_t>(dkey)) : kABins;
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
                                gather(lo, cur, st.kbound);
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
                st.pending_kind = 1;
                gather(b, cur, st.kbound);
            } else {
                st.err = 4;
            }
        }
        cluster.sync();  // ============================================ one barrier per round
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
// launch of one (mode, dtype) instance family; defined in smp_inst.cu, compiled once per pair

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

// elements per thread of the instantiated kernels
int pick_ept(uint32_t chunk);

}  // namespace sixi_b200
