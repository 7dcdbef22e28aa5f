#pragma once
// sixi_sharded.hpp - the vocab-sharded sampling step in C++ over the NCCL C API (header-only; link
// NCCL and cudart). For models whose output layer is split over ranks by vocabulary, so that each
// rank holds a slice of every logits row; the engine itself runs on one device and has no
// counterpart. One step on each rank:
//
//   stage 1   sixi_smp_shard_candidates on this rank's slice: per row the slice's best top_n
//             candidates (adjusted logit, global id) and (max, sum of exp, allowed count)
//   exchange  ncclAllGather of both arrays on the caller's stream (one NCCL group), rank-major
//   stage 2   sixi_smp_merge_shards, identical on every rank: every row's token where the merged
//             candidates decide it, SIXI_OUT_OF_BOUNDS where the row's kept set or draw reaches past
//             them (possible for top_k = 0 or top_k > top_n)
//   round 2   only for those rows (one stream synchronisation learns how many): their slice rows
//             are packed (sixi_smp_gather_rows), all-gathered, rebuilt into full rows and sampled
//             with sixi_smp_sample_indexed as their batch rows
//
// Every rank ends with the same tokens and statuses for every row: the tokens sixi_smp_sample draws
// on the full rows wherever stage 2 certifies the row or round 2 samples it. No PyTorch, no host
// copy of any logits. Rank r owns ids [offset(r), offset(r) + width(r)) of the vocabulary, the first
// vocab % n_shards ranks one id more than the rest.
#include <nccl.h>

#include <algorithm>
#include <memory>
#include <vector>

#include "sixi_sampler.hpp"

namespace sixi_b200 {

struct ShardLayout {
    uint32_t vocab = 0, n_shards = 1;
    uint32_t width(uint32_t r) const { return vocab / n_shards + (r < vocab % n_shards ? 1u : 0u); }
    uint32_t offset(uint32_t r) const { return r * (vocab / n_shards) + std::min(r, vocab % n_shards); }
    uint32_t max_width() const { return width(0); }
};

// CUDA-event split of one step on this rank (milliseconds), filled when requested.
struct ShardStepTimes {
    float stage1_ms = 0.0f, exchange_ms = 0.0f, stage2_ms = 0.0f, round2_ms = 0.0f;
    uint32_t round2_rows = 0;
};

class ShardedSampler {
public:
    // A sampler for batches of up to `max_rows` rows of a `full_vocab`-wide vocabulary split over
    // the ranks of `comm` (ncclCommInitRank / ncclCommInitAll; not owned, must outlive the sampler),
    // on `device`, which must be the communicator's device for this rank.
    static Result<std::unique_ptr<ShardedSampler>> create(int device, uint32_t max_rows, uint32_t full_vocab,
                                                          ncclComm_t comm, uint32_t top_n = 64) {
        using R = Result<std::unique_ptr<ShardedSampler>>;
        int nranks = 0, rank = 0;
        if (comm == nullptr || ncclCommCount(comm, &nranks) != ncclSuccess ||
            ncclCommUserRank(comm, &rank) != ncclSuccess || nranks < 1)
            return R(ErrorCode::InvalidArgument, "ShardedSampler: invalid NCCL communicator");
        if (top_n == 0 || top_n > 64 || static_cast<uint32_t>(nranks) > 16)
            return R(ErrorCode::InvalidArgument, "ShardedSampler: top_n in 1..64 and at most 16 ranks");
        sixi_smp* h = nullptr;
        const int32_t st = sixi_smp_create(device, max_rows, full_vocab, &h);
        if (st != SIXI_OK) return R(detail::status_of(st, "sixi_smp_create"));
        std::unique_ptr<ShardedSampler> s(new ShardedSampler());
        s->h_ = h;
        s->device_ = device;
        s->max_rows_ = max_rows;
        s->comm_ = comm;
        s->rank_ = static_cast<uint32_t>(rank);
        s->layout_ = ShardLayout{full_vocab, static_cast<uint32_t>(nranks)};
        s->top_n_ = top_n;
        detail::DeviceGuard g(device);
        for (detail::DeviceBuffer* b : {&s->cand_, &s->stats_, &s->gcand_, &s->gstats_, &s->index_, &s->pack_,
                                        &s->gathered_, &s->full_})
            b->device = device;
        const size_t n = max_rows, S = static_cast<size_t>(nranks);
        if (!s->cand_.ensure(n * top_n * 8) || !s->stats_.ensure(n * 24) || !s->gcand_.ensure(S * n * top_n * 8) ||
            !s->gstats_.ensure(S * n * 24) || !s->index_.ensure(n * 4 + 4))
            return R(ErrorCode::OutOfMemoryVRAM, "ShardedSampler: device buffers");
        if (cudaMallocHost(&s->h_status_, n * 4 + 4) != cudaSuccess ||
            cudaMallocHost(&s->h_index_, n * 4 + 4) != cudaSuccess)
            return R(ErrorCode::OutOfMemoryVRAM, "ShardedSampler: pinned host buffers");
        for (cudaEvent_t* e : {&s->ev_[0], &s->ev_[1], &s->ev_[2], &s->ev_[3], &s->ev_[4]})
            if (cudaEventCreate(e) != cudaSuccess) return R(ErrorCode::BackendError, "ShardedSampler: events");
        return R(std::move(s));
    }

    ~ShardedSampler() {
        detail::DeviceGuard g(device_);
        for (cudaEvent_t e : ev_)
            if (e != nullptr) cudaEventDestroy(e);
        if (h_status_ != nullptr) cudaFreeHost(h_status_);
        if (h_index_ != nullptr) cudaFreeHost(h_index_);
        sixi_smp_destroy(h_);
    }
    ShardedSampler(const ShardedSampler&) = delete;
    ShardedSampler& operator=(const ShardedSampler&) = delete;

    const ShardLayout& layout() const noexcept { return layout_; }
    uint32_t rank() const noexcept { return rank_; }
    sixi_smp* handle() const noexcept { return h_; }

    // One step on this rank. shard_rows: n_rows rows of this rank's slice (device, fp32 or bf16,
    // width(rank) <= row_stride). d_params [n_rows], d_masks (full-vocabulary rows, nullable),
    // d_hist / d_hist_off (CSR of global ids, nullable), d_uniforms ([n_rows] or NULL for Philox):
    // the whole batch's device arrays, the same on every rank. Writes every row's token and status
    // to d_out_tokens / d_out_status; synchronises `stream` once (before round 2). Every rank must
    // make the same calls in the same order (NCCL collectives).
    Status sample(const sixi_smp_rows& shard_rows, const sixi_smp_params* d_params, const uint32_t* d_masks,
                  const int32_t* d_hist, const int64_t* d_hist_off, const double* d_uniforms, uint64_t step,
                  int32_t* d_out_tokens, int32_t* d_out_status, cudaStream_t stream, ShardStepTimes* times = nullptr) {
        const uint32_t n = shard_rows.n_rows, S = layout_.n_shards, w = layout_.width(rank_);
        if (n > max_rows_) return Status::Error(ErrorCode::OutOfBounds, "ShardedSampler: batch above max_rows");
        if (shard_rows.data == nullptr || shard_rows.row_stride < w || d_params == nullptr ||
            d_out_tokens == nullptr || d_out_status == nullptr)
            return Status::Error(ErrorCode::InvalidArgument, "ShardedSampler: null buffer or slice narrower than its width");
        if (n == 0) return Status::Ok();
        detail::DeviceGuard g(device_);
        const size_t esz = shard_rows.dtype == SIXI_SMP_BF16 ? 2 : 4;
        if (times != nullptr) cudaEventRecord(ev_[0], stream);
        int32_t rc = sixi_smp_shard_candidates(h_, &shard_rows, layout_.offset(rank_), w, layout_.vocab, d_params,
                                               d_masks, d_hist, d_hist_off, top_n_, cand_.p, stats_.p, stream);
        if (rc != SIXI_OK) return detail::status_of(rc, "sixi_smp_shard_candidates");
        if (times != nullptr) cudaEventRecord(ev_[1], stream);
        ncclResult_t nr = ncclGroupStart();
        if (nr == ncclSuccess) nr = ncclAllGather(cand_.p, gcand_.p, static_cast<size_t>(n) * top_n_ * 8, ncclChar, comm_, stream);
        if (nr == ncclSuccess) nr = ncclAllGather(stats_.p, gstats_.p, static_cast<size_t>(n) * 24, ncclChar, comm_, stream);
        const ncclResult_t ne = ncclGroupEnd();
        if (nr != ncclSuccess || ne != ncclSuccess) return nccl_error(nr != ncclSuccess ? nr : ne);
        if (times != nullptr) cudaEventRecord(ev_[2], stream);
        rc = sixi_smp_merge_shards(h_, n, S, top_n_, gcand_.p, gstats_.p, d_params, d_uniforms, step, d_out_tokens,
                                   d_out_status, stream);
        if (rc != SIXI_OK) return detail::status_of(rc, "sixi_smp_merge_shards");
        if (times != nullptr) cudaEventRecord(ev_[3], stream);
        // the rows stage 2 could not certify: the same set on every rank (stage 2 is deterministic)
        if (cudaMemcpyAsync(h_status_, d_out_status, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToHost, stream) !=
                cudaSuccess ||
            cudaStreamSynchronize(stream) != cudaSuccess)
            return Status::Error(ErrorCode::BackendError, "ShardedSampler: status read-back");
        uint32_t nf = 0;
        for (uint32_t r = 0; r < n; ++r)
            if (h_status_[r] == SIXI_OUT_OF_BOUNDS) h_index_[nf++] = static_cast<int32_t>(r);
        if (nf > 0) {
            const size_t wmax = layout_.max_width();
            if (!pack_.ensure(nf * wmax * esz) || !gathered_.ensure(static_cast<size_t>(S) * nf * wmax * esz) ||
                !full_.ensure(static_cast<size_t>(nf) * layout_.vocab * esz))
                return Status::Error(ErrorCode::OutOfMemoryVRAM, "ShardedSampler: round-2 buffers");
            cudaMemcpyAsync(index_.p, h_index_, nf * 4, cudaMemcpyHostToDevice, stream);
            rc = sixi_smp_gather_rows(h_, &shard_rows, index_.as<int32_t>(), nf, w, pack_.p, wmax, stream);
            if (rc != SIXI_OK) return detail::status_of(rc, "sixi_smp_gather_rows");
            nr = ncclAllGather(pack_.p, gathered_.p, nf * wmax * esz, ncclChar, comm_, stream);
            if (nr != ncclSuccess) return nccl_error(nr);
            for (uint32_t r = 0; r < S; ++r) {  // slice r of every flagged row into its columns
                const char* src = gathered_.as<char>() + static_cast<size_t>(r) * nf * wmax * esz;
                char* dst = full_.as<char>() + static_cast<size_t>(layout_.offset(r)) * esz;
                if (cudaMemcpy2DAsync(dst, layout_.vocab * esz, src, wmax * esz, layout_.width(r) * esz, nf,
                                      cudaMemcpyDeviceToDevice, stream) != cudaSuccess)
                    return Status::Error(ErrorCode::BackendError, "ShardedSampler: row rebuild");
            }
            const sixi_smp_rows full{full_.p, shard_rows.dtype, nf, layout_.vocab};
            rc = sixi_smp_sample_indexed(h_, &full, index_.as<uint32_t>(), d_params, d_masks, d_hist, d_hist_off,
                                         d_uniforms, step, d_out_tokens, d_out_status, stream);
            if (rc != SIXI_OK) return detail::status_of(rc, "sixi_smp_sample_indexed");
        }
        if (times != nullptr) {
            cudaEventRecord(ev_[4], stream);
            if (cudaEventSynchronize(ev_[4]) != cudaSuccess)
                return Status::Error(ErrorCode::BackendError, "ShardedSampler: timing events");
            cudaEventElapsedTime(&times->stage1_ms, ev_[0], ev_[1]);
            cudaEventElapsedTime(&times->exchange_ms, ev_[1], ev_[2]);
            cudaEventElapsedTime(&times->stage2_ms, ev_[2], ev_[3]);
            cudaEventElapsedTime(&times->round2_ms, ev_[3], ev_[4]);
            times->round2_rows = nf;
        }
        return Status::Ok();
    }

private:
    ShardedSampler() = default;

    static Status nccl_error(ncclResult_t r) {
        return Status::Error(ErrorCode::BackendError, std::string("NCCL: ") + ncclGetErrorString(r));
    }

    sixi_smp* h_ = nullptr;
    int device_ = 0;
    uint32_t max_rows_ = 0;
    ncclComm_t comm_ = nullptr;
    uint32_t rank_ = 0;
    ShardLayout layout_;
    uint32_t top_n_ = 64;
    detail::DeviceBuffer cand_, stats_, gcand_, gstats_, index_, pack_, gathered_, full_;
    int32_t* h_status_ = nullptr;
    int32_t* h_index_ = nullptr;
    cudaEvent_t ev_[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
};

}  // namespace sixi_b200
