// sixi_sampler.hpp - C++ host adapter of the B200 logits-to-token path (header only, C++17).
//
// Mirrors the engine's host-side sampler/verifier interface so that a caller can swap it in:
//   - DeterministicSampler (include/sixi_asi/core_execution.hpp:146-183): sample_greedy_argmax,
//     sample_token, compute_sampling_candidates, sample_from_candidates, with the same argument
//     meaning, the same Result/ErrorCode error behaviour and the same RNG consumption
//     (src/core/core_execution.cpp:586-619: greedy draws nothing, a sampled row draws one uniform).
//   - the verification half of SpeculativeDecoder::step (include/sixi_asi/speculative.hpp:164-168;
//     src/speculative/speculative.cpp:589-692 one-hot drafts, 801-916 dense draft probabilities),
//     returning the fields of SpeculativeStepResult that verification fills.
// Every compute call goes through the C ABI (include/sixi_smp.h) to the sm_100a kernels; there is
// no host compute path. The single-row methods take HOST logits like the engine's functions and
// stage them on the device; batched callers use sample_rows / verify_rows with device buffers.
//
// Templates accept the engine's own types: any params struct with temperature, top_k, top_p,
// repetition_penalty, presence_penalty, seed and mode (min_p and frequency_penalty are read when
// present), and any RNG with next_uniform01(), checkpoint() and restore() (DeterministicRng).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <memory>
#include <optional>
#include <string>
#include <type_traits>
#include <utility>
#include <vector>

#include "../../include/sixi_json.h"
#include "../../include/sixi_smp.h"

namespace sixi_b200 {

// Same values as the engine's ErrorCode (include/sixi_asi/common.hpp:40-66); the kernels report
// these per row.
enum class ErrorCode : int32_t {
    Ok = 0,
    InvalidArgument = 1,
    OutOfBounds = 2,
    OutOfMemoryVRAM = 11,
    NumericNaNOrInf = 16,
    BackendError = 23,
    UnsupportedHardware = 24,
};

struct Status {
    ErrorCode code = ErrorCode::Ok;
    std::string message{};
    bool ok() const noexcept { return code == ErrorCode::Ok; }
    static Status Ok() { return Status{}; }
    static Status Error(ErrorCode c, std::string msg) { return Status{c, std::move(msg)}; }
};

// Shape of the engine's Result<T> (include/sixi_asi/common.hpp:79-104).
template <typename T>
class Result {
public:
    Result(T v) : status_(Status::Ok()), value_(std::move(v)) {}
    Result(Status st) : status_(std::move(st)) {}
    Result(ErrorCode c, std::string msg) : status_(Status::Error(c, std::move(msg))) {}
    bool ok() const noexcept { return status_.ok() && value_.has_value(); }
    const Status& status() const noexcept { return status_; }
    ErrorCode code() const noexcept { return status_.code; }
    const std::string& message() const noexcept { return status_.message; }
    T& value() & { return *value_; }
    const T& value() const& { return *value_; }
    T&& value() && { return std::move(*value_); }

private:
    Status status_;
    std::optional<T> value_;
};

// The engine's SamplingParams (include/sixi_asi/core_execution.hpp:137-145) plus the two
// extensions of the device path (min_p and frequency_penalty, 0 = off as in the engine).
enum class ExecutionMode : uint8_t { StrictReplay = 0, Adaptive = 1 };

struct SamplingParams {
    float temperature = 0.0f;
    int32_t top_k = 20;
    float top_p = 0.95f;
    float repetition_penalty = 1.0f;
    float presence_penalty = 0.0f;
    uint64_t seed = 42ULL;
    ExecutionMode mode = ExecutionMode::StrictReplay;
    float min_p = 0.0f;
    float frequency_penalty = 0.0f;
};

struct Candidate {
    int32_t id = 0;
    double prob = 0.0;
};

// Verification fields of SpeculativeStepResult (include/sixi_asi/speculative.hpp:119-129).
struct VerifyResult {
    uint32_t proposed_k = 0;
    uint32_t accepted_draft_count = 0;
    int32_t first_rejected_position = -1;
    std::vector<int32_t> committed_tokens;  // accepted drafts + the recovered or bonus token
    uint32_t uniforms_used = 0;
};

// Draft fields of DraftProposal (include/sixi_asi/speculative.hpp:24-30) for the suffix drafter.
struct SuffixProposal {
    std::vector<int32_t> draft_tokens;              // length k
    std::vector<std::vector<float>> draft_probs;    // [k][vocab_size] one-hot (empty when vocab_size == 0)
    uint32_t match_len = 0;
};

namespace detail {

template <class P, class = void>
struct has_min_p : std::false_type {};
template <class P>
struct has_min_p<P, std::void_t<decltype(std::declval<const P&>().min_p)>> : std::true_type {};
template <class P, class = void>
struct has_freq : std::false_type {};
template <class P>
struct has_freq<P, std::void_t<decltype(std::declval<const P&>().frequency_penalty)>> : std::true_type {};

inline ErrorCode code_of(int32_t st) { return static_cast<ErrorCode>(st); }

inline Status status_of(int32_t st, const char* where) {
    if (st == SIXI_OK) return Status::Ok();
    return Status::Error(code_of(st), std::string(where) + ": " + sixi_smp_status_string(st));
}

// Makes `device` current for a scope and restores the caller's device afterwards.
struct DeviceGuard {
    int prev = 0;
    explicit DeviceGuard(int device) {
        cudaGetDevice(&prev);
        cudaSetDevice(device);
    }
    ~DeviceGuard() { cudaSetDevice(prev); }
};

// Device buffer that grows on demand (cudaMalloc on growth only).
struct DeviceBuffer {
    void* p = nullptr;
    size_t bytes = 0;
    int device = 0;
    ~DeviceBuffer() { release(); }
    void release() {
        if (p != nullptr) {
            int prev = 0;
            cudaGetDevice(&prev);
            cudaSetDevice(device);
            cudaFree(p);
            cudaSetDevice(prev);
        }
        p = nullptr;
        bytes = 0;
    }
    bool ensure(size_t need) {
        if (need <= bytes) return true;
        release();
        if (cudaMalloc(&p, need) != cudaSuccess) {
            p = nullptr;
            return false;
        }
        bytes = need;
        return true;
    }
    template <class T>
    T* as() const {
        return static_cast<T*>(p);
    }
};

}  // namespace detail

// Converts any engine-style params struct into the C ABI record.
template <class P>
sixi_smp_params to_smp_params(const P& p, bool masked = false, uint64_t counter = 0) {
    sixi_smp_params r{};
    r.temperature = p.temperature;
    r.top_k = p.top_k;
    r.top_p = p.top_p;
    r.repetition_penalty = p.repetition_penalty;
    r.presence_penalty = p.presence_penalty;
    r.min_p = 0.0f;
    r.frequency_penalty = 0.0f;
    if constexpr (detail::has_min_p<P>::value) r.min_p = p.min_p;
    if constexpr (detail::has_freq<P>::value) r.frequency_penalty = p.frequency_penalty;
    r.mode = static_cast<uint32_t>(p.mode);
    r.flags = masked ? static_cast<uint32_t>(SIXI_SMP_ROW_MASKED) : 0u;
    r.seed = p.seed;
    r.counter = counter;
    return r;
}

class DeviceSampler {
public:
    // Creates a sampler for `vocab`-wide rows on `device`, batches of up to `max_rows` rows.
    static Result<std::unique_ptr<DeviceSampler>> create(int device, size_t max_rows, uint32_t vocab) {
        sixi_smp* h = nullptr;
        const int32_t st = sixi_smp_create(device, max_rows, vocab, &h);
        if (st != SIXI_OK) return Result<std::unique_ptr<DeviceSampler>>(detail::status_of(st, "sixi_smp_create"));
        std::unique_ptr<DeviceSampler> s(new DeviceSampler(h, device, max_rows, vocab));
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(device);
        const cudaError_t e = cudaStreamCreateWithFlags(&s->stream_, cudaStreamNonBlocking);
        cudaSetDevice(prev);
        if (e != cudaSuccess)
            return Result<std::unique_ptr<DeviceSampler>>(ErrorCode::BackendError, cudaGetErrorString(e));
        return Result<std::unique_ptr<DeviceSampler>>(std::move(s));
    }

    ~DeviceSampler() {
        if (stream_ != nullptr) {
            cudaStreamSynchronize(stream_);
            cudaStreamDestroy(stream_);
        }
        sixi_smp_destroy(h_);
    }
    DeviceSampler(const DeviceSampler&) = delete;
    DeviceSampler& operator=(const DeviceSampler&) = delete;

    uint32_t vocab() const noexcept { return vocab_; }
    size_t max_rows() const noexcept { return max_rows_; }
    sixi_smp* handle() const noexcept { return h_; }
    cudaStream_t stream() const noexcept { return stream_; }

    // ---- DeterministicSampler mirror (host logits, one row, synchronous) ----------------------

    // Argmax of the raw logits, lowest id on ties; -1 for null or empty input or any failure
    // (DeterministicSampler::sample_greedy_argmax, src/core/core_execution.cpp:394-407).
    int32_t sample_greedy_argmax(const float* logits, uint64_t vocab_size) noexcept {
        if (logits == nullptr || vocab_size == 0 || vocab_size != vocab_) return -1;
        detail::DeviceGuard g(device_);
        if (!stage_logits(logits, 1, vocab_size)) return -1;
        sixi_smp_rows rows{d_logits_.p, SIXI_SMP_F32, 1, vocab_size};
        int32_t* out = d_out_.as<int32_t>();
        if (sixi_smp_greedy_argmax(h_, &rows, nullptr, out, out + 1, stream_) != SIXI_OK) return -1;
        int32_t r[2] = {-1, 0};
        if (cudaMemcpyAsync(r, out, sizeof r, cudaMemcpyDeviceToHost, stream_) != cudaSuccess) return -1;
        if (cudaStreamSynchronize(stream_) != cudaSuccess) return -1;
        return r[1] == SIXI_OK ? r[0] : -1;
    }

    // NaN / Inf inspection and policy of one host row, in place, with the engine's signature and
    // Status (inspect_and_apply_numeric_policy, src/core/numeric.cpp:628-699): `policy` is the
    // engine's NumericPolicy (0 FailAndInvalidate, 1 EmergencyClampAndReport) and `out_report` any
    // type with NumericHealthReport's fields (include/sixi_asi/numeric.hpp:131-139). A row with a
    // NaN or an infinity under the fail policy returns NumericNaNOrInf with the engine's message.
    // The row is the sampler's vocabulary wide (n == vocab()), or empty.
    template <class Policy, class Report>
    Status inspect_and_apply_numeric_policy(float* data, int64_t n, Policy policy, float clamp_abs_max,
                                            Report* out_report) {
        if (n < 0 || (n > 0 && data == nullptr))
            return Status::Error(ErrorCode::InvalidArgument, "invalid data pointer or element count");
        sixi_smp_numeric_report r{};
        r.healthy = 1;
        r.first_bad_index = -1;
        const uint32_t pol = static_cast<uint32_t>(policy) == 1u ? SIXI_SMP_NUMERIC_CLAMP : SIXI_SMP_NUMERIC_FAIL;
        if (n > 0) {
            if (static_cast<uint64_t>(n) != vocab_)
                return Status::Error(ErrorCode::InvalidArgument, "element count differs from the sampler's vocabulary");
            detail::DeviceGuard g(device_);
            if (!stage_logits(data, 1, static_cast<uint64_t>(n)) || !d_rep_.ensure(sizeof r)) return oom();
            const int32_t rc = sixi_smp_numeric_policy(h_, d_logits_.as<float>(), 1, static_cast<uint64_t>(n), pol,
                                                       clamp_abs_max, d_rep_.as<sixi_smp_numeric_report>(), stream_);
            if (rc != SIXI_OK) return detail::status_of(rc, "sixi_smp_numeric_policy");
            cudaError_t e = cudaMemcpyAsync(&r, d_rep_.p, sizeof r, cudaMemcpyDeviceToHost, stream_);
            if (e == cudaSuccess && pol == SIXI_SMP_NUMERIC_CLAMP)
                e = cudaMemcpyAsync(data, d_logits_.p, static_cast<size_t>(n) * sizeof(float), cudaMemcpyDeviceToHost,
                                    stream_);
            if (e == cudaSuccess) e = cudaStreamSynchronize(stream_);
            if (e != cudaSuccess) return Status::Error(ErrorCode::BackendError, cudaGetErrorString(e));
        }
        if (out_report != nullptr) {
            out_report->healthy = r.healthy != 0;
            out_report->request_corrupted = r.request_corrupted != 0;
            out_report->state_invalidated = r.state_invalidated != 0;
            out_report->emergency_clamped = r.emergency_clamped != 0;
            out_report->nan_count = r.nan_count;
            out_report->inf_count = r.inf_count;
            out_report->first_bad_index = r.first_bad_index;
        }
        if (r.status != SIXI_OK)
            return Status::Error(ErrorCode::NumericNaNOrInf,
                                 "NaN/Inf detected at index " + std::to_string(r.first_bad_index) +
                                     " (nan_count=" + std::to_string(r.nan_count) +
                                     ", inf_count=" + std::to_string(r.inf_count) + ")");
        return Status::Ok();
    }

    // SuffixDrafter::propose / ::propose_anchored on one host history (src/speculative/
    // speculative.cpp:28-176), with the engine's defaults SuffixDrafter(3, 16384): an empty optional
    // where the engine returns none. propose fills one-hot draft_probs when vocab_size > 0, as the
    // engine does. For many streams at once call sixi_smp_suffix_draft on device histories.
    std::optional<SuffixProposal> suffix_propose(const std::vector<int32_t>& token_history, uint32_t k,
                                                 uint64_t vocab_size, uint32_t min_match_len = 3,
                                                 uint32_t max_window_tokens = 16384) {
        return suffix_call(token_history, nullptr, k, vocab_size, min_match_len, max_window_tokens);
    }
    std::optional<SuffixProposal> suffix_propose_anchored(const std::vector<int32_t>& token_history,
                                                          int32_t anchor_token, uint32_t k,
                                                          uint32_t min_match_len = 3,
                                                          uint32_t max_window_tokens = 16384) {
        return suffix_call(token_history, &anchor_token, k, 0, min_match_len, max_window_tokens);
    }

    // The sparse normalised distribution sample_token draws from (penalties -> top-k ->
    // temperature softmax -> top-p [-> min-p]); greedy yields one candidate with prob 1
    // (src/core/core_execution.cpp:449-584). `mask_words` (host, ceil(V/32) words) is optional.
    template <class P>
    Result<std::vector<Candidate>> compute_sampling_candidates(const float* logits, uint64_t vocab_size,
                                                               const P& params,
                                                               const std::vector<int32_t>& recent_tokens = {},
                                                               const uint32_t* mask_words = nullptr) {
        using R = Result<std::vector<Candidate>>;
        Status st = check_row(logits, vocab_size);
        if (!st.ok()) return R(st);
        detail::DeviceGuard g(device_);
        if (!stage_logits(logits, 1, vocab_size)) return R(oom());
        st = stage_inputs(to_smp_params(params, mask_words != nullptr), recent_tokens, mask_words, nullptr);
        if (!st.ok()) return R(st);
        const uint32_t max_out = 256;
        if (!d_cand_.ensure(2 * max_out * sizeof(double))) return R(oom());
        int32_t* ids = d_cand_.as<int32_t>();
        double* probs = reinterpret_cast<double*>(d_cand_.as<char>() + max_out * sizeof(double));
        int32_t* out = d_out_.as<int32_t>();
        sixi_smp_rows rows{d_logits_.p, SIXI_SMP_F32, 1, vocab_size};
        int32_t rc = sixi_smp_candidates(h_, &rows, d_params_.as<sixi_smp_params>(),
                                         mask_words ? d_mask_.as<uint32_t>() : nullptr, d_hist_.as<int32_t>(),
                                         d_hoff_.as<int64_t>(), max_out, ids, probs, out, out + 1, stream_);
        if (rc != SIXI_OK) return R(detail::status_of(rc, "sixi_smp_candidates"));
        int32_t cnt_st[2] = {0, 0};
        std::vector<int32_t> hid(max_out);
        std::vector<double> hp(max_out);
        cudaMemcpyAsync(cnt_st, out, sizeof cnt_st, cudaMemcpyDeviceToHost, stream_);
        cudaMemcpyAsync(hid.data(), ids, max_out * sizeof(int32_t), cudaMemcpyDeviceToHost, stream_);
        cudaMemcpyAsync(hp.data(), probs, max_out * sizeof(double), cudaMemcpyDeviceToHost, stream_);
        if (cudaStreamSynchronize(stream_) != cudaSuccess) return R(ErrorCode::BackendError, "stream failed");
        if (cnt_st[1] != SIXI_OK) return R(detail::status_of(cnt_st[1], "compute_sampling_candidates"));
        if (cnt_st[0] > static_cast<int32_t>(max_out))
            return R(ErrorCode::OutOfBounds, "candidate list longer than 256 entries (top_k = 0 or > 256)");
        std::vector<Candidate> c(static_cast<size_t>(cnt_st[0]));
        for (size_t i = 0; i < c.size(); ++i) c[i] = Candidate{hid[i], hp[i]};
        return R(std::move(c));
    }

    // Draws one token exactly like DeterministicSampler::sample_token
    // (src/core/core_execution.cpp:603-619): greedy rows consume no uniform, sampled rows one, and
    // a row that fails leaves the RNG untouched.
    template <class P, class Rng>
    Result<int32_t> sample_token(const float* logits, uint64_t vocab_size, const P& params, Rng& rng,
                                 const std::vector<int32_t>& recent_tokens = {},
                                 const uint32_t* mask_words = nullptr) {
        Status st = check_row(logits, vocab_size);
        if (!st.ok()) return Result<int32_t>(st);
        detail::DeviceGuard g(device_);
        if (!stage_logits(logits, 1, vocab_size)) return Result<int32_t>(oom());
        return sample_staged(sixi_smp_rows{d_logits_.p, SIXI_SMP_F32, 1, vocab_size}, params, rng, recent_tokens,
                             mask_words);
    }

    // ---- device-resident rows ------------------------------------------------------------------
    // The same calls on rows the caller already holds in device memory on this sampler's device
    // (fp32 or bf16, any row stride >= vocab()): the backend's logits buffer for the output
    // positions, so that the V * 4 bytes of a row never cross PCIe. Only the parameters, the
    // history and the uniforms go to the device, and a few bytes per row come back. The device
    // rows must stay valid and unchanged until the call returns (every call here synchronises).

    // sample_token on one device row (`row.n_rows` == 1).
    template <class P, class Rng>
    Result<int32_t> sample_token(const sixi_smp_rows& row, const P& params, Rng& rng,
                                 const std::vector<int32_t>& recent_tokens = {},
                                 const uint32_t* mask_words = nullptr) {
        if (row.data == nullptr || row.n_rows != 1 || row.row_stride < vocab_)
            return Result<int32_t>(ErrorCode::InvalidArgument, "sample_token: one device row of the vocabulary's width");
        detail::DeviceGuard g(device_);
        return sample_staged(row, params, rng, recent_tokens, mask_words);
    }

    // Raw argmax of one device row (sample_greedy_argmax); -1 on any failure.
    int32_t sample_greedy_argmax(const sixi_smp_rows& row) noexcept {
        if (row.data == nullptr || row.n_rows != 1 || row.row_stride < vocab_) return -1;
        detail::DeviceGuard g(device_);
        int32_t* out = d_out_.as<int32_t>();
        if (sixi_smp_greedy_argmax(h_, &row, nullptr, out, out + 1, stream_) != SIXI_OK) return -1;
        int32_t r[2] = {-1, 0};
        if (cudaMemcpyAsync(r, out, sizeof r, cudaMemcpyDeviceToHost, stream_) != cudaSuccess) return -1;
        if (cudaStreamSynchronize(stream_) != cudaSuccess) return -1;
        return r[1] == SIXI_OK ? r[0] : -1;
    }

    // The candidate-list draw of DeterministicSampler::sample_from_candidates
    // (src/core/core_execution.cpp:586-601): one uniform, first cdf > u, else the last id. Host-side
    // by nature (its input is a host list of at most a few hundred entries).
    template <class Rng>
    static int32_t sample_from_candidates(const std::vector<Candidate>& cands, Rng& rng) noexcept {
        if (cands.empty()) return -1;
        const double u = rng.next_uniform01();
        double cdf = 0.0;
        for (const Candidate& c : cands) {
            cdf += c.prob;
            if (u < cdf) return c.id;
        }
        return cands.back().id;
    }

    // ---- speculative verification (one stream, host buffers) ----------------------------------

    // Verifies `drafts` (k tokens) against k + 1 target rows [k + 1][V] (host fp32): row i judges
    // draft i, row k draws the bonus token. `draft_probs` [k][V] selects the dense-q rule
    // (speculative.cpp:801-916), nullptr the one-hot rule (speculative.cpp:589-692).
    // `context_tokens` is the penalty history before the first draft. Uniforms are taken from
    // `rng` in the engine's order and the RNG is advanced by exactly the number used.
    template <class P, class Rng>
    Result<VerifyResult> verify(const float* target_rows, const float* draft_probs, const std::vector<int32_t>& drafts,
                                const P& params, Rng& rng, const std::vector<int32_t>& context_tokens,
                                const uint32_t* mask_words = nullptr) {
        using R = Result<VerifyResult>;
        const size_t k = drafts.size();
        if (target_rows == nullptr) return R(ErrorCode::InvalidArgument, "verify: target rows are null");
        if (k + 1 > max_rows_) return R(ErrorCode::OutOfBounds, "verify: k + 1 exceeds max_rows");
        detail::DeviceGuard g(device_);
        const uint64_t V = vocab_;
        if (!stage_logits(target_rows, k + 1, V)) return R(oom());
        if (draft_probs != nullptr && k > 0) {
            if (!d_q_.ensure(k * V * 4 + 16)) return R(oom());
            cudaMemcpyAsync(d_q_.p, draft_probs, k * V * 4, cudaMemcpyHostToDevice, stream_);
        }
        return verify_staged(sixi_smp_rows{d_logits_.p, SIXI_SMP_F32, static_cast<uint32_t>(k + 1), V},
                             draft_probs != nullptr ? d_q_.as<float>() : nullptr, drafts, params, rng, context_tokens,
                             mask_words);
    }

    // verify on k + 1 device rows (`target.n_rows` == drafts.size() + 1: the rows of one stream's
    // verify pass) with dense draft probabilities in device memory (`d_draft_probs`: k fp32 rows,
    // target.row_stride elements apart, as the verifier reads them) or none (one-hot rule).
    template <class P, class Rng>
    Result<VerifyResult> verify(const sixi_smp_rows& target, const float* d_draft_probs,
                                const std::vector<int32_t>& drafts, const P& params, Rng& rng,
                                const std::vector<int32_t>& context_tokens, const uint32_t* mask_words = nullptr) {
        using R = Result<VerifyResult>;
        if (target.data == nullptr || target.n_rows != drafts.size() + 1 || target.row_stride < vocab_)
            return R(ErrorCode::InvalidArgument, "verify: k + 1 device rows of the vocabulary's width");
        if (target.n_rows > max_rows_) return R(ErrorCode::OutOfBounds, "verify: k + 1 exceeds max_rows");
        detail::DeviceGuard g(device_);
        return verify_staged(target, d_draft_probs, drafts, params, rng, context_tokens, mask_words);
    }

    // ---- batched device path -------------------------------------------------------------------

    // One token per row for a device batch; asynchronous on `stream` (sixi_smp_sample).
    Status sample_rows(const sixi_smp_rows& rows, const sixi_smp_params* d_params, const uint32_t* d_masks,
                       const int32_t* d_hist, const int64_t* d_hist_off, const double* d_uniforms, uint64_t step,
                       int32_t* d_out_tokens, int32_t* d_out_status, cudaStream_t stream) {
        return detail::status_of(sixi_smp_sample(h_, &rows, d_params, d_masks, d_hist, d_hist_off, d_uniforms, step,
                                                 d_out_tokens, d_out_status, stream),
                                 "sixi_smp_sample");
    }

private:
    DeviceSampler(sixi_smp* h, int device, size_t max_rows, uint32_t vocab)
        : h_(h), device_(device), max_rows_(max_rows), vocab_(vocab) {
        for (detail::DeviceBuffer* b : {&d_logits_, &d_params_, &d_mask_, &d_hist_, &d_hoff_, &d_u_, &d_out_,
                                        &d_cand_, &d_q_, &d_drafts_, &d_vout_})
            b->device = device;
        detail::DeviceGuard g(device);
        d_out_.ensure(64);
    }

    static Status oom() { return Status::Error(ErrorCode::OutOfMemoryVRAM, "device staging allocation failed"); }

    std::optional<SuffixProposal> suffix_call(const std::vector<int32_t>& hist, const int32_t* anchor, uint32_t k,
                                              uint64_t vocab_size, uint32_t min_match_len, uint32_t window) {
        if (k == 0 || k > 4096u || min_match_len > 64u) return std::nullopt;
        detail::DeviceGuard g(device_);
        const int64_t off[2] = {0, static_cast<int64_t>(hist.size())};
        if (!d_hist_.ensure(hist.size() * 4 + 4) || !d_hoff_.ensure(sizeof off) || !d_drafts_.ensure((k + 2) * 4))
            return std::nullopt;
        int32_t* d_out = d_drafts_.as<int32_t>();
        cudaError_t e = cudaSuccess;
        if (!hist.empty()) e = cudaMemcpyAsync(d_hist_.p, hist.data(), hist.size() * 4, cudaMemcpyHostToDevice, stream_);
        if (e == cudaSuccess) e = cudaMemcpyAsync(d_hoff_.p, off, sizeof off, cudaMemcpyHostToDevice, stream_);
        if (e == cudaSuccess && anchor != nullptr)
            e = cudaMemcpyAsync(d_out + k + 1, anchor, 4, cudaMemcpyHostToDevice, stream_);
        if (e != cudaSuccess) return std::nullopt;
        if (sixi_smp_suffix_draft(h_, d_hist_.as<int32_t>(), d_hoff_.as<int64_t>(), 1, min_match_len, window,
                                  anchor != nullptr ? d_out + k + 1 : nullptr, k, d_out, d_out + k,
                                  stream_) != SIXI_OK)
            return std::nullopt;
        std::vector<int32_t> res(k + 1);
        if (cudaMemcpyAsync(res.data(), d_out, (k + 1) * 4, cudaMemcpyDeviceToHost, stream_) != cudaSuccess ||
            cudaStreamSynchronize(stream_) != cudaSuccess || res[k] == 0)
            return std::nullopt;
        SuffixProposal p;
        p.match_len = static_cast<uint32_t>(res[k]);
        p.draft_tokens.assign(res.begin(), res.begin() + k);
        if (vocab_size > 0) {
            p.draft_probs.assign(k, std::vector<float>(vocab_size, 0.0f));
            for (uint32_t i = 0; i < k; ++i) {
                const int32_t t = p.draft_tokens[i];
                if (t >= 0 && static_cast<uint64_t>(t) < vocab_size) p.draft_probs[i][static_cast<size_t>(t)] = 1.0f;
            }
        }
        return p;
    }

    // sample_token on rows already on the device (staged or the caller's): uniforms drawn in the
    // engine's order, the RNG restored when the row fails.
    template <class P, class Rng>
    Result<int32_t> sample_staged(const sixi_smp_rows& rows, const P& params, Rng& rng,
                                  const std::vector<int32_t>& recent_tokens, const uint32_t* mask_words) {
        using R = Result<int32_t>;
        const auto ck = rng.checkpoint();
        const bool sampled = params.temperature > 0.0f;
        const double u = sampled ? rng.next_uniform01() : 0.0;
        Status st = stage_inputs(to_smp_params(params, mask_words != nullptr), recent_tokens, mask_words, &u);
        if (!st.ok()) {
            rng.restore(ck);
            return R(st);
        }
        int32_t* out = d_out_.as<int32_t>();
        const int32_t rc = sixi_smp_sample(h_, &rows, d_params_.as<sixi_smp_params>(),
                                           mask_words ? d_mask_.as<uint32_t>() : nullptr, d_hist_.as<int32_t>(),
                                           d_hoff_.as<int64_t>(), d_u_.as<double>(), 0, out, out + 1, stream_);
        int32_t r[2] = {-1, 0};
        if (rc == SIXI_OK) {
            cudaMemcpyAsync(r, out, sizeof r, cudaMemcpyDeviceToHost, stream_);
            if (cudaStreamSynchronize(stream_) != cudaSuccess) r[1] = SIXI_BACKEND_ERROR;
        } else {
            r[1] = rc;
        }
        if (r[1] != SIXI_OK) {
            rng.restore(ck);
            return R(detail::status_of(r[1], "sample_token"));
        }
        return R(r[0]);
    }

    // verify on device rows (staged or the caller's), with device draft probabilities or none.
    template <class P, class Rng>
    Result<VerifyResult> verify_staged(const sixi_smp_rows& rows, const float* d_q, const std::vector<int32_t>& drafts,
                                       const P& params, Rng& rng, const std::vector<int32_t>& context_tokens,
                                       const uint32_t* mask_words) {
        using R = Result<VerifyResult>;
        const size_t k = drafts.size();
        const sixi_smp_params pr = to_smp_params(params, mask_words != nullptr);
        const size_t mw = sixi_smp_mask_words(h_);
        const auto ck = rng.checkpoint();
        std::vector<double> u(k + 1);
        for (double& x : u) x = rng.next_uniform01();
        const int64_t hoff[2] = {0, static_cast<int64_t>(context_tokens.size())};
        const bool ok = d_params_.ensure(sizeof pr) && d_hist_.ensure(context_tokens.size() * 4 + 4) &&
                        d_hoff_.ensure(sizeof hoff) && d_u_.ensure(u.size() * 8) && d_drafts_.ensure(k * 4 + 4) &&
                        d_vout_.ensure((6 + k + 1) * 4) && (mask_words == nullptr || d_mask_.ensure((k + 1) * mw * 4));
        if (!ok) {
            rng.restore(ck);
            return R(oom());
        }
        cudaMemcpyAsync(d_params_.p, &pr, sizeof pr, cudaMemcpyHostToDevice, stream_);
        if (!context_tokens.empty())
            cudaMemcpyAsync(d_hist_.p, context_tokens.data(), context_tokens.size() * 4, cudaMemcpyHostToDevice,
                            stream_);
        cudaMemcpyAsync(d_hoff_.p, hoff, sizeof hoff, cudaMemcpyHostToDevice, stream_);
        cudaMemcpyAsync(d_u_.p, u.data(), u.size() * 8, cudaMemcpyHostToDevice, stream_);
        if (k > 0) cudaMemcpyAsync(d_drafts_.p, drafts.data(), k * 4, cudaMemcpyHostToDevice, stream_);
        if (mask_words != nullptr)
            cudaMemcpyAsync(d_mask_.p, mask_words, (k + 1) * mw * 4, cudaMemcpyHostToDevice, stream_);
        int32_t* o = d_vout_.as<int32_t>();  // accepted, n_tokens, first_reject, used, status, tokens[k+1]
        const int32_t rc = sixi_smp_verify(h_, &rows, d_q, d_drafts_.as<int32_t>(), nullptr, 1,
                                           static_cast<uint32_t>(k), d_params_.as<sixi_smp_params>(),
                                           mask_words ? d_mask_.as<uint32_t>() : nullptr, d_hist_.as<int32_t>(),
                                           d_hoff_.as<int64_t>(), d_u_.as<double>(), 0, o, o + 5, o + 1, o + 2,
                                           o + 3, o + 4, stream_);
        std::vector<int32_t> h(5 + k + 1, 0);
        if (rc == SIXI_OK) {
            cudaMemcpyAsync(h.data(), o, h.size() * 4, cudaMemcpyDeviceToHost, stream_);
            if (cudaStreamSynchronize(stream_) != cudaSuccess) h[4] = SIXI_BACKEND_ERROR;
        } else {
            h[4] = rc;
        }
        rng.restore(ck);
        if (h[4] != SIXI_OK) return R(detail::status_of(h[4], "verify"));
        for (int32_t i = 0; i < h[3]; ++i) rng.next_uniform01();
        VerifyResult res;
        res.proposed_k = static_cast<uint32_t>(k);
        res.accepted_draft_count = static_cast<uint32_t>(h[0]);
        res.first_rejected_position = h[2];
        res.uniforms_used = static_cast<uint32_t>(h[3]);
        res.committed_tokens.assign(h.begin() + 5, h.begin() + 5 + h[1]);
        return R(std::move(res));
    }

    Status check_row(const float* logits, uint64_t vocab_size) const {
        if (logits == nullptr || vocab_size == 0)
            return Status::Error(ErrorCode::InvalidArgument, "logits must be non-null with vocab_size > 0");
        if (vocab_size != vocab_)
            return Status::Error(ErrorCode::InvalidArgument, "vocab_size differs from the sampler's vocabulary");
        return Status::Ok();
    }

    bool stage_logits(const float* logits, size_t n_rows, uint64_t vocab_size) {
        if (!d_logits_.ensure(n_rows * vocab_size * sizeof(float))) return false;
        return cudaMemcpyAsync(d_logits_.p, logits, n_rows * vocab_size * sizeof(float), cudaMemcpyHostToDevice,
                               stream_) == cudaSuccess;
    }

    // params, history, mask and uniform of one row to the device staging buffers
    Status stage_inputs(const sixi_smp_params& p, const std::vector<int32_t>& hist, const uint32_t* mask_words,
                        const double* u) {
        const size_t mw = sixi_smp_mask_words(h_);
        const int64_t hoff[2] = {0, static_cast<int64_t>(hist.size())};
        if (!d_params_.ensure(sizeof p) || !d_hist_.ensure(hist.size() * 4 + 4) || !d_hoff_.ensure(sizeof hoff) ||
            !d_u_.ensure(8) || (mask_words != nullptr && !d_mask_.ensure(mw * 4)))
            return oom();
        cudaMemcpyAsync(d_params_.p, &p, sizeof p, cudaMemcpyHostToDevice, stream_);
        if (!hist.empty()) cudaMemcpyAsync(d_hist_.p, hist.data(), hist.size() * 4, cudaMemcpyHostToDevice, stream_);
        cudaMemcpyAsync(d_hoff_.p, hoff, sizeof hoff, cudaMemcpyHostToDevice, stream_);
        if (u != nullptr) cudaMemcpyAsync(d_u_.p, u, 8, cudaMemcpyHostToDevice, stream_);
        if (mask_words != nullptr) cudaMemcpyAsync(d_mask_.p, mask_words, mw * 4, cudaMemcpyHostToDevice, stream_);
        return Status::Ok();
    }

    sixi_smp* h_ = nullptr;
    int device_ = 0;
    size_t max_rows_ = 0;
    uint32_t vocab_ = 0;
    cudaStream_t stream_ = nullptr;
    detail::DeviceBuffer d_logits_, d_params_, d_mask_, d_hist_, d_hoff_, d_u_, d_out_, d_cand_, d_q_, d_drafts_,
        d_vout_, d_rep_;
};

// Device-side grammar masks for `response_format: {"type": "json_object"}` answers
// (include/sixi_json.h): one uploaded vocabulary, automaton states in caller-owned device memory,
// asynchronous calls on the caller's stream. Together with DeviceSampler::sample_rows (masked
// rows) a constrained step never leaves the device.
class JsonMaskProducer {
public:
    // `texts[i]` is token i's text (the tokenizer's bytes), `special[i]` marks control tokens
    // (may be empty), `eos_id` the end-of-sequence token (or -1).
    static Result<std::unique_ptr<JsonMaskProducer>> create(int device, const std::vector<std::string>& texts,
                                                            const std::vector<uint8_t>& special, int32_t eos_id) {
        std::vector<uint64_t> off(texts.size() + 1, 0);
        for (size_t i = 0; i < texts.size(); ++i) off[i + 1] = off[i] + texts[i].size();
        std::string bytes;
        bytes.reserve(off.back());
        for (const auto& t : texts) bytes += t;
        std::vector<uint8_t> flags(texts.size(), 0);
        for (size_t i = 0; i < special.size() && i < flags.size(); ++i)
            flags[i] = special[i] ? static_cast<uint8_t>(SIXI_JSON_TOKEN_SPECIAL) : 0u;
        sixi_json_vocab* v = nullptr;
        const int32_t st = sixi_json_vocab_create(device, reinterpret_cast<const uint8_t*>(bytes.data()), off.data(),
                                                  static_cast<uint32_t>(texts.size()), flags.data(), eos_id, &v);
        if (st != SIXI_OK)
            return Result<std::unique_ptr<JsonMaskProducer>>(detail::status_of(st, "sixi_json_vocab_create"));
        return Result<std::unique_ptr<JsonMaskProducer>>(std::unique_ptr<JsonMaskProducer>(new JsonMaskProducer(v)));
    }
    ~JsonMaskProducer() { sixi_json_vocab_destroy(v_); }
    JsonMaskProducer(const JsonMaskProducer&) = delete;
    JsonMaskProducer& operator=(const JsonMaskProducer&) = delete;

    uint32_t vocab() const noexcept { return sixi_json_vocab_size(v_); }
    uint32_t mask_words() const noexcept { return (vocab() + 31u) / 32u; }

    Status reset(sixi_json_state* states, uint32_t n, cudaStream_t stream) const {
        return detail::status_of(sixi_json_reset(v_, states, n, stream), "sixi_json_reset");
    }
    Status fill_masks(const sixi_json_state* states, uint32_t n, uint32_t* masks, cudaStream_t stream) const {
        return detail::status_of(sixi_json_fill_masks(v_, states, n, masks, mask_words(), stream),
                                 "sixi_json_fill_masks");
    }
    Status advance(sixi_json_state* states, uint32_t n, const int32_t* tokens, int32_t* status,
                   cudaStream_t stream) const {
        return detail::status_of(sixi_json_advance(v_, states, n, tokens, 1, nullptr, status, stream),
                                 "sixi_json_advance");
    }
    // committed tokens of a speculative step: tokens[r * stride + j], j < counts[r]
    Status advance_many(sixi_json_state* states, uint32_t n, const int32_t* tokens, uint64_t stride,
                        const int32_t* counts, int32_t* status, cudaStream_t stream) const {
        return detail::status_of(sixi_json_advance(v_, states, n, tokens, stride, counts, status, stream),
                                 "sixi_json_advance");
    }
    Status expand_drafts(const sixi_json_state* states, uint32_t n_streams, const int32_t* drafts, uint32_t k,
                         const int32_t* n_drafts, sixi_json_state* out_states, cudaStream_t stream) const {
        return detail::status_of(
            sixi_json_expand_drafts(v_, states, n_streams, drafts, k, n_drafts, out_states, stream),
            "sixi_json_expand_drafts");
    }

private:
    explicit JsonMaskProducer(sixi_json_vocab* v) : v_(v) {}
    sixi_json_vocab* v_ = nullptr;
};

}  // namespace sixi_b200
