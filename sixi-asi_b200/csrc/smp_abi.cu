// smp_abi.cu - extern "C" boundary of the B200 logits-to-token path (include/sixi_smp.h).
//
// The entry points validate arguments, pick the launch plan for the handle's vocabulary and
// enqueue the row-engine kernels on the caller's stream. They never synchronise, except
// sixi_smp_sample_host, whose contract is the engine's host-side sample_token call shape.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <cstring>
#include <new>

#include "../../include/sixi_smp.h"
#include "smp_device.cuh"
#include "smp_kernels.cuh"

using sixi_b200::LaunchPlan;
using sixi_b200::RowArgs;
using sixi_b200::VerifyRowResult;

// Device staging of the host-buffer entry points: one slot per call in flight.
struct HostSlot {
    void* d_logits;
    size_t logits_cap;  // bytes
    sixi_smp_params* d_params;
    uint32_t* d_mask;
    int32_t* d_hist;
    size_t hist_cap;    // tokens
    int64_t* d_hoff;
    double* d_u;
    int32_t* d_tok;
    int32_t* d_status;
    size_t rows_cap;
    cudaEvent_t copied;    // its inputs are on the device (recorded on the copy stream)
    cudaEvent_t consumed;  // the call that used it has read its inputs and written its outputs
};

struct sixi_smp {
    int32_t device;
    uint32_t max_rows;
    uint32_t vocab;
    uint32_t mask_words;
    VerifyRowResult* ws;         // verifier per-row workspace [max_rows]
    sixi_b200::DraftStat* qstat; // draft-row distribution statistics [max_rows]
    sixi_smp_params* d_default;  // default params (raw argmax entry)
    // staging of sixi_smp_sample_host(_async): two slots used alternately, so that a call's
    // host->device copy (on copy_stream) overlaps the previous call's kernel
    HostSlot slot[2];
    uint32_t next_slot;
    cudaStream_t copy_stream;
};

namespace {

int32_t from_cuda(cudaError_t e) {
    if (e == cudaSuccess) return SIXI_OK;
    if (e == cudaErrorMemoryAllocation) return SIXI_OUT_OF_MEMORY_VRAM;
    return SIXI_BACKEND_ERROR;
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

// Verifier workspace of sixi_smp_verify_static: a file-scope device array (no allocation). Its
// address on each device is resolved once, by the first call on that device.
constexpr uint32_t kStaticVerifyRows = SIXI_SMP_STATIC_VERIFY_ROWS;
__device__ __align__(256) VerifyRowResult g_static_verify_ws[kStaticVerifyRows];
constexpr int kMaxDevices = 64;
std::atomic<VerifyRowResult*> g_static_ws_addr[kMaxDevices];

bool rows_ok(const sixi_smp* h, const sixi_smp_rows* rows) {
    if (rows == nullptr || (rows->n_rows > 0 && rows->data == nullptr)) return false;
    if (rows->dtype != SIXI_SMP_F32 && rows->dtype != SIXI_SMP_BF16) return false;
    if (rows->row_stride < h->vocab) return false;
    return true;
}

RowArgs base_args(const sixi_smp* h, const sixi_smp_rows* rows, LaunchPlan* plan) {
    RowArgs a;
    std::memset(&a, 0, sizeof(a));
    sixi_b200::plan_rows(h->vocab, rows->n_rows, sixi_b200::device_sm_count(h->device), plan, h->device);
    a.data = rows->data;
    a.row_stride = rows->row_stride;
    a.dtype = rows->dtype;
    a.vocab = h->vocab;
    a.n_rows = rows->n_rows;
    a.chunk = plan->chunk;
    const size_t esz = rows->dtype == SIXI_SMP_BF16 ? 2 : 4;
    a.use_tma = ((reinterpret_cast<uintptr_t>(rows->data) & 15u) == 0 &&
                 (rows->row_stride * esz) % 16 == 0)
                    ? 1u
                    : 0u;
    a.mask_words = h->mask_words;
    return a;
}

template <typename T>
cudaError_t grow(T** p, size_t* cap, size_t need) {
    if (*cap >= need && *p != nullptr) return cudaSuccess;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), need * sizeof(T));
    if (e == cudaSuccess) *cap = need;
    return e;
}

// Verification with dense q stored (draft_probs), evaluated from draft logits (qlog with their
// temperatures: a statistics pass first), or one-hot (neither).
int32_t verify_impl(sixi_smp* h, const sixi_smp_rows* target, const float* draft_probs,
                    const sixi_smp_rows* qlog, const float* qlog_temps, const int32_t* drafts,
                    const int32_t* n_drafts, uint32_t n_streams, uint32_t k, const sixi_smp_params* params,
                    const uint32_t* mask_words, const int32_t* hist_tokens, const int64_t* hist_offsets,
                    const double* uniforms, uint64_t step, int32_t* out_accepted, int32_t* out_tokens,
                    int32_t* out_n_tokens, int32_t* out_first_reject, int32_t* out_uniforms_used,
                    int32_t* out_status, void* stream) {
    if (h == nullptr || !rows_ok(h, target) || params == nullptr || drafts == nullptr ||
        out_accepted == nullptr || out_tokens == nullptr || out_n_tokens == nullptr ||
        out_first_reject == nullptr || out_uniforms_used == nullptr || out_status == nullptr ||
        (hist_tokens != nullptr && hist_offsets == nullptr) || k == 0)
        return SIXI_INVALID_ARGUMENT;
    if (static_cast<uint64_t>(n_streams) * (k + 1) != target->n_rows) return SIXI_INVALID_ARGUMENT;
    if (target->n_rows > h->max_rows) return SIXI_INVALID_ARGUMENT;
    if (n_streams == 0) return SIXI_OK;
    if (draft_probs != nullptr && (reinterpret_cast<uintptr_t>(draft_probs) & 3u) != 0)
        return SIXI_INVALID_ARGUMENT;
    DeviceGuard g(h->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSuccess;
    if (qlog != nullptr) {
        // the draft rows' maxima and sums, with the plan sixi_smp_full_distribution uses for them
        LaunchPlan dplan{};
        if (!sixi_b200::plan_rows(h->vocab, qlog->n_rows, sixi_b200::device_sm_count(h->device), &dplan))
            return SIXI_INVALID_ARGUMENT;
        sixi_b200::DistArgs d{};
        d.data = qlog->data;
        d.row_stride = qlog->row_stride;
        d.dtype = qlog->dtype;
        d.vocab = h->vocab;
        d.n_rows = qlog->n_rows;
        d.chunk = dplan.chunk;
        d.temperatures = qlog_temps;
        d.out = nullptr;
        d.stats = h->qstat;
        e = sixi_b200::launch_full_distribution(d, dplan, s);
    }
    LaunchPlan plan{};
    RowArgs a = base_args(h, target, &plan);
    a.params = params;
    a.mask = mask_words;
    a.hist = hist_tokens;
    a.hist_off = hist_tokens ? hist_offsets : nullptr;
    a.uniforms = uniforms;
    a.step = step;
    a.q = draft_probs;
    if (qlog != nullptr) {
        a.qlog = qlog->data;
        a.qlog_stride = qlog->row_stride;
        a.qlog_dtype = qlog->dtype;
        a.qstat = h->qstat;
    }
    a.drafts = drafts;
    a.n_drafts = n_drafts;
    a.k = k;
    a.ws = h->ws;
    if (e == cudaSuccess) e = sixi_b200::launch_rows(sixi_b200::kModeVerify, a, plan, s);
    if (e == cudaSuccess)
        e = sixi_b200::launch_verify_finalize(a, n_streams, out_accepted, out_tokens, out_n_tokens,
                                              out_first_reject, out_uniforms_used, out_status, s);
    return from_cuda(e);
}

}  // namespace

extern "C" {

int32_t sixi_smp_create(int32_t device, uint32_t max_rows, uint32_t vocab, sixi_smp** out) {
    if (out == nullptr) return SIXI_INVALID_ARGUMENT;
    *out = nullptr;
    LaunchPlan plan{};
    if (vocab == 0 || !sixi_b200::plan_rows(vocab, 1, 0, &plan)) return SIXI_INVALID_ARGUMENT;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return SIXI_INVALID_ARGUMENT;
    DeviceGuard g(device);
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return SIXI_BACKEND_ERROR;
    if (prop.major < 10) return SIXI_UNSUPPORTED_HARDWARE;
    sixi_smp* h = new (std::nothrow) sixi_smp;
    if (h == nullptr) return SIXI_OUT_OF_MEMORY_VRAM;
    std::memset(h, 0, sizeof(*h));
    h->device = device;
    h->max_rows = max_rows;
    h->vocab = vocab;
    h->mask_words = (vocab + 31u) / 32u;
    cudaError_t e = cudaSuccess;
    if (max_rows > 0) e = cudaMalloc(&h->ws, sizeof(VerifyRowResult) * max_rows);
    if (e == cudaSuccess && max_rows > 0) e = cudaMalloc(&h->qstat, sizeof(sixi_b200::DraftStat) * max_rows);
    if (e == cudaSuccess) e = cudaMalloc(&h->d_default, sizeof(sixi_smp_params));
    if (e == cudaSuccess) {
        sixi_smp_params p;
        std::memset(&p, 0, sizeof(p));
        p.top_k = 0;
        p.top_p = 1.0f;
        p.repetition_penalty = 1.0f;
        e = cudaMemcpy(h->d_default, &p, sizeof(p), cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess) e = sixi_b200::prepare_kernels(device);
    // resident-cluster counts for the launch plans; without them the plans use the SM count alone
    if (e == cudaSuccess && sixi_b200::prepare_plans(device, vocab) != cudaSuccess) (void)cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&h->copy_stream, cudaStreamNonBlocking);
    for (int i = 0; i < 2 && e == cudaSuccess; ++i) {
        e = cudaEventCreateWithFlags(&h->slot[i].copied, cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&h->slot[i].consumed, cudaEventDisableTiming);
    }
    if (e != cudaSuccess) {
        sixi_smp_destroy(h);
        return from_cuda(e);
    }
    *out = h;
    return SIXI_OK;
}

int32_t sixi_smp_destroy(sixi_smp* h) {
    if (h == nullptr) return SIXI_OK;
    DeviceGuard g(h->device);
    if (h->copy_stream != nullptr) cudaStreamSynchronize(h->copy_stream);
    for (HostSlot& sl : h->slot) {
        if (sl.consumed != nullptr) cudaEventSynchronize(sl.consumed);
        cudaFree(sl.d_logits);
        cudaFree(sl.d_params);
        cudaFree(sl.d_mask);
        cudaFree(sl.d_hist);
        cudaFree(sl.d_hoff);
        cudaFree(sl.d_u);
        cudaFree(sl.d_tok);
        cudaFree(sl.d_status);
        if (sl.copied != nullptr) cudaEventDestroy(sl.copied);
        if (sl.consumed != nullptr) cudaEventDestroy(sl.consumed);
    }
    if (h->copy_stream != nullptr) cudaStreamDestroy(h->copy_stream);
    cudaFree(h->ws);
    cudaFree(h->qstat);
    cudaFree(h->d_default);
    delete h;
    return SIXI_OK;
}

uint32_t sixi_smp_vocab(const sixi_smp* h) { return h ? h->vocab : 0u; }
uint32_t sixi_smp_mask_words(const sixi_smp* h) { return h ? h->mask_words : 0u; }

const char* sixi_smp_status_string(int32_t status) {
    switch (status) {
        case SIXI_OK: return "Ok";
        case SIXI_INVALID_ARGUMENT: return "InvalidArgument";
        case SIXI_OUT_OF_BOUNDS: return "OutOfBounds";
        case SIXI_OUT_OF_MEMORY_VRAM: return "OutOfMemoryVRAM";
        case SIXI_NUMERIC_NAN_OR_INF: return "NumericNaNOrInf";
        case SIXI_BACKEND_ERROR: return "BackendError";
        case SIXI_UNSUPPORTED_HARDWARE: return "UnsupportedHardware";
        default: return "Unknown";
    }
}

double sixi_smp_philox_uniform(uint64_t seed, uint64_t counter, uint32_t slot) {
    return sixi_b200::philox_uniform(seed, counter, slot);
}

int32_t sixi_smp_sample(sixi_smp* h, const sixi_smp_rows* rows, const sixi_smp_params* params,
                        const uint32_t* mask_words, const int32_t* hist_tokens,
                        const int64_t* hist_offsets, const double* uniforms, uint64_t step,
                        int32_t* out_tokens, int32_t* out_status, void* stream) {
    if (h == nullptr || !rows_ok(h, rows) || params == nullptr || out_tokens == nullptr ||
        out_status == nullptr || (hist_tokens != nullptr && hist_offsets == nullptr))
        return SIXI_INVALID_ARGUMENT;
    if (rows->n_rows == 0) return SIXI_OK;
    DeviceGuard g(h->device);
    LaunchPlan plan{};
    RowArgs a = base_args(h, rows, &plan);
    a.params = params;
    a.mask = mask_words;
    a.hist = hist_tokens;
    a.hist_off = hist_tokens ? hist_offsets : nullptr;
    a.uniforms = uniforms;
    a.step = step;
    a.out_tok = out_tokens;
    a.out_status = out_status;
    return from_cuda(sixi_b200::launch_rows(sixi_b200::kModeSample, a, plan,
                                            static_cast<cudaStream_t>(stream)));
}

int32_t sixi_smp_sample_indexed(sixi_smp* h, const sixi_smp_rows* rows, const uint32_t* row_map,
                                const sixi_smp_params* params, const uint32_t* mask_words, const int32_t* hist_tokens,
                                const int64_t* hist_offsets, const double* uniforms, uint64_t step,
                                int32_t* out_tokens, int32_t* out_status, void* stream) {
    if (h == nullptr || !rows_ok(h, rows) || row_map == nullptr || params == nullptr || out_tokens == nullptr ||
        out_status == nullptr || (hist_tokens != nullptr && hist_offsets == nullptr))
        return SIXI_INVALID_ARGUMENT;
    if (rows->n_rows == 0) return SIXI_OK;
    DeviceGuard g(h->device);
    LaunchPlan plan{};
    RowArgs a = base_args(h, rows, &plan);
    a.params = params;
    a.mask = mask_words;
    a.hist = hist_tokens;
    a.hist_off = hist_tokens ? hist_offsets : nullptr;
    a.uniforms = uniforms;
    a.step = step;
    a.row_map = row_map;
    a.out_tok = out_tokens;
    a.out_status = out_status;
    return from_cuda(sixi_b200::launch_rows(sixi_b200::kModeSample, a, plan, static_cast<cudaStream_t>(stream)));
}

int32_t sixi_smp_gather_rows(sixi_smp* h, const sixi_smp_rows* src, const int32_t* row_index, uint32_t n,
                             uint32_t width, void* dst, uint64_t dst_stride, void* stream) {
    if (h == nullptr || src == nullptr || (src->dtype != SIXI_SMP_F32 && src->dtype != SIXI_SMP_BF16) ||
        width > src->row_stride || width > dst_stride || n > 65535u ||
        (n > 0 && (src->data == nullptr || row_index == nullptr || dst == nullptr)))
        return SIXI_INVALID_ARGUMENT;
    if (n == 0 || width == 0) return SIXI_OK;
    DeviceGuard g(h->device);
    return from_cuda(sixi_b200::launch_gather_rows(src->data, src->row_stride, src->dtype == SIXI_SMP_BF16 ? 2u : 4u,
                                                   row_index, n, width, dst, dst_stride,
                                                   static_cast<cudaStream_t>(stream)));
}

int32_t sixi_smp_sample_host_async(sixi_smp* h, const void* host_logits, uint32_t dtype, uint32_t n_rows,
                                   uint64_t row_stride, const sixi_smp_params* host_params,
                                   const uint32_t* host_mask_words, const int32_t* host_hist_tokens,
                                   const int64_t* host_hist_offsets, const double* host_uniforms, uint64_t step,
                                   int32_t* host_out_tokens, int32_t* host_out_status, void* stream) {
    if (h == nullptr || host_logits == nullptr || host_params == nullptr ||
        host_out_tokens == nullptr || host_out_status == nullptr || row_stride < h->vocab ||
        (dtype != SIXI_SMP_F32 && dtype != SIXI_SMP_BF16) ||
        (host_hist_tokens != nullptr && host_hist_offsets == nullptr))
        return SIXI_INVALID_ARGUMENT;
    if (n_rows == 0) return SIXI_OK;
    DeviceGuard g(h->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    HostSlot& sl = h->slot[h->next_slot];
    const size_t esz = dtype == SIXI_SMP_BF16 ? 2 : 4;
    const size_t lbytes = static_cast<size_t>(n_rows) * row_stride * esz;
    const int64_t nh = host_hist_tokens != nullptr ? host_hist_offsets[n_rows] : 0;
    cudaError_t e = cudaSuccess;
    // growth reallocates the slot: wait for the call that last used it first
    const bool grow_rows = sl.d_params == nullptr || sl.rows_cap < n_rows;
    if (sl.logits_cap < lbytes || grow_rows || (nh > 0 && sl.hist_cap < static_cast<size_t>(nh)))
        e = cudaEventSynchronize(sl.consumed);
    if (e == cudaSuccess) e = grow(reinterpret_cast<uint8_t**>(&sl.d_logits), &sl.logits_cap, lbytes);
    if (e == cudaSuccess && grow_rows) {
        cudaFree(sl.d_params);
        cudaFree(sl.d_u);
        cudaFree(sl.d_tok);
        cudaFree(sl.d_status);
        cudaFree(sl.d_mask);
        cudaFree(sl.d_hoff);
        sl.d_params = nullptr;
        sl.d_u = nullptr;
        sl.d_tok = nullptr;
        sl.d_status = nullptr;
        sl.d_mask = nullptr;
        sl.d_hoff = nullptr;
        e = cudaMalloc(&sl.d_params, sizeof(sixi_smp_params) * n_rows);
        if (e == cudaSuccess) e = cudaMalloc(&sl.d_u, sizeof(double) * n_rows);
        if (e == cudaSuccess) e = cudaMalloc(&sl.d_tok, sizeof(int32_t) * n_rows);
        if (e == cudaSuccess) e = cudaMalloc(&sl.d_status, sizeof(int32_t) * n_rows);
        if (e == cudaSuccess) e = cudaMalloc(&sl.d_mask, sizeof(uint32_t) * h->mask_words * n_rows);
        if (e == cudaSuccess) e = cudaMalloc(&sl.d_hoff, sizeof(int64_t) * (n_rows + 1));
        sl.rows_cap = (e == cudaSuccess) ? n_rows : 0;
    }
    if (e == cudaSuccess && nh > 0) e = grow(&sl.d_hist, &sl.hist_cap, static_cast<size_t>(nh));
    if (e != cudaSuccess) return from_cuda(e);
    // inputs -> the slot on the copy stream, once the call that last used the slot is done with it
    cudaStream_t c = h->copy_stream;
    e = cudaStreamWaitEvent(c, sl.consumed, 0);
    if (e == cudaSuccess) e = cudaMemcpyAsync(sl.d_logits, host_logits, lbytes, cudaMemcpyHostToDevice, c);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(sl.d_params, host_params, sizeof(sixi_smp_params) * n_rows, cudaMemcpyHostToDevice, c);
    if (e == cudaSuccess && host_mask_words)
        e = cudaMemcpyAsync(sl.d_mask, host_mask_words, sizeof(uint32_t) * h->mask_words * n_rows,
                            cudaMemcpyHostToDevice, c);
    if (e == cudaSuccess && nh > 0) {
        e = cudaMemcpyAsync(sl.d_hist, host_hist_tokens, sizeof(int32_t) * static_cast<size_t>(nh),
                            cudaMemcpyHostToDevice, c);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(sl.d_hoff, host_hist_offsets, sizeof(int64_t) * (n_rows + 1), cudaMemcpyHostToDevice, c);
    }
    if (e == cudaSuccess && host_uniforms)
        e = cudaMemcpyAsync(sl.d_u, host_uniforms, sizeof(double) * n_rows, cudaMemcpyHostToDevice, c);
    if (e == cudaSuccess) e = cudaEventRecord(sl.copied, c);
    // the kernel and the read-back on the caller's stream, after the copies
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s, sl.copied, 0);
    if (e != cudaSuccess) return from_cuda(e);
    h->next_slot ^= 1u;
    sixi_smp_rows rows{sl.d_logits, dtype, n_rows, row_stride};
    const int32_t st = sixi_smp_sample(h, &rows, sl.d_params, host_mask_words ? sl.d_mask : nullptr,
                                       nh > 0 ? sl.d_hist : nullptr, nh > 0 ? sl.d_hoff : nullptr,
                                       host_uniforms ? sl.d_u : nullptr, step, sl.d_tok, sl.d_status, stream);
    if (st != SIXI_OK) {
        cudaEventRecord(sl.consumed, s);
        return st;
    }
    e = cudaMemcpyAsync(host_out_tokens, sl.d_tok, sizeof(int32_t) * n_rows, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(host_out_status, sl.d_status, sizeof(int32_t) * n_rows, cudaMemcpyDeviceToHost, s);
    const cudaError_t e2 = cudaEventRecord(sl.consumed, s);
    return from_cuda(e != cudaSuccess ? e : e2);
}

int32_t sixi_smp_sample_host(sixi_smp* h, const void* host_logits, uint32_t dtype,
                             uint32_t n_rows, uint64_t row_stride,
                             const sixi_smp_params* host_params, const uint32_t* host_mask_words,
                             const int32_t* host_hist_tokens, const int64_t* host_hist_offsets,
                             const double* host_uniforms, uint64_t step, int32_t* host_out_tokens,
                             int32_t* host_out_status, void* stream) {
    const int32_t st = sixi_smp_sample_host_async(h, host_logits, dtype, n_rows, row_stride, host_params,
                                                  host_mask_words, host_hist_tokens, host_hist_offsets,
                                                  host_uniforms, step, host_out_tokens, host_out_status, stream);
    if (st != SIXI_OK || n_rows == 0) return st;
    DeviceGuard g(h->device);
    return from_cuda(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
}

int32_t sixi_smp_greedy_argmax(sixi_smp* h, const sixi_smp_rows* rows, const uint32_t* mask_words,
                               int32_t* out_tokens, int32_t* out_status, void* stream) {
    if (h == nullptr || !rows_ok(h, rows) || out_tokens == nullptr || out_status == nullptr)
        return SIXI_INVALID_ARGUMENT;
    if (rows->n_rows == 0) return SIXI_OK;
    DeviceGuard g(h->device);
    LaunchPlan plan{};
    RowArgs a = base_args(h, rows, &plan);
    a.params = h->d_default;
    a.mask = mask_words;
    a.out_tok = out_tokens;
    a.out_status = out_status;
    return from_cuda(sixi_b200::launch_rows(sixi_b200::kModeGreedy, a, plan,
                                            static_cast<cudaStream_t>(stream)));
}

int32_t sixi_smp_candidates(sixi_smp* h, const sixi_smp_rows* rows, const sixi_smp_params* params,
                            const uint32_t* mask_words, const int32_t* hist_tokens,
                            const int64_t* hist_offsets, uint32_t max_out, int32_t* out_ids,
                            double* out_probs, int32_t* out_count, int32_t* out_status,
                            void* stream) {
    if (h == nullptr || !rows_ok(h, rows) || params == nullptr || max_out == 0 || max_out > 256 ||
        out_ids == nullptr || out_probs == nullptr || out_count == nullptr || out_status == nullptr ||
        (hist_tokens != nullptr && hist_offsets == nullptr))
        return SIXI_INVALID_ARGUMENT;
    if (rows->n_rows == 0) return SIXI_OK;
    DeviceGuard g(h->device);
    LaunchPlan plan{};
    RowArgs a = base_args(h, rows, &plan);
    a.params = params;
    a.mask = mask_words;
    a.hist = hist_tokens;
    a.hist_off = hist_tokens ? hist_offsets : nullptr;
    a.max_out = max_out;
    a.out_ids = out_ids;
    a.out_probs = out_probs;
    a.out_count = out_count;
    a.out_status = out_status;
    return from_cuda(sixi_b200::launch_rows(sixi_b200::kModeCandidates, a, plan,
                                            static_cast<cudaStream_t>(stream)));
}

int32_t sixi_smp_verify(sixi_smp* h, const sixi_smp_rows* target, const float* draft_probs,
                        const int32_t* drafts, const int32_t* n_drafts, uint32_t n_streams,
                        uint32_t k, const sixi_smp_params* params, const uint32_t* mask_words,
                        const int32_t* hist_tokens, const int64_t* hist_offsets,
                        const double* uniforms, uint64_t step, int32_t* out_accepted,
                        int32_t* out_tokens, int32_t* out_n_tokens, int32_t* out_first_reject,
                        int32_t* out_uniforms_used, int32_t* out_status, void* stream) {
    return verify_impl(h, target, draft_probs, nullptr, nullptr, drafts, n_drafts, n_streams, k, params, mask_words,
                       hist_tokens, hist_offsets, uniforms, step, out_accepted, out_tokens, out_n_tokens,
                       out_first_reject, out_uniforms_used, out_status, stream);
}

int32_t sixi_smp_verify_draft_logits(sixi_smp* h, const sixi_smp_rows* target, const sixi_smp_rows* draft_logits,
                                     const float* draft_temperatures, const int32_t* drafts,
                                     const int32_t* n_drafts, uint32_t n_streams, uint32_t k,
                                     const sixi_smp_params* params, const uint32_t* mask_words,
                                     const int32_t* hist_tokens, const int64_t* hist_offsets,
                                     const double* uniforms, uint64_t step, int32_t* out_accepted,
                                     int32_t* out_tokens, int32_t* out_n_tokens, int32_t* out_first_reject,
                                     int32_t* out_uniforms_used, int32_t* out_status, void* stream) {
    if (h == nullptr || draft_logits == nullptr || !rows_ok(h, draft_logits) || draft_temperatures == nullptr ||
        static_cast<uint64_t>(n_streams) * k != draft_logits->n_rows)
        return SIXI_INVALID_ARGUMENT;
    return verify_impl(h, target, nullptr, draft_logits, draft_temperatures, drafts, n_drafts, n_streams, k, params,
                       mask_words, hist_tokens, hist_offsets, uniforms, step, out_accepted, out_tokens,
                       out_n_tokens, out_first_reject, out_uniforms_used, out_status, stream);
}

int32_t sixi_smp_full_distribution(sixi_smp* h, const sixi_smp_rows* rows, const float* temperatures,
                                   float* out_probs, uint64_t out_stride, void* stream) {
    if (h == nullptr || !rows_ok(h, rows) || temperatures == nullptr || out_probs == nullptr ||
        out_stride < h->vocab)
        return SIXI_INVALID_ARGUMENT;
    if (rows->n_rows == 0) return SIXI_OK;
    DeviceGuard g(h->device);
    LaunchPlan plan{};
    if (!sixi_b200::plan_rows(h->vocab, rows->n_rows, sixi_b200::device_sm_count(h->device), &plan))
        return SIXI_INVALID_ARGUMENT;
    sixi_b200::DistArgs a{};
    a.data = rows->data;
    a.row_stride = rows->row_stride;
    a.dtype = rows->dtype;
    a.vocab = h->vocab;
    a.n_rows = rows->n_rows;
    a.chunk = plan.chunk;
    a.temperatures = temperatures;
    a.out = out_probs;
    a.out_stride = out_stride;
    return from_cuda(sixi_b200::launch_full_distribution(a, plan, static_cast<cudaStream_t>(stream)));
}

int32_t sixi_smp_numeric_policy(sixi_smp* h, float* rows, uint32_t n_rows, uint64_t row_stride, uint32_t policy,
                                float clamp_abs_max, sixi_smp_numeric_report* out_reports, void* stream) {
    if (h == nullptr || out_reports == nullptr || (n_rows > 0 && rows == nullptr) || row_stride < h->vocab ||
        (policy != SIXI_SMP_NUMERIC_FAIL && policy != SIXI_SMP_NUMERIC_CLAMP) ||
        (reinterpret_cast<uintptr_t>(rows) & 3u) != 0 || (reinterpret_cast<uintptr_t>(out_reports) & 7u) != 0)
        return SIXI_INVALID_ARGUMENT;
    if (n_rows == 0) return SIXI_OK;
    DeviceGuard g(h->device);
    // numeric.cpp:641: the clamp bound is the magnitude of clamp_abs_max
    const float limit = fabsf(clamp_abs_max);
    return from_cuda(sixi_b200::launch_numeric_policy(rows, n_rows, row_stride, h->vocab, policy, limit, out_reports,
                                                      static_cast<cudaStream_t>(stream)));
}

int32_t sixi_smp_suffix_draft(sixi_smp* h, const int32_t* hist_tokens, const int64_t* hist_offsets, uint32_t n_streams,
                              uint32_t min_match_len, uint32_t max_window_tokens, const int32_t* anchors, uint32_t k,
                              int32_t* out_drafts, int32_t* out_match_len, void* stream) {
    if (h == nullptr || hist_offsets == nullptr || out_match_len == nullptr || (k > 0 && out_drafts == nullptr) ||
        min_match_len > 64u || k > 4096u)
        return SIXI_INVALID_ARGUMENT;
    if (n_streams == 0) return SIXI_OK;
    DeviceGuard g(h->device);
    return from_cuda(sixi_b200::launch_suffix_draft(hist_tokens, hist_offsets, n_streams, min_match_len,
                                                    max_window_tokens, anchors, k, out_drafts, out_match_len,
                                                    static_cast<cudaStream_t>(stream)));
}

int32_t sixi_smp_verify_static(int32_t device, uint32_t vocab, const sixi_smp_rows* target,
                               const float* draft_probs, const int32_t* drafts, const int32_t* n_drafts,
                               uint32_t n_streams, uint32_t k, const sixi_smp_params* params,
                               const uint32_t* mask_words, const int32_t* hist_tokens,
                               const int64_t* hist_offsets, const double* uniforms, uint64_t step,
                               int32_t* out_accepted, int32_t* out_tokens, int32_t* out_n_tokens,
                               int32_t* out_first_reject, int32_t* out_uniforms_used, int32_t* out_status,
                               void* stream) {
    LaunchPlan plan{};
    if (device < 0 || device >= kMaxDevices || vocab == 0 || !sixi_b200::plan_rows(vocab, 1, 0, &plan))
        return SIXI_INVALID_ARGUMENT;
    if (target == nullptr || (target->n_rows > 0 && target->data == nullptr) ||
        (target->dtype != SIXI_SMP_F32 && target->dtype != SIXI_SMP_BF16) || target->row_stride < vocab ||
        params == nullptr || drafts == nullptr || out_accepted == nullptr || out_tokens == nullptr ||
        out_n_tokens == nullptr || out_first_reject == nullptr || out_uniforms_used == nullptr ||
        out_status == nullptr || (hist_tokens != nullptr && hist_offsets == nullptr) || k == 0)
        return SIXI_INVALID_ARGUMENT;
    if (static_cast<uint64_t>(n_streams) * (k + 1) != target->n_rows) return SIXI_INVALID_ARGUMENT;
    if (target->n_rows > kStaticVerifyRows) return SIXI_OUT_OF_BOUNDS;  // larger than the static workspace
    if (n_streams == 0) return SIXI_OK;
    if (draft_probs != nullptr && (reinterpret_cast<uintptr_t>(draft_probs) & 3u) != 0)
        return SIXI_INVALID_ARGUMENT;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device >= n) return SIXI_INVALID_ARGUMENT;
    DeviceGuard g(device);
    VerifyRowResult* ws = g_static_ws_addr[device].load(std::memory_order_acquire);
    if (ws == nullptr) {  // first call on this device: check the architecture, set the launch
                          // attributes of every kernel instance, resolve the workspace address
        cudaDeviceProp prop;
        if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return SIXI_BACKEND_ERROR;
        if (prop.major < 10) return SIXI_UNSUPPORTED_HARDWARE;
        if (sixi_b200::prepare_kernels(device) != cudaSuccess) return SIXI_BACKEND_ERROR;
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_static_verify_ws) != cudaSuccess || p == nullptr) return SIXI_BACKEND_ERROR;
        ws = static_cast<VerifyRowResult*>(p);
        g_static_ws_addr[device].store(ws, std::memory_order_release);
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    sixi_smp probe_h;  // the fields base_args reads; no memory is attached to it
    std::memset(&probe_h, 0, sizeof(probe_h));
    probe_h.device = device;
    probe_h.vocab = vocab;
    probe_h.mask_words = (vocab + 31u) / 32u;
    RowArgs a = base_args(&probe_h, target, &plan);
    a.params = params;
    a.mask = mask_words;
    a.hist = hist_tokens;
    a.hist_off = hist_tokens ? hist_offsets : nullptr;
    a.uniforms = uniforms;
    a.step = step;
    a.q = draft_probs;
    a.drafts = drafts;
    a.n_drafts = n_drafts;
    a.k = k;
    a.ws = ws;
    cudaError_t e = sixi_b200::launch_rows(sixi_b200::kModeVerify, a, plan, s);
    if (e == cudaSuccess)
        e = sixi_b200::launch_verify_finalize(a, n_streams, out_accepted, out_tokens, out_n_tokens,
                                              out_first_reject, out_uniforms_used, out_status, s);
    return from_cuda(e);
}

int32_t sixi_smp_shard_candidates(sixi_smp* h, const sixi_smp_rows* shard_rows, uint32_t vocab_offset,
                                  uint32_t shard_vocab, uint32_t full_vocab, const sixi_smp_params* params,
                                  const uint32_t* mask_words, const int32_t* hist_tokens,
                                  const int64_t* hist_offsets, uint32_t top_n, void* out_cand, void* out_stats,
                                  void* stream) {
    if (h == nullptr || shard_rows == nullptr || params == nullptr || out_cand == nullptr || out_stats == nullptr ||
        (shard_rows->n_rows > 0 && shard_rows->data == nullptr) ||
        (shard_rows->dtype != SIXI_SMP_F32 && shard_rows->dtype != SIXI_SMP_BF16) ||
        (hist_tokens != nullptr && hist_offsets == nullptr))
        return SIXI_INVALID_ARGUMENT;
    if (full_vocab != h->vocab || shard_vocab == 0 || shard_vocab > shard_rows->row_stride ||
        static_cast<uint64_t>(vocab_offset) + shard_vocab > full_vocab || top_n == 0 ||
        top_n > sixi_b200::kMaxShardTopN || sixi_b200::shard_smem_bytes(shard_vocab) > sixi_b200::kMaxShardSmem)
        return SIXI_INVALID_ARGUMENT;
    if (shard_rows->n_rows == 0) return SIXI_OK;
    DeviceGuard g(h->device);
    sixi_b200::ShardArgs a{};
    a.data = shard_rows->data;
    a.row_stride = shard_rows->row_stride;
    a.dtype = shard_rows->dtype;
    a.shard_vocab = shard_vocab;
    a.vocab_offset = vocab_offset;
    a.full_vocab = full_vocab;
    a.mask_words = h->mask_words;
    a.n_rows = shard_rows->n_rows;
    a.top_n = top_n;
    a.params = params;
    a.mask = mask_words;
    a.hist = hist_tokens;
    a.hist_off = hist_tokens ? hist_offsets : nullptr;
    a.out_cand = static_cast<sixi_b200::ShardCand*>(out_cand);
    a.out_stats = static_cast<sixi_b200::ShardStats*>(out_stats);
    return from_cuda(sixi_b200::launch_shard_candidates(a, static_cast<cudaStream_t>(stream)));
}

int32_t sixi_smp_merge_shards(sixi_smp* h, uint32_t n_rows, uint32_t n_shards, uint32_t top_n,
                              const void* gathered_cand, const void* gathered_stats, const sixi_smp_params* params,
                              const double* uniforms, uint64_t step, int32_t* out_tokens, int32_t* out_status,
                              void* stream) {
    if (h == nullptr || gathered_cand == nullptr || gathered_stats == nullptr || params == nullptr ||
        out_tokens == nullptr || out_status == nullptr || n_shards == 0 || n_shards > sixi_b200::kMaxShards ||
        top_n == 0 || top_n > sixi_b200::kMaxShardTopN || n_shards * top_n > 1024u)
        return SIXI_INVALID_ARGUMENT;
    if (n_rows == 0) return SIXI_OK;
    DeviceGuard g(h->device);
    sixi_b200::MergeArgs a{};
    a.n_rows = n_rows;
    a.n_shards = n_shards;
    a.top_n = top_n;
    a.cand = static_cast<const sixi_b200::ShardCand*>(gathered_cand);
    a.stats = static_cast<const sixi_b200::ShardStats*>(gathered_stats);
    a.params = params;
    a.uniforms = uniforms;
    a.step = step;
    a.out_tok = out_tokens;
    a.out_status = out_status;
    return from_cuda(sixi_b200::launch_merge_shards(a, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
