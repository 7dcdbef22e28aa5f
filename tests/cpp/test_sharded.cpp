// test_sharded.cpp - the C++ vocab-sharded step (sixi-asi_b200/host/sixi_sharded.hpp, NCCL C API)
// against the same stages composed on one GPU.
//
// Config-2 rows (N(0, 2.5^2) logits with 16 ids per row boosted by +8; temperature 0.3-1.2 with a
// quarter greedy, top-k in {0, 20, 40, 100}, top-p 0.7-1.0, repetition penalty 1.0-1.3, Adaptive
// mode, histories of 64-2,048 ids) are split by vocabulary over S ranks, one thread and one GPU
// per rank, with communicators from ncclCommInitAll. Expected on every rank and every row:
//   - rows stage 2 certifies: the token and status of sixi_smp_merge_shards run on device 0 over
//     the slices' stage-1 outputs stacked rank-major (what the all-gather must deliver);
//   - rows it flags (SIXI_OUT_OF_BOUNDS): the token and status of sixi_smp_sample on the full row
//     (what round 2 must rebuild and sample).
// Runs S = 1 (V = 50,000: one slice holds the whole row) and, with two or more GPUs, S = 2
// (V = 151,936). Exit status 0 when every check passes.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>

#include "sixi_sharded.hpp"

using namespace sixi_b200;

namespace {

int g_fail = 0;
#define CHECK(cond)                                                                       \
    do {                                                                                  \
        if (!(cond)) {                                                                    \
            std::fprintf(stderr, "CHECK failed %s:%d: %s\n", __FILE__, __LINE__, #cond);  \
            ++g_fail;                                                                     \
            return false;                                                                 \
        }                                                                                 \
    } while (0)

struct Gen {  // SplitMix64 + Box-Muller (test data only)
    uint64_t s;
    explicit Gen(uint64_t seed) : s(seed) {}
    uint64_t next() {
        uint64_t z = (s += 0x9E3779B97F4A7C15ull);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    }
    double uni() { return static_cast<double>(next() >> 11) * 0x1.0p-53; }
    float normal(float sigma) {
        const double u1 = std::max(uni(), 1e-300), u2 = uni();
        return static_cast<float>(sigma * std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2));
    }
};

struct Batch {
    uint32_t n = 0, V = 0;
    std::vector<float> logits;  // [n][V]
    std::vector<sixi_smp_params> params;
    std::vector<int32_t> hist;
    std::vector<int64_t> hoff;
    std::vector<double> u;
};

Batch make_batch(uint32_t n, uint32_t V, uint64_t seed) {
    Gen g(seed);
    Batch b;
    b.n = n;
    b.V = V;
    b.logits.resize(static_cast<size_t>(n) * V);
    for (auto& x : b.logits) x = g.normal(2.5f);
    const int32_t ks[4] = {0, 20, 40, 100};
    b.hoff.push_back(0);
    for (uint32_t r = 0; r < n; ++r) {
        for (int j = 0; j < 16; ++j) b.logits[static_cast<size_t>(r) * V + g.next() % V] += 8.0f;
        sixi_smp_params p{};
        p.temperature = g.uni() < 0.25 ? 0.0f : static_cast<float>(0.3 + 0.9 * g.uni());
        p.top_k = ks[g.next() % 4];
        p.top_p = static_cast<float>(0.7 + 0.3 * g.uni());
        p.repetition_penalty = static_cast<float>(1.0 + 0.3 * g.uni());
        p.mode = SIXI_SMP_ADAPTIVE;
        p.seed = g.next();
        b.params.push_back(p);
        const uint32_t nh = 64 + static_cast<uint32_t>(g.next() % 1985);
        for (uint32_t i = 0; i < nh; ++i) b.hist.push_back(static_cast<int32_t>(g.next() % V));
        b.hoff.push_back(static_cast<int64_t>(b.hist.size()));
        b.u.push_back(g.uni());
    }
    return b;
}

template <class T>
T* upload(const std::vector<T>& v) {
    T* d = nullptr;
    cudaMalloc(&d, v.size() * sizeof(T) + 16);
    cudaMemcpy(d, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice);
    return d;
}

// The expected tokens and statuses, on device 0 from the C ABI alone.
bool expected(const Batch& b, uint32_t S, uint32_t top_n, std::vector<int32_t>& tok, std::vector<int32_t>& st) {
    cudaSetDevice(0);
    sixi_smp* h = nullptr;
    CHECK(sixi_smp_create(0, b.n, b.V, &h) == SIXI_OK);
    const ShardLayout lay{b.V, S};
    float* d_full = upload(b.logits);
    auto* d_p = upload(b.params);
    int32_t* d_h = upload(b.hist);
    int64_t* d_ho = upload(b.hoff);
    double* d_u = upload(b.u);
    void *gc = nullptr, *gs = nullptr;
    int32_t *d_tok = nullptr, *d_st = nullptr, *d_tf = nullptr, *d_sf = nullptr;
    cudaMalloc(&gc, static_cast<size_t>(S) * b.n * top_n * 8);
    cudaMalloc(&gs, static_cast<size_t>(S) * b.n * 24);
    for (int32_t** p : {&d_tok, &d_st, &d_tf, &d_sf}) cudaMalloc(p, b.n * 4);
    for (uint32_t r = 0; r < S; ++r) {
        const sixi_smp_rows slice{d_full + lay.offset(r), SIXI_SMP_F32, b.n, b.V};
        CHECK(sixi_smp_shard_candidates(h, &slice, lay.offset(r), lay.width(r), b.V, d_p, nullptr, d_h, d_ho, top_n,
                                        static_cast<char*>(gc) + static_cast<size_t>(r) * b.n * top_n * 8,
                                        static_cast<char*>(gs) + static_cast<size_t>(r) * b.n * 24,
                                        nullptr) == SIXI_OK);
    }
    CHECK(sixi_smp_merge_shards(h, b.n, S, top_n, gc, gs, d_p, d_u, 0, d_tok, d_st, nullptr) == SIXI_OK);
    const sixi_smp_rows full{d_full, SIXI_SMP_F32, b.n, b.V};
    CHECK(sixi_smp_sample(h, &full, d_p, nullptr, d_h, d_ho, d_u, 0, d_tf, d_sf, nullptr) == SIXI_OK);
    std::vector<int32_t> tm(b.n), sm(b.n), tf(b.n), sf(b.n);
    cudaMemcpy(tm.data(), d_tok, b.n * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(sm.data(), d_st, b.n * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(tf.data(), d_tf, b.n * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(sf.data(), d_sf, b.n * 4, cudaMemcpyDeviceToHost);
    CHECK(cudaDeviceSynchronize() == cudaSuccess);
    tok.resize(b.n);
    st.resize(b.n);
    uint32_t flagged = 0;
    for (uint32_t r = 0; r < b.n; ++r) {
        const bool oob = sm[r] == SIXI_OUT_OF_BOUNDS;
        flagged += oob ? 1u : 0u;
        tok[r] = oob ? tf[r] : tm[r];
        st[r] = oob ? sf[r] : sm[r];
    }
    std::printf("S=%u V=%u: %u of %u rows go to round 2\n", S, b.V, flagged, b.n);
    for (void* p : {static_cast<void*>(d_full), static_cast<void*>(d_p), static_cast<void*>(d_h),
                    static_cast<void*>(d_ho), static_cast<void*>(d_u), gc, gs, static_cast<void*>(d_tok),
                    static_cast<void*>(d_st), static_cast<void*>(d_tf), static_cast<void*>(d_sf)})
        cudaFree(p);
    sixi_smp_destroy(h);
    return true;
}

// One rank: its slice (a contiguous [n][width] copy, as a vocab-parallel output layer writes it)
// and the batch arrays on its own GPU, one ShardedSampler step.
bool run_rank(const Batch& b, uint32_t S, uint32_t rank, ncclComm_t comm, uint32_t top_n, std::vector<int32_t>& tok,
              std::vector<int32_t>& st) {
    CHECK(cudaSetDevice(static_cast<int>(rank)) == cudaSuccess);
    auto made = ShardedSampler::create(static_cast<int>(rank), b.n, b.V, comm, top_n);
    CHECK(made.ok());
    ShardedSampler& s = *made.value();
    const ShardLayout& lay = s.layout();
    CHECK(lay.n_shards == S && s.rank() == rank);
    const uint32_t w = lay.width(rank);
    std::vector<float> slice(static_cast<size_t>(b.n) * w);
    for (uint32_t r = 0; r < b.n; ++r)
        std::memcpy(&slice[static_cast<size_t>(r) * w], &b.logits[static_cast<size_t>(r) * b.V + lay.offset(rank)],
                    w * 4);
    float* d_slice = upload(slice);
    auto* d_p = upload(b.params);
    int32_t* d_h = upload(b.hist);
    int64_t* d_ho = upload(b.hoff);
    double* d_u = upload(b.u);
    int32_t *d_tok = nullptr, *d_st = nullptr;
    cudaMalloc(&d_tok, b.n * 4);
    cudaMalloc(&d_st, b.n * 4);
    cudaStream_t stream = nullptr;
    CHECK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) == cudaSuccess);
    ShardStepTimes t;
    const sixi_smp_rows rows{d_slice, SIXI_SMP_F32, b.n, w};
    for (int rep = 0; rep < 3; ++rep) {  // repeated steps reuse the round-2 buffers
        const Status ss = s.sample(rows, d_p, nullptr, d_h, d_ho, d_u, 0, d_tok, d_st, stream, &t);
        if (!ss.ok()) std::fprintf(stderr, "rank %u: %s\n", rank, ss.message.c_str());
        CHECK(ss.ok());
    }
    tok.resize(b.n);
    st.resize(b.n);
    cudaMemcpyAsync(tok.data(), d_tok, b.n * 4, cudaMemcpyDeviceToHost, stream);
    cudaMemcpyAsync(st.data(), d_st, b.n * 4, cudaMemcpyDeviceToHost, stream);
    CHECK(cudaStreamSynchronize(stream) == cudaSuccess);
    std::printf("  rank %u: stage1 %.3f ms, exchange %.3f ms, stage2 %.3f ms, round2 %.3f ms (%u rows)\n", rank,
                t.stage1_ms, t.exchange_ms, t.stage2_ms, t.round2_ms, t.round2_rows);
    cudaStreamDestroy(stream);
    for (void* p : {static_cast<void*>(d_slice), static_cast<void*>(d_p), static_cast<void*>(d_h),
                    static_cast<void*>(d_ho), static_cast<void*>(d_u), static_cast<void*>(d_tok),
                    static_cast<void*>(d_st)})
        cudaFree(p);
    return true;
}

bool sharded_case(uint32_t S, uint32_t V, uint32_t n, uint64_t seed) {
    const uint32_t top_n = 64;
    const Batch b = make_batch(n, V, seed);
    std::vector<int32_t> etok, est;
    CHECK(expected(b, S, top_n, etok, est));
    std::vector<ncclComm_t> comms(S);
    std::vector<int> devs(S);
    for (uint32_t r = 0; r < S; ++r) devs[r] = static_cast<int>(r);
    CHECK(ncclCommInitAll(comms.data(), static_cast<int>(S), devs.data()) == ncclSuccess);
    std::vector<std::vector<int32_t>> tok(S), st(S);
    std::vector<int> ok(S, 0);
    std::vector<std::thread> th;
    for (uint32_t r = 0; r < S; ++r)
        th.emplace_back([&, r]() { ok[r] = run_rank(b, S, r, comms[r], top_n, tok[r], st[r]) ? 1 : 0; });
    for (auto& t : th) t.join();
    for (uint32_t r = 0; r < S; ++r) ncclCommDestroy(comms[r]);
    for (uint32_t r = 0; r < S; ++r) {
        CHECK(ok[r] == 1);
        CHECK(st[r] == est);
        CHECK(tok[r] == etok);
    }
    return true;
}

}  // namespace

int main() {
    int n_dev = 0;
    if (cudaGetDeviceCount(&n_dev) != cudaSuccess || n_dev < 1) {
        std::fprintf(stderr, "no CUDA device\n");
        return 2;
    }
    int passed = 0, total = 0;
    ++total;
    passed += sharded_case(1, 50000, 48, 7) ? 1 : 0;
    if (n_dev >= 2) {
        ++total;
        passed += sharded_case(2, 151936, 64, 8) ? 1 : 0;
    }
    if (n_dev >= 4) {  // every GPU of the box, up to 8 slices
        ++total;
        passed += sharded_case(n_dev < 8 ? n_dev : 8, 151936, 64, 9) ? 1 : 0;
    }
    std::printf("%d/%d sharded cases passed (%d GPUs)\n", passed, total, n_dev);
    return passed == total && g_fail == 0 ? 0 : 1;
}
