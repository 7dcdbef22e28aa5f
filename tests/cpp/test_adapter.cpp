// test_adapter.cpp - parity of the C++ host adapter (sixi-asi_b200/host/sixi_sampler.hpp) against
// the CPU oracle (oracle/sixi_oracle.h, port build), written like the engine's own C++ tests.
//
//   engine_topk_topp        restates test_sampler_candidates_topk_topp
//                           (tests/test_routing_and_numerics.cpp:485-545) through the adapter
//   random_rows             sample_token / compute_sampling_candidates / sample_greedy_argmax on
//                           seeded rows vs the oracle (V = 1, 33, 4097, 151,936)
//   rng_consumption         greedy draws nothing, sampled rows draw one uniform, failing rows
//                           leave the RNG untouched (core_execution.cpp:586-619)
//   errors                  the engine's error behaviour (null / empty / wrong vocab / NaN)
//   verify_random           SpeculativeDecoder verification (dense q and one-hot) vs orc_verify,
//                           and the RNG advanced by exactly the uniforms used
//   verify_forced_rejection greedy rejection positions (tests/test_determinism_and_speculative.cpp
//                           forced-rejection checks)
//   json_constrained        JsonMaskProducer + masked sample_rows: a greedy constrained decode
//                           writes the intended JSON object although a disallowed token scores
//                           higher, and every mask equals the CPU automaton's (sixi_json_oracle.h)
//   numeric_policy          inspect_and_apply_numeric_policy through the adapter vs the oracle
//                           (both policies, the engine's unit vectors of
//                           tests/test_routing_and_numerics.cpp:415-460, and a 151,936-wide row)
//   suffix_drafter          suffix_propose / suffix_propose_anchored vs orc_suffix_draft (match
//                           length, drafts, one-hot draft_probs)
//   device_rows             a fake backend that keeps its logits in device memory (fp32 rows with a
//                           padded stride, and bf16 rows): sample_token, sample_greedy_argmax and
//                           verify on its device rows equal the host-row calls on the same values,
//                           tokens and RNG state alike
// Exit status 0 when every check passes. Needs a CUDA device.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <numeric>
#include <string>
#include <vector>

#include "../../oracle/sixi_json_oracle.h"
#include "../../oracle/sixi_oracle.h"
#include "sixi_sampler.hpp"

using namespace sixi_b200;

namespace {

int g_fail = 0;
#define CHECK(cond)                                                                   \
    do {                                                                              \
        if (!(cond)) {                                                                \
            std::fprintf(stderr, "CHECK failed %s:%d: %s\n", __FILE__, __LINE__, #cond); \
            ++g_fail;                                                                 \
            return false;                                                             \
        }                                                                             \
    } while (0)

// Test RNG with the engine RNG's interface (next_uniform01, checkpoint, restore): SplitMix64.
struct TestRng {
    uint64_t s;
    explicit TestRng(uint64_t seed) : s(seed) {}
    uint64_t next_u64() {
        uint64_t z = (s += 0x9E3779B97F4A7C15ull);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    }
    double next_uniform01() { return static_cast<double>(next_u64() >> 11) * 0x1.0p-53; }
    uint64_t checkpoint() const { return s; }
    void restore(uint64_t st) { s = st; }
};

std::vector<float> normal_row(TestRng& r, size_t v, float sigma) {
    std::vector<float> x(v);
    for (size_t i = 0; i < v; ++i) {  // Box-Muller
        const double u1 = std::max(r.next_uniform01(), 1e-300), u2 = r.next_uniform01();
        x[i] = static_cast<float>(sigma * std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2));
    }
    return x;
}

// True when u is within 1e-6 of a cumulative boundary of the oracle's candidate list.
bool near_boundary(const std::vector<float>& x, const sixi_smp_params& p, const std::vector<int32_t>& h, double u) {
    std::vector<int32_t> ids(x.size());
    std::vector<double> pr(x.size());
    uint64_t n = 0;
    orc_candidates(x.data(), SIXI_SMP_F32, x.size(), &p, h.data(), h.size(), nullptr, x.size(), ids.data(),
                   pr.data(), &n);
    double c = 0.0;
    for (uint64_t i = 0; i < n; ++i) {
        c += pr[i];
        if (std::fabs(c - u) < 1e-6) return true;
    }
    return false;
}

bool engine_topk_topp() {
    const uint64_t V = 5000;
    auto made = DeviceSampler::create(0, 64, V);
    CHECK(made.ok());
    DeviceSampler& s = *made.value();
    std::vector<float> logits(V);
    for (uint64_t i = 0; i < V; ++i)
        logits[i] = std::sin(static_cast<float>(i) * 0.37f) * 3.0f + ((i % 97 == 0) ? 2.5f : 0.0f);
    SamplingParams p;
    p.temperature = 1.0f;
    p.top_k = 20;
    p.top_p = 1.0f;
    p.mode = ExecutionMode::StrictReplay;
    auto cr = s.compute_sampling_candidates(logits.data(), V, p);
    CHECK(cr.ok());
    const auto& cands = cr.value();
    CHECK(cands.size() == 20);
    std::vector<int32_t> ids(V);
    std::iota(ids.begin(), ids.end(), 0);
    std::sort(ids.begin(), ids.end(), [&](int32_t a, int32_t b) {
        if (logits[a] != logits[b]) return logits[a] > logits[b];
        return a < b;
    });
    double psum = 0.0;
    for (size_t i = 0; i < 20; ++i) {
        CHECK(cands[i].id == ids[i]);
        if (i > 0) CHECK(cands[i - 1].prob >= cands[i].prob);
        psum += cands[i].prob;
    }
    CHECK(std::fabs(psum - 1.0) < 1e-9);
    CHECK(cands.front().id == s.sample_greedy_argmax(logits.data(), V));
    p.top_p = 0.5f;
    auto tp = s.compute_sampling_candidates(logits.data(), V, p);
    CHECK(tp.ok() && !tp.value().empty() && tp.value().size() < 20);
    CHECK(tp.value().front().id == ids[0]);
    double tsum = 0.0;
    for (const auto& c : tp.value()) tsum += c.prob;
    CHECK(std::fabs(tsum - 1.0) < 1e-9);
    TestRng r1(99), r2(99);
    auto t1 = s.sample_token(logits.data(), V, p, r1);
    auto t2 = s.sample_token(logits.data(), V, p, r2);
    CHECK(t1.ok() && t2.ok() && t1.value() == t2.value());
    bool in_set = false;
    for (const auto& c : tp.value()) in_set = in_set || c.id == t1.value();
    CHECK(in_set);
    p.temperature = 0.0f;
    TestRng r3(5);
    const uint64_t before = r3.checkpoint();
    auto g = s.sample_token(logits.data(), V, p, r3);
    CHECK(g.ok() && g.value() == ids[0]);
    CHECK(r3.checkpoint() == before);
    return true;
}

bool random_rows() {
    const uint64_t vocabs[] = {1, 33, 4097, 151936};
    TestRng gen(20261201);
    for (uint64_t V : vocabs) {
        auto made = DeviceSampler::create(0, 16, V);
        CHECK(made.ok());
        DeviceSampler& s = *made.value();
        for (int it = 0; it < 12; ++it) {
            auto x = normal_row(gen, V, it % 3 == 0 ? 6.0f : 2.5f);
            SamplingParams p;
            const float temps[] = {0.0f, 0.3f, 0.7f, 1.0f, 1.5f};
            const int32_t tks[] = {0, 1, 5, 20, 40, 100, 256};
            p.temperature = temps[it % 5];
            p.top_k = tks[(it * 3) % 7];
            p.top_p = it % 4 == 0 ? 1.0f : 0.6f + 0.1f * static_cast<float>(it % 4);
            p.repetition_penalty = it % 2 ? 1.2f : 1.0f;
            p.presence_penalty = it % 3 == 1 ? 0.5f : 0.0f;
            p.mode = it % 2 ? ExecutionMode::Adaptive : ExecutionMode::StrictReplay;
            std::vector<int32_t> hist(static_cast<size_t>(gen.next_u64() % 300));
            for (auto& h : hist) h = static_cast<int32_t>(gen.next_u64() % V);
            const sixi_smp_params sp = to_smp_params(p);
            // greedy argmax of the raw row
            CHECK(s.sample_greedy_argmax(x.data(), V) == orc_greedy_argmax(x.data(), V));
            // sampled token with the RNG's next uniform
            TestRng r(1000 + it), peek(1000 + it);
            const double u = p.temperature > 0.0f ? peek.next_uniform01() : 0.0;
            auto t = s.sample_token(x.data(), V, p, r, hist);
            CHECK(t.ok());
            int32_t ot = -1;
            CHECK(orc_sample(x.data(), SIXI_SMP_F32, V, &sp, hist.data(), hist.size(), nullptr, u, &ot) == 0);
            if (t.value() != ot && !near_boundary(x, sp, hist, u)) {
                std::fprintf(stderr, "V=%llu it=%d token %d vs oracle %d\n", (unsigned long long)V, it, t.value(), ot);
                CHECK(false);
            }
            // candidate list (only lists of at most 256 entries come back through the adapter)
            std::vector<int32_t> oid(V);
            std::vector<double> opr(V);
            uint64_t on = 0;
            orc_candidates(x.data(), SIXI_SMP_F32, V, &sp, hist.data(), hist.size(), nullptr, V, oid.data(),
                           opr.data(), &on);
            auto c = s.compute_sampling_candidates(x.data(), V, p, hist);
            if (on <= 256) {
                CHECK(c.ok() && c.value().size() == on);
                for (uint64_t i = 0; i < on; ++i) {
                    CHECK(c.value()[i].id == oid[i]);
                    CHECK(std::fabs(c.value()[i].prob - opr[i]) <= 1e-5 * opr[i] + 1e-300);
                }
            } else {
                CHECK(!c.ok() && c.code() == ErrorCode::OutOfBounds);
            }
        }
    }
    return true;
}

bool rng_consumption() {
    const uint64_t V = 4097;
    auto made = DeviceSampler::create(0, 4, V);
    CHECK(made.ok());
    DeviceSampler& s = *made.value();
    TestRng gen(7);
    auto x = normal_row(gen, V, 2.5f);
    SamplingParams p;
    p.temperature = 0.0f;
    TestRng r(11);
    uint64_t st0 = r.checkpoint();
    CHECK(s.sample_token(x.data(), V, p, r).ok());
    CHECK(r.checkpoint() == st0);  // greedy: no uniform
    p.temperature = 0.8f;
    CHECK(s.sample_token(x.data(), V, p, r).ok());
    TestRng one(11);
    one.next_uniform01();
    CHECK(r.checkpoint() == one.checkpoint());  // sampled: exactly one uniform
    x[17] = std::nanf("");
    st0 = r.checkpoint();
    auto bad = s.sample_token(x.data(), V, p, r);
    CHECK(!bad.ok() && bad.code() == ErrorCode::NumericNaNOrInf);
    CHECK(r.checkpoint() == st0);  // a failing row draws nothing
    return true;
}

bool errors() {
    const uint64_t V = 100;
    auto made = DeviceSampler::create(0, 4, V);
    CHECK(made.ok());
    DeviceSampler& s = *made.value();
    std::vector<float> x(V, 0.0f);
    CHECK(s.sample_greedy_argmax(nullptr, V) == -1);
    CHECK(s.sample_greedy_argmax(x.data(), 0) == -1);
    SamplingParams p;
    TestRng r(1);
    auto e1 = s.sample_token(nullptr, V, p, r);
    CHECK(!e1.ok() && e1.code() == ErrorCode::InvalidArgument);
    auto e2 = s.sample_token(x.data(), V + 1, p, r);
    CHECK(!e2.ok() && e2.code() == ErrorCode::InvalidArgument);
    // all-equal logits: lowest id wins (engine tie rule)
    CHECK(s.sample_greedy_argmax(x.data(), V) == 0);
    auto bad_create = DeviceSampler::create(0, 4, 0);
    CHECK(!bad_create.ok() && bad_create.code() == ErrorCode::InvalidArgument);
    return true;
}

bool verify_random() {
    const uint64_t vocabs[] = {700, 151936};
    TestRng gen(4242);
    for (uint64_t V : vocabs) {
        auto made = DeviceSampler::create(0, 32, V);
        CHECK(made.ok());
        DeviceSampler& s = *made.value();
        for (int it = 0; it < 8; ++it) {
            const uint32_t k = 1 + static_cast<uint32_t>(it % 6);
            std::vector<float> tgt((k + 1) * V), q(k * V);
            for (uint32_t i = 0; i <= k; ++i) {
                auto row = normal_row(gen, V, 3.0f);
                std::copy(row.begin(), row.end(), tgt.begin() + i * V);
            }
            std::vector<int32_t> drafts(k);
            for (uint32_t i = 0; i < k; ++i) {  // q = softmax(target + noise), draft = argmax of q
                double m = -1e300, z = 0.0;
                std::vector<double> t(V);
                for (uint64_t j = 0; j < V; ++j) {
                    t[j] = tgt[i * V + j] + 0.8 * (gen.next_uniform01() - 0.5);
                    m = std::max(m, t[j]);
                }
                for (uint64_t j = 0; j < V; ++j) z += std::exp(t[j] - m);
                int32_t best = 0;
                for (uint64_t j = 0; j < V; ++j) {
                    q[i * V + j] = static_cast<float>(std::exp(t[j] - m) / z);
                    if (q[i * V + j] > q[i * V + best]) best = static_cast<int32_t>(j);
                }
                drafts[i] = (it % 3 == 2) ? static_cast<int32_t>(gen.next_u64() % V) : best;
            }
            SamplingParams p;
            p.temperature = it % 4 == 3 ? 0.0f : 0.9f;
            p.top_k = it % 2 ? 0 : 40;
            p.top_p = 0.9f;
            p.repetition_penalty = 1.1f;
            p.mode = ExecutionMode::Adaptive;
            std::vector<int32_t> ctx(50);
            for (auto& c : ctx) c = static_cast<int32_t>(gen.next_u64() % V);
            for (int dense = 0; dense < 2; ++dense) {
                TestRng r(77 + it), peek(77 + it);
                std::vector<double> u(k + 1);
                for (auto& v : u) v = peek.next_uniform01();
                auto res = s.verify(tgt.data(), dense ? q.data() : nullptr, drafts, p, r, ctx);
                CHECK(res.ok());
                const sixi_smp_params sp = to_smp_params(p);
                const int64_t hoff[2] = {0, static_cast<int64_t>(ctx.size())};
                int32_t acc = 0, ntok = 0, frej = 0, used = 0, st = 0;
                std::vector<int32_t> toks(k + 1);
                orc_verify(tgt.data(), SIXI_SMP_F32, V, V, dense ? q.data() : nullptr, drafts.data(), nullptr, 1, k,
                           &sp, nullptr, ctx.data(), hoff, u.data(), 0, &acc, toks.data(), &ntok, &frej, &used, &st, 1);
                CHECK(st == 0);
                CHECK(res.value().accepted_draft_count == static_cast<uint32_t>(acc));
                CHECK(res.value().first_rejected_position == frej);
                CHECK(res.value().uniforms_used == static_cast<uint32_t>(used));
                CHECK(res.value().committed_tokens.size() == static_cast<size_t>(ntok));
                for (int32_t i = 0; i < ntok; ++i) CHECK(res.value().committed_tokens[i] == toks[i]);
                TestRng adv(77 + it);
                for (int32_t i = 0; i < used; ++i) adv.next_uniform01();
                CHECK(r.checkpoint() == adv.checkpoint());
            }
        }
    }
    return true;
}

bool verify_forced_rejection() {
    const uint64_t V = 4096;
    const uint32_t k = 4;
    auto made = DeviceSampler::create(0, 16, V);
    CHECK(made.ok());
    DeviceSampler& s = *made.value();
    TestRng gen(3);
    std::vector<float> tgt((k + 1) * V);
    std::vector<int32_t> am(k + 1);
    for (uint32_t i = 0; i <= k; ++i) {
        auto row = normal_row(gen, V, 1.0f);
        std::copy(row.begin(), row.end(), tgt.begin() + i * V);
        am[i] = orc_greedy_argmax(row.data(), V);
    }
    SamplingParams p;
    p.temperature = 0.0f;
    for (uint32_t pos = 0; pos <= k; ++pos) {
        std::vector<int32_t> drafts(am.begin(), am.begin() + k);
        if (pos < k) drafts[pos] = (am[pos] + 17) % static_cast<int32_t>(V);
        TestRng r(1);
        auto res = s.verify(tgt.data(), nullptr, drafts, p, r, {});
        CHECK(res.ok());
        CHECK(res.value().accepted_draft_count == pos);
        CHECK(res.value().first_rejected_position == (pos < k ? static_cast<int32_t>(pos) : -1));
        CHECK(res.value().committed_tokens.size() == pos + 1);
        for (uint32_t i = 0; i <= pos; ++i) CHECK(res.value().committed_tokens[i] == am[i]);
        CHECK(res.value().uniforms_used == 0 && r.checkpoint() == 1);
    }
    return true;
}

bool json_constrained() {
    // vocabulary: every byte, a few multi-byte pieces, one control token and end-of-sequence
    std::vector<std::string> texts;
    for (int b = 0; b < 256; ++b) texts.push_back(std::string(1, static_cast<char>(b)));
    for (const char* t : {"{\"", "\":", "\": ", " [", "true", "false", "], ", "}}", ", \"", "12", "ab"})
        texts.push_back(t);
    const int32_t ctl = static_cast<int32_t>(texts.size());
    texts.push_back("<|ctl|>");
    const int32_t eos = static_cast<int32_t>(texts.size());
    texts.push_back("<|endoftext|>");
    std::vector<uint8_t> special(texts.size(), 0);
    special[ctl] = 1;
    const uint32_t V = static_cast<uint32_t>(texts.size());
    auto jp = JsonMaskProducer::create(0, texts, special, eos);
    CHECK(jp.ok());
    auto made = DeviceSampler::create(0, 4, V);
    CHECK(made.ok());
    JsonMaskProducer& g = *jp.value();
    DeviceSampler& s = *made.value();
    // the intended answer, greedily tokenised by longest match
    const std::string doc = "{\"ab\": [12, true, {\"x\": false}], \"c\": {\"d\": {}}}";
    std::vector<int32_t> want;
    for (size_t i = 0; i < doc.size();) {
        int32_t best = -1;
        size_t bl = 0;
        for (int32_t t = 0; t < ctl; ++t)
            if (texts[t].size() > bl && doc.compare(i, texts[t].size(), texts[t]) == 0) best = t, bl = texts[t].size();
        want.push_back(best);
        i += bl;
    }
    want.push_back(eos);
    const uint32_t W = g.mask_words();
    sixi_json_state* d_st = nullptr;
    uint32_t* d_mask = nullptr;
    float* d_logits = nullptr;
    sixi_smp_params* d_p = nullptr;
    int32_t *d_tok = nullptr, *d_sts = nullptr, *d_gst = nullptr;
    cudaMalloc(&d_st, sizeof(sixi_json_state));
    cudaMalloc(&d_mask, 4 * W);
    cudaMalloc(&d_logits, 4 * V);
    cudaMalloc(&d_p, sizeof(sixi_smp_params));
    cudaMalloc(&d_tok, 4);
    cudaMalloc(&d_sts, 4);
    cudaMalloc(&d_gst, 4);
    SamplingParams sp;
    sp.temperature = 0.0f;
    const sixi_smp_params p = to_smp_params(sp, true);
    cudaStream_t st = s.stream();
    cudaMemcpyAsync(d_p, &p, sizeof p, cudaMemcpyHostToDevice, st);
    CHECK(g.reset(d_st, 1, st).ok());
    std::vector<uint8_t> flat;
    std::vector<uint64_t> off(V + 1, 0);
    for (uint32_t i = 0; i < V; ++i) {
        off[i + 1] = off[i] + texts[i].size();
        flat.insert(flat.end(), texts[i].begin(), texts[i].end());
    }
    TestRng gen(11);
    std::vector<int32_t> got;
    for (size_t step = 0; step < want.size(); ++step) {
        std::vector<float> x = normal_row(gen, V, 1.0f);
        x[want[step]] += 20.0f;
        x[eos] += 30.0f;  // end-of-sequence scores highest but is allowed only after the object
        x[ctl] += 40.0f;  // a control token is never allowed
        cudaMemcpyAsync(d_logits, x.data(), 4 * V, cudaMemcpyHostToDevice, st);
        CHECK(g.fill_masks(d_st, 1, d_mask, st).ok());
        sixi_smp_rows rows{d_logits, SIXI_SMP_F32, 1, V};
        CHECK(s.sample_rows(rows, d_p, d_mask, nullptr, nullptr, nullptr, step, d_tok, d_sts, st).ok());
        // the device mask of this state equals the CPU automaton's
        sixi_json_state hs;
        std::vector<uint32_t> m(W), om(W);
        cudaMemcpyAsync(&hs, d_st, sizeof hs, cudaMemcpyDeviceToHost, st);
        cudaMemcpyAsync(m.data(), d_mask, 4 * W, cudaMemcpyDeviceToHost, st);
        CHECK(g.advance(d_st, 1, d_tok, d_gst, st).ok());
        int32_t tok = -1, sts = -1, gst = -1;
        cudaMemcpyAsync(&tok, d_tok, 4, cudaMemcpyDeviceToHost, st);
        cudaMemcpyAsync(&sts, d_sts, 4, cudaMemcpyDeviceToHost, st);
        cudaMemcpyAsync(&gst, d_gst, 4, cudaMemcpyDeviceToHost, st);
        CHECK(cudaStreamSynchronize(st) == cudaSuccess);
        orc_json_fill_masks(flat.data(), off.data(), special.data(), V, eos, &hs, 1, om.data(), W, 1);
        CHECK(m == om);
        CHECK(sts == SIXI_OK && gst == SIXI_OK);
        got.push_back(tok);
    }
    CHECK(got == want);
    sixi_json_state fin;
    cudaMemcpy(&fin, d_st, sizeof fin, cudaMemcpyDeviceToHost);
    CHECK(fin.mode == SIXI_JSON_DONE && fin.failed == 0);
    cudaFree(d_st);
    cudaFree(d_mask);
    cudaFree(d_logits);
    cudaFree(d_p);
    cudaFree(d_tok);
    cudaFree(d_sts);
    cudaFree(d_gst);
    return true;
}

}  // namespace

// the engine's NumericPolicy / NumericHealthReport shapes (include/sixi_asi/numeric.hpp:127-139)
enum class EnginePolicy : uint8_t { FailAndInvalidate = 0, EmergencyClampAndReport = 1 };
struct EngineReport {
    bool healthy = true, request_corrupted = false, state_invalidated = false, emergency_clamped = false;
    uint64_t nan_count = 0, inf_count = 0;
    int64_t first_bad_index = -1;
};

bool numeric_policy() {
    const float nan = std::nanf(""), inf = INFINITY;
    {  // the engine's unit vectors
        auto made = DeviceSampler::create(0, 1, 5);
        CHECK(made.ok());
        DeviceSampler& s = *made.value();
        std::vector<float> d = {1.0f, 2.5f, nan, -3.0f, inf};
        EngineReport r;
        Status st = s.inspect_and_apply_numeric_policy(d.data(), 5, EnginePolicy::FailAndInvalidate, 100.0f, &r);
        CHECK(!st.ok() && st.code == ErrorCode::NumericNaNOrInf);
        CHECK(!r.healthy && r.request_corrupted && r.state_invalidated && !r.emergency_clamped);
        CHECK(r.nan_count == 1 && r.inf_count == 1 && r.first_bad_index == 2 && std::isnan(d[2]));
        std::vector<float> c = {1.0f, nan, inf, -inf, 500.0f};
        st = s.inspect_and_apply_numeric_policy(c.data(), 5, EnginePolicy::EmergencyClampAndReport, 100.0f, &r);
        CHECK(st.ok() && r.emergency_clamped && r.nan_count == 1 && r.inf_count == 2);
        CHECK(c == std::vector<float>({1.0f, 0.0f, 100.0f, -100.0f, 100.0f}));
    }
    const uint32_t V = 151936;
    auto made = DeviceSampler::create(0, 1, V);
    CHECK(made.ok());
    DeviceSampler& s = *made.value();
    TestRng rng(41);
    for (int it = 0; it < 6; ++it) {
        std::vector<float> x = normal_row(rng, V, 40.0f);
        for (int k = 0; k < it * 3; ++k) x[rng.next_u64() % V] = (k % 3 == 0) ? nan : ((k % 3 == 1) ? inf : -inf);
        for (int pol = 0; pol < 2; ++pol) {
            std::vector<float> a = x, b = x;
            EngineReport r;
            const Status st = s.inspect_and_apply_numeric_policy(a.data(), V, static_cast<EnginePolicy>(pol), 50.0f, &r);
            sixi_smp_numeric_report o{};
            const int32_t ost = orc_numeric_policy(b.data(), V, static_cast<uint32_t>(pol), 50.0f, &o);
            CHECK(static_cast<int32_t>(st.code) == ost);
            CHECK(r.healthy == (o.healthy != 0) && r.request_corrupted == (o.request_corrupted != 0));
            CHECK(r.state_invalidated == (o.state_invalidated != 0) && r.emergency_clamped == (o.emergency_clamped != 0));
            CHECK(r.nan_count == o.nan_count && r.inf_count == o.inf_count && r.first_bad_index == o.first_bad_index);
            CHECK(std::memcmp(a.data(), b.data(), V * sizeof(float)) == 0);
        }
    }
    EngineReport r;
    CHECK(s.inspect_and_apply_numeric_policy(static_cast<float*>(nullptr), 0, EnginePolicy::FailAndInvalidate, 0.0f, &r).ok());
    CHECK(!s.inspect_and_apply_numeric_policy(static_cast<float*>(nullptr), 5, EnginePolicy::FailAndInvalidate, 0.0f, &r).ok());
    return true;
}

bool suffix_drafter() {
    auto made = DeviceSampler::create(0, 1, 64);
    CHECK(made.ok());
    DeviceSampler& s = *made.value();
    TestRng rng(17);
    int found = 0;
    for (int it = 0; it < 40; ++it) {
        const size_t n = static_cast<size_t>(rng.next_u64() % 3000);
        const uint64_t vocab = (it % 3 == 0) ? 4 : 64;
        std::vector<int32_t> h(n);
        for (auto& t : h) t = static_cast<int32_t>(rng.next_u64() % vocab);
        if (n > 100 && it % 2 == 0) {  // a repeated tail
            for (size_t i = 0; i < 10; ++i) h[n / 3 + i] = h[n - 10 + i];
        }
        const uint32_t k = 1 + static_cast<uint32_t>(rng.next_u64() % 9);
        for (int anchored = 0; anchored < 2; ++anchored) {
            const int32_t anchor = n ? h[rng.next_u64() % n] : 1;
            auto p = anchored ? s.suffix_propose_anchored(h, anchor, k) : s.suffix_propose(h, k, 64);
            std::vector<int32_t> od(k);
            const int32_t om = orc_suffix_draft(h.data(), n, 3, 16384, anchored, anchor, k, od.data());
            CHECK(p.has_value() == (om > 0));
            if (!p.has_value()) continue;
            ++found;
            CHECK(static_cast<int32_t>(p->match_len) == om && p->draft_tokens == od);
            if (!anchored) {
                CHECK(p->draft_probs.size() == k);
                for (uint32_t i = 0; i < k; ++i) CHECK(p->draft_probs[i][static_cast<size_t>(od[i])] == 1.0f);
            }
        }
    }
    CHECK(found > 10);
    return true;
}

// A backend whose output logits stay in device memory (the device-resident hand-off): a
// [positions][stride] buffer, fp32 or bf16, with a view of any run of rows.
struct FakeDeviceBackend {
    void* d = nullptr;
    uint32_t dtype = SIXI_SMP_F32;
    uint64_t V = 0, stride = 0;
    uint32_t n = 0;
    FakeDeviceBackend(const std::vector<float>& rows, uint64_t vocab, uint64_t row_stride, uint32_t n_rows, bool bf16)
        : dtype(bf16 ? SIXI_SMP_BF16 : SIXI_SMP_F32), V(vocab), stride(row_stride), n(n_rows) {
        if (bf16) {
            std::vector<uint16_t> h(static_cast<size_t>(n_rows) * row_stride, 0);
            for (uint32_t r = 0; r < n_rows; ++r)
                for (uint64_t i = 0; i < vocab; ++i) {
                    uint32_t u;
                    std::memcpy(&u, &rows[r * vocab + i], 4);
                    h[r * row_stride + i] = static_cast<uint16_t>(u >> 16);  // rows are bf16 values already
                }
            cudaMalloc(&d, h.size() * 2);
            cudaMemcpy(d, h.data(), h.size() * 2, cudaMemcpyHostToDevice);
        } else {
            std::vector<float> h(static_cast<size_t>(n_rows) * row_stride, 0.0f);
            for (uint32_t r = 0; r < n_rows; ++r)
                std::copy(rows.begin() + r * vocab, rows.begin() + (r + 1) * vocab, h.begin() + r * row_stride);
            cudaMalloc(&d, h.size() * 4);
            cudaMemcpy(d, h.data(), h.size() * 4, cudaMemcpyHostToDevice);
        }
    }
    ~FakeDeviceBackend() { cudaFree(d); }
    sixi_smp_rows rows(uint32_t first, uint32_t count) const {
        const size_t esz = dtype == SIXI_SMP_BF16 ? 2 : 4;
        return sixi_smp_rows{static_cast<char*>(d) + first * stride * esz, dtype, count, stride};
    }
};

float to_bf16_value(float x) {  // truncating conversion: the value a bf16 buffer holds exactly
    uint32_t u;
    std::memcpy(&u, &x, 4);
    u &= 0xFFFF0000u;
    std::memcpy(&x, &u, 4);
    return x;
}

bool device_rows() {
    const uint64_t V = 151936;
    const uint32_t k = 6;
    TestRng gen(99);
    auto made = DeviceSampler::create(0, 32, V);
    CHECK(made.ok());
    DeviceSampler& s = *made.value();
    for (int it = 0; it < 6; ++it) {
        const bool bf16 = it % 2 == 1;
        std::vector<float> rows((k + 1) * V);
        for (uint32_t r = 0; r <= k; ++r) {
            auto x = normal_row(gen, V, 3.0f);
            for (uint64_t i = 0; i < V; ++i) rows[r * V + i] = bf16 ? to_bf16_value(x[i]) : x[i];
        }
        std::vector<float> q(k * V);
        std::vector<int32_t> drafts(k);
        for (uint32_t i = 0; i < k; ++i) {
            double z = 0.0, m = -1e300;
            for (uint64_t j = 0; j < V; ++j) m = std::max(m, static_cast<double>(rows[i * V + j]));
            for (uint64_t j = 0; j < V; ++j) z += std::exp(rows[i * V + j] - m);
            int32_t best = 0;
            for (uint64_t j = 0; j < V; ++j) {
                q[i * V + j] = static_cast<float>(std::exp(rows[i * V + j] - m) / z);
                if (rows[i * V + j] > rows[i * V + best]) best = static_cast<int32_t>(j);
            }
            drafts[i] = (i + static_cast<uint32_t>(it)) % 3 == 0 ? static_cast<int32_t>(gen.next_u64() % V) : best;
        }
        const FakeDeviceBackend be(rows, V, V + 64 * (it % 3), k + 1, bf16);
        // q rows on the device are the target rows' stride apart, as the verifier reads them
        float* dq = nullptr;
        CHECK(cudaMalloc(&dq, k * be.stride * 4) == cudaSuccess);
        CHECK(cudaMemcpy2D(dq, be.stride * 4, q.data(), V * 4, V * 4, k, cudaMemcpyHostToDevice) == cudaSuccess);
        SamplingParams p;
        p.temperature = it == 4 ? 0.0f : 0.8f;
        p.top_k = it % 3 == 0 ? 0 : 40;
        p.top_p = 0.9f;
        p.repetition_penalty = 1.15f;
        p.mode = ExecutionMode::Adaptive;
        std::vector<int32_t> ctx(300);
        for (auto& c : ctx) c = static_cast<int32_t>(gen.next_u64() % V);
        // sample_token and the raw argmax, row by row
        for (uint32_t r = 0; r <= k; ++r) {
            TestRng a(1000 + r), b(1000 + r);
            auto th = s.sample_token(&rows[r * V], V, p, a, ctx);
            auto td = s.sample_token(be.rows(r, 1), p, b, ctx);
            CHECK(th.ok() && td.ok());
            CHECK(th.value() == td.value());
            CHECK(a.checkpoint() == b.checkpoint());
            CHECK(s.sample_greedy_argmax(&rows[r * V], V) == s.sample_greedy_argmax(be.rows(r, 1)));
        }
        // verify: dense q and one-hot
        for (int dense = 0; dense < 2; ++dense) {
            TestRng a(55 + it), b(55 + it);
            auto vh = s.verify(rows.data(), dense ? q.data() : nullptr, drafts, p, a, ctx);
            auto vd = s.verify(be.rows(0, k + 1), dense ? dq : nullptr, drafts, p, b, ctx);
            CHECK(vh.ok() && vd.ok());
            CHECK(vh.value().committed_tokens == vd.value().committed_tokens);
            CHECK(vh.value().accepted_draft_count == vd.value().accepted_draft_count);
            CHECK(vh.value().first_rejected_position == vd.value().first_rejected_position);
            CHECK(a.checkpoint() == b.checkpoint());
        }
        cudaFree(dq);
    }
    // wrong shapes are refused without touching the RNG
    TestRng r(5);
    const uint64_t before = r.checkpoint();
    SamplingParams p;
    p.temperature = 0.7f;
    CHECK(!s.sample_token(sixi_smp_rows{nullptr, SIXI_SMP_F32, 1, V}, p, r).ok());
    CHECK(!s.verify(sixi_smp_rows{reinterpret_cast<void*>(16), SIXI_SMP_F32, 3, V}, nullptr,
                    std::vector<int32_t>{1, 2, 3}, p, r, {}).ok());
    CHECK(r.checkpoint() == before);
    return true;
}

int main() {
    struct {
        const char* name;
        bool (*fn)();
    } tests[] = {{"engine_topk_topp", engine_topk_topp},
                 {"random_rows", random_rows},
                 {"rng_consumption", rng_consumption},
                 {"errors", errors},
                 {"verify_random", verify_random},
                 {"verify_forced_rejection", verify_forced_rejection},
                 {"json_constrained", json_constrained},
                 {"numeric_policy", numeric_policy},
                 {"suffix_drafter", suffix_drafter},
                 {"device_rows", device_rows}};
    int passed = 0, n = 0;
    for (auto& t : tests) {
        ++n;
        const bool ok = t.fn();
        std::printf("%s %s\n", ok ? "PASS" : "FAIL", t.name);
        passed += ok ? 1 : 0;
    }
    std::printf("%d/%d passed\n", passed, n);
    return passed == n && g_fail == 0 ? 0 : 1;
}
