// test_spec_step.cpp - the C++ host adapter's speculative verification (DeviceSampler::verify in
// sixi-asi_b200/host/sixi_sampler.hpp, on the GPU) against the engine's own
// SpeculativeDecoder::step (src/speculative/speculative.cpp:367-976), run on the CPU by the
// reference build (oracle/_ref/libsixiref.so: a replay IBackend and a fixed-draft INeuralDrafter).
// Both sides draw from the engine's DeterministicRng (core_execution.cpp:33-61) seeded alike.
//
//   slow path  dense draft probabilities, no rollback ring (speculative.cpp:739-976): the adapter's
//              verify(rows, q, drafts) must commit the step's tokens, accept as many drafts,
//              reject at the same position and leave the RNG in the same state
//   fast path  one-hot drafts after an anchor (speculative.cpp:471-737): the adapter draws the
//              anchor with sample_token, then verify(rows, nullptr, drafts) with the anchor in the
//              penalty history; the step's committed tokens are the anchor plus the accepted drafts,
//              followed by the token it carries to the next step
//   forced     a rejection forced at every draft position, sampled and greedy
// Rows follow config 4: target ~ N(0, 3^2) rounded to bf16, q = softmax(target + N(0, 1)), drafts
// drawn from q; per-stream parameters from the config-2 mix (temperature, top-p, repetition penalty,
// Adaptive mode) with top-k in {20, 40, 100}: every draw is then over at most 100 candidates with
// the engine's fp64 arithmetic, so the test requires exact equality. Rows with top_k = 0 (drawn on
// the full-vocabulary path, exact except within 1e-6 of a CDF boundary) are covered by the Python
// tests, which carry that allowance. Exit status 0 when every check passes. Needs a CUDA device.
#include <array>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>

#include "sixi_sampler.hpp"

extern "C" {
double orc_ref_rng_uniform(uint64_t* rng_io);
void orc_ref_rng_seed(uint64_t seed, uint64_t seq, uint64_t* rng_out);
int32_t orc_ref_spec_step(int32_t fast, const float* anchor_row, const float* rows, uint64_t vocab,
                          const float* draft_probs, const int32_t* drafts, uint32_t k, const sixi_smp_params* p,
                          const int32_t* hist, uint64_t n_hist, uint64_t* rng_io, int32_t* out_tokens,
                          int32_t* out_n, int32_t* out_accepted, int32_t* out_first_reject);
}

using namespace sixi_b200;

namespace {

int g_fail = 0;
int g_checks = 0;
#define CHECK(cond)                                                                        \
    do {                                                                                   \
        ++g_checks;                                                                        \
        if (!(cond)) {                                                                     \
            std::fprintf(stderr, "CHECK failed %s:%d: %s\n", __FILE__, __LINE__, #cond);   \
            ++g_fail;                                                                      \
            return false;                                                                  \
        }                                                                                  \
    } while (0)

// The engine's DeterministicRng, driven through the reference build (the adapter's Rng concept:
// next_uniform01, checkpoint, restore).
struct EngineRng {
    std::array<uint64_t, 2> st{};
    explicit EngineRng(uint64_t seed) { orc_ref_rng_seed(seed, 54, st.data()); }
    double next_uniform01() { return orc_ref_rng_uniform(st.data()); }
    std::array<uint64_t, 2> checkpoint() const { return st; }
    void restore(const std::array<uint64_t, 2>& s) { st = s; }
};

// Input generator (SplitMix64 + Box-Muller; test data only).
struct Gen {
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

float bf16_round(float x) {  // round to nearest even bf16, back to fp32
    uint32_t u;
    std::memcpy(&u, &x, 4);
    u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
    std::memcpy(&x, &u, 4);
    return x;
}

struct Stream {
    uint64_t V = 0;
    uint32_t k = 0;
    std::vector<float> rows;   // [k+1][V]
    std::vector<float> q;      // [k][V]
    std::vector<float> anchor; // [V] (fast path)
    std::vector<int32_t> drafts, hist;
    SamplingParams p;
};

Stream make_stream(uint64_t V, uint32_t k, uint64_t seed, bool greedy) {
    Gen g(seed);
    Stream s;
    s.V = V;
    s.k = k;
    s.rows.resize((k + 1) * V);
    for (auto& x : s.rows) x = bf16_round(g.normal(3.0f));
    s.anchor.resize(V);
    for (auto& x : s.anchor) x = g.normal(3.0f);
    s.q.resize(k * V);
    s.drafts.resize(k);
    for (uint32_t i = 0; i < k; ++i) {
        float* qi = &s.q[i * V];
        double mx = -1e300;
        for (uint64_t j = 0; j < V; ++j) {
            qi[j] = s.rows[i * V + j] + g.normal(1.0f);
            mx = std::max(mx, static_cast<double>(qi[j]));
        }
        double sum = 0.0;
        std::vector<double> e(V);
        for (uint64_t j = 0; j < V; ++j) sum += (e[j] = std::exp(static_cast<double>(qi[j]) - mx));
        const double u = g.uni() * sum;
        double c = 0.0;
        int32_t d = static_cast<int32_t>(V - 1);
        for (uint64_t j = 0; j < V; ++j) {
            qi[j] = static_cast<float>(e[j] / sum);
            c += e[j];
            if (d == static_cast<int32_t>(V - 1) && u < c) d = static_cast<int32_t>(j);
        }
        s.drafts[i] = d;
    }
    const uint32_t nh = 64 + static_cast<uint32_t>(g.next() % 448);
    for (uint32_t i = 0; i < nh; ++i) s.hist.push_back(static_cast<int32_t>(g.next() % V));
    const int32_t ks[3] = {20, 40, 100};
    s.p.temperature = greedy ? 0.0f : static_cast<float>(0.3 + 0.9 * g.uni());
    s.p.top_k = ks[g.next() % 3];
    s.p.top_p = static_cast<float>(0.7 + 0.3 * g.uni());
    s.p.repetition_penalty = static_cast<float>(1.0 + 0.3 * g.uni());
    s.p.mode = ExecutionMode::Adaptive;
    return s;
}

struct EngineOut {
    int32_t status = 0, n = 0, accepted = 0, first_reject = -1;
    std::vector<int32_t> tokens;
    std::array<uint64_t, 2> rng{};
};

EngineOut engine_step(const Stream& s, bool fast, const float* q, uint64_t seed) {
    EngineOut o;
    EngineRng r(seed);
    o.tokens.assign(s.k + 2, -1);
    const sixi_smp_params sp = to_smp_params(s.p);
    o.status = orc_ref_spec_step(fast ? 1 : 0, s.anchor.data(), s.rows.data(), s.V, q, s.drafts.data(), s.k, &sp,
                                 s.hist.data(), s.hist.size(), r.st.data(), o.tokens.data(), &o.n, &o.accepted,
                                 &o.first_reject);
    o.tokens.resize(static_cast<size_t>(o.n));
    o.rng = r.st;
    return o;
}

bool slow_path(DeviceSampler& dev, const Stream& s, uint64_t seed) {
    const EngineOut e = engine_step(s, false, s.q.data(), seed);
    CHECK(e.status == 0);
    EngineRng rng(seed);
    auto r = dev.verify(s.rows.data(), s.q.data(), s.drafts, s.p, rng, s.hist);
    CHECK(r.ok());
    const VerifyResult& v = r.value();
    CHECK(v.committed_tokens == e.tokens);
    CHECK(static_cast<int32_t>(v.accepted_draft_count) == e.accepted);
    CHECK(v.first_rejected_position == e.first_reject);
    CHECK(rng.st == e.rng);
    return true;
}

bool fast_path(DeviceSampler& dev, const Stream& s, uint64_t seed) {
    const EngineOut e = engine_step(s, true, nullptr, seed);
    CHECK(e.status == 0);
    EngineRng rng(seed);
    // the anchor: a sampled token, or for greedy the raw argmax without penalties
    // (speculative.cpp:480-490)
    int32_t anchor = -1;
    if (s.p.temperature <= 0.0f) {
        anchor = dev.sample_greedy_argmax(s.anchor.data(), s.V);
    } else {
        auto a = dev.sample_token(s.anchor.data(), s.V, s.p, rng, s.hist);
        CHECK(a.ok());
        anchor = a.value();
    }
    std::vector<int32_t> h2 = s.hist;
    h2.push_back(anchor);
    auto r = dev.verify(s.rows.data(), nullptr, s.drafts, s.p, rng, h2);
    CHECK(r.ok());
    std::vector<int32_t> mine{anchor};
    mine.insert(mine.end(), r.value().committed_tokens.begin(), r.value().committed_tokens.end());
    CHECK(mine == e.tokens);
    CHECK(static_cast<int32_t>(r.value().accepted_draft_count) == e.accepted);
    CHECK(r.value().first_rejected_position == e.first_reject);
    CHECK(rng.st == e.rng);
    return true;
}

// A rejection forced at position j: the drafts before j are the rows' best entries with a tiny q
// (accepted whatever the uniform; greedy: the raw argmax), draft j lies outside the kept
// candidates (p = 0: rejected; greedy: not the argmax).
bool forced(DeviceSampler& dev, Stream s, uint32_t j, uint64_t seed) {
    const bool greedy = s.p.temperature <= 0.0f;
    std::vector<int32_t> recent = s.hist;
    for (uint32_t i = 0; i <= j; ++i) {
        const float* row = &s.rows[i * s.V];
        int32_t best = 0;
        for (uint64_t x = 1; x < s.V; ++x)
            if (row[x] > row[best]) best = static_cast<int32_t>(x);
        if (greedy) {
            s.drafts[i] = i < j ? best : (best + 1) % static_cast<int32_t>(s.V);
            continue;
        }
        auto c = dev.compute_sampling_candidates(row, s.V, s.p, recent);
        CHECK(c.ok());
        if (i < j) {
            s.drafts[i] = c.value().front().id;
            s.q[i * s.V + static_cast<uint64_t>(s.drafts[i])] = 1e-9f;
            recent.push_back(s.drafts[i]);
        } else {
            std::vector<char> kept(s.V, 0);
            for (const auto& cc : c.value()) kept[static_cast<size_t>(cc.id)] = 1;
            int32_t out = 0;
            while (kept[static_cast<size_t>(out)]) ++out;
            s.drafts[i] = out;
        }
    }
    CHECK(slow_path(dev, s, seed));
    const EngineOut e = engine_step(s, false, s.q.data(), seed);
    CHECK(e.first_reject == static_cast<int32_t>(j));
    CHECK(e.accepted == static_cast<int32_t>(j));
    return true;
}

}  // namespace

int main() {
    const uint32_t k = 8;
    int cases = 0;
    for (uint64_t V : {4097ull, 151936ull}) {
        auto made = DeviceSampler::create(0, 64, static_cast<uint32_t>(V));
        if (!made.ok()) {
            std::fprintf(stderr, "create failed\n");
            return 2;
        }
        DeviceSampler& dev = *made.value();
        const int n = V < 10000 ? 12 : 4;
        for (int i = 0; i < n; ++i) {
            for (bool greedy : {false, true}) {
                const uint64_t seed = V * 31 + static_cast<uint64_t>(i) * 2 + (greedy ? 1 : 0);
                const Stream s = make_stream(V, k, seed, greedy);
                const int before = g_fail;
                slow_path(dev, s, seed + 7);
                fast_path(dev, s, seed + 9);
                if (g_fail != before)
                    std::fprintf(stderr, "  case V=%llu seed=%llu greedy=%d T=%.3f top_k=%d top_p=%.3f\n",
                                 static_cast<unsigned long long>(V), static_cast<unsigned long long>(seed),
                                 greedy ? 1 : 0, s.p.temperature, s.p.top_k, s.p.top_p);
                cases += 2;
            }
        }
        if (V < 10000) {
            for (uint32_t j = 0; j < k; ++j) {
                for (bool greedy : {false, true}) {
                    forced(dev, make_stream(V, k, 900 + j * 2 + (greedy ? 1 : 0), greedy), j, 4000 + j);
                    ++cases;
                }
            }
        }
    }
    std::printf("adapter vs SpeculativeDecoder::step: %d cases, %d checks, %d failed\n", cases, g_checks, g_fail);
    return g_fail == 0 ? 0 : 1;
}
