// ref_shim.cpp - TEST INFRASTRUCTURE ONLY (parity checker and the timed CPU reference arm).
//
// Wraps the Sixi-ASI engine's own sampler, compiled from its sources by oracle/Makefile into
// oracle/_ref/libsixiref.so, behind the oracle signatures of oracle/sixi_oracle.h:
//   - DeterministicSampler::sample_greedy_argmax / compute_sampling_candidates are called as-is
//     (src/core/core_execution.cpp:394-407, 449-584);
//   - the grammar mask is applied by compaction (allowed ids in ascending order, history ids
//     remapped, results mapped back), which the engine's API can express;
//   - the draw with a supplied uniform restates sample_from_candidates' CDF walk
//     (src/core/core_execution.cpp:586-601), since the engine draws from its own PCG32 stream;
//   - verification restates SpeculativeDecoder::step's accept/residual/bonus logic
//     (src/speculative/speculative.cpp:630-692 one-hot, :801-916 dense q) around the engine's
//     compute_sampling_candidates, taking the uniforms from the supplied slots;
//   - orc_ref_spec_step runs the engine's real SpeculativeDecoder::step with its own
//     DeterministicRng, through a replay IBackend (pre-supplied target rows) and a fixed-draft
//     INeuralDrafter: the slow path (no rollback ring, dense draft probs, :739-976) or the fast
//     path (O(1) rollback, one-hot drafts after a sampled anchor, :471-737). It pins the restated
//     verifier and the C++ adapter's RNG contract, and times config 4 on the host cores.
// Inputs the engine cannot express (min_p, frequency penalty) return ORC_UNSUPPORTED.
#include "sixi_asi/core_execution.hpp"
#include "sixi_asi/numeric.hpp"
#include "sixi_asi/speculative.hpp"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

extern "C" {
#include "sixi_oracle.h"
}

using sixi_asi::ErrorCode;
using sixi_asi::ExecutionMode;
using sixi_asi::core::DeterministicSampler;
using sixi_asi::core::SamplingParams;
using Cand = DeterministicSampler::Candidate;
using sixi_asi::Result;
using sixi_asi::Status;
using sixi_asi::core::BackendSequenceState;
using sixi_asi::core::DeterministicRng;
using sixi_asi::core::IBackend;
using sixi_asi::core::RngState;
namespace spec = sixi_asi::speculative;

#define EXPORT extern "C" __attribute__((visibility("default")))

namespace {

bool allowed(const uint32_t* mask, uint64_t i) {
    return mask == nullptr || ((mask[i >> 5] >> (i & 31u)) & 1u);
}

void load_row(const void* row, uint32_t dtype, uint64_t vocab, std::vector<float>& out) {
    out.resize(vocab);
    if (dtype == SIXI_SMP_BF16) {
        const uint16_t* r = static_cast<const uint16_t*>(row);
        for (uint64_t i = 0; i < vocab; ++i) out[i] = sixi_asi::bf16_to_fp32(r[i]);
    } else {
        std::memcpy(out.data(), row, vocab * sizeof(float));
    }
}

SamplingParams to_engine(const sixi_smp_params* p) {
    SamplingParams s;
    s.temperature = p->temperature;
    s.top_k = p->top_k;
    s.top_p = p->top_p;
    s.repetition_penalty = p->repetition_penalty;
    s.presence_penalty = p->presence_penalty;
    s.seed = p->seed;
    s.mode = p->mode == SIXI_SMP_ADAPTIVE ? ExecutionMode::Adaptive : ExecutionMode::StrictReplay;
    return s;
}

bool expressible(const sixi_smp_params* p) {
    return p->min_p == 0.0f && p->frequency_penalty == 0.0f;
}

// Engine candidates for one fp32 row with the mask applied by compaction.
int32_t engine_candidates(const std::vector<float>& x, const sixi_smp_params* p,
                          const int32_t* hist, uint64_t n_hist, const uint32_t* mask,
                          std::vector<Cand>& out) {
    const uint64_t vocab = x.size();
    const SamplingParams sp = to_engine(p);
    std::vector<int32_t> recent;
    if (mask == nullptr) {
        recent.assign(hist, hist + n_hist);
        auto r = DeterministicSampler::compute_sampling_candidates(x.data(), vocab, sp, recent);
        if (!r.ok()) return static_cast<int32_t>(r.code());
        out = r.value();
        return SIXI_OK;
    }
    std::vector<float> comp;
    std::vector<int32_t> ids;
    std::vector<int32_t> remap(vocab, -1);
    for (uint64_t i = 0; i < vocab; ++i) {
        if (!allowed(mask, i)) continue;
        remap[i] = static_cast<int32_t>(ids.size());
        ids.push_back(static_cast<int32_t>(i));
        comp.push_back(x[i]);
    }
    if (ids.empty()) return SIXI_INVALID_ARGUMENT;
    for (uint64_t j = 0; j < n_hist; ++j) {
        const int32_t t = hist[j];
        if (t >= 0 && static_cast<uint64_t>(t) < vocab && remap[t] >= 0) recent.push_back(remap[t]);
    }
    auto r = DeterministicSampler::compute_sampling_candidates(comp.data(), comp.size(), sp, recent);
    if (!r.ok()) return static_cast<int32_t>(r.code());
    out = r.value();
    for (auto& c : out) c.id = ids[static_cast<size_t>(c.id)];
    return SIXI_OK;
}

int32_t draw(const std::vector<Cand>& c, double u) {
    if (c.empty()) return -1;
    double cdf = 0.0;
    for (const auto& x : c) {
        cdf += x.prob;
        if (u < cdf) return x.id;
    }
    return c.back().id;
}

int32_t sample_one(const void* row, uint32_t dtype, uint64_t vocab, const sixi_smp_params* p,
                   const int32_t* hist, uint64_t n_hist, const uint32_t* mask, double u,
                   int32_t* out_token) {
    *out_token = -1;
    if (!expressible(p)) return ORC_UNSUPPORTED;
    std::vector<float> x;
    load_row(row, dtype, vocab, x);
    std::vector<Cand> c;
    const int32_t st = engine_candidates(x, p, hist, n_hist, mask, c);
    if (st != SIXI_OK) return st;
    // sample_token: greedy returns the front candidate and consumes no uniform
    *out_token = p->temperature <= 0.0f ? (c.empty() ? -1 : c.front().id) : draw(c, u);
    return SIXI_OK;
}

int32_t greedy_row(const void* row, uint32_t dtype, uint64_t vocab, const uint32_t* mask,
                   int32_t* out_token) {
    std::vector<float> x;
    load_row(row, dtype, vocab, x);
    int32_t st = SIXI_OK;
    std::vector<float> comp;
    std::vector<int32_t> ids;
    for (uint64_t i = 0; i < vocab; ++i) {
        if (!allowed(mask, i)) continue;
        if (std::isnan(x[i]) || std::isinf(x[i])) st = SIXI_NUMERIC_NAN_OR_INF;
        comp.push_back(x[i]);
        ids.push_back(static_cast<int32_t>(i));
    }
    if (ids.empty()) {
        *out_token = -1;
        return SIXI_INVALID_ARGUMENT;
    }
    const int32_t a = DeterministicSampler::sample_greedy_argmax(comp.data(), comp.size());
    *out_token = ids[static_cast<size_t>(a)];
    return st;
}

const uint32_t* row_mask(const uint32_t* masks, uint64_t vocab, const sixi_smp_params* p,
                         uint64_t r) {
    if (masks == nullptr || !(p->flags & SIXI_SMP_ROW_MASKED)) return nullptr;
    return masks + r * ((vocab + 31) / 32);
}

template <typename F>
void parallel_for(uint32_t n, int32_t n_threads, F fn) {
    if (n_threads <= 0) n_threads = static_cast<int32_t>(std::thread::hardware_concurrency());
    if (n_threads < 1) n_threads = 1;
    if (static_cast<uint32_t>(n_threads) > n) n_threads = static_cast<int32_t>(n ? n : 1);
    if (n_threads == 1) {
        for (uint32_t i = 0; i < n; ++i) fn(i);
        return;
    }
    std::vector<std::thread> th;
    const uint32_t per = (n + static_cast<uint32_t>(n_threads) - 1) / static_cast<uint32_t>(n_threads);
    for (int32_t t = 0; t < n_threads; ++t) {
        const uint32_t b = std::min(n, static_cast<uint32_t>(t) * per), e = std::min(n, b + per);
        th.emplace_back([=]() {
            for (uint32_t i = b; i < e; ++i) fn(i);
        });
    }
    for (auto& t : th) t.join();
}

}  // namespace

EXPORT int32_t orc_kind(void) { return 1; }

EXPORT double orc_philox_uniform(uint64_t, uint64_t, uint32_t) { return -1.0; /* not provided */ }

EXPORT int32_t orc_greedy_argmax(const float* logits, uint64_t vocab) {
    return DeterministicSampler::sample_greedy_argmax(logits, vocab);
}

EXPORT void orc_full_distribution(const void* row, uint32_t dtype, uint64_t vocab, float temperature,
                                  float* out) {
    std::vector<float> x;
    load_row(row, dtype, vocab, x);
    std::vector<float> probs;
    DeterministicSampler::compute_full_distribution(x.data(), vocab, temperature, probs);
    for (uint64_t i = 0; i < vocab; ++i) out[i] = i < probs.size() ? probs[i] : 0.0f;
}

// The engine's own SuffixDrafter (src/speculative/speculative.cpp:24-176).
EXPORT int32_t orc_suffix_draft(const int32_t* hist, uint64_t n, uint32_t min_match_len, uint32_t max_window_tokens,
                                int32_t use_anchor, int32_t anchor, uint32_t k, int32_t* out_drafts) {
    const std::vector<int32_t> h(hist, hist + n);
    const sixi_asi::speculative::SuffixDrafter d(min_match_len, max_window_tokens);
    const auto p = use_anchor ? d.propose_anchored(h, anchor, k) : d.propose(h, k, 0);
    for (uint32_t i = 0; i < k; ++i) out_drafts[i] = p.has_value() ? p->draft_tokens[i] : -1;
    return p.has_value() ? static_cast<int32_t>(p->match_len) : 0;
}

// The engine's own inspect_and_apply_numeric_policy (src/core/numeric.cpp:628-699), its report
// copied field by field into the sixi_smp_numeric_report layout.
EXPORT int32_t orc_numeric_policy(float* data, int64_t n, uint32_t policy, float clamp_abs_max,
                                  sixi_smp_numeric_report* out) {
    sixi_asi::NumericHealthReport rep{};
    const sixi_asi::NumericPolicy pol = policy == SIXI_SMP_NUMERIC_CLAMP ? sixi_asi::NumericPolicy::EmergencyClampAndReport
                                                                          : sixi_asi::NumericPolicy::FailAndInvalidate;
    const sixi_asi::Status st = sixi_asi::inspect_and_apply_numeric_policy(data, n, pol, clamp_abs_max, &rep);
    const int32_t code = static_cast<int32_t>(st.code);
    if (out != nullptr) {
        out->healthy = rep.healthy ? 1 : 0;
        out->request_corrupted = rep.request_corrupted ? 1 : 0;
        out->state_invalidated = rep.state_invalidated ? 1 : 0;
        out->emergency_clamped = rep.emergency_clamped ? 1 : 0;
        out->status = code;
        out->nan_count = rep.nan_count;
        out->inf_count = rep.inf_count;
        out->first_bad_index = rep.first_bad_index;
    }
    return code;
}

EXPORT int32_t orc_greedy_row(const void* row, uint32_t dtype, uint64_t vocab,
                              const uint32_t* mask, int32_t* out_token) {
    return greedy_row(row, dtype, vocab, mask, out_token);
}

EXPORT int32_t orc_candidates(const void* row, uint32_t dtype, uint64_t vocab,
                              const sixi_smp_params* p, const int32_t* hist, uint64_t n_hist,
                              const uint32_t* mask, uint64_t cap, int32_t* out_ids,
                              double* out_probs, uint64_t* out_n) {
    *out_n = 0;
    if (!expressible(p)) return ORC_UNSUPPORTED;
    std::vector<float> x;
    load_row(row, dtype, vocab, x);
    std::vector<Cand> c;
    const int32_t st = engine_candidates(x, p, hist, n_hist, mask, c);
    if (st != SIXI_OK) return st;
    for (uint64_t i = 0; i < c.size() && i < cap; ++i) {
        out_ids[i] = c[i].id;
        out_probs[i] = c[i].prob;
    }
    *out_n = c.size();
    return SIXI_OK;
}

EXPORT int32_t orc_sample(const void* row, uint32_t dtype, uint64_t vocab,
                          const sixi_smp_params* p, const int32_t* hist, uint64_t n_hist,
                          const uint32_t* mask, double u, int32_t* out_token) {
    return sample_one(row, dtype, vocab, p, hist, n_hist, mask, u, out_token);
}

EXPORT int32_t orc_sample_batch(const void* logits, uint32_t dtype, uint32_t n_rows,
                                uint64_t row_stride, uint64_t vocab, const sixi_smp_params* params,
                                const uint32_t* masks, const int32_t* hist_tokens,
                                const int64_t* hist_offsets, const double* uniforms, uint64_t,
                                int32_t* out_tokens, int32_t* out_status, int32_t n_threads) {
    if (uniforms == nullptr) return ORC_UNSUPPORTED;
    const size_t esz = dtype == SIXI_SMP_BF16 ? 2 : 4;
    parallel_for(n_rows, n_threads, [&](uint32_t r) {
        const sixi_smp_params* p = &params[r];
        const void* row = static_cast<const char*>(logits) + static_cast<size_t>(r) * row_stride * esz;
        const int32_t* hist = nullptr;
        uint64_t nh = 0;
        if (hist_tokens && hist_offsets) {
            hist = hist_tokens + hist_offsets[r];
            nh = static_cast<uint64_t>(hist_offsets[r + 1] - hist_offsets[r]);
        }
        out_status[r] = sample_one(row, dtype, vocab, p, hist, nh, row_mask(masks, vocab, p, r),
                                   uniforms[r], &out_tokens[r]);
    });
    return SIXI_OK;
}

EXPORT int32_t orc_verify(const void* target, uint32_t dtype, uint64_t row_stride, uint64_t vocab,
                          const float* draft_probs, const int32_t* drafts, const int32_t* n_drafts,
                          uint32_t n_streams, uint32_t k, const sixi_smp_params* params,
                          const uint32_t* masks, const int32_t* hist_tokens,
                          const int64_t* hist_offsets, const double* uniforms, uint64_t,
                          int32_t* out_accepted, int32_t* out_tokens, int32_t* out_n_tokens,
                          int32_t* out_first_reject, int32_t* out_uniforms_used,
                          int32_t* out_status, int32_t n_threads) {
    if (uniforms == nullptr) return ORC_UNSUPPORTED;
    const size_t esz = dtype == SIXI_SMP_BF16 ? 2 : 4;
    const uint64_t V = vocab;
    parallel_for(n_streams, n_threads, [&](uint32_t s) {
        const sixi_smp_params* p = &params[s];
        const uint32_t nd = n_drafts ? static_cast<uint32_t>(n_drafts[s]) : k;
        const int32_t* d = drafts + static_cast<size_t>(s) * k;
        int32_t* out = out_tokens + static_cast<size_t>(s) * (k + 1);
        auto row = [&](uint32_t i) {
            return static_cast<const char*>(target) + (static_cast<size_t>(s) * (k + 1) + i) * row_stride * esz;
        };
        auto mask = [&](uint32_t i) { return row_mask(masks, V, p, static_cast<uint64_t>(s) * (k + 1) + i); };
        auto uni = [&](uint32_t j) { return uniforms[static_cast<size_t>(s) * (k + 1) + j]; };
        std::vector<int32_t> committed;
        uint32_t used = 0, acc = 0;
        int32_t first_reject = -1, status = SIXI_OK;
        for (uint32_t i = 0; i <= k; ++i) out[i] = -1;
        if (!expressible(p) || nd > k) {
            status = expressible(p) ? SIXI_INVALID_ARGUMENT : ORC_UNSUPPORTED;
        } else if (p->temperature <= 0.0f) {
            for (uint32_t i = 0; i <= nd; ++i) {
                int32_t t = -1;
                const int32_t gs = greedy_row(row(i), dtype, V, mask(i), &t);
                if (gs == SIXI_INVALID_ARGUMENT) {
                    status = gs;
                    break;
                }
                if (gs != SIXI_OK && status == SIXI_OK) status = gs;
                if (i == nd) {
                    committed.push_back(t);
                    break;
                }
                if (d[i] == t) {
                    committed.push_back(d[i]);
                    ++acc;
                } else {
                    committed.push_back(t);
                    first_reject = static_cast<int32_t>(i);
                    break;
                }
            }
        } else {
            std::vector<int32_t> base;
            if (hist_tokens && hist_offsets) {
                base.assign(hist_tokens + hist_offsets[s], hist_tokens + hist_offsets[s + 1]);
            }
            std::vector<int32_t> recent = base;
            std::vector<float> x;
            bool rejected = false;
            for (uint32_t i = 0; i < nd && status == SIXI_OK; ++i) {
                load_row(row(i), dtype, V, x);
                std::vector<Cand> cands;
                const int32_t cs = engine_candidates(x, p, recent.data(), recent.size(), mask(i), cands);
                if (cs != SIXI_OK) {
                    status = cs;
                    break;
                }
                const int32_t di = d[i];
                const bool in_range = di >= 0 && static_cast<uint64_t>(di) < V;
                if (draft_probs) {
                    const float* q = draft_probs + (static_cast<size_t>(s) * k + i) * row_stride;
                    std::vector<float> pt(V, 0.0f);
                    for (const auto& c : cands) pt[static_cast<size_t>(c.id)] = static_cast<float>(c.prob);
                    const float p_d = in_range ? pt[static_cast<size_t>(di)] : 0.0f;
                    const float q_d = in_range ? q[di] : 1.0f;
                    const double accept_prob = (q_d <= 0.0f)
                        ? (p_d > 0.0f ? 1.0 : 0.0)
                        : std::min(1.0, static_cast<double>(p_d) / std::max(1e-12, static_cast<double>(q_d)));
                    const double r = uni(used++);
                    if (r < accept_prob) {
                        committed.push_back(di);
                        ++acc;
                        recent.push_back(di);
                        continue;
                    }
                    first_reject = static_cast<int32_t>(i);
                    std::vector<double> residual(V, 0.0);
                    double res_sum = 0.0;
                    for (uint64_t xx = 0; xx < V; ++xx) {
                        const double diff = std::max(0.0, static_cast<double>(pt[xx]) - static_cast<double>(q[xx]));
                        residual[xx] = diff;
                        res_sum += diff;
                    }
                    const double u = uni(used++);
                    int32_t repl = static_cast<int32_t>(V - 1);
                    double cdf = 0.0;
                    for (uint64_t xx = 0; xx < V; ++xx) {
                        cdf += res_sum > 1e-12 ? residual[xx] / res_sum : static_cast<double>(pt[xx]);
                        if (u < cdf) {
                            repl = static_cast<int32_t>(xx);
                            break;
                        }
                    }
                    committed.push_back(repl);
                    rejected = true;
                    break;
                }
                double p_d = 0.0;
                for (const auto& c : cands) {
                    if (c.id == di) {
                        p_d = c.prob;
                        break;
                    }
                }
                const double r = uni(used++);
                if (r < p_d) {
                    committed.push_back(di);
                    ++acc;
                    recent.push_back(di);
                    continue;
                }
                first_reject = static_cast<int32_t>(i);
                std::vector<Cand> residual;
                double res_sum = 0.0;
                for (const auto& c : cands) {
                    if (c.id != di) {
                        residual.push_back(c);
                        res_sum += c.prob;
                    }
                }
                const double u = uni(used++);
                int32_t repl;
                if (!residual.empty() && res_sum > 0.0) {
                    for (auto& c : residual) c.prob /= res_sum;
                    repl = draw(residual, u);
                } else {
                    repl = draw(cands, u);
                }
                committed.push_back(repl);
                rejected = true;
                break;
            }
            if (status == SIXI_OK && !rejected) {
                const std::vector<int32_t>& h = draft_probs ? base : recent;
                int32_t t = -1;
                const double u = uni(used++);
                const int32_t bs = sample_one(row(nd), dtype, V, p, h.data(), h.size(), mask(nd), u, &t);
                if (bs != SIXI_OK) {
                    status = bs;
                } else {
                    committed.push_back(t);
                }
            }
        }
        if (status != SIXI_OK && status != SIXI_NUMERIC_NAN_OR_INF) {
            committed.clear();
            acc = 0;
            first_reject = -1;
        }
        for (size_t i = 0; i < committed.size(); ++i) out[i] = committed[i];
        out_accepted[s] = static_cast<int32_t>(acc);
        out_n_tokens[s] = static_cast<int32_t>(committed.size());
        out_first_reject[s] = first_reject;
        out_uniforms_used[s] = static_cast<int32_t>(used);
        out_status[s] = status;
    });
    return SIXI_OK;
}

// ---------------------------------------------------------------------------------------------
// The engine's SpeculativeDecoder::step over pre-supplied rows

namespace {

// An IBackend that replays target logits: forward_sequence_all_logits returns the supplied rows
// (rows 1..k on the slow path, where the caller's current_last_logits is row 0; rows 0..k on the
// fast path, after the anchor's row). Other forwards return a zero row; the state it checkpoints
// is the RNG's, as a real backend's checkpoint carries it (core_execution.hpp:184-190).
class ReplayBackend final : public IBackend {
public:
    ReplayBackend(const float* rows, uint32_t n_rows, uint64_t vocab, bool fast, uint32_t window)
        : rows_(rows), n_rows_(n_rows), vocab_(vocab), fast_(fast), window_(window) {}
    std::string backend_name() const override { return "replay"; }
    uint64_t vocab_size() const override { return vocab_; }
    int32_t eos_token_id() const override { return -1; }
    Result<std::vector<int32_t>> tokenize(const std::string&, bool) override {
        return Result<std::vector<int32_t>>(ErrorCode::BackendError, "replay backend has no tokenizer");
    }
    Result<std::string> detokenize(const std::vector<int32_t>&) override {
        return Result<std::string>(ErrorCode::BackendError, "replay backend has no tokenizer");
    }
    Status reset_state() override { return Status::Ok(); }
    Result<BackendSequenceState> checkpoint_state(const DeterministicRng& rng) override {
        BackendSequenceState st;
        st.seq_len = seq_len_;
        st.rng_state = rng.checkpoint();
        return Result<BackendSequenceState>(std::move(st));
    }
    Status restore_state(const BackendSequenceState& ck, DeterministicRng& rng) override {
        seq_len_ = ck.seq_len;
        rng.restore(ck.rng_state);
        return Status::Ok();
    }
    Result<std::vector<float>> forward_tokens(const std::vector<int32_t>& t, uint32_t) override {
        seq_len_ += t.size();
        return Result<std::vector<float>>(std::vector<float>(vocab_, 0.0f));
    }
    Result<std::vector<std::vector<float>>> forward_sequence_all_logits(const std::vector<int32_t>& t) override {
        using R = Result<std::vector<std::vector<float>>>;
        const uint32_t first = fast_ ? 0u : 1u;
        if (first + t.size() > n_rows_) return R(ErrorCode::BackendError, "replay backend: too few rows");
        std::vector<std::vector<float>> out;
        for (size_t i = 0; i < t.size(); ++i) {
            const float* r = rows_ + (first + i) * vocab_;
            out.emplace_back(r, r + vocab_);
        }
        seq_len_ += t.size();
        return R(std::move(out));
    }
    bool supports_fast_prefix_rollback() const noexcept override { return fast_; }
    uint32_t fast_rollback_window() const noexcept override { return fast_ ? window_ : 0u; }
    uint64_t current_seq_len() const noexcept override { return seq_len_; }
    Status rollback_to_position(uint64_t n) override {
        if (!fast_) return Status::Error(ErrorCode::BackendError, "no rollback ring");
        seq_len_ = n;
        return Status::Ok();
    }

private:
    const float* rows_;
    uint32_t n_rows_;
    uint64_t vocab_;
    bool fast_;
    uint32_t window_;
    uint64_t seq_len_ = 1000;
};

// An INeuralDrafter that proposes the given drafts, with dense draft probabilities when given.
class FixedDrafter final : public spec::INeuralDrafter {
public:
    FixedDrafter(const int32_t* drafts, uint32_t k, const float* q, uint64_t vocab) {
        p_.source = spec::DraftSource::NeuralMTP;
        p_.draft_tokens.assign(drafts, drafts + k);
        if (q != nullptr)
            for (uint32_t i = 0; i < k; ++i) p_.draft_probs.emplace_back(q + i * vocab, q + (i + 1) * vocab);
    }
    sixi_asi::NeuralDrafterType drafter_type() const noexcept override { return sixi_asi::NeuralDrafterType::MTP; }
    std::string drafter_name() const override { return "fixed"; }
    Result<spec::DraftProposal> propose_k(const std::vector<int32_t>&, const std::vector<float>&, uint32_t) override {
        return Result<spec::DraftProposal>(p_);
    }

private:
    spec::DraftProposal p_;
};

int32_t spec_step(int32_t fast, const float* anchor_row, const float* rows, uint64_t vocab, const float* draft_probs,
                  const int32_t* drafts, uint32_t k, const sixi_smp_params* p, const int32_t* hist, uint64_t n_hist,
                  uint64_t* rng_io, int32_t* out_tokens, int32_t* out_n, int32_t* out_accepted,
                  int32_t* out_first_reject) {
    *out_n = 0;
    *out_accepted = 0;
    *out_first_reject = -1;
    if (!expressible(p) || k == 0) return ORC_UNSUPPORTED;
    spec::SpeculativeConfig cfg;
    cfg.execution_mode = p->mode == SIXI_SMP_ADAPTIVE ? ExecutionMode::Adaptive : ExecutionMode::StrictReplay;
    cfg.enable_suffix_drafter = false;
    cfg.neural_drafter = sixi_asi::NeuralDrafterType::MTP;
    cfg.draft_k = k;
    cfg.adaptive_k = false;
    cfg.min_adaptive_k = 1;
    cfg.max_adaptive_k = k;
    auto backend = std::make_shared<ReplayBackend>(rows, k + 1, vocab, fast != 0, k);
    auto drafter = std::make_shared<FixedDrafter>(drafts, k, fast ? nullptr : draft_probs, vocab);
    spec::SpeculativeDecoder dec(cfg, backend, drafter);
    std::vector<int32_t> ctx(hist, hist + n_hist);
    const float* first = fast ? anchor_row : rows;
    std::vector<float> last(first, first + vocab);
    DeterministicRng rng;
    rng.restore(RngState{rng_io[0], rng_io[1]});
    const SamplingParams sp = to_engine(p);
    auto r = dec.step(ctx, last, sp, rng);
    if (!r.ok()) return static_cast<int32_t>(r.code());
    const auto& res = r.value();
    std::vector<int32_t> toks = res.committed_tokens;
    if (fast) {
        // the fast path keeps the token after the last committed one for the next step: carried for
        // sampling, the argmax of the returned logits for greedy (speculative.cpp:704-714)
        if (sp.temperature > 0.0f) {
            const auto c = dec.carried_token(ctx);
            toks.push_back(c.has_value() ? *c : -1);
        } else {
            toks.push_back(DeterministicSampler::sample_greedy_argmax(last.data(), vocab));
        }
    }
    for (size_t i = 0; i < toks.size(); ++i) out_tokens[i] = toks[i];
    *out_n = static_cast<int32_t>(toks.size());
    *out_accepted = static_cast<int32_t>(res.accepted_draft_count);
    *out_first_reject = res.first_rejected_position;
    const RngState after = rng.checkpoint();
    rng_io[0] = after.state;
    rng_io[1] = after.inc;
    return SIXI_OK;
}

}  // namespace

// One uniform of the engine's DeterministicRng from the state (state, inc) in rng_io, which is
// advanced in place (core_execution.cpp:33-61).
EXPORT double orc_ref_rng_uniform(uint64_t* rng_io) {
    DeterministicRng rng;
    rng.restore(RngState{rng_io[0], rng_io[1]});
    const double u = rng.next_uniform01();
    const RngState after = rng.checkpoint();
    rng_io[0] = after.state;
    rng_io[1] = after.inc;
    return u;
}

// The engine's seeded RNG state: DeterministicRng(seed, seq).
EXPORT void orc_ref_rng_seed(uint64_t seed, uint64_t seq, uint64_t* rng_out) {
    const DeterministicRng rng(seed, seq);
    const RngState st = rng.checkpoint();
    rng_out[0] = st.state;
    rng_out[1] = st.inc;
}

// One SpeculativeDecoder::step (speculative.cpp:367-976) of one stream with fp32 rows.
//   fast = 0: slow path. rows [k+1][V]: row 0 is current_last_logits, rows 1..k are returned by
//             forward_sequence_all_logits(drafts); draft_probs [k][V] (dense q) or NULL.
//             out_tokens = committed_tokens (accepted drafts, then the replacement or the bonus).
//   fast = 1: fast path. anchor_row is current_last_logits (the anchor is drawn from it), rows
//             [k+1][V] are the verify batch after the anchor; drafts are one-hot proposals.
//             out_tokens = committed_tokens (anchor, accepted drafts), then the token the step
//             determined for the next position (replacement or bonus).
// rng_io = the engine RNG's (state, inc) before the step, replaced by the state after it.
// out_tokens needs k + 2 slots. Returns the step's ErrorCode.
EXPORT int32_t orc_ref_spec_step(int32_t fast, const float* anchor_row, const float* rows, uint64_t vocab,
                                 const float* draft_probs, const int32_t* drafts, uint32_t k, const sixi_smp_params* p,
                                 const int32_t* hist, uint64_t n_hist, uint64_t* rng_io, int32_t* out_tokens,
                                 int32_t* out_n, int32_t* out_accepted, int32_t* out_first_reject) {
    return spec_step(fast, anchor_row, rows, vocab, draft_probs, drafts, k, p, hist, n_hist, rng_io, out_tokens,
                     out_n, out_accepted, out_first_reject);
}

// The slow-path step for S streams (config 4 on the host cores): target rows [S][k+1][V] (fp32,
// or bf16 converted by the engine's bf16_to_fp32), q [S][k][V], drafts [S][k], one RNG state per
// stream (rng_io [S][2], advanced in place), out_tokens [S][k+2]; statuses in out_status.
EXPORT int32_t orc_ref_spec_step_batch(const void* rows, uint32_t dtype, uint64_t vocab, const float* draft_probs,
                                       const int32_t* drafts, uint32_t n_streams, uint32_t k,
                                       const sixi_smp_params* params, const int32_t* hist_tokens,
                                       const int64_t* hist_offsets, uint64_t* rng_io, int32_t* out_tokens,
                                       int32_t* out_n, int32_t* out_accepted, int32_t* out_first_reject,
                                       int32_t* out_status, int32_t n_threads) {
    const size_t esz = dtype == SIXI_SMP_BF16 ? 2 : 4;
    parallel_for(n_streams, n_threads, [&](uint32_t s) {
        std::vector<float> x;
        std::vector<float> tr(static_cast<size_t>(k + 1) * vocab);
        for (uint32_t i = 0; i <= k; ++i) {
            load_row(static_cast<const char*>(rows) + (static_cast<size_t>(s) * (k + 1) + i) * vocab * esz, dtype,
                     vocab, x);
            std::copy(x.begin(), x.end(), tr.begin() + static_cast<size_t>(i) * vocab);
        }
        const int32_t* h = hist_tokens ? hist_tokens + hist_offsets[s] : nullptr;
        const uint64_t nh = hist_tokens ? static_cast<uint64_t>(hist_offsets[s + 1] - hist_offsets[s]) : 0;
        out_status[s] = spec_step(0, nullptr, tr.data(), vocab,
                                  draft_probs ? draft_probs + static_cast<size_t>(s) * k * vocab : nullptr,
                                  drafts + static_cast<size_t>(s) * k, k, &params[s], h, nh, rng_io + 2 * s,
                                  out_tokens + static_cast<size_t>(s) * (k + 2), &out_n[s], &out_accepted[s],
                                  &out_first_reject[s]);
    });
    return SIXI_OK;
}
