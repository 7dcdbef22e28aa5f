/*
 * sixi_oracle.c - TEST INFRASTRUCTURE ONLY (parity checker; never linked by the product).
 *
 * Plain-C restatement of the Sixi-ASI engine's per-step logits-to-token path:
 *   - DeterministicSampler::sample_greedy_argmax   src/core/core_execution.cpp:394-407
 *   - DeterministicSampler::compute_sampling_candidates  src/core/core_execution.cpp:449-584
 *   - DeterministicSampler::sample_from_candidates src/core/core_execution.cpp:586-601
 *   - DeterministicSampler::sample_token          src/core/core_execution.cpp:603-619
 *   - SpeculativeDecoder::step verification, fast path (one-hot drafts)
 *                                                  src/speculative/speculative.cpp:630-692
 *   - SpeculativeDecoder::step verification with draft probabilities (dense q)
 *                                                  src/speculative/speculative.cpp:801-916
 *   - numeric::bf16_to_fp32                        src/core/numeric.cpp:108-111
 * with three additions the engine cannot express, each identity when unused:
 *   - grammar mask: masked tokens are removed before everything else, i.e. the row is compacted
 *     to its allowed ids (ascending), which keeps relative order and tie-breaks;
 *   - supplied uniforms (or Philox4x32-10) instead of the engine's PCG32 stream;
 *   - frequency penalty (subtracted once per history occurrence, after the per-unique-id
 *     repetition/presence penalty) and min-p (after top-p: keep prob >= min_p * max prob,
 *     renormalise).
 * Arithmetic follows the engine's order and precision (fp32 penalties, fp64 softmax with libm exp,
 * sequential sums in candidate order), so the port is bit-identical to the reference build on the
 * engine-expressible inputs; tests/test_oracle.py checks this against oracle/_ref and the golden
 * vectors in tests/golden/.
 */
#define _GNU_SOURCE
#include "sixi_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

int32_t orc_kind(void) { return 0; }

/* ------------------------------------------------------------------------------------------ */
/* Philox4x32-10, from Salmon, Moraes, Dror, Shaw: "Parallel Random Numbers: As Easy as 1, 2, 3"
 * (SC'11): 10 rounds of two 32x32->64 multiplies with a Weyl-sequence key schedule. */
#define PHILOX_M0 0xD2511F53u
#define PHILOX_M1 0xCD9E8D57u
#define PHILOX_W0 0x9E3779B9u
#define PHILOX_W1 0xBB67AE85u

void orc_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
    uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3];
    uint32_t k0 = key[0], k1 = key[1];
    for (int r = 0; r < 10; ++r) {
        const uint64_t p0 = (uint64_t)PHILOX_M0 * c0;
        const uint64_t p1 = (uint64_t)PHILOX_M1 * c2;
        const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
        const uint32_t n1 = (uint32_t)p1;
        const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
        const uint32_t n3 = (uint32_t)p0;
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        k0 += PHILOX_W0;
        k1 += PHILOX_W1;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

double orc_philox_uniform(uint64_t seed, uint64_t counter, uint32_t slot) {
    const uint32_t ctr[4] = {slot, 0u, (uint32_t)counter, (uint32_t)(counter >> 32)};
    const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    uint32_t o[4];
    orc_philox4x32_10(ctr, key, o);
    /* same 53-bit construction as DeterministicRng::next_uniform01 (core_execution.cpp:55-61) */
    const uint64_t v = ((uint64_t)o[0] << 32) | (uint64_t)o[1];
    return (double)(v >> 11) * (1.0 / 9007199254740992.0);
}

/* ------------------------------------------------------------------------------------------ */
static float bf16_to_f32(uint16_t b) {
    const uint32_t bits = (uint32_t)b << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static void load_row(const void* row, uint32_t dtype, uint64_t vocab, float* out) {
    if (dtype == SIXI_SMP_BF16) {
        const uint16_t* r = (const uint16_t*)row;
        for (uint64_t i = 0; i < vocab; ++i) out[i] = bf16_to_f32(r[i]);
    } else {
        memcpy(out, row, vocab * sizeof(float));
    }
}

static inline int allowed(const uint32_t* mask, uint64_t i) {
    return mask == NULL || ((mask[i >> 5] >> (i & 31u)) & 1u);
}

int32_t orc_greedy_argmax(const float* logits, uint64_t vocab) {
    if (logits == NULL || vocab == 0) return -1;
    int32_t best_id = 0;
    float best = logits[0];
    for (uint64_t i = 1; i < vocab; ++i) {
        if (logits[i] > best) {
            best = logits[i];
            best_id = (int32_t)i;
        }
    }
    return best_id;
}

/* SuffixDrafter::propose (speculative.cpp:28-113): positions from the most recent backwards, the
 * suffix compared from the end of a window of up to 16 tokens ending at pos + L - 1; a strictly
 * longer match replaces the best. Without one of min_match_len, exact matches of the history's
 * tail, longest first, most recent first. propose_anchored (speculative.cpp:115-176): the pattern
 * is the history's tail followed by the anchor, matched backwards from each occurrence of the
 * anchor. The k drafts repeat the continuation after the match. */
int32_t orc_suffix_draft(const int32_t* h, uint64_t n, uint32_t min_match_len, uint32_t max_window_tokens,
                         int32_t use_anchor, int32_t anchor, uint32_t k, int32_t* out_drafts) {
    uint64_t best_len = 0, best_cont = 0;
    int ok = 0;
    const uint64_t ws = n > max_window_tokens ? n - max_window_tokens : 0;
    if (!use_anchor) {
        if (k != 0 && min_match_len != 0 && n > min_match_len) {
            const uint64_t maxp = (n - 1) < 16 ? (n - 1) : 16;
            for (uint64_t pos = n - min_match_len - 1;; --pos) {
                if (pos < ws) break;
                uint64_t m = 0;
                const uint64_t L = maxp < n - 1 - pos ? maxp : n - 1 - pos;
                while (m < L && h[pos + L - 1 - m] == h[n - 1 - m]) ++m;
                if (m >= min_match_len && m > best_len) {
                    best_len = m;
                    best_cont = pos + L;
                }
                if (pos == ws) break;
            }
            if (best_len < min_match_len) {
                for (uint64_t len = maxp; len >= min_match_len; --len) {
                    if (len >= n) continue;
                    const int32_t* tail = h + (n - len);
                    for (uint64_t pos = n - len - 1;; --pos) {
                        if (pos < ws) break;
                        uint64_t i = 0;
                        while (i < len && h[pos + i] == tail[i]) ++i;
                        if (i == len) {
                            best_len = len;
                            best_cont = pos + len;
                            break;
                        }
                        if (pos == ws) break;
                    }
                    if (best_len >= min_match_len) break;
                    if (len == min_match_len) break;
                }
            }
            ok = best_len >= min_match_len && best_cont < n;
        }
    } else if (k != 0 && n >= 2) {
        const uint64_t min_total = (uint64_t)min_match_len + 1 > 2 ? (uint64_t)min_match_len + 1 : 2;
        const uint64_t max_total = n < 16 ? n : 16;
        for (uint64_t pos = n - 1;; --pos) {
            if (pos < ws) break;
            if (h[pos] == anchor && pos + 1 < n) {
                uint64_t m = 1;
                const uint64_t max_here = max_total < pos + 1 ? max_total : pos + 1;
                while (m < max_here && h[pos - m] == h[n - m]) ++m;
                if (m >= min_total && m > best_len) {
                    best_len = m;
                    best_cont = pos + 1;
                }
            }
            if (pos == ws) break;
        }
        ok = best_len >= min_total && best_cont < n;
    }
    for (uint32_t i = 0; i < k; ++i) out_drafts[i] = ok ? h[best_cont + (i % (n - best_cont))] : -1;
    return ok ? (int32_t)best_len : 0;
}

/* inspect_and_apply_numeric_policy (numeric.cpp:628-699): one forward scan; NaN and infinity are
 * counted and the first of either is remembered; the clamp policy rewrites NaN as 0, infinities as
 * the signed bound |clamp_abs_max|, and (bound > 0) finite values beyond the bound; the report's
 * flags follow numeric.cpp:674-692. */
int32_t orc_numeric_policy(float* data, int64_t n, uint32_t policy, float clamp_abs_max,
                           sixi_smp_numeric_report* out) {
    sixi_smp_numeric_report r;
    memset(&r, 0, sizeof(r));
    r.healthy = 1;
    r.first_bad_index = -1;
    if (n < 0 || (n > 0 && data == NULL)) {
        r.status = SIXI_INVALID_ARGUMENT;
        if (out) *out = r;
        return SIXI_INVALID_ARGUMENT;
    }
    const int clamp = policy == SIXI_SMP_NUMERIC_CLAMP;
    const float limit = fabsf(clamp_abs_max);
    for (int64_t i = 0; i < n; ++i) {
        const float v = data[i];
        if (isnan(v)) {
            ++r.nan_count;
            if (r.first_bad_index < 0) r.first_bad_index = i;
            if (clamp) data[i] = 0.0f;
        } else if (isinf(v)) {
            ++r.inf_count;
            if (r.first_bad_index < 0) r.first_bad_index = i;
            if (clamp) data[i] = (v > 0.0f) ? limit : -limit;
        } else if (clamp && limit > 0.0f) {
            if (v > limit) {
                data[i] = limit;
                r.emergency_clamped = 1;
            } else if (v < -limit) {
                data[i] = -limit;
                r.emergency_clamped = 1;
            }
        }
    }
    if (r.nan_count > 0 || r.inf_count > 0) {
        r.healthy = 0;
        if (!clamp) {
            r.request_corrupted = 1;
            r.state_invalidated = 1;
            r.emergency_clamped = 0;
            r.status = SIXI_NUMERIC_NAN_OR_INF;
        } else {
            r.emergency_clamped = 1;
        }
    }
    if (out) *out = r;
    return r.status;
}

/* compute_full_distribution (core_execution.cpp:409-447): the scaled maximum ignores NaN; a NaN
 * or +inf logit makes the sum NaN and every probability 0. Built with -ffp-contract=off like the
 * engine, so x * inv_temp - max is a multiply then a subtract. */
void orc_full_distribution(const void* row, uint32_t dtype, uint64_t vocab, float temperature, float* out) {
    for (uint64_t i = 0; i < vocab; ++i) out[i] = 0.0f;
    if (row == NULL || vocab == 0) return;
    float* x = (float*)malloc(vocab * sizeof(float));
    double* e = (double*)malloc(vocab * sizeof(double));
    if (x == NULL || e == NULL) {
        free(x);
        free(e);
        return;
    }
    load_row(row, dtype, vocab, x);
    if (temperature <= 0.0f) {
        out[orc_greedy_argmax(x, vocab)] = 1.0f;
    } else {
        const double inv_temp = 1.0 / (double)temperature;
        double max_scaled = -INFINITY;
        for (uint64_t i = 0; i < vocab; ++i) {
            const double s = (double)x[i] * inv_temp;
            if (s > max_scaled) max_scaled = s;
        }
        double sum = 0.0;
        for (uint64_t i = 0; i < vocab; ++i) {
            e[i] = exp((double)x[i] * inv_temp - max_scaled);
            sum += e[i];
        }
        if (sum > 0.0) {
            for (uint64_t i = 0; i < vocab; ++i) out[i] = (float)(e[i] / sum);
        }
    }
    free(x);
    free(e);
}

/* argmax of the compacted allowed logits (first allowed element plays the role of index 0) */
static int32_t masked_argmax(const float* x, uint64_t vocab, const uint32_t* mask) {
    int32_t best_id = -1;
    float best = 0.0f;
    for (uint64_t i = 0; i < vocab; ++i) {
        if (!allowed(mask, i)) continue;
        if (best_id < 0) {
            best_id = (int32_t)i;
            best = x[i];
        } else if (x[i] > best) {
            best = x[i];
            best_id = (int32_t)i;
        }
    }
    return best_id;
}

/* per-thread scratch */
typedef struct {
    int32_t id;
    float logit;
    double prob;
} tc_t;

typedef struct {
    uint64_t vocab;
    float* x;        /* row as fp32, then adjusted in place */
    uint8_t* seen;   /* unique-history marker */
    tc_t* cands;
    float* ptarget;  /* dense verify */
} scratch_t;

static int scratch_init(scratch_t* s, uint64_t vocab) {
    s->vocab = vocab;
    s->x = (float*)malloc(vocab * sizeof(float));
    s->seen = (uint8_t*)calloc(vocab, 1);
    s->cands = (tc_t*)malloc(vocab * sizeof(tc_t));
    s->ptarget = (float*)malloc(vocab * sizeof(float));
    return s->x && s->seen && s->cands && s->ptarget;
}

static void scratch_free(scratch_t* s) {
    free(s->x);
    free(s->seen);
    free(s->cands);
    free(s->ptarget);
}

/* ordering: higher logit first; equal logits -> lower id first (core_execution.cpp:521-527) */
static inline int better(const tc_t* a, const tc_t* b) {
    if (a->logit != b->logit) return a->logit > b->logit;
    return a->id < b->id;
}

static int cmp_better(const void* A, const void* B) {
    const tc_t* a = (const tc_t*)A;
    const tc_t* b = (const tc_t*)B;
    if (better(a, b)) return -1;
    if (better(b, a)) return 1;
    return 0;
}

/* bounded heap whose root is the worst kept candidate */
static void heap_sift_down(tc_t* h, uint64_t n, uint64_t i) {
    for (;;) {
        uint64_t l = 2 * i + 1, r = l + 1, w = i;
        if (l < n && better(&h[w], &h[l])) w = l; /* h[l] is worse than h[w] */
        if (r < n && better(&h[w], &h[r])) w = r;
        if (w == i) return;
        tc_t t = h[i]; h[i] = h[w]; h[w] = t;
        i = w;
    }
}

static void heap_sift_up(tc_t* h, uint64_t i) {
    while (i > 0) {
        uint64_t p = (i - 1) / 2;
        if (better(&h[p], &h[i])) { /* child worse than parent -> move up */
            tc_t t = h[i]; h[i] = h[p]; h[p] = t;
            i = p;
        } else {
            return;
        }
    }
}

/*
 * Core of compute_sampling_candidates on the fp32 row s->x (modified in place). On success the
 * sorted candidates are in s->cands[0..*out_n) and *greedy_tok is -1, or (greedy shortcut) the
 * single token is in *greedy_tok.
 */
static int32_t candidates_core(scratch_t* s, uint64_t vocab, const sixi_smp_params* p,
                               const int32_t* hist, uint64_t n_hist, const uint32_t* mask,
                               uint64_t* out_n, int32_t* greedy_tok) {
    float* x = s->x;
    *greedy_tok = -1;
    *out_n = 0;
    uint64_t n_allowed = 0;
    for (uint64_t i = 0; i < vocab; ++i) {
        if (!allowed(mask, i)) continue;
        ++n_allowed;
        if (isnan(x[i]) || isinf(x[i])) return SIXI_NUMERIC_NAN_OR_INF;
    }
    if (n_allowed == 0) return SIXI_INVALID_ARGUMENT;

    const int apply_penalties = (p->mode != SIXI_SMP_STRICT_REPLAY) && n_hist > 0 &&
        (p->repetition_penalty != 1.0f || p->presence_penalty != 0.0f ||
         p->frequency_penalty != 0.0f);
    if (!apply_penalties && p->temperature <= 0.0f) {
        *greedy_tok = masked_argmax(x, vocab, mask);
        return SIXI_OK;
    }
    if (apply_penalties) {
        /* once per unique in-range allowed id (core_execution.cpp:477-491) */
        for (uint64_t j = 0; j < n_hist; ++j) {
            const int32_t t = hist[j];
            if (t < 0 || (uint64_t)t >= vocab || !allowed(mask, (uint64_t)t) || s->seen[t]) continue;
            s->seen[t] = 1;
            float v = x[t];
            if (p->repetition_penalty != 1.0f && p->repetition_penalty > 0.0f) {
                v = (v < 0.0f) ? (v * p->repetition_penalty) : (v / p->repetition_penalty);
            }
            v -= p->presence_penalty;
            x[t] = v;
        }
        for (uint64_t j = 0; j < n_hist; ++j) { /* reset the marker */
            const int32_t t = hist[j];
            if (t >= 0 && (uint64_t)t < vocab) s->seen[t] = 0;
        }
        if (p->frequency_penalty != 0.0f) { /* extension: once per occurrence */
            for (uint64_t j = 0; j < n_hist; ++j) {
                const int32_t t = hist[j];
                if (t < 0 || (uint64_t)t >= vocab || !allowed(mask, (uint64_t)t)) continue;
                x[t] -= p->frequency_penalty;
            }
        }
    }
    if (p->temperature <= 0.0f) {
        *greedy_tok = masked_argmax(x, vocab, mask);
        return SIXI_OK;
    }

    const uint64_t k = (p->top_k > 0 && (uint64_t)p->top_k < n_allowed) ? (uint64_t)p->top_k
                                                                         : n_allowed;
    tc_t* c = s->cands;
    uint64_t n = 0;
    if (k < n_allowed) {
        for (uint64_t i = 0; i < vocab; ++i) {
            if (!allowed(mask, i)) continue;
            const tc_t t = {(int32_t)i, x[i], 0.0};
            if (n < k) {
                c[n] = t;
                heap_sift_up(c, n);
                ++n;
            } else if (better(&t, &c[0])) {
                c[0] = t;
                heap_sift_down(c, n, 0);
            }
        }
    } else {
        for (uint64_t i = 0; i < vocab; ++i) {
            if (!allowed(mask, i)) continue;
            c[n].id = (int32_t)i;
            c[n].logit = x[i];
            c[n].prob = 0.0;
            ++n;
        }
    }
    qsort(c, n, sizeof(tc_t), cmp_better);

    /* temperature softmax over the k candidates in fp64 (core_execution.cpp:538-549) */
    const double inv_temp = 1.0 / (double)p->temperature;
    const double max_scaled = (double)c[0].logit * inv_temp;
    double sum_exp = 0.0;
    for (uint64_t i = 0; i < n; ++i) {
        c[i].prob = exp((double)c[i].logit * inv_temp - max_scaled);
        sum_exp += c[i].prob;
    }
    if (sum_exp > 0.0) {
        for (uint64_t i = 0; i < n; ++i) c[i].prob /= sum_exp;
    }
    /* top-p, crossing token kept, renormalised (core_execution.cpp:551-575) */
    if (p->top_p > 0.0f && p->top_p < 1.0f) {
        double cum = 0.0;
        uint64_t keep = 0;
        for (; keep < n; ++keep) {
            cum += c[keep].prob;
            if (cum >= (double)p->top_p) {
                ++keep;
                break;
            }
        }
        if (keep == 0) keep = 1;
        if (keep < n) {
            n = keep;
            double renorm = 0.0;
            for (uint64_t i = 0; i < n; ++i) renorm += c[i].prob;
            if (renorm > 0.0) {
                for (uint64_t i = 0; i < n; ++i) c[i].prob /= renorm;
            }
        }
    }
    /* extension: min-p relative to the most likely candidate */
    if (p->min_p > 0.0f) {
        const double thr = (double)p->min_p * c[0].prob;
        uint64_t keep = 1;
        while (keep < n && c[keep].prob >= thr) ++keep;
        if (keep < n) {
            n = keep;
            double renorm = 0.0;
            for (uint64_t i = 0; i < n; ++i) renorm += c[i].prob;
            if (renorm > 0.0) {
                for (uint64_t i = 0; i < n; ++i) c[i].prob /= renorm;
            }
        }
    }
    *out_n = n;
    return SIXI_OK;
}

/* sample_from_candidates with a supplied uniform (core_execution.cpp:586-601) */
static int32_t draw_cdf(const tc_t* c, uint64_t n, double u) {
    if (n == 0) return -1;
    double cdf = 0.0;
    for (uint64_t i = 0; i < n; ++i) {
        cdf += c[i].prob;
        if (u < cdf) return c[i].id;
    }
    return c[n - 1].id;
}

static int32_t sample_core(scratch_t* s, const void* row, uint32_t dtype, uint64_t vocab,
                           const sixi_smp_params* p, const int32_t* hist, uint64_t n_hist,
                           const uint32_t* mask, double u, int32_t* out_token) {
    load_row(row, dtype, vocab, s->x);
    uint64_t n = 0;
    int32_t g = -1;
    const int32_t st = candidates_core(s, vocab, p, hist, n_hist, mask, &n, &g);
    if (st != SIXI_OK) {
        *out_token = -1;
        return st;
    }
    if (g >= 0) {
        *out_token = g;
        return SIXI_OK;
    }
    /* temperature > 0 here (greedy rows took the shortcut) */
    *out_token = draw_cdf(s->cands, n, u);
    return SIXI_OK;
}

int32_t orc_greedy_row(const void* row, uint32_t dtype, uint64_t vocab, const uint32_t* mask,
                       int32_t* out_token) {
    float* x = (float*)malloc(vocab * sizeof(float));
    if (!x) return SIXI_BACKEND_ERROR;
    load_row(row, dtype, vocab, x);
    int32_t st = SIXI_OK;
    uint64_t n_allowed = 0;
    for (uint64_t i = 0; i < vocab; ++i) {
        if (!allowed(mask, i)) continue;
        ++n_allowed;
        if (isnan(x[i]) || isinf(x[i])) st = SIXI_NUMERIC_NAN_OR_INF;
    }
    if (n_allowed == 0) {
        *out_token = -1;
        free(x);
        return SIXI_INVALID_ARGUMENT;
    }
    *out_token = masked_argmax(x, vocab, mask);
    free(x);
    return st;
}

int32_t orc_candidates(const void* row, uint32_t dtype, uint64_t vocab, const sixi_smp_params* p,
                       const int32_t* hist, uint64_t n_hist, const uint32_t* mask, uint64_t cap,
                       int32_t* out_ids, double* out_probs, uint64_t* out_n) {
    scratch_t s;
    if (!scratch_init(&s, vocab)) return SIXI_BACKEND_ERROR;
    load_row(row, dtype, vocab, s.x);
    uint64_t n = 0;
    int32_t g = -1;
    const int32_t st = candidates_core(&s, vocab, p, hist, n_hist, mask, &n, &g);
    if (st == SIXI_OK) {
        if (g >= 0) {
            s.cands[0].id = g;
            s.cands[0].prob = 1.0;
            n = 1;
        }
        for (uint64_t i = 0; i < n && i < cap; ++i) {
            out_ids[i] = s.cands[i].id;
            out_probs[i] = s.cands[i].prob;
        }
    }
    *out_n = n;
    scratch_free(&s);
    return st;
}

int32_t orc_sample(const void* row, uint32_t dtype, uint64_t vocab, const sixi_smp_params* p,
                   const int32_t* hist, uint64_t n_hist, const uint32_t* mask, double u,
                   int32_t* out_token) {
    scratch_t s;
    if (!scratch_init(&s, vocab)) return SIXI_BACKEND_ERROR;
    const int32_t st = sample_core(&s, row, dtype, vocab, p, hist, n_hist, mask, u, out_token);
    scratch_free(&s);
    return st;
}

/* ------------------------------------------------------------------------------------------ */
/* simple static partition of [0, n) over threads */
typedef struct {
    void (*fn)(void* ctx, scratch_t* s, uint32_t i);
    void* ctx;
    uint32_t begin, end;
    uint64_t vocab;
} job_t;

static void* job_run(void* arg) {
    job_t* j = (job_t*)arg;
    scratch_t s;
    if (!scratch_init(&s, j->vocab)) return NULL;
    for (uint32_t i = j->begin; i < j->end; ++i) j->fn(j->ctx, &s, i);
    scratch_free(&s);
    return NULL;
}

static void parallel_for(uint32_t n, int32_t n_threads, uint64_t vocab,
                         void (*fn)(void*, scratch_t*, uint32_t), void* ctx) {
    if (n_threads <= 0) n_threads = (int32_t)sysconf(_SC_NPROCESSORS_ONLN);
    if (n_threads < 1) n_threads = 1;
    if ((uint32_t)n_threads > n) n_threads = (int32_t)(n ? n : 1);
    job_t* jobs = (job_t*)calloc((size_t)n_threads, sizeof(job_t));
    pthread_t* th = (pthread_t*)calloc((size_t)n_threads, sizeof(pthread_t));
    const uint32_t per = (n + (uint32_t)n_threads - 1) / (uint32_t)n_threads;
    for (int32_t t = 0; t < n_threads; ++t) {
        jobs[t].fn = fn;
        jobs[t].ctx = ctx;
        jobs[t].vocab = vocab;
        jobs[t].begin = (uint32_t)t * per < n ? (uint32_t)t * per : n;
        jobs[t].end = jobs[t].begin + per < n ? jobs[t].begin + per : n;
    }
    if (n_threads == 1) {
        job_run(&jobs[0]);
    } else {
        for (int32_t t = 0; t < n_threads; ++t) pthread_create(&th[t], NULL, job_run, &jobs[t]);
        for (int32_t t = 0; t < n_threads; ++t) pthread_join(th[t], NULL);
    }
    free(jobs);
    free(th);
}

typedef struct {
    const void* logits;
    uint32_t dtype;
    uint64_t row_stride, vocab;
    const sixi_smp_params* params;
    const uint32_t* masks;
    const int32_t* hist_tokens;
    const int64_t* hist_offsets;
    const double* uniforms;
    uint64_t step;
    int32_t* out_tokens;
    int32_t* out_status;
} batch_ctx_t;

static const uint32_t* row_mask(const uint32_t* masks, uint64_t vocab, const sixi_smp_params* p,
                                uint64_t r) {
    if (masks == NULL || !(p->flags & SIXI_SMP_ROW_MASKED)) return NULL;
    return masks + r * ((vocab + 31) / 32);
}

static void batch_row(void* vctx, scratch_t* s, uint32_t r) {
    batch_ctx_t* c = (batch_ctx_t*)vctx;
    const sixi_smp_params* p = &c->params[r];
    const size_t esz = c->dtype == SIXI_SMP_BF16 ? 2 : 4;
    const void* row = (const char*)c->logits + (size_t)r * c->row_stride * esz;
    const int32_t* hist = NULL;
    uint64_t nh = 0;
    if (c->hist_tokens && c->hist_offsets) {
        hist = c->hist_tokens + c->hist_offsets[r];
        nh = (uint64_t)(c->hist_offsets[r + 1] - c->hist_offsets[r]);
    }
    const double u = c->uniforms ? c->uniforms[r]
                                 : orc_philox_uniform(p->seed, p->counter + c->step, 0u);
    c->out_status[r] = sample_core(s, row, c->dtype, c->vocab, p, hist, nh,
                                   row_mask(c->masks, c->vocab, p, r), u, &c->out_tokens[r]);
}

int32_t orc_sample_batch(const void* logits, uint32_t dtype, uint32_t n_rows, uint64_t row_stride,
                         uint64_t vocab, const sixi_smp_params* params, const uint32_t* masks,
                         const int32_t* hist_tokens, const int64_t* hist_offsets,
                         const double* uniforms, uint64_t step, int32_t* out_tokens,
                         int32_t* out_status, int32_t n_threads) {
    batch_ctx_t c = {logits, dtype, row_stride, vocab, params, masks, hist_tokens, hist_offsets,
                     uniforms, step, out_tokens, out_status};
    parallel_for(n_rows, n_threads, vocab, batch_row, &c);
    return SIXI_OK;
}

/* ------------------------------------------------------------------------------------------ */
typedef struct {
    const void* target;
    uint32_t dtype;
    uint64_t row_stride, vocab;
    const float* q;
    const int32_t* drafts;
    const int32_t* n_drafts;
    uint32_t k;
    const sixi_smp_params* params;
    const uint32_t* masks;
    const int32_t* hist_tokens;
    const int64_t* hist_offsets;
    const double* uniforms;
    uint64_t step;
    int32_t *acc, *tok, *ntok, *frej, *used, *status;
} verify_ctx_t;

static void verify_stream(void* vctx, scratch_t* s, uint32_t st) {
    verify_ctx_t* c = (verify_ctx_t*)vctx;
    const sixi_smp_params* p = &c->params[st];
    const uint64_t V = c->vocab;
    const uint32_t k = c->k;
    const uint32_t nd = c->n_drafts ? (uint32_t)c->n_drafts[st] : k;
    const size_t esz = c->dtype == SIXI_SMP_BF16 ? 2 : 4;
    const int32_t* d = c->drafts + (size_t)st * k;
    int32_t* out = c->tok + (size_t)st * (k + 1);
    for (uint32_t i = 0; i <= k; ++i) out[i] = -1;
    uint32_t used = 0, acc = 0, n_out = 0;
    int32_t first_reject = -1, status = SIXI_OK;

#define ROW(i) ((const char*)c->target + ((size_t)st * (k + 1) + (i)) * c->row_stride * esz)
#define MASK(i) row_mask(c->masks, V, p, (uint64_t)st * (k + 1) + (i))
#define UNI(j) (c->uniforms ? c->uniforms[(size_t)st * (k + 1) + (j)] \
                            : orc_philox_uniform(p->seed, p->counter + c->step, (uint32_t)(j)))

    if (nd > k) {
        status = SIXI_INVALID_ARGUMENT;
        goto done;
    }
    if (p->temperature <= 0.0f) {
        /* greedy match: target argmax of the raw logits (speculative.cpp:801-822, 617-629) */
        for (uint32_t i = 0; i <= nd; ++i) {
            int32_t t = -1;
            const int32_t gs = orc_greedy_row(ROW(i), c->dtype, V, MASK(i), &t);
            if (gs == SIXI_INVALID_ARGUMENT) {
                status = gs;
                goto done;
            }
            if (gs != SIXI_OK && status == SIXI_OK) status = gs;
            if (i == nd) {
                out[n_out++] = t; /* bonus */
                break;
            }
            if (d[i] == t) {
                out[n_out++] = d[i];
                ++acc;
            } else {
                out[n_out++] = t;
                first_reject = (int32_t)i;
                break;
            }
        }
        goto done;
    }

    /* stochastic: history = base + accepted drafts */
    const int32_t* base = NULL;
    uint64_t nb = 0;
    if (c->hist_tokens && c->hist_offsets) {
        base = c->hist_tokens + c->hist_offsets[st];
        nb = (uint64_t)(c->hist_offsets[st + 1] - c->hist_offsets[st]);
    }
    int32_t* hist = (int32_t*)malloc((nb + k + 1) * sizeof(int32_t));
    if (nb) memcpy(hist, base, nb * sizeof(int32_t));
    uint64_t nh = nb;
    int rejected = 0;
    for (uint32_t i = 0; i < nd; ++i) {
        load_row(ROW(i), c->dtype, V, s->x);
        uint64_t n = 0;
        int32_t g = -1;
        const int32_t cs = candidates_core(s, V, p, hist, nh, MASK(i), &n, &g);
        if (cs != SIXI_OK) {
            status = cs;
            free(hist);
            goto done;
        }
        const int32_t di = d[i];
        const int in_range = di >= 0 && (uint64_t)di < V;
        if (c->q) {
            /* dense draft probabilities (speculative.cpp:823-903) */
            const float* q = c->q + ((size_t)st * k + i) * c->row_stride;
            for (uint64_t x = 0; x < V; ++x) s->ptarget[x] = 0.0f;
            for (uint64_t j = 0; j < n; ++j) s->ptarget[s->cands[j].id] = (float)s->cands[j].prob;
            const float p_d = in_range ? s->ptarget[di] : 0.0f;
            const float q_d = in_range ? q[di] : 1.0f;
            const double accept_prob =
                (q_d <= 0.0f) ? (p_d > 0.0f ? 1.0 : 0.0)
                              : fmin(1.0, (double)p_d / fmax(1e-12, (double)q_d));
            const double r = UNI(used);
            ++used;
            if (r < accept_prob) {
                out[n_out++] = di;
                ++acc;
                hist[nh++] = di;
                continue;
            }
            first_reject = (int32_t)i;
            double res_sum = 0.0;
            for (uint64_t x = 0; x < V; ++x) {
                const double diff = fmax(0.0, (double)s->ptarget[x] - (double)q[x]);
                res_sum += diff;
            }
            const double u = UNI(used);
            ++used;
            int32_t repl = 0;
            if (res_sum > 1e-12) {
                double cdf = 0.0;
                repl = (int32_t)(V - 1);
                for (uint64_t x = 0; x < V; ++x) {
                    const double diff = fmax(0.0, (double)s->ptarget[x] - (double)q[x]);
                    cdf += diff / res_sum;
                    if (u < cdf) {
                        repl = (int32_t)x;
                        break;
                    }
                }
            } else {
                double cdf = 0.0;
                repl = (int32_t)(V - 1);
                for (uint64_t x = 0; x < V; ++x) {
                    cdf += (double)s->ptarget[x];
                    if (u < cdf) {
                        repl = (int32_t)x;
                        break;
                    }
                }
            }
            out[n_out++] = repl;
            rejected = 1;
            break;
        } else {
            /* one-hot drafts (speculative.cpp:630-681) */
            double p_d = 0.0;
            for (uint64_t j = 0; j < n; ++j) {
                if (s->cands[j].id == di) {
                    p_d = s->cands[j].prob;
                    break;
                }
            }
            const double r = UNI(used);
            ++used;
            if (r < p_d) {
                out[n_out++] = di;
                ++acc;
                hist[nh++] = di;
                continue;
            }
            first_reject = (int32_t)i;
            double res_sum = 0.0;
            uint64_t m = 0;
            for (uint64_t j = 0; j < n; ++j) {
                if (s->cands[j].id != di) {
                    ++m;
                    res_sum += s->cands[j].prob;
                }
            }
            const double u = UNI(used);
            ++used;
            int32_t repl;
            if (m > 0 && res_sum > 0.0) {
                uint64_t w = 0;
                for (uint64_t j = 0; j < n; ++j) {
                    if (s->cands[j].id != di) s->cands[w++] = s->cands[j];
                }
                for (uint64_t j = 0; j < m; ++j) s->cands[j].prob /= res_sum;
                repl = draw_cdf(s->cands, m, u);
            } else {
                /* residual empty: draw from the full candidate list */
                repl = draw_cdf(s->cands, n, u);
            }
            out[n_out++] = repl;
            rejected = 1;
            break;
        }
    }
    if (!rejected) {
        /* bonus: dense q uses the pre-step history (speculative.cpp:908-915), one-hot the full
         * history (speculative.cpp:683-691) */
        const uint64_t nbonus = c->q ? nb : nh;
        int32_t t = -1;
        const double u = UNI(used);
        ++used;
        const int32_t bs = sample_core(s, ROW(nd), c->dtype, V, p, hist, nbonus, MASK(nd), u, &t);
        if (bs != SIXI_OK) {
            status = bs;
            free(hist);
            goto done;
        }
        out[n_out++] = t;
    }
    free(hist);

done:
    if (status != SIXI_OK && status != SIXI_NUMERIC_NAN_OR_INF) {
        for (uint32_t i = 0; i <= k; ++i) out[i] = -1;
        n_out = 0;
        acc = 0;
        first_reject = -1;
    }
    c->acc[st] = (int32_t)acc;
    c->ntok[st] = (int32_t)n_out;
    c->frej[st] = first_reject;
    c->used[st] = (int32_t)used;
    c->status[st] = status;
#undef ROW
#undef MASK
#undef UNI
}

int32_t orc_verify(const void* target, uint32_t dtype, uint64_t row_stride, uint64_t vocab,
                   const float* draft_probs, const int32_t* drafts, const int32_t* n_drafts,
                   uint32_t n_streams, uint32_t k, const sixi_smp_params* params,
                   const uint32_t* masks, const int32_t* hist_tokens, const int64_t* hist_offsets,
                   const double* uniforms, uint64_t step, int32_t* out_accepted,
                   int32_t* out_tokens, int32_t* out_n_tokens, int32_t* out_first_reject,
                   int32_t* out_uniforms_used, int32_t* out_status, int32_t n_threads) {
    verify_ctx_t c = {target, dtype, row_stride, vocab, draft_probs, drafts, n_drafts, k, params,
                      masks, hist_tokens, hist_offsets, uniforms, step, out_accepted, out_tokens,
                      out_n_tokens, out_first_reject, out_uniforms_used, out_status};
    parallel_for(n_streams, n_threads, vocab, verify_stream, &c);
    return SIXI_OK;
}
