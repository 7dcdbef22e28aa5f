/* TEST INFRASTRUCTURE ONLY: CPU restatement of the JSON-object grammar automaton that produces
 * the per-row allowed-token masks (include/sixi_json.h). Parity checker for the device producer
 * (tests/, __graft_entry__.smoke(), bench.py's CPU-baseline leg); the product never calls it.
 *
 * The engine's own automaton for `response_format: {"type": "json_object"}` (docs/API.md:45-76 in
 * the engine) is binary-only, so this is written from the grammar: RFC 8259 JSON text whose top
 * level is one object, strings in RFC 3629 UTF-8 without raw control characters, nesting at most
 * SIXI_JSON_MAX_DEPTH containers, and the end-of-sequence token only after the closing brace. It
 * is pinned against Python's json module (an independent RFC 8259 parser) by tests/test_json.py.
 *
 * The walk keeps an explicit stack of container kinds and re-reads the byte that ends a number in
 * the enclosing context; states are exchanged in the sixi_json_state layout so that the device
 * states can be compared field by field.
 */
#include <pthread.h>
#include <stdint.h>
#include <string.h>

#include "sixi_json_oracle.h"

typedef struct {
    int mode, aux, pos, rem, rng, depth;
    unsigned char obj[SIXI_JSON_MAX_DEPTH]; /* 1 object, 0 array */
} walker;

static void from_state(const sixi_json_state* s, walker* w) {
    w->mode = s->mode;
    w->aux = s->aux;
    w->pos = s->pos;
    w->rem = s->utf8 & 3;
    w->rng = s->utf8 >> 2;
    w->depth = s->depth;
    for (int d = 0; d < (int)SIXI_JSON_MAX_DEPTH; ++d) w->obj[d] = (unsigned char)((s->stack[d / 32] >> (d % 32)) & 1u);
}

static void to_state(const walker* w, int failed, sixi_json_state* s) {
    memset(s, 0, sizeof(*s));
    s->mode = (uint8_t)w->mode;
    s->aux = (uint8_t)w->aux;
    s->pos = (uint8_t)w->pos;
    s->utf8 = (uint8_t)(w->rem | (w->rng << 2));
    s->depth = (uint16_t)w->depth;
    s->failed = (uint8_t)failed;
    /* bits above the depth are whatever the last push at that level left; keep them as pushed */
    for (int d = 0; d < (int)SIXI_JSON_MAX_DEPTH; ++d)
        if (w->obj[d]) s->stack[d / 32] |= 1u << (d % 32);
}

static int ws(unsigned c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r'; }
static int digit(unsigned c) { return c >= '0' && c <= '9'; }
static int hexd(unsigned c) { return digit(c) || (c >= 'a' && c <= 'f') || (c >= 'A' && c <= 'F'); }

static const char* const LIT[3] = {"true", "false", "null"};

static int open_container(walker* w, int is_obj) {
    if (w->depth >= (int)SIXI_JSON_MAX_DEPTH) return 0;
    w->obj[w->depth++] = (unsigned char)is_obj;
    w->mode = is_obj ? SIXI_JSON_OBJ_FIRST : SIXI_JSON_ARR_FIRST;
    return 1;
}

static void close_container(walker* w) {
    --w->depth;
    w->mode = w->depth == 0 ? SIXI_JSON_DONE : SIXI_JSON_AFTER;
}

static int begin_value(walker* w, unsigned c) {
    switch (c) {
        case '"': w->mode = SIXI_JSON_STRING; w->aux = 0; w->rem = 0; w->rng = 0; return 1;
        case '{': return open_container(w, 1);
        case '[': return open_container(w, 0);
        case '-': w->mode = SIXI_JSON_NEG; return 1;
        case '0': w->mode = SIXI_JSON_ZERO; return 1;
        case 't': w->mode = SIXI_JSON_LITERAL; w->aux = 0; w->pos = 1; return 1;
        case 'f': w->mode = SIXI_JSON_LITERAL; w->aux = 1; w->pos = 1; return 1;
        case 'n': w->mode = SIXI_JSON_LITERAL; w->aux = 2; w->pos = 1; return 1;
        default:
            if (c >= '1' && c <= '9') { w->mode = SIXI_JSON_INT; return 1; }
            return 0;
    }
}

/* RFC 3629 table: the allowed range of the first continuation byte after each lead byte */
static int utf8_lead(walker* w, unsigned c) {
    if (c >= 0xC2 && c <= 0xDF) { w->rem = 1; w->rng = 0; return 1; }
    if (c == 0xE0) { w->rem = 2; w->rng = 1; return 1; }
    if ((c >= 0xE1 && c <= 0xEC) || c == 0xEE || c == 0xEF) { w->rem = 2; w->rng = 0; return 1; }
    if (c == 0xED) { w->rem = 2; w->rng = 2; return 1; }
    if (c == 0xF0) { w->rem = 3; w->rng = 3; return 1; }
    if (c >= 0xF1 && c <= 0xF3) { w->rem = 3; w->rng = 0; return 1; }
    if (c == 0xF4) { w->rem = 3; w->rng = 4; return 1; }
    return 0;
}

static int utf8_cont(walker* w, unsigned c) {
    static const unsigned lo[5] = {0x80, 0xA0, 0x80, 0x90, 0x80};
    static const unsigned hi[5] = {0xBF, 0xBF, 0x9F, 0xBF, 0x8F};
    if (c < lo[w->rng] || c > hi[w->rng]) return 0;
    w->rem -= 1;
    w->rng = 0;
    return 1;
}

static int feed(walker* w, unsigned c) {
    switch (w->mode) {
        case SIXI_JSON_START:
            if (ws(c)) return 1;
            return c == '{' && open_container(w, 1);
        case SIXI_JSON_OBJ_FIRST:
        case SIXI_JSON_OBJ_KEY:
            if (ws(c)) return 1;
            if (c == '"') { w->mode = SIXI_JSON_STRING; w->aux = 1; w->rem = 0; w->rng = 0; return 1; }
            if (c == '}' && w->mode == SIXI_JSON_OBJ_FIRST) { close_container(w); return 1; }
            return 0;
        case SIXI_JSON_COLON:
            if (ws(c)) return 1;
            if (c == ':') { w->mode = SIXI_JSON_VALUE; return 1; }
            return 0;
        case SIXI_JSON_VALUE:
        case SIXI_JSON_ARR_FIRST:
            if (ws(c)) return 1;
            if (c == ']' && w->mode == SIXI_JSON_ARR_FIRST) { close_container(w); return 1; }
            return begin_value(w, c);
        case SIXI_JSON_AFTER: {
            if (ws(c)) return 1;
            const int in_obj = w->obj[w->depth - 1];
            if (c == ',') { w->mode = in_obj ? SIXI_JSON_OBJ_KEY : SIXI_JSON_VALUE; return 1; }
            if (c == (in_obj ? '}' : ']')) { close_container(w); return 1; }
            return 0;
        }
        case SIXI_JSON_DONE:
            return 0;
        case SIXI_JSON_STRING:
            if (w->rem > 0) return utf8_cont(w, c);
            if (c == '"') { w->mode = w->aux ? SIXI_JSON_COLON : SIXI_JSON_AFTER; return 1; }
            if (c == '\\') { w->mode = SIXI_JSON_ESCAPE; return 1; }
            if (c < 0x20) return 0;
            if (c < 0x80) return 1;
            return utf8_lead(w, c);
        case SIXI_JSON_ESCAPE:
            if (c == 'u') { w->mode = SIXI_JSON_HEX; w->pos = 4; return 1; }
            if (strchr("\"\\/bfnrt", (int)c) && c != 0) { w->mode = SIXI_JSON_STRING; return 1; }
            return 0;
        case SIXI_JSON_HEX:
            if (!hexd(c)) return 0;
            if (--w->pos == 0) w->mode = SIXI_JSON_STRING;
            return 1;
        case SIXI_JSON_NEG:
            if (c == '0') { w->mode = SIXI_JSON_ZERO; return 1; }
            if (c >= '1' && c <= '9') { w->mode = SIXI_JSON_INT; return 1; }
            return 0;
        case SIXI_JSON_ZERO:
        case SIXI_JSON_INT:
        case SIXI_JSON_FRAC:
        case SIXI_JSON_EXP_DIGITS:
            if (digit(c) && w->mode != SIXI_JSON_ZERO) return 1;
            if (c == '.' && (w->mode == SIXI_JSON_ZERO || w->mode == SIXI_JSON_INT)) { w->mode = SIXI_JSON_DOT; return 1; }
            if ((c == 'e' || c == 'E') && w->mode != SIXI_JSON_EXP_DIGITS) { w->mode = SIXI_JSON_EXP; return 1; }
            /* the number is complete: this byte belongs to the enclosing container */
            w->mode = SIXI_JSON_AFTER;
            return feed(w, c);
        case SIXI_JSON_DOT:
            if (!digit(c)) return 0;
            w->mode = SIXI_JSON_FRAC;
            return 1;
        case SIXI_JSON_EXP:
            if (c == '+' || c == '-') { w->mode = SIXI_JSON_EXP_SIGN; return 1; }
            if (!digit(c)) return 0;
            w->mode = SIXI_JSON_EXP_DIGITS;
            return 1;
        case SIXI_JSON_EXP_SIGN:
            if (!digit(c)) return 0;
            w->mode = SIXI_JSON_EXP_DIGITS;
            return 1;
        case SIXI_JSON_LITERAL:
            if (c != (unsigned char)LIT[w->aux][w->pos]) return 0;
            if (LIT[w->aux][++w->pos] == '\0') w->mode = SIXI_JSON_AFTER;
            return 1;
        default:
            return 0;
    }
}

/* Feeds n bytes to *st; 1 (state advanced) or 0 (refused, state unchanged). */
int orc_json_feed(sixi_json_state* st, const uint8_t* p, uint64_t n) {
    if (st->failed) return 0;
    walker w;
    from_state(st, &w);
    for (uint64_t i = 0; i < n; ++i)
        if (!feed(&w, p[i])) return 0;
    to_state(&w, 0, st);
    return 1;
}

/* 1 when the token may follow the state (the token's text, or end-of-sequence / a control token) */
static int token_ok(const sixi_json_state* st, const uint8_t* p, uint64_t n, int is_eos, int is_special) {
    if (st->failed) return 0;
    if (is_eos) return st->mode == SIXI_JSON_DONE;
    if (is_special || n == 0) return 0;
    sixi_json_state t = *st;
    return orc_json_feed(&t, p, n);
}

typedef struct {
    const uint8_t* bytes;
    const uint64_t* offs;
    const uint8_t* flags;
    uint32_t vocab;
    int32_t eos;
    const sixi_json_state* states;
    uint32_t n_rows;
    uint32_t* masks;
    uint64_t stride;
    uint32_t r0, r1;
} mask_job;

static void* mask_rows(void* arg) {
    const mask_job* j = (const mask_job*)arg;
    const uint32_t words = (j->vocab + 31) / 32;
    for (uint32_t r = j->r0; r < j->r1; ++r) {
        uint32_t* m = j->masks + (uint64_t)r * j->stride;
        memset(m, 0, sizeof(uint32_t) * words);
        for (uint32_t i = 0; i < j->vocab; ++i) {
            const int sp = j->flags ? (j->flags[i] & SIXI_JSON_TOKEN_SPECIAL) != 0 : 0;
            if (token_ok(&j->states[r], j->bytes + j->offs[i], j->offs[i + 1] - j->offs[i], (int32_t)i == j->eos, sp))
                m[i / 32] |= 1u << (i % 32);
        }
    }
    return 0;
}

/* The allowed-token masks of n_rows states (rows spread over n_threads threads, 0 = 1). */
void orc_json_fill_masks(const uint8_t* bytes, const uint64_t* offs, const uint8_t* flags, uint32_t vocab,
                         int32_t eos, const sixi_json_state* states, uint32_t n_rows, uint32_t* masks,
                         uint64_t stride, int n_threads) {
    if (n_threads < 1) n_threads = 1;
    if ((uint32_t)n_threads > n_rows) n_threads = (int)(n_rows ? n_rows : 1);
    pthread_t th[256];
    mask_job jobs[256];
    if (n_threads > 256) n_threads = 256;
    for (int t = 0; t < n_threads; ++t) {
        mask_job j = {bytes, offs, flags, vocab, eos, states, n_rows, masks, stride,
                      (uint32_t)((uint64_t)n_rows * t / n_threads), (uint32_t)((uint64_t)n_rows * (t + 1) / n_threads)};
        jobs[t] = j;
    }
    int joined[256] = {0};
    for (int t = 1; t < n_threads; ++t) {
        if (pthread_create(&th[t], 0, mask_rows, &jobs[t]) == 0)
            joined[t] = 1;
        else
            mask_rows(&jobs[t]);
    }
    mask_rows(&jobs[0]);
    for (int t = 1; t < n_threads; ++t)
        if (joined[t]) pthread_join(th[t], 0);
}

/* Applies tokens[r * stride + j], j < n_tokens[r] (NULL: 1), to each row; status per row as the
 * device producer reports it (0 ok, 1 refused: the row keeps its state and is marked failed). */
void orc_json_advance(const uint8_t* bytes, const uint64_t* offs, const uint8_t* flags, uint32_t vocab, int32_t eos,
                      sixi_json_state* states, uint32_t n_rows, const int32_t* tokens, uint64_t stride,
                      const int32_t* n_tokens, int32_t* status) {
    for (uint32_t r = 0; r < n_rows; ++r) {
        sixi_json_state* st = &states[r];
        int ok = !st->failed;
        sixi_json_state cur = *st;
        const int32_t n = n_tokens ? n_tokens[r] : 1;
        for (int32_t j = 0; ok && j < n; ++j) {
            const int32_t id = tokens[(uint64_t)r * stride + (uint64_t)j];
            if (id < 0 || (uint32_t)id >= vocab) { ok = 0; break; }
            const int sp = flags ? (flags[id] & SIXI_JSON_TOKEN_SPECIAL) != 0 : 0;
            const uint64_t len = offs[id + 1] - offs[id];
            if (!token_ok(&cur, bytes + offs[id], len, id == eos, sp)) { ok = 0; break; }
            if (id != eos) orc_json_feed(&cur, bytes + offs[id], len);
        }
        if (!st->failed) {
            cur.failed = (uint8_t)(ok ? 0 : 1);
            *st = cur;
        }
        if (status) status[r] = ok ? SIXI_OK : SIXI_INVALID_ARGUMENT;
    }
}

/* out[s * (k + 1) + j]: states[s] after drafts[s * k + 0 .. j - 1]; after a refused draft the later
 * rows repeat the last accepted state. */
void orc_json_expand(const uint8_t* bytes, const uint64_t* offs, const uint8_t* flags, uint32_t vocab, int32_t eos,
                     const sixi_json_state* states, uint32_t n_streams, const int32_t* drafts, uint32_t k,
                     const int32_t* n_drafts, sixi_json_state* out) {
    for (uint32_t s = 0; s < n_streams; ++s) {
        sixi_json_state cur = states[s];
        sixi_json_state* o = out + (uint64_t)s * (k + 1);
        o[0] = cur;
        int valid = !cur.failed;
        uint32_t nd = n_drafts ? (uint32_t)(n_drafts[s] < 0 ? 0 : n_drafts[s]) : k;
        if (nd > k) nd = k;
        for (uint32_t j = 0; j < k; ++j) {
            if (valid && j < nd) {
                const int32_t id = drafts[(uint64_t)s * k + j];
                int sp = 0;
                uint64_t len = 0;
                if (id >= 0 && (uint32_t)id < vocab) {
                    sp = flags ? (flags[id] & SIXI_JSON_TOKEN_SPECIAL) != 0 : 0;
                    len = offs[id + 1] - offs[id];
                }
                if (id >= 0 && (uint32_t)id < vocab && token_ok(&cur, bytes + offs[id], len, id == eos, sp)) {
                    if (id != eos) orc_json_feed(&cur, bytes + offs[id], len);
                } else {
                    valid = 0;
                }
            }
            o[j + 1] = cur;
        }
    }
}
