// smp_json.cu - device-side grammar-mask producer for JSON-object answers (include/sixi_json.h).
//
// The engine constrains `response_format: {"type": "json_object"}` answers to tokens that keep the
// text a prefix of one JSON object (docs/API.md:45-76 in the engine); its automaton is binary-only.
// This is a byte-level pushdown automaton for RFC 8259 JSON with a top-level object, run on the
// device for every (row, token) pair:
//   json_ctx_kernel      at upload, one thread per token and 32 contexts: the token's verdict in
//                        each context (a class of states, see "Contexts"), giving one mask row per
//                        context and a short list of tokens whose verdict the context leaves open.
//   json_mask_kernel     per row: a copy of its context's mask row, then the open tokens walked
//                        through a register copy of the row's state (rows without a context walk
//                        every token); blocks stage their words in shared memory.
//   json_advance_kernel  one thread per row: applies the sampled (or committed) tokens.
//   json_expand_kernel   one thread per stream: the per-draft states of a speculative step.
// The vocabulary is uploaded once: the first 16 bytes of every token inline (one 16-byte load per
// token and row, served from L2 after the first row), longer tails in a byte array, and a 32-bit
// word of length and flags.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <initializer_list>
#include <new>
#include <vector>

#include "../../include/sixi_json.h"

namespace {

// Meta of a token: x = length in bytes; y = flags (bits 0..7), first byte (bits 8..15), first
// byte that is not JSON whitespace (bits 16..23), count of '{' and '[' bytes (bits 24..31, capped).
constexpr uint32_t kTokSpecial = 1u << 0;
constexpr uint32_t kTokEos = 1u << 1;
constexpr uint32_t kTokPlain = 1u << 2;  // clean string state -> same clean string state
constexpr uint32_t kTokAllWs = 1u << 3;  // only whitespace
constexpr uint64_t kMaxTokenBytes = 0xFFFFFFFFull;

constexpr uint32_t M_START = SIXI_JSON_START, M_OBJ_FIRST = SIXI_JSON_OBJ_FIRST, M_OBJ_KEY = SIXI_JSON_OBJ_KEY,
                   M_COLON = SIXI_JSON_COLON, M_VALUE = SIXI_JSON_VALUE, M_ARR_FIRST = SIXI_JSON_ARR_FIRST,
                   M_AFTER = SIXI_JSON_AFTER, M_DONE = SIXI_JSON_DONE, M_STR = SIXI_JSON_STRING,
                   M_ESC = SIXI_JSON_ESCAPE, M_HEX = SIXI_JSON_HEX, M_NEG = SIXI_JSON_NEG, M_ZERO = SIXI_JSON_ZERO,
                   M_INT = SIXI_JSON_INT, M_DOT = SIXI_JSON_DOT, M_FRAC = SIXI_JSON_FRAC, M_EXP = SIXI_JSON_EXP,
                   M_EXPS = SIXI_JSON_EXP_SIGN, M_EXPD = SIXI_JSON_EXP_DIGITS, M_LIT = SIXI_JSON_LITERAL;

static_assert(sizeof(sixi_json_state) == 32, "state layout");

// The automaton state in registers. The container stack is four words indexed with selects, so
// that it never spills to local memory.
struct JS {
    uint32_t mode, aux, pos, utf8, depth;
    uint32_t s0, s1, s2, s3;
};

__host__ __device__ inline JS js_load(const sixi_json_state& t) {
    JS s;
    s.mode = t.mode;
    s.aux = t.aux;
    s.pos = t.pos;
    s.utf8 = t.utf8;
    s.depth = t.depth;
    s.s0 = t.stack[0];
    s.s1 = t.stack[1];
    s.s2 = t.stack[2];
    s.s3 = t.stack[3];
    return s;
}

__host__ __device__ inline void js_store(const JS& s, uint32_t failed, sixi_json_state& t) {
    t.mode = static_cast<uint8_t>(s.mode);
    t.aux = static_cast<uint8_t>(s.aux);
    t.pos = static_cast<uint8_t>(s.pos);
    t.utf8 = static_cast<uint8_t>(s.utf8);
    t.depth = static_cast<uint16_t>(s.depth);
    t.failed = static_cast<uint8_t>(failed);
    t.reserved0 = 0;
    t.stack[0] = s.s0;
    t.stack[1] = s.s1;
    t.stack[2] = s.s2;
    t.stack[3] = s.s3;
    t.reserved1[0] = 0;
    t.reserved1[1] = 0;
}

// 1 when the innermost open container is an object (depth > 0)
__host__ __device__ inline uint32_t js_top_is_obj(const JS& s) {
    const uint32_t d = s.depth - 1u;
    const uint32_t w = d < 64u ? (d < 32u ? s.s0 : s.s1) : (d < 96u ? s.s2 : s.s3);
    return (w >> (d & 31u)) & 1u;
}

__host__ __device__ inline bool js_push(JS& s, uint32_t is_obj, uint32_t next_mode) {
    if (s.depth >= SIXI_JSON_MAX_DEPTH) return false;
    const uint32_t d = s.depth, m = 1u << (d & 31u), q = d >> 5;
    const uint32_t set = is_obj ? m : 0u;
    if (q == 0u) s.s0 = (s.s0 & ~m) | set;
    if (q == 1u) s.s1 = (s.s1 & ~m) | set;
    if (q == 2u) s.s2 = (s.s2 & ~m) | set;
    if (q == 3u) s.s3 = (s.s3 & ~m) | set;
    s.depth = d + 1u;
    s.mode = next_mode;
    return true;
}

__host__ __device__ inline void js_pop(JS& s) {
    s.depth -= 1u;
    s.mode = s.depth == 0u ? M_DONE : M_AFTER;
}

__host__ __device__ inline bool is_ws(uint32_t c) { return c == 0x20u || c == 0x09u || c == 0x0Au || c == 0x0Du; }
__host__ __device__ inline bool is_digit(uint32_t c) { return c - 0x30u < 10u; }
__host__ __device__ inline bool is_hex(uint32_t c) {
    return c - 0x30u < 10u || (c | 0x20u) - 0x61u < 6u;
}

// character `pos` of literal `which` (0 "true", 1 "false", 2 "null"); 0 past its end
__host__ __device__ inline uint32_t lit_char(uint32_t which, uint32_t pos) {
    const uint64_t packed = which == 0u ? 0x65757274ull : (which == 1u ? 0x65736c6166ull : 0x6c6c756eull);
    return pos < 8u ? static_cast<uint32_t>(packed >> (8u * pos)) & 0xFFu : 0u;
}
__host__ __device__ inline uint32_t lit_len(uint32_t which) { return which == 1u ? 5u : 4u; }

// first byte of a value (modes VALUE and ARR_FIRST)
__host__ __device__ inline bool js_value_start(JS& s, uint32_t c) {
    if (c == 0x22u) {  // "
        s.mode = M_STR;
        s.aux = 0u;
        s.utf8 = 0u;
        return true;
    }
    if (c == 0x7Bu) return js_push(s, 1u, M_OBJ_FIRST);  // {
    if (c == 0x5Bu) return js_push(s, 0u, M_ARR_FIRST);  // [
    if (c == 0x2Du) {                                    // -
        s.mode = M_NEG;
        return true;
    }
    if (c == 0x30u) {
        s.mode = M_ZERO;
        return true;
    }
    if (c - 0x31u < 9u) {
        s.mode = M_INT;
        return true;
    }
    const uint32_t which = c == 0x74u ? 0u : (c == 0x66u ? 1u : (c == 0x6Eu ? 2u : 3u));  // t f n
    if (which < 3u) {
        s.mode = M_LIT;
        s.aux = which;
        s.pos = 1u;
        return true;
    }
    return false;
}

// Feeds one byte; false when the byte cannot continue the text (the state is then meaningless).
__host__ __device__ inline bool js_byte(JS& s, uint32_t c) {
    // a number ends at the first byte that cannot continue it; that byte is then read in AFTER
    if (s.mode == M_ZERO || s.mode == M_INT || s.mode == M_FRAC || s.mode == M_EXPD) {
        const bool digit = is_digit(c);
        const bool e = (c | 0x20u) == 0x65u;
        if (s.mode == M_ZERO) {
            if (c == 0x2Eu) { s.mode = M_DOT; return true; }
            if (e) { s.mode = M_EXP; return true; }
        } else if (s.mode == M_INT) {
            if (digit) return true;
            if (c == 0x2Eu) { s.mode = M_DOT; return true; }
            if (e) { s.mode = M_EXP; return true; }
        } else if (s.mode == M_FRAC) {
            if (digit) return true;
            if (e) { s.mode = M_EXP; return true; }
        } else if (digit) {
            return true;
        }
        s.mode = M_AFTER;
    }
    switch (s.mode) {
        case M_START:
            if (is_ws(c)) return true;
            return c == 0x7Bu && js_push(s, 1u, M_OBJ_FIRST);
        case M_OBJ_FIRST:
            if (c == 0x7Du) {  // }
                js_pop(s);
                return true;
            }
            [[fallthrough]];  // whitespace or a key
        case M_OBJ_KEY:
            if (is_ws(c)) return true;
            if (c == 0x22u) {
                s.mode = M_STR;
                s.aux = 1u;
                s.utf8 = 0u;
                return true;
            }
            return false;
        case M_COLON:
            if (is_ws(c)) return true;
            if (c == 0x3Au) {
                s.mode = M_VALUE;
                return true;
            }
            return false;
        case M_ARR_FIRST:
            if (c == 0x5Du) {  // ]
                js_pop(s);
                return true;
            }
            [[fallthrough]];  // whitespace or a value
        case M_VALUE:
            if (is_ws(c)) return true;
            return js_value_start(s, c);
        case M_AFTER: {
            if (is_ws(c)) return true;
            const uint32_t obj = js_top_is_obj(s);
            if (c == 0x2Cu) {  // ,
                s.mode = obj ? M_OBJ_KEY : M_VALUE;
                return true;
            }
            if ((obj && c == 0x7Du) || (!obj && c == 0x5Du)) {
                js_pop(s);
                return true;
            }
            return false;
        }
        case M_STR: {
            const uint32_t rem = s.utf8 & 3u;
            if (rem != 0u) {
                const uint32_t r = s.utf8 >> 2;
                const uint32_t lo = r == 1u ? 0xA0u : (r == 3u ? 0x90u : 0x80u);
                const uint32_t hi = r == 2u ? 0x9Fu : (r == 4u ? 0x8Fu : 0xBFu);
                if (c < lo || c > hi) return false;
                s.utf8 = rem - 1u;
                return true;
            }
            if (c == 0x22u) {
                s.mode = s.aux ? M_COLON : M_AFTER;
                return true;
            }
            if (c == 0x5Cu) {
                s.mode = M_ESC;
                return true;
            }
            if (c < 0x20u) return false;
            if (c < 0x80u) return true;
            if (c < 0xC2u || c > 0xF4u) return false;
            if (c < 0xE0u) {
                s.utf8 = 1u;
            } else if (c < 0xF0u) {
                s.utf8 = 2u | ((c == 0xE0u ? 1u : (c == 0xEDu ? 2u : 0u)) << 2);
            } else {
                s.utf8 = 3u | ((c == 0xF0u ? 3u : (c == 0xF4u ? 4u : 0u)) << 2);
            }
            return true;
        }
        case M_ESC:
            if (c == 0x75u) {  // u
                s.mode = M_HEX;
                s.pos = 4u;
                return true;
            }
            if (c == 0x22u || c == 0x5Cu || c == 0x2Fu || c == 0x62u || c == 0x66u || c == 0x6Eu || c == 0x72u ||
                c == 0x74u) {
                s.mode = M_STR;
                return true;
            }
            return false;
        case M_HEX:
            if (!is_hex(c)) return false;
            s.pos -= 1u;
            if (s.pos == 0u) s.mode = M_STR;
            return true;
        case M_NEG:
            if (c == 0x30u) {
                s.mode = M_ZERO;
                return true;
            }
            if (c - 0x31u < 9u) {
                s.mode = M_INT;
                return true;
            }
            return false;
        case M_DOT:
            if (!is_digit(c)) return false;
            s.mode = M_FRAC;
            return true;
        case M_EXP:
            if (c == 0x2Bu || c == 0x2Du) {
                s.mode = M_EXPS;
                return true;
            }
            if (!is_digit(c)) return false;
            s.mode = M_EXPD;
            return true;
        case M_EXPS:
            if (!is_digit(c)) return false;
            s.mode = M_EXPD;
            return true;
        case M_LIT:
            if (c != lit_char(s.aux, s.pos)) return false;
            s.pos += 1u;
            if (s.pos == lit_len(s.aux)) s.mode = M_AFTER;
            return true;
        default:  // DONE: nothing but end-of-sequence (a token, not a byte)
            return false;
    }
}

// ---------------------------------------------------------------------------------------------
// Contexts. A context fixes the mode, the part of the state that the mode reads (string kind and
// open UTF-8 sequence, literal position, \u digits left) and the kind of the innermost open
// container. At upload every (token, context) pair gets a verdict bit and a dependency bit; the
// verdict holds for every state of that context unless the token closes the innermost container
// and goes on (then the container below decides: dependency bit, the token is walked). A row's
// context is found through a 64K-entry table indexed by ctx_key.
constexpr uint32_t kMaxCtx = 96;
constexpr uint32_t kCtxWords = kMaxCtx / 32;
constexpr uint32_t kNoCtx = 0xFFu;
constexpr uint32_t kCtxKeys = 1u << 16;
constexpr uint32_t kCtxMaxDepth = 64;  // rows at least this deep are walked (push limit)
constexpr uint32_t kCtxMaxOpens = SIXI_JSON_MAX_DEPTH - kCtxMaxDepth;  // tokens opening more: walked

__host__ __device__ inline uint32_t ctx_key(uint32_t mode, uint32_t aux, uint32_t pos, uint32_t utf8,
                                            uint32_t top) {
    const bool str_like = mode == M_STR || mode == M_ESC || mode == M_HEX;
    const uint32_t a = (str_like || mode == M_LIT) ? aux : 0u;
    const uint32_t p = (mode == M_LIT || mode == M_HEX) ? pos : 0u;
    const uint32_t u = mode == M_STR ? utf8 : 0u;
    return (mode & 31u) | ((a & 3u) << 5) | ((p & 7u) << 7) | ((u & 31u) << 10) | ((top & 1u) << 15);
}

__host__ __device__ inline uint32_t ctx_key_of(const JS& s) {
    return ctx_key(s.mode, s.aux, s.pos, s.utf8, s.depth > 0 ? js_top_is_obj(s) : 0u);
}

struct JVocab {
    const uint4* head;      // [V] first 16 bytes of each token (zero padded)
    const uint2* meta;      // [V] length; flags and first bytes
    const uint8_t* bytes;   // all token bytes
    const uint64_t* off;    // [V] offset of each token in `bytes`
    const uint8_t* ctx_table;  // [kCtxKeys] context index of a ctx_key, kNoCtx when none
    const uint32_t* ctx_mask;  // [n_ctx][wpad] allowed-token bits of each context (dependent pairs 0)
    const uint32_t* dep_off;   // [n_ctx + 1] each context's dependent tokens in dep_ids
    const int32_t* dep_ids;    // ascending ids per context
    uint32_t vocab;
    uint32_t wpad;             // mask words per context row (ceil(V / 32) rounded up to 4)
    int32_t eos;
};

__device__ __forceinline__ uint32_t head_byte(const uint4& h, uint32_t i) {
    const uint32_t w = i < 8u ? (i < 4u ? h.x : h.y) : (i < 12u ? h.z : h.w);
    return (w >> (8u * (i & 3u))) & 0xFFu;
}

// The bytes of token `id` applied to s; false when one is refused.
__device__ __forceinline__ bool js_token(JS& s, const JVocab& v, uint32_t id, uint32_t len, const uint4& h) {
    const uint32_t n16 = len < 16u ? len : 16u;
    for (uint32_t i = 0; i < n16; ++i) {
        if (!js_byte(s, head_byte(h, i))) return false;
    }
    if (len > 16u) {
        const uint8_t* p = v.bytes + v.off[id];
        for (uint32_t i = 16; i < len; ++i) {
            if (!js_byte(s, p[i])) return false;
        }
    }
    return true;
}

// Applies token `id` to the state; false when it is not allowed there.
__device__ __forceinline__ bool js_apply(JS& s, const JVocab& v, uint32_t id) {
    const uint2 meta = v.meta[id];
    if (meta.y & kTokEos) return s.mode == M_DONE;
    const uint32_t len = meta.x;
    if ((meta.y & kTokSpecial) || len == 0u) return false;
    if (s.mode == M_STR && s.utf8 == 0u && (meta.y & kTokPlain)) return true;
    JS t = s;
    if (!js_token(t, v, id, len, v.head[id])) return false;
    s = t;
    return true;
}

// One thread per (token, context word): the verdict and dependency bits of 32 contexts.
__global__ void json_ctx_kernel(const JVocab v, const sixi_json_state* reps, uint32_t n_ctx, uint32_t* acc,
                                uint32_t* dep) {
    const uint32_t id = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t cw = blockIdx.y;
    if (id >= v.vocab) return;
    const uint2 meta = v.meta[id];
    const uint32_t len = meta.x;
    uint32_t a = 0u, d = 0u;
    if (!(meta.y & (kTokEos | kTokSpecial)) && len > 0u) {
        const uint4 h = v.head[id];
        const uint8_t* tail = v.bytes + v.off[id];
        const bool many_opens = (meta.y >> 24) > kCtxMaxOpens;
        for (uint32_t j = 0; j < 32u; ++j) {
            const uint32_t c = cw * 32u + j;
            if (c >= n_ctx) break;
            JS s = js_load(reps[c]);
            const uint32_t d0 = s.depth;
            bool ok = true, dp = many_opens;
            for (uint32_t i = 0; i < len && !dp; ++i) {
                if (!js_byte(s, i < 16u ? head_byte(h, i) : tail[i])) {
                    ok = false;
                    break;
                }
                if (s.depth < d0 && i + 1u < len) dp = true;  // closed the innermost container, goes on
            }
            if (dp) {
                d |= 1u << j;
            } else if (ok) {
                a |= 1u << j;
            }
        }
    }
    acc[static_cast<uint64_t>(cw) * v.vocab + id] = a;
    dep[static_cast<uint64_t>(cw) * v.vocab + id] = d;
}

constexpr int kMaskThreads = 256;
constexpr uint32_t kMaskSplit = 4;  // blocks per row
constexpr uint32_t kMaskMaxWords = 2048;  // words per block (shared memory)

// Verdict of token `id` by walking it (rows without a context and dependent pairs). A token whose
// first byte the state refuses (per-block table of the 256 byte values) is refused without a walk;
// in modes where whitespace changes nothing the first byte that is not whitespace is screened.
__device__ __noinline__ bool walk_verdict(const sixi_json_state& st, const JVocab& v, uint32_t id,
                                          const uint32_t* first_ok) {
    const uint2 meta = v.meta[id];
    const uint32_t len = meta.x;
    if ((meta.y & (kTokSpecial | kTokEos)) || len == 0u) return false;
    if (st.mode == M_STR && st.utf8 == 0u && (meta.y & kTokPlain)) return true;
    const bool ws_noop = st.mode <= M_AFTER;
    if (ws_noop && (meta.y & kTokAllWs)) return true;
    const uint32_t b = ws_noop ? (meta.y >> 16) & 0xFFu : (meta.y >> 8) & 0xFFu;
    if (!((first_ok[b >> 5] >> (b & 31u)) & 1u)) return false;
    JS s = js_load(st);
    return js_token(s, v, id, len, v.head[id]);
}

// Block (x, row) builds mask words [w0, w1) of one row in shared memory. With a context: a copy of
// the context's mask row, then the context's dependent tokens in range are walked and or-ed in.
// Without one (rows 64 or more containers deep): every token in range is walked. Done rows allow
// only end-of-sequence; failed rows nothing.
__global__ void __launch_bounds__(kMaskThreads) json_mask_kernel(const JVocab v, const sixi_json_state* states,
                                                                  uint32_t* mask, uint64_t stride,
                                                                  uint32_t words_per_block) {
    __shared__ uint32_t first_ok[8];
    __shared__ __align__(16) uint32_t sw[kMaskMaxWords];
    const uint32_t row = blockIdx.y;
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t words = (v.vocab + 31u) / 32u;
    const uint32_t w0 = blockIdx.x * words_per_block;
    const uint32_t w1 = w0 + words_per_block < words ? w0 + words_per_block : words;
    if (w0 >= w1) return;
    const sixi_json_state st = states[row];
    const bool live = st.failed == 0u && st.mode != M_DONE;
    const JS s0 = js_load(st);
    const uint32_t ctx = (live && st.depth < kCtxMaxDepth) ? v.ctx_table[ctx_key_of(s0)] : kNoCtx;
    {
        JS s = s0;
        const bool okb = live && js_byte(s, threadIdx.x);
        const uint32_t w = __ballot_sync(0xFFFFFFFFu, okb);
        if (lane == 0u) first_ok[threadIdx.x >> 5] = w;
    }
    const uint32_t n = w1 - w0;
    if (ctx != kNoCtx) {
        // w0 and wpad are multiples of 4: 16-byte copies
        const uint4* src = reinterpret_cast<const uint4*>(v.ctx_mask + static_cast<uint64_t>(ctx) * v.wpad + w0);
        for (uint32_t i = threadIdx.x; i < (n + 3u) / 4u; i += kMaskThreads) reinterpret_cast<uint4*>(sw)[i] = src[i];
    } else {
        for (uint32_t i = threadIdx.x; i < n; i += kMaskThreads) sw[i] = 0u;
    }
    __syncthreads();
    if (ctx != kNoCtx) {
        const uint32_t d0 = v.dep_off[ctx], d1 = v.dep_off[ctx + 1];
        for (uint32_t k = d0 + threadIdx.x; k < d1; k += kMaskThreads) {
            const uint32_t id = static_cast<uint32_t>(v.dep_ids[k]);
            if (id / 32u < w0 || id / 32u >= w1) continue;
            if (walk_verdict(st, v, id, first_ok)) atomicOr(&sw[id / 32u - w0], 1u << (id & 31u));
        }
    } else if (live) {
        for (uint32_t id = w0 * 32u + threadIdx.x; id < w1 * 32u && id < v.vocab; id += kMaskThreads) {
            const bool ok = walk_verdict(st, v, id, first_ok);
            const uint32_t word = __ballot_sync(__activemask(), ok);
            if (lane == 0u) sw[id / 32u - w0] = word;
        }
    } else if (st.failed == 0u && v.eos >= 0 && static_cast<uint32_t>(v.eos) / 32u >= w0 &&
               static_cast<uint32_t>(v.eos) / 32u < w1 && threadIdx.x == 0) {
        sw[static_cast<uint32_t>(v.eos) / 32u - w0] = 1u << (v.eos & 31);  // complete: end-of-sequence only
    }
    __syncthreads();
    uint32_t* dst = mask + static_cast<uint64_t>(row) * stride + w0;
    for (uint32_t i = threadIdx.x; i < n; i += kMaskThreads) dst[i] = sw[i];
}

__global__ void json_advance_kernel(const JVocab v, sixi_json_state* states, uint32_t n_rows, const int32_t* tokens,
                                    uint64_t token_stride, const int32_t* n_tokens, int32_t* out_status) {
    const uint32_t row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= n_rows) return;
    sixi_json_state st = states[row];
    int32_t status = SIXI_OK;
    if (st.failed) {
        status = SIXI_INVALID_ARGUMENT;
    } else {
        JS s = js_load(st);
        const int32_t n = n_tokens ? n_tokens[row] : 1;
        for (int32_t j = 0; j < n; ++j) {
            const int32_t id = tokens[static_cast<uint64_t>(row) * token_stride + static_cast<uint64_t>(j)];
            if (id < 0 || static_cast<uint32_t>(id) >= v.vocab || !js_apply(s, v, static_cast<uint32_t>(id))) {
                status = SIXI_INVALID_ARGUMENT;
                break;
            }
        }
        js_store(s, status != SIXI_OK ? 1u : 0u, st);
        states[row] = st;
    }
    if (out_status) out_status[row] = status;
}

__global__ void json_expand_kernel(const JVocab v, const sixi_json_state* states, uint32_t n_streams,
                                   const int32_t* drafts, uint32_t k, const int32_t* n_drafts,
                                   sixi_json_state* out) {
    const uint32_t s_i = blockIdx.x * blockDim.x + threadIdx.x;
    if (s_i >= n_streams) return;
    const sixi_json_state st = states[s_i];
    sixi_json_state* o = out + static_cast<uint64_t>(s_i) * (k + 1u);
    o[0] = st;
    JS s = js_load(st);
    uint32_t nd = n_drafts ? static_cast<uint32_t>(n_drafts[s_i] < 0 ? 0 : n_drafts[s_i]) : k;
    nd = nd < k ? nd : k;
    bool valid = st.failed == 0u;
    sixi_json_state cur = st;
    for (uint32_t j = 0; j < k; ++j) {
        if (valid && j < nd) {
            const int32_t id = drafts[static_cast<uint64_t>(s_i) * k + j];
            if (id >= 0 && static_cast<uint32_t>(id) < v.vocab && js_apply(s, v, static_cast<uint32_t>(id))) {
                js_store(s, 0u, cur);
            } else {
                valid = false;
            }
        }
        o[j + 1u] = cur;
    }
}

// The same walk on the host, for the per-token flags computed at upload: a token is plain string
// content when, from a string with no UTF-8 sequence open, every byte keeps the walk inside the
// string (content, escapes) and the token ends there with no sequence open. Such a token leaves
// any such state unchanged, whatever encloses the string.
bool host_plain(const uint8_t* p, uint64_t len) {
    JS s{};
    s.mode = M_STR;
    for (uint64_t i = 0; i < len; ++i) {
        if (!js_byte(s, p[i])) return false;
        if (s.mode != M_STR && s.mode != M_ESC && s.mode != M_HEX) return false;
    }
    return s.mode == M_STR && s.utf8 == 0u;
}

}  // namespace

struct sixi_json_vocab {
    int32_t device;
    uint32_t vocab;
    int32_t eos_id;
    uint4* head;
    uint2* meta;
    uint8_t* bytes;
    uint64_t* off;
    uint8_t* ctx_table;
    sixi_json_state* ctx_rep;
    uint32_t* ctx_mask;
    uint32_t* dep_off;
    int32_t* dep_ids;
    uint32_t wpad;
};

namespace {

struct DevGuard {
    int prev = -1;
    explicit DevGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DevGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

int32_t status_of(cudaError_t e) {
    if (e == cudaSuccess) return SIXI_OK;
    if (e == cudaErrorMemoryAllocation) return SIXI_OUT_OF_MEMORY_VRAM;
    return SIXI_BACKEND_ERROR;
}

JVocab view(const sixi_json_vocab* v) {
    return JVocab{v->head, v->meta, v->bytes, v->off, v->ctx_table, v->ctx_mask, v->dep_off, v->dep_ids,
                  v->vocab, v->wpad, v->eos_id};
}

void free_vocab(sixi_json_vocab* v) {
    cudaFree(v->head);
    cudaFree(v->meta);
    cudaFree(v->bytes);
    cudaFree(v->off);
    cudaFree(v->ctx_table);
    cudaFree(v->ctx_rep);
    cudaFree(v->ctx_mask);
    cudaFree(v->dep_off);
    cudaFree(v->dep_ids);
    delete v;
}

// Every context with its representative state (innermost container at depth 2, or the start).
void build_contexts(std::vector<sixi_json_state>& reps, std::vector<uint8_t>& table) {
    table.assign(kCtxKeys, static_cast<uint8_t>(kNoCtx));
    auto add = [&](uint32_t mode, uint32_t aux, uint32_t pos, uint32_t utf8, uint32_t top) {
        sixi_json_state t;
        std::memset(&t, 0, sizeof(t));
        t.mode = static_cast<uint8_t>(mode);
        t.aux = static_cast<uint8_t>(aux);
        t.pos = static_cast<uint8_t>(pos);
        t.utf8 = static_cast<uint8_t>(utf8);
        if (mode != M_START) {
            t.depth = 2;
            t.stack[0] = 1u | (top << 1);
        }
        table[ctx_key(mode, aux, pos, utf8, mode == M_START ? 0u : top)] = static_cast<uint8_t>(reps.size());
        reps.push_back(t);
    };
    add(M_START, 0, 0, 0, 0);
    add(M_OBJ_FIRST, 0, 0, 0, 1);
    add(M_OBJ_KEY, 0, 0, 0, 1);
    add(M_COLON, 0, 0, 0, 1);
    add(M_ARR_FIRST, 0, 0, 0, 0);
    const uint32_t str_slots[3][2] = {{1, 1}, {0, 0}, {0, 1}};  // (aux, top): key, value in array/object
    const uint32_t utf8_codes[8] = {0, 1, 2, 6, 10, 3, 15, 19};
    for (const auto& sl : str_slots) {
        for (uint32_t u : utf8_codes) add(M_STR, sl[0], 0, u, sl[1]);
        add(M_ESC, sl[0], 0, 0, sl[1]);
        for (uint32_t p = 1; p <= 4; ++p) add(M_HEX, sl[0], p, 0, sl[1]);
    }
    for (uint32_t top = 0; top < 2; ++top) {
        add(M_VALUE, 0, 0, 0, top);
        add(M_AFTER, 0, 0, 0, top);
        for (uint32_t m : {M_NEG, M_ZERO, M_INT, M_DOT, M_FRAC, M_EXP, M_EXPS, M_EXPD}) add(m, 0, 0, 0, top);
        for (uint32_t w = 0; w < 3; ++w)
            for (uint32_t p = 1; p < lit_len(w); ++p) add(M_LIT, w, p, 0, top);
    }
}

}  // namespace

extern "C" {

int32_t sixi_json_vocab_create(int32_t device, const uint8_t* host_bytes, const uint64_t* host_offsets,
                               uint32_t vocab, const uint8_t* host_flags, int32_t eos_id,
                               sixi_json_vocab** out) {
    if (out == nullptr || host_offsets == nullptr || vocab == 0u || (host_bytes == nullptr && host_offsets[vocab] > 0) ||
        eos_id >= static_cast<int64_t>(vocab) || eos_id < -1)
        return SIXI_INVALID_ARGUMENT;
    *out = nullptr;
    const uint64_t total = host_offsets[vocab];
    std::vector<uint4> head(vocab);
    std::vector<uint2> meta(vocab);
    for (uint32_t i = 0; i < vocab; ++i) {
        if (host_offsets[i + 1] < host_offsets[i] || host_offsets[i + 1] > total) return SIXI_INVALID_ARGUMENT;
        const uint64_t len = host_offsets[i + 1] - host_offsets[i];
        if (len > kMaxTokenBytes) return SIXI_INVALID_ARGUMENT;
        const uint8_t* p = host_bytes + host_offsets[i];
        uint8_t h[16] = {};
        std::memcpy(h, p, len < 16 ? len : 16);
        std::memcpy(&head[i], h, 16);
        uint32_t f = 0u;
        if (host_flags && (host_flags[i] & SIXI_JSON_TOKEN_SPECIAL)) f |= kTokSpecial;
        if (static_cast<int64_t>(i) == eos_id) f |= kTokEos;
        if (len > 0 && !(f & (kTokSpecial | kTokEos)) && host_plain(p, len)) f |= kTokPlain;
        uint64_t nws = 0, opens = 0;
        while (nws < len && is_ws(p[nws])) ++nws;
        for (uint64_t k = 0; k < len; ++k) opens += (p[k] == 0x7Bu || p[k] == 0x5Bu) ? 1u : 0u;
        if (len > 0 && nws == len) f |= kTokAllWs;
        const uint32_t b0 = len > 0 ? p[0] : 0u, bn = nws < len ? p[nws] : 0u;
        const uint32_t no = static_cast<uint32_t>(opens < 255 ? opens : 255);
        meta[i] = make_uint2(static_cast<uint32_t>(len), f | (b0 << 8) | (bn << 16) | (no << 24));
    }
    DevGuard g(device);
    sixi_json_vocab* v = new (std::nothrow) sixi_json_vocab{};
    if (v == nullptr) return SIXI_OUT_OF_MEMORY_VRAM;
    v->device = device;
    v->vocab = vocab;
    v->eos_id = eos_id;
    cudaError_t e = cudaMalloc(&v->head, sizeof(uint4) * vocab);
    if (e == cudaSuccess) e = cudaMalloc(&v->meta, sizeof(uint2) * vocab);
    if (e == cudaSuccess) e = cudaMalloc(&v->bytes, total > 0 ? total : 1);
    if (e == cudaSuccess) e = cudaMalloc(&v->off, sizeof(uint64_t) * vocab);
    if (e == cudaSuccess) e = cudaMemcpy(v->head, head.data(), sizeof(uint4) * vocab, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(v->meta, meta.data(), sizeof(uint2) * vocab, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && total > 0) e = cudaMemcpy(v->bytes, host_bytes, total, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(v->off, host_offsets, sizeof(uint64_t) * vocab, cudaMemcpyHostToDevice);
    // per-(token, context) verdicts, computed on the device once
    std::vector<sixi_json_state> reps;
    std::vector<uint8_t> table;
    build_contexts(reps, table);
    if (reps.size() > kMaxCtx) e = cudaErrorInvalidValue;
    if (e == cudaSuccess) e = cudaMalloc(&v->ctx_table, kCtxKeys);
    if (e == cudaSuccess) e = cudaMalloc(&v->ctx_rep, sizeof(sixi_json_state) * reps.size());
    uint32_t* d_acc = nullptr;
    uint32_t* d_dep = nullptr;
    if (e == cudaSuccess) e = cudaMalloc(&d_acc, sizeof(uint32_t) * kCtxWords * vocab);
    if (e == cudaSuccess) e = cudaMalloc(&d_dep, sizeof(uint32_t) * kCtxWords * vocab);
    if (e == cudaSuccess) e = cudaMemcpy(v->ctx_table, table.data(), kCtxKeys, cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy(v->ctx_rep, reps.data(), sizeof(sixi_json_state) * reps.size(), cudaMemcpyHostToDevice);
    const uint32_t n_ctx = static_cast<uint32_t>(reps.size());
    if (e == cudaSuccess) {
        const dim3 grid((vocab + 255u) / 256u, kCtxWords);
        JVocab jv = view(v);
        json_ctx_kernel<<<grid, 256>>>(jv, v->ctx_rep, n_ctx, d_acc, d_dep);
        e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
    }
    // per context: the mask row of its verdicts and the ascending list of its dependent tokens
    std::vector<uint32_t> acc, dep;
    if (e == cudaSuccess) {
        acc.resize(static_cast<size_t>(kCtxWords) * vocab);
        dep.resize(static_cast<size_t>(kCtxWords) * vocab);
        e = cudaMemcpy(acc.data(), d_acc, sizeof(uint32_t) * acc.size(), cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemcpy(dep.data(), d_dep, sizeof(uint32_t) * dep.size(), cudaMemcpyDeviceToHost);
    }
    cudaFree(d_acc);
    cudaFree(d_dep);
    v->wpad = ((vocab + 31u) / 32u + 3u) / 4u * 4u;
    if (e == cudaSuccess) {
        std::vector<uint32_t> cmask(static_cast<size_t>(n_ctx) * v->wpad, 0u);
        std::vector<uint32_t> doff(n_ctx + 1, 0u);
        std::vector<int32_t> dids;
        for (uint32_t c = 0; c < n_ctx; ++c) {
            const uint32_t* a = acc.data() + static_cast<size_t>(c / 32u) * vocab;
            const uint32_t* d = dep.data() + static_cast<size_t>(c / 32u) * vocab;
            uint32_t* m = cmask.data() + static_cast<size_t>(c) * v->wpad;
            for (uint32_t i = 0; i < vocab; ++i) {
                if ((d[i] >> (c & 31u)) & 1u) {
                    dids.push_back(static_cast<int32_t>(i));
                } else if ((a[i] >> (c & 31u)) & 1u) {
                    m[i / 32u] |= 1u << (i & 31u);
                }
            }
            doff[c + 1] = static_cast<uint32_t>(dids.size());
        }
        if (dids.empty()) dids.push_back(0);
        e = cudaMalloc(&v->ctx_mask, sizeof(uint32_t) * cmask.size());
        if (e == cudaSuccess) e = cudaMalloc(&v->dep_off, sizeof(uint32_t) * doff.size());
        if (e == cudaSuccess) e = cudaMalloc(&v->dep_ids, sizeof(int32_t) * dids.size());
        if (e == cudaSuccess)
            e = cudaMemcpy(v->ctx_mask, cmask.data(), sizeof(uint32_t) * cmask.size(), cudaMemcpyHostToDevice);
        if (e == cudaSuccess)
            e = cudaMemcpy(v->dep_off, doff.data(), sizeof(uint32_t) * doff.size(), cudaMemcpyHostToDevice);
        if (e == cudaSuccess)
            e = cudaMemcpy(v->dep_ids, dids.data(), sizeof(int32_t) * dids.size(), cudaMemcpyHostToDevice);
    }
    if (e != cudaSuccess) {
        free_vocab(v);
        return status_of(e);
    }
    *out = v;
    return SIXI_OK;
}

void sixi_json_vocab_destroy(sixi_json_vocab* v) {
    if (v == nullptr) return;
    DevGuard g(v->device);
    free_vocab(v);
}

uint32_t sixi_json_vocab_size(const sixi_json_vocab* v) { return v ? v->vocab : 0u; }

int32_t sixi_json_reset(const sixi_json_vocab* v, sixi_json_state* states, uint32_t n_rows, void* stream) {
    if (v == nullptr || (n_rows > 0 && states == nullptr)) return SIXI_INVALID_ARGUMENT;
    if (n_rows == 0) return SIXI_OK;
    DevGuard g(v->device);
    return status_of(cudaMemsetAsync(states, 0, sizeof(sixi_json_state) * n_rows, static_cast<cudaStream_t>(stream)));
}

int32_t sixi_json_fill_masks(const sixi_json_vocab* v, const sixi_json_state* states, uint32_t n_rows,
                             uint32_t* mask_words, uint64_t mask_stride, void* stream) {
    if (v == nullptr || (n_rows > 0 && (states == nullptr || mask_words == nullptr)) ||
        mask_stride < (v->vocab + 31u) / 32u || n_rows > 65535u)
        return SIXI_INVALID_ARGUMENT;
    if (n_rows == 0) return SIXI_OK;
    DevGuard g(v->device);
    // words per block: a multiple of 4 (16-byte copies), at most kMaskMaxWords
    const uint32_t words = (v->vocab + 31u) / 32u;
    uint32_t split = kMaskSplit;
    while ((words + split - 1) / split > kMaskMaxWords - 3u) ++split;
    const uint32_t wpb = ((words + split - 1) / split + 3u) / 4u * 4u;
    const dim3 grid((words + wpb - 1) / wpb, n_rows);
    json_mask_kernel<<<grid, kMaskThreads, 0, static_cast<cudaStream_t>(stream)>>>(view(v), states, mask_words,
                                                                                   mask_stride, wpb);
    return status_of(cudaGetLastError());
}

int32_t sixi_json_advance(const sixi_json_vocab* v, sixi_json_state* states, uint32_t n_rows,
                          const int32_t* tokens, uint64_t token_stride, const int32_t* n_tokens,
                          int32_t* out_status, void* stream) {
    if (v == nullptr || (n_rows > 0 && (states == nullptr || tokens == nullptr)) ||
        (n_tokens != nullptr && token_stride == 0))
        return SIXI_INVALID_ARGUMENT;
    if (n_rows == 0) return SIXI_OK;
    DevGuard g(v->device);
    const uint32_t nb = (n_rows + 127u) / 128u;
    json_advance_kernel<<<nb, 128, 0, static_cast<cudaStream_t>(stream)>>>(view(v), states, n_rows, tokens,
                                                                          token_stride, n_tokens, out_status);
    return status_of(cudaGetLastError());
}

int32_t sixi_json_expand_drafts(const sixi_json_vocab* v, const sixi_json_state* states, uint32_t n_streams,
                                const int32_t* drafts, uint32_t k, const int32_t* n_drafts,
                                sixi_json_state* out_states, void* stream) {
    if (v == nullptr || (n_streams > 0 && (states == nullptr || out_states == nullptr || (k > 0 && drafts == nullptr))))
        return SIXI_INVALID_ARGUMENT;
    if (n_streams == 0) return SIXI_OK;
    DevGuard g(v->device);
    const uint32_t nb = (n_streams + 127u) / 128u;
    json_expand_kernel<<<nb, 128, 0, static_cast<cudaStream_t>(stream)>>>(view(v), states, n_streams, drafts, k,
                                                                         n_drafts, out_states);
    return status_of(cudaGetLastError());
}

}  // extern "C"
