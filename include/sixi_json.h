/* sixi_json.h - C ABI of the device-side grammar-mask producer for JSON-object answers.
 *
 * The engine decodes `response_format: {"type": "json_object"}` answers under a grammar: the
 * model may only choose tokens that keep the answer a prefix of exactly one JSON object, and
 * generation stops at the end of the document (docs/API.md:45-76 in the engine). The engine's own
 * automaton ships only in binary form; the mask it produces is the packed per-row allowed-token
 * bitmask that the sampler consumes (bit i % 32 of word i / 32, masked logits -> -inf before
 * penalties; hot-path row a12, `sixi_smp_sample` / `sixi_smp_verify` `mask_words`).
 *
 * This producer keeps the automaton state of every row on the device and writes the masks there,
 * so a constrained decoding step is three launches on one stream and no host round trip:
 *     sixi_json_fill_masks(states) -> sixi_smp_sample(..., masks) -> sixi_json_advance(tokens)
 * The grammar is RFC 8259 JSON with an object at the top level: leading whitespace, then one
 * object, then nothing but the end-of-sequence token. Strings must be valid UTF-8 (RFC 3629) with
 * no raw control characters; numbers, literals and escapes follow RFC 8259 exactly. Containers
 * nest at most SIXI_JSON_MAX_DEPTH deep.
 *
 * Conventions are those of sixi_smp.h: every call is asynchronous on the caller's stream, status
 * codes are the engine's ErrorCode values (SIXI_OK, SIXI_INVALID_ARGUMENT, ...), and per-row
 * failures go to out_status, never to a trap.
 */
#ifndef SIXI_JSON_H
#define SIXI_JSON_H

#include <stddef.h>
#include <stdint.h>

#include "sixi_smp.h"

#ifdef __cplusplus
extern "C" {
#endif

#define SIXI_JSON_MAX_DEPTH 128u

/* automaton modes (sixi_json_state.mode) */
#define SIXI_JSON_START 0u       /* before the document: whitespace or '{' */
#define SIXI_JSON_OBJ_FIRST 1u   /* after '{': whitespace, a key or '}' */
#define SIXI_JSON_OBJ_KEY 2u     /* after ',' in an object: whitespace or a key */
#define SIXI_JSON_COLON 3u       /* after a key: whitespace or ':' */
#define SIXI_JSON_VALUE 4u       /* after ':' or after ',' in an array: whitespace or a value */
#define SIXI_JSON_ARR_FIRST 5u   /* after '[': whitespace, a value or ']' */
#define SIXI_JSON_AFTER 6u       /* after a value in a container: whitespace, ',' or the close */
#define SIXI_JSON_DONE 7u        /* the top-level object is closed: only end-of-sequence */
#define SIXI_JSON_STRING 8u      /* inside a string (aux 1: an object key) */
#define SIXI_JSON_ESCAPE 9u      /* after a backslash in a string */
#define SIXI_JSON_HEX 10u        /* inside \uXXXX (pos: hex digits left) */
#define SIXI_JSON_NEG 11u        /* number: after '-' */
#define SIXI_JSON_ZERO 12u       /* number: a leading 0 */
#define SIXI_JSON_INT 13u        /* number: integer digits */
#define SIXI_JSON_DOT 14u        /* number: after '.' */
#define SIXI_JSON_FRAC 15u       /* number: fraction digits */
#define SIXI_JSON_EXP 16u        /* number: after 'e' / 'E' */
#define SIXI_JSON_EXP_SIGN 17u   /* number: after the exponent sign */
#define SIXI_JSON_EXP_DIGITS 18u /* number: exponent digits */
#define SIXI_JSON_LITERAL 19u    /* inside true / false / null (aux: which, pos: next char) */

/* per-token flags of sixi_json_vocab_create */
#define SIXI_JSON_TOKEN_SPECIAL 1u /* a control token with no text: never allowed */

/* Automaton state of one row (32 bytes, plain data; all-zero bytes are the start state). */
typedef struct sixi_json_state {
    uint8_t mode;       /* SIXI_JSON_* */
    uint8_t aux;        /* string: 1 for an object key, 0 for a value; literal: 0 true, 1 false, 2 null */
    uint8_t pos;        /* literal: index of the next character; \u escape: hex digits left */
    uint8_t utf8;       /* string: continuation bytes still due (bits 0-1) and the range of the next
                           one (bits 2-4: 0 80-BF, 1 A0-BF, 2 80-9F, 3 90-BF, 4 80-8F) */
    uint16_t depth;     /* open containers */
    uint8_t failed;     /* 1 after a disallowed token was applied: the row is frozen, its mask empty */
    uint8_t reserved0;
    uint32_t stack[4];  /* bit d (word d / 32) is 1 when the container at depth d (0 = outermost) is
                           an object, 0 for an array */
    uint32_t reserved1[2];
} sixi_json_state;

typedef struct sixi_json_vocab sixi_json_vocab;

/* Uploads a tokenizer vocabulary: token i's text is host_bytes[host_offsets[i], host_offsets[i+1]).
 * host_flags (nullable, [vocab]) marks control tokens (SIXI_JSON_TOKEN_SPECIAL); eos_id (or -1) is
 * the end-of-sequence token, allowed exactly when the document is complete. Tokens with empty text
 * are never allowed. Synchronous (it copies from host memory once). */
SIXI_SMP_API int32_t sixi_json_vocab_create(int32_t device, const uint8_t* host_bytes,
                                            const uint64_t* host_offsets, uint32_t vocab,
                                            const uint8_t* host_flags, int32_t eos_id,
                                            sixi_json_vocab** out);
SIXI_SMP_API void sixi_json_vocab_destroy(sixi_json_vocab* v);
SIXI_SMP_API uint32_t sixi_json_vocab_size(const sixi_json_vocab* v);

/* Sets n_rows device states to the start state. */
SIXI_SMP_API int32_t sixi_json_reset(const sixi_json_vocab* v, sixi_json_state* states, uint32_t n_rows,
                                     void* stream);

/* Writes the allowed-token mask of every row: mask_words[r * mask_stride + w], w < ceil(V / 32),
 * bit i % 32 of word i / 32 set when token i may follow the row's text (bits past V are 0). A
 * failed row gets an empty mask. mask_stride >= ceil(V / 32); sixi_smp_sample and sixi_smp_verify
 * read masks with stride ceil(V / 32). */
SIXI_SMP_API int32_t sixi_json_fill_masks(const sixi_json_vocab* v, const sixi_json_state* states,
                                          uint32_t n_rows, uint32_t* mask_words, uint64_t mask_stride,
                                          void* stream);

/* Advances each row by its tokens: tokens[r * token_stride + j] for j < n_tokens[r] (n_tokens NULL:
 * one token per row). out_status[r] (nullable) is SIXI_OK, or SIXI_INVALID_ARGUMENT when a token
 * was not allowed (or is out of range); such a row stays frozen at the state before that token
 * with its failed flag set. */
SIXI_SMP_API int32_t sixi_json_advance(const sixi_json_vocab* v, sixi_json_state* states, uint32_t n_rows,
                                       const int32_t* tokens, uint64_t token_stride, const int32_t* n_tokens,
                                       int32_t* out_status, void* stream);

/* Speculative verification needs one mask per target row: target row j of stream s sees the text
 * extended by the first j drafts. Writes out_states[s * (k + 1) + j] = states[s] advanced by
 * drafts[s * k + 0 .. j - 1] for j <= n_drafts[s] (n_drafts NULL: k). From a disallowed draft on,
 * the later rows repeat the last valid state (the verifier rejects that draft first, so their
 * masks are never consulted). Feed out_states to sixi_json_fill_masks with S * (k + 1) rows. */
SIXI_SMP_API int32_t sixi_json_expand_drafts(const sixi_json_vocab* v, const sixi_json_state* states,
                                             uint32_t n_streams, const int32_t* drafts, uint32_t k,
                                             const int32_t* n_drafts, sixi_json_state* out_states,
                                             void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SIXI_JSON_H */
