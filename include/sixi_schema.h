/* sixi_schema.h - C ABI of the grammar-mask producer for `response_format: json_schema` answers.
 *
 * The engine decodes `{"type": "json_schema", "json_schema": {"schema": {...}}}` answers under a
 * grammar: the model may only choose tokens that keep the answer a prefix of a document matching
 * the schema, and generation stops at the end of the document (docs/API.md:45-76 in the engine,
 * whose automaton ships only in binary form). This producer compiles the schema once on the host
 * (sixi_schema_compile), keeps one automaton state per row in device memory and writes the packed
 * allowed-token masks that sixi_smp_sample / sixi_smp_verify consume (bit i % 32 of word i / 32):
 *     sixi_schema_fill_masks(states) -> sixi_smp_sample(..., masks) -> sixi_schema_advance(tokens)
 *
 * Supported keywords (the engine's list): type (a name or a list), properties, required,
 * additionalProperties (true, false or a schema), items (a schema or false), prefixItems, minItems,
 * maxItems, enum, const, anyOf, allOf, $ref with $defs (and "#"), minimum / maximum /
 * exclusiveMinimum / exclusiveMaximum for integers, minLength, maxLength, pattern (anchored with ^
 * and $), format (date, time, date-time, uuid); the annotations title, description, default,
 * examples, $schema, $id and $comment are accepted and have no effect. Anything else is refused
 * with SIXI_INVALID_ARGUMENT and a message naming the place, as the engine's API does, e.g.
 * "JSON schema: #/properties/a: keyword 'uniqueItems' is not supported".
 * Limits of this implementation, refused the same way: anyOf / type-list alternatives must begin
 * with different characters (a string and null, an object and an array, ...; integer with number
 * is read as number), allOf merges object schemas (properties and required) or identical types;
 * at most 64 properties per object and 64 enum / const values per node; patterns use literals,
 * ., [...] classes with ranges, \d \w \s, groups, |, ?, *, + and {m,n} over ASCII; enum and const
 * values are matched in compact JSON form (no whitespace inside them).
 * Grammar details: whitespace is allowed wherever JSON allows it except after the top-level value,
 * which is followed by nothing but the end-of-sequence token. Object keys are the declared names
 * written literally; an additional property's key is any other string. String lengths count code
 * points (an escape counts as one). Containers nest at most SIXI_SCHEMA_MAX_DEPTH deep, and a
 * token that opens more than SIXI_SCHEMA_MASK_OPENS containers at once is not allowed by the
 * masks (sixi_schema_advance still applies it).
 *
 * Conventions are those of sixi_smp.h: calls on device states are asynchronous on the caller's
 * stream, status codes are the engine's ErrorCode values, per-row failures go to out_status.
 */
#ifndef SIXI_SCHEMA_H
#define SIXI_SCHEMA_H

#include <stddef.h>
#include <stdint.h>

#include "sixi_smp.h"

#ifdef __cplusplus
extern "C" {
#endif

#define SIXI_SCHEMA_MAX_DEPTH 32u
#define SIXI_SCHEMA_MASK_OPENS 6u
#define SIXI_SCHEMA_STATE_BYTES 800u

/* Automaton state of one row: plain data, SIXI_SCHEMA_STATE_BYTES bytes, set by sixi_schema_reset. */
typedef struct sixi_schema_state {
    uint8_t bytes[SIXI_SCHEMA_STATE_BYTES];
} sixi_schema_state;

typedef struct sixi_schema sixi_schema;

/* Compiles a JSON schema (UTF-8 JSON text of the "schema" object) against a tokenizer vocabulary
 * (token i's text is host_bytes[host_offsets[i], host_offsets[i+1]); host_flags (nullable) marks
 * control tokens with SIXI_JSON_TOKEN_SPECIAL = 1, never allowed; eos_id or -1 is the
 * end-of-sequence token) and uploads both to `device`. On a schema error returns
 * SIXI_INVALID_ARGUMENT and writes a NUL-terminated message into err (err_cap bytes, nullable).
 * Synchronous. */
SIXI_SMP_API int32_t sixi_schema_compile(int32_t device, const char* schema_json, size_t schema_len,
                                         const uint8_t* host_bytes, const uint64_t* host_offsets, uint32_t vocab,
                                         const uint8_t* host_flags, int32_t eos_id, char* err, size_t err_cap,
                                         sixi_schema** out);
SIXI_SMP_API void sixi_schema_destroy(sixi_schema* g);
SIXI_SMP_API uint32_t sixi_schema_vocab_size(const sixi_schema* g);

/* Sets n_rows device states to the start state. */
SIXI_SMP_API int32_t sixi_schema_reset(const sixi_schema* g, sixi_schema_state* states, uint32_t n_rows,
                                       void* stream);

/* Allowed-token masks: mask_words[r * mask_stride + w], w < ceil(V / 32), bit i % 32 of word i / 32
 * set when token i keeps row r's text a prefix of a matching document (the end-of-sequence token:
 * when the document is complete). A failed row gets an empty mask. */
SIXI_SMP_API int32_t sixi_schema_fill_masks(const sixi_schema* g, const sixi_schema_state* states, uint32_t n_rows,
                                            uint32_t* mask_words, uint64_t mask_stride, void* stream);

/* Advances each row by tokens[r * token_stride + j], j < n_tokens[r] (n_tokens NULL: one token);
 * out_status[r] (nullable): SIXI_OK, or SIXI_INVALID_ARGUMENT for a token that was not allowed
 * (the row then stays at the state before it, failed). */
SIXI_SMP_API int32_t sixi_schema_advance(const sixi_schema* g, sixi_schema_state* states, uint32_t n_rows,
                                         const int32_t* tokens, uint64_t token_stride, const int32_t* n_tokens,
                                         int32_t* out_status, void* stream);

/* Host-side check of one text against the compiled schema (no device work): returns 1 when the
 * bytes are a prefix of a matching document (2 when they are a complete one), 0 otherwise. For
 * tests and tooling. */
SIXI_SMP_API int32_t sixi_schema_check_text(const sixi_schema* g, const uint8_t* text, size_t len);

#ifdef __cplusplus
}
#endif

#endif /* SIXI_SCHEMA_H */
