/* TEST INFRASTRUCTURE ONLY: the CPU automaton of the JSON-object grammar (sixi_json_oracle.c), the
 * parity checker of the device mask producer (include/sixi_json.h). */
#ifndef SIXI_JSON_ORACLE_H
#define SIXI_JSON_ORACLE_H

#include <stdint.h>

#include "../include/sixi_json.h"

#ifdef __cplusplus
extern "C" {
#endif

int orc_json_feed(sixi_json_state* st, const uint8_t* p, uint64_t n);
void orc_json_fill_masks(const uint8_t* bytes, const uint64_t* offs, const uint8_t* flags, uint32_t vocab,
                         int32_t eos, const sixi_json_state* states, uint32_t n_rows, uint32_t* masks,
                         uint64_t stride, int n_threads);
void orc_json_advance(const uint8_t* bytes, const uint64_t* offs, const uint8_t* flags, uint32_t vocab, int32_t eos,
                      sixi_json_state* states, uint32_t n_rows, const int32_t* tokens, uint64_t stride,
                      const int32_t* n_tokens, int32_t* status);
void orc_json_expand(const uint8_t* bytes, const uint64_t* offs, const uint8_t* flags, uint32_t vocab, int32_t eos,
                     const sixi_json_state* states, uint32_t n_streams, const int32_t* drafts, uint32_t k,
                     const int32_t* n_drafts, sixi_json_state* out);

#ifdef __cplusplus
}
#endif

#endif /* SIXI_JSON_ORACLE_H */
