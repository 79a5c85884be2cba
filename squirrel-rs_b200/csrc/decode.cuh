// decode.cuh — persistent single-token decode kernel (decode.cu).
#pragma once
#include <stdint.h>

struct sq_ctx;
namespace sq {
int decode_prepare(sq_ctx *c);           // allocate per-context resources; SQ_OK when unsupported
bool decode_available(const sq_ctx *c);  // the persistent kernel handles this model
// one decode step: token id at d_tok (device); writes logits, argmax, the next
// token id back into d_tok and, when out_ids != null, out_ids[step]
int decode_launch(sq_ctx *c, uint32_t *d_tok, uint32_t *out_ids, int step);
int decode_check(sq_ctx *c);             // after a sync: SQ_ERR_TIMEOUT if a bounded wait gave up
unsigned *decode_err_ptr(const sq_ctx *c);  // the kernel's error word (null without the kernel)
bool decode_check_always(const sq_ctx *c);  // profiling builds: decode_check after every call
void decode_release(sq_ctx *c);
}  // namespace sq
