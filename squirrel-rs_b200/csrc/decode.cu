// decode.cu — persistent single-token decode kernel (placeholder until enabled).
#include "../host/model.h"
#include "common.cuh"
#include "decode.cuh"

namespace sq {
int decode_prepare(sq_ctx *) { return SQ_OK; }
bool decode_available(const sq_ctx *) { return false; }
int decode_launch(sq_ctx *, uint32_t *, uint32_t *, int) { return fail(SQ_ERR_ARG, "decode kernel unavailable"); }
int decode_check(sq_ctx *) { return SQ_OK; }
void decode_release(sq_ctx *) {}
}  // namespace sq
