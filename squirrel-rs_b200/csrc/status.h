// status.h — host-usable pieces shared by the CUDA sources and the host code:
// GGUF block sizes and the error plumbing behind sq_last_error().
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/squirrel_cuda.h"

namespace sq {

// GGUF block sizes (kernels/tensor.rs:10-35): 32 elements per block.
constexpr int QK = 32;
constexpr int Q8_BYTES = 34;  // f16 scale + 32 x i8
constexpr int Q4_BYTES = 18;  // f16 scale + 16 bytes: low nibble = elt j, high = elt j+16
constexpr int BF16_BYTES = 64;

inline int block_bytes(int t) {
  switch (t) {
    case SQ_Q8_0: return Q8_BYTES;
    case SQ_Q4_0: return Q4_BYTES;
    case SQ_BF16: return BF16_BYTES;
    default: return 0;
  }
}
inline bool is_weight_type(int t) { return t == SQ_Q8_0 || t == SQ_Q4_0 || t == SQ_BF16; }
// Bytes of a tensor of numel elements (0 for an unsupported type or a partial block).
inline size_t tensor_nbytes(int type, uint64_t numel) {
  if (type == SQ_F32) return numel * 4;
  const int bb = block_bytes(type);
  if (!bb || numel % QK) return 0;
  return numel / QK * bb;
}

// ---- error plumbing -------------------------------------------------------------
void set_error(const std::string &msg);
int fail(int code, const std::string &msg);
int cuda_fail(cudaError_t e, const char *what);

#define SQ_CUDA(call)                                  \
  do {                                                 \
    cudaError_t _e = (call);                           \
    if (_e != cudaSuccess) return ::sq::cuda_fail(_e, #call); \
  } while (0)

#define SQ_CHECK_LAUNCH(what)                              \
  do {                                                     \
    cudaError_t _e = cudaGetLastError();                   \
    if (_e != cudaSuccess) return ::sq::cuda_fail(_e, what); \
  } while (0)

}  // namespace sq
