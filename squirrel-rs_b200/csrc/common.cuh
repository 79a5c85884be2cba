// common.cuh — shared device helpers: exact dequant, warp reductions, greedy fold state.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "status.h"

namespace sq {

// ---- device helpers ---------------------------------------------------------------

// f16 -> f32 is exact (half::f16::to_f32).
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ float bf2f(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

__device__ __forceinline__ uint16_t ld_u16(const uint8_t *p) {
  return *reinterpret_cast<const uint16_t *>(p);  // blocks are 2-byte aligned
}

// Exact dequantization of element j (0..31) of one block (dot_prod.rs:409-414, 440-446, 524-528).
template <int T>
__device__ __forceinline__ float dequant_elem(const uint8_t *blk, int j) {
  if constexpr (T == SQ_Q8_0) {
    return h2f(ld_u16(blk)) * (float)(int8_t)blk[2 + j];
  } else if constexpr (T == SQ_Q4_0) {
    uint8_t byte = blk[2 + (j & 15)];
    int q = j < 16 ? (byte & 0x0F) : (byte >> 4);
    return h2f(ld_u16(blk)) * (float)(q - 8);
  } else {
    return bf2f(ld_u16(blk + 2 * j));
  }
}

template <int T>
constexpr int type_bytes() {
  return T == SQ_Q8_0 ? Q8_BYTES : (T == SQ_Q4_0 ? Q4_BYTES : BF16_BYTES);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// State of GreedySampler's fold over a contiguous index range (greedy.rs:6-15).
// Iterator::max_by keeps the running best only when it compares Greater than the
// next item, so a NaN (which compares Equal) replaces the best and is itself replaced
// by the following item: the answer is the last-max of the items after the last NaN,
// or that NaN's index when it is the final item. `best` < 0 means "no item after the
// last NaN", `nan` < 0 means "no NaN". combine(L, R) needs L to precede R.
struct ArgState {
  float v;
  long long best;
  long long nan;
};
__device__ __forceinline__ ArgState arg_empty() { return {0.f, -1, -1}; }
__device__ __forceinline__ ArgState arg_elem(float x, long long i) {
  if (x != x) return {0.f, -1, i};
  return {x, i, -1};
}
__device__ __forceinline__ ArgState arg_combine(ArgState L, ArgState R) {
  if (R.nan >= 0) return R;
  if (L.best < 0) return {R.v, R.best, L.nan};
  if (R.best < 0) return L;
  if (L.v > R.v) return L;  // Greater keeps the earlier; Equal / Less take the later
  return {R.v, R.best, L.nan};
}
__device__ __forceinline__ long long arg_result(ArgState s) { return s.best >= 0 ? s.best : s.nan; }

}  // namespace sq
