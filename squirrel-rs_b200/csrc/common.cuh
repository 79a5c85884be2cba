// common.cuh — shared device helpers: exact dequant, warp reductions, greedy fold state.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "status.h"

namespace sq {

// ---- device helpers ---------------------------------------------------------------

// Programmatic dependent launch. A kernel launched with programmatic stream
// serialization may start while the previous kernel of the stream is still running;
// every thread calls pdl_wait() before it reads anything an earlier kernel wrote or
// writes anything an earlier kernel may still read (it returns at once for a plain
// launch). pdl_trigger() lets the next such kernel be scheduled early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

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


// Words of one lane's block pair: Q8_0 / Q4_0 two 34 / 18-byte blocks (68 / 36 bytes,
// 4-byte aligned when the pair is), BF16 two 64-byte blocks.
template <int T>
constexpr int pair_words() {
  return T == SQ_Q8_0 ? 17 : (T == SQ_Q4_0 ? 9 : 32);
}

// Packed f32x2 arithmetic (sm_100): one instruction does two lanes' worth of the
// float work, element pairs (2j, 2j+1) sharing a 64-bit register.
typedef unsigned long long f2x;
__device__ __forceinline__ f2x pk2(float a, float b) {
  f2x r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ f2x pk2u(uint32_t a, uint32_t b) {
  f2x r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ float2 up2(f2x v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ f2x ffma2(f2x a, f2x b, f2x c) {
  f2x d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ f2x fadd2(f2x a, f2x b) {
  f2x d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2x fmul2(f2x a, f2x b) {
  f2x d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float hsum2(f2x a, f2x b) {  // (a.x + a.y) + (b.x + b.y)
  const float2 u = up2(a), v = up2(b);
  return (u.x + u.y) + (v.x + v.y);
}

// Bytes b0, b1 of one word -> two exact floats (as q8f / nibf).
__device__ __forceinline__ f2x q8f2(uint32_t wx, int b0, int b1) {
  const f2x bias = pk2(-8388736.0f, -8388736.0f);
  return fadd2(pk2u(__byte_perm(wx, 0x4B000000u, 0x7540u | (unsigned)b0), __byte_perm(wx, 0x4B000000u, 0x7540u | (unsigned)b1)),
               bias);
}
__device__ __forceinline__ f2x nibf2(uint32_t nib4, int b0, int b1) {
  const f2x bias = pk2(-8388616.0f, -8388616.0f);
  return fadd2(pk2u(__byte_perm(nib4, 0x4B000000u, 0x7540u | (unsigned)b0), __byte_perm(nib4, 0x4B000000u, 0x7540u | (unsigned)b1)),
               bias);
}

// Dot of the lane's 64 activations (x2[j] = elements 2j, 2j+1) with its 64 weights
// (f32 activations: W8A32 / W4A32 / BF16 — dot_prod.rs:86-96, 255-270, 464-472; per
// block the products are summed first and scaled once).
template <int T>
__device__ __forceinline__ float pair_dot(const uint32_t (&w)[pair_words<T>()], const f2x (&x2)[32]) {
  if constexpr (T == SQ_Q8_0) {
    const float s0 = __half2float(__ushort_as_half((unsigned short)(w[0] & 0xFFFF)));
    const float s1 = __half2float(__ushort_as_half((unsigned short)(w[8] >> 16)));
    f2x a[2] = {0ull, 0ull}, b[2] = {0ull, 0ull};
#pragma unroll
    for (int i = 0; i < 32; i += 2) {  // block 0: bytes 2..33 (a pair's bytes share a word)
      const int c0 = 2 + i;
      const uint32_t wx = w[c0 >> 2] ^ 0x80808080u;
      a[(i >> 1) & 1] = ffma2(x2[i >> 1], q8f2(wx, c0 & 3, (c0 & 3) + 1), a[(i >> 1) & 1]);
    }
#pragma unroll
    for (int i = 0; i < 32; i += 2) {  // block 1: bytes 36..67
      const int c0 = 36 + i;
      const uint32_t wx = w[c0 >> 2] ^ 0x80808080u;
      b[(i >> 1) & 1] = ffma2(x2[16 + (i >> 1)], q8f2(wx, c0 & 3, (c0 & 3) + 1), b[(i >> 1) & 1]);
    }
    return fmaf(hsum2(a[0], a[1]), s0, hsum2(b[0], b[1]) * s1);
  } else if constexpr (T == SQ_Q4_0) {
    const float s0 = __half2float(__ushort_as_half((unsigned short)(w[0] & 0xFFFF)));
    const float s1 = __half2float(__ushort_as_half((unsigned short)(w[4] >> 16)));
    f2x a[2] = {0ull, 0ull}, b[2] = {0ull, 0ull};
#pragma unroll
    for (int j = 0; j < 16; j += 2) {  // block 0: quant bytes 2..17 (element j low nibble, j+16 high)
      const int c0 = 2 + j;               // even: the pair's two bytes share a word
      const uint32_t w0 = w[c0 >> 2];
      a[0] = ffma2(x2[j >> 1], nibf2(w0 & 0x0F0F0F0Fu, c0 & 3, (c0 & 3) + 1), a[0]);
      a[1] = ffma2(x2[8 + (j >> 1)], nibf2((w0 >> 4) & 0x0F0F0F0Fu, c0 & 3, (c0 & 3) + 1), a[1]);
    }
#pragma unroll
    for (int j = 0; j < 16; j += 2) {  // block 1: quant bytes 20..35
      const int c0 = 20 + j;
      const uint32_t w0 = w[c0 >> 2];
      b[0] = ffma2(x2[16 + (j >> 1)], nibf2(w0 & 0x0F0F0F0Fu, c0 & 3, (c0 & 3) + 1), b[0]);
      b[1] = ffma2(x2[24 + (j >> 1)], nibf2((w0 >> 4) & 0x0F0F0F0Fu, c0 & 3, (c0 & 3) + 1), b[1]);
    }
    return fmaf(hsum2(a[0], a[1]), s0, hsum2(b[0], b[1]) * s1);
  } else {
    f2x a[2] = {0ull, 0ull};
#pragma unroll
    for (int k = 0; k < 8; k++) {
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const uint32_t u = w[4 * k + j];
        a[j & 1] = ffma2(x2[4 * k + j], pk2u(u << 16, u & 0xFFFF0000u), a[j & 1]);
      }
    }
    return hsum2(a[0], a[1]);
  }
}

// 4-byte / 16-byte shared-memory loads by 32-bit shared address.
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}

// Sum four values over the warp: a butterfly that halves the values it carries at
// each of the first two steps (6 shuffles in all, against 4 x 5 for four separate
// sums), then every lane gets all four totals.
__device__ __forceinline__ void warp_sum4(float (&v)[4]) {
  const int lane = threadIdx.x & 31;
  const bool b4 = lane & 16, b3 = lane & 8;
  float k0 = b4 ? v[2] : v[0], k1 = b4 ? v[3] : v[1];
  const float s0 = b4 ? v[0] : v[2], s1 = b4 ? v[1] : v[3];
  k0 += __shfl_xor_sync(0xffffffffu, s0, 16);
  k1 += __shfl_xor_sync(0xffffffffu, s1, 16);
  float k = b3 ? k1 : k0;
  k += __shfl_xor_sync(0xffffffffu, b3 ? k0 : k1, 8);
  k += __shfl_xor_sync(0xffffffffu, k, 4);
  k += __shfl_xor_sync(0xffffffffu, k, 2);
  k += __shfl_xor_sync(0xffffffffu, k, 1);
  // lanes 8g .. 8g+7 now hold the total of value g
#pragma unroll
  for (int r = 0; r < 4; r++) v[r] = __shfl_sync(0xffffffffu, k, 8 * r);
}

// Launch kernel k on stream s, with programmatic stream serialization when pdl (the
// kernel must then call pdl_wait() as described above).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_ex(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                             Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

}  // namespace sq
