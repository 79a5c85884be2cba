// gemm.cu — prefill projections: Y[m][N] = X[m][K] @ W^T for m > 1 rows of f32
// activations against native GGUF weight rows (Q8_0 / Q4_0 / BF16), the m-row
// case of ops/linear.rs:26-37 (kernels/matmul.rs:68-128, which runs one matvec
// per row).
//
// A CTA computes a 64 x BN tile of Y. Each K step is one 32-element quant block:
// the CTA stages the 64 x 32 activation tile and the BN x 32 weight tile in shared
// memory, the weights dequantized to f32 as q * scale (exact: an 8-bit integer
// times an f16 scale has at most 19 significant bits), then every thread
// accumulates a 4 x TN register tile with FMAs. The next K step's tiles are read
// into registers while the current one is multiplied (two shared buffers).
// When the grid would not cover the SMs, K is split across gridDim.z; the partial
// tiles land in a caller-provided workspace and a second kernel sums them in
// split order, so results do not depend on scheduling.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "common.cuh"
#include "ops.cuh"
#include "status.h"

namespace sq {
namespace {

constexpr int GM = 64;        // rows of X per CTA tile
constexpr int GT = 256;       // threads per CTA
constexpr int APAD = GM + 4;  // shared row stride (floats) of the activation tile

template <int T>
constexpr int blk_bytes() {
  return T == SQ_Q8_0 ? Q8_BYTES : (T == SQ_Q4_0 ? Q4_BYTES : BF16_BYTES);
}

// Elements [8*part .. 8*part + EPT) of weight row n's block b, dequantized (q * scale).
template <int T, int EPT>
__device__ __forceinline__ void load_w(const uint8_t *blk, int first, float (&v)[EPT]) {
  if constexpr (T == SQ_Q8_0) {
    const float sc = h2f(ld_u16(blk));
    const uint8_t *q = blk + 2 + first;
#pragma unroll
    for (int i = 0; i < EPT; i += 2) {
      const uint16_t u = ld_u16(q + i);  // 2-byte aligned: blocks are 34 bytes, quants start at byte 2
      v[i] = sc * (float)(int8_t)(u & 0xFF);
      v[i + 1] = sc * (float)(int8_t)(u >> 8);
    }
  } else if constexpr (T == SQ_Q4_0) {
    const float sc = h2f(ld_u16(blk));
    const bool hi = first >= 16;  // elements 16..31 are the high nibbles of bytes 0..15
    const uint8_t *q = blk + 2 + (first & 15);
#pragma unroll
    for (int i = 0; i < EPT; i += 2) {
      const uint16_t u = ld_u16(q + i);
      const int b0 = u & 0xFF, b1 = u >> 8;
      v[i] = sc * (float)((hi ? (b0 >> 4) : (b0 & 15)) - 8);
      v[i + 1] = sc * (float)((hi ? (b1 >> 4) : (b1 & 15)) - 8);
    }
  } else {
    const uint8_t *q = blk + 2 * first;
#pragma unroll
    for (int i = 0; i < EPT; i += 2) {
      const uint32_t u = __ldg(reinterpret_cast<const uint32_t *>(q + 2 * i));
      v[i] = __uint_as_float(u << 16);
      v[i + 1] = __uint_as_float(u & 0xFFFF0000u);
    }
  }
}

template <int T, int BN>
__global__ void __launch_bounds__(GT) k_gemm(const float *__restrict__ x, int m, int K, const uint8_t *__restrict__ w,
                                             int N, float *__restrict__ y, float *__restrict__ part) {
  constexpr int TN = BN / 16;         // columns per thread
  constexpr int EPT = BN * 32 / GT;   // weight elements each thread stages per K step
  constexpr int BPAD = BN + 4;
  constexpr int BB = blk_bytes<T>();
  __shared__ __align__(16) float As[2][32][APAD];
  __shared__ __align__(16) float Bs[2][32][BPAD];
  const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * GM;
  const int nb = K / QK;
  const int kb0 = (int)((long long)nb * blockIdx.z / gridDim.z), kb1 = (int)((long long)nb * (blockIdx.z + 1) / gridDim.z);
  // staging roles: activations (row am, 8 elements from ak), weights (row wn, EPT from wk)
  const int am = tid % GM, ak = (tid / GM) * 8;
  const int wn = tid % BN, wk = (tid / BN) * EPT;
  const bool arow = m0 + am < m, wrow = n0 + wn < N;
  const float *xr = x + (size_t)(m0 + am) * K + ak;
  const uint8_t *wr = w + (size_t)(n0 + wn) * nb * BB;
  float ra[8], rw[EPT];
  auto fetch = [&](int kb) {
    if (arow) {
      const float4 u = __ldg(reinterpret_cast<const float4 *>(xr + (size_t)kb * QK));
      const float4 v = __ldg(reinterpret_cast<const float4 *>(xr + (size_t)kb * QK + 4));
      ra[0] = u.x, ra[1] = u.y, ra[2] = u.z, ra[3] = u.w, ra[4] = v.x, ra[5] = v.y, ra[6] = v.z, ra[7] = v.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; i++) ra[i] = 0.f;
    }
    if (wrow) {
      load_w<T, EPT>(wr + (size_t)kb * BB, wk, rw);
    } else {
#pragma unroll
      for (int i = 0; i < EPT; i++) rw[i] = 0.f;
    }
  };
  auto stash = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 8; i++) As[buf][ak + i][am] = ra[i];
#pragma unroll
    for (int i = 0; i < EPT; i++) Bs[buf][wk + i][wn] = rw[i];
  };
  float acc[4][TN];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < TN; j++) acc[i][j] = 0.f;
  if (kb0 < kb1) {
    fetch(kb0);
    stash(0);
    __syncthreads();
    for (int kb = kb0; kb < kb1; kb++) {
      const int buf = (kb - kb0) & 1;
      if (kb + 1 < kb1) fetch(kb + 1);
#pragma unroll 8
      for (int k = 0; k < 32; k++) {
        const float4 a = *reinterpret_cast<const float4 *>(&As[buf][k][ty * 4]);
        float b[TN];
        if constexpr (TN == 4) {
          const float4 u = *reinterpret_cast<const float4 *>(&Bs[buf][k][tx * 4]);
          b[0] = u.x, b[1] = u.y, b[2] = u.z, b[3] = u.w;
        } else {
          const float2 u = *reinterpret_cast<const float2 *>(&Bs[buf][k][tx * 2]);
          b[0] = u.x, b[1] = u.y;
        }
        const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
          for (int j = 0; j < TN; j++) acc[i][j] = fmaf(av[i], b[j], acc[i][j]);
      }
      if (kb + 1 < kb1) {
        stash(buf ^ 1);
        __syncthreads();
      }
    }
  }
  float *out = gridDim.z > 1 ? part + (size_t)blockIdx.z * m * N : y;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int mm = m0 + ty * 4 + i;
    if (mm >= m) continue;
#pragma unroll
    for (int j = 0; j < TN; j++) {
      const int nn = n0 + tx * TN + j;
      if (nn < N) out[(size_t)mm * N + nn] = acc[i][j];
    }
  }
}

// y = sum over splits of part, in split order.
__global__ void k_split_sum(const float *__restrict__ part, int splits, size_t n, float *__restrict__ y) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    float s = part[i];
    for (int z = 1; z < splits; z++) s += part[(size_t)z * n + i];
    y[i] = s;
  }
}

template <int T, int BN>
cudaError_t gemm_t(cudaStream_t s, const float *x, int m, int K, const uint8_t *w, int N, float *y, int splits,
                   float *part) {
  const dim3 grid((N + BN - 1) / BN, (m + GM - 1) / GM, splits);
  k_gemm<T, BN><<<grid, GT, 0, s>>>(x, m, K, w, N, y, part);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || splits == 1) return e;
  const size_t n = (size_t)m * N;
  k_split_sum<<<(unsigned)std::min<size_t>((n + 255) / 256, 4096), 256, 0, s>>>(part, splits, n, y);
  return cudaGetLastError();
}

int g_sms = 0;

}  // namespace

cudaError_t launch_gemm_f32w(cudaStream_t s, const float *x, int m, int K, const void *w, int wtype, int N, float *y,
                             float *ws, size_t ws_floats) {
  if (!g_sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_sms <= 0) g_sms = 148;
  }
  const int target = 2 * g_sms;
  const int mt = (m + GM - 1) / GM;
  const bool wide = (long long)((N + 63) / 64) * mt >= target;
  const long long tiles = wide ? (long long)((N + 63) / 64) * mt : (long long)((N + 31) / 32) * mt;
  int splits = 1;
  if (ws && tiles < target) {
    splits = (int)std::min<long long>((target + tiles - 1) / tiles, 8);
    splits = std::min(splits, std::max(1, K / QK / 8));  // at least 8 blocks per split
    while (splits > 1 && (size_t)splits * m * N > ws_floats) splits--;
  }
  const uint8_t *wb = (const uint8_t *)w;
  switch (wtype) {
    case SQ_Q8_0:
      return wide ? gemm_t<SQ_Q8_0, 64>(s, x, m, K, wb, N, y, splits, ws) : gemm_t<SQ_Q8_0, 32>(s, x, m, K, wb, N, y, splits, ws);
    case SQ_Q4_0:
      return wide ? gemm_t<SQ_Q4_0, 64>(s, x, m, K, wb, N, y, splits, ws) : gemm_t<SQ_Q4_0, 32>(s, x, m, K, wb, N, y, splits, ws);
    default:
      return wide ? gemm_t<SQ_BF16, 64>(s, x, m, K, wb, N, y, splits, ws) : gemm_t<SQ_BF16, 32>(s, x, m, K, wb, N, y, splits, ws);
  }
}

}  // namespace sq
