// gemm_tc.cu — tensor-core prefill projections for BF16 weights:
// Y[m][N] = X[m][K] @ W^T with f32 activations X and bf16 weight rows W (GGUF BF16),
// the m-row case of ops/linear.rs:26-37 (kernels/matmul.rs:68-128 runs one f32
// matvec per row; the bf16 weights are widened to f32 exactly).
//
// Accuracy: every f32 activation is split into three bf16 terms x = h + d + l
// (h = bf16(x), d = bf16(x - h), l = bf16(x - h - d); each difference is exact and
// the three terms carry all 24 significant bits), so W·x = W·h + W·d + W·l exactly in
// real arithmetic. Products of two bf16 values are exact; the tensor core sums them
// in an f32 accumulator. The split runs once per call (k_split3) into a workspace
// laid out [3][m][K] bf16.
//
// Kernel (one 128 x BN output tile per CTA, 4 warps):
//   warp 0   TMA producer: per 64-element K block, the 128 x 64 weight tile and the
//            three BN x 64 activation-term tiles, 128-byte swizzled, into a ring of
//            shared-memory stages completing on an mbarrier;
//   warp 1   one thread issues tcgen05.mma (kind::f16, bf16 inputs, f32 accumulator
//            in tensor memory, M = 128 weight rows, N = BN rows of X), three terms x
//            four K steps of 16 per stage, then tcgen05.commit frees the stage;
//   all      epilogue: tcgen05.ld of the accumulator (lane = weight row, column =
//            activation row), coalesced f32 stores of Y (or of a split-K partial).
// K is split across gridDim.z when the tiles alone do not cover the SMs; partials
// are summed in split order by k_split_sum (deterministic).
// Every mbarrier wait is bounded; on expiry the CTA records an error, drains its
// copies in flight, frees its tensor memory and returns (gemm_tc_status()).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <mutex>

#include "ops.cuh"
#include "status.h"
#include "tc.cuh"

namespace sq {
namespace {

using namespace tc;

constexpr int TC_M = 128;       // weight rows per tile (MMA M)
constexpr int TC_KB = 64;       // K elements per stage: one 128-byte swizzle row of bf16
constexpr int TC_TERMS = 3;     // bf16 terms per f32 activation
constexpr int TC_THREADS = 128;

__device__ unsigned g_tc_err;  // set when a bounded wait of a tensor-core kernel gave up

template <int BN>
struct TcCfg {
  static constexpr int A_BYTES = TC_M * TC_KB * 2;     // 16 KB weight tile
  static constexpr int B_BYTES = BN * TC_KB * 2;       // one activation-term tile
  static constexpr int STAGE = A_BYTES + TC_TERMS * B_BYTES;
  static constexpr int STAGES = BN >= 256 ? 2 : (BN >= 128 ? 3 : 5);
  static constexpr int BAR_OFF = STAGES * STAGE;       // mbarriers after the stages
  static constexpr int SMEM = 1024 + BAR_OFF + 128;    // + alignment slack
  static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;  // f32 accumulator: one column per activation row
  static constexpr uint32_t IDESC = idesc_bf16(TC_M, BN);
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "MMA N for M = 128");
  static_assert(B_BYTES % 1024 == 0 && A_BYTES % 1024 == 0, "tiles keep 1024-byte swizzle alignment");
  static_assert(SMEM <= 232448, "shared memory per CTA");
};

// grid: (ceil(N/128), ceil(m/BN), splits). kb_per: K blocks of 64 per split.
template <int BN>
__global__ void __launch_bounds__(TC_THREADS, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx, int m, int N,
              int nkb, int kb_per, float *__restrict__ y, float *__restrict__ part, unsigned *err) {
  using C = TcCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = su32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // swizzled tiles start on 1024-byte boundaries
  const uint32_t bars = base + C::BAR_OFF;       // full[STAGES], empty[STAGES], done, tmem slot, abort
  auto full = [&](int s) { return bars + 8u * s; };
  auto empty = [&](int s) { return bars + 8u * (C::STAGES + s); };
  const uint32_t done = bars + 8u * (2 * C::STAGES);
  uint8_t *gen = smem_raw + (base - raw);  // generic pointer to the aligned base
  volatile uint32_t *tmem_slot = (volatile uint32_t *)(gen + C::BAR_OFF + 8 * (2 * C::STAGES + 1));
  volatile int *abort_flag = (volatile int *)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int f0 = blockIdx.x * TC_M, t0 = blockIdx.y * BN;
  const int kb0 = blockIdx.z * kb_per;
  const int nk = min(nkb, kb0 + kb_per) - kb0;  // >= 1 (the host sizes the splits)

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; s++) {
      bar_init(full(s), 1);
      bar_init(empty(s), 1);
    }
    bar_init(done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_map(&tw);
    prefetch_map(&tx);
  }
  __syncwarp();
  if (warp == 0) tmem_alloc(su32((const void *)tmem_slot), C::TMEM_COLS);  // the whole warp
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  int issued = 0;  // producer: K blocks whose copies were started
  if (warp == 0) {
    for (int i = 0; i < nk; i++) {
      const int s = i % C::STAGES;
      int ok = 1;
      if (lane == 0) {
        if (i >= C::STAGES) ok = bar_wait(empty(s), (unsigned)((i / C::STAGES) - 1) & 1u, err, abort_flag);
        if (ok) {
          const uint32_t a = base + (uint32_t)s * C::STAGE;
          const int k = (kb0 + i) * TC_KB;
          bar_expect_tx(full(s), (unsigned)C::STAGE);
          tma_load_2d(a, &tw, k, f0, full(s));
#pragma unroll
          for (int t = 0; t < TC_TERMS; t++)
            tma_load_3d(a + C::A_BYTES + (uint32_t)t * C::B_BYTES, &tx, k, t0, t, full(s));
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      issued = i + 1;
    }
  } else if (warp == 1) {
    for (int i = 0; i < nk; i++) {
      const int s = i % C::STAGES;
      int ok = 1;
      if (lane == 0) {
        ok = bar_wait(full(s), (unsigned)(i / C::STAGES) & 1u, err, abort_flag);
        if (ok) {
          fence_after();
          const uint32_t a = base + (uint32_t)s * C::STAGE;
#pragma unroll
          for (int t = 0; t < TC_TERMS; t++) {
            const uint32_t b = a + C::A_BYTES + (uint32_t)t * C::B_BYTES;
#pragma unroll
            for (int kk = 0; kk < TC_KB / 16; kk++)
              mma_bf16(tmem, sw128_desc(a + 32u * kk), sw128_desc(b + 32u * kk), C::IDESC,
                       (i | t | kk) != 0 ? 1u : 0u);
          }
          mma_commit(empty(s));  // the stage is free once these MMAs have read it
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
    }
    if (lane == 0) mma_commit(done);  // arrives when every MMA above has completed
    __syncwarp();
  }

  // Epilogue: every warp reads its 32 accumulator lanes (weight rows f0+32*warp ..).
  int ok = 1;
  if (lane == 0) ok = bar_wait(done, 0u, err, abort_flag);
  ok = __shfl_sync(0xffffffffu, ok, 0);
  fence_after();
  if (ok && !*abort_flag) {
    float *out = part ? part + (size_t)blockIdx.z * m * N : y;
    const int f = f0 + 32 * warp + lane;
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      if (t0 + c >= m) break;  // warp-uniform
      uint32_t r[16];
      tmem_ld16(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)c, r);
      tmem_wait_ld(r);
      if (f < N) {
#pragma unroll
        for (int j = 0; j < 16; j++) {
          const int t = t0 + c + j;
          if (t < m) out[(size_t)t * N + f] = __uint_as_float(r[j]);
        }
      }
    }
  }
  // Drain (only after an abort): copies started but not consumed land before the
  // CTA's shared memory goes away, and the MMAs finish before the columns are freed.
  if (warp == 0 && lane == 0) {
    for (int i = std::max(0, issued - C::STAGES); i < issued; i++) bar_drain(full(i % C::STAGES), (unsigned)(i / C::STAGES) & 1u);
  }
  if (warp == 1 && lane == 0) bar_drain(done, 0u);
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// xs[t][r][k] (t = 0, 1, 2): the three bf16 terms of x[r][k]; n = m*K elements,
// plane = n, four elements per thread (n % 4 == 0).
__global__ void k_split3(const float4 *__restrict__ x, size_t n4, __nv_bfloat16 *__restrict__ xs, size_t plane) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    const float4 v = x[i];
    const float in[4] = {v.x, v.y, v.z, v.w};
    __nv_bfloat16 h[4], d[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      h[j] = __float2bfloat16_rn(in[j]);
      const float r1 = in[j] - __bfloat162float(h[j]);
      d[j] = __float2bfloat16_rn(r1);
      const float r2 = r1 - __bfloat162float(d[j]);
      l[j] = __float2bfloat16_rn(r2);
    }
    uint2 *o = reinterpret_cast<uint2 *>(xs + 4 * i);
    auto pack = [](const __nv_bfloat16 (&a)[4]) {
      uint2 u;
      u.x = (uint32_t)__bfloat16_as_ushort(a[0]) | ((uint32_t)__bfloat16_as_ushort(a[1]) << 16);
      u.y = (uint32_t)__bfloat16_as_ushort(a[2]) | ((uint32_t)__bfloat16_as_ushort(a[3]) << 16);
      return u;
    };
    o[0] = pack(h);
    o[plane / 4] = pack(d);
    o[plane / 2] = pack(l);
  }
}

__global__ void k_split_sum_tc(const float *__restrict__ part, int splits, size_t n, float *__restrict__ y) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    float s = part[i];
    for (int z = 1; z < splits; z++) s += part[(size_t)z * n + i];
    y[i] = s;
  }
}

}  // namespace

// Device address of the error word of the tensor-core kernels on the current device.
unsigned *tc_err_ptr() {
  static unsigned *ptrs[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  if (!ptrs[dev]) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_tc_err) != cudaSuccess) return nullptr;
    ptrs[dev] = (unsigned *)p;
  }
  return ptrs[dev];
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
int g_sms_tc = 0;
std::once_flag g_once;

void init_once() {
  std::call_once(g_once, [] {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sms_tc, cudaDevAttrMultiProcessorCount, dev);
    if (g_sms_tc <= 0) g_sms_tc = 148;
  });
}

// A bf16 tensor map with a 64-element (128-byte) inner box, 128-byte swizzle and
// zero fill outside the tensor.
bool encode(CUtensorMap *map, const void *ptr, int rank, const cuuint64_t *dims, const cuuint64_t *strides,
            const cuuint32_t *box) {
  const cuuint32_t es[3] = {1, 1, 1};
  return g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)rank, const_cast<void *>(ptr), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN>
cudaError_t run_tc(cudaStream_t s, const __nv_bfloat16 *xs, int m, int K, const void *w, int N, float *y,
                   int splits, float *part) {
  using C = TcCfg<BN>;
  CUtensorMap tw, tx;
  const cuuint64_t wd[2] = {(cuuint64_t)K, (cuuint64_t)N}, ws_[1] = {(cuuint64_t)K * 2};
  const cuuint32_t wb[2] = {TC_KB, TC_M};
  const cuuint64_t xd[3] = {(cuuint64_t)K, (cuuint64_t)m, TC_TERMS},
                   xst[2] = {(cuuint64_t)K * 2, (cuuint64_t)m * K * 2};
  const cuuint32_t xb[3] = {TC_KB, BN, 1};
  if (!encode(&tw, w, 2, wd, ws_, wb) || !encode(&tx, xs, 3, xd, xst, xb)) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(k_gemm_tc<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const int nkb = (K + TC_KB - 1) / TC_KB;
  const int kb_per = (nkb + splits - 1) / splits;
  splits = (nkb + kb_per - 1) / kb_per;  // every split gets at least one block
  const dim3 grid((N + TC_M - 1) / TC_M, (m + BN - 1) / BN, splits);
  k_gemm_tc<BN><<<grid, TC_THREADS, C::SMEM, s>>>(tw, tx, m, N, nkb, kb_per, y, splits > 1 ? part : nullptr,
                                                  tc_err_ptr());
  e = cudaGetLastError();
  if (e != cudaSuccess || splits == 1) return e;
  const size_t n = (size_t)m * N;
  k_split_sum_tc<<<(unsigned)std::min<size_t>((n + 255) / 256, 4096), 256, 0, s>>>(part, splits, n, y);
  return cudaGetLastError();
}

}  // namespace

bool gemm_tc_supported(int m, int K, const float *x, const void *w, int wtype, const float *ws, size_t ws_floats) {
  init_once();
  return g_encode && wtype == SQ_BF16 && m >= 2 && K % 16 == 0 && x && ws && ((uintptr_t)x & 15) == 0 &&
         ((uintptr_t)w & 15) == 0 && ((uintptr_t)ws & 255) == 0 && (size_t)3 * m * K / 2 + 64 <= ws_floats;
}

cudaError_t launch_gemm_tc_bf16(cudaStream_t s, const float *x, int m, int K, const void *w, int N, float *y,
                                float *ws, size_t ws_floats) {
  if (!gemm_tc_supported(m, K, x, w, SQ_BF16, ws, ws_floats)) return cudaErrorNotSupported;
  // workspace: [3][m][K] bf16 terms, then split-K partials (256-byte aligned)
  __nv_bfloat16 *xs = reinterpret_cast<__nv_bfloat16 *>(ws);
  const size_t xs_floats = ((size_t)3 * m * K / 2 + 63) & ~(size_t)63;
  float *part = ws + xs_floats;
  const size_t part_floats = ws_floats - xs_floats;
  const size_t n = (size_t)m * K;  // a multiple of 16
  k_split3<<<(unsigned)std::min<size_t>((n / 4 + 255) / 256, 8 * (size_t)g_sms_tc), 256, 0, s>>>(
      reinterpret_cast<const float4 *>(x), n / 4, xs, n);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int ft = (N + TC_M - 1) / TC_M;
  const int nkb = (K + TC_KB - 1) / TC_KB;
  const bool wide = (long long)ft * ((m + 127) / 128) >= g_sms_tc;
  const long long tiles = wide ? (long long)ft * ((m + 127) / 128) : (long long)ft * ((m + 63) / 64);
  int splits = 1;
  if (tiles < g_sms_tc) {
    splits = (int)std::min<long long>((g_sms_tc + tiles - 1) / tiles, 8);
    splits = std::min(splits, std::max(1, nkb / 4));  // at least 4 K blocks per split
    while (splits > 1 && (size_t)splits * m * N > part_floats) splits--;
  }
  return wide ? run_tc<128>(s, xs, m, K, w, N, y, splits, part) : run_tc<64>(s, xs, m, K, w, N, y, splits, part);
}

bool gemm_tc_enabled() {
  static const bool on = [] {
    const char *v = getenv("SQB200_GEMM");
    return !(v && strcmp(v, "simt") == 0);
  }();
  return on;
}

unsigned gemm_tc_status(bool clear) {
  unsigned v = 0;
  cudaMemcpyFromSymbol(&v, g_tc_err, sizeof(v));
  if (clear && v) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(g_tc_err, &z, sizeof(z));
  }
  return v;
}

}  // namespace sq
