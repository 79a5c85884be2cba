// gemm_tc.cu — tensor-core prefill projections: Y[m][N] = X[m][K] @ W^T with f32
// activations X and native GGUF weight rows W (BF16, Q8_0, Q4_0), the m-row case of
// ops/linear.rs:26-37 (kernels/matmul.rs:68-128 runs one f32 matvec per row).
// k_gemm_tc serves BF16 rows (widened to f32 exactly by the reference); k_gemm_tcq
// serves Q8_0 / Q4_0 rows with per-block scaling (further below).
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
//   warps 1-3  one thread each issues tcgen05.mma (kind::f16, bf16 inputs, f32
//            accumulator in tensor memory, M = 128 weight rows, N = BN rows of X) for
//            one activation term into that term's own accumulator, four K steps of
//            16 per stage, then tcgen05.commit; the stage is free once all three
//            have committed;
//   all      epilogue: tcgen05.ld of the three accumulators (lane = weight row,
//            column = activation row), summed in a fixed order (deterministic),
//            coalesced f32 stores of Y (or of a split-K partial).
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
  // one f32 accumulator per activation term (one column per activation row each)
  static constexpr int TMEM_COLS = TC_TERMS * BN <= 32 ? 32 : (TC_TERMS * BN <= 64 ? 64 : (TC_TERMS * BN <= 128 ? 128 : (TC_TERMS * BN <= 256 ? 256 : 512)));
  static constexpr uint32_t IDESC = idesc_bf16(TC_M, BN);
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "MMA N for M = 128");
  static_assert(B_BYTES % 1024 == 0 && A_BYTES % 1024 == 0, "tiles keep 1024-byte swizzle alignment");
  static_assert(SMEM <= 232448, "shared memory per CTA");
};

// Up to three weight matrices that share one input (q / k / v, gate / up): one launch
// covers all their 128-row tiles, tile x of matrix i for blockIdx.x in [t[i], t[i+1]).
struct TcW {
  CUtensorMap map[3];
  float *y[3];
  int N[3];
  int t[4];  // first tile of each matrix; t[3] = the grid's x extent
};

// grid: (tiles of all matrices, ceil(m/BN), splits). kb_per: K blocks of 64 per split
// (split-K only with one matrix).
template <int BN>
__global__ void __launch_bounds__(TC_THREADS, 1)
    k_gemm_tc(const __grid_constant__ TcW W, const __grid_constant__ CUtensorMap tx, int m, int nkb, int kb_per,
              float *__restrict__ part, unsigned *err) {
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
  const int bx = blockIdx.x, mi = bx < W.t[1] ? 0 : (bx < W.t[2] ? 1 : 2);  // this tile's matrix
  const CUtensorMap *tw = &W.map[mi];
  const int N = W.N[mi];
  float *__restrict__ y = W.y[mi];
  const int f0 = (bx - W.t[mi]) * TC_M, t0 = blockIdx.y * BN;
  const int kb0 = blockIdx.z * kb_per;
  const int nk = min(nkb, kb0 + kb_per) - kb0;  // >= 1 (the host sizes the splits)

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; s++) {
      bar_init(full(s), 1);
      bar_init(empty(s), TC_TERMS);  // one commit per issuing thread
    }
    bar_init(done, TC_TERMS);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_map(tw);
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
          tma_load_2d(a, tw, k, f0, full(s));
#pragma unroll
          for (int t = 0; t < TC_TERMS; t++)
            tma_load_3d(a + C::A_BYTES + (uint32_t)t * C::B_BYTES, &tx, k, t0, t, full(s));
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      issued = i + 1;
    }
  } else {
    // warps 1-3: one issuing thread per activation term (term t = warp - 1), each
    // into its own accumulator (columns t*BN ..)
    const int t = warp - 1;
    for (int i = 0; i < nk; i++) {
      const int s = i % C::STAGES;
      int ok = 1;
      if (lane == 0) {
        ok = bar_wait(full(s), (unsigned)(i / C::STAGES) & 1u, err, abort_flag);
        if (ok) {
          fence_after();
          const uint32_t a = base + (uint32_t)s * C::STAGE;
          const uint32_t b = a + C::A_BYTES + (uint32_t)t * C::B_BYTES;
#pragma unroll
          for (int kk = 0; kk < TC_KB / 16; kk++)
            mma_bf16(tmem + (uint32_t)(t * BN), sw128_desc(a + 32u * kk), sw128_desc(b + 32u * kk), C::IDESC,
                     (i | kk) != 0 ? 1u : 0u);
          mma_commit(empty(s));  // the stage is free once all three threads' MMAs have read it
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
    }
    if (lane == 0) mma_commit(done);  // arrives when every MMA of this thread has completed
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
      uint32_t r[3][16];
      const uint32_t lb = tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)c;
      tmem_ld16(lb, r[0]);
      tmem_ld16(lb + BN, r[1]);
      tmem_ld16(lb + 2 * BN, r[2]);
      tmem_wait_ld(r[0]);
      tmem_tie(r[1]);
      tmem_tie(r[2]);
      if (f < N) {
#pragma unroll
        for (int j = 0; j < 16; j++) {
          const int t = t0 + c + j;  // the terms' sums in a fixed order: deterministic
          const float v = (__uint_as_float(r[0][j]) + __uint_as_float(r[1][j])) + __uint_as_float(r[2][j]);
          if (t < m) out[(size_t)t * N + f] = v;
        }
      }
    }
  }
  // Drain (only after an abort): copies started but not consumed land before the
  // CTA's shared memory goes away, and the MMAs finish before the columns are freed.
  if (warp == 0 && lane == 0) {
    for (int i = std::max(0, issued - C::STAGES); i < issued; i++) bar_drain(full(i % C::STAGES), (unsigned)(i / C::STAGES) & 1u);
  }
  if (warp >= 1 && lane == 0) bar_drain(done, 0u);
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------
// Q8_0 / Q4_0 weights (kernels/dot_prod.rs W8A32 / W4A32: each 32-element block's
// products are summed, then the sum is multiplied by the block's f16 scale and added
// to the row's f32 accumulator). The quants become exact bf16 values for the MMA;
// each block's sum over the three activation terms lands in its own tensor-memory
// buffer (four in rotation); the epilogue threads fold sum * scale into f32
// registers block by block, in block order.
//
// Warps 0-3: thread r owns weight row f0 + r: converts its row of each 64-element
// step from the raw block bytes into the 128-byte swizzled bf16 A tile, and folds the
// block sums of tensor-memory lane r. Warp 4: TMA of the raw weight rows (eight
// blocks = 256 elements per copy, 128 rows, one chunk ahead) and of the activation
// terms. Warp 5: MMA issue (one thread: the block sums keep a fixed order).
// ---------------------------------------------------------------------------------
constexpr int Q_CHUNK = 256;  // K elements per raw weight copy (eight blocks)
constexpr int Q_THREADS = 192;  // 6 warps: at most 2 per SM sub-partition, so 255 registers fit

template <int T, int BN>
struct QCfg {
  static constexpr int BB = T == SQ_Q8_0 ? Q8_BYTES : Q4_BYTES;
  static constexpr int CB = 8 * BB;                   // bytes of one row's chunk: 272 / 144
  static constexpr int RAW = TC_M * CB;               // 34816 / 18432: multiples of 1024
  static constexpr int A_TILE = TC_M * TC_KB * 2;     // 16 KB
  static constexpr int B_TERM = BN * TC_KB * 2;
  static constexpr int B_STAGE = TC_TERMS * B_TERM;
  static constexpr int NB = BN >= 128 ? 2 : 3;        // activation-term stages
  static constexpr int OFF_RAW = 0;
  static constexpr int OFF_A = 2 * RAW;
  static constexpr int OFF_B = OFF_A + 2 * A_TILE;
  static constexpr int OFF_BAR = OFF_B + NB * B_STAGE;
  static constexpr int SMEM = 1024 + OFF_BAR + 256;
  static constexpr int NP = 4;                        // tensor-memory block-sum buffers
  static constexpr uint32_t TMEM_COLS = NP * BN < 32 ? 32 : NP * BN;
  static constexpr uint32_t IDESC = idesc_bf16(TC_M, BN);
  static_assert(RAW % 1024 == 0 && B_TERM % 1024 == 0, "1024-byte tile alignment");
  static_assert(SMEM <= 232448, "shared memory per CTA");
  static_assert(TMEM_COLS <= 512, "tensor memory columns");
};

// barrier slots
enum : int {
  QB_RAWFULL = 0,   // [2]
  QB_RAWEMPTY = 2,  // [2]
  QB_AFULL = 4,     // [2]
  QB_AEMPTY = 6,    // [2]
  QB_PFULL = 8,     // [4]
  QB_PEMPTY = 12,   // [4]
  QB_FIN = 16,
  QB_BFULL = 17,    // [NB]
  QB_BEMPTY = 20,   // [NB]
  QB_N = 23
};

__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t a) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return v;
}
// four unsigned bytes b (value b + bias_off) of u -> two bf16x2 words of (b - bias), exact
__device__ __forceinline__ void bytes_to_bf16(uint32_t u, float bias, uint32_t &lo, uint32_t &hi) {
  const float f0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440)) - bias;
  const float f1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441)) - bias;
  const float f2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442)) - bias;
  const float f3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443)) - bias;
  const __nv_bfloat162 a = __floats2bfloat162_rn(f0, f1), b = __floats2bfloat162_rn(f2, f3);
  lo = *reinterpret_cast<const uint32_t *>(&a);
  hi = *reinterpret_cast<const uint32_t *>(&b);
}
// Four bytes starting at shared address a (2-byte aligned).
__device__ __forceinline__ uint32_t lds_4at(uint32_t a) {
  if (a & 2u) return __byte_perm(lds_u32(a - 2), lds_u32(a + 2), 0x5432);
  return lds_u32(a);
}

// Row r's 64 elements of blocks (2*sub, 2*sub + 1) of the raw chunk at `row` into
// the swizzled A tile row at `dst` (chunk c of 8 elements at c ^ (r % 8)).
template <int T>
__device__ __forceinline__ void convert_step(uint32_t row, int sub, uint32_t dst, int r7) {
  constexpr int BB = T == SQ_Q8_0 ? Q8_BYTES : Q4_BYTES;
#pragma unroll
  for (int c = 0; c < 8; c++) {
    const int blk = 2 * sub + c / 4;
    uint32_t w0, w1;
    float bias;
    if constexpr (T == SQ_Q8_0) {  // elements 8*(c%4) .. +7 of block blk: int8, stored as value + 128
      const uint32_t a = row + (uint32_t)(blk * BB + 2 + 8 * (c % 4));
      w0 = lds_4at(a) ^ 0x80808080u;
      w1 = lds_4at(a + 4) ^ 0x80808080u;
      bias = 8388736.0f;  // 2^23 + 128
    } else {  // low nibbles of bytes 0..15 are elements 0..15, high nibbles 16..31; value = nibble - 8
      const int hi = (c % 4) / 2, part = c % 2;
      const uint32_t a = row + (uint32_t)(blk * BB + 2 + 8 * part);
      const uint32_t b0 = lds_4at(a), b1 = lds_4at(a + 4);
      w0 = hi ? (b0 >> 4) & 0x0F0F0F0Fu : b0 & 0x0F0F0F0Fu;
      w1 = hi ? (b1 >> 4) & 0x0F0F0F0Fu : b1 & 0x0F0F0F0Fu;
      bias = 8388616.0f;  // 2^23 + 8
    }
    uint32_t v0, v1, v2, v3;
    bytes_to_bf16(w0, bias, v0, v1);
    bytes_to_bf16(w1, bias, v2, v3);
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst + (uint32_t)((c ^ r7) << 4)), "r"(v0), "r"(v1),
                 "r"(v2), "r"(v3)
                 : "memory");
  }
}

// grid: (ceil(N/128), ceil(m/BN), splits); ch_per: 256-element chunks per split.
template <int T, int BN>
__global__ void __launch_bounds__(Q_THREADS, 1)
    k_gemm_tcq(const __grid_constant__ TcW W, const __grid_constant__ CUtensorMap tx, int m, int nch, int ch_per,
               float *__restrict__ part, unsigned *err) {
  using C = QCfg<T, BN>;
  const int bx = blockIdx.x, mi = bx < W.t[1] ? 0 : (bx < W.t[2] ? 1 : 2);  // this tile's matrix
  const CUtensorMap *tw = &W.map[mi];
  const int N = W.N[mi];
  float *__restrict__ y = W.y[mi];
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw0 = su32(smem_raw);
  const uint32_t base = (raw0 + 1023u) & ~1023u;
  const uint32_t bars = base + C::OFF_BAR;
  auto bar = [&](int i) { return bars + 8u * (uint32_t)i; };
  uint8_t *gen = smem_raw + (base - raw0);
  volatile uint32_t *tmem_slot = (volatile uint32_t *)(gen + C::OFF_BAR + 8 * QB_N);
  volatile int *abort_flag = (volatile int *)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int f0 = (bx - W.t[mi]) * TC_M, t0 = blockIdx.y * BN;
  const int c0 = blockIdx.z * ch_per;
  const int nc = min(nch, c0 + ch_per) - c0;  // >= 1
  const int nsub = 4 * nc;                    // 64-element steps

  if (threadIdx.x == 0) {
    for (int i = 0; i < QB_N; i++) {
      const bool rows = (i >= QB_RAWEMPTY && i < QB_RAWEMPTY + 2) || (i >= QB_AFULL && i < QB_AFULL + 2) ||
                        (i >= QB_PEMPTY && i < QB_PEMPTY + 4);
      bar_init(bar(i), rows ? TC_M : 1);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_map(tw);
    prefetch_map(&tx);
  }
  __syncwarp();
  if (warp == 0) tmem_alloc(su32((const void *)tmem_slot), C::TMEM_COLS);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // TMA: raw weight rows (one 256-element chunk = eight blocks per copy, issued a
    // chunk ahead) and the activation terms of each 64-element step
    if (lane == 0) {
      int raw_issued = 0, issued = 0;
      auto load_raw = [&](int c) -> bool {
        const int rb = c & 1;
        if (c >= 2 && !bar_wait(bar(QB_RAWEMPTY + rb), (unsigned)((c >> 1) - 1) & 1u, err, abort_flag)) return false;
        bar_expect_tx(bar(QB_RAWFULL + rb), (unsigned)C::RAW);
        tma_load_2d(base + C::OFF_RAW + rb * C::RAW, tw, (c0 + c) * (C::CB / 2), f0, bar(QB_RAWFULL + rb));
        raw_issued = c + 1;
        return true;
      };
      bool ok = load_raw(0);
      for (int i = 0; ok && i < nsub; i++) {
        if (i % 4 == 1 && i / 4 + 1 < nc && !(ok = load_raw(i / 4 + 1))) break;
        const int bb = i % C::NB;
        if (i >= C::NB && !bar_wait(bar(QB_BEMPTY + bb), (unsigned)((i / C::NB) - 1) & 1u, err, abort_flag)) break;
        bar_expect_tx(bar(QB_BFULL + bb), (unsigned)C::B_STAGE);
        const int k = c0 * Q_CHUNK + i * TC_KB;
#pragma unroll
        for (int t = 0; t < TC_TERMS; t++)
          tma_load_3d(base + C::OFF_B + bb * C::B_STAGE + t * C::B_TERM, &tx, k, t0, t, bar(QB_BFULL + bb));
        issued = i + 1;
      }
      for (int c = std::max(0, raw_issued - 2); c < raw_issued; c++)
        bar_drain(bar(QB_RAWFULL + (c & 1)), (unsigned)(c >> 1) & 1u);
      for (int i = std::max(0, issued - C::NB); i < issued; i++)
        bar_drain(bar(QB_BFULL + i % C::NB), (unsigned)(i / C::NB) & 1u);
    }
    __syncwarp();
  } else if (warp == 5) {  // MMA issue: per step two blocks, each 3 terms x 2 K steps into its own buffer
    if (lane == 0) {
      for (int i = 0; i < nsub; i++) {
        const int ab = i & 1, bb = i % C::NB;
        if (!bar_wait(bar(QB_AFULL + ab), (unsigned)(i >> 1) & 1u, err, abort_flag)) break;
        if (!bar_wait(bar(QB_BFULL + bb), (unsigned)(i / C::NB) & 1u, err, abort_flag)) break;
        bool ok = true;
        for (int blk = 0; blk < 2 && ok; blk++) {
          const int gb = 2 * i + blk, pb = gb & 3;
          if (gb >= C::NP && !bar_wait(bar(QB_PEMPTY + pb), (unsigned)((gb >> 2) - 1) & 1u, err, abort_flag)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t a = base + C::OFF_A + ab * C::A_TILE, b = base + C::OFF_B + bb * C::B_STAGE;
#pragma unroll
          for (int t = 0; t < TC_TERMS; t++)
#pragma unroll
            for (int kk = 0; kk < 2; kk++) {
              const uint32_t ko = 32u * (uint32_t)(2 * blk + kk);
              mma_bf16(tmem + (uint32_t)(pb * BN), sw128_desc(a + ko), sw128_desc(b + t * C::B_TERM + ko), C::IDESC,
                       (t | kk) != 0 ? 1u : 0u);
            }
          mma_commit(bar(QB_PFULL + pb));
        }
        if (!ok) break;
        mma_commit(bar(QB_AEMPTY + ab));
        mma_commit(bar(QB_BEMPTY + bb));
      }
      mma_commit(bar(QB_FIN));
      bar_drain(bar(QB_FIN), 0u);
    }
    __syncwarp();
  } else {  // warps 0-3: row r converts and folds
    const int r = threadIdx.x, r7 = r & 7;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * warp) << 16);
    float acc[BN];
#pragma unroll
    for (int j = 0; j < BN; j++) acc[j] = 0.f;
    float sc[8], scp[8];
    bool ok = true;
    auto wait_all = [&](uint32_t b, unsigned par) -> bool {
      int v = 1;
      if (lane == 0) v = bar_wait(b, par, err, abort_flag);
      return __shfl_sync(0xffffffffu, v, 0) != 0;
    };
    auto fold = [&](int gb, float s) -> bool {  // acc += s * block sum gb
      const int pb = gb & 3;
      if (!wait_all(bar(QB_PFULL + pb), (unsigned)(gb >> 2) & 1u)) return false;
      fence_after();
#pragma unroll
      for (int c = 0; c < BN / 16; c++) {
        uint32_t v[16];
        tmem_ld16(lane_base + (uint32_t)(pb * BN + 16 * c), v);
        tmem_wait_ld(v);
#pragma unroll
        for (int j = 0; j < 16; j++) acc[16 * c + j] = fmaf(s, __uint_as_float(v[j]), acc[16 * c + j]);
      }
      fence_before();
      bar_arrive(bar(QB_PEMPTY + pb));
      return true;
    };
    for (int c = 0; c < nc && ok; c++) {
      const int rb = c & 1;
      if (!(ok = wait_all(bar(QB_RAWFULL + rb), (unsigned)(c >> 1) & 1u))) break;
      const uint32_t row = base + C::OFF_RAW + rb * C::RAW + (uint32_t)(r * C::CB);
#pragma unroll
      for (int j = 0; j < 8; j++) sc[j] = __half2float(__ushort_as_half((uint16_t)lds_u16(row + j * C::BB)));
#pragma unroll
      for (int sub = 0; sub < 4; sub++) {
        const int i = 4 * c + sub, ab = i & 1;
        if (i >= 2 && !(ok = wait_all(bar(QB_AEMPTY + ab), (unsigned)((i >> 1) - 1) & 1u))) break;
        convert_step<T>(row, sub, base + C::OFF_A + ab * C::A_TILE + (uint32_t)((r >> 3) * 1024 + r7 * 128), r7);
        fence_proxy_async();
        bar_arrive(bar(QB_AFULL + ab));
        if (sub == 3) bar_arrive(bar(QB_RAWEMPTY + rb));  // scales are in registers
        if (i >= 1) {  // fold the previous step's two blocks
          const float s0 = sub == 0 ? scp[6] : sc[2 * sub - 2];
          const float s1 = sub == 0 ? scp[7] : sc[2 * sub - 1];
          if (!(ok = fold(2 * (i - 1), s0)) || !(ok = fold(2 * (i - 1) + 1, s1))) break;
        }
      }
#pragma unroll
      for (int j = 0; j < 8; j++) scp[j] = sc[j];
    }
    if (ok) ok = fold(2 * (nsub - 1), scp[6]) && fold(2 * (nsub - 1) + 1, scp[7]);
    if (ok && !*abort_flag) {
      float *out = part ? part + (size_t)blockIdx.z * m * N : y;
      const int f = f0 + r;
      if (f < N) {
#pragma unroll
        for (int j = 0; j < BN; j++)
          if (t0 + j < m) out[(size_t)(t0 + j) * N + f] = acc[j];
      }
    }
  }
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

// nmat (1-3) weight matrices of K columns against the same activation terms; splits
// > 1 only with one matrix.
template <int BN>
cudaError_t run_tc(cudaStream_t s, const __nv_bfloat16 *xs, int m, int K, int nmat, const void *const *w,
                   const int *N, float *const *y, int splits, float *part) {
  using C = TcCfg<BN>;
  TcW W{};
  CUtensorMap tx;
  const cuuint64_t ws_[1] = {(cuuint64_t)K * 2};
  const cuuint32_t wb[2] = {TC_KB, TC_M};
  W.t[0] = 0;
  for (int i = 0; i < 3; i++) {
    const int j = i < nmat ? i : nmat - 1;  // unused entries repeat the last matrix (never selected)
    const cuuint64_t wd[2] = {(cuuint64_t)K, (cuuint64_t)N[j]};
    if (!encode(&W.map[i], w[j], 2, wd, ws_, wb)) return cudaErrorInvalidValue;
    W.y[i] = y[j];
    W.N[i] = N[j];
    W.t[i + 1] = W.t[i] + (i < nmat ? (N[i] + TC_M - 1) / TC_M : 0);
  }
  const cuuint64_t xd[3] = {(cuuint64_t)K, (cuuint64_t)m, TC_TERMS},
                   xst[2] = {(cuuint64_t)K * 2, (cuuint64_t)m * K * 2};
  const cuuint32_t xb[3] = {TC_KB, BN, 1};
  if (!encode(&tx, xs, 3, xd, xst, xb)) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(k_gemm_tc<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const int nkb = (K + TC_KB - 1) / TC_KB;
  if (nmat > 1) splits = 1;
  const int kb_per = (nkb + splits - 1) / splits;
  splits = (nkb + kb_per - 1) / kb_per;  // every split gets at least one block
  const dim3 grid(W.t[3], (m + BN - 1) / BN, splits);
  k_gemm_tc<BN><<<grid, TC_THREADS, C::SMEM, s>>>(W, tx, m, nkb, kb_per, splits > 1 ? part : nullptr, tc_err_ptr());
  e = cudaGetLastError();
  if (e != cudaSuccess || splits == 1) return e;
  const size_t n = (size_t)m * N[0];
  k_split_sum_tc<<<(unsigned)std::min<size_t>((n + 255) / 256, 4096), 256, 0, s>>>(part, splits, n, y[0]);
  return cudaGetLastError();
}

template <int T, int BN>
cudaError_t run_tcq(cudaStream_t s, const __nv_bfloat16 *xs, int m, int K, int nmat, const void *const *w,
                    const int *N, float *const *y, int splits, float *part) {
  using C = QCfg<T, BN>;
  TcW W{};
  CUtensorMap tx;
  const cuuint64_t rowbytes = (cuuint64_t)(K / QK) * C::BB;
  const cuuint64_t wst[1] = {rowbytes};
  const cuuint32_t wb[2] = {(cuuint32_t)(C::CB / 2), TC_M}, es[2] = {1, 1};
  W.t[0] = 0;
  for (int i = 0; i < 3; i++) {
    const int j = i < nmat ? i : nmat - 1;  // unused entries repeat the last matrix (never selected)
    const cuuint64_t wd[2] = {rowbytes / 2, (cuuint64_t)N[j]};
    if (g_encode(&W.map[i], CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(w[j]), wd, wst, wb, es,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
    W.y[i] = y[j];
    W.N[i] = N[j];
    W.t[i + 1] = W.t[i] + (i < nmat ? (N[i] + TC_M - 1) / TC_M : 0);
  }
  const cuuint64_t xd[3] = {(cuuint64_t)K, (cuuint64_t)m, TC_TERMS},
                   xst[2] = {(cuuint64_t)K * 2, (cuuint64_t)m * K * 2};
  const cuuint32_t xb[3] = {TC_KB, BN, 1};
  if (!encode(&tx, xs, 3, xd, xst, xb)) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(k_gemm_tcq<T, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const int nch = K / Q_CHUNK;
  if (nmat > 1) splits = 1;
  const int ch_per = (nch + splits - 1) / splits;
  splits = (nch + ch_per - 1) / ch_per;
  const dim3 grid(W.t[3], (m + BN - 1) / BN, splits);
  k_gemm_tcq<T, BN><<<grid, Q_THREADS, C::SMEM, s>>>(W, tx, m, nch, ch_per, splits > 1 ? part : nullptr,
                                                     tc_err_ptr());
  e = cudaGetLastError();
  if (e != cudaSuccess || splits == 1) return e;
  const size_t n = (size_t)m * N[0];
  k_split_sum_tc<<<(unsigned)std::min<size_t>((n + 255) / 256, 4096), 256, 0, s>>>(part, splits, n, y[0]);
  return cudaGetLastError();
}

template <int T>
cudaError_t run_tcq_bn(int bn, cudaStream_t s, const __nv_bfloat16 *xs, int m, int K, const void *w, int N, float *y,
                       int splits, float *part) {
  if (bn == 32) return run_tcq<T, 32>(s, xs, m, K, 1, &w, &N, &y, splits, part);
  if (bn == 64) return run_tcq<T, 64>(s, xs, m, K, 1, &w, &N, &y, splits, part);
  return run_tcq<T, 128>(s, xs, m, K, 1, &w, &N, &y, splits, part);
}

}  // namespace

bool gemm_tc_supported(int m, int K, const float *x, const void *w, int wtype, const float *ws, size_t ws_floats) {
  init_once();
  bool ok = g_encode && m >= 2 && K % 16 == 0 && x && ws && ((uintptr_t)x & 15) == 0 && ((uintptr_t)w & 15) == 0 &&
            ((uintptr_t)ws & 255) == 0 && (size_t)3 * m * K / 2 + 64 <= ws_floats;
  if (wtype == SQ_BF16) return ok;
  if (wtype != SQ_Q8_0 && wtype != SQ_Q4_0) return false;
  const size_t rowbytes = (size_t)(K / QK) * (wtype == SQ_Q8_0 ? Q8_BYTES : Q4_BYTES);
  return ok && K % Q_CHUNK == 0 && rowbytes % 16 == 0;  // whole eight-block chunks on 16-byte boundaries
}

cudaError_t launch_split_terms(cudaStream_t s, const float *x, int m, int K, float *ws) {
  init_once();
  const size_t n = (size_t)m * K;  // a multiple of 16
  k_split3<<<(unsigned)std::min<size_t>((n / 4 + 255) / 256, 8 * (size_t)g_sms_tc), 256, 0, s>>>(
      reinterpret_cast<const float4 *>(x), n / 4, reinterpret_cast<__nv_bfloat16 *>(ws), n);
  return cudaGetLastError();
}

cudaError_t launch_gemm_tc(cudaStream_t s, const float *x, int m, int K, const void *w, int wtype, int N, float *y,
                           float *ws, size_t ws_floats) {
  if (!gemm_tc_supported(m, K, x, w, wtype, ws, ws_floats)) return cudaErrorNotSupported;
  cudaError_t e = launch_split_terms(s, x, m, K, ws);
  if (e != cudaSuccess) return e;
  return launch_gemm_tc_terms(s, m, K, w, wtype, N, y, ws, ws_floats);
}

cudaError_t launch_gemm_tc_terms(cudaStream_t s, int m, int K, const void *w, int wtype, int N, float *y, float *ws,
                                 size_t ws_floats) {
  // the terms' source is only checked for alignment: pass the workspace itself
  if (!gemm_tc_supported(m, K, ws, w, wtype, ws, ws_floats)) return cudaErrorNotSupported;
  // workspace: [3][m][K] bf16 terms, then split-K partials (256-byte aligned)
  __nv_bfloat16 *xs = reinterpret_cast<__nv_bfloat16 *>(ws);
  const size_t xs_floats = ((size_t)3 * m * K / 2 + 63) & ~(size_t)63;
  float *part = ws + xs_floats;
  const size_t part_floats = ws_floats - xs_floats;
  const int ft = (N + TC_M - 1) / TC_M;
  if (wtype != SQ_BF16) {  // quantized rows: 256-element chunks, BN by the row count
    const int bn = m <= 32 ? 32 : (m <= 64 ? 64 : 128);
    const long long tiles = (long long)ft * ((m + bn - 1) / bn);
    const int nch = K / Q_CHUNK;
    int splits = 1;
    if (tiles < g_sms_tc) {
      splits = (int)std::min<long long>((g_sms_tc + tiles - 1) / tiles, 16);
      splits = std::min(splits, nch);
      while (splits > 1 && (size_t)splits * m * N > part_floats) splits--;
    }
    return wtype == SQ_Q8_0 ? run_tcq_bn<SQ_Q8_0>(bn, s, xs, m, K, w, N, y, splits, part)
                            : run_tcq_bn<SQ_Q4_0>(bn, s, xs, m, K, w, N, y, splits, part);
  }
  const int nkb = (K + TC_KB - 1) / TC_KB;
  const bool wide = (long long)ft * ((m + 127) / 128) >= g_sms_tc;
  const long long tiles = wide ? (long long)ft * ((m + 127) / 128) : (long long)ft * ((m + 63) / 64);
  int splits = 1;
  if (tiles < g_sms_tc) {
    splits = (int)std::min<long long>((g_sms_tc + tiles - 1) / tiles, 8);
    splits = std::min(splits, std::max(1, nkb / 4));  // at least 4 K blocks per split
    while (splits > 1 && (size_t)splits * m * N > part_floats) splits--;
  }
  return wide ? run_tc<128>(s, xs, m, K, 1, &w, &N, &y, splits, part)
              : run_tc<64>(s, xs, m, K, 1, &w, &N, &y, splits, part);
}

cudaError_t launch_gemm_tc_terms_multi(cudaStream_t s, int m, int K, int nmat, const void *const *w, int wtype,
                                       const int *N, float *const *y, float *ws, size_t ws_floats) {
  // one launch over every matrix's tiles when the kernel takes them without a K split
  // (enough tiles of 128 weight rows x 128 activation rows for the SMs); otherwise one
  // launch per matrix
  long long tiles = 0;
  bool ok = nmat >= 1 && nmat <= 3;
  for (int i = 0; i < nmat && ok; i++) {
    ok = gemm_tc_supported(m, K, ws, w[i], wtype, ws, ws_floats);
    tiles += (long long)((N[i] + TC_M - 1) / TC_M) * ((m + 127) / 128);
  }
  if (ok && tiles >= g_sms_tc) {
    const __nv_bfloat16 *xs = reinterpret_cast<const __nv_bfloat16 *>(ws);
    if (wtype == SQ_BF16) return run_tc<128>(s, xs, m, K, nmat, w, N, y, 1, nullptr);
    if (wtype == SQ_Q8_0) return run_tcq<SQ_Q8_0, 128>(s, xs, m, K, nmat, w, N, y, 1, nullptr);
    return run_tcq<SQ_Q4_0, 128>(s, xs, m, K, nmat, w, N, y, 1, nullptr);
  }
  for (int i = 0; i < nmat; i++) {
    const cudaError_t e = launch_gemm_tc_terms(s, m, K, w[i], wtype, N[i], y[i], ws, ws_floats);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
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
