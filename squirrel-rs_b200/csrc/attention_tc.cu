// attention_tc.cu — tensor-core causal GQA attention for prefill, head_dim 64
// (kernels/attention.rs:11-70 semantics: scores = (q.k) * 1/sqrt(hd) over keys
// 0..=offset+t, max-subtracted softmax, probability-weighted sum of V; f32 inputs).
//
// Accuracy: q, k, v and the probabilities p are each split into three bf16 terms
// that sum to the f32 value exactly (x = h + d + l). A product of two split values
// is formed from the six term products whose weight is at least 2^-16 of the leading
// one (hh, hd, dh, hl, dd, lh); each bf16 x bf16 product is exact and the tensor core
// accumulates in f32, so scores and outputs keep f32-level accuracy.
//
// Pre-pass (k_split_rows, k_split_vt): the chunk's queries as [3][H][n][64], the
// keys 0..seq_k-1 as [3][G][seq_k][64] and the values transposed as
// [3][G][64][seq_k padded to 8] (bf16), in a caller-provided workspace.
//
// Kernel: one CTA per (128-query block, q head); the heaviest (last) query blocks
// start first. 14 warps:
//   warps 8, 10  TMA: the query block's three term tiles once, then per 64-key block
//            the key (warp 8) and transposed-value (warp 10) term tiles into separate
//            double buffers (a key buffer is released when its S is done, a value
//            buffer when its O is);
//   warps 9, 12  MMA issue for S_j = Q K_j^T (M = 128 queries, N = 64 keys), three of
//            the six term pairs each, into one of two tensor-memory score buffers;
//   warps 11, 13  MMA issue for O_j = P_j V_j (N = 64 dims, A = P read from tensor
//            memory), three term pairs each, into one of two output buffers. The
//            softmax threads zero each score / output buffer after reading it, so
//            every MMA accumulates and the issuing threads need no mutual order;
//   warps 0-7  two threads per query row (warps w and w + 4 share tensor-memory
//            lanes), each with 32 keys and 32 output dims: scores of block j from
//            tensor memory, causal mask near the diagonal, online softmax in base 2
//            (running max combined through shared memory, ex2), P_j split into terms
//            and stored into one of two tensor-memory P buffers (so P_{j+1} is
//            written while O_j is computed), then the f32 running output
//            o = o * 2^(m_old - m_new) + O_j in registers (one block behind).
// Every wait is bounded; on expiry the CTA records the error, stops, drains its
// copies and MMAs, frees its tensor memory and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>

#include "ops.cuh"
#include "tc.cuh"

namespace sq {
namespace {

using namespace tc;

constexpr int FA_M = 128;   // query rows per CTA
constexpr int FA_BK = 64;   // keys per block
constexpr int FA_HD = 64;   // head dim
constexpr int FA_PARTS = 2;                 // softmax threads per query row
constexpr int FA_SOFTMAX = 128 * FA_PARTS;  // softmax threads
constexpr int FA_WARP_TMA = FA_SOFTMAX / 32, FA_WARP_MMA = FA_WARP_TMA + 1, FA_WARP_V = FA_WARP_TMA + 2,
              FA_WARP_PV = FA_WARP_TMA + 3, FA_WARP_S2 = FA_WARP_TMA + 4, FA_WARP_PV2 = FA_WARP_TMA + 5;
constexpr int FA_THREADS = FA_SOFTMAX + 192;

constexpr int Q_TERM = FA_M * FA_HD * 2;   // 16 KB
constexpr int K_TERM = FA_BK * FA_HD * 2;  // 8 KB
constexpr int V_TERM = FA_HD * FA_BK * 2;  // 8 KB (transposed: 64 dims x 64 keys)
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + 3 * Q_TERM;      // two buffers of three key terms
constexpr int OFF_V = OFF_K + 2 * 3 * K_TERM;  // two buffers of three value terms
constexpr int OFF_XCHG = OFF_V + 2 * 3 * V_TERM;  // row maxima / sums exchanged by a row's threads
constexpr int OFF_BAR = OFF_XCHG + 3 * FA_PARTS * FA_M * 4;
constexpr int FA_SMEM = 1024 + OFF_BAR + 256;
static_assert(FA_SMEM <= 232448, "shared memory per CTA");
static_assert(OFF_K % 1024 == 0 && OFF_V % 1024 == 0 && OFF_BAR % 8 == 0, "alignment");

// barrier slots (8 bytes each)
enum : int {
  B_QFULL = 0,
  B_KFULL = 1,    // [2] key terms of a block landed
  B_KEMPTY = 3,   // [2] S of that block done: the key buffer is free
  B_VFULL = 5,    // [2]
  B_VEMPTY = 7,   // [2] O of that block done: the value buffer is free
  B_SFULL = 9,    // [2] both score accumulators of a block done
  B_SPFREE = 11,  // [2] O of the block done: its score / P buffer is free
  B_PFULL = 13,   // [2] P of a block written to tensor memory
  B_OFULL = 15,   // [2] both output accumulators of a block done
  B_OFREE = 17,   // [2] the softmax threads have read them
  B_FIN = 19,     // the score issuers' MMAs all done
  B_FIN2 = 20,    // the output issuers' MMAs all done
  N_BARS = 21
};
// tensor-memory columns. SP[2] at 0 / 128: the two score accumulators (issuer A at
// +0, issuer B at +64, f32, column = key); once read, the same columns take P as
// three bf16 terms of 32 columns (two keys per 32-bit column). O[2] at 256 / 384:
// the two output accumulators (+0, +64; column = head dim). Lane = query row.
constexpr uint32_t TM_SP = 0, TM_O = 256, TM_COLS = 512;
constexpr uint32_t IDESC = idesc_bf16(FA_M, 64);

// term pairs (a, b) with a + b <= 2: the products kept
__device__ __constant__ int8_t kPairs[6][2] = {{0, 0}, {0, 1}, {1, 0}, {0, 2}, {1, 1}, {2, 0}};

__device__ __forceinline__ void split3(float x, __nv_bfloat16 &h, __nv_bfloat16 &d, __nv_bfloat16 &l) {
  h = __float2bfloat16_rn(x);
  const float r1 = x - __bfloat162float(h);
  d = __float2bfloat16_rn(r1);
  l = __float2bfloat16_rn(r1 - __bfloat162float(d));
}
// 2^x (hardware approximation, relative error ~2^-22; results below 2^-126 flush
// to zero, far below any probability that reaches the output).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack2(__nv_bfloat16 a, __nv_bfloat16 b) {
  return (uint32_t)__bfloat16_as_ushort(a) | ((uint32_t)__bfloat16_as_ushort(b) << 16);
}

// grid: n_heads * nqb CTAs. offset = seq_k - n (keys before the chunk's first query).
// scale2 = log2(e) / sqrt(hd): scores in base-2 units, p = 2^(s2 - m2).
__global__ void __launch_bounds__(FA_THREADS, 1)
    k_attn_tc(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
              const __grid_constant__ CUtensorMap tv, float *__restrict__ out, int n, int offset, int n_heads,
              int group, int nqb, float scale2, unsigned *err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = su32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t bars = base + OFF_BAR;
  auto bar = [&](int i) { return bars + 8u * (uint32_t)i; };
  uint8_t *gen = smem_raw + (base - raw);
  volatile uint32_t *tmem_slot = (volatile uint32_t *)(gen + OFF_BAR + 8 * N_BARS);
  volatile int *abort_flag = (volatile int *)(tmem_slot + 1);
  float *xchg = (float *)(gen + OFF_XCHG);  // [2 blocks][parts][128 rows] row maxima, then [parts][128] sums

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qb = nqb - 1 - (int)blockIdx.x / n_heads;  // heaviest blocks first
  const int h = (int)blockIdx.x % n_heads, g = h / group;
  const int G = n_heads / group;
  const int q0 = qb * FA_M;
  const int q_last = min(q0 + FA_M, n) - 1;
  const int nkb = (offset + q_last) / FA_BK + 1;  // key blocks this query block sees

  if (threadIdx.x == 0) {
    for (int i = 0; i < N_BARS; i++) {  // every softmax thread arrives on P-full and O-free
      const bool rows = i == B_PFULL || i == B_PFULL + 1 || i == B_OFREE || i == B_OFREE + 1;
      const bool by_issuers = !rows && i != B_QFULL && !(i >= B_KFULL && i < B_KFULL + 2) &&
                              !(i >= B_VFULL && i < B_VFULL + 2);  // committed by two issuing threads
      bar_init(bar(i), rows ? FA_SOFTMAX : (by_issuers ? 2 : 1));
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_map(&tq);
    prefetch_map(&tk);
    prefetch_map(&tv);
  }
  __syncwarp();
  if (warp == 0) tmem_alloc(su32((const void *)tmem_slot), TM_COLS);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  constexpr int KP = FA_BK / FA_PARTS;  // keys (and output dims) per softmax thread

  if (warp == FA_WARP_TMA) {
    // ---------------- TMA producer ----------------
    int issued = 0;
    if (lane == 0) {
      bar_expect_tx(bar(B_QFULL), 3 * Q_TERM);
      for (int t = 0; t < 3; t++) tma_load_3d(base + OFF_Q + t * Q_TERM, &tq, 0, q0, t * n_heads + h, bar(B_QFULL));
      // keys of block j+2 load once S_j is done (the value copies run in their own
      // warp, released by O_j): the key copy overlaps the softmax and P.V between
      for (int j = 0; j < nkb; j++) {
        const int b = j & 1;
        if (j >= 2 && !bar_wait(bar(B_KEMPTY + b), (unsigned)((j >> 1) - 1) & 1u, err, abort_flag)) break;
        bar_expect_tx(bar(B_KFULL + b), 3 * K_TERM);
        for (int t = 0; t < 3; t++)
          tma_load_3d(base + OFF_K + (b * 3 + t) * K_TERM, &tk, 0, j * FA_BK, t * G + g, bar(B_KFULL + b));
        issued = j + 1;
      }
      // drain: every started copy lands before the CTA exits
      bar_drain(bar(B_QFULL), 0u);
      for (int j = std::max(0, issued - 2); j < issued; j++) bar_drain(bar(B_KFULL + (j & 1)), (unsigned)(j >> 1) & 1u);
    }
    __syncwarp();
  } else if (warp == FA_WARP_V) {
    // ---------------- TMA producer: transposed values ----------------
    if (lane == 0) {
      int issued = 0;
      for (int j = 0; j < nkb; j++) {
        const int b = j & 1;
        if (j >= 2 && !bar_wait(bar(B_VEMPTY + b), (unsigned)((j >> 1) - 1) & 1u, err, abort_flag)) break;
        bar_expect_tx(bar(B_VFULL + b), 3 * V_TERM);
        for (int t = 0; t < 3; t++)
          tma_load_3d(base + OFF_V + (b * 3 + t) * V_TERM, &tv, j * FA_BK, 0, t * G + g, bar(B_VFULL + b));
        issued = j + 1;
      }
      for (int j = std::max(0, issued - 2); j < issued; j++) bar_drain(bar(B_VFULL + (j & 1)), (unsigned)(j >> 1) & 1u);
    }
    __syncwarp();
  } else if (warp == FA_WARP_MMA || warp == FA_WARP_S2) {
    // ---------------- MMA issue: scores (two threads, three term pairs each, own accumulators) ----------------
    const int p0 = warp == FA_WARP_MMA ? 0 : 3;
    if (lane == 0) {
      bool ok = bar_wait(bar(B_QFULL), 0u, err, abort_flag);
      for (int i = 0; ok && i < nkb; i++) {
        const int b = i & 1;
        if (!bar_wait(bar(B_KFULL + b), (unsigned)(i >> 1) & 1u, err, abort_flag)) break;
        if (i >= 2 && !bar_wait(bar(B_SPFREE + b), (unsigned)((i >> 1) - 1) & 1u, err, abort_flag)) break;
        fence_after();
        const uint32_t d = tmem + TM_SP + 128u * b + (p0 ? 64u : 0u);
        const uint32_t qa = base + OFF_Q, ka = base + OFF_K + b * 3 * K_TERM;
#pragma unroll
        for (int q = 0; q < 3; q++) {
          const int pr = p0 + q;
          const uint32_t a0 = qa + kPairs[pr][0] * Q_TERM, b0 = ka + kPairs[pr][1] * K_TERM;
#pragma unroll
          for (int kk = 0; kk < FA_HD / 16; kk++)
            mma_bf16(d, sw128_desc(a0 + 32u * kk), sw128_desc(b0 + 32u * kk), IDESC, (q | kk) != 0 ? 1u : 0u);
        }
        mma_commit(bar(B_SFULL + b));
        mma_commit(bar(B_KEMPTY + b));
      }
      mma_commit(bar(B_FIN));
      bar_drain(bar(B_FIN), 0u);  // every MMA done before the columns are freed
    }
    __syncwarp();
  } else if (warp == FA_WARP_PV || warp == FA_WARP_PV2) {
    // ---------------- MMA issue: outputs (two threads, three term pairs each, own accumulators) ----------------
    const int p0 = warp == FA_WARP_PV ? 0 : 3;
    if (lane == 0) {
      for (int j = 0; j < nkb; j++) {
        const int b = j & 1;
        if (!bar_wait(bar(B_PFULL + b), (unsigned)(j >> 1) & 1u, err, abort_flag)) break;
        if (j >= 2 && !bar_wait(bar(B_OFREE + b), (unsigned)((j >> 1) - 1) & 1u, err, abort_flag)) break;
        if (!bar_wait(bar(B_VFULL + b), (unsigned)(j >> 1) & 1u, err, abort_flag)) break;
        fence_after();
        const uint32_t d = tmem + TM_O + 128u * b + (p0 ? 64u : 0u);
        const uint32_t pa = tmem + TM_SP + 128u * b, va = base + OFF_V + b * 3 * V_TERM;
#pragma unroll
        for (int q = 0; q < 3; q++) {
          const int pr = p0 + q;
          const uint32_t a0 = pa + 32u * kPairs[pr][0], b0 = va + kPairs[pr][1] * V_TERM;
#pragma unroll
          for (int kk = 0; kk < FA_BK / 16; kk++)  // A = P from tensor memory: 16 keys = 8 columns
            mma_bf16_ts(d, a0 + 8u * kk, sw128_desc(b0 + 32u * kk), IDESC, (q | kk) != 0 ? 1u : 0u);
        }
        mma_commit(bar(B_OFULL + b));
        mma_commit(bar(B_VEMPTY + b));
        mma_commit(bar(B_SPFREE + b));
      }
      mma_commit(bar(B_FIN2));
      bar_drain(bar(B_FIN2), 0u);
    }
    __syncwarp();
  } else {
    // ---------------- softmax / output ----------------
    // FA_PARTS threads per query row: warps w, w + 4, .. share tensor-memory lanes
    // 32*(w%4) ..; part pt owns keys [KP*pt, KP*pt + KP) of each block and output
    // dims [KP*pt, KP*pt + KP). Row maxima and sums are combined through shared
    // memory at named barrier 1 + quarter.
    const int quarter = warp & 3, pt = warp >> 2;
    const int r = 32 * quarter + lane;  // query row = tensor-memory lane
    const int qpos = offset + q0 + r;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * quarter) << 16);
    const uint32_t col = (uint32_t)(KP * pt);
    float o[KP];
#pragma unroll
    for (int d = 0; d < KP; d++) o[d] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 1.f;  // m in base-2 units (scores * scale2)
    bool ok = true;
    auto wait_all = [&](uint32_t b, unsigned par) -> bool {  // lane 0 waits, the warp follows
      int v = 1;
      if (lane == 0) v = bar_wait(b, par, err, abort_flag);
      return __shfl_sync(0xffffffffu, v, 0) != 0;
    };
    // Every wait is followed by a vote of the row group's warps, so they leave the
    // loop together and never leave one of them at a barrier alone.
    auto group_sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(1 + quarter), "r"(32 * FA_PARTS) : "memory"); };
    auto group_and = [&](bool v) -> bool {
      unsigned res;
      asm volatile(
          "{\n\t.reg .pred p, q;\n\t"
          "setp.ne.u32 p, %1, 0;\n\t"
          "bar.red.and.pred q, %2, %3, p;\n\t"
          "selp.u32 %0, 1, 0, q;\n\t}"
          : "=r"(res)
          : "r"((unsigned)v), "r"(1 + quarter), "r"(32 * FA_PARTS)
          : "memory");
      return res != 0;
    };
    auto add_block = [&](int j) -> bool {  // o = o * alpha_prev + O_j (this part's dims)
      const int b = j & 1;
      if (!group_and(wait_all(bar(B_OFULL + b), (unsigned)(j >> 1) & 1u))) return false;
      fence_after();
      uint32_t va[KP / 16][16], vb[KP / 16][16];
      const uint32_t oa = lane_base + TM_O + 128u * b + col;
#pragma unroll
      for (int c = 0; c < KP / 16; c++) {
        tmem_ld16(oa + 16u * c, va[c]);
        tmem_ld16(oa + 64u + 16u * c, vb[c]);
      }
      tmem_wait_ld(va[0]);
#pragma unroll
      for (int c = 0; c < KP / 16; c++) {
        if (c) tmem_tie(va[c]);
        tmem_tie(vb[c]);
      }
      fence_before();
      bar_arrive(bar(B_OFREE + b));
#pragma unroll
      for (int i = 0; i < KP; i++)  // the two accumulators in a fixed order: deterministic
        o[i] = fmaf(o[i], alpha_prev, __uint_as_float(va[i >> 4][i & 15]) + __uint_as_float(vb[i >> 4][i & 15]));
      return true;
    };
    // keys below the query block's first position need no mask
    const int unmasked_blocks = (offset + q0 + 1) / FA_BK;
    for (int j = 0; j < nkb; j++) {
      const int b = j & 1;
      const bool got = wait_all(bar(B_SFULL + b), (unsigned)(j >> 1) & 1u);
      float sc[KP];  // raw scores q.k (masked: -inf)
      float mx = -INFINITY;
      if (got) {
        fence_after();
        uint32_t sv[KP / 16][16], sw[KP / 16][16];
        const uint32_t sa = lane_base + TM_SP + 128u * b + col;
#pragma unroll
        for (int c = 0; c < KP / 16; c++) {
          tmem_ld16(sa + 16u * c, sv[c]);
          tmem_ld16(sa + 64u + 16u * c, sw[c]);
        }
        tmem_wait_ld(sv[0]);
#pragma unroll
        for (int c = 0; c < KP / 16; c++) {
          if (c) tmem_tie(sv[c]);
          tmem_tie(sw[c]);
        }
#pragma unroll
        for (int c = 0; c < KP / 16; c++)  // S = accumulator A + accumulator B, fixed order
#pragma unroll
          for (int e = 0; e < 16; e++) sv[c][e] = __float_as_uint(__uint_as_float(sv[c][e]) + __uint_as_float(sw[c][e]));
        if (j < unmasked_blocks) {
#pragma unroll
          for (int c = 0; c < KP; c++) sc[c] = __uint_as_float(sv[c >> 4][c & 15]);
        } else {
          const int k0 = j * FA_BK + KP * pt;
#pragma unroll
          for (int c = 0; c < KP; c++) sc[c] = (k0 + c <= qpos) ? __uint_as_float(sv[c >> 4][c & 15]) : -INFINITY;
        }
        float m4[4] = {sc[0], sc[1], sc[2], sc[3]};  // four independent chains
#pragma unroll
        for (int c = 4; c < KP; c++) m4[c & 3] = fmaxf(m4[c & 3], sc[c]);
        mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * scale2;  // scale2 > 0: max commutes
        xchg[(b * FA_PARTS + pt) * FA_M + r] = mx;
      }
      // the vote doubles as the exchange barrier of the row maxima, and orders every
      // thread's score loads before any thread's P stores into the same columns
      fence_before();
      ok = group_and(got);
      fence_after();
      if (!ok) break;
#pragma unroll
      for (int q = 1; q < FA_PARTS; q++) mx = fmaxf(mx, xchg[(b * FA_PARTS + ((pt + q) % FA_PARTS)) * FA_M + r]);
      const float m_new = fmaxf(m, mx);  // finite: key 0 is visible to every row in block 0
      const float alpha = ex2(m - m_new);  // 0 on the first block (m = -inf)
      float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < KP; c++) {
        sc[c] = ex2(fmaf(sc[c], scale2, -m_new));  // 2^(s*scale2 - m); 0 for masked keys
        s4[c & 3] += sc[c];
      }
      const float sum = (s4[0] + s4[1]) + (s4[2] + s4[3]);
      l = fmaf(l, alpha, sum);
      m = m_new;
      // P_j, this part's keys: three bf16 terms into the columns that held S_j (every
      // thread of the row has read its scores: the vote above is a barrier)
      {
        uint32_t w[3][KP / 2];
#pragma unroll
        for (int i = 0; i < KP / 2; i++) {
          const float p0 = sc[2 * i], p1 = sc[2 * i + 1];
          const __nv_bfloat162 t0 = __floats2bfloat162_rn(p0, p1);
          const float2 f0 = __bfloat1622float2(t0);
          const float r0 = p0 - f0.x, r1 = p1 - f0.y;
          const __nv_bfloat162 t1 = __floats2bfloat162_rn(r0, r1);
          const float2 f1 = __bfloat1622float2(t1);
          const __nv_bfloat162 t2 = __floats2bfloat162_rn(r0 - f1.x, r1 - f1.y);
          w[0][i] = *reinterpret_cast<const uint32_t *>(&t0);
          w[1][i] = *reinterpret_cast<const uint32_t *>(&t1);
          w[2][i] = *reinterpret_cast<const uint32_t *>(&t2);
        }
        const uint32_t pcol = lane_base + TM_SP + 128u * b + (uint32_t)(KP / 2 * pt);
#pragma unroll
        for (int t = 0; t < 3; t++)
#pragma unroll
          for (int h8 = 0; h8 < KP / 16; h8++) tmem_st8(pcol + 32u * t + 8u * h8, &w[t][8 * h8]);
        tmem_wait_st();
      }
      fence_before();
      bar_arrive(bar(B_PFULL + b));
      if (j >= 1 && !(ok = add_block(j - 1))) break;
      alpha_prev = alpha;
    }
    if (ok) ok = add_block(nkb - 1);
    // row sum = the parts' partial sums (same running maximum)
    if (ok) {
      xchg[(2 * FA_PARTS + pt) * FA_M + r] = l;
      group_sync();
#pragma unroll
      for (int q = 1; q < FA_PARTS; q++) l += xchg[(2 * FA_PARTS + ((pt + q) % FA_PARTS)) * FA_M + r];
    }
    if (ok && !*abort_flag && q0 + r < n) {
      const float inv = 1.0f / l;
      float4 *dst = reinterpret_cast<float4 *>(out + ((size_t)(q0 + r) * n_heads + h) * FA_HD + KP * pt);
#pragma unroll
      for (int d = 0; d < KP; d += 4)
        dst[d / 4] = make_float4(o[d] * inv, o[d + 1] * inv, o[d + 2] * inv, o[d + 3] * inv);
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    tmem_dealloc(tmem, TM_COLS);
  }
}

// dst[t][a][b][0..63] = term t of src[a*sa + b*sb + 0..63] for a < A, b < B.
__global__ void k_split_rows(const float *__restrict__ src, long long sa, long long sb, int A, int B,
                             __nv_bfloat16 *__restrict__ dst) {
  const size_t plane = (size_t)A * B * FA_HD;
  const size_t total = plane / 4;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t e = 4 * i;
    const int d = (int)(e % FA_HD);
    const size_t ab = e / FA_HD;
    const int bb = (int)(ab % B), a = (int)(ab / B);
    const float4 v = *reinterpret_cast<const float4 *>(src + a * sa + bb * sb + d);
    const float in[4] = {v.x, v.y, v.z, v.w};
    __nv_bfloat16 th[4], td[4], tl[4];
#pragma unroll
    for (int k = 0; k < 4; k++) split3(in[k], th[k], td[k], tl[k]);
    *reinterpret_cast<uint2 *>(dst + e) = make_uint2(pack2(th[0], th[1]), pack2(th[2], th[3]));
    *reinterpret_cast<uint2 *>(dst + plane + e) = make_uint2(pack2(td[0], td[1]), pack2(td[2], td[3]));
    *reinterpret_cast<uint2 *>(dst + 2 * plane + e) = make_uint2(pack2(tl[0], tl[1]), pack2(tl[2], tl[3]));
  }
}

// dst[t][g][d][s] = term t of v[g*ga + s*sp + d], s < seq_k (rows padded to skp).
// grid (ceil(seq_k/64), G), 256 threads: a 64-key x 64-dim tile through shared memory.
__global__ void k_split_vt(const float *__restrict__ v, long long ga, long long sp, int seq_k, int skp,
                           __nv_bfloat16 *__restrict__ dst) {
  __shared__ float tile[64][65];
  const int s0 = blockIdx.x * 64, g = blockIdx.y, G = gridDim.y;
  for (int i = threadIdx.x; i < 64 * 64; i += blockDim.x) {
    const int s = i / 64, d = i % 64;
    tile[s][d] = (s0 + s < seq_k) ? v[g * ga + (long long)(s0 + s) * sp + d] : 0.f;
  }
  __syncthreads();
  const size_t plane = (size_t)G * FA_HD * skp;
  for (int i = threadIdx.x; i < 64 * 64; i += blockDim.x) {
    const int d = i / 64, s = i % 64;
    if (s0 + s >= skp) continue;
    __nv_bfloat16 th, td, tl;
    split3(tile[s][d], th, td, tl);
    const size_t at = ((size_t)g * FA_HD + d) * skp + s0 + s;
    dst[at] = th;
    dst[plane + at] = td;
    dst[2 * plane + at] = tl;
  }
}

PFN_cuTensorMapEncodeTiled_v12000 g_enc = nullptr;

bool encode3(CUtensorMap *map, const void *ptr, cuuint64_t d0, cuuint64_t d1, cuuint64_t d2, cuuint64_t stride1,
             cuuint64_t stride2, cuuint32_t b0, cuuint32_t b1) {
  const cuuint64_t dims[3] = {d0, d1, d2}, strides[2] = {stride1, stride2};
  const cuuint32_t box[3] = {b0, b1, 1}, es[3] = {1, 1, 1};
  return g_enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(ptr), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

}  // namespace

size_t attn_tc_workspace_bytes(int seq_q, int seq_k, int n_heads, int n_kv_heads) {
  const size_t skp = ((size_t)seq_k + 7) & ~(size_t)7;
  return align256((size_t)6 * n_heads * seq_q * FA_HD) + align256((size_t)6 * n_kv_heads * seq_k * FA_HD) +
         align256((size_t)6 * n_kv_heads * FA_HD * skp);
}

bool attn_tc_supported(int seq_q, int seq_k, int n_heads, int n_kv_heads, int head_dim, long long kps, long long khs,
                       const void *q, const void *k, const void *v, size_t ws_bytes) {
  if (!g_enc) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      g_enc = (PFN_cuTensorMapEncodeTiled_v12000)fn;
  }
  return g_enc && head_dim == FA_HD && seq_q >= 64 && seq_k >= seq_q && n_kv_heads > 0 &&
         n_heads % n_kv_heads == 0 && kps % 4 == 0 && khs % 4 == 0 && ((uintptr_t)q & 15) == 0 &&
         ((uintptr_t)k & 15) == 0 && ((uintptr_t)v & 15) == 0 &&
         ws_bytes >= attn_tc_workspace_bytes(seq_q, seq_k, n_heads, n_kv_heads);
}

cudaError_t launch_attn_tc(cudaStream_t s, const float *q, const float *k, const float *v, float *out, int seq_q,
                           int seq_k, int n_heads, int n_kv_heads, int head_dim, long long kps, long long khs,
                           void *ws, size_t ws_bytes) {
  if (!attn_tc_supported(seq_q, seq_k, n_heads, n_kv_heads, head_dim, kps, khs, q, k, v, ws_bytes))
    return cudaErrorNotSupported;
  const int H = n_heads, G = n_kv_heads, n = seq_q;
  const int skp = (seq_k + 7) & ~7;
  uint8_t *w = (uint8_t *)ws;
  __nv_bfloat16 *qs = (__nv_bfloat16 *)w;
  __nv_bfloat16 *ks = (__nv_bfloat16 *)(w + align256((size_t)6 * H * n * FA_HD));
  __nv_bfloat16 *vt = (__nv_bfloat16 *)((uint8_t *)ks + align256((size_t)6 * G * seq_k * FA_HD));
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  auto grid_for = [&](size_t work) { return (unsigned)std::max<size_t>(1, std::min<size_t>((work + 255) / 256, 8 * (size_t)sms)); };
  k_split_rows<<<grid_for((size_t)H * n * 16), 256, 0, s>>>(q, FA_HD, (long long)H * FA_HD, H, n, qs);
  k_split_rows<<<grid_for((size_t)G * seq_k * 16), 256, 0, s>>>(k, khs, kps, G, seq_k, ks);
  k_split_vt<<<dim3((skp + 63) / 64, G), 256, 0, s>>>(v, khs, kps, seq_k, skp, vt);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  CUtensorMap tq, tk, tv;
  if (!encode3(&tq, qs, FA_HD, n, 3 * H, FA_HD * 2, (cuuint64_t)n * FA_HD * 2, 64, FA_M) ||
      !encode3(&tk, ks, FA_HD, seq_k, 3 * G, FA_HD * 2, (cuuint64_t)seq_k * FA_HD * 2, 64, FA_BK) ||
      !encode3(&tv, vt, seq_k, FA_HD, 3 * G, (cuuint64_t)skp * 2, (cuuint64_t)FA_HD * skp * 2, FA_BK, FA_HD))
    return cudaErrorInvalidValue;
  e = cudaFuncSetAttribute(k_attn_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, FA_SMEM);
  if (e != cudaSuccess) return e;
  const int nqb = (n + FA_M - 1) / FA_M;
  // scores * 1/sqrt(hd) (attention.rs:37), in base-2 units for exp2f
  const float scale2 = (float)(1.4426950408889634 / sqrt((double)head_dim));
  k_attn_tc<<<H * nqb, FA_THREADS, FA_SMEM, s>>>(tq, tk, tv, out, n, seq_k - n, H, H / G, nqb, scale2, tc_err_ptr());
  return cudaGetLastError();
}

}  // namespace sq
