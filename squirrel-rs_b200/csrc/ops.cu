// ops.cu — op-level kernels for sm_100a and the C-ABI entry points that replace
// squirrel-rs's `src/ops` functions. Decode of one token runs in the persistent
// decode kernel (decode.cu); these kernels serve the op-level ABI and prefill.
#include <cuda_bf16.h>
#include <math.h>
#include <stdio.h>

#include <atomic>
#include <mutex>
#include <string>

#include "common.cuh"
#include "ops.cuh"

namespace sq {

static thread_local std::string g_last_error;

void set_error(const std::string &msg) { g_last_error = msg; }
int fail(int code, const std::string &msg) {
  g_last_error = msg;
  return code;
}
int cuda_fail(cudaError_t e, const char *what) {
  g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return SQ_ERR_CUDA;
}

// ------------------------------------------------------------------------------------
// linear, f32 activations (W8A32 / W4A32 / BF16): dot_prod.rs:86-96, 255-270, 464-472.
// One warp per output row; lanes take the row's blocks; up to MT activation rows reuse
// each decoded block from registers. Per block the 32 products are summed first and
// scaled once (the reference's block_acc * scale), with FMA accumulation.
// ------------------------------------------------------------------------------------
template <int T>
__device__ __forceinline__ void load_block_f32(const uint8_t *blk, float (&q)[32], float &scale) {
  if constexpr (T == SQ_Q8_0) {
    scale = h2f(ld_u16(blk));
    const uint16_t *p = reinterpret_cast<const uint16_t *>(blk + 2);
#pragma unroll
    for (int i = 0; i < 16; i++) {
      uint16_t v = p[i];
      q[2 * i] = (float)(int8_t)(v & 0xFF);
      q[2 * i + 1] = (float)(int8_t)(v >> 8);
    }
  } else if constexpr (T == SQ_Q4_0) {
    scale = h2f(ld_u16(blk));
    const uint16_t *p = reinterpret_cast<const uint16_t *>(blk + 2);
#pragma unroll
    for (int i = 0; i < 8; i++) {
      uint16_t v = p[i];
      uint8_t b0 = v & 0xFF, b1 = v >> 8;
      q[2 * i] = (float)((b0 & 15) - 8);
      q[2 * i + 16] = (float)((b0 >> 4) - 8);
      q[2 * i + 1] = (float)((b1 & 15) - 8);
      q[2 * i + 17] = (float)((b1 >> 4) - 8);
    }
  } else {
    scale = 1.0f;
    const uint4 *p = reinterpret_cast<const uint4 *>(blk);  // BF16 blocks are 64-byte aligned rows
#pragma unroll
    for (int i = 0; i < 4; i++) {
      uint4 u = p[i];
      uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int k = 0; k < 4; k++) {
        q[8 * i + 2 * k] = __uint_as_float(w[k] << 16);
        q[8 * i + 2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
      }
    }
  }
}

template <int T, int MT>
__global__ void __launch_bounds__(256) k_linear_f32(const float *__restrict__ x, int m, int in_dim,
                                                     const uint8_t *__restrict__ w, int out_dim,
                                                     float *__restrict__ y) {
  constexpr int BB = type_bytes<T>();
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int bpr = in_dim / QK;
  for (int n = gw; n < out_dim; n += nw) {
    const uint8_t *wr = w + (size_t)n * bpr * BB;
    for (int m0 = 0; m0 < m; m0 += MT) {
      float acc[MT];
#pragma unroll
      for (int r = 0; r < MT; r++) acc[r] = 0.f;
      for (int b = lane; b < bpr; b += 32) {
        float q[32], scale;
        load_block_f32<T>(wr + (size_t)b * BB, q, scale);
#pragma unroll
        for (int r = 0; r < MT; r++) {
          if (m0 + r < m) {
            const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)(m0 + r) * in_dim + b * QK);
            float s = 0.f;
#pragma unroll
            for (int k = 0; k < 8; k++) {
              float4 v = __ldg(xr + k);
              s = fmaf(v.x, q[4 * k], s);
              s = fmaf(v.y, q[4 * k + 1], s);
              s = fmaf(v.z, q[4 * k + 2], s);
              s = fmaf(v.w, q[4 * k + 3], s);
            }
            acc[r] = (T == SQ_BF16) ? acc[r] + s : fmaf(s, scale, acc[r]);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < MT; r++) {
        float v = warp_sum(acc[r]);
        if (lane == 0 && m0 + r < m) y[(size_t)(m0 + r) * out_dim + n] = v;
      }
    }
  }
}

// m = 1 (decode through the op level): a matvec streamed through shared memory.
// Each CTA owns a contiguous block of rows. A producer warp streams it as tiles of
// whole consecutive rows (at most 36 KB, one bulk copy each, L2 evict-first: the
// weights are read once) into a ring of MV_NS slots completing on mbarriers. A row is
// split into segments of 2048 inputs (32 block pairs); the 8 consumer warps form
// groups of nseg warps, warp `seg` of a group keeps its input segment in registers
// (lane j holds elements 64j .. 64j+63, read once) and takes that segment of rows
// g, g + G, .. of every tile (two rows at a time, four for Q4_0: independent dots,
// one joint reduction); lane j reads pair j of the row from shared memory. With one
// segment the warp writes the row; otherwise the partial sums go to the slot's
// buffer in shared memory and the producer warp adds them in segment order
// (deterministic) once every consumer has released the slot, so consumers never
// wait on each other. The input may be RMS-normalised or formed as silu(x) * up as
// it is read, outputs may be added to a residual row, and a gate/up pair may leave
// only SiLU(gate) * up (MvArgs::gate_act). Rows must be whole multiples of 256
// elements (16-byte row starts) and in_dim <= 8 * 2048 (the caller checks).
// Waits are bounded (~2 s); on expiry the warp records an error and stops.
constexpr int MV_CONS = 8;                     // consumer warps
constexpr int MV_THREADS = 32 * (MV_CONS + 1);  // + the producer warp
constexpr int MV_SLOT = 36864;                 // bytes per ring slot
constexpr int MV_NS = 5;                       // ring slots
constexpr int MV_TRMAX = 64;                   // rows per tile at most
constexpr int MV_REDROWS = 32;                 // rows per tile when rows are split into segments
constexpr int MV_GATE_ROWS = 1024;             // gate rows per CTA kept for SiLU(gate) * up (gate_act)
constexpr int MV_HDR = 2 * MV_NS * 8 + ((MV_NS * MV_REDROWS + 1) * MV_CONS + MV_GATE_ROWS) * 4;  // mbarriers, sums, gates
constexpr int MV_RING_OFF = (MV_HDR + 127) & ~127;

__device__ unsigned g_mv_err;  // set when a bounded wait of k_matvec gave up (matvec_status)

__device__ __forceinline__ uint32_t mv_su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ bool mv_try_wait(uint32_t b, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(b), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mv_wait(uint32_t b, unsigned parity) {
  if (mv_try_wait(b, parity)) return true;
  const long long t0 = clock64();
  while (!mv_try_wait(b, parity)) {
    if (clock64() - t0 > 4000000000LL) {
      atomicExch(&g_mv_err, 1u);
      return false;
    }
  }
  return true;
}

template <int T>
__device__ __forceinline__ void mv_load_pair(uint32_t a, int lane, uint32_t (&wv)[pair_words<T>()]) {
  constexpr int PW = pair_words<T>();
  if constexpr (PW % 4 == 0) {  // BF16: 128 bytes a lane, 16-byte aligned. Step i reads the
    // lane's 16-byte chunk i ^ (lane % 8): the 8 lanes of a quarter-warp hit 8 different
    // bank groups (the input registers are permuted the same way)
#pragma unroll
    for (int i = 0; i < PW / 4; i++)
      asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(wv[4 * i]), "=r"(wv[4 * i + 1]), "=r"(wv[4 * i + 2]), "=r"(wv[4 * i + 3])
                   : "r"(a + 16u * (uint32_t)(i ^ (lane & 7))));
  } else {  // odd word stride between lanes: conflict-free 4-byte loads
#pragma unroll
    for (int i = 0; i < PW; i++) asm volatile("ld.shared.u32 %0, [%1];" : "=r"(wv[i]) : "r"(a + 4 * i));
  }
}

__device__ __forceinline__ float silu_ref(float x);

// MODE: what is folded into the input read (MV_PLAIN, MV_NORM, MV_SILU): a separate
// instantiation each, so the plain matvec carries none of that code.
constexpr int MV_PLAIN = 0, MV_NORM = 1, MV_SILU = 2, MV_GENERAL = 3;  // GENERAL: several matrices or residuals

template <int T, int MODE>
__global__ void __launch_bounds__(MV_THREADS, 1) k_matvec(const __grid_constant__ MvArgs a) {
  constexpr int PW = pair_words<T>(), CB = 32 * PW * 4;
  extern __shared__ __align__(128) uint8_t mv_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int in_dim = a.in_dim;
  const int nseg = (in_dim + 2047) / 2048;
  const int G = MV_CONS / nseg;  // row groups (consumer warps past G * nseg idle)
  const int ncons = G * nseg;
  const int np = in_dim / 64;               // pairs per row
  const int rb = np * PW * 4;               // row bytes (a multiple of 16)
  int TR = min(nseg > 1 ? MV_REDROWS : MV_TRMAX, MV_SLOT / rb);  // rows per tile (>= 1: rows fit a slot) ...
  if (TR >= G) TR -= TR % G;             // ... a multiple of the row groups: even work per warp
  // Fields of `a` are read by name only (never through its address, e.g. by a
  // lambda's reference capture), so they stay operands from the parameter bank.
#define MV_SEL(f, mi) ((mi) == 0 ? a.f[0] : ((mi) == 1 ? a.f[1] : a.f[2]))
  // each CTA owns a contiguous block of rows of every matrix: [sX0, sX1) of matrix X
  // the plain mode has one matrix and no residual (known at compile time)
  const int od0 = a.out_dim[0], od1 = MODE != MV_PLAIN && a.n > 1 ? a.out_dim[1] : 0,
            od2 = MODE != MV_PLAIN && a.n > 2 ? a.out_dim[2] : 0;
  const int pe0 = (od0 + gridDim.x - 1) / gridDim.x, pe1 = (od1 + gridDim.x - 1) / gridDim.x,
            pe2 = (od2 + gridDim.x - 1) / gridDim.x;
  const int s00 = blockIdx.x * pe0, s01 = min(od0, s00 + pe0);
  const int s10 = blockIdx.x * pe1, s11 = min(od1, s10 + pe1);
  const int s20 = blockIdx.x * pe2, s21 = min(od2, s20 + pe2);
  auto ntile = [&](int b0, int b1) { return b1 > b0 ? (b1 - b0 + TR - 1) / TR : 0; };
  const int nt0 = ntile(s00, s01), nt1 = ntile(s10, s11), nt2 = ntile(s20, s21);
  const int ntiles = nt0 + nt1 + nt2;
  // tile t -> (matrix, first row, rows)
  auto tile_of = [&](int t, int &mi, int &r0, int &rows) {
    int b0 = s00, b1 = s01;
    mi = 0;
    if (t >= nt0) {
      t -= nt0;
      mi = 1;
      b0 = s10;
      b1 = s11;
      if (t >= nt1) {
        t -= nt1;
        mi = 2;
        b0 = s20;
        b1 = s21;
      }
    }
    r0 = b0 + t * TR;
    rows = min(TR, b1 - r0);
  };
  const uint32_t full = mv_su32(mv_smem), empty = full + 8u * MV_NS;
  float *red = reinterpret_cast<float *>(mv_smem + 2 * MV_NS * 8);  // [MV_NS][MV_REDROWS][nseg], then [MV_CONS]
  // gate_act: the gate rows of this CTA, by row within its block; the thread that
  // writes gate row i is the one that later finishes up row i (same tile slot)
  float *gsm = red + (MV_NS * MV_REDROWS + 1) * MV_CONS;
  const uint32_t ring = mv_su32(mv_smem + MV_RING_OFF);
#define MV_OUT_ROW(mi, row, v)                                    \
  do {                                                            \
    if constexpr (MODE == MV_PLAIN) {                             \
      a.y[0][row] = (v);                                          \
    } else if (a.gate_act) {                                      \
      if ((mi) == 0) gsm[(row) - s00] = (v);                      \
      else a.y[1][row] = __fmul_rn(silu_ref(gsm[(row) - s00]), (v)); \
    } else {                                                      \
      const float *rs_ = MV_SEL(res, mi);                          \
      MV_SEL(y, mi)[row] = rs_ ? __fadd_rn(rs_[row], (v)) : (v);  \
    }                                                             \
  } while (0)
  if (threadIdx.x == 0) {
    for (int i = 0; i < MV_NS; i++) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(full + 8u * i) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(empty + 8u * i), "r"(ncons) : "memory");
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (warp == MV_CONS) {
    // producer: streams the tiles; with segments it also adds each tile's partial
    // sums (in segment order) once every consumer has released the tile's slot
    uint64_t pol = 0;
    if (lane == 0) asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    // the outputs as locals (the lambda below must not capture `a`)
    float *const py0 = a.y[0], *const py1 = a.y[1], *const py2 = a.y[2];
    const float *const pr0 = a.res[0], *const pr1 = a.res[1], *const pr2 = a.res[2];
    const bool gact = MODE != MV_PLAIN && a.gate_act != 0;
    auto finish = [&](int t) {
      int mi, r0, rows;
      tile_of(t, mi, r0, rows);
      float *yp = mi == 0 ? py0 : (mi == 1 ? py1 : py2);
      const float *rp = mi == 0 ? pr0 : (mi == 1 ? pr1 : pr2);
      const float *rd = red + (t % MV_NS) * MV_REDROWS * nseg;
      for (int r = lane; r < rows; r += 32) {
        float sum = rd[r * nseg];
        for (int q = 1; q < nseg; q++) sum += rd[r * nseg + q];
        if (gact) {
          if (mi == 0) gsm[r0 + r - s00] = sum;
          else py1[r0 + r] = __fmul_rn(silu_ref(gsm[r0 + r - s00]), sum);
        } else {
          yp[r0 + r] = rp ? __fadd_rn(rp[r0 + r], sum) : sum;
        }
      }
    };
    const bool solo = nseg == 1;  // nothing to finish: lane 0 alone streams the tiles
    if (solo && lane != 0) return;
    auto wait_empty = [&](int t) -> bool {  // the consumers are done with tile t
      if (solo) return mv_wait(empty + 8u * (t % MV_NS), (unsigned)(t / MV_NS) & 1u);
      int ok = 1;
      if (lane == 0) ok = mv_wait(empty + 8u * (t % MV_NS), (unsigned)(t / MV_NS) & 1u);
      return __shfl_sync(0xffffffffu, ok, 0) != 0;
    };
    int issued = 0, finished = 0;
    for (int t = 0; t < ntiles; t++) {
      const int slot = t % MV_NS;
      if (t == MV_NS) {  // the first ring fill (weights only) went out before the previous kernel ended
        pdl_wait();
        if (lane == 0) pdl_trigger();
      }
      if (t >= MV_NS) {
        if (!wait_empty(t - MV_NS)) break;
        if (nseg > 1) finish(t - MV_NS);
        finished = t - MV_NS + 1;
      }
      if (lane == 0 && t + 1 != a.test_skip) {  // a skipped tile's barrier never completes (tests)
        int mi, r0, rows;
        tile_of(t, mi, r0, rows);
        const unsigned bytes = (unsigned)(rows * rb);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(full + 8u * slot), "r"(bytes)
                     : "memory");
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
                ring + (uint32_t)slot * MV_SLOT),
            "l"(MV_SEL(w, mi) + (size_t)r0 * rb), "r"(bytes), "r"(full + 8u * slot), "l"(pol)
            : "memory");
      }
      issued = t + 1;
    }
    if (ntiles <= MV_NS) {
      pdl_wait();
      if (lane == 0) pdl_trigger();
    }
    if (nseg > 1 && issued == ntiles)  // the last tiles' partial sums
      for (int t = finished; t < ntiles; t++) {
        if (!wait_empty(t)) break;
        finish(t);
      }
    if (lane == 0)
      for (int t = max(0, issued - MV_NS); t < issued; t++) {  // drain: copies land before exit
        const long long t0 = clock64();
        while (!mv_try_wait(full + 8u * (t % MV_NS), (unsigned)(t / MV_NS) & 1u) && clock64() - t0 < 4000000000LL) {
        }
      }
    return;
  }
  if (warp >= ncons) return;
  pdl_wait();  // the input row (and residual rows) come from earlier kernels
  const int g = warp / nseg, seg = warp % nseg;
  const int pairs = min(32, np - seg * 32);  // pairs in this segment (>= 1)
  const bool active = lane < pairs;
  float inv_rms = 1.f;
  if constexpr (MODE == MV_NORM) {  // the consumers' sum of squares over the whole row, in a fixed order
    float ss = 0.f;
    for (int e = 4 * (warp * 32 + lane); e < in_dim; e += 4 * 32 * ncons) {
      const float4 v = __ldg(reinterpret_cast<const float4 *>(a.x + e));
      ss = fmaf(v.x, v.x, ss);
      ss = fmaf(v.y, v.y, ss);
      ss = fmaf(v.z, v.z, ss);
      ss = fmaf(v.w, v.w, ss);
    }
    ss = warp_sum(ss);
    float *part = red + MV_NS * MV_REDROWS * MV_CONS;  // [MV_CONS]
    if (lane == 0) part[warp] = ss;
    asm volatile("bar.sync 1, %0;" ::"r"(32 * ncons) : "memory");
    float tot = part[0];
    for (int q = 1; q < ncons; q++) tot += part[q];
    inv_rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)in_dim), a.eps)));
  }
  f2x x2[32];
  if (active) {
    const int base = seg * 2048 + lane * 64;
#pragma unroll
    for (int k = 0; k < 16; k++) {  // BF16: 8-element chunk i holds chunk i ^ (lane % 8), as the weights
      const int src = T == SQ_BF16 ? ((((k >> 1) ^ (lane & 7)) << 1) | (k & 1)) : k;
      float4 f = __ldg(reinterpret_cast<const float4 *>(a.x + base) + src);
      if constexpr (MODE == MV_SILU) {  // SiLU(gate) * up (silu.rs, elementwise_mul.rs)
        const float4 u = __ldg(reinterpret_cast<const float4 *>(a.xu + base) + src);
        f = make_float4(__fmul_rn(silu_ref(f.x), u.x), __fmul_rn(silu_ref(f.y), u.y), __fmul_rn(silu_ref(f.z), u.z),
                        __fmul_rn(silu_ref(f.w), u.w));
      }
      if constexpr (MODE == MV_NORM) {  // (x * w) * (1/rms): one multiply a element (the
        // reference divides by rms, one rounding apart; a division per element per CTA
        // cost this launch ~1 us)
        const float4 gw = __ldg(reinterpret_cast<const float4 *>(a.norm_w + base) + src);
        f = make_float4(__fmul_rn(__fmul_rn(f.x, gw.x), inv_rms), __fmul_rn(__fmul_rn(f.y, gw.y), inv_rms),
                        __fmul_rn(__fmul_rn(f.z, gw.z), inv_rms), __fmul_rn(__fmul_rn(f.w, gw.w), inv_rms));
      }
      x2[2 * k] = pk2(f.x, f.y);
      x2[2 * k + 1] = pk2(f.z, f.w);
    }
  } else {
#pragma unroll
    for (int k = 0; k < 32; k++) x2[k] = 0ull;
  }
  for (int t = 0; t < ntiles; t++) {
    const int slot = t % MV_NS;
    int ok = 1;
    if (lane == 0) ok = mv_wait(full + 8u * slot, (unsigned)(t / MV_NS) & 1u);
    if (!__shfl_sync(0xffffffffu, ok, 0)) break;
    int mi, r0, rows;
    tile_of(t, mi, r0, rows);
    const uint32_t tile = ring + (uint32_t)slot * MV_SLOT + (uint32_t)seg * CB + (uint32_t)lane * PW * 4;
    float *rd = red + slot * MV_REDROWS * nseg;  // partial sums, added by the producer
    constexpr int RI = T == SQ_Q4_0 ? 4 : 2;  // rows an iteration: independent dot chains
    for (int r = g; r < rows; r += RI * G) {  // rows r, r + G, .. of the tile
      float d[RI];
#pragma unroll
      for (int q = 0; q < RI; q++) d[q] = 0.f;
      if (active) {
        uint32_t wv[RI][PW];
#pragma unroll
        for (int q = 0; q < RI; q++)
          if (r + q * G < rows) mv_load_pair<T>(tile + (uint32_t)((r + q * G) * rb), lane, wv[q]);
#pragma unroll
        for (int q = 0; q < RI; q++)
          if (r + q * G < rows) d[q] = pair_dot<T>(wv[q], x2);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int q = 0; q < RI; q++) d[q] += __shfl_xor_sync(0xffffffffu, d[q], o);
      if (lane == 0) {
#pragma unroll
        for (int q = 0; q < RI; q++) {
          const int rr = r + q * G;
          if (rr < rows) {
            if (nseg == 1) MV_OUT_ROW(mi, r0 + rr, d[q]);
            else rd[rr * nseg + seg] = d[q];
          }
        }
      }
    }
    __syncwarp();  // every lane is done with the slot (and lane 0's partial sums are written)
    if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(empty + 8u * slot) : "memory");
  }
#undef MV_OUT_ROW
#undef MV_SEL
}

template <int T>
size_t mv_smem_bytes(int in_dim) {
  (void)in_dim;
  return (size_t)MV_RING_OFF + (size_t)MV_NS * MV_SLOT;
}

// ------------------------------------------------------------------------------------
// linear, Q8_0 activations (W8A8 / W4A8): dot_prod.rs:378-403 (scalar twins). The
// integer block sums are exact (dp4a); each block adds (isum * sa) * sb.
// ------------------------------------------------------------------------------------
__device__ __forceinline__ void load_q8_words(const uint8_t *blk, int (&w)[8], float &scale) {
  scale = h2f(ld_u16(blk));
  const uint16_t *p = reinterpret_cast<const uint16_t *>(blk + 2);
#pragma unroll
  for (int i = 0; i < 8; i++) w[i] = (int)((uint32_t)p[2 * i] | ((uint32_t)p[2 * i + 1] << 16));
}

template <int T, int MT>
__global__ void __launch_bounds__(256) k_linear_q8(const uint8_t *__restrict__ xq, int m, int in_dim,
                                                    const uint8_t *__restrict__ w, int out_dim,
                                                    float *__restrict__ y) {
  constexpr int BB = type_bytes<T>();
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int bpr = in_dim / QK;
  for (int n = gw; n < out_dim; n += nw) {
    const uint8_t *wr = w + (size_t)n * bpr * BB;
    for (int m0 = 0; m0 < m; m0 += MT) {
      float acc[MT];
#pragma unroll
      for (int r = 0; r < MT; r++) acc[r] = 0.f;
      for (int b = lane; b < bpr; b += 32) {
        const uint8_t *blk = wr + (size_t)b * BB;
        int wq[8];
        float sb;
        if constexpr (T == SQ_Q8_0) {
          load_q8_words(blk, wq, sb);
        } else {
          sb = h2f(ld_u16(blk));
          const uint16_t *p = reinterpret_cast<const uint16_t *>(blk + 2);
#pragma unroll
          for (int i = 0; i < 4; i++) {
            uint32_t v = (uint32_t)p[2 * i] | ((uint32_t)p[2 * i + 1] << 16);
            wq[i] = (int)__vsub4(v & 0x0F0F0F0Fu, 0x08080808u);             // elements 4i..4i+3
            wq[i + 4] = (int)__vsub4((v >> 4) & 0x0F0F0F0Fu, 0x08080808u);  // elements 16+4i..
          }
        }
#pragma unroll
        for (int r = 0; r < MT; r++) {
          if (m0 + r < m) {
            int aw[8];
            float sa;
            load_q8_words(xq + ((size_t)(m0 + r) * bpr + b) * Q8_BYTES, aw, sa);
            int isum = 0;
#pragma unroll
            for (int i = 0; i < 8; i++) isum = __dp4a(aw[i], wq[i], isum);
            acc[r] += ((float)isum * sa) * sb;
          }
        }
      }
#pragma unroll
      for (int r = 0; r < MT; r++) {
        float v = warp_sum(acc[r]);
        if (lane == 0 && m0 + r < m) y[(size_t)(m0 + r) * out_dim + n] = v;
      }
    }
  }
}

// quantize_row_q8_0_scalar (dot_prod.rs:21-31), one warp per block, bit-exact.
__global__ void k_quantize_q8_0(const float *__restrict__ x, size_t nblocks, uint8_t *__restrict__ out) {
  const int lane = threadIdx.x & 31;
  size_t b = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const size_t stride = ((size_t)gridDim.x * blockDim.x) >> 5;
  for (; b < nblocks; b += stride) {
    float v = x[b * QK + lane];
    float amax = warp_max(fabsf(v));
    float scale = __fdiv_rn(amax, 127.0f);
    float inv = scale > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
    float r = roundf(__fmul_rn(v, inv));  // ties away from zero, like f32::round
    int8_t q = (r != r) ? 0 : (int8_t)fminf(fmaxf(r, -127.0f), 127.0f);
    uint8_t *blk = out + b * Q8_BYTES;
    blk[2 + lane] = (uint8_t)q;
    if (lane == 0) *reinterpret_cast<uint16_t *>(blk) = __half_as_ushort(__float2half_rn(scale));
  }
}

// embed (ops/embedding.rs:10-52): exact dequantized rows. A token id >= vocab (the
// reference panics on the slice) yields a NaN row instead of an out-of-bounds read.
template <int T>
__global__ void k_embed(const uint32_t *__restrict__ tokens, const uint8_t *__restrict__ w, int dim, int vocab,
                        float *__restrict__ out) {
  constexpr int BB = type_bytes<T>();
  const int t = blockIdx.y;
  const uint32_t tok = tokens[t];
  const uint8_t *row = w + (size_t)(tok < (uint32_t)vocab ? tok : 0) * (dim / QK) * BB;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x)
    out[(size_t)t * dim + i] = tok < (uint32_t)vocab ? dequant_elem<T>(row + (i / QK) * BB, i % QK) : __int_as_float(0x7fc00000);
}

template <int T>
__global__ void k_dequant(const uint8_t *__restrict__ blocks, size_t n, float *__restrict__ out) {
  constexpr int BB = type_bytes<T>();
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    out[i] = dequant_elem<T>(blocks + (i / QK) * BB, (int)(i % QK));
}

// rms_norm_f32_into (kernels/rms_norm.rs:40-56): y = (x*w) / sqrt(mean(x^2) + eps), one CTA per row.
// Rows of dim <= 8 * 4 * 256 with 16-byte row starts: every float4 of a thread loaded
// at once and kept in registers for the output (one pass over global memory).
constexpr int RMS_V = 8;

// Four f32 values -> their three exact bf16 terms (x = h + d + l), stored at element
// offset e of the three planes [3][plane] (the tensor-core GEMM's activation input).
__device__ __forceinline__ void store_terms4(__nv_bfloat16 *terms, size_t plane, size_t e, float4 v) {
  const float in[4] = {v.x, v.y, v.z, v.w};
  uint32_t hw[2], dw[2], lw[2];
#pragma unroll
  for (int k = 0; k < 2; k++) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(in[2 * k], in[2 * k + 1]);
    const float2 hf = __bfloat1622float2(h);
    const float r0 = in[2 * k] - hf.x, r1 = in[2 * k + 1] - hf.y;
    const __nv_bfloat162 d = __floats2bfloat162_rn(r0, r1);
    const float2 df = __bfloat1622float2(d);
    const __nv_bfloat162 l = __floats2bfloat162_rn(r0 - df.x, r1 - df.y);
    hw[k] = *reinterpret_cast<const uint32_t *>(&h);
    dw[k] = *reinterpret_cast<const uint32_t *>(&d);
    lw[k] = *reinterpret_cast<const uint32_t *>(&l);
  }
  *reinterpret_cast<uint2 *>(terms + e) = make_uint2(hw[0], hw[1]);
  *reinterpret_cast<uint2 *>(terms + plane + e) = make_uint2(dw[0], dw[1]);
  *reinterpret_cast<uint2 *>(terms + 2 * plane + e) = make_uint2(lw[0], lw[1]);
}

// y (may be null) and / or the three bf16 terms of the output (terms may be null;
// plane = rows * dim). add (may be null): the residual add first, x += add
// (elementwise_add.rs:47-61), written back to x, then the norm of the sum.
__global__ void __launch_bounds__(256) k_rms_norm_v(float *x, const float *__restrict__ w, float *y, int dim,
                                                    float eps, __nv_bfloat16 *terms, size_t plane,
                                                    const float *__restrict__ add) {
  __shared__ float red[8];
  float4 *xr = reinterpret_cast<float4 *>(x + (size_t)blockIdx.x * dim);
  const float4 *ar = add ? reinterpret_cast<const float4 *>(add + (size_t)blockIdx.x * dim) : nullptr;
  const float4 *wr = reinterpret_cast<const float4 *>(w);
  float4 *yr = reinterpret_cast<float4 *>(y + (size_t)blockIdx.x * dim);
  const int nv = dim / 4;
  float4 v[RMS_V], g[RMS_V];
#pragma unroll
  for (int k = 0; k < RMS_V; k++) {
    const int i = threadIdx.x + k * 256;
    v[k] = i < nv ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    g[k] = i < nv ? __ldg(wr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (add) {
#pragma unroll
    for (int k = 0; k < RMS_V; k++) {
      const int i = threadIdx.x + k * 256;
      if (i < nv) {
        const float4 a = ar[i];
        v[k] = make_float4(__fadd_rn(v[k].x, a.x), __fadd_rn(v[k].y, a.y), __fadd_rn(v[k].z, a.z),
                           __fadd_rn(v[k].w, a.w));
        xr[i] = v[k];
      }
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < RMS_V; k++) {
    ss = fmaf(v[k].x, v[k].x, ss);
    ss = fmaf(v[k].y, v[k].y, ss);
    ss = fmaf(v[k].z, v[k].z, ss);
    ss = fmaf(v[k].w, v[k].w, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < 8 ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(red[0], (float)dim), eps));
#pragma unroll
  for (int k = 0; k < RMS_V; k++) {
    const int i = threadIdx.x + k * 256;
    if (i < nv) {
      const float4 o = make_float4(__fdiv_rn(__fmul_rn(v[k].x, g[k].x), rms), __fdiv_rn(__fmul_rn(v[k].y, g[k].y), rms),
                                   __fdiv_rn(__fmul_rn(v[k].z, g[k].z), rms), __fdiv_rn(__fmul_rn(v[k].w, g[k].w), rms));
      if (y) yr[i] = o;
      if (terms) store_terms4(terms, plane, (size_t)blockIdx.x * dim + 4 * i, o);
    }
  }
}

__global__ void __launch_bounds__(256) k_rms_norm(const float *__restrict__ x, const float *__restrict__ w,
                                                  float *y, int dim, float eps) {
  __shared__ float red[8];
  const float *xr = x + (size_t)blockIdx.x * dim;
  float *yr = y + (size_t)blockIdx.x * dim;
  float ss = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(red[0], (float)dim), eps));
  for (int i = threadIdx.x; i < dim; i += blockDim.x) yr[i] = __fdiv_rn(__fmul_rn(xr[i], w[i]), rms);
}

// rope_f32_interleaved (kernels/rope.rs:7-36): rotate (x[2j], x[2j+1]) by pos*inv_freq[j].
// sin/cos are evaluated in double and rounded once to float.
__global__ void k_rope(float *x, int seq, int row_dim, int base_pos, const float *__restrict__ inv_freq,
                       int half) {
  const int pairs = row_dim / 2;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < (long long)seq * pairs;
       idx += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(idx / pairs), p = (int)(idx % pairs), j = p % half;
    const float theta = __fmul_rn((float)(base_pos + r), inv_freq[j]);
    double sd, cd;
    sincos((double)theta, &sd, &cd);
    const float s = (float)sd, c = (float)cd;
    float *e = x + (size_t)r * row_dim + 2 * p;
    const float a = e[0], b = e[1];
    e[0] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    e[1] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
  }
}

__global__ void k_rope_table(float *x, int seq, int row_dim, int base_pos, const float *__restrict__ cos_t,
                             const float *__restrict__ sin_t, int half, const int *__restrict__ pos_dev) {
  if (pos_dev) base_pos = *pos_dev;
  const int pairs = row_dim / 2;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < (long long)seq * pairs;
       idx += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(idx / pairs), p = (int)(idx % pairs), j = p % half;
    const size_t t = (size_t)(base_pos + r) * half + j;
    const float c = cos_t[t], s = sin_t[t];
    float *e = x + (size_t)r * row_dim + 2 * p;
    const float a = e[0], b = e[1];
    e[0] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    e[1] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
  }
}

// sigmoid_f32 (kernels/sigmoid.rs:2-9) and silu (silu.rs:4-8).
__device__ __forceinline__ float sigmoid_ref(float x) {
  if (x >= 0.0f) return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
  const float z = expf(x);
  return __fdiv_rn(z, __fadd_rn(1.0f, z));
}
__device__ __forceinline__ float silu_ref(float x) { return __fmul_rn(x, sigmoid_ref(x)); }

__global__ void k_silu(float *x, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    x[i] = silu_ref(x[i]);
}
__global__ void k_mul(const float *a, const float *b, float *out, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    out[i] = __fmul_rn(a[i], b[i]);
}
__global__ void k_add(float *a, const float *b, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    a[i] = __fadd_rn(a[i], b[i]);
}
__global__ void k_silu_mul(const float *g, const float *u, float *out, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    out[i] = __fmul_rn(silu_ref(g[i]), u[i]);
}
// silu(g) * u written only as its three bf16 terms (n % 4 == 0, 16-byte aligned).
__global__ void k_silu_mul_terms(const float4 *__restrict__ g, const float4 *__restrict__ u, size_t n4,
                                 __nv_bfloat16 *__restrict__ terms) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    const float4 a = g[i], b = u[i];
    const float4 o = make_float4(__fmul_rn(silu_ref(a.x), b.x), __fmul_rn(silu_ref(a.y), b.y),
                                 __fmul_rn(silu_ref(a.z), b.z), __fmul_rn(silu_ref(a.w), b.w));
    store_terms4(terms, 4 * n4, 4 * i, o);
  }
}

// GreedySampler (greedy.rs:6-15): per-CTA ordered reduction of a contiguous chunk,
// then one CTA combines the chunk states in index order.
constexpr int ARGMAX_THREADS = 256;
constexpr int ARGMAX_CHUNK = 4096;

__device__ ArgState block_arg_reduce(ArgState s) {
  __shared__ ArgState sh[ARGMAX_THREADS / 32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {  // combine with the neighbour range to the right
    ArgState r;
    r.v = __shfl_down_sync(0xffffffffu, s.v, o);
    r.best = __shfl_down_sync(0xffffffffu, s.best, o);
    r.nan = __shfl_down_sync(0xffffffffu, s.nan, o);
    if ((lane & (2 * o - 1)) == 0) s = arg_combine(s, r);
  }
  if (lane == 0) sh[wid] = s;
  __syncthreads();
  ArgState t = arg_empty();
  if (threadIdx.x == 0)
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) t = arg_combine(t, sh[i]);
  __syncthreads();
  return t;
}

__global__ void __launch_bounds__(ARGMAX_THREADS) k_argmax_partial(const float *__restrict__ x, size_t n,
                                                                   ArgState *part) {
  const size_t lo = (size_t)blockIdx.x * ARGMAX_CHUNK;
  const size_t hi = lo + ARGMAX_CHUNK < n ? lo + ARGMAX_CHUNK : n;
  // each thread scans a contiguous sub-range so its sequential fold keeps index order
  const size_t per = (ARGMAX_CHUNK + ARGMAX_THREADS - 1) / ARGMAX_THREADS;
  ArgState s = arg_empty();
  for (size_t i = lo + threadIdx.x * per; i < lo + (threadIdx.x + 1) * per && i < hi; i++)
    s = arg_combine(s, arg_elem(x[i], (long long)i));
  s = block_arg_reduce(s);
  if (threadIdx.x == 0) part[blockIdx.x] = s;
}

__global__ void __launch_bounds__(ARGMAX_THREADS) k_argmax_final(const ArgState *part, int np, long long *out) {
  const int per = (np + ARGMAX_THREADS - 1) / ARGMAX_THREADS;
  ArgState s = arg_empty();
  for (int i = threadIdx.x * per; i < (threadIdx.x + 1) * per && i < np; i++) s = arg_combine(s, part[i]);
  s = block_arg_reduce(s);
  if (threadIdx.x == 0) *out = arg_result(s);
}

// The greedy argmax state of one vocabulary shard, indices shifted to the whole
// vocabulary; and the fold of the shards' states in shard (= index) order.
__global__ void __launch_bounds__(ARGMAX_THREADS) k_argmax_state(const ArgState *part, int np, long long offset,
                                                                 ArgState *out) {
  const int per = (np + ARGMAX_THREADS - 1) / ARGMAX_THREADS;
  ArgState s = arg_empty();
  for (int i = threadIdx.x * per; i < (threadIdx.x + 1) * per && i < np; i++) s = arg_combine(s, part[i]);
  s = block_arg_reduce(s);
  if (threadIdx.x == 0) {
    if (s.best >= 0) s.best += offset;
    if (s.nan >= 0) s.nan += offset;
    *out = s;
  }
}
__global__ void k_argmax_fold(const ArgState *states, int n, long long *out) {
  ArgState s = arg_empty();
  for (int i = 0; i < n; i++) s = arg_combine(s, states[i]);
  *out = arg_result(s);
}

// ------------------------------------------------------------------------------------
// launchers
// ------------------------------------------------------------------------------------
static int g_num_sms = 0;
static int num_sms() {
  if (!g_num_sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  return g_num_sms;
}

static inline int grid_for(size_t work, int per_block, int cap) {
  size_t g = (work + per_block - 1) / per_block;
  if (g < 1) g = 1;
  if (g > (size_t)cap) g = cap;
  return (int)g;
}

cudaError_t launch_quantize_q8_0(cudaStream_t s, const float *x, size_t n, void *out) {
  size_t nb = n / QK;
  k_quantize_q8_0<<<grid_for(nb, 8, 65535), 256, 0, s>>>(x, nb, (uint8_t *)out);
  return cudaGetLastError();
}

// The fused single-row matvec (k_matvec with MvArgs): every matrix must take the
// streaming path (whole 256-element multiples, 16-byte rows and pointers).
bool matvec_fused_ok(const MvArgs &a, int wtype) {
  if (a.n < 1 || a.n > 3 || !a.x || a.in_dim <= 0 || a.in_dim % 256 || a.in_dim > MV_CONS * 2048) return false;
  if (wtype != SQ_Q8_0 && wtype != SQ_Q4_0 && wtype != SQ_BF16) return false;
  const int pw = wtype == SQ_Q8_0 ? pair_words<SQ_Q8_0>() : (wtype == SQ_Q4_0 ? pair_words<SQ_Q4_0>() : pair_words<SQ_BF16>());
  if ((size_t)(a.in_dim / 64) * pw * 4 > MV_SLOT) return false;
  auto al = [](const void *p) { return ((uintptr_t)p & 15) == 0; };
  if (!al(a.x) || (a.xu && !al(a.xu)) || (a.norm_w && !al(a.norm_w)) || (a.xu && a.norm_w)) return false;
  for (int i = 0; i < a.n; i++)
    if (!a.w[i] || !al(a.w[i]) || !a.y[i] || a.out_dim[i] <= 0) return false;
  if (a.gate_act && (a.n != 2 || a.out_dim[0] != a.out_dim[1] || a.res[0] || a.res[1] || a.xu ||
                     (a.out_dim[0] + num_sms() - 1) / num_sms() > MV_GATE_ROWS))
    return false;
  return true;
}

// Failure-detection tests only: SQ_TEST_SKIP_MATVEC=n (read at the first k_matvec
// launch of the process) makes the process's n-th k_matvec launch leave its first
// tile uncopied, so the consumers' bounded wait for it expires, the kernel sets
// g_mv_err and returns, and the next status check reports a timeout.
static int mv_test_skip() {
  static const long n = [] {
    const char *v = getenv("SQ_TEST_SKIP_MATVEC");
    return v ? strtol(v, nullptr, 10) : 0L;
  }();
  static std::atomic<long> launches{0};
  return n > 0 && ++launches == n ? 1 : 0;
}

template <int T, int MODE>
static cudaError_t matvec_mode_t(cudaStream_t s, const MvArgs &a, bool pdl = false) {
  const size_t mv_smem = mv_smem_bytes<T>(a.in_dim);
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(k_matvec<T, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mv_smem);
    attr_set = true;
  }
  MvArgs b = a;
  b.test_skip = mv_test_skip();
  return launch_ex(k_matvec<T, MODE>, dim3(num_sms()), dim3(MV_THREADS), mv_smem, s, pdl, b);
}
template <int T>
static cudaError_t matvec_fused_t(cudaStream_t s, const MvArgs &a, bool pdl) {
  if (a.norm_w) return matvec_mode_t<T, MV_NORM>(s, a, pdl);
  if (a.xu) return matvec_mode_t<T, MV_SILU>(s, a, pdl);
  if (a.n > 1 || a.res[0]) return matvec_mode_t<T, MV_GENERAL>(s, a, pdl);
  return matvec_mode_t<T, MV_PLAIN>(s, a, pdl);
}

cudaError_t launch_matvec_fused(cudaStream_t s, const MvArgs &a, int wtype, bool pdl) {
  if (!matvec_fused_ok(a, wtype)) return cudaErrorNotSupported;
  if (wtype == SQ_Q8_0) return matvec_fused_t<SQ_Q8_0>(s, a, pdl);
  if (wtype == SQ_Q4_0) return matvec_fused_t<SQ_Q4_0>(s, a, pdl);
  return matvec_fused_t<SQ_BF16>(s, a, pdl);
}

bool pdl_enabled() {
  static const bool on = [] {
    const char *e = getenv("SQB200_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <int T>
static void linear_f32_t(cudaStream_t s, const float *x, int m, int in_dim, const uint8_t *w, int out_dim,
                         float *y) {
  const int grid = grid_for((size_t)out_dim, 8, num_sms() * 8);
  const size_t mv_smem = mv_smem_bytes<T>(in_dim);
  if (m == 1 && in_dim % 256 == 0 && in_dim <= MV_CONS * 2048 && (size_t)(in_dim / 64) * pair_words<T>() * 4 <= MV_SLOT &&
      ((uintptr_t)w & 15) == 0 && ((uintptr_t)x & 15) == 0) {  // 16-byte row starts; a row fits a slot
    MvArgs a{};
    a.x = x;
    a.in_dim = in_dim;
    a.n = 1;
    a.w[0] = w;
    a.out_dim[0] = out_dim;
    a.y[0] = y;
    matvec_mode_t<T, MV_PLAIN>(s, a);
  } else if (m <= 1)
    k_linear_f32<T, 1><<<grid, 256, 0, s>>>(x, m, in_dim, w, out_dim, y);
  else if (m <= 4)
    k_linear_f32<T, 4><<<grid, 256, 0, s>>>(x, m, in_dim, w, out_dim, y);
  else
    k_linear_f32<T, 8><<<grid, 256, 0, s>>>(x, m, in_dim, w, out_dim, y);
}

template <int T>
static void linear_q8_t(cudaStream_t s, const uint8_t *xq, int m, int in_dim, const uint8_t *w, int out_dim,
                        float *y) {
  const int grid = grid_for((size_t)out_dim, 8, num_sms() * 8);
  if (m <= 1)
    k_linear_q8<T, 1><<<grid, 256, 0, s>>>(xq, m, in_dim, w, out_dim, y);
  else if (m <= 4)
    k_linear_q8<T, 4><<<grid, 256, 0, s>>>(xq, m, in_dim, w, out_dim, y);
  else
    k_linear_q8<T, 8><<<grid, 256, 0, s>>>(xq, m, in_dim, w, out_dim, y);
}

cudaError_t launch_linear(cudaStream_t s, const float *x, int m, int in_dim, const void *w, int wtype,
                          int out_dim, float *y, int acts_q8, void *xq, float *ws, size_t ws_floats) {
  const uint8_t *wb = (const uint8_t *)w;
  if (acts_q8 && wtype != SQ_BF16) {
    if (x) {
      cudaError_t e = launch_quantize_q8_0(s, x, (size_t)m * in_dim, xq);
      if (e != cudaSuccess) return e;
    }
    if (wtype == SQ_Q8_0) linear_q8_t<SQ_Q8_0>(s, (const uint8_t *)xq, m, in_dim, wb, out_dim, y);
    else linear_q8_t<SQ_Q4_0>(s, (const uint8_t *)xq, m, in_dim, wb, out_dim, y);
  } else if (m >= 2) {  // several rows (prefill): tensor cores, else the CUDA-core tiled GEMM
    if (gemm_tc_enabled() && gemm_tc_supported(m, in_dim, x, w, wtype, ws, ws_floats))
      return launch_gemm_tc(s, x, m, in_dim, w, wtype, out_dim, y, ws, ws_floats);
    return launch_gemm_f32w(s, x, m, in_dim, w, wtype, out_dim, y, ws, ws_floats);
  } else {
    if (wtype == SQ_Q8_0) linear_f32_t<SQ_Q8_0>(s, x, m, in_dim, wb, out_dim, y);
    else if (wtype == SQ_Q4_0) linear_f32_t<SQ_Q4_0>(s, x, m, in_dim, wb, out_dim, y);
    else linear_f32_t<SQ_BF16>(s, x, m, in_dim, wb, out_dim, y);
  }
  return cudaGetLastError();
}

cudaError_t launch_embed(cudaStream_t s, const uint32_t *tokens, int n, const void *w, int wtype, int dim, int vocab,
                         float *out) {
  dim3 grid(grid_for((size_t)dim, 256, 64), n);
  const uint8_t *wb = (const uint8_t *)w;
  if (wtype == SQ_Q8_0) k_embed<SQ_Q8_0><<<grid, 256, 0, s>>>(tokens, wb, dim, vocab, out);
  else if (wtype == SQ_Q4_0) k_embed<SQ_Q4_0><<<grid, 256, 0, s>>>(tokens, wb, dim, vocab, out);
  else k_embed<SQ_BF16><<<grid, 256, 0, s>>>(tokens, wb, dim, vocab, out);
  return cudaGetLastError();
}

cudaError_t launch_dequantize(cudaStream_t s, const void *blocks, int wtype, size_t n, float *out) {
  const int grid = grid_for(n, 256, num_sms() * 16);
  const uint8_t *b = (const uint8_t *)blocks;
  if (wtype == SQ_Q8_0) k_dequant<SQ_Q8_0><<<grid, 256, 0, s>>>(b, n, out);
  else if (wtype == SQ_Q4_0) k_dequant<SQ_Q4_0><<<grid, 256, 0, s>>>(b, n, out);
  else k_dequant<SQ_BF16><<<grid, 256, 0, s>>>(b, n, out);
  return cudaGetLastError();
}

cudaError_t launch_rms_norm(cudaStream_t s, const float *x, const float *w, float *y, int rows, int dim,
                            float eps) {
  if (dim % 4 == 0 && dim <= RMS_V * 4 * 256 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)w & 15) == 0 &&
      ((uintptr_t)y & 15) == 0)
    k_rms_norm_v<<<rows, 256, 0, s>>>(const_cast<float *>(x), w, y, dim, eps, nullptr, 0, nullptr);
  else
    k_rms_norm<<<rows, 256, 0, s>>>(x, w, y, dim, eps);
  return cudaGetLastError();
}

cudaError_t launch_rope_rows(cudaStream_t s, float *x, int seq, int row_dim, int base_pos,
                             const float *inv_freq, int half) {
  k_rope<<<grid_for((size_t)seq * row_dim / 2, 256, num_sms() * 8), 256, 0, s>>>(x, seq, row_dim, base_pos,
                                                                                 inv_freq, half);
  return cudaGetLastError();
}

cudaError_t launch_rope_rows_table(cudaStream_t s, float *x, int seq, int row_dim, int base_pos,
                                   const float *cos_t, const float *sin_t, int half, const int *pos_dev) {
  k_rope_table<<<grid_for((size_t)seq * row_dim / 2, 256, num_sms() * 8), 256, 0, s>>>(
      x, seq, row_dim, base_pos, cos_t, sin_t, half, pos_dev);
  return cudaGetLastError();
}

cudaError_t launch_silu(cudaStream_t s, float *x, size_t n) {
  k_silu<<<grid_for(n, 256, num_sms() * 8), 256, 0, s>>>(x, n);
  return cudaGetLastError();
}
cudaError_t launch_mul(cudaStream_t s, const float *a, const float *b, float *out, size_t n) {
  k_mul<<<grid_for(n, 256, num_sms() * 8), 256, 0, s>>>(a, b, out, n);
  return cudaGetLastError();
}
cudaError_t launch_add(cudaStream_t s, float *a, const float *b, size_t n) {
  k_add<<<grid_for(n, 256, num_sms() * 8), 256, 0, s>>>(a, b, n);
  return cudaGetLastError();
}
bool rms_norm_terms_ok(const float *x, const float *w, int dim) {
  return dim % 4 == 0 && dim <= RMS_V * 4 * 256 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)w & 15) == 0;
}
cudaError_t launch_rms_norm_terms(cudaStream_t s, const float *x, const float *w, void *terms, int rows, int dim,
                                  float eps) {
  if (!rms_norm_terms_ok(x, w, dim) || ((uintptr_t)terms & 15)) return cudaErrorNotSupported;
  k_rms_norm_v<<<rows, 256, 0, s>>>(const_cast<float *>(x), w, nullptr, dim, eps, (__nv_bfloat16 *)terms,
                                    (size_t)rows * dim, nullptr);
  return cudaGetLastError();
}
cudaError_t launch_add_rms_norm_terms(cudaStream_t s, float *x, const float *add, const float *w, void *terms,
                                      int rows, int dim, float eps) {
  if (!rms_norm_terms_ok(x, w, dim) || ((uintptr_t)terms & 15) || ((uintptr_t)add & 15)) return cudaErrorNotSupported;
  k_rms_norm_v<<<rows, 256, 0, s>>>(x, w, nullptr, dim, eps, (__nv_bfloat16 *)terms, (size_t)rows * dim, add);
  return cudaGetLastError();
}
cudaError_t launch_silu_mul_terms(cudaStream_t s, const float *g, const float *u, void *terms, size_t n) {
  if (n % 4 || ((uintptr_t)g & 15) || ((uintptr_t)u & 15) || ((uintptr_t)terms & 15)) return cudaErrorNotSupported;
  k_silu_mul_terms<<<grid_for(n / 4, 256, num_sms() * 8), 256, 0, s>>>(
      reinterpret_cast<const float4 *>(g), reinterpret_cast<const float4 *>(u), n / 4, (__nv_bfloat16 *)terms);
  return cudaGetLastError();
}

cudaError_t launch_silu_mul(cudaStream_t s, const float *g, const float *u, float *out, size_t n) {
  k_silu_mul<<<grid_for(n, 256, num_sms() * 8), 256, 0, s>>>(g, u, out, n);
  return cudaGetLastError();
}

int argmax_partials(size_t n) { return (int)((n + ARGMAX_CHUNK - 1) / ARGMAX_CHUNK); }

cudaError_t launch_argmax_state(cudaStream_t s, const float *x, size_t n, long long offset, void *partials,
                                void *state) {
  const int np = argmax_partials(n);
  k_argmax_partial<<<np, ARGMAX_THREADS, 0, s>>>(x, n, (ArgState *)partials);
  k_argmax_state<<<1, ARGMAX_THREADS, 0, s>>>((const ArgState *)partials, np, offset, (ArgState *)state);
  return cudaGetLastError();
}
cudaError_t launch_argmax_fold(cudaStream_t s, const void *states, int n, long long *out) {
  k_argmax_fold<<<1, 1, 0, s>>>((const ArgState *)states, n, out);
  return cudaGetLastError();
}
size_t argmax_state_bytes() { return sizeof(ArgState); }

unsigned *mv_err_ptr() {
  static unsigned *ptrs[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  if (!ptrs[dev]) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_mv_err) != cudaSuccess) return nullptr;
    ptrs[dev] = (unsigned *)p;
  }
  return ptrs[dev];
}

__global__ void k_collect_status(const long long *argmax, const unsigned *e0, const unsigned *e1, const unsigned *e2,
                                 const unsigned *e3, unsigned long long *out) {
  if (threadIdx.x != 0) return;
  out[0] = (unsigned long long)*argmax;
  out[1] = e0 ? *(volatile const unsigned *)e0 : 0u;
  out[2] = e1 ? *(volatile const unsigned *)e1 : 0u;
  out[3] = e2 ? *(volatile const unsigned *)e2 : 0u;
  out[4] = e3 ? *(volatile const unsigned *)e3 : 0u;
}

cudaError_t launch_collect_status(cudaStream_t s, const long long *argmax, const unsigned *e0, const unsigned *e1,
                                  const unsigned *e2, const unsigned *e3, unsigned long long *out) {
  k_collect_status<<<1, 32, 0, s>>>(argmax, e0, e1, e2, e3, out);
  return cudaGetLastError();
}

unsigned matvec_status(bool clear) {
  unsigned v = 0;
  cudaMemcpyFromSymbol(&v, g_mv_err, sizeof(v));
  if (clear && v) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(g_mv_err, &z, sizeof(z));
  }
  return v;
}

int device_wait_status(bool clear, const char *what) {
  const unsigned mv = matvec_status(clear), tc = gemm_tc_status(clear);
  if (!mv && !tc) return SQ_OK;
  std::string who = mv ? "the streaming matvec" : "";
  if (tc) who += std::string(mv ? " and " : "") + "a tensor-core kernel";
  return fail(SQ_ERR_TIMEOUT, std::string(what) + ": a bounded wait of " + who + " expired");
}

cudaError_t launch_argmax(cudaStream_t s, const float *x, size_t n, void *partials, long long *out) {
  const int np = argmax_partials(n);
  k_argmax_partial<<<np, ARGMAX_THREADS, 0, s>>>(x, n, (ArgState *)partials);
  k_argmax_final<<<1, ARGMAX_THREADS, 0, s>>>((const ArgState *)partials, np, out);
  return cudaGetLastError();
}

}  // namespace sq

// =====================================================================================
// C ABI, op level. Validation mirrors the reference's checks before any launch.
// =====================================================================================
using namespace sq;

static inline bool aligned16(const void *p) { return ((uintptr_t)p & 15) == 0; }

// Stream-ordered scratch for the op-level calls. The device's default memory pool
// is told to keep freed memory, so repeated calls reuse it instead of returning
// it to the driver at every synchronization.
static cudaError_t scratch_alloc(void **p, size_t bytes, cudaStream_t s) {
  static bool pool_set[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 64 && !pool_set[dev]) {
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
      uint64_t keep = UINT64_MAX;
      cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    }
    pool_set[dev] = true;
  }
  return cudaMallocAsync(p, bytes, s);
}

extern "C" const char *sq_last_error(void) { return g_last_error.c_str(); }
extern "C" const char *sq_version(void) { return "squirrel-b200 0.1 (sm_100a)"; }
extern "C" int sq_wait_status(int clear) { return sq::device_wait_status(clear != 0, "wait_status"); }

// Workspace of the tensor-core GEMM for an op-level call (m >= 2, f32 activations):
// the three bf16 activation terms plus up to 16 split-K partials.
static size_t tc_workspace_floats(int m, int in_dim, int out_dim, int wtype, bool q8) {
  (void)wtype;
  if (q8 || m < 2) return 0;
  return (size_t)3 * m * in_dim / 2 + 64 + (size_t)16 * m * out_dim;
}

static int check_linear(const float *input, int m, int in_dim, const void *weight, int wtype, int out_dim,
                        float *output) {
  if (!input || !weight || !output) return fail(SQ_ERR_ARG, "linear: null pointer");
  if (!is_weight_type(wtype)) return fail(SQ_ERR_INVALID_TYPE, "linear: weight type must be Q8_0, Q4_0 or BF16");
  if (m <= 0 || in_dim <= 0 || out_dim <= 0 || in_dim % QK)
    return fail(SQ_ERR_SHAPE, "linear: in_dim must be a positive multiple of 32 and m, out_dim positive");
  if (!aligned16(input) || ((uintptr_t)weight & 1) || (wtype == SQ_BF16 && !aligned16(weight)))
    return fail(SQ_ERR_ALIGN, "linear: input must be 16-byte aligned, blocks 2-byte aligned (BF16: 16)");
  return SQ_OK;
}

extern "C" int sq_linear(void *stream, const float *input, int m, int in_dim, const void *weight, int wtype,
                         int out_dim, float *output, int acts) {
  int st = check_linear(input, m, in_dim, weight, wtype, out_dim, output);
  if (st) return st;
  cudaStream_t s = (cudaStream_t)stream;
  void *xq = nullptr;
  const bool q8 = acts == SQ_ACTS_Q8 && wtype != SQ_BF16;
  if (q8) SQ_CUDA(scratch_alloc(&xq, (size_t)m * (in_dim / QK) * Q8_BYTES, s));
  void *ws = nullptr;
  const size_t ws_floats = tc_workspace_floats(m, in_dim, out_dim, wtype, q8);
  if (ws_floats) SQ_CUDA(scratch_alloc(&ws, ws_floats * sizeof(float), s));
  cudaError_t e = launch_linear(s, input, m, in_dim, weight, wtype, out_dim, output, q8, xq, (float *)ws, ws_floats);
  if (xq) cudaFreeAsync(xq, s);
  if (ws) cudaFreeAsync(ws, s);
  if (e != cudaSuccess) return cuda_fail(e, "sq_linear");
  return SQ_OK;
}

extern "C" int sq_linear_shared(void *stream, const float *input, int m, int in_dim, int n,
                                const void *const *weights, const int *out_dims, int wtype,
                                float *const *outputs, int acts, void *act_scratch) {
  if (n <= 0 || !weights || !out_dims || !outputs) return fail(SQ_ERR_SHAPE, "linear_shared: no projections");
  for (int i = 0; i < n; i++) {
    int st = check_linear(input, m, in_dim, weights[i], wtype, out_dims[i], outputs[i]);
    if (st) return st;
  }
  const bool q8 = acts == SQ_ACTS_Q8 && wtype != SQ_BF16;
  if (q8 && !act_scratch) return fail(SQ_ERR_ARG, "linear_shared: Q8 activations need act_scratch");
  cudaStream_t s = (cudaStream_t)stream;
  if (q8) {  // quantize the shared input once (linear.rs:117-127)
    cudaError_t e = launch_quantize_q8_0(s, input, (size_t)m * in_dim, act_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "linear_shared quantize");
  }
  int widest = 0;
  for (int i = 0; i < n; i++) widest = std::max(widest, out_dims[i]);
  void *ws = nullptr;
  const size_t ws_floats = tc_workspace_floats(m, in_dim, widest, wtype, q8);
  if (ws_floats) SQ_CUDA(scratch_alloc(&ws, ws_floats * sizeof(float), s));
  for (int i = 0; i < n; i++) {
    cudaError_t e = launch_linear(s, q8 ? nullptr : input, m, in_dim, weights[i], wtype, out_dims[i],
                                  outputs[i], q8, act_scratch, (float *)ws, ws_floats);
    if (e != cudaSuccess) {
      if (ws) cudaFreeAsync(ws, s);
      return cuda_fail(e, "sq_linear_shared");
    }
  }
  if (ws) cudaFreeAsync(ws, s);
  return SQ_OK;
}

extern "C" int sq_embed(void *stream, const uint32_t *tokens, int n_tokens, const void *weight, int wtype,
                        int embed_dim, int vocab, float *out) {
  if (!tokens || !weight || !out) return fail(SQ_ERR_ARG, "embed: null pointer");
  if (!is_weight_type(wtype)) return fail(SQ_ERR_INVALID_TYPE, "embed: weight type must be Q8_0, Q4_0 or BF16");
  if (n_tokens <= 0) return fail(SQ_ERR_EMPTY, "embed: no tokens");
  if (embed_dim <= 0 || embed_dim % QK || vocab <= 0) return fail(SQ_ERR_SHAPE, "embed: embed_dim must be a multiple of 32");
  cudaError_t e = launch_embed((cudaStream_t)stream, tokens, n_tokens, weight, wtype, embed_dim, vocab, out);
  if (e != cudaSuccess) return cuda_fail(e, "sq_embed");
  return SQ_OK;
}

extern "C" int sq_rms_norm(void *stream, const float *input, const float *weight, float *output, int rows,
                           int dim, float eps) {
  if (!input || !weight || !output) return fail(SQ_ERR_ARG, "rms_norm: null pointer");
  if (rows < 0 || dim <= 0) return fail(SQ_ERR_SHAPE, "rms_norm: bad shape");
  if (rows == 0) return SQ_OK;
  cudaError_t e = launch_rms_norm((cudaStream_t)stream, input, weight, output, rows, dim, eps);
  if (e != cudaSuccess) return cuda_fail(e, "sq_rms_norm");
  return SQ_OK;
}

extern "C" int sq_rms_norm_inplace(void *stream, float *x, const float *weight, int rows, int dim, float eps) {
  return sq_rms_norm(stream, x, weight, x, rows, dim, eps);
}

extern "C" int sq_rope_rows(void *stream, float *x, int seq, int row_dim, int base_pos, const float *inv_freq,
                            int half) {
  if (!x || !inv_freq) return fail(SQ_ERR_ARG, "rope_rows: null pointer");
  if (half <= 0 || seq <= 0 || row_dim <= 0 || row_dim % (2 * half) || base_pos < 0)
    return fail(SQ_ERR_SHAPE, "rope_rows: row width must be a multiple of head_dim = 2*half");
  cudaError_t e = launch_rope_rows((cudaStream_t)stream, x, seq, row_dim, base_pos, inv_freq, half);
  if (e != cudaSuccess) return cuda_fail(e, "sq_rope_rows");
  return SQ_OK;
}

extern "C" int sq_silu(void *stream, float *x, size_t n) {
  if (!x) return fail(SQ_ERR_ARG, "silu: null pointer");
  if (!n) return SQ_OK;
  cudaError_t e = launch_silu((cudaStream_t)stream, x, n);
  return e == cudaSuccess ? SQ_OK : cuda_fail(e, "sq_silu");
}
extern "C" int sq_elementwise_mul(void *stream, const float *a, const float *b, float *out, size_t n) {
  if (!a || !b || !out) return fail(SQ_ERR_ARG, "elementwise_mul: null pointer");
  if (!n) return SQ_OK;
  cudaError_t e = launch_mul((cudaStream_t)stream, a, b, out, n);
  return e == cudaSuccess ? SQ_OK : cuda_fail(e, "sq_elementwise_mul");
}
extern "C" int sq_elementwise_add(void *stream, float *a, const float *b, size_t n) {
  if (!a || !b) return fail(SQ_ERR_ARG, "elementwise_add: null pointer");
  if (!n) return SQ_OK;
  cudaError_t e = launch_add((cudaStream_t)stream, a, b, n);
  return e == cudaSuccess ? SQ_OK : cuda_fail(e, "sq_elementwise_add");
}
extern "C" int sq_silu_mul(void *stream, const float *gate, const float *up, float *out, size_t n) {
  if (!gate || !up || !out) return fail(SQ_ERR_ARG, "silu_mul: null pointer");
  if (!n) return SQ_OK;
  cudaError_t e = launch_silu_mul((cudaStream_t)stream, gate, up, out, n);
  return e == cudaSuccess ? SQ_OK : cuda_fail(e, "sq_silu_mul");
}

extern "C" int sq_quantize_row_q8_0(void *stream, const float *src, size_t n, void *out_blocks) {
  if (!src || !out_blocks) return fail(SQ_ERR_ARG, "quantize_row_q8_0: null pointer");
  if (n % QK) return fail(SQ_ERR_SHAPE, "quantize_row_q8_0: length must be a multiple of 32");
  if ((uintptr_t)out_blocks & 1) return fail(SQ_ERR_ALIGN, "quantize_row_q8_0: output must be 2-byte aligned");
  if (!n) return SQ_OK;
  cudaError_t e = launch_quantize_q8_0((cudaStream_t)stream, src, n, out_blocks);
  return e == cudaSuccess ? SQ_OK : cuda_fail(e, "sq_quantize_row_q8_0");
}

extern "C" int sq_dequantize(void *stream, const void *blocks, int wtype, size_t n_elems, float *out) {
  if (!blocks || !out) return fail(SQ_ERR_ARG, "dequantize: null pointer");
  if (!is_weight_type(wtype)) return fail(SQ_ERR_INVALID_TYPE, "dequantize: type must be Q8_0, Q4_0 or BF16");
  if (n_elems % QK) return fail(SQ_ERR_SHAPE, "dequantize: length must be a multiple of 32");
  if ((uintptr_t)blocks & 1) return fail(SQ_ERR_ALIGN, "dequantize: blocks must be 2-byte aligned");
  if (!n_elems) return SQ_OK;
  cudaError_t e = launch_dequantize((cudaStream_t)stream, blocks, wtype, n_elems, out);
  return e == cudaSuccess ? SQ_OK : cuda_fail(e, "sq_dequantize");
}

extern "C" int sq_argmax(void *stream, const float *logits, size_t n, int64_t *out_index) {
  if (!logits || !out_index) return fail(SQ_ERR_ARG, "argmax: null pointer");
  if (!n) return fail(SQ_ERR_EMPTY, "argmax: empty logits");
  cudaStream_t s = (cudaStream_t)stream;
  void *part = nullptr;
  SQ_CUDA(scratch_alloc(&part, (size_t)argmax_partials(n) * sizeof(ArgState), s));
  cudaError_t e = launch_argmax(s, logits, n, part, (long long *)out_index);
  cudaFreeAsync(part, s);
  return e == cudaSuccess ? SQ_OK : cuda_fail(e, "sq_argmax");
}

extern "C" int sq_sdpa_cached(void *stream, const float *q, const float *k, const float *v, float *out,
                              int seq_q, int seq_k, int n_heads, int n_kv_heads, int head_dim) {
  if (!q || !k || !v || !out) return fail(SQ_ERR_ARG, "sdpa_cached: null pointer");
  if (n_kv_heads <= 0 || head_dim <= 0 || n_heads <= 0 || n_heads % n_kv_heads)
    return fail(SQ_ERR_SHAPE, "sdpa_cached: n_heads must be a positive multiple of n_kv_heads");
  if (seq_q <= 0 || seq_k < seq_q) return fail(SQ_ERR_SHAPE, "sdpa_cached: need 0 < seq_q <= seq_k");
  if (head_dim > 256 || head_dim % 32) return fail(SQ_ERR_SHAPE, "sdpa_cached: head_dim must be a multiple of 32, <= 256");
  cudaStream_t s = (cudaStream_t)stream;
  const long long kps = (long long)n_kv_heads * head_dim, khs = head_dim;
  const size_t tc_bytes = attn_tc_workspace_bytes(seq_q, seq_k, n_heads, n_kv_heads);
  if (attn_tc_supported(seq_q, seq_k, n_heads, n_kv_heads, head_dim, kps, khs, q, k, v, tc_bytes)) {
    void *ws = nullptr;  // tensor cores: workspace for the bf16 terms of q, k and v
    SQ_CUDA(scratch_alloc(&ws, tc_bytes, s));
    cudaError_t e = launch_attn_tc(s, q, k, v, out, seq_q, seq_k, n_heads, n_kv_heads, head_dim, kps, khs, ws, tc_bytes);
    cudaFreeAsync(ws, s);
    return e == cudaSuccess ? SQ_OK : cuda_fail(e, "sq_sdpa_cached");
  }
  const int ns = sdpa_num_splits(seq_q, seq_k, n_heads);
  float *part = nullptr;
  if (ns > 1) SQ_CUDA(scratch_alloc((void **)&part, sdpa_partials_floats(seq_q, n_heads, head_dim, ns) * 4, s));
  cudaError_t e = launch_sdpa(s, q, k, v, out, seq_q, seq_k, n_heads, n_kv_heads, head_dim,
                              (long long)n_kv_heads * head_dim, head_dim, ns, part);
  if (part) cudaFreeAsync(part, s);
  return e == cudaSuccess ? SQ_OK : cuda_fail(e, "sq_sdpa_cached");
}

namespace sq {
__global__ void k_kv_append(const float *__restrict__ k, const float *__restrict__ v, float *kc, float *vc, int n,
                            int n_kv, int hd, int pos, int max_ctx, const int *__restrict__ pos_dev) {
  if (pos_dev) pos = *pos_dev;
  const long long total = (long long)n * n_kv * hd;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int d = (int)(i % hd);
    const int g = (int)((i / hd) % n_kv);
    const int r = (int)(i / ((long long)hd * n_kv));
    const size_t dst = ((size_t)g * max_ctx + pos + r) * hd + d;
    kc[dst] = k[i];
    vc[dst] = v[i];
  }
}

cudaError_t launch_kv_append(cudaStream_t s, const float *k, const float *v, float *kc, float *vc, int n,
                             int n_kv, int hd, int pos, int max_ctx, const int *pos_dev) {
  k_kv_append<<<grid_for((size_t)n * n_kv * hd, 256, num_sms() * 8), 256, 0, s>>>(k, v, kc, vc, n, n_kv, hd,
                                                                                  pos, max_ctx, pos_dev);
  return cudaGetLastError();
}

// RoPE of the q and k rows (rope.rs:7-36, the cos/sin table of k_rope_table) and the
// append of the rotated K and the V rows to the cache (kv_cache.rs:8-78), one launch:
// work item p of a row is q pair p (p < Q/2), k pair p - Q/2, or v pair p - Q/2 - KVd/2.
// The arithmetic is k_rope_table's and k_kv_append's; q is rotated in place, k only
// into the cache.
__global__ void k_rope_append(float *q, const float *__restrict__ k, const float *__restrict__ v, float *kc,
                              float *vc, int n, int Q, int KVd, int hd, int max_ctx, int pos,
                              const float *__restrict__ cos_t, const float *__restrict__ sin_t,
                              const int *__restrict__ pos_dev) {
  pdl_wait();
  pdl_trigger();
  if (pos_dev) pos = *pos_dev;
  const int half = hd / 2, qp = Q / 2, kp = KVd / 2, per = qp + 2 * kp;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < (long long)n * per;
       idx += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(idx / per), p = (int)(idx % per);
    if (p < qp + kp) {
      const int pr = p < qp ? p : p - qp;  // pair index within the q or k row
      const size_t t = (size_t)(pos + r) * half + pr % half;
      const float c = cos_t[t], sn = sin_t[t];
      const float *src = p < qp ? q + (size_t)r * Q + 2 * pr : k + (size_t)r * KVd + 2 * pr;
      const float a = src[0], b = src[1];
      const float ra = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn));
      const float rb = __fadd_rn(__fmul_rn(a, sn), __fmul_rn(b, c));
      if (p < qp) {
        float *e = q + (size_t)r * Q + 2 * pr;
        e[0] = ra;
        e[1] = rb;
      } else {
        const int g = 2 * pr / hd, d = 2 * pr % hd;
        float *dst = kc + ((size_t)g * max_ctx + pos + r) * hd + d;
        dst[0] = ra;
        dst[1] = rb;
      }
    } else {
      const int pv = p - qp - kp, g = 2 * pv / hd, d = 2 * pv % hd;
      const float *src = v + (size_t)r * KVd + 2 * pv;
      float *dst = vc + ((size_t)g * max_ctx + pos + r) * hd + d;
      dst[0] = src[0];
      dst[1] = src[1];
    }
  }
}

cudaError_t launch_rope_append(cudaStream_t s, float *q, const float *k, const float *v, float *kc, float *vc,
                               int n, int Q, int KVd, int hd, int pos, int max_ctx, const float *cos_t,
                               const float *sin_t, const int *pos_dev, bool pdl) {
  const size_t items = (size_t)n * (Q / 2 + KVd);
  return launch_ex(k_rope_append, dim3(grid_for(items, 256, num_sms() * 8)), dim3(256), 0, s, pdl, q, k, v, kc, vc,
                   n, Q, KVd, hd, max_ctx, pos, cos_t, sin_t, pos_dev);
}
__global__ void k_add_int(int *p, int v) { *p += v; }
__global__ void k_store_int(int *p, int v) { *p = v; }
cudaError_t launch_set_int(cudaStream_t s, int *p, int v) {
  k_store_int<<<1, 1, 0, s>>>(p, v);
  return cudaGetLastError();
}
cudaError_t launch_add_int(cudaStream_t s, int *p, int v) {
  k_add_int<<<1, 1, 0, s>>>(p, v);
  return cudaGetLastError();
}

__global__ void k_feedback(const long long *argmax, uint32_t *tok, uint32_t *out_ids, int step) {
  const uint32_t t = (uint32_t)argmax[0];
  tok[0] = t;
  if (out_ids) out_ids[step] = t;
}

cudaError_t launch_feedback(cudaStream_t s, const long long *argmax, uint32_t *tok, uint32_t *out_ids, int step) {
  k_feedback<<<1, 1, 0, s>>>(argmax, tok, out_ids, step);
  return cudaGetLastError();
}
}  // namespace sq
