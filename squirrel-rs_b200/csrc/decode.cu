// decode.cu — the persistent single-token decode kernel for sm_100a.
//
// One cooperative launch per token runs the whole of Llama3_2::forward for one
// token (models/llama/model.rs:45-97 with layers.rs:81-109) plus GreedySampler
// (greedy.rs:6-15): embedding, L x [RMSNorm + QKV + RoPE + KV append, GQA
// attention, O + residual, RMSNorm + gate/up + SiLU*up, down + residual], final
// RMSNorm, LM head, argmax — and feeds the argmax back as the next token id.
//
// Layout: one CTA of NC warps (NGRP groups of four) per SM. Every weight row the
// CTA owns for the whole token streams through a ring of NSLOT shared-memory slots
// with 1-D bulk async copies (cp.async.bulk ... mbarrier::complete_tx): the last
// warp to finish with a slot immediately refills it with the tile NSLOT positions
// ahead in the CTA's tile table (built once per context), so NSLOT tiles are always
// in flight, also while the warps wait for another stage's output. The warps decode
// the GGUF blocks straight from shared memory (native 34/18/64-byte layout) against
// the stage input, staged once per CTA in shared memory (f32, or quantized to Q8_0
// blocks for W8A8 contexts), four weight rows per warp at a time, and finish each
// row inside the warp (RoPE, residual add, SiLU*up, logits). CTAs hand vectors to
// each other as tagged words that the consumers poll (no grid barrier): after QKV,
// attention, O, gate/up and down.
//
// Every wait (mbarrier, exchange word) is bounded by a clock limit; on expiry the
// kernel records an error, drains its in-flight copies and returns, and the host
// reports SQ_ERR_TIMEOUT.
#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <vector>

#include "../host/model.h"
#include "common.cuh"
#include "decode.cuh"
#include "ops.cuh"

namespace sq {
namespace dk {

#ifndef SQ_DECODE_GROUPS
#define SQ_DECODE_GROUPS 2
#endif
constexpr int NG = 4;                    // warps per group (one per SM sub-partition)
constexpr int NGRP = SQ_DECODE_GROUPS;   // groups per CTA: tile k goes to group k % NGRP
constexpr int NC = NG * NGRP;            // warps per CTA
constexpr int NTHREADS = NC * 32;
constexpr int SLOT = 36864;              // largest ring slot in bytes (the context's slot: Params::slot_bytes)
constexpr int NSLOT = 5;
constexpr int MAX_LAYERS = 128;
constexpr int MAX_TILE_ITEMS = 64;       // rows x segments per tile
constexpr int MAX_X = 8192;              // longest stage input staged in shared memory (floats)
constexpr int MAX_LM_ROWS = 896;         // LM-head rows per CTA kept in shared memory (128256 / 148 = 867)
constexpr int GROUP = 4;                 // q heads per kv head supported here
constexpr long long WAIT_LIMIT = 4000000000LL;  // ~2 s of SM clocks

// ST_DOWN2: the second input part of a down projection wider than MAX_X (Params::split)
enum { ST_QKV = 0, ST_O = 1, ST_GU = 2, ST_DOWN = 3, ST_LM = 4, ST_DOWN2 = 5 };

struct LayerW {
  const uint8_t *q, *k, *v, *o, *gate, *up, *down;
  const float *attn_norm, *ffn_norm;
};

struct Params {  // passed by value to the decode kernel: at most the 32 KB of kernel parameters
  int L, E, Q, KVd, F, V, H, KVH, hd, max_ctx, G;
  int nseg_E, nseg_Q, nseg_F;
  int rb_E, rb_Q, rb_F;        // bytes per weight row with in_dim = E / Q / F
  // FFN inputs wider than the staging buffer (F > MAX_X, e.g. 14336) are taken in two
  // parts: ST_DOWN over elements [0, xa), ST_DOWN2 over [xa, F), the same output rows;
  // part 1's sums wait in shared memory for part 2's
  int split, xa, rb_FA, rb_FB, nseg_FA, nseg_FB;
  int tile_rows[6];            // rows per tile per stage kind (gate/up: per matrix)
  int slot_bytes;              // ring slot stride (the largest tile, <= SLOT)
  int max_chunks;
  float eps, attn_scale;
  const uint8_t *embd, *out_w;
  const float *out_norm, *cos_t, *sin_t;
  float *kc, *vc, *hidden, *qbuf, *attn_out, *act, *logits, *attn_part;
  unsigned *attn_cnt, *bar, *ticket, *err;
  ArgState *arg_part;
  long long *argmax;
  int *pos;
  unsigned long long *hid_ll, *q_ll, *kv_ll, *attn_ll, *act_ll;  // tagged exchange vectors
  unsigned *launch;              // launches so far (the high bits of every tag)
#ifdef SQ_DECODE_TIMELINE
  // profiling builds only (-DSQ_DECODE_TIMELINE): per-CTA stage timestamps, and per
  // tile {issued, landed, done} clocks [G][max_tiles][3]
  unsigned long long *timeline;
  int tl_stride;
  unsigned long long *tile_tl;
#endif
  int2 *tiles;                   // [G][max_tiles] tile table: {row, layer<<16 | kind<<12 | rows}
  int *ntiles;                   // [G]
  int max_tiles;
  // Failure-detection tests only (SQ_TEST_DROP_EXCHANGE=n, read when the context is
  // created): in the context's n-th launch the producer of residual word 0 after
  // layer 0's O projection (under tensor parallelism: of this rank's partial of that
  // row) does not write it, so a bounded poll for it expires and the kernel reports
  // a timeout. 0 = off.
  unsigned drop_tag;
  // Tensor parallel (tp_world > 1): this rank's shard of the model (local heads, FFN
  // rows, vocabulary rows; full hidden size). The O and down projections leave
  // partial sums of every hidden row: a producer stores them, tagged, into row block
  // [kind][tp_rank] of every rank's exchange area (tp_box[r], peer memory mapped
  // with CUDA IPC; plain stores, no bulk or TMA access), and after the stage each
  // CTA sums its own rows over the ranks in rank order, adds the residual and
  // publishes the result locally, where the next stage's staging reads it. The
  // greedy argmax folds the ranks' states (area [2][world][E] onwards) in rank
  // order, which is vocabulary order. tp_box[] is in rank order.
  int tp_world, tp_rank, vocab_local;
  unsigned long long *tp_box[8];
  LayerW layers[MAX_LAYERS];
};
static_assert(sizeof(Params) + 64 <= 32764, "Params fits the kernel parameter space");

// ---------------------------------------------------------------------------------
// PTX helpers: mbarrier, bulk copy, shared loads, grid barrier
// ---------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *b, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned ld_volatile(const unsigned *p) {
  return *(const volatile unsigned *)p;
}
// Bounded wait on an mbarrier phase; false (and the error flag set) on timeout or
// when another CTA already failed.
__device__ __forceinline__ bool mbar_wait(uint64_t *b, unsigned parity, unsigned *err) {
  if (mbar_try_wait(b, parity)) return true;
  const long long t0 = clock64();
  for (unsigned it = 1;; it++) {
    if (mbar_try_wait(b, parity)) return true;
    if ((it & 63u) == 0) {  // the global error flag and the clock only now and then
      if (ld_volatile(err)) return false;
      if (clock64() - t0 > WAIT_LIMIT) {
        atomicExch(err, 1u);
        return false;
      }
    }
  }
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// The same copy with an L2 eviction-priority policy for the lines it reads.
__device__ __forceinline__ void bulk_g2s_hint(void *dst, const void *src, unsigned bytes, uint64_t *bar,
                                              uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void cta_sync() { asm volatile("bar.sync 1, %0;" ::"n"(NC * 32) : "memory"); }

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(unsigned *p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

#ifdef SQ_DECODE_TIMELINE
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Profiling builds only. Timeline slot k of this CTA: 0 = start; for stage s (5 per
// layer, the LM head is stage 5L) 8s+1 = input words arrived, 8s+3 = input staged in
// shared memory, 8s+2 = input in registers, 8s+4 / 8s+5 = first / last tile landed,
// 8s+6 = stage done; stride-2 = LM head done, stride-1 = end. Stamps are SM clock
// counts; each CTA also records one (global ns, clock) pair at a tick of the global
// timer at start and at end (slots stride-6..stride-3), which maps its clocks onto
// global time more finely than the timer's own resolution.
__device__ __forceinline__ void stamp(const Params &p, int k) {
  if (p.timeline && threadIdx.x == 0) p.timeline[(size_t)blockIdx.x * p.tl_stride + k] = (unsigned long long)clock64();
}
__device__ __forceinline__ void stamp_now(const Params &p, int k) {  // by whichever thread calls it
  if (p.timeline) p.timeline[(size_t)blockIdx.x * p.tl_stride + k] = (unsigned long long)clock64();
}
__device__ __forceinline__ void stamp_sync(const Params &p, int k) {
  if (p.timeline && threadIdx.x == 0) {
    const unsigned long long g0 = global_ns();
    unsigned long long g = g0;
    for (int it = 0; it < 1000000 && g == g0; it++) g = global_ns();  // the next tick
    const long long c = clock64();
    p.timeline[(size_t)blockIdx.x * p.tl_stride + k] = g;
    p.timeline[(size_t)blockIdx.x * p.tl_stride + k + 1] = (unsigned long long)c;
  }
}
__device__ __forceinline__ void stamp_tile(const Params &p, int j, int which) {
  if (p.tile_tl) p.tile_tl[((size_t)blockIdx.x * p.max_tiles + j) * 3 + which] = (unsigned long long)clock64();
}
#define TL_STRIDE(p) ((p).tl_stride)
#else
__device__ __forceinline__ void stamp(const Params &, int) {}
__device__ __forceinline__ void stamp_now(const Params &, int) {}
__device__ __forceinline__ void stamp_sync(const Params &, int) {}
__device__ __forceinline__ void stamp_tile(const Params &, int, int) {}
#define TL_STRIDE(p) 6
#endif

// ---------------------------------------------------------------------------------
// work split (the same in the tile tables and in the consumers)
// ---------------------------------------------------------------------------------
__device__ __forceinline__ void unit_range(int units, int stage, int cta, int G, int &u0, int &u1) {
  const int c = (cta + stage * 61) % G;  // rotate which CTAs get the larger shares
  u0 = (int)((long long)units * c / G);
  u1 = (int)((long long)units * (c + 1) / G);
}

// rows of stage `kind` of layer l owned by this CTA, in the stage's row space
__device__ __forceinline__ void stage_rows(const Params &p, int kind, int l, int cta, int &r0, int &r1) {
  const int stage = l * 5 + (kind == ST_DOWN2 ? ST_DOWN : kind);  // both parts: the same rows
  int u0, u1;
  switch (kind) {
    case ST_QKV:
      unit_range((p.Q + 2 * p.KVd) / 2, stage, cta, p.G, u0, u1);
      r0 = 2 * u0;
      r1 = 2 * u1;
      return;
    case ST_O: unit_range(p.E, stage, cta, p.G, r0, r1); return;
    case ST_GU: unit_range(p.F, stage, cta, p.G, r0, r1); return;
    case ST_DOWN:
    case ST_DOWN2: unit_range(p.E, stage, cta, p.G, r0, r1); return;
    default: unit_range(p.V, stage, cta, p.G, r0, r1); return;
  }
}

__device__ __forceinline__ int stage_rb(const Params &p, int kind) {
  if (kind == ST_DOWN) return p.split ? p.rb_FA : p.rb_F;
  if (kind == ST_DOWN2) return p.rb_FB;
  return kind == ST_O ? p.rb_Q : p.rb_E;
}
__device__ __forceinline__ int stage_nseg(const Params &p, int kind) {
  if (kind == ST_DOWN) return p.split ? p.nseg_FA : p.nseg_F;
  if (kind == ST_DOWN2) return p.nseg_FB;
  return kind == ST_O ? p.nseg_Q : p.nseg_E;
}
__device__ __forceinline__ int stage_in_dim(const Params &p, int kind) {
  if (kind == ST_DOWN) return p.split ? p.xa : p.F;
  if (kind == ST_DOWN2) return p.F - p.xa;
  return kind == ST_O ? p.Q : p.E;
}

// ---------------------------------------------------------------------------------
// consumers: block decode against register-resident activations
// ---------------------------------------------------------------------------------
constexpr unsigned FULL = 0xffffffffu;

struct Ring {
  uint8_t *slots;
  uint64_t *full;  // full[s]: the bytes of the tile in slot s have landed
};

// Element index of activation register i (0..63) of `lane` in segment `seg`.
// Q8_0 / Q4_0: each lane owns one pair of consecutive 32-element blocks of the
// segment (the segment = 32 pairs = 2048 elements). BF16: each lane owns 8
// consecutive elements of each 256-element stripe (16-byte shared-memory reads).
template <int T>
__device__ __forceinline__ int xelem(int seg, int lane, int i) {
  if constexpr (T == SQ_BF16) return seg * 2048 + (i >> 3) * 256 + lane * 8 + (i & 7);
  return seg * 2048 + lane * 64 + i;
}

// Whether lane's elements in segment seg exist for a row of `in_dim` elements.
template <int T>
__device__ __forceinline__ bool lane_active(int seg, int lane, int in_dim) {
  if constexpr (T == SQ_BF16) return seg * 2048 < in_dim;  // BF16 rows are whole segments (host check)
  return seg * 2048 + lane * 64 < in_dim;
}

// Load this lane's activations of segment seg from a global vector written in this
// kernel (L2 reads: other SMs wrote it).
// 16-byte global loads issued as written (volatile asm keeps them ahead of their
// uses, so a lane's whole vector is one round trip, not sixteen).
__device__ __forceinline__ float4 ldcg4(const float *p) {  // data other SMs wrote in this kernel: L2
  float4 v;
  asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ float4 ldnc4(const float *p) {  // constant data (norm weights)
  float4 v;
  asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ float sigmoid_ref(float v) {  // kernels/sigmoid.rs:2-9
  if (v >= 0.0f) return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v)));
  const float z = expf(v);
  return __fdiv_rn(z, __fadd_rn(1.0f, z));
}

// int8 / nibble -> exact float: place the byte under the exponent of 2^23 and
// subtract the bias (2^23 + 128 for sign-flipped int8, 2^23 + 8 for Q4_0's -8).
__device__ __forceinline__ float q8f(uint32_t wx, int byte) {  // wx = word ^ 0x80808080
  return __uint_as_float(__byte_perm(wx, 0x4B000000u, 0x7540u | (unsigned)byte)) - 8388736.0f;
}
__device__ __forceinline__ float nibf(uint32_t nib4, int byte) {  // nib4 = 4 nibbles in byte lanes
  return __uint_as_float(__byte_perm(nib4, 0x4B000000u, 0x7540u | (unsigned)byte)) - 8388616.0f;
}

__device__ __forceinline__ uint32_t ldnc32(const uint8_t *p) {
  uint32_t v;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

struct AttScratch {
  float m[NC][GROUP], l[NC][GROUP];
  float a[NC][GROUP][128];
};

// The stage input of a W8A8 context (SQ_ACTS_Q8): int8 activations laid out word for
// word against the weight words the integer dot products read (see stage_q), and the
// f32 value of each block's f16 scale.
struct QStage {
  uint32_t xq[MAX_X / 2048 * 18 * 32];  // Q8_0 weights: [seg][17][lane]; Q4_0: [seg][9][low / high][lane]
  float2 xsc[MAX_X / 64];               // scales of the two blocks of each lane's pair
  int2 xsum[MAX_X / 64];                // Q4_0: sums of the quants of the two blocks
};

struct Smem {
  float red[2 * NGRP][MAX_TILE_ITEMS];  // segment partial sums: two buffers per warp group
  union {
    float xs[MAX_X / 2048 * 2176];  // the stage input, lane-interleaved (see xs_index)
    QStage qs;                      // the quantized stage input (W8A8)
    AttScratch at;    // attention-stage partials (a different phase of the layer)
  };
  float ssp[NC];      // per-warp partial squared sums of the RMS norm
  float qh[128];      // one q head (head_dim <= 128)
  float lm[MAX_LM_ROWS];
  float dpart[32];    // split down projection: part 1's sums of this CTA's rows
  int rel[NSLOT];     // warps done with the tile in each slot
  int slot_tile[NSLOT];  // tile index last issued into each slot
  int pad_[3];
  int issued[NSLOT];  // copies issued into each slot (for the error-path drain)
  int ntiles;
  int flag;
};
static_assert(sizeof(Smem) % 16 == 0, "the tile table after Smem is a bulk-copy target (16-byte aligned)");

enum { XS_PLAIN = 0, XS_NORM = 1, XS_EMBED = 2 };

// ---- tagged exchange between CTAs ------------------------------------------------
// Every vector one stage hands to the next (the residual stream, q / the new K/V
// row, attention output, SiLU*up) lives in 64-bit words: the float in the low half,
// the tag of the write in the high half. A reader polls the words themselves until
// every one carries the tag it expects, so receiving the data is the
// synchronization — no grid barrier, no flag round trip. Tags are
// launch << 10 | layer << 3 | kind (kind below), so a stale word never matches.
enum { TG_EMBED = 0, TG_QKV = 1, TG_ATTN = 2, TG_POST_O = 3, TG_ACT = 4, TG_POST_DOWN = 5, TG_ARG = 6 };
__host__ __device__ __forceinline__ unsigned mk_tag(unsigned launch, int l, int kind) {
  return (launch << 10) | ((unsigned)l << 3) | (unsigned)kind;
}
__device__ __forceinline__ void st_ll(unsigned long long *a, float v, unsigned tag) {
  const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
  asm volatile("st.global.u64 [%0], %1;" ::"l"(a), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_ll(const unsigned long long *a) {
  unsigned long long v;
  asm volatile("ld.global.cg.u64 %0, [%1];" : "=l"(v) : "l"(a));
  return v;
}
// Tensor-parallel exchange words: stored by any rank (peer memory over NVLink) and
// read by the owner, so both sides use system scope.
__device__ __forceinline__ void st_ll_sys(unsigned long long *a, float v, unsigned tag) {
  const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_ll_sys(const unsigned long long *a) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
  return v;
}
__device__ __forceinline__ ulonglong2 ld_ll2(const unsigned long long *a) {  // two words, 16-byte aligned
  ulonglong2 v;
  asm volatile("ld.global.cg.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(a));
  return v;
}
__device__ __forceinline__ bool ll_ok(unsigned long long w, unsigned tag) { return (unsigned)(w >> 32) == tag; }
__device__ __forceinline__ float ll_val(unsigned long long w) { return __uint_as_float((unsigned)w); }

// A bounded poll gives up when another CTA failed or after WAIT_LIMIT clocks (then
// it sets the error flag).
__device__ __forceinline__ bool poll_expired(const Params &p, long long t0) {
  if (ld_volatile(p.err)) return true;
  if (clock64() - t0 > WAIT_LIMIT) {
    atomicExch(p.err, 3u);
    return true;
  }
  return false;
}

// Re-read one word until it carries `tag` (bounded: on expiry the error flag is set
// and 0 returned).
__device__ __noinline__ unsigned long long ll_wait(const Params &p, const unsigned long long *a, unsigned tag) {
  const long long t0 = clock64();
  for (unsigned it = 0;; it++) {
    const unsigned long long w = ld_ll(a);
    if (ll_ok(w, tag)) return w;
    if ((it & 63u) == 63u) {
      if (ld_volatile(p.err)) return 0ull;
      if (clock64() - t0 > WAIT_LIMIT) {
        atomicExch(p.err, 3u);
        return 0ull;
      }
    }
  }
}
__device__ __forceinline__ float poll_ll(const Params &p, const unsigned long long *a, unsigned tag) {
  unsigned long long w = ld_ll(a);
  if (!ll_ok(w, tag)) w = ll_wait(p, a, tag);
  return ll_val(w);
}
// N words at once: every stale word is re-read in the same pass, so a retry costs
// one L2 round trip however many words are still missing.
template <int N, bool SYS = false>
__device__ __forceinline__ void poll_ll_n(const Params &p, const unsigned long long *const (&a)[N], unsigned tag,
                                          float (&out)[N]) {
  unsigned long long w[N];
#pragma unroll
  for (int i = 0; i < N; i++) w[i] = SYS ? ld_ll_sys(a[i]) : ld_ll(a[i]);
  const long long t0 = clock64();
  for (unsigned it = 0;; it++) {
    bool all = true;
#pragma unroll
    for (int i = 0; i < N; i++) all = all && ll_ok(w[i], tag);
    if (all) break;
#pragma unroll
    for (int i = 0; i < N; i++)
      if (!ll_ok(w[i], tag)) w[i] = SYS ? ld_ll_sys(a[i]) : ld_ll(a[i]);
    if ((it & 15u) == 15u && poll_expired(p, t0)) break;
  }
#pragma unroll
  for (int i = 0; i < N; i++) out[i] = ll_val(w[i]);
}

// ---- stage inputs: one cooperative load per CTA into shared memory -------------
// Every CTA needs the whole input vector of a stage (all elements of the residual
// for a norm, all of attn / act). Reading it once per CTA — not once per warp —
// keeps the CTAs' simultaneous reads of the same few KB from piling up on a
// handful of L2 slices. The layout is the one the dot products read, with
// conflict-free 16-byte loads that the four rows of a step share (lane `lane` of a
// warp on segment `seg`, its 64 elements i of the segment's 2048):
//  Q8_0: [seg][k 0..16][lane] float4: step k of quad_dot_xs (word k of the lane's
//        68-byte block pair) takes slot k; the lane's element i sits at position
//        i + 2 (i < 32) or i + 4 of its 68 floats, so the two scales' positions are
//        padding. (Sharing one slot between steps 0 and 8, as Q4_0 does, measured
//        4 % slower on Q8_0: the staging index arithmetic sits on every stage's
//        critical path.)
//  Q4_0: [seg][slot 0..7][low / high][lane] float4: word k of the 36-byte pair
//        holds bytes whose low nibbles are elements j and high nibbles j + 16, so a
//        step loads both halves of slot k (k 1..3), k - 1 (k 5..8), or slot 0
//        (bytes 14, 15, 0, 1 of block 0), shared by steps 0 and 4;
//  BF16: [seg][i / 4][lane] float4 for the lane's element i = 8k .. 8k+7 of step k.
// Element pairs (2j, 2j + 1) are adjacent in every layout.
template <int T>
__device__ __forceinline__ int xs_index(int e) {
  const int seg = e >> 11, r = e & 2047;
  if constexpr (T == SQ_Q8_0) {
    const int ln = r >> 6, i = r & 63, pos = i < 32 ? i + 2 : i + 4;
    return ((seg * 17 + (pos >> 2)) * 32 + ln) * 4 + (pos & 3);
  }
  if constexpr (T == SQ_Q4_0) {
    const int ln = r >> 6, i = r & 63, j = i & 31, byte = j & 15, half = j >> 4;
    int slot, c;
    if (i >= 32) {
      slot = 4 + (byte >> 2);
      c = byte & 3;
    } else if (byte < 2 || byte >= 14) {
      slot = 0;
      c = byte < 2 ? byte + 2 : byte - 14;
    } else {
      slot = (byte + 2) >> 2;
      c = (byte + 2) & 3;
    }
    return (((seg * 8 + slot) * 2 + half) * 32 + ln) * 4 + c;
  }
  int lane, i;
  if constexpr (T == SQ_BF16) {
    lane = (r & 255) >> 3;
    i = ((r >> 8) << 3) | (r & 7);
  } else {
    lane = r >> 6;
    i = r & 63;
  }
  return (seg << 11) + ((i >> 2) << 7) + (lane << 2) + (i & 3);
}

// Stage the n-element input of a stage into sm.xs. XS_PLAIN copies the tagged
// vector v; XS_NORM stages h*w for the RMS norm of h (rms_norm.rs:40-56) and
// returns 1/rms; XS_EMBED dequantizes the embedding row (ops/embedding.rs:10-52,
// exact scale*q) as h — optionally publishing it as the layer-0 residual — and
// normalizes it like XS_NORM. The squared sum is combined in a fixed order, so
// every CTA computes the same rms.
template <int T, int MODE>
__device__ float stage_x(const Params &p, Smem &sm, const unsigned long long *v, unsigned tag, const float *w, int n,
                         const uint8_t *emb_row, bool write_hidden, unsigned emb_tag, int stamp_at) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float ss = 0.f;
  if constexpr (MODE == XS_EMBED) {
    for (int g0 = 0; g0 < n / 8; g0 += NC * 32) {  // 8 elements (a quarter block) per thread per pass
      const int g = g0 + tid;
      if (g < n / 8) {
        const int e = g * 8, b = e >> 5, j0 = e & 31;
        float d[8];
        if constexpr (T == SQ_BF16) {
          const uint8_t *a = emb_row + (size_t)b * 64 + j0 * 2;
          const uint32_t u[4] = {ldnc32(a), ldnc32(a + 4), ldnc32(a + 8), ldnc32(a + 12)};
#pragma unroll
          for (int k = 0; k < 4; k++) {
            d[2 * k] = __uint_as_float(u[k] << 16);
            d[2 * k + 1] = __uint_as_float(u[k] & 0xFFFF0000u);
          }
        } else if constexpr (T == SQ_Q8_0) {
          const uint8_t *blk = emb_row + (size_t)b * Q8_BYTES;
          const float sc = h2f(ld_u16(blk));
#pragma unroll
          for (int k = 0; k < 8; k++) d[k] = sc * (float)(int8_t)__ldg(blk + 2 + j0 + k);
        } else {
          const uint8_t *blk = emb_row + (size_t)b * Q4_BYTES;
          const float sc = h2f(ld_u16(blk));
#pragma unroll
          for (int k = 0; k < 8; k++) {
            const uint8_t byte = __ldg(blk + 2 + ((j0 + k) & 15));
            d[k] = sc * (float)((j0 < 16 ? (byte & 0x0F) : (byte >> 4)) - 8);
          }
        }
        const float4 w0 = ldnc4(w + e), w1 = ldnc4(w + e + 4);
        if (write_hidden) {
#pragma unroll
          for (int k = 0; k < 8; k++) st_ll(p.hid_ll + e + k, d[k], emb_tag);
        }
#pragma unroll
        for (int k = 0; k < 8; k++) ss = fmaf(d[k], d[k], ss);
        if constexpr (T != SQ_BF16) {  // element pairs are adjacent in these layouts, quads are not
          const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
          for (int k = 0; k < 8; k += 2)
            *reinterpret_cast<float2 *>(&sm.xs[xs_index<T>(e + k)]) =
                make_float2(__fmul_rn(d[k], ww[k]), __fmul_rn(d[k + 1], ww[k + 1]));
        } else {
          *reinterpret_cast<float4 *>(&sm.xs[xs_index<T>(e)]) =
              make_float4(__fmul_rn(d[0], w0.x), __fmul_rn(d[1], w0.y), __fmul_rn(d[2], w0.z), __fmul_rn(d[3], w0.w));
          *reinterpret_cast<float4 *>(&sm.xs[xs_index<T>(e + 4)]) =
              make_float4(__fmul_rn(d[4], w1.x), __fmul_rn(d[5], w1.y), __fmul_rn(d[6], w1.z), __fmul_rn(d[7], w1.w));
        }
      }
    }
  } else {
    // word pairs (two elements), every load of this thread in flight before any use
    constexpr int MAXC = (MAX_X / 2 + NC * 32 - 1) / (NC * 32);
    ulonglong2 c[MAXC];
    float2 wv[MAXC];
    const int nc = n / 2;
#pragma unroll
    for (int k = 0; k < MAXC; k++) {
      const int ci = k * NC * 32 + tid;
      c[k] = ci < nc ? ld_ll2(v + 2 * ci) : make_ulonglong2(0ull, 0ull);
      if (MODE == XS_NORM) wv[k] = ci < nc ? *reinterpret_cast<const float2 *>(w + 2 * ci) : make_float2(0.f, 0.f);
    }
    const long long t0 = clock64();
    for (unsigned it = 0;; it++) {  // re-read all stale pairs together
      bool all = true;
#pragma unroll
      for (int k = 0; k < MAXC; k++)
        if (k * NC * 32 + tid < nc && !(ll_ok(c[k].x, tag) && ll_ok(c[k].y, tag))) all = false;
      if (all) break;
#pragma unroll
      for (int k = 0; k < MAXC; k++) {
        const int ci = k * NC * 32 + tid;
        if (ci < nc && !(ll_ok(c[k].x, tag) && ll_ok(c[k].y, tag))) c[k] = ld_ll2(v + 2 * ci);
      }
      if ((it & 15u) == 15u && poll_expired(p, t0)) break;
    }
    if (stamp_at >= 0) stamp(p, stamp_at);
#pragma unroll
    for (int k = 0; k < MAXC; k++) {
      const int ci = k * NC * 32 + tid;
      if (ci < nc) {
        float a = ll_val(c[k].x), b = ll_val(c[k].y);
        if (MODE == XS_NORM) {
          ss = fmaf(a, a, ss);
          ss = fmaf(b, b, ss);
          a = __fmul_rn(a, wv[k].x);
          b = __fmul_rn(b, wv[k].y);
        }
        *reinterpret_cast<float2 *>(&sm.xs[xs_index<T>(2 * ci)]) = make_float2(a, b);
      }
    }
  }
  if (MODE != XS_PLAIN) {
    ss = warp_sum(ss);
    if (lane == 0) sm.ssp[warp] = ss;
  }
  cta_sync();
  if (stamp_at >= 0) stamp(p, stamp_at + 2);
  if (MODE == XS_PLAIN) return 1.0f;
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < NC; k++) tot += sm.ssp[k];
  return 1.0f / __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)n), p.eps));
}

// Byte offset in QStage::xq of activation element j (0..31) of block h (0, 1) of a
// lane's block pair, for the weight type the dots read. Q8_0: the pair is 17 words
// (scale, 32 quants, scale, 32 quants), so element j of block h lines up with byte
// 2 + 34h + j of the weight words. Q4_0: 9 words (scale, 16 bytes, scale, 16 bytes);
// byte 2 + 18h + (j & 15) holds element j in its low nibble (j < 16) or high nibble,
// so the low and high elements go to two word planes. Positions under a scale stay 0.
template <int T>
__device__ __forceinline__ uint32_t xq_byte(int seg, int lane, int h, int j) {
  if constexpr (T == SQ_Q8_0) {
    const int pos = 2 + 34 * h + j;
    return (uint32_t)(((seg * 17 + (pos >> 2)) * 32 + lane) * 4 + (pos & 3));
  } else {
    const int pos = 2 + 18 * h + (j & 15);
    return (uint32_t)((((seg * 9 + (pos >> 2)) * 2 + (j >> 4)) * 32 + lane) * 4 + (pos & 3));
  }
}

__device__ __forceinline__ void sts16(uint32_t a, uint32_t v) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(a), "h"((unsigned short)v) : "memory");
}

// W8A8 (SQ_ACTS_Q8): the stage's n-element input quantized to Q8_0 blocks
// (quantize_row_q8_0, dot_prod.rs:21-31) into sm.qs, after the RMS norm for XS_NORM /
// XS_EMBED in the reference's form y = (h*w) / rms (rms_norm.rs:40-56; the squared
// sum in a fixed order of our own). Every linear quantizes its input this way
// (matmul.rs:89-100). Thread t takes eight consecutive elements (a quarter block) per
// pass; the four threads of a block meet through shuffles for its absolute maximum
// and (Q4_0) the sum of its quants. Returns 1: the norm is applied before quantizing.
template <int T, int MODE>
__device__ float stage_q(const Params &p, Smem &sm, const unsigned long long *v, unsigned tag, const float *w, int n,
                         const uint8_t *emb_row, bool write_hidden, unsigned emb_tag, int stamp_at) {
  constexpr int MAXG = MAX_X / 8 / NTHREADS;  // passes of eight elements a thread
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ng = n / 8;  // n is a multiple of 256 (host check): whole warps take part in a pass
  float x[MAXG][8];
  float ss = 0.f;

  if constexpr (MODE == XS_EMBED) {
#pragma unroll
    for (int k = 0; k < MAXG; k++) {
      const int g = k * NTHREADS + tid;
      if (g < ng) {
        const int e = g * 8, b = e >> 5, j0 = e & 31;
        const uint8_t *blk = emb_row + (size_t)b * (T == SQ_Q8_0 ? Q8_BYTES : Q4_BYTES);
        const float sc = h2f(ld_u16(blk));
#pragma unroll
        for (int i = 0; i < 8; i++) {
          if constexpr (T == SQ_Q8_0) {
            x[k][i] = sc * (float)(int8_t)__ldg(blk + 2 + j0 + i);
          } else {
            const uint8_t byte = __ldg(blk + 2 + ((j0 + i) & 15));
            x[k][i] = sc * (float)((j0 < 16 ? (byte & 0x0F) : (byte >> 4)) - 8);
          }
        }
        if (write_hidden) {
#pragma unroll
          for (int i = 0; i < 8; i++) st_ll(p.hid_ll + e + i, x[k][i], emb_tag);
        }
      }
    }
  } else {
    ulonglong2 c[MAXG][4];
#pragma unroll
    for (int k = 0; k < MAXG; k++) {
      const int g = k * NTHREADS + tid;
#pragma unroll
      for (int i = 0; i < 4; i++) c[k][i] = g < ng ? ld_ll2(v + 8 * g + 2 * i) : make_ulonglong2(0ull, 0ull);
    }
    const long long t0 = clock64();
    for (unsigned it = 0;; it++) {  // re-read all stale pairs together
      bool all = true;
#pragma unroll
      for (int k = 0; k < MAXG; k++)
#pragma unroll
        for (int i = 0; i < 4; i++)
          if (k * NTHREADS + tid < ng && !(ll_ok(c[k][i].x, tag) && ll_ok(c[k][i].y, tag))) all = false;
      if (all) break;
#pragma unroll
      for (int k = 0; k < MAXG; k++) {
        const int g = k * NTHREADS + tid;
#pragma unroll
        for (int i = 0; i < 4; i++)
          if (g < ng && !(ll_ok(c[k][i].x, tag) && ll_ok(c[k][i].y, tag))) c[k][i] = ld_ll2(v + 8 * g + 2 * i);
      }
      if ((it & 15u) == 15u && poll_expired(p, t0)) break;
    }
#pragma unroll
    for (int k = 0; k < MAXG; k++)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        x[k][2 * i] = ll_val(c[k][i].x);
        x[k][2 * i + 1] = ll_val(c[k][i].y);
      }
  }
  if (stamp_at >= 0) stamp(p, stamp_at);
  float rms = 1.0f;
  if constexpr (MODE != XS_PLAIN) {
#pragma unroll
    for (int k = 0; k < MAXG; k++)
      if (k * NTHREADS + tid < ng) {
#pragma unroll
        for (int i = 0; i < 8; i++) ss = fmaf(x[k][i], x[k][i], ss);
      }
    ss = warp_sum(ss);
    if (lane == 0) sm.ssp[warp] = ss;
    cta_sync();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < NC; k++) tot += sm.ssp[k];
    rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)n), p.eps));
  }
  const uint32_t xq = smem_u32(sm.qs.xq);
  float *xsc = reinterpret_cast<float *>(sm.qs.xsc);
  int *xsum = reinterpret_cast<int *>(sm.qs.xsum);
#pragma unroll
  for (int k = 0; k < MAXG; k++) {
    const int g = k * NTHREADS + tid;
    if (g >= ng) continue;  // warp-uniform (ng is a multiple of 32), so the shuffles below see whole warps
    float y[8];
    if constexpr (MODE != XS_PLAIN) {
      const float4 w0 = ldnc4(w + 8 * g), w1 = ldnc4(w + 8 * g + 4);
      const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int i = 0; i < 8; i++) y[i] = __fdiv_rn(__fmul_rn(x[k][i], ww[i]), rms);
    } else {
#pragma unroll
      for (int i = 0; i < 8; i++) y[i] = x[k][i];
    }
    float am = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) am = fmaxf(am, fabsf(y[i]));
    am = fmaxf(am, __shfl_xor_sync(FULL, am, 1));
    am = fmaxf(am, __shfl_xor_sync(FULL, am, 2));
    const float scale = __fdiv_rn(am, 127.0f);
    const float inv = scale > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
    int q[8], qs = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const float r = roundf(__fmul_rn(y[i], inv));  // ties away from zero, like f32::round
      q[i] = (r != r) ? 0 : (int)fminf(fmaxf(r, -127.0f), 127.0f);
      qs += q[i];
    }
    const int b = g >> 2, qq = g & 3;  // block of the stage input, quarter of the block
    const int seg = b >> 6, ln = (b >> 1) & 31, h = b & 1;
#pragma unroll
    for (int i = 0; i < 8; i += 2)
      sts16(xq + xq_byte<T>(seg, ln, h, 8 * qq + i), (uint32_t)(q[i] & 0xFF) | ((uint32_t)(q[i + 1] & 0xFF) << 8));
    if constexpr (T == SQ_Q8_0) {
      if (qq == 0) sts16(xq + xq_byte<T>(seg, ln, h, -2), 0u);  // under the block's scale
    } else {
      if ((qq & 1) == 0) {  // this plane (low for qq 0, high for qq 2) under the block's scale (byte 18h)
        const int pos = 18 * h;
        sts16(xq + (uint32_t)((((seg * 9 + (pos >> 2)) * 2 + (qq >> 1)) * 32 + ln) * 4 + (pos & 3)), 0u);
      }
      qs += __shfl_xor_sync(FULL, qs, 1);
      qs += __shfl_xor_sync(FULL, qs, 2);
      if (qq == 0) xsum[b] = qs;
    }
    if (qq == 0) xsc[b] = __half2float(__float2half_rn(scale));
  }
  cta_sync();
  if (stamp_at >= 0) stamp(p, stamp_at + 2);
  return 1.0f;
}

// Stage a stage's input into the staging buffer, where the dot products read it.
// Returns the factor the stage's dot products take: the norm's 1/rms (1 for a plain
// input), applied to each row's sum (the reference scales the input, (h*w)/rms:
// one rounding apart). W8A8 contexts (AQ) stage the quantized input instead.
template <int T, int MODE, bool AQ>
__device__ __forceinline__ float stage_in(const Params &p, Smem &sm, const unsigned long long *v, unsigned tag,
                                         const float *w, int n, int stamp_at, const uint8_t *emb_row = nullptr,
                                         bool write_hidden = false, unsigned emb_tag = 0u) {
  if constexpr (AQ) return stage_q<T, MODE>(p, sm, v, tag, w, n, emb_row, write_hidden, emb_tag, stamp_at);
  else return stage_x<T, MODE>(p, sm, v, tag, w, n, emb_row, write_hidden, emb_tag, stamp_at);
}

// Q4_0 step k of a lane's block pair: the staging slot holding its inputs.
__host__ __device__ constexpr int xs_slot_q4(int k) { return k == 0 || k == 4 ? 0 : (k < 4 ? k : k - 1); }

// Four weight rows at a time: the lane's partial dot products of rows at shared
// addresses ra[0..3] with its 64 inputs in the staging buffer (xs, layout at
// xs_index). Q8_0 / Q4_0 one 68 / 36-byte block pair of segment `seg` (4-byte words
// at an odd word stride between lanes: conflict-free), BF16 eight 16-byte chunks.
// The loop runs word by word with the four rows innermost: each step loads its
// inputs once (one or two 16-byte loads the four rows share) and has four
// independent load -> convert -> FMA chains. int8 / nibble -> f32 by byte permute
// into a float magic constant, packed f32x2 adds and FMAs. Per block the products
// are summed first and scaled once, as the reference does (dot_prod.rs:86-96,
// 255-270; BF16 one running sum, :464-472). Keeping the inputs here instead of in 64
// registers a lane measured 5 % (1B) and 11 % (8B) faster on Q8_0.
template <int T>
__device__ __forceinline__ void quad_dot_xs(const uint32_t (&ra)[4], int seg, int lane, uint32_t xs, float (&out)[4]) {
  if constexpr (T == SQ_Q8_0) {
    const uint32_t off = (uint32_t)(seg * 32 + lane) * 68u;
    const uint32_t xa = xs + (uint32_t)((seg * 17 * 32 + lane) * 16);
    const f2x bias = pk2(-8388736.0f, -8388736.0f);  // 2^23 + 128: sign-flipped int8 under 2^23
    f2x A[4], B[4];
    float s0[4], s1[4];
#pragma unroll
    for (int r = 0; r < 4; r++) A[r] = B[r] = 0ull;
#pragma unroll
    for (int k = 0; k < 17; k++) {
      uint32_t w[4];
#pragma unroll
      for (int r = 0; r < 4; r++) w[r] = lds32(ra[r] + off + 4u * k);
      const uint4 xv = lds128(xa + (uint32_t)k * 512u);  // elements 4k-2 .. 4k+1 (block 0) / 4k-4 .. 4k-1
      const f2x xlo = pk2u(xv.x, xv.y), xhi = pk2u(xv.z, xv.w);
#pragma unroll
      for (int r = 0; r < 4; r++) {
        const uint32_t wx = w[r] ^ 0x80808080u;
        const f2x lo = fadd2(pk2u(__byte_perm(wx, 0x4B000000u, 0x7540u), __byte_perm(wx, 0x4B000000u, 0x7541u)), bias);
        const f2x hi = fadd2(pk2u(__byte_perm(wx, 0x4B000000u, 0x7542u), __byte_perm(wx, 0x4B000000u, 0x7543u)), bias);
        if (k == 0) {  // scale of block 0, quants 0, 1
          s0[r] = h2f((uint16_t)(w[r] & 0xFFFFu));
          A[r] = ffma2(xhi, hi, A[r]);
        } else if (k < 8) {  // quants 4k-2 .. 4k+1 of block 0
          A[r] = ffma2(xlo, lo, A[r]);
          A[r] = ffma2(xhi, hi, A[r]);
        } else if (k == 8) {  // quants 30, 31 of block 0, scale of block 1
          A[r] = ffma2(xlo, lo, A[r]);
          s1[r] = h2f((uint16_t)(w[r] >> 16));
        } else {  // quants 4k-36 .. 4k-33 of block 1
          B[r] = ffma2(xlo, lo, B[r]);
          B[r] = ffma2(xhi, hi, B[r]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const float2 a = up2(A[r]), b = up2(B[r]);
      out[r] = fmaf(a.x + a.y, s0[r], (b.x + b.y) * s1[r]);
    }
  } else if constexpr (T == SQ_Q4_0) {
    const uint32_t off = (uint32_t)(seg * 32 + lane) * 36u;
    const uint32_t xa = xs + (uint32_t)((seg * 16 * 32 + lane) * 16);  // [slot][half][lane] float4
    const f2x bias = pk2(-8388616.0f, -8388616.0f);  // 2^23 + 8: nibble q under 2^23, value q - 8
    f2x A[4], B[4];
    float s0[4], s1[4];
#pragma unroll
    for (int r = 0; r < 4; r++) A[r] = B[r] = 0ull;
#pragma unroll
    for (int k = 0; k < 9; k++) {
      uint32_t w[4];
#pragma unroll
      for (int r = 0; r < 4; r++) w[r] = lds32(ra[r] + off + 4u * k);
      const uint32_t sa = xa + (uint32_t)xs_slot_q4(k) * 1024u;
      const uint4 xl = lds128(sa), xh = lds128(sa + 512u);  // low-nibble and high-nibble elements
      const f2x l01x = pk2u(xl.x, xl.y), l23x = pk2u(xl.z, xl.w), h01x = pk2u(xh.x, xh.y), h23x = pk2u(xh.z, xh.w);
#pragma unroll
      for (int r = 0; r < 4; r++) {
        const uint32_t nl = w[r] & 0x0F0F0F0Fu, nh = (w[r] >> 4) & 0x0F0F0F0Fu;
        const f2x l01 = fadd2(pk2u(__byte_perm(nl, 0x4B000000u, 0x7540u), __byte_perm(nl, 0x4B000000u, 0x7541u)), bias);
        const f2x l23 = fadd2(pk2u(__byte_perm(nl, 0x4B000000u, 0x7542u), __byte_perm(nl, 0x4B000000u, 0x7543u)), bias);
        const f2x h01 = fadd2(pk2u(__byte_perm(nh, 0x4B000000u, 0x7540u), __byte_perm(nh, 0x4B000000u, 0x7541u)), bias);
        const f2x h23 = fadd2(pk2u(__byte_perm(nh, 0x4B000000u, 0x7542u), __byte_perm(nh, 0x4B000000u, 0x7543u)), bias);
        if (k == 0) {  // scale of block 0, its bytes 0, 1 (slot 0's upper halves)
          s0[r] = h2f((uint16_t)(w[r] & 0xFFFFu));
          A[r] = ffma2(l23x, l23, A[r]);
          A[r] = ffma2(h23x, h23, A[r]);
        } else if (k < 4) {  // bytes 4k-2 .. 4k+1 of block 0
          A[r] = ffma2(l01x, l01, A[r]);
          A[r] = ffma2(l23x, l23, A[r]);
          A[r] = ffma2(h01x, h01, A[r]);
          A[r] = ffma2(h23x, h23, A[r]);
        } else if (k == 4) {  // bytes 14, 15 of block 0 (slot 0's lower halves), scale of block 1
          A[r] = ffma2(l01x, l01, A[r]);
          A[r] = ffma2(h01x, h01, A[r]);
          s1[r] = h2f((uint16_t)(w[r] >> 16));
        } else {  // bytes 4k-20 .. 4k-17 of block 1
          B[r] = ffma2(l01x, l01, B[r]);
          B[r] = ffma2(l23x, l23, B[r]);
          B[r] = ffma2(h01x, h01, B[r]);
          B[r] = ffma2(h23x, h23, B[r]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const float2 a = up2(A[r]), b = up2(B[r]);
      out[r] = fmaf(a.x + a.y, s0[r], (b.x + b.y) * s1[r]);
    }
  } else {
    const uint32_t xa = xs + (uint32_t)(seg * 2048 + lane * 4) * 4u;
    f2x A[4];
#pragma unroll
    for (int r = 0; r < 4; r++) A[r] = 0ull;
#pragma unroll
    for (int k = 0; k < 8; k++) {
      uint4 u[4];
#pragma unroll
      for (int r = 0; r < 4; r++) u[r] = lds128(ra[r] + (uint32_t)(seg * 2048 + k * 256 + lane * 8) * 2u);
      const uint4 xa4 = lds128(xa + (uint32_t)(2 * k) * 512u), xb4 = lds128(xa + (uint32_t)(2 * k + 1) * 512u);
      const f2x x0 = pk2u(xa4.x, xa4.y), x1 = pk2u(xa4.z, xa4.w), x2 = pk2u(xb4.x, xb4.y), x3 = pk2u(xb4.z, xb4.w);
#pragma unroll
      for (int r = 0; r < 4; r++) {
        A[r] = ffma2(x0, pk2u(u[r].x << 16, u[r].x & 0xFFFF0000u), A[r]);
        A[r] = ffma2(x1, pk2u(u[r].y << 16, u[r].y & 0xFFFF0000u), A[r]);
        A[r] = ffma2(x2, pk2u(u[r].z << 16, u[r].z & 0xFFFF0000u), A[r]);
        A[r] = ffma2(x3, pk2u(u[r].w << 16, u[r].w & 0xFFFF0000u), A[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const float2 a = up2(A[r]);
      out[r] = a.x + a.y;
    }
  }
}

__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {  // signed bytes x signed bytes
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {  // unsigned bytes x signed bytes
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// W8A8 block dots, four weight rows at a time: the lane's block pair of segment seg
// of rows ra[0..3] against the quantized input in sm.qs (stage_q). Each weight word
// meets the activation word built against it (zeros under the scales), so a step is
// one dp4a a row (Q8_0) or two on the word's low and high nibbles (Q4_0, quants
// q in 0..15: the block's sum is fixed up by -8 x the sum of the activation quants).
// Per block the integer sum is scaled as the reference does, (isum * d_a) * d_w
// (dot_q8_0_q8_0_scalar / dot_q8_0_q4_0_scalar, dot_prod.rs:378-403).
template <int T>
__device__ __forceinline__ void quad_dot_q(const uint32_t (&ra)[4], int seg, int lane, const QStage &qs,
                                           float (&out)[4]) {
  const uint32_t xq = smem_u32(qs.xq);
  int i0[4] = {0, 0, 0, 0}, i1[4] = {0, 0, 0, 0};
  float s0[4], s1[4];
  if constexpr (T == SQ_Q8_0) {
    const uint32_t off = (uint32_t)(seg * 32 + lane) * 68u;
    const uint32_t xa = xq + (uint32_t)((seg * 17 * 32 + lane) * 4);
#pragma unroll
    for (int k = 0; k < 17; k++) {
      uint32_t w[4];
#pragma unroll
      for (int r = 0; r < 4; r++) w[r] = lds32(ra[r] + off + 4u * k);
      const uint32_t a = lds32(xa + (uint32_t)k * 128u);
#pragma unroll
      for (int r = 0; r < 4; r++) {
        if (k <= 8) i0[r] = dp4a_ss(w[r], a, i0[r]);  // word 8: block 0's last two quants, block 1's scale
        else i1[r] = dp4a_ss(w[r], a, i1[r]);
        if (k == 0) s0[r] = h2f((uint16_t)(w[r] & 0xFFFFu));
        if (k == 8) s1[r] = h2f((uint16_t)(w[r] >> 16));
      }
    }
  } else {
    const uint32_t off = (uint32_t)(seg * 32 + lane) * 36u;
    const uint32_t xa = xq + (uint32_t)((seg * 9 * 2 * 32 + lane) * 4);
#pragma unroll
    for (int k = 0; k < 9; k++) {
      uint32_t w[4];
#pragma unroll
      for (int r = 0; r < 4; r++) w[r] = lds32(ra[r] + off + 4u * k);
      const uint32_t alo = lds32(xa + (uint32_t)(2 * k) * 128u), ahi = lds32(xa + (uint32_t)(2 * k + 1) * 128u);
#pragma unroll
      for (int r = 0; r < 4; r++) {
        const uint32_t lo = w[r] & 0x0F0F0F0Fu, hi = (w[r] >> 4) & 0x0F0F0F0Fu;
        if (k <= 4) {  // word 4: block 0's bytes 14, 15 and block 1's scale
          i0[r] = dp4a_us(lo, alo, i0[r]);
          i0[r] = dp4a_us(hi, ahi, i0[r]);
        } else {
          i1[r] = dp4a_us(lo, alo, i1[r]);
          i1[r] = dp4a_us(hi, ahi, i1[r]);
        }
        if (k == 0) s0[r] = h2f((uint16_t)(w[r] & 0xFFFFu));
        if (k == 4) s1[r] = h2f((uint16_t)(w[r] >> 16));
      }
    }
    const int2 qsum = qs.xsum[seg * 32 + lane];
#pragma unroll
    for (int r = 0; r < 4; r++) {
      i0[r] -= 8 * qsum.x;
      i1[r] -= 8 * qsum.y;
    }
  }
  const float2 da = qs.xsc[seg * 32 + lane];
#pragma unroll
  for (int r = 0; r < 4; r++)
    out[r] = __fadd_rn(__fmul_rn(__fmul_rn((float)i0[r], da.x), s0[r]), __fmul_rn(__fmul_rn((float)i1[r], da.y), s1[r]));
}

// The bulk copies of tile entry d: f(byte offset in the slot, global source, bytes).
// Rows of a QKV tile may span Wq / Wk / Wv; a gate/up tile carries its gate rows,
// then the same rows of Wup. Returns the tile's total bytes.
template <class F>
__device__ __forceinline__ unsigned tile_copies(const Params &p, int2 d, F &&f) {
  const int r = d.x, n = d.y & 0xFFF, kind = (d.y >> 12) & 0xF, l = d.y >> 16;
  const int rb = stage_rb(p, kind);
  const LayerW &W = p.layers[l < p.L ? l : 0];
  if (kind == ST_GU) {
    f(0u, W.gate + (size_t)r * rb, (unsigned)(n * rb));
    f((unsigned)(n * rb), W.up + (size_t)r * rb, (unsigned)(n * rb));
    return 2u * n * rb;
  }
  if (kind == ST_QKV) {
    int a = r, off = 0;
    const int bounds[3] = {p.Q, p.Q + p.KVd, p.Q + 2 * p.KVd};
    const uint8_t *base[3] = {W.q, W.k, W.v};
    const int start[3] = {0, p.Q, p.Q + p.KVd};
#pragma unroll
    for (int t = 0; t < 3; t++) {
      const int hi = min(r + n, bounds[t]);
      if (a < hi) {
        f((unsigned)(off * rb), base[t] + (size_t)(a - start[t]) * rb, (unsigned)((hi - a) * rb));
        off += hi - a;
        a = hi;
      }
    }
    return (unsigned)(n * rb);
  }
  if ((kind == ST_DOWN && p.split) || kind == ST_DOWN2) {  // one input part of each row: a copy per row
    const size_t off = kind == ST_DOWN2 ? (size_t)p.rb_FA : 0;
    for (int i = 0; i < n; i++) f((unsigned)(i * rb), W.down + (size_t)(r + i) * p.rb_F + off, (unsigned)rb);
    return (unsigned)(n * rb);
  }
  const uint8_t *src = kind == ST_O ? W.o : (kind == ST_DOWN ? W.down : p.out_w);
  f(0u, src + (size_t)r * rb, (unsigned)(n * rb));
  return (unsigned)(n * rb);
}

// Issue tile j of this CTA's table into `slot`: bulk copies completing on full[slot].
// The weights are read once per token, so the copies mark their L2 lines
// evict-first.
__device__ void issue_tile(const Params &p, const Ring &rg, Smem &sm, const int2 *tbl, int j, int slot) {
  const int2 d = tbl[j];
  stamp_tile(p, j, 0);
  uint8_t *dst = rg.slots + (size_t)slot * p.slot_bytes;
  uint64_t *bar = &rg.full[slot];
  sm.issued[slot]++;
  *(volatile int *)&sm.slot_tile[slot] = j;
  const int n = d.y & 0xFFF, kind = (d.y >> 12) & 0xF;
  mbar_expect_tx(bar, (kind == ST_GU ? 2u : 1u) * n * stage_rb(p, kind));
  const uint64_t pol = policy_evict_first();
  tile_copies(p, d, [&](unsigned off, const uint8_t *src, unsigned bytes) { bulk_g2s_hint(dst + off, src, bytes, bar, pol); });
}

// A warp is done reading tile `k` in `slot`; the last of the `nwarps` warps that
// read it refills the slot with tile k + NSLOT. It refills only when its own wait on
// the slot succeeded (`landed`): after a failed wait the slot's copy may still be in
// flight, and a second copy into the same barrier phase would leave the exit drain
// waiting on the wrong phase. A slot left empty makes the next wait on it give up.
__device__ __forceinline__ void release_slot(const Params &p, const Ring &rg, Smem &sm, const int2 *tbl, int slot,
                                             int k, int nwarps, bool landed) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) {
    if (atomicAdd(&sm.rel[slot], 1) == nwarps - 1) {
      sm.rel[slot] = 0;
      if (landed && k + NSLOT < sm.ntiles) issue_tile(p, rg, sm, tbl, k + NSLOT, slot);
    }
  }
}

// Per-stage values each warp holds in registers: RoPE cos/sin of the token's
// position for frequency index lane and lane+32, and hidden[r0 + lane] (the
// residual of this CTA's rows of the O / down stages).
struct StageRegs {
  float c0, c1, s0, s1, hres;
};

// Finish output row(s) of a stage (warp-uniform arguments; lane 0 stores).
// rows a / b are absolute rows of the stage's row space; vb is ignored when !hasb.
// Outputs other CTAs read go out as tagged words (`tag`); the K/V row also lands
// in the cache for later tokens.
__device__ __forceinline__ void finish_rows(const Params &p, Smem &sm, int kind, int l, int pos, int r0, int a,
                                            float va, int b, float vb, bool hasb, const StageRegs &sr, unsigned tag) {
  const int lane = threadIdx.x & 31;
  if (kind == ST_QKV) {  // a even, b = a + 1: RoPE pair (rope.rs:25-31), then q / K / V
    const int j = (a % p.hd) >> 1;
    const float c = __shfl_sync(FULL, j < 32 ? sr.c0 : sr.c1, j & 31);
    const float s = __shfl_sync(FULL, j < 32 ? sr.s0 : sr.s1, j & 31);
    if (lane == 0) {
      if (a < p.Q + p.KVd) {
        const float ra = __fsub_rn(__fmul_rn(va, c), __fmul_rn(vb, s));
        const float rb = __fadd_rn(__fmul_rn(va, s), __fmul_rn(vb, c));
        if (a < p.Q) {
          st_ll(p.q_ll + a, ra, tag);
          st_ll(p.q_ll + a + 1, rb, tag);
        } else {
          const int kr = a - p.Q, g = kr / p.hd, d = kr % p.hd;
          float *dst = p.kc + (((size_t)l * p.KVH + g) * p.max_ctx + pos) * p.hd + d;
          dst[0] = ra;
          dst[1] = rb;
          st_ll(p.kv_ll + kr, ra, tag);
          st_ll(p.kv_ll + kr + 1, rb, tag);
        }
      } else {
        const int vr = a - p.Q - p.KVd, g = vr / p.hd, d = vr % p.hd;
        float *dst = p.vc + (((size_t)l * p.KVH + g) * p.max_ctx + pos) * p.hd + d;
        dst[0] = va;
        dst[1] = vb;
        st_ll(p.kv_ll + p.KVd + vr, va, tag);
        st_ll(p.kv_ll + p.KVd + vr + 1, vb, tag);
      }
    }
  } else if ((kind == ST_O || kind == ST_DOWN) && p.tp_world > 1) {  // a row-parallel partial, to every rank
    if (lane == 0) {
      const size_t off = ((size_t)(kind == ST_DOWN) * p.tp_world + p.tp_rank) * p.E;
      for (int d = 0; d < p.tp_world; d++) {
        if (a != 0 || tag != p.drop_tag) st_ll_sys(p.tp_box[d] + off + a, va, tag);
        if (hasb) st_ll_sys(p.tp_box[d] + off + b, vb, tag);
      }
    }
  } else if (kind == ST_O || kind == ST_DOWN) {  // residual (elementwise_add.rs:47-61)
    const float ha = __shfl_sync(FULL, sr.hres, (a - r0) & 31);
    const float hb = __shfl_sync(FULL, sr.hres, (b - r0) & 31);
    if (lane == 0) {
      if (a != 0 || tag != p.drop_tag) st_ll(p.hid_ll + a, __fadd_rn(ha, va), tag);
      if (hasb) st_ll(p.hid_ll + b, __fadd_rn(hb, vb), tag);
    }
  } else if (kind == ST_GU) {  // a = gate row, vb = up (silu.rs:4-8, elementwise_mul.rs:3-17)
    if (lane == 0) st_ll(p.act_ll + a, __fmul_rn(__fmul_rn(va, sigmoid_ref(va)), vb), tag);
  } else {  // LM head logits
    if (lane == 0) {
      p.logits[a] = va;
      sm.lm[a - r0] = va;
      if (hasb) {
        p.logits[b] = vb;
        sm.lm[b - r0] = vb;
      }
    }
  }
}

// Wait until `slot` holds tile k and its bytes have landed. The two warp groups
// consume alternate tiles, so a group can be two phases of a slot's barrier ahead
// of the slot's last completed phase; the parity wait is meaningful only once the
// slot's current phase is tile k's, which sm.slot_tile tells.
__device__ __forceinline__ bool slot_wait(const Params &p, const Ring &rg, const Smem &sm, int slot, int k,
                                          unsigned phase) {
  if (*(volatile const int *)&sm.slot_tile[slot] != k) {
    const long long t0 = clock64();
    for (unsigned it = 0; *(volatile const int *)&sm.slot_tile[slot] != k; it++)
      if ((it & 63u) == 63u && poll_expired(p, t0)) return false;
  }
  return mbar_wait(&rg.full[slot], phase, p.err);
}

__device__ __forceinline__ void group_sync(int grp) {
  asm volatile("bar.sync %0, %1;" ::"r"(2 + grp), "n"(NG * 32) : "memory");
}

// One matvec stage of this CTA. The CTA's tiles rotate over NGRP groups of NG warps
// (tile k goes to group k % NGRP), so one group's reductions, epilogues and slot
// refills overlap the other groups' dot products. Within a tile a warp takes four
// rows at a time (two row pairs, or four rows of its input segment when the rows
// are split into segments) and reduces them together.
template <int T, bool AQ>
__device__ __forceinline__ void matvec_stage(const Params &p, const Ring &rg, Smem &sm, const int2 *tbl, int kind, int l,
                             float osc, int &slot, unsigned &phase, int &tile_ctr, int pos,
                             const StageRegs &sr, unsigned tag) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = warp / NG, wig = warp % NG;
  const int nseg = stage_nseg(p, kind), rb = stage_rb(p, kind), Tr = p.tile_rows[kind];
  const int in_dim = stage_in_dim(p, kind);
  const bool gu = kind == ST_GU;
  const int seg = wig % nseg, rpw = NG / nseg, rs = wig / nseg;
  const bool active = lane_active<T>(seg, lane, in_dim);
  const uint32_t slots = smem_u32(rg.slots);
  const bool lead = wig == 0 && lane == 0;  // stamps of the group that has the tile
  int r0, r1;
  stage_rows(p, kind, l, blockIdx.x, r0, r1);
  const int stage_id = kind == ST_LM ? 5 * p.L : 5 * l + (kind == ST_QKV ? 0 : (kind == ST_DOWN2 ? ST_DOWN : kind) + 1);
  for (int r = r0; r < r1; r += Tr) {
    if (tile_ctr % NGRP == grp) {
      const int n = min(Tr, r1 - r);
      const int rows = gu ? 2 * n : n;
      const uint32_t tile = slots + (uint32_t)slot * (uint32_t)p.slot_bytes;
      float *red = sm.red[2 * grp + ((tile_ctr / NGRP) & 1)];
      const bool ok = slot_wait(p, rg, sm, slot, tile_ctr, phase);
      if (lead) stamp_tile(p, tile_ctr, 1);
      if (lead && r == r0) stamp_now(p, 8 * stage_id + 4);
      if (lead && r + Tr >= r1) stamp_now(p, 8 * stage_id + 5);
      if (ok) {
        if (nseg == 1) {
          // warp-owned row pairs (2i, 2i+1), or (gate i, up i): pairs i and i + NG
          // together (four rows, one reduction)
          const int npairs = gu ? n : (n + 1) >> 1;
          for (int i = wig; i < npairs; i += 2 * NG) {
            const int i2 = i + NG;
            const bool has2 = i2 < npairs;
            int rw[4];
            rw[0] = gu ? i : 2 * i;
            rw[1] = gu ? n + i : 2 * i + 1;
            rw[2] = gu ? i2 : 2 * i2;
            rw[3] = gu ? n + i2 : 2 * i2 + 1;
            const bool hasb = rw[1] < rows, hasb2 = has2 && rw[3] < rows;
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            if (active) {
              // a missing row reads row rw[0] again (in bounds) and is not used
              const uint32_t ra[4] = {tile + (uint32_t)rw[0] * rb, tile + (uint32_t)(hasb ? rw[1] : rw[0]) * rb,
                                      tile + (uint32_t)(has2 ? rw[2] : rw[0]) * rb,
                                      tile + (uint32_t)(hasb2 ? rw[3] : rw[0]) * rb};
              if constexpr (AQ) quad_dot_q<T>(ra, 0, lane, sm.qs, v);
              else quad_dot_xs<T>(ra, 0, lane, smem_u32(sm.xs), v);
            }
            warp_sum4(v);
            if (gu) {
              finish_rows(p, sm, kind, l, pos, r0, r + i, v[0] * osc, r + i, v[1] * osc, true, sr, tag);
              if (has2) finish_rows(p, sm, kind, l, pos, r0, r + i2, v[2] * osc, r + i2, v[3] * osc, true, sr, tag);
            } else {
              finish_rows(p, sm, kind, l, pos, r0, r + rw[0], v[0] * osc, r + rw[1], v[1] * osc, hasb, sr, tag);
              if (has2)
                finish_rows(p, sm, kind, l, pos, r0, r + rw[2], v[2] * osc, r + rw[3], v[3] * osc, hasb2, sr, tag);
            }
          }
        } else {
          // segment-split rows: this warp's segment of rows rs, rs + rpw, rs + 2 rpw,
          // rs + 3 rpw, ...; the partial sums meet in shared memory
          for (int i = rs; i < rows; i += 4 * rpw) {
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            if (active) {
              uint32_t ra[4];
#pragma unroll
              for (int q = 0; q < 4; q++) ra[q] = tile + (uint32_t)(i + q * rpw < rows ? i + q * rpw : i) * rb;
              if constexpr (AQ) quad_dot_q<T>(ra, seg, lane, sm.qs, v);
              else quad_dot_xs<T>(ra, seg, lane, smem_u32(sm.xs), v);
            }
            warp_sum4(v);
            if (lane == 0) {
#pragma unroll
              for (int q = 0; q < 4; q++)
                if (i + q * rpw < rows) red[(i + q * rpw) * nseg + seg] = v[q];
            }
          }
        }
      }
      release_slot(p, rg, sm, tbl, slot, tile_ctr, NG, ok);
      if (lead) stamp_tile(p, tile_ctr, 2);
      if (nseg > 1) {
        group_sync(grp);
        // finish the tile's rows: warp wig takes row pairs wig, wig + NG, ...
        if (ok) {
          const int npairs = gu ? n : (n + 1) >> 1;
          for (int i = wig; i < npairs; i += NG) {
            const int a = gu ? i : 2 * i, b = gu ? n + i : 2 * i + 1;
            const bool hasb = b < rows;
            float va = 0.f, vb = 0.f;
            for (int s = 0; s < nseg; s++) {
              va += red[a * nseg + s];
              if (hasb) vb += red[b * nseg + s];
            }
            va *= osc;
            vb *= osc;
            if (kind == ST_DOWN && p.split) {  // part 1 of a split down row: kept for part 2
              if (lane == 0) {
                sm.dpart[r + a - r0] = va;
                if (hasb) sm.dpart[r + b - r0] = vb;
              }
            } else if (kind == ST_DOWN2) {  // part 2: part 1 + part 2, then the residual
              finish_rows(p, sm, ST_DOWN, l, pos, r0, r + a, sm.dpart[r + a - r0] + va, r + b,
                          hasb ? sm.dpart[r + b - r0] + vb : 0.f, hasb, sr, tag);
            } else if (gu) {
              finish_rows(p, sm, kind, l, pos, r0, r + i, va, r + i, vb, true, sr, tag);
            } else {
              finish_rows(p, sm, kind, l, pos, r0, r + a, va, r + b, vb, hasb, sr, tag);
            }
          }
        }
      }
    }
    if (++slot == NSLOT) {
      slot = 0;
      phase ^= 1u;
    }
    tile_ctr++;
  }
  stamp(p, 8 * stage_id + 6);
}

// Tensor parallel: after this CTA's O (or down) stage, its hidden rows summed over the
// ranks' partials in rank order (layers.rs:57 / :76 row-parallel sums), plus the
// residual (layers.rs:96 / :106), published locally for the next stage's staging.
// One warp; lane i takes row r0 + i (a CTA owns at most 32 rows).
__device__ __forceinline__ void tp_reduce_rows(const Params &p, int kind, int l, const StageRegs &sr, unsigned tag) {
  const int lane = threadIdx.x & 31;
  int r0, r1;
  stage_rows(p, kind, l, blockIdx.x, r0, r1);
  if (r1 <= r0) return;
  const int a = r0 + lane;
  const bool mine = lane < r1 - r0;
  const unsigned long long *box = p.tp_box[p.tp_rank] + (size_t)(kind == ST_O ? 0 : 1) * p.tp_world * p.E;
  const unsigned long long *w[8];
#pragma unroll
  for (int r = 0; r < 8; r++) w[r] = box + (size_t)(r < p.tp_world ? r : 0) * p.E + (mine ? a : r0);
  float v[8];
  poll_ll_n<8, true>(p, w, tag, v);
  float sum = v[0];
#pragma unroll
  for (int r = 1; r < 8; r++)
    if (r < p.tp_world) sum += v[r];
  if (mine) st_ll(p.hid_ll + a, __fadd_rn(sr.hres, sum), tag);
}

// Causal GQA attention for one token at position pos (attention.rs:11-70), reading
// q and the new K/V row from the tagged words of the QKV stage and the older
// positions from the KV cache; the output goes out tagged for the O stage.
//
// Short contexts (head_dim 64, pos < SHORT_CTX): one item per q head. The warps
// split the cached positions 32 at a time; lane = position for q.k (q broadcast from
// shared memory, no reductions), lane = dimension for p.V; each warp keeps a running
// max / sum / accumulator, the warps merge in shared memory, and warp 0 adds the
// current position.
constexpr int SHORT_CTX = 512;

template <int DPL>
__device__ void attention_heads(const Params &p, Smem &sm, int l, int pos, unsigned tag_in, unsigned tag_out) {
  constexpr int HD = DPL * 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int h = blockIdx.x; h < p.H; h += p.G) {
    const int g = h / GROUP;
    if (warp == 0) {
#pragma unroll
      for (int i = 0; i < DPL; i++) sm.qh[lane + 32 * i] = poll_ll(p, p.q_ll + (size_t)h * HD + lane + 32 * i, tag_in);
    }
    cta_sync();
    const float *kb = p.kc + ((size_t)l * p.KVH + g) * p.max_ctx * HD;
    const float *vb = p.vc + ((size_t)l * p.KVH + g) * p.max_ctx * HD;
    float m = -INFINITY, lsum = 0.f, acc[DPL];
#pragma unroll
    for (int i = 0; i < DPL; i++) acc[i] = 0.f;
    for (int base = warp * 32; base < pos; base += NC * 32) {
      const int s = base + lane;
      const bool valid = s < pos;
      float4 kr[HD / 4];
#pragma unroll
      for (int k = 0; k < HD / 4; k++)
        kr[k] = valid ? ldcg4(kb + (size_t)s * HD + 4 * k) : make_float4(0.f, 0.f, 0.f, 0.f);
      constexpr int VJ = 64 / DPL;  // V rows per batch (64 registers): in flight with q.K and the softmax
      float vv[VJ][DPL];
      auto load_v = [&](int j0) {
#pragma unroll
        for (int j = 0; j < VJ; j++)
#pragma unroll
          for (int i = 0; i < DPL; i++)
            vv[j][i] = base + j0 + j < pos ? __ldcg(vb + (size_t)(base + j0 + j) * HD + lane + 32 * i) : 0.f;
      };
      load_v(0);
      float d = 0.f;
#pragma unroll
      for (int k = 0; k < HD / 4; k++) {
        const float4 q4 = *reinterpret_cast<const float4 *>(&sm.qh[4 * k]);
        d = fmaf(q4.x, kr[k].x, d);
        d = fmaf(q4.y, kr[k].y, d);
        d = fmaf(q4.z, kr[k].z, d);
        d = fmaf(q4.w, kr[k].w, d);
      }
      const float sc = valid ? d * p.attn_scale : -INFINITY;
      const float mn = fmaxf(m, warp_max(sc));
      const float corr = expf(m - mn);
      const float pj = valid ? expf(sc - mn) : 0.f;
      lsum = fmaf(lsum, corr, warp_sum(pj));
#pragma unroll
      for (int i = 0; i < DPL; i++) acc[i] *= corr;
#pragma unroll
      for (int j0 = 0; j0 < 32; j0 += VJ) {
        if (j0) load_v(j0);
#pragma unroll
        for (int j = 0; j < VJ; j++) {
          const float pjj = __shfl_sync(FULL, pj, j0 + j);
#pragma unroll
          for (int i = 0; i < DPL; i++) acc[i] = fmaf(pjj, vv[j][i], acc[i]);
        }
      }
      m = mn;
    }
    if (lane == 0) {
      sm.at.m[warp][0] = m;
      sm.at.l[warp][0] = lsum;
    }
#pragma unroll
    for (int i = 0; i < DPL; i++) sm.at.a[warp][0][lane + 32 * i] = acc[i];
    cta_sync();
    if (warp == 0) {
      float M = -INFINITY;
      for (int w = 0; w < NC; w++) M = fmaxf(M, sm.at.m[w][0]);
      float Ls = 0.f, A[DPL];
#pragma unroll
      for (int i = 0; i < DPL; i++) A[i] = 0.f;
      for (int w = 0; w < NC; w++) {
        const float f = sm.at.l[w][0] > 0.f ? expf(sm.at.m[w][0] - M) : 0.f;
        Ls = fmaf(sm.at.l[w][0], f, Ls);
#pragma unroll
        for (int i = 0; i < DPL; i++) A[i] = fmaf(sm.at.a[w][0][lane + 32 * i], f, A[i]);
      }
      // the current position
      float kq[DPL], vq[DPL], d = 0.f;
#pragma unroll
      for (int i = 0; i < DPL; i++) {
        kq[i] = poll_ll(p, p.kv_ll + (size_t)g * HD + lane + 32 * i, tag_in);
        vq[i] = poll_ll(p, p.kv_ll + p.KVd + (size_t)g * HD + lane + 32 * i, tag_in);
        d = fmaf(sm.qh[lane + 32 * i], kq[i], d);
      }
      const float sc = warp_sum(d) * p.attn_scale;
      const float mn = fmaxf(M, sc);
      const float corr = expf(M - mn), pp = expf(sc - mn);
      Ls = fmaf(Ls, corr, pp);
      const float inv = 1.0f / Ls;
#pragma unroll
      for (int i = 0; i < DPL; i++)
        st_ll(p.attn_ll + (size_t)h * HD + lane + 32 * i, fmaf(pp, vq[i], A[i] * corr) * inv, tag_out);
    }
    cta_sync();
  }
}

// Long contexts, grouped: split-KV over (kv head, chunk) items, so each K / V row a
// chunk covers is read once for the GROUP q heads that share it (GQA), not once per
// q head. Warp w takes q heads 2 * (w / 4) and 2 * (w / 4) + 1 of the group and the
// chunk's 32-position blocks w % 4, w % 4 + 4, ...: a lane owns a position for q.k
// (its K row in registers, both heads' dots from it), the warp's online softmax per
// head over its blocks, then lane = dimension for p.V with each V row loaded once
// for both heads. The four warps of a head merge in shared memory into the chunk's
// partial per head; the chunk that holds the token's own position adds it from the
// QKV stage's tagged words; the last CTA to finish a kv head combines the chunks of
// its four heads (one warp per head) and publishes their outputs.
// Chunks of the (kv head, chunk) attention items at key length Lk: ~128 positions a
// chunk (four 32-position blocks, one per warp pair), at most max_chunks per head.
__device__ __forceinline__ void attn_chunking(const Params &p, int Lk, int &n_chunks, int &CH) {
  n_chunks = (Lk + 127) / 128;
  if (n_chunks > p.max_chunks) n_chunks = p.max_chunks;
  CH = (Lk + n_chunks - 1) / n_chunks;
}

template <int DPL>
__device__ void attention_groups(const Params &p, Smem &sm, int l, int pos, unsigned tag_in, unsigned tag_out) {
  constexpr int HD = DPL * 32;
  static_assert(GROUP == 4 && NC >= 8, "two heads x four position lanes of warps (warps past 8 only keep step)");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int Lk = pos + 1;
  int n_chunks, CH;
  attn_chunking(p, Lk, n_chunks, CH);
  const int items = p.KVH * n_chunks;
  const int hp = warp >> 2, bw = warp & 3;  // head pair, block lane of this warp
  for (int item = blockIdx.x; item < items; item += p.G) {
    const int g = item / n_chunks, c = item % n_chunks;
    const int s0 = c * CH, s1 = min(Lk, s0 + CH);
    const int cached_end = min(s1, pos);  // positions below pos come from the cache
    const float *kb = p.kc + ((size_t)l * p.KVH + g) * p.max_ctx * HD;
    const float *vb = p.vc + ((size_t)l * p.KVH + g) * p.max_ctx * HD;
    float4 kr[HD / 4];
    auto load_k = [&](int base) {
      const int s = base + lane;
      const bool valid = s < cached_end;
#pragma unroll
      for (int k = 0; k < HD / 4; k++)
        kr[k] = valid ? ldcg4(kb + (size_t)s * HD + 4 * k) : make_float4(0.f, 0.f, 0.f, 0.f);
    };
    if (s0 + bw * 32 < cached_end) load_k(s0 + bw * 32);
    if (warp < GROUP) {  // the group's four q heads into shared memory
      const unsigned long long *qa[DPL];
      float qv[DPL];
#pragma unroll
      for (int i = 0; i < DPL; i++) qa[i] = p.q_ll + (size_t)(g * GROUP + warp) * HD + lane + 32 * i;
      poll_ll_n<DPL>(p, qa, tag_in, qv);
#pragma unroll
      for (int i = 0; i < DPL; i++) sm.at.a[warp][0][lane + 32 * i] = qv[i];  // head j's q in slot [j][0]
    }
    cta_sync();
    const float *q0 = sm.at.a[2 * hp][0], *q1 = sm.at.a[2 * hp + 1][0];
    float m[2] = {-INFINITY, -INFINITY}, lsum[2] = {0.f, 0.f}, acc[2][DPL];
#pragma unroll
    for (int i = 0; i < DPL; i++) acc[0][i] = acc[1][i] = 0.f;
    // V rows per batch: head_dim 64 all 32 rows of the block (64 registers), loaded
    // before q.K so that they are in flight with it and the softmax; head_dim 128
    // (whose keys already take 128 registers) 8 rows at a time after the softmax
    constexpr int VJ = DPL <= 2 ? 32 : 8;
    for (int base = s0 + bw * 32; base < cached_end; base += 4 * 32) {
      const int s = base + lane;
      const bool valid = s < cached_end;
      float vv[VJ][DPL];
      auto load_v = [&](int j0) {
#pragma unroll
        for (int j = 0; j < VJ; j++)
#pragma unroll
          for (int i = 0; i < DPL; i++)
            vv[j][i] = base + j0 + j < cached_end ? __ldcg(vb + (size_t)(base + j0 + j) * HD + lane + 32 * i) : 0.f;
      };
      if constexpr (DPL <= 2) load_v(0);
      float d0 = 0.f, d1 = 0.f;
#pragma unroll
      for (int k = 0; k < HD / 4; k++) {
        const float4 a = *reinterpret_cast<const float4 *>(q0 + 4 * k), b = *reinterpret_cast<const float4 *>(q1 + 4 * k);
        d0 = fmaf(a.x, kr[k].x, d0);
        d0 = fmaf(a.y, kr[k].y, d0);
        d0 = fmaf(a.z, kr[k].z, d0);
        d0 = fmaf(a.w, kr[k].w, d0);
        d1 = fmaf(b.x, kr[k].x, d1);
        d1 = fmaf(b.y, kr[k].y, d1);
        d1 = fmaf(b.z, kr[k].z, d1);
        d1 = fmaf(b.w, kr[k].w, d1);
      }
      if (base + 4 * 32 < cached_end) load_k(base + 4 * 32);  // the next block's keys while this one finishes
      float pj[2];
#pragma unroll
      for (int t = 0; t < 2; t++) {
        const float sc = valid ? (t ? d1 : d0) * p.attn_scale : -INFINITY;
        const float mn = fmaxf(m[t], warp_max(sc));
        const float corr = expf(m[t] - mn);
        pj[t] = valid ? expf(sc - mn) : 0.f;
        lsum[t] = fmaf(lsum[t], corr, warp_sum(pj[t]));
#pragma unroll
        for (int i = 0; i < DPL; i++) acc[t][i] *= corr;
        m[t] = mn;
      }
#pragma unroll
      for (int j0 = 0; j0 < 32; j0 += VJ) {
        if (j0 > 0 || DPL > 2) load_v(j0);
#pragma unroll
        for (int j = 0; j < VJ; j++) {
          const float p0 = __shfl_sync(FULL, pj[0], j0 + j), p1 = __shfl_sync(FULL, pj[1], j0 + j);
#pragma unroll
          for (int i = 0; i < DPL; i++) {
            acc[0][i] = fmaf(p0, vv[j][i], acc[0][i]);
            acc[1][i] = fmaf(p1, vv[j][i], acc[1][i]);
          }
        }
      }
    }
    // per-warp partials in slots [warp][2 + t] for local head t (q stays in [j][0] for the merge)
    cta_sync();
#pragma unroll
    for (int t = 0; t < 2; t++) {
      if (lane == 0) {
        sm.at.m[warp][t] = m[t];
        sm.at.l[warp][t] = lsum[t];
      }
#pragma unroll
      for (int i = 0; i < DPL; i++) sm.at.a[warp][2 + t][lane + 32 * i] = acc[t][i];
    }
    cta_sync();
    if (warp < GROUP) {  // warp j merges head j of the group over its four warps, adds the token's own position
      const int j = warp, hpj = j >> 1, t = j & 1, h = g * GROUP + j;
      float M = -INFINITY;
      for (int w = 4 * hpj; w < 4 * hpj + 4; w++) M = fmaxf(M, sm.at.m[w][t]);
      float Ls = 0.f, A[DPL];
#pragma unroll
      for (int i = 0; i < DPL; i++) A[i] = 0.f;
      for (int w = 4 * hpj; w < 4 * hpj + 4; w++) {
        const float f = sm.at.l[w][t] > 0.f ? expf(sm.at.m[w][t] - M) : 0.f;
        Ls = fmaf(sm.at.l[w][t], f, Ls);
#pragma unroll
        for (int i = 0; i < DPL; i++) A[i] = fmaf(sm.at.a[w][2 + t][lane + 32 * i], f, A[i]);
      }
      if (s1 == Lk) {
        const unsigned long long *kva[2 * DPL];
        float kvq[2 * DPL], d = 0.f;
#pragma unroll
        for (int i = 0; i < DPL; i++) {
          kva[i] = p.kv_ll + (size_t)g * HD + lane + 32 * i;
          kva[DPL + i] = p.kv_ll + p.KVd + (size_t)g * HD + lane + 32 * i;
        }
        poll_ll_n<2 * DPL>(p, kva, tag_in, kvq);
#pragma unroll
        for (int i = 0; i < DPL; i++) d = fmaf(sm.at.a[j][0][lane + 32 * i], kvq[i], d);
        const float sc = warp_sum(d) * p.attn_scale;
        const float mn = fmaxf(M, sc);
        const float corr = Ls > 0.f ? expf(M - mn) : 0.f, pp = expf(sc - mn);
        Ls = fmaf(Ls, corr, pp);
#pragma unroll
        for (int i = 0; i < DPL; i++) A[i] = fmaf(pp, kvq[DPL + i], A[i] * corr);
        M = mn;
      }
      float *pp = p.attn_part + ((size_t)h * p.max_chunks + c) * (HD + 2);
      if (lane == 0) {
        pp[0] = M;
        pp[1] = Ls;
      }
#pragma unroll
      for (int i = 0; i < DPL; i++) pp[2 + lane + 32 * i] = A[i];
      __threadfence();
    }
    cta_sync();
    if (threadIdx.x == 0) {
      const unsigned old = atomicAdd(p.attn_cnt + (size_t)l * p.H + g, 1u);
      sm.flag = old == (unsigned)(n_chunks - 1);
    }
    cta_sync();
    if (sm.flag && warp < GROUP) {  // the kv head's last chunk: warp j combines head j's chunks
      __threadfence();
      const int h = g * GROUP + warp;
      float M = -INFINITY;
      for (int cc = 0; cc < n_chunks; cc++) {
        const float *pp = p.attn_part + ((size_t)h * p.max_chunks + cc) * (HD + 2);
        if (__ldcg(pp + 1) > 0.f) M = fmaxf(M, __ldcg(pp));
      }
      float Ls = 0.f, A[DPL];
#pragma unroll
      for (int i = 0; i < DPL; i++) A[i] = 0.f;
      for (int cc = 0; cc < n_chunks; cc++) {
        const float *pp = p.attn_part + ((size_t)h * p.max_chunks + cc) * (HD + 2);
        const float lc = __ldcg(pp + 1);
        if (lc > 0.f) {
          const float f = expf(__ldcg(pp) - M);
          Ls = fmaf(lc, f, Ls);
#pragma unroll
          for (int i = 0; i < DPL; i++) A[i] = fmaf(__ldcg(pp + 2 + lane + 32 * i), f, A[i]);
        }
      }
      const float inv = 1.0f / Ls;
#pragma unroll
      for (int i = 0; i < DPL; i++) st_ll(p.attn_ll + (size_t)h * HD + lane + 32 * i, A[i] * inv, tag_out);
    }
    cta_sync();
    if (sm.flag && threadIdx.x == 0) p.attn_cnt[(size_t)l * p.H + g] = 0;  // ready for the next token
  }
}

// Ordered greedy fold (greedy.rs:6-15) over n values in shared memory by one warp:
// lanes take contiguous sub-ranges, combined left to right. Valid in lane 0.
__device__ ArgState warp_argmax_smem(const float *v, int n, long long base) {
  const int lane = threadIdx.x & 31;
  const int per = (n + 31) / 32;
  ArgState s = arg_empty();
  for (int i = lane * per; i < (lane + 1) * per && i < n; i++) s = arg_combine(s, arg_elem(v[i], base + i));
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    ArgState r;
    r.v = __shfl_down_sync(FULL, s.v, o);
    r.best = __shfl_down_sync(FULL, s.best, o);
    r.nan = __shfl_down_sync(FULL, s.nan, o);
    if ((lane & (2 * o - 1)) == 0) s = arg_combine(s, r);
  }
  return s;
}

__device__ __forceinline__ void load_stage_regs(const Params &p, int kind, int l, int pos, StageRegs &sr,
                                                unsigned hid_tag) {
  const int lane = threadIdx.x & 31;
  if (kind == ST_QKV) {
    const int half = p.hd >> 1;
    const size_t base = (size_t)pos * half;
    sr.c0 = lane < half ? __ldg(p.cos_t + base + lane) : 0.f;
    sr.s0 = lane < half ? __ldg(p.sin_t + base + lane) : 0.f;
    sr.c1 = lane + 32 < half ? __ldg(p.cos_t + base + 32 + lane) : 0.f;
    sr.s1 = lane + 32 < half ? __ldg(p.sin_t + base + 32 + lane) : 0.f;
  } else if (kind == ST_O || kind == ST_DOWN || kind == ST_DOWN2) {  // the residual of this CTA's rows (<= 32)
    int r0, r1;
    stage_rows(p, kind, l, blockIdx.x, r0, r1);
    sr.hres = lane < r1 - r0 ? poll_ll(p, p.hid_ll + r0 + lane, hid_tag) : 0.f;
  }
}

template <int T, int DPL, bool AQ>
__global__ void __launch_bounds__(NTHREADS, 1)
    k_decode(const __grid_constant__ Params p, const uint32_t *tok_in, uint32_t *tok_out, uint32_t *out_ids,
             int step) {
  extern __shared__ __align__(128) uint8_t dsm[];
  Ring rg;
  rg.slots = dsm;
  rg.full = reinterpret_cast<uint64_t *>(dsm + (size_t)NSLOT * p.slot_bytes);
  uint64_t *tbl_bar = rg.full + NSLOT;
  Smem &sm = *reinterpret_cast<Smem *>(tbl_bar + 1);  // 16-byte aligned: 5 + 1 barriers of 8 bytes
  int2 *tbl = reinterpret_cast<int2 *>(&sm + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  stamp_sync(p, TL_STRIDE(p) - 6);
  stamp(p, 0);
  if (threadIdx.x == 0) {
    for (int s = 0; s < NSLOT; s++) {
      mbar_init(&rg.full[s], 1);
      sm.rel[s] = 0;
      sm.issued[s] = 0;
      sm.slot_tile[s] = -1;
    }
    mbar_init(tbl_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // this CTA's tile table (8 bytes a tile, padded to 16) into shared memory, then the first NSLOT tiles
    const int nt = p.ntiles[blockIdx.x];
    sm.ntiles = nt;
    const unsigned tb = (unsigned)((nt * 8 + 15) & ~15);
    mbar_expect_tx(tbl_bar, tb);
    bulk_g2s(tbl, p.tiles + (size_t)blockIdx.x * p.max_tiles, tb, tbl_bar);
    if (mbar_wait(tbl_bar, 0, p.err)) {
      for (int j = 0; j < NSLOT && j < nt; j++) issue_tile(p, rg, sm, tbl, j, j);
    }
  }
  __syncthreads();
  const int pos = *p.pos;
  const uint32_t tok = *tok_in;
  const unsigned launch = *p.launch;
  int slot = 0, tile_ctr = 0;
  unsigned phase = 0;
  StageRegs sr = {0.f, 0.f, 0.f, 0.f, 0.f};
  // One pass per projection stage: QKV, O, gate/up, down (in two input parts when
  // split) of every layer, then the LM head; a single matvec call site keeps one copy
  // of the tile loop in the instruction cache for all of them.
  const int spl = p.split ? 5 : 4;  // stages per layer
  for (int si = 0; si <= spl * p.L; si++) {
    const int l = si / spl, sk = si - l * spl;
    const int kind = l == p.L ? ST_LM : (sk == 4 ? ST_DOWN2 : sk);  // ST_QKV, ST_O, ST_GU, ST_DOWN are 0..3
    const int stage_id = kind == ST_LM ? 5 * p.L : 5 * l + (kind == ST_QKV ? 0 : (kind == ST_DOWN2 ? ST_DOWN : kind) + 1);
    const LayerW &W = p.layers[l < p.L ? l : 0];
    const unsigned hid_in = l == 0 ? mk_tag(launch, 0, TG_EMBED) : mk_tag(launch, l - 1, TG_POST_DOWN);
    load_stage_regs(p, kind, l, pos, sr, kind == ST_DOWN || kind == ST_DOWN2 ? mk_tag(launch, l, TG_POST_O) : hid_in);
    if (si > 0) cta_sync();  // every warp is done with the previous input: the staging buffer is rewritten
    float osc;
    unsigned tag_out;
    if (kind == ST_QKV) {
      if (l == 0)
        osc = stage_in<T, XS_EMBED, AQ>(p, sm, nullptr, 0u, W.attn_norm, p.E, 8 * stage_id + 1,
                                    p.embd + (size_t)tok * p.rb_E, blockIdx.x == 0, hid_in);
      else
        osc = stage_in<T, XS_NORM, AQ>(p, sm, p.hid_ll, hid_in, W.attn_norm, p.E, 8 * stage_id + 1);
      tag_out = mk_tag(launch, l, TG_QKV);
    } else if (kind == ST_O) {
      osc = stage_in<T, XS_PLAIN, AQ>(p, sm, p.attn_ll, mk_tag(launch, l, TG_ATTN), nullptr, p.Q, 8 * stage_id + 1);
      tag_out = mk_tag(launch, l, TG_POST_O);
    } else if (kind == ST_DOWN || kind == ST_DOWN2) {
      const int x0 = kind == ST_DOWN2 ? p.xa : 0;
      osc = stage_in<T, XS_PLAIN, AQ>(p, sm, p.act_ll + x0, mk_tag(launch, l, TG_ACT), nullptr, stage_in_dim(p, kind),
                                  8 * stage_id + 1);
      tag_out = mk_tag(launch, l, TG_POST_DOWN);
    } else {  // gate/up after the FFN norm, or the LM head after the final norm (model.rs:72-95)
      const bool lm = kind == ST_LM;
      osc = stage_in<T, XS_NORM, AQ>(p, sm, p.hid_ll, lm ? mk_tag(launch, p.L - 1, TG_POST_DOWN) : mk_tag(launch, l, TG_POST_O),
                                 lm ? p.out_norm : W.ffn_norm, p.E, 8 * stage_id + 1);
      tag_out = lm ? 0u : mk_tag(launch, l, TG_ACT);
    }
    stamp(p, 8 * stage_id + 2);
    matvec_stage<T, AQ>(p, rg, sm, tbl, kind, l, osc, slot, phase, tile_ctr, pos, sr, tag_out);
    if (p.tp_world > 1 && warp == 0 && (kind == ST_O || kind == (p.split ? ST_DOWN2 : ST_DOWN)))
      tp_reduce_rows(p, kind == ST_O ? ST_O : ST_DOWN, l, sr, tag_out);
    if (kind == ST_QKV) {
      // ---- attention (waits on q / K / V words, not on a barrier)
      cta_sync();  // shared scratch of the staging buffer is reused below
      if (DPL <= 2 && pos < SHORT_CTX) attention_heads<DPL <= 2 ? DPL : 2>(p, sm, l, pos, tag_out, mk_tag(launch, l, TG_ATTN));
      else attention_groups<DPL>(p, sm, l, pos, tag_out, mk_tag(launch, l, TG_ATTN));
      stamp(p, 8 * (5 * l + 1) + 6);
    }
  }
  cta_sync();
  stamp(p, TL_STRIDE(p) - 2);
  // ---- greedy argmax: this CTA's rows (kept in shared memory) in order, then the
  // last CTA to finish folds the per-CTA states in row order
  if (warp == 0) {
    int r0, r1;
    stage_rows(p, ST_LM, p.L, blockIdx.x, r0, r1);
    const ArgState s = warp_argmax_smem(sm.lm, r1 - r0, r0);
    unsigned last = 0;
    if (lane == 0) {
      p.arg_part[blockIdx.x] = s;
      __threadfence();
      last = atomicAdd(p.ticket, 1u) == (unsigned)(p.G - 1);
    }
    last = __shfl_sync(FULL, last, 0);
    if (last) {
      __threadfence();
      ArgState acc = arg_empty();
      const int stage = p.L * 5 + ST_LM;
      for (int base = 0; base < p.G; base += 32) {
        ArgState mine = arg_empty();
        const int i = base + lane;  // rotated index i owns the i-th row range
        if (i < p.G) {
          const int owner = ((i - stage * 61) % p.G + p.G) % p.G;
          mine.v = __ldcg(&p.arg_part[owner].v);
          mine.best = __ldcg(&p.arg_part[owner].best);
          mine.nan = __ldcg(&p.arg_part[owner].nan);
        }
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          ArgState r;
          r.v = __shfl_down_sync(FULL, mine.v, o);
          r.best = __shfl_down_sync(FULL, mine.best, o);
          r.nan = __shfl_down_sync(FULL, mine.nan, o);
          if ((lane & (2 * o - 1)) == 0) mine = arg_combine(mine, r);
        }
        if (lane == 0) acc = arg_combine(acc, mine);
      }
      if (p.tp_world > 1) {  // this rank's state to every rank, then all ranks' states in rank order
        acc.v = __shfl_sync(FULL, acc.v, 0);
        acc.best = __shfl_sync(FULL, acc.best, 0);
        acc.nan = __shfl_sync(FULL, acc.nan, 0);
        const unsigned tag = mk_tag(launch, p.L, TG_ARG);
        const size_t off = (size_t)2 * p.tp_world * p.E + (size_t)p.tp_rank * 3;
        if (lane < p.tp_world) {
          unsigned long long *d = p.tp_box[lane] + off;
          st_ll_sys(d, acc.v, tag);
          st_ll_sys(d + 1, __int_as_float((int)acc.best), tag);
          st_ll_sys(d + 2, __int_as_float((int)acc.nan), tag);
        }
        ArgState all = arg_empty();
        if (lane == 0) {
          const unsigned long long *src = p.tp_box[p.tp_rank] + (size_t)2 * p.tp_world * p.E;
          for (int r = 0; r < p.tp_world; r++) {
            const unsigned long long *w3[3] = {src + r * 3, src + r * 3 + 1, src + r * 3 + 2};
            float v3[3];
            poll_ll_n<3, true>(p, w3, tag, v3);
            const long long base = (long long)r * p.vocab_local;
            const int best = __float_as_int(v3[1]), nan = __float_as_int(v3[2]);
            ArgState st = {v3[0], best >= 0 ? base + best : -1, nan >= 0 ? base + nan : -1};
            all = arg_combine(all, st);
          }
        }
        acc = all;
      }
      if (lane == 0) {
        const long long id = arg_result(acc);
        *p.argmax = id;
        *tok_out = (uint32_t)id;
        if (out_ids) out_ids[step] = (uint32_t)id;
        *p.pos = pos + 1;
        *p.launch = launch + 1;  // every CTA read the launch count at its start
        *p.ticket = 0;
      }
    }
  }
  // after a failed wait, let every copy this CTA issued land before the CTA exits
  if (threadIdx.x == 0 && ld_volatile(p.err)) {
    for (int s = 0; s < NSLOT; s++) {
      if (!sm.issued[s]) continue;
      const long long t0 = clock64();
      while (!mbar_try_wait(&rg.full[s], (unsigned)(sm.issued[s] - 1) & 1u) && clock64() - t0 < WAIT_LIMIT) {
      }
    }
  }
  stamp(p, TL_STRIDE(p) - 1);
  stamp_sync(p, TL_STRIDE(p) - 4);
}

// Per-CTA tile tables, built once per context with the same row split the kernel
// uses: the tiles of every stage of every layer in consumption order.
__global__ void k_build_tiles(const Params *__restrict__ pp, int2 *tiles, int *ntiles, int max_tiles) {
  const Params &p = *pp;
  if (threadIdx.x != 0) return;
  const int cta = blockIdx.x;
  int nt = 0;
  const int spl = p.split ? 5 : 4;  // stages per layer, in the kernel's order
  for (int l = 0; l <= p.L; l++) {
    for (int sk = 0; sk < (l < p.L ? spl : 1); sk++) {
      const int kind = l == p.L ? ST_LM : (sk == 4 ? ST_DOWN2 : sk);
      int r0, r1;
      stage_rows(p, kind, l, cta, r0, r1);
      for (int r = r0; r < r1; r += p.tile_rows[kind]) {
        const int n = min(p.tile_rows[kind], r1 - r);
        if (nt < max_tiles) tiles[(size_t)cta * max_tiles + nt] = make_int2(r, (l << 16) | (kind << 12) | n);
        nt++;
      }
    }
  }
  ntiles[cta] = nt;
}

}  // namespace dk

// ---------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------
struct DecodeState {
  bool available = false;
  int dev_pos = 0;  // position the device counter holds once queued launches finish
  dk::Params *d_params = nullptr;  // for the tile-table builder
  dk::Params hp{};                 // the decode kernel's by-value parameter (constant bank)
  void *kernel = nullptr;
  size_t smem = 0;
  int grid = 0;
  unsigned *d_err = nullptr, *d_bar = nullptr, *d_ticket = nullptr, *d_attn_cnt = nullptr;
  int *d_pos = nullptr;
  int n_kv_heads = 0, n_heads = 0, n_layers = 0;
#ifdef SQ_DECODE_TIMELINE
  // profiling builds: SQ_DECODE_TIMELINE=<file> writes the stamps of the last launch
  unsigned long long *d_timeline = nullptr;
  unsigned long long *d_tile_tl = nullptr;
  const int2 *d_tiles = nullptr;
  int max_tiles = 0;
  int tl_stride = 0;
  std::string tl_path;
#endif
  std::vector<void *> allocs;
};

template <int T, int DPL, bool AQ = false>
static void *pick_kernel() {
  return (void *)dk::k_decode<T, DPL, AQ>;
}

static int nseg_for(int in_dim) {
  const int s = (in_dim + 2047) / 2048;
  for (int c : {1, 2, 4, 8})
    if (s <= c) return c;
  return 0;
}

int decode_prepare(sq_ctx *c) {
  const sq_model *m = c->m;
  const sq_llama_config &cf = m->lc;  // this rank's shard (the whole model on one GPU)
  auto *st = new DecodeState();
  c->dec = st;
  if (getenv("SQ_DISABLE_DECODE_KERNEL")) return SQ_OK;
  unsigned long long *boxes[8] = {};
  int tp_world = 1;
  if (m->tp_size > 1) {  // tensor parallel: the kernel exchanges partial sums through the peer mailboxes
    if (const char *v = getenv("SQB200_TP_DECODE"))
      if (strcmp(v, "op") == 0) return SQ_OK;  // the op-level step with its all-reduce kernels (A/B)
    tp_world = tp_decode_boxes(m->ar, boxes, 8);
    if (tp_world != m->tp_size) return SQ_OK;  // no peer mailboxes: the op-level step serves this model
  }
  const int E = cf.embed_dim, Q = cf.n_heads * cf.head_dim, KVd = cf.n_kv_heads * cf.head_dim, F = cf.ffn_dim;
  const int wt = cf.weight_type, bb = block_bytes(wt);
  // supported shapes: same type everywhere, rows multiple of 16 bytes, <= 8 segments, GQA group 4
  bool ok = m->out_type == wt && m->embd_type == wt && cf.n_blocks <= dk::MAX_LAYERS &&
            cf.n_heads == dk::GROUP * cf.n_kv_heads && (cf.head_dim == 64 || cf.head_dim == 128);
  // an FFN input wider than the staging buffer is taken in two parts of <= MAX_X
  const int split = F > dk::MAX_X, xa = split ? dk::MAX_X : F, xb = F - xa;
  const int nE = nseg_for(E), nQ = nseg_for(Q), nF = nseg_for(F), nFA = nseg_for(xa), nFB = split ? nseg_for(xb) : 1;
  ok = ok && nE && nQ && nFA && nFB && (split || nF);
  // W8A8 (Q8_0 activations) for Q8_0 / Q4_0 weights; BF16 weights keep f32 activations
  // under either setting, as the reference's BF16 linear does (matmul.rs:106-108)
  const bool aq = m->acts == SQ_ACTS_Q8 && wt != SQ_BF16;
  for (int d : {E, Q, xa, split ? xb : xa}) {
    ok = ok && d > 0 && (d / QK) % 8 == 0 && ((size_t)(d / QK) * bb) % 16 == 0;  // pairs, 16-byte rows and parts
    if (wt == SQ_BF16) ok = ok && d % 2048 == 0;  // BF16 lanes stripe whole 2048-element segments
  }
  const int rbE = E / QK * bb, rbQ = Q / QK * bb, rbF = F / QK * bb, rbFA = xa / QK * bb, rbFB = xb / QK * bb;
  auto rows_fit = [&](int rb, int mult) {
    int t = dk::SLOT / (rb * mult);
    if (t >= 2) t &= ~1;
    return t;
  };
  dk::Params h{};
  h.split = split;
  h.xa = xa;
  h.rb_FA = rbFA;
  h.rb_FB = rbFB;
  h.nseg_FA = nFA;
  h.nseg_FB = nFB;
  h.tile_rows[dk::ST_QKV] = rows_fit(rbE, 1);
  h.tile_rows[dk::ST_O] = rows_fit(rbQ, 1);
  h.tile_rows[dk::ST_GU] = rows_fit(rbE, 2);
  h.tile_rows[dk::ST_DOWN] = rows_fit(split ? rbFA : rbF, 1);
  h.tile_rows[dk::ST_LM] = rows_fit(rbE, 1);
  h.tile_rows[dk::ST_DOWN2] = split ? rows_fit(rbFB, 1) : 2;
  int slot_bytes = 0;
  for (int k = 0; k < 6; k++) {
    const int nseg = k == dk::ST_O ? nQ : (k == dk::ST_DOWN ? (split ? nFA : nF) : (k == dk::ST_DOWN2 ? nFB : nE));
    const int rb = k == dk::ST_O ? rbQ : (k == dk::ST_DOWN ? (split ? rbFA : rbF) : (k == dk::ST_DOWN2 ? rbFB : rbE));
    // segment partial sums of a tile (rows x segments) go through shared memory
    ok = ok && h.tile_rows[k] >= 2 && (nseg == 1 || h.tile_rows[k] * (k == dk::ST_GU ? 2 : 1) * nseg <= dk::MAX_TILE_ITEMS);
    if (k != dk::ST_DOWN2 || split) slot_bytes = std::max(slot_bytes, h.tile_rows[k] * rb * (k == dk::ST_GU ? 2 : 1));
  }
  h.slot_bytes = (slot_bytes + 127) & ~127;  // the largest tile; mbarriers after the ring stay 8-byte aligned
  int dev = m->device, nsm = 0;
  SQ_CUDA(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
  // residual rows per CTA live in one register per lane (and part sums in dpart[32]);
  // LM rows per CTA in shared memory
  ok = ok && (E + nsm - 1) / nsm <= 32 && (cf.vocab_size + nsm - 1) / nsm <= dk::MAX_LM_ROWS;
  ok = ok && std::max(std::max(E, Q), std::max(xa, xb)) <= dk::MAX_X;  // stage inputs fit the staging buffer
  if (!ok) return SQ_OK;  // the op-level path serves this model
  void *kern = nullptr;
  if (wt == SQ_Q8_0 && aq)
    kern = cf.head_dim == 64 ? pick_kernel<SQ_Q8_0, 2, true>() : pick_kernel<SQ_Q8_0, 4, true>();
  else if (wt == SQ_Q4_0 && aq)
    kern = cf.head_dim == 64 ? pick_kernel<SQ_Q4_0, 2, true>() : pick_kernel<SQ_Q4_0, 4, true>();
  else if (wt == SQ_Q8_0) kern = cf.head_dim == 64 ? pick_kernel<SQ_Q8_0, 2>() : pick_kernel<SQ_Q8_0, 4>();
  else if (wt == SQ_Q4_0) kern = cf.head_dim == 64 ? pick_kernel<SQ_Q4_0, 2>() : pick_kernel<SQ_Q4_0, 4>();
  else kern = cf.head_dim == 64 ? pick_kernel<SQ_BF16, 2>() : pick_kernel<SQ_BF16, 4>();
  h.tp_world = tp_world;
  h.tp_rank = m->tp_rank;
  h.vocab_local = cf.vocab_size;
  for (int r = 0; r < tp_world && r < 8; r++) h.tp_box[r] = boxes[r];
  h.L = cf.n_blocks;
  h.E = E;
  h.Q = Q;
  h.KVd = KVd;
  h.F = F;
  h.V = cf.vocab_size;
  h.H = cf.n_heads;
  h.KVH = cf.n_kv_heads;
  h.hd = cf.head_dim;
  h.max_ctx = c->max_ctx;
  h.G = nsm;
  h.nseg_E = nE;
  h.nseg_Q = nQ;
  h.nseg_F = nF;
  h.rb_E = rbE;
  h.rb_Q = rbQ;
  h.rb_F = rbF;
  // grouped long-context attention: ~128 positions a chunk, up to one item per CTA
  h.max_chunks = std::max(1, nsm / cf.n_kv_heads);
  h.eps = cf.rms_eps;
  h.attn_scale = 1.0f / sqrtf((float)cf.head_dim);
  h.embd = (const uint8_t *)m->embd;
  h.out_w = (const uint8_t *)m->out_w;
  h.out_norm = m->out_norm;
  h.cos_t = c->d_cos;
  h.sin_t = c->d_sin;
  h.kc = c->kc;
  h.vc = c->vc;
  h.hidden = c->hidden;
  h.qbuf = c->q;
  h.attn_out = c->attn;
  h.act = c->act;
  h.logits = c->logits;
  h.argmax = c->d_argmax;
  for (int l = 0; l < cf.n_blocks; l++) {
    const auto &Lw = m->layers[l];
    h.layers[l] = {(const uint8_t *)Lw.q, (const uint8_t *)Lw.k, (const uint8_t *)Lw.v, (const uint8_t *)Lw.o,
                   (const uint8_t *)Lw.gate, (const uint8_t *)Lw.up, (const uint8_t *)Lw.down, Lw.attn_norm,
                   Lw.ffn_norm};
  }
  auto alloc = [&](void **p, size_t bytes) -> cudaError_t {
    cudaError_t e = cudaMalloc(p, bytes);
    if (e == cudaSuccess) {
      st->allocs.push_back(*p);
      e = cudaMemset(*p, 0, bytes);
    }
    return e;
  };
  SQ_CUDA(alloc((void **)&h.attn_part, (size_t)cf.n_heads * h.max_chunks * (cf.head_dim + 2) * 4));
  SQ_CUDA(alloc((void **)&h.attn_cnt, (size_t)cf.n_blocks * cf.n_heads * 4));
  SQ_CUDA(alloc((void **)&h.hid_ll, (size_t)E * 8));
  SQ_CUDA(alloc((void **)&h.q_ll, (size_t)Q * 8));
  SQ_CUDA(alloc((void **)&h.kv_ll, (size_t)2 * KVd * 8));
  SQ_CUDA(alloc((void **)&h.attn_ll, (size_t)Q * 8));
  SQ_CUDA(alloc((void **)&h.act_ll, (size_t)F * 8));
  SQ_CUDA(alloc((void **)&h.launch, 4));
  {
    const unsigned one = 1;  // tags of launch 0 would match the zeroed words
    SQ_CUDA(cudaMemcpy(h.launch, &one, 4, cudaMemcpyHostToDevice));
  }
  SQ_CUDA(alloc((void **)&h.bar, 4));
  SQ_CUDA(alloc((void **)&h.ticket, 4));
  SQ_CUDA(alloc((void **)&h.err, 4));
  SQ_CUDA(alloc((void **)&h.arg_part, (size_t)nsm * sizeof(ArgState)));
  SQ_CUDA(alloc((void **)&h.pos, 4));
  SQ_CUDA(alloc((void **)&st->d_params, sizeof(dk::Params)));
  if (const char *v = getenv("SQ_TEST_DROP_EXCHANGE")) {  // failure-detection tests (see Params::drop_tag)
    const int n = atoi(v);
    if (n > 0) h.drop_tag = dk::mk_tag((unsigned)n, 0, dk::TG_POST_O);
  }
#ifdef SQ_DECODE_TIMELINE
  if (const char *tl = getenv("SQ_DECODE_TIMELINE")) {  // stage timestamps of profiling builds
    st->tl_path = tl;
    st->tl_stride = 8 * (5 * cf.n_blocks + 1) + 6;
    SQ_CUDA(alloc((void **)&st->d_timeline, (size_t)nsm * st->tl_stride * 8));
    h.timeline = st->d_timeline;
    h.tl_stride = st->tl_stride;
  }
#endif
  // tile tables: count pass, then fill (same row split as the kernel)
  SQ_CUDA(alloc((void **)&h.ntiles, (size_t)nsm * sizeof(int)));
  SQ_CUDA(cudaMemcpy(st->d_params, &h, sizeof(dk::Params), cudaMemcpyHostToDevice));
  dk::k_build_tiles<<<nsm, 32>>>(st->d_params, nullptr, h.ntiles, 0);
  SQ_CHECK_LAUNCH("build tiles");
  std::vector<int> counts(nsm);
  SQ_CUDA(cudaMemcpy(counts.data(), h.ntiles, nsm * sizeof(int), cudaMemcpyDeviceToHost));
  h.max_tiles = (*std::max_element(counts.begin(), counts.end()) + 1) & ~1;
  SQ_CUDA(alloc((void **)&h.tiles, (size_t)nsm * h.max_tiles * sizeof(int2)));
#ifdef SQ_DECODE_TIMELINE
  if (h.timeline) {
    SQ_CUDA(alloc((void **)&h.tile_tl, (size_t)nsm * h.max_tiles * 3 * 8));
    st->d_tile_tl = h.tile_tl;
    st->d_tiles = h.tiles;
    st->max_tiles = h.max_tiles;
  }
#endif
  SQ_CUDA(cudaMemcpy(st->d_params, &h, sizeof(dk::Params), cudaMemcpyHostToDevice));
  dk::k_build_tiles<<<nsm, 32>>>(st->d_params, h.tiles, h.ntiles, h.max_tiles);
  SQ_CHECK_LAUNCH("build tiles");
  SQ_CUDA(cudaDeviceSynchronize());
  const size_t smem = (size_t)dk::NSLOT * h.slot_bytes + (dk::NSLOT + 1) * sizeof(uint64_t) + sizeof(dk::Smem) +
                      (size_t)h.max_tiles * sizeof(int2);
  int smem_max = 0;
  SQ_CUDA(cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  if (smem > (size_t)smem_max) return SQ_OK;  // tile table too long: the op-level path serves this model
  SQ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 0;
  SQ_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, dk::NTHREADS, smem));
  if (per_sm < 1) return SQ_OK;
  st->d_err = h.err;
  st->d_bar = h.bar;
  st->d_ticket = h.ticket;
  st->d_attn_cnt = h.attn_cnt;
  st->n_kv_heads = cf.n_kv_heads;
  st->n_heads = cf.n_heads;
  st->n_layers = cf.n_blocks;
  st->d_pos = h.pos;
  st->hp = h;
  st->kernel = kern;
  st->smem = smem;
  st->grid = nsm;
  st->available = true;
  return SQ_OK;
}

bool decode_available(const sq_ctx *c) { return c->dec && c->dec->available; }

unsigned *decode_err_ptr(const sq_ctx *c) { return decode_available(c) ? c->dec->d_err : nullptr; }

bool decode_check_always(const sq_ctx *c) {
#ifdef SQ_DECODE_TIMELINE
  return c->dec && c->dec->d_timeline;  // the stamps of the last launch are written by decode_check
#else
  (void)c;
  return false;
#endif
}

__global__ void k_set_int(int *p, int v) { *p = v; }

int decode_launch(sq_ctx *c, uint32_t *d_tok, uint32_t *out_ids, int step) {
  DecodeState *st = c->dec;
  // the kernel reads the position from device memory and advances it itself; resync
  // only after prefill or reset moved the host's count
  if (st->dev_pos != c->seq_len) {
    k_set_int<<<1, 1, 0, c->stream>>>(st->d_pos, c->seq_len);
    SQ_CHECK_LAUNCH("decode pos");
    st->dev_pos = c->seq_len;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(st->grid);
  cfg.blockDim = dim3(dk::NTHREADS);
  cfg.dynamicSmemBytes = st->smem;
  cfg.stream = c->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void *args[] = {&st->hp, &d_tok, &d_tok, &out_ids, &step};
  SQ_CUDA(cudaLaunchKernelExC(&cfg, st->kernel, args));
  c->seq_len += 1;
  st->dev_pos += 1;
  return SQ_OK;
}

int decode_check(sq_ctx *c) {
  DecodeState *st = c->dec;
  if (!st || !st->available) return SQ_OK;
  unsigned err = 0;
  SQ_CUDA(cudaMemcpy(&err, st->d_err, 4, cudaMemcpyDeviceToHost));
#ifdef SQ_DECODE_TIMELINE
  if (st->d_timeline) {
    std::vector<unsigned long long> tl((size_t)st->grid * st->tl_stride);
    SQ_CUDA(cudaMemcpy(tl.data(), st->d_timeline, tl.size() * 8, cudaMemcpyDeviceToHost));
    if (FILE *f = fopen(st->tl_path.c_str(), "wb")) {
      const int hdr[2] = {st->grid, st->tl_stride};
      fwrite(hdr, sizeof hdr, 1, f);
      fwrite(tl.data(), 8, tl.size(), f);
      std::vector<unsigned long long> tt((size_t)st->grid * st->max_tiles * 3);
      if (st->d_tile_tl && cudaMemcpy(tt.data(), st->d_tile_tl, tt.size() * 8, cudaMemcpyDeviceToHost) == cudaSuccess) {
        fwrite(&st->max_tiles, 4, 1, f);
        fwrite(tt.data(), 8, tt.size(), f);
        std::vector<int2> tb((size_t)st->grid * st->max_tiles);
        if (cudaMemcpy(tb.data(), st->d_tiles, tb.size() * sizeof(int2), cudaMemcpyDeviceToHost) == cudaSuccess)
          fwrite(tb.data(), sizeof(int2), tb.size(), f);
      }
      fclose(f);
    }
  }
#endif
  if (err) {
    // reset the kernel's flag and counters so the context stays usable
    cudaMemset(st->d_err, 0, 4);
    cudaMemset(st->d_bar, 0, 4);
    cudaMemset(st->d_ticket, 0, 4);
    cudaMemset(st->d_attn_cnt, 0, (size_t)st->n_heads * st->n_layers * 4);
    st->dev_pos = -1;  // force a position resync
    return fail(SQ_ERR_TIMEOUT, "decode kernel: a bounded wait expired (code " + std::to_string(err) + ")");
  }
  return SQ_OK;
}

void decode_release(sq_ctx *c) {
  if (!c->dec) return;
  for (void *p : c->dec->allocs) cudaFree(p);
  delete c->dec;
  c->dec = nullptr;
}

}  // namespace sq
