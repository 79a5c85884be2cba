// ops.cuh — internal launchers of the op-level kernels (used by the C ABI in ops.cu
// and by the model orchestration in host/model.cpp). No validation here: callers
// validate shapes first.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace sq {

// out[m][out_dim] = x[m][in_dim] @ w; acts_q8 uses `xq` (m*in/32 Q8_0 blocks) when non-null.
// f32 activations with m >= 2 run the tiled GEMM; `ws` (ws_floats floats, may be null)
// lets it split K when the output tiles alone would not cover the SMs.
cudaError_t launch_linear(cudaStream_t s, const float *x, int m, int in_dim, const void *w, int wtype,
                          int out_dim, float *y, int acts_q8, void *xq, float *ws = nullptr, size_t ws_floats = 0);
// The tiled GEMM itself (gemm.cu): y[m][N] = x[m][K] @ w^T, native weight rows.
cudaError_t launch_gemm_f32w(cudaStream_t s, const float *x, int m, int K, const void *w, int wtype, int N, float *y,
                             float *ws, size_t ws_floats);
// A fused single-row matvec (one launch of the streaming matvec): up to three
// matrices of one type and input width over one input row; the input optionally
// RMS-normalised (weight norm_w; (x * w) * (1/rms), one rounding from the reference's
// (x * w) / rms) or formed as
// silu(x) * xu; each output optionally added to a residual row (may be the output).
struct MvArgs {
  const float *x;       // input row [in_dim]
  const float *xu;      // optional: input = silu(x) * xu
  const float *norm_w;  // optional: input = (x * norm_w) / sqrt(mean(x^2) + eps)
  float eps;
  int in_dim;
  int n;  // matrices (1..3)
  const uint8_t *w[3];
  int out_dim[3];
  float *y[3];
  const float *res[3];  // optional residual rows: y[r] = res[r] + dot
  int gate_act;         // n == 2 (gate, up; same rows, no residual): y[1] = silu(gate . x) * (up . x); y[0] unused
  int test_skip;        // failure-detection tests only (set by the launcher): k > 0 = tile k - 1 is never copied
};
bool matvec_fused_ok(const MvArgs &a, int wtype);
// pdl: launched with programmatic stream serialization (the kernel streams its first
// weight tiles while the previous kernel finishes; see pdl_enabled()).
cudaError_t launch_matvec_fused(cudaStream_t s, const MvArgs &a, int wtype, bool pdl = false);
// Programmatic dependent launches for the one-row decode step (SQB200_PDL=0 turns them off).
bool pdl_enabled();

// Tensor-core GEMM (gemm_tc.cu) for BF16, Q8_0 and Q4_0 weight rows: the f32
// activations are split into three bf16 terms in `ws` (3*m*K/2 floats, then split-K
// partials). Supported when m >= 2, K % 16 == 0 (quantized: K % 256 == 0 and 16-byte
// rows), x and w 16-byte aligned, ws 256-byte aligned and large enough.
bool gemm_tc_supported(int m, int K, const float *x, const void *w, int wtype, const float *ws, size_t ws_floats);
cudaError_t launch_gemm_tc(cudaStream_t s, const float *x, int m, int K, const void *w, int wtype, int N, float *y,
                           float *ws, size_t ws_floats);
// Non-zero when a bounded wait of a tensor-core kernel gave up (read after a sync).
unsigned gemm_tc_status(bool clear);
// Non-zero when a bounded wait of the streaming matvec (k_matvec) gave up (read after a sync).
unsigned matvec_status(bool clear);
unsigned *mv_err_ptr();  // device address of that error word (current device)
// One launch that copies the argmax and up to four error words (null: skipped, 0)
// into out[0..4], so a call ends with one small device-to-host copy.
cudaError_t launch_collect_status(cudaStream_t s, const long long *argmax, const unsigned *e0, const unsigned *e1,
                                  const unsigned *e2, const unsigned *e3, unsigned long long *out);
// Both words of the current device, read (and cleared when `clear`) after a sync:
// SQ_OK, or SQ_ERR_TIMEOUT with a message naming `what` and the kernels that gave up.
int device_wait_status(bool clear, const char *what);
unsigned *tc_err_ptr();  // device address of that error word (current device)
// False when SQB200_GEMM=simt selects the CUDA-core GEMM for every weight type.
bool gemm_tc_enabled();
// Tensor-core causal attention (attention_tc.cu), head_dim 64, seq_q >= 64: the same
// arguments as launch_sdpa plus a workspace of attn_tc_workspace_bytes() bytes for the
// bf16 terms of q, k and v.
size_t attn_tc_workspace_bytes(int seq_q, int seq_k, int n_heads, int n_kv_heads);
bool attn_tc_supported(int seq_q, int seq_k, int n_heads, int n_kv_heads, int head_dim, long long kps, long long khs,
                       const void *q, const void *k, const void *v, size_t ws_bytes);
cudaError_t launch_attn_tc(cudaStream_t s, const float *q, const float *k, const float *v, float *out, int seq_q,
                           int seq_k, int n_heads, int n_kv_heads, int head_dim, long long kps, long long khs,
                           void *ws, size_t ws_bytes);
// The same GEMM on activation terms already in ws ([3][m][K] bf16 at its start), e.g.
// written by launch_rms_norm_terms / launch_silu_mul_terms / launch_split_terms.
cudaError_t launch_gemm_tc_terms(cudaStream_t s, int m, int K, const void *w, int wtype, int N, float *y, float *ws,
                                 size_t ws_floats);
// The same for nmat (1-3) weight matrices that share the input terms (q / k / v,
// gate / up): one launch over all their tiles when the kernel takes them without a K
// split, else one launch per matrix.
cudaError_t launch_gemm_tc_terms_multi(cudaStream_t s, int m, int K, int nmat, const void *const *w, int wtype,
                                       const int *N, float *const *y, float *ws, size_t ws_floats);
cudaError_t launch_split_terms(cudaStream_t s, const float *x, int m, int K, float *ws);
// RMSNorm / SiLU.mul writing only the three bf16 terms of their output ([3][rows][dim]).
bool rms_norm_terms_ok(const float *x, const float *w, int dim);
cudaError_t launch_rms_norm_terms(cudaStream_t s, const float *x, const float *w, void *terms, int rows, int dim,
                                  float eps);
// The residual add x += add first (written back to x), then the same norm of the sum.
cudaError_t launch_add_rms_norm_terms(cudaStream_t s, float *x, const float *add, const float *w, void *terms,
                                      int rows, int dim, float eps);
cudaError_t launch_silu_mul_terms(cudaStream_t s, const float *g, const float *u, void *terms, size_t n);
cudaError_t launch_quantize_q8_0(cudaStream_t s, const float *x, size_t n, void *out);
cudaError_t launch_embed(cudaStream_t s, const uint32_t *tokens, int n, const void *w, int wtype,
                         int embed_dim, int vocab, float *out);
cudaError_t launch_rms_norm(cudaStream_t s, const float *x, const float *w, float *y, int rows, int dim,
                            float eps);
// RoPE with on-device double-precision sin/cos of pos*inv_freq[j].
cudaError_t launch_rope_rows(cudaStream_t s, float *x, int seq, int row_dim, int base_pos,
                             const float *inv_freq, int half);
// RoPE from a host-computed (C library sinf/cosf) table [n_pos][half].
// pos_dev (optional): base_pos is read from the device instead (CUDA-graph replay).
cudaError_t launch_rope_rows_table(cudaStream_t s, float *x, int seq, int row_dim, int base_pos,
                                   const float *cos_t, const float *sin_t, int half, const int *pos_dev = nullptr);
cudaError_t launch_silu(cudaStream_t s, float *x, size_t n);
cudaError_t launch_mul(cudaStream_t s, const float *a, const float *b, float *out, size_t n);
cudaError_t launch_add(cudaStream_t s, float *a, const float *b, size_t n);
cudaError_t launch_silu_mul(cudaStream_t s, const float *g, const float *u, float *out, size_t n);
cudaError_t launch_dequantize(cudaStream_t s, const void *blocks, int wtype, size_t n, float *out);
// Two-stage greedy argmax; `partials` holds at least argmax_partials(n) states
// (sizeof(ArgState) = 24 bytes each).
int argmax_partials(size_t n);
cudaError_t launch_argmax(cudaStream_t s, const float *x, size_t n, void *partials, long long *out);
// Tensor parallel: the argmax state of a vocabulary shard starting at `offset`
// (argmax_state_bytes() bytes), and the fold of n shard states in shard order.
cudaError_t launch_argmax_state(cudaStream_t s, const float *x, size_t n, long long offset, void *partials,
                                void *state);
cudaError_t launch_argmax_fold(cudaStream_t s, const void *states, int n, long long *out);
size_t argmax_state_bytes();

// Causal GQA attention. q/out rows: [seq_q][n_heads*hd]; key s of kv head g lives at
// k + s*k_pos_stride + g*k_head_stride (same for v). `part` is scratch for split-KV
// partials of sdpa_partials_floats(...) floats (may be null when n_split == 1).
constexpr long long SDPA_MAX_ROW_SPLITS = 1024;
int sdpa_num_splits(int seq_q, int seq_k, int n_heads);
size_t sdpa_partials_floats(int seq_q, int n_heads, int head_dim, int n_split);
size_t sdpa_max_partials_floats(int head_dim);
// pos_dev (optional): seq_k is *pos_dev + seq_q, read on the device (CUDA-graph replay).
cudaError_t launch_sdpa(cudaStream_t s, const float *q, const float *k, const float *v, float *out,
                        int seq_q, int seq_k, int n_heads, int n_kv_heads, int head_dim,
                        long long k_pos_stride, long long k_head_stride, int n_split, float *part,
                        const int *pos_dev = nullptr, int *split_cnt = nullptr, bool pdl = false);
// split_cnt (optional, seq_q * n_heads ints, zero before the first call): the last CTA of
// a query row to finish merges the splits itself (and re-zeroes its counter) instead
// of a separate combine launch; same arithmetic, same order.

}  // namespace sq

namespace sq {
// KV append into the head-major cache [n_kv][max_ctx][hd] of one layer:
// cache[g][pos + r][d] = src[r][g*hd + d] for r < n (kv_cache.rs:38-53 semantics).
cudaError_t launch_kv_append(cudaStream_t s, const float *k, const float *v, float *kc, float *vc, int n,
                             int n_kv, int hd, int pos, int max_ctx, const int *pos_dev = nullptr);
// RoPE of q (in place) and k rows from the cos/sin table, then the rotated K and the V
// rows appended to the cache, in one launch (q: [n][Q], k / v: [n][KVd]).
cudaError_t launch_rope_append(cudaStream_t s, float *q, const float *k, const float *v, float *kc, float *vc,
                               int n, int Q, int KVd, int hd, int pos, int max_ctx, const float *cos_t,
                               const float *sin_t, const int *pos_dev = nullptr, bool pdl = false);
// *p += v / *p = v (the device position counter of a replayed decode step)
cudaError_t launch_add_int(cudaStream_t s, int *p, int v);
cudaError_t launch_set_int(cudaStream_t s, int *p, int v);
// dst_tok[0] = (uint32)argmax[0]; out_ids[step] = dst_tok[0]  (device-side token feedback)
cudaError_t launch_feedback(cudaStream_t s, const long long *argmax, uint32_t *tok, uint32_t *out_ids, int step);
}  // namespace sq
