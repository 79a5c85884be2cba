/*
 * oracle.h — CPU restatement of squirrel-rs's Llama token loop, used ONLY as the
 * parity checker (tests/, __graft_entry__.smoke(), bench.py's cpu_baseline and
 * --impl reference arms). It is test infrastructure, never the product path.
 *
 * What it restates (paths are relative to the squirrel-rs crate):
 *   - x86_64 path of the reference (W8A32 / W4A32 / BF16 with f32 activations):
 *     src/kernels/dot_prod.rs:86-96, :255-270, :464-472, src/kernels/matmul.rs:102-128
 *   - aarch64 activation-quantization semantics, scalar twins (W8A8 / W4A8):
 *     src/kernels/dot_prod.rs:21-31 (quantizer), :378-403 (integer block dots),
 *     src/ops/linear.rs:73-158 (shared quantization of one input)
 *   - every other op on the path: rms_norm.rs:40-74, rope.rs:7-36, softmax.rs:4-27,
 *     attention.rs:11-70, silu.rs:4-8, sigmoid.rs:2-9, elementwise_{add,mul}.rs,
 *     samplers/greedy.rs:6-15, ops/embedding.rs:10-52
 *   - model orchestration: models/llama/{config,weights,layers,model}.rs,
 *     models/common/kv_cache.rs, text_generator.rs:58-97
 *   - GGUF reading: file_parser/{gguf_file,gguf_header,gguf_metadata_value,
 *     gguf_tensor_info,ggml_type}.rs
 *
 * Build: gcc -O2 -ffp-contract=off -fopenmp (Rust never contracts a*b+c into an
 * FMA, and each output row's summation order here equals the reference's).
 * Transcendentals are glibc's expf/sinf/cosf/powf/sqrtf, which is what Rust's
 * f32::{exp,sin_cos,powf,sqrt} call on x86_64-linux-gnu.
 *
 * Parity status: op-level functions are pinned by the reference's own unit-test
 * vectors (tests/test_oracle_pins.py). End-to-end output is NOT pinned by the
 * reference (it has no golden files and cannot be compiled here: no Rust
 * toolchain); end-to-end fixtures are this oracle's own output.
 */
#ifndef SQ_ORACLE_H
#define SQ_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML type ids (file_parser/ggml_type.rs:8-41). */
enum { OR_F32 = 0, OR_Q4_0 = 2, OR_Q8_0 = 8, OR_BF16 = 30 };
/* KernelError (kernels/kernel_error.rs:2-7) mapped to ints, 0 = Ok. */
enum { OR_OK = 0, OR_SHAPE = 1, OR_INVALID_TYPE = 2, OR_EMPTY = 3, OR_ALIGN = 4, OR_IO = 5 };

/* half / bf16 conversions (crate `half` 2.7.1 semantics: exact widening, RNE narrowing). */
float or_f16_to_f32(uint16_t h);
uint16_t or_f32_to_f16(float f);
float or_bf16_to_f32(uint16_t b);

/* Block sizes in bytes per 32 elements for a GGML type, 0 if unsupported. */
size_t or_block_bytes(int type);

/* WeightBlock::dequantize_into (dot_prod.rs:409-414, 440-446, 524-528). */
void or_dequantize(int type, const uint8_t *blocks, size_t nblocks, float *out);
/* quantize_row_q8_0_scalar (dot_prod.rs:21-31); n multiple of 32. */
void or_quantize_row_q8_0(const float *src, size_t n, uint8_t *out);

/* Row dots. */
float or_dot_f32_q8_0(const float *a, const uint8_t *b, size_t nblocks);  /* :86-96 */
float or_dot_f32_q4_0(const float *a, const uint8_t *b, size_t nblocks);  /* :255-270 */
float or_dot_f32_bf16(const float *a, const uint8_t *b, size_t nblocks);  /* :464-472 */
float or_dot_q8_0_q8_0(const uint8_t *a, const uint8_t *b, size_t nblocks); /* :378-388 */
float or_dot_q8_0_q4_0(const uint8_t *a, const uint8_t *b, size_t nblocks); /* :391-403 */
float or_dot_f32_f32(const float *a, const float *b, size_t n);            /* :540-549 */

/* linear: out[m][out_dim] = in[m][in_dim] @ w (out_dim rows of in_dim/32 blocks).
 * acts_q8 = 0: f32 activations (x86 path); 1: Q8_0-quantized activations
 * (aarch64 scalar semantics; BF16 ignores it, ops/linear.rs:34). */
int or_linear(const float *in, int m, int in_dim, const uint8_t *w, int type, int out_dim,
              float *out, int acts_q8, int nthreads);

int or_rms_norm(const float *in, const float *w, float *out, int rows, int dim, float eps);
int or_rms_norm_inplace(float *x, const float *w, int rows, int dim, float eps);
int or_rope_rows(float *x, int seq, int row_dim, int base_pos, const float *inv_freq, int half);
int or_softmax(const float *a, float *out, int n);
int or_sdpa(const float *q, const float *k, const float *v, float *out, int seq_q, int seq_k,
            int n_heads, int n_kv_heads, int head_dim, int nthreads);
float or_sigmoid(float x);
void or_silu(float *x, int n);
int or_mul(const float *a, const float *b, float *out, int n);
int or_add_inplace(float *a, const float *b, int n);
/* GreedySampler::sample (greedy.rs:6-15): Iterator::max_by with partial_cmp, Equal on NaN. */
int64_t or_greedy(const float *logits, size_t n);
int or_embed(const uint32_t *tokens, int n, const uint8_t *w, int type, int embed_dim, int vocab,
             float *out);
/* compute_rope_inv_freq (config.rs:83-127). */
void or_rope_inv_freq(int head_dim, float base, float factor, float low, float high,
                      float orig_ctx, float *out);

/* ---- model level ---- */
typedef struct or_model or_model;
typedef struct or_ctx or_ctx;

typedef struct {
    int n_blocks, embed_dim, ffn_dim, n_heads, n_kv_heads, head_dim, vocab_size, context_length;
    float rope_base, rms_eps;
    uint32_t bos_token_id, eos_token_id;
    int weight_type; /* type of the projection weights (attn_q of block 0) */
} or_config;

/* Load a GGUF (llama arch). acts_q8 selects the activation scheme for Q8_0/Q4_0. */
or_model *or_model_load(const char *path, int acts_q8, int *status);
void or_model_free(or_model *m);
void or_model_config(const or_model *m, or_config *out);
const float *or_model_inv_freq(const or_model *m);
or_ctx *or_ctx_new(const or_model *m);
void or_ctx_free(or_ctx *c);
void or_ctx_reset(or_ctx *c);
int or_ctx_seq_len(const or_ctx *c);
/* Model::forward (model.rs:45-97). */
int or_forward(const or_model *m, or_ctx *c, const uint32_t *ids, int n, int nthreads);
const float *or_ctx_logits(const or_ctx *c);
/* TextTokenGenerator::generate with SQUIRREL_IGNORE_EOS semantics when ignore_eos != 0
 * (text_generator.rs:58-97), token ids in and out; step_ms may be NULL.
 * Returns the number of generated tokens, or a negative status. If logits_out is
 * non-NULL it receives the logits of every step, [max_tokens][vocab]. */
int or_generate(const or_model *m, const uint32_t *prompt, int n_prompt, int max_tokens,
                int ignore_eos, uint32_t *out_ids, double *step_ms, float *logits_out,
                int nthreads);

#ifdef __cplusplus
}
#endif
#endif
