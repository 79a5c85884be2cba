/*
 * squirrel_cuda.h — C ABI of the B200 (sm_100a) implementation of squirrel-rs's
 * Llama token loop. Plain pointers and sizes only; no torch or CUDA types in the
 * signatures (a stream is passed as `void*`, a cudaStream_t; NULL = the legacy
 * default stream).
 *
 * Two levels, both drop-ins for the reference's Rust interfaces (paths relative
 * to the squirrel-rs crate):
 *   - op level  : replaces the `src/ops` free functions (and the `src/kernels`
 *                 they dispatch to). Arguments are DEVICE pointers; calls are
 *                 asynchronous on `stream`; shapes are validated on the host
 *                 before any launch, with the reference's error kinds.
 *   - model level: replaces `Llama3_2` / `ModelContext` / `TextTokenGenerator`
 *                 internals behind `trait Model` (models/common/model.rs:6-26).
 *                 Host pointers; one sync point per forward (the argmax id).
 *
 * Status codes: 0 = Ok; 1-4 mirror `KernelError` (kernels/kernel_error.rs:2-7).
 * Every non-zero return also sets a message readable with sq_last_error().
 */
#ifndef SQUIRREL_CUDA_H
#define SQUIRREL_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status ---------------------------------------------------------------- */
enum {
    SQ_OK = 0,
    SQ_ERR_SHAPE = 1,        /* KernelError::ShapeMismatch */
    SQ_ERR_INVALID_TYPE = 2, /* KernelError::InvalidType */
    SQ_ERR_EMPTY = 3,        /* KernelError::EmptyInput */
    SQ_ERR_ALIGN = 4,        /* KernelError::TensorAlignmentError */
    SQ_ERR_ARG = 5,          /* NULL pointer or out-of-range argument (no Rust analogue) */
    SQ_ERR_IO = 6,           /* GGUF file could not be read (std::io::Error, gguf_file.rs:22-35) */
    SQ_ERR_CONFIG = 7,       /* LLMError::InvalidConfig / InvalidWeights (models/common/error.rs:5-10) */
    SQ_ERR_CUDA = 16,        /* CUDA runtime error */
    SQ_ERR_NCCL = 17,        /* NCCL error (tensor-parallel contexts) */
    SQ_ERR_TIMEOUT = 18,     /* a bounded device-side wait gave up */
    SQ_ERR_CAPACITY = 19     /* KV cache of the context is full */
};

/* GGML type ids (file_parser/ggml_type.rs:8-41); the kernels take these four. */
enum { SQ_F32 = 0, SQ_Q4_0 = 2, SQ_Q8_0 = 8, SQ_BF16 = 30 };

/* Activation scheme of the Q8_0 / Q4_0 projections (ops/linear.rs:14-37):
 *  SQ_ACTS_F32: f32 activations against dequantized weights — the reference's
 *               x86_64 path and its SQUIRREL_F32_ACTS=1 ablation (W8A32 / W4A32);
 *  SQ_ACTS_Q8 : activations quantized to Q8_0 once per input (quantize_row_q8_0,
 *               dot_prod.rs:10-31), integer block dots (dot_prod.rs:378-403) —
 *               the reference's aarch64 default (W8A8 / W4A8).
 * BF16 weights always use f32 activations (ops/linear.rs:34). */
enum { SQ_ACTS_F32 = 0, SQ_ACTS_Q8 = 1 };

/* Message of the last failing call on this thread ("" if none). */
const char *sq_last_error(void);
/* Library build string (arch, version). */
const char *sq_version(void);

/* Bounded-wait status of the current device. Every device-side wait in this
 * library gives up after a time limit instead of hanging. The model-level calls
 * (sq_forward, sq_decode_steps, sq_generate) check this themselves and return
 * SQ_ERR_TIMEOUT. Op-level calls are asynchronous and cannot: a wait that expired
 * inside sq_linear / sq_linear_shared (the streaming matvec, m = 1) or sq_linear /
 * sq_sdpa_cached (the tensor-core GEMM and attention, m >= 2) is recorded in a word
 * of the device. After synchronizing the stream, this returns SQ_OK, or
 * SQ_ERR_TIMEOUT when such a wait expired since the record was last cleared (the
 * outputs of the calls since then are not valid); `clear` != 0 resets the record.
 * The record covers every stream and context of the device. No counterpart in the
 * reference, whose CPU kernels cannot time out (kernels/kernel_error.rs:2-7). */
int sq_wait_status(int clear);

/* ---- op level (device pointers; async on stream) ---------------------------- */

/* ops/linear.rs:26-37 `linear`: output[m][out_dim] = input[m][in_dim] @ weight,
 * weight = out_dim rows of in_dim/32 blocks of `wtype` in native GGUF layout. */
int sq_linear(void *stream, const float *input, int m, int in_dim, const void *weight, int wtype,
              int out_dim, float *output, int acts);

/* ops/linear.rs:73-168 `linear_shared`: n projections of one input (Q/K/V or
 * gate/up); under SQ_ACTS_Q8 the input is quantized once into `act_scratch`
 * (m * in_dim/32 * 34 bytes of device memory, the reference's `act_q`), which
 * may be NULL under SQ_ACTS_F32. All weights must share `wtype`. */
int sq_linear_shared(void *stream, const float *input, int m, int in_dim, int n,
                     const void *const *weights, const int *out_dims, int wtype,
                     float *const *outputs, int acts, void *act_scratch);

/* ops/embedding.rs:10-52 `embed`: out[t] = dequant(weight row tokens[t]). */
int sq_embed(void *stream, const uint32_t *tokens, int n_tokens, const void *weight, int wtype,
             int embed_dim, int vocab, float *out);

/* ops/rms_norm.rs:13-43 `rms_norm` and :50-66 `rms_norm_inplace` (rows of dim). */
int sq_rms_norm(void *stream, const float *input, const float *weight, float *output, int rows,
                int dim, float eps);
int sq_rms_norm_inplace(void *stream, float *x, const float *weight, int rows, int dim, float eps);

/* ops/rope.rs:6-32 `rope_rows`: row i rotated at position base_pos + i, interleaved
 * pairs (kernels/rope.rs:7-36); inv_freq is a device array of `half` floats. */
int sq_rope_rows(void *stream, float *x, int seq, int row_dim, int base_pos, const float *inv_freq,
                 int half);

/* ops/sdpa.rs:8-38 `sdpa_cached`: causal GQA attention of q [seq_q][n_heads*hd]
 * against k/v [seq_k][n_kv_heads*hd]; out like q. */
int sq_sdpa_cached(void *stream, const float *q, const float *k, const float *v, float *out,
                   int seq_q, int seq_k, int n_heads, int n_kv_heads, int head_dim);

/* ops/silu.rs:4-8, ops/elementwise_mul.rs:8-22, ops/elementwise_add.rs:8-15. */
int sq_silu(void *stream, float *x, size_t n);
int sq_elementwise_mul(void *stream, const float *a, const float *b, float *out, size_t n);
int sq_elementwise_add(void *stream, float *a, const float *b, size_t n);
/* silu(gate) * up in one pass (layers.rs:73-74 fused): out may alias gate. */
int sq_silu_mul(void *stream, const float *gate, const float *up, float *out, size_t n);

/* kernels/dot_prod.rs:10-31 `quantize_row_q8_0`: n f32 -> n/32 Q8_0 blocks (bit-exact). */
int sq_quantize_row_q8_0(void *stream, const float *src, size_t n, void *out_blocks);
/* WeightBlock::dequantize_into (dot_prod.rs:409-414, 440-446, 524-528), bit-exact. */
int sq_dequantize(void *stream, const void *blocks, int wtype, size_t n_elems, float *out);
/* samplers/greedy.rs:6-15 `GreedySampler::sample`: index of the max; ties and NaN
 * resolve like Iterator::max_by with partial_cmp (the later element wins). */
int sq_argmax(void *stream, const float *logits, size_t n, int64_t *out_index);

/* No counterpart in the reference. sq_argmax without any device allocation, for
 * callers that must not allocate device memory on the call path: sq_argmax takes
 * its per-chunk partial states from the stream-ordered pool (cudaMallocAsync) on
 * every call, which can fail with out-of-memory when a caller has sized its KV
 * caches and buffers to fill the GPU, and a caller that budgets device memory up
 * front cannot allow it. This variant keeps the partial states in a fixed 96 KiB
 * buffer of the library's static device memory and returns the same index as
 * sq_argmax (same kernels).
 *   - n up to SQ_ARGMAX_NOALLOC_MAX_N elements; larger n fails with SQ_ERR_ARG
 *     before any launch (use sq_argmax for those).
 *   - The buffer's device address is looked up on the first call on each device
 *     (with that device current); make that first call before capturing the
 *     stream into a CUDA graph.
 *   - All calls on one device share the buffer: calls that can overlap on the
 *     device (unordered streams, concurrent host threads) race and may return a
 *     wrong index. Order them, e.g. on one stream. */
#define SQ_ARGMAX_NOALLOC_MAX_N (1u << 24)
int sq_argmax_noalloc(void *stream, const float *logits, size_t n, int64_t *out_index);

/* ---- model level (host pointers) ------------------------------------------------ */

typedef struct sq_model sq_model;
typedef struct sq_ctx sq_ctx;

/* models/llama/config.rs:9-27 LlamaConfig (without the inv_freq table). */
typedef struct {
    int n_blocks, embed_dim, ffn_dim, n_heads, n_kv_heads, head_dim, vocab_size, context_length;
    float rope_base, rms_eps;
    uint32_t bos_token_id, eos_token_id;
    int weight_type; /* GGML type of the projection weights */
    /* llama3 RoPE scaling (config.rs:83-127 defaults: 32, 1, 4, 8192) */
    float rope_factor, rope_low_freq, rope_high_freq, rope_orig_ctx;
} sq_llama_config;

/* Upload path used by the reference's own GGUF parser (file_parser stays on the
 * host): create, upload each tensor in its native block layout, finalize. Names
 * follow models/llama/weights.rs:69-89 ("blk.{i}.attn_q.weight", ...); a missing
 * "output.weight" falls back to "token_embd.weight" (tied, weights.rs:89).
 * dims are the GGUF ne[] (ne[0] = in_dim). */
int sq_model_create(const sq_llama_config *cfg, int device, int acts, sq_model **out);
int sq_model_upload_tensor(sq_model *m, const char *name, int ggml_type, const uint64_t *dims,
                           int n_dims, const void *host_data, size_t nbytes);
int sq_model_finalize(sq_model *m);
/* Convenience: GGUFFile::from_file + LlamaConfig::from_gguf + upload, in one call. */
int sq_model_load_gguf(const char *path, int device, int acts, sq_model **out);
int sq_model_config(const sq_model *m, sq_llama_config *out);
void sq_model_free(sq_model *m);

/* Model::new_context (model.rs:36-43): KV cache for max_ctx positions (0 = min(context_length, 8192)). */
int sq_ctx_create(sq_model *m, int max_ctx, sq_ctx **out);
void sq_ctx_free(sq_ctx *c);
/* ModelContext::reset_cache (context.rs:25-27): forget positions, keep memory. */
int sq_ctx_reset(sq_ctx *c);
int sq_ctx_seq_len(const sq_ctx *c, int *out);
/* Model::forward (model.rs:45-97) + GreedySampler on the device: consumes n token
 * ids (prefill when n > 1), appends them to the KV cache, leaves the last row's
 * logits on the device and returns the greedy id in *out_argmax (may be NULL). */
int sq_forward(sq_ctx *c, const uint32_t *ids, size_t n, uint32_t *out_argmax);
/* ModelContext::logits (context.rs:20-22): copy the last logits to host. */
int sq_ctx_logits(sq_ctx *c, float *out, size_t n);
/* TextTokenGenerator::generate (text_generator.rs:38-101) on token ids: prefill the
 * prompt, then greedy steps until max_tokens or EOS (unless ignore_eos). out_ids
 * gets the generated ids, step_ms (optional) the host-measured ms per step. */
int sq_generate(sq_ctx *c, const uint32_t *prompt, size_t n_prompt, int max_tokens, int ignore_eos,
                uint32_t *out_ids, float *step_ms, int *n_out);
/* n_steps greedy decode steps chained on the device (each step's argmax feeds the
 * next), no host round trip between steps; the ids land in out_ids (host). The
 * context must hold at least one position (a prior sq_forward). */
int sq_decode_steps(sq_ctx *c, int n_steps, uint32_t *out_ids);
/* ---- tensor parallelism (several GPUs, one process per GPU) -----------------------
 * No counterpart in the reference (a CPU engine): the multi-GPU form of the model
 * level above, Megatron column/row sharding with an all-reduce after the O and down
 * projections and a greedy argmax across the vocabulary shards. Every rank makes
 * the same calls in the same order (sq_forward, sq_decode_steps, sq_generate,
 * sq_ctx_logits, sq_tp_recover are collective); each rank's result is the whole
 * model's. Rank 0 makes the id with sq_nccl_unique_id and shares its bytes with
 * the other ranks (e.g. over torch.distributed). NCCL is loaded at first use.
 * Decode rows run on the persistent decode kernel, one launch a token on every rank:
 * the O and down projections store their partial sums into every rank's mailbox
 * (NVLink peer memory, plain stores) and each CTA sums its own hidden rows over the
 * ranks in rank order with the residual add; the greedy argmax folds the ranks'
 * states the same way. SQB200_TP_DECODE=op (read when a context is created) runs
 * the op-level step instead, whose all-reduces use a one-shot peer-memory kernel,
 * or NCCL's with SQB200_TP_ALLREDUCE=nccl (read when the model is created). Prefill
 * rows, and groups whose GPUs cannot map each other's memory, use NCCL's.
 * Contexts of one tensor-parallel model must not run concurrently. */
/* ncclGetUniqueId into out (n >= 128 bytes). */
int sq_nccl_unique_id(void *out, size_t n);
/* After SQ_ERR_TIMEOUT on any rank (a peer's partial sum did not arrive in time,
 * e.g. because a rank stopped issuing steps), the ranks' all-reduce sequence
 * numbers may differ. Once every rank has stopped issuing work, every rank calls
 * this (collective, over NCCL): it clears the mailboxes (the all-reduce's and the
 * decode kernel's exchange words), sequence numbers and error word. Contexts must then be reset (sq_ctx_reset):
 * their KV cache past the last good position is undefined. SQ_OK without effect for
 * a model on one GPU or one on NCCL's all-reduce. */
int sq_tp_recover(sq_model *m);
/* sq_model_create / sq_model_load_gguf as rank tp_rank of tp_size GPUs. n_heads,
 * n_kv_heads, vocab_size and ffn_dim/32 must divide by tp_size. */
int sq_model_create_tp(const sq_llama_config *cfg, int device, int acts, int tp_rank, int tp_size,
                       const void *nccl_id, sq_model **out);
int sq_model_load_gguf_tp(const char *path, int device, int acts, int tp_rank, int tp_size, const void *nccl_id,
                          sq_model **out);
/* The shard of one GGUF tensor that rank tp_rank holds (host memory, no GPU):
 * attn_q/k/v, ffn_gate/up and output keep their rank's rows; attn_output and
 * ffn_down keep their rank's whole blocks of every row; everything else is copied.
 * dst == NULL only reports out_dims / out_bytes. */
int sq_tp_shard_tensor(const char *name, int ggml_type, const uint64_t *dims, int n_dims, int tp_rank, int tp_size,
                       const void *src, size_t src_bytes, void *dst, size_t dst_cap, uint64_t *out_dims,
                       size_t *out_bytes);

/* Device stream of the context (cudaStream_t), for timing with events. */
void *sq_ctx_stream(sq_ctx *c);
/* Kernel launches one decode step of this context issues: 1 when the persistent
 * decode kernel serves the model, else the count of the op-level sequence. */
int sq_ctx_launches_per_token(const sq_ctx *c, int *out);

#ifdef __cplusplus
}
#endif
#endif
