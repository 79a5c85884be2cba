// model.h — host-side structs behind the opaque sq_model / sq_ctx handles.
#pragma once
#include <cuda_runtime.h>

#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/squirrel_cuda.h"

namespace sq {
struct DevTensor {
  void *ptr = nullptr;
  int type = 0;
  std::vector<uint64_t> dims;
  size_t nbytes = 0;
};
struct DecodeState;  // persistent decode kernel resources (decode.cu)
struct TpAllReduce;  // one-shot NVLink all-reduce of a tensor-parallel model (allreduce.cu)
void rope_inv_freq(const sq_llama_config &c, std::vector<float> &out);
int forward_device(sq_ctx *c, const uint32_t *d_ids, int n);
// NCCL (tp.cpp): loaded on first use
int nccl_comm_init(const void *id, int rank, int size, void **comm);
void nccl_comm_destroy(void *comm);
int nccl_all_reduce_sum(void *comm, float *buf, size_t n, cudaStream_t s);
int nccl_all_gather_bytes(void *comm, const void *src, void *dst, size_t bytes_per_rank, cudaStream_t s);
int nccl_all_reduce_min_int(void *comm, int *buf, cudaStream_t s);
// One-shot all-reduce over NVLink peer memory (allreduce.cu): set up collectively at
// model creation (m->ar stays null when a rank cannot map its peers: NCCL then serves),
// launched for one decode row with the residual add fused, error word read after a sync.
int tp_allreduce_create(sq_model *m);
void tp_allreduce_release(TpAllReduce *ar);
cudaError_t launch_allreduce_add(cudaStream_t s, TpAllReduce *ar, float *hidden, const float *part, bool pdl);
unsigned tp_allreduce_status(const TpAllReduce *ar, bool clear);
unsigned *tp_allreduce_err_ptr(const TpAllReduce *ar);
// The persistent decode kernel's exchange area of every rank's mailbox (this process's
// mappings, rank order); returns the number of ranks (0: none).
int tp_decode_boxes(const TpAllReduce *ar, unsigned long long **boxes, int max);
int tp_allreduce_recover(sq_model *m);  // collective re-synchronization after a timeout
}  // namespace sq

// LlamaWeights (models/llama/weights.rs:18-47) resolved to device pointers.
struct sq_model {
  sq_llama_config cfg{};  // the whole model's configuration
  sq_llama_config lc{};   // this rank's shard of it (q / kv heads, FFN rows, vocabulary rows)
  int device = 0;
  int acts = SQ_ACTS_F32;
  bool finalized = false;
  int tp_rank = 0, tp_size = 1;  // tensor-parallel group (tp.cpp)
  void *nccl = nullptr;          // ncclComm_t when tp_size > 1
  sq::TpAllReduce *ar = nullptr;  // the decode step's peer-memory all-reduce (null: NCCL's)
  int vocab0 = 0;                // first vocabulary row of this rank's LM-head shard
  std::unordered_map<std::string, sq::DevTensor> tensors;
  struct Layer {
    const float *attn_norm = nullptr, *ffn_norm = nullptr;
    const void *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr, *gate = nullptr, *up = nullptr,
               *down = nullptr;
  };
  std::vector<Layer> layers;
  const void *embd = nullptr, *out_w = nullptr;
  int embd_type = 0, out_type = 0;
  const float *out_norm = nullptr;
  std::vector<float> inv_freq;
  float *d_inv_freq = nullptr;
  ~sq_model();
};

// ModelContext (models/common/context.rs:9-28): KV cache + workspace, on one stream.
struct sq_ctx {
  sq_model *m = nullptr;
  int max_ctx = 0;
  int seq_len = 0;  // KvCache::seq_len: position of the next token
  bool have_logits = false;
  cudaStream_t stream = nullptr;
  // head-major KV cache: [layer][kv_head][max_ctx][head_dim] f32
  float *kc = nullptr, *vc = nullptr;
  int ws_rows = 0;
  float *hidden = nullptr, *normed = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn = nullptr,
        *attn_out = nullptr, *gate = nullptr, *up = nullptr, *act = nullptr, *ffn_out = nullptr, *logits = nullptr;
  void *xq = nullptr;  // Q8_0 activation scratch (the reference's act_q)
  float *sdpa_part = nullptr;
  size_t sdpa_part_floats = 0;
  int *sdpa_cnt = nullptr;  // per query row: split CTAs finished (the last one merges; self-resetting)
  float *gemm_ws = nullptr;  // split-K partial tiles of the prefill GEMM
  size_t gemm_ws_floats = 0;
  void *argmax_part = nullptr;
  long long *d_argmax = nullptr;
  uint32_t *d_tokens = nullptr;
  float *d_cos = nullptr, *d_sin = nullptr;  // RoPE table [max_ctx][head_dim/2]
  sq::DecodeState *dec = nullptr;
  cudaGraphExec_t step_graph = nullptr;  // the op-level decode step, captured once
  int *d_gpos = nullptr;  // its device position counter
  int gpos = -1;          // the value d_gpos holds once queued work finishes (-1: unknown)
  int eager_steps = 0;
  bool graph_failed = false;
  float *logits_full = nullptr;  // tensor parallel: the gathered vocabulary
  void *arg_local = nullptr, *arg_all = nullptr;  // tensor parallel: per-rank argmax states
  uint32_t *d_out_ids = nullptr;  // ids of sq_decode_steps
  // pinned host staging: the ids a call copies in or out (max_ctx of them), and the
  // argmax with the error words every call reads back in one copy
  uint32_t *h_ids = nullptr;
  unsigned long long *h_status = nullptr, *d_status = nullptr;
  int out_cap = 0;
  std::vector<void *> allocs;
  ~sq_ctx();
};
