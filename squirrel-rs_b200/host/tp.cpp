// tp.cpp — tensor parallelism for the multi-GPU decode configuration: Megatron
// column/row sharding of the GGUF tensors and the NCCL plumbing around it.
//
// Column-parallel (output rows split): attn_q by q heads, attn_k / attn_v by kv
// heads, ffn_gate / ffn_up by FFN rows, output (LM head) by vocabulary rows.
// Row-parallel (input split, whole 32-element blocks of every row): attn_output by
// q heads, ffn_down by FFN rows. Norms and token_embd are replicated. A rank's
// shard keeps the native block layout, so the single-GPU kernels run on it
// unchanged; the forward adds an all-reduce after the O and down projections and
// a cross-rank greedy argmax over the vocabulary shards.
//
// NCCL is loaded with dlopen when the first tensor-parallel model is created (a
// process that also loaded PyTorch reuses the copy already mapped), so the
// library itself does not depend on it.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include <mutex>
#include <string>

#include "../csrc/status.h"
#include "model.h"

using namespace sq;

namespace sq {

namespace {
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  const char *(*error_string)(ncclResult_t) = nullptr;
  std::string why;
  bool ok = false;
};

NcclApi &api() {
  static NcclApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      a.why = std::string("cannot load libnccl.so.2: ") + dlerror();
      return;
    }
    a.get_unique_id = (decltype(a.get_unique_id))dlsym(h, "ncclGetUniqueId");
    a.comm_init_rank = (decltype(a.comm_init_rank))dlsym(h, "ncclCommInitRank");
    a.all_reduce = (decltype(a.all_reduce))dlsym(h, "ncclAllReduce");
    a.all_gather = (decltype(a.all_gather))dlsym(h, "ncclAllGather");
    a.comm_destroy = (decltype(a.comm_destroy))dlsym(h, "ncclCommDestroy");
    a.error_string = (decltype(a.error_string))dlsym(h, "ncclGetErrorString");
    a.ok = a.get_unique_id && a.comm_init_rank && a.all_reduce && a.all_gather && a.comm_destroy && a.error_string;
    if (!a.ok) a.why = "libnccl.so.2 lacks an expected symbol";
  });
  return a;
}

int nccl_fail(ncclResult_t r, const char *what) {
  return fail(SQ_ERR_NCCL, std::string(what) + ": " + (api().error_string ? api().error_string(r) : "NCCL error"));
}

bool ends_with(const std::string &s, const char *suffix) {
  const size_t n = strlen(suffix);
  return s.size() >= n && s.compare(s.size() - n, n, suffix) == 0;
}

enum { SHARD_REPLICATE = 0, SHARD_ROWS = 1, SHARD_COLS = 2 };

int shard_kind(const std::string &name) {
  if (name.rfind("blk.", 0) == 0) {
    if (ends_with(name, ".attn_q.weight") || ends_with(name, ".attn_k.weight") || ends_with(name, ".attn_v.weight") ||
        ends_with(name, ".ffn_gate.weight") || ends_with(name, ".ffn_up.weight"))
      return SHARD_ROWS;
    if (ends_with(name, ".attn_output.weight") || ends_with(name, ".ffn_down.weight")) return SHARD_COLS;
    return SHARD_REPLICATE;
  }
  return name == "output.weight" ? SHARD_ROWS : SHARD_REPLICATE;
}
}  // namespace

int nccl_all_reduce_sum(void *comm, float *buf, size_t n, cudaStream_t s) {
  const ncclResult_t r = api().all_reduce(buf, buf, n, ncclFloat32, ncclSum, (ncclComm_t)comm, s);
  return r == ncclSuccess ? SQ_OK : nccl_fail(r, "ncclAllReduce");
}

int nccl_all_reduce_min_int(void *comm, int *buf, cudaStream_t s) {
  const ncclResult_t r = api().all_reduce(buf, buf, 1, ncclInt32, ncclMin, (ncclComm_t)comm, s);
  return r == ncclSuccess ? SQ_OK : nccl_fail(r, "ncclAllReduce");
}

int nccl_all_gather_bytes(void *comm, const void *src, void *dst, size_t bytes_per_rank, cudaStream_t s) {
  const ncclResult_t r = api().all_gather(src, dst, bytes_per_rank, ncclUint8, (ncclComm_t)comm, s);
  return r == ncclSuccess ? SQ_OK : nccl_fail(r, "ncclAllGather");
}

int nccl_comm_init(const void *id, int rank, int size, void **comm) {
  NcclApi &a = api();
  if (!a.ok) return fail(SQ_ERR_NCCL, a.why);
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclComm_t c = nullptr;
  const ncclResult_t r = a.comm_init_rank(&c, size, uid, rank);
  if (r != ncclSuccess) return nccl_fail(r, "ncclCommInitRank");
  *comm = (void *)c;
  return SQ_OK;
}

void nccl_comm_destroy(void *comm) {
  if (comm && api().ok) api().comm_destroy((ncclComm_t)comm);
}

}  // namespace sq

extern "C" int sq_nccl_unique_id(void *out, size_t n) {
  if (!out) return fail(SQ_ERR_ARG, "nccl_unique_id: null pointer");
  if (n < sizeof(ncclUniqueId)) return fail(SQ_ERR_ARG, "nccl_unique_id: buffer smaller than 128 bytes");
  NcclApi &a = api();
  if (!a.ok) return fail(SQ_ERR_NCCL, a.why);
  ncclUniqueId uid;
  const ncclResult_t r = a.get_unique_id(&uid);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  memcpy(out, &uid, sizeof(uid));
  return SQ_OK;
}

extern "C" int sq_tp_shard_tensor(const char *name, int ggml_type, const uint64_t *dims, int n_dims, int tp_rank,
                                  int tp_size, const void *src, size_t src_bytes, void *dst, size_t dst_cap,
                                  uint64_t *out_dims, size_t *out_bytes) {
  if (!name || !dims || !out_dims || !out_bytes) return fail(SQ_ERR_ARG, "tp_shard_tensor: null pointer");
  if (tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size) return fail(SQ_ERR_ARG, "tp_shard_tensor: bad rank or size");
  if (n_dims <= 0 || n_dims > 4) return fail(SQ_ERR_SHAPE, std::string("tp_shard_tensor: bad rank for ") + name);
  uint64_t numel = 1;
  for (int i = 0; i < n_dims; i++) numel *= dims[i];
  const size_t full = tensor_nbytes(ggml_type, numel);
  if (!full) return fail(SQ_ERR_INVALID_TYPE, std::string("tp_shard_tensor: unsupported type for ") + name);
  if (src && src_bytes != full) return fail(SQ_ERR_SHAPE, std::string("tp_shard_tensor: byte size mismatch for ") + name);
  int kind = tp_size == 1 ? SHARD_REPLICATE : shard_kind(name);
  if (kind != SHARD_REPLICATE && n_dims != 2)
    return fail(SQ_ERR_SHAPE, std::string("tp_shard_tensor: expected a matrix: ") + name);
  for (int i = 0; i < n_dims; i++) out_dims[i] = dims[i];
  size_t bytes = full;
  const uint64_t in = dims[0], rows = n_dims == 2 ? dims[1] : 0;
  if (kind == SHARD_ROWS) {
    if (rows % (uint64_t)tp_size) return fail(SQ_ERR_SHAPE, std::string("tp_shard_tensor: rows not divisible: ") + name);
    out_dims[1] = rows / tp_size;
    bytes = full / tp_size;
  } else if (kind == SHARD_COLS) {
    if (in % (32ull * tp_size))
      return fail(SQ_ERR_SHAPE, std::string("tp_shard_tensor: row length not a whole number of blocks per rank: ") + name);
    out_dims[0] = in / tp_size;
    bytes = tensor_nbytes(ggml_type, out_dims[0] * rows);
  }
  *out_bytes = bytes;
  if (!dst) return SQ_OK;  // size query
  if (!src) return fail(SQ_ERR_ARG, "tp_shard_tensor: null source");
  if (dst_cap < bytes) return fail(SQ_ERR_ARG, std::string("tp_shard_tensor: destination too small for ") + name);
  const uint8_t *s = (const uint8_t *)src;
  uint8_t *d = (uint8_t *)dst;
  if (kind == SHARD_REPLICATE) {
    memcpy(d, s, bytes);
  } else if (kind == SHARD_ROWS) {
    memcpy(d, s + (size_t)tp_rank * bytes, bytes);
  } else {  // each row: its rank's contiguous run of whole blocks
    const size_t row_full = tensor_nbytes(ggml_type, in), row_part = tensor_nbytes(ggml_type, in / tp_size);
    for (uint64_t r = 0; r < rows; r++) memcpy(d + r * row_part, s + r * row_full + (size_t)tp_rank * row_part, row_part);
  }
  return SQ_OK;
}
