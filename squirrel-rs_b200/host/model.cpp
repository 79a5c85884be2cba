// model.cpp — host side of the model-level C ABI: the B200 counterpart of the
// reference's GGUF upload (file_parser/*.rs -> HBM), LlamaConfig / LlamaWeights
// (models/llama/{config,weights}.rs), ModelContext / KvCache / Workspace
// (models/common/*.rs), Llama3_2::forward (models/llama/model.rs:45-97) and the
// TextTokenGenerator step loop (text_generator.rs:58-97). Everything numeric
// runs in CUDA kernels; this file validates, allocates and sequences launches.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <math.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <chrono>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "../csrc/status.h"
#include "../csrc/decode.cuh"
#include "../csrc/ops.cuh"
#include "model.h"

using namespace sq;

// ------------------------------------------------------------------------------------
// GGUF reader (file_parser/gguf_file.rs:22-49, gguf_header.rs, gguf_metadata_value.rs,
// gguf_tensor_info.rs). Data starts at the next multiple of a hard-coded 32 bytes.
// ------------------------------------------------------------------------------------
namespace {

enum { GT_U8 = 0, GT_I8, GT_U16, GT_I16, GT_U32, GT_I32, GT_F32, GT_BOOL, GT_STR, GT_ARR, GT_U64, GT_I64, GT_F64 };

struct KV {
  int type = -1;
  uint64_t u = 0;
  float f = 0;
  uint64_t arr_len = 0;
};

struct TInfo {
  std::vector<uint64_t> dims;
  int type;
  uint64_t offset;
};

struct Reader {
  const uint8_t *p, *end;
  bool bad = false;
  uint64_t u(int n) {
    if (p + n > end) {
      bad = true;
      return 0;
    }
    uint64_t v = 0;
    for (int i = 0; i < n; i++) v |= (uint64_t)p[i] << (8 * i);
    p += n;
    return v;
  }
  std::string str() {
    uint64_t n = u(8);
    if (bad || p + n > end) {
      bad = true;
      return {};
    }
    std::string s((const char *)p, n);
    p += n;
    return s;
  }
  void value(int type, KV *kv, int depth) {
    static const int sz[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (type < 0 || type > 12) {
      bad = true;
      return;
    }
    if (type == GT_STR) {
      str();
    } else if (type == GT_ARR) {
      int at = (int)u(4);
      uint64_t n = u(8);
      if (kv && depth == 0) kv->arr_len = n;
      for (uint64_t i = 0; i < n && !bad; i++) value(at, nullptr, depth + 1);
    } else {
      uint64_t v = u(sz[type]);
      if (kv && depth == 0) {
        kv->u = v;
        if (type == GT_F32) {
          uint32_t w = (uint32_t)v;
          memcpy(&kv->f, &w, 4);
        }
      }
    }
  }
};

struct GgufFile {
  void *map = MAP_FAILED;
  size_t len = 0;
  std::unordered_map<std::string, KV> kv;
  std::unordered_map<std::string, TInfo> tensors;
  uint64_t data_off = 0;
  ~GgufFile() {
    if (map != MAP_FAILED) munmap(map, len);
  }
  int open(const char *path) {
    int fd = ::open(path, O_RDONLY);
    if (fd < 0) return fail(SQ_ERR_IO, std::string("cannot open ") + path);
    struct stat sb;
    fstat(fd, &sb);
    len = (size_t)sb.st_size;
    map = mmap(nullptr, len, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (map == MAP_FAILED) return fail(SQ_ERR_IO, std::string("cannot map ") + path);
    Reader r{(const uint8_t *)map, (const uint8_t *)map + len};
    r.u(4);  // magic (read, not checked, like gguf_header.rs:13-24)
    r.u(4);  // version
    uint64_t nt = r.u(8), nkv = r.u(8);
    for (uint64_t i = 0; i < nkv && !r.bad; i++) {
      std::string key = r.str();
      int type = (int)r.u(4);
      KV k;
      k.type = type;
      r.value(type, &k, 0);
      kv[key] = k;
    }
    for (uint64_t i = 0; i < nt && !r.bad; i++) {
      std::string name = r.str();
      TInfo t;
      uint32_t nd = (uint32_t)r.u(4);
      if (nd > 8) {
        r.bad = true;
        break;
      }
      for (uint32_t d = 0; d < nd; d++) t.dims.push_back(r.u(8));
      t.type = (int)r.u(4);
      t.offset = r.u(8);
      tensors[name] = t;
    }
    if (r.bad) return fail(SQ_ERR_IO, std::string("truncated or malformed GGUF ") + path);
    uint64_t pos = (uint64_t)(r.p - (const uint8_t *)map);
    data_off = (pos + 31) & ~(uint64_t)31;
    return SQ_OK;
  }
  bool u32(const char *key, uint32_t *out) const {  // config.rs:129-138: strictly U32
    auto it = kv.find(key);
    if (it == kv.end() || it->second.type != GT_U32) return false;
    *out = (uint32_t)it->second.u;
    return true;
  }
  bool f32(const char *key, float *out) const {  // config.rs:140-149: strictly F32
    auto it = kv.find(key);
    if (it == kv.end() || it->second.type != GT_F32) return false;
    *out = it->second.f;
    return true;
  }
};

}  // namespace

// ------------------------------------------------------------------------------------
// model
// ------------------------------------------------------------------------------------
namespace sq {

// compute_rope_inv_freq (models/llama/config.rs:83-127), host single precision, C library powf.
void rope_inv_freq(const sq_llama_config &c, std::vector<float> &out) {
  const int half = c.head_dim / 2;
  const float inv_head_dim = 1.0f / (float)c.head_dim;
  out.resize(half);
  for (int j = 0; j < half; j++) out[j] = powf(c.rope_base, -2.0f * (float)j * inv_head_dim);
  const float two_pi = 6.28318548202514648438f;  // std::f32::consts::TAU
  const float low_wl = c.rope_orig_ctx / c.rope_low_freq, high_wl = c.rope_orig_ctx / c.rope_high_freq;
  for (int j = 0; j < half; j++) {
    const float f = out[j];
    const float wavelen = two_pi / f;
    if (wavelen > low_wl) {
      out[j] = f / c.rope_factor;
    } else if (wavelen >= high_wl) {
      const float smooth = (c.rope_orig_ctx / wavelen - c.rope_low_freq) / (c.rope_high_freq - c.rope_low_freq);
      const float a = 1.0f - smooth, b = f / c.rope_factor;
      const volatile float t1 = a * b;  // keep the two products separately rounded (Rust never contracts)
      const volatile float t2 = smooth * f;
      out[j] = t1 + t2;
    }
  }
}

}  // namespace sq

sq_model::~sq_model() {
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  for (auto &kv : tensors) cudaFree(kv.second.ptr);
  cudaFree(d_inv_freq);
  tp_allreduce_release(ar);  // every peer's last write into this mailbox preceded its last flag
  nccl_comm_destroy(nccl);
  cudaSetDevice(prev);
}

static int validate_config(const sq_llama_config &c) {
  if (c.n_blocks <= 0 || c.embed_dim <= 0 || c.ffn_dim <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 ||
      c.head_dim <= 0 || c.vocab_size <= 0)
    return fail(SQ_ERR_CONFIG, "config: non-positive dimension");
  if (c.n_heads % c.n_kv_heads) return fail(SQ_ERR_CONFIG, "config: n_heads must be a multiple of n_kv_heads");
  if (c.head_dim % 32 || c.head_dim > 256) return fail(SQ_ERR_CONFIG, "config: head_dim must be a multiple of 32, <= 256");
  if (c.embed_dim % 32 || c.ffn_dim % 32 || (c.n_heads * c.head_dim) % 32)
    return fail(SQ_ERR_CONFIG, "config: projection widths must be multiples of 32");
  if (!is_weight_type(c.weight_type)) return fail(SQ_ERR_INVALID_TYPE, "config: weight type must be Q8_0, Q4_0 or BF16");
  return SQ_OK;
}

// Model creation, alone (tp_size 1) or as rank tp_rank of a tensor-parallel group
// whose members share the NCCL unique id `nccl_id`.
static int model_create(const sq_llama_config *cfg, int device, int acts, int tp_rank, int tp_size,
                        const void *nccl_id, sq_model **out) {
  if (!cfg || !out) return fail(SQ_ERR_ARG, "model_create: null pointer");
  *out = nullptr;
  int st = validate_config(*cfg);
  if (st) return st;
  if (tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size) return fail(SQ_ERR_ARG, "model_create: bad tp rank / size");
  if (tp_size > 1) {
    if (!nccl_id) return fail(SQ_ERR_ARG, "model_create: tensor parallel needs an NCCL unique id");
    if (cfg->n_heads % tp_size || cfg->n_kv_heads % tp_size || cfg->ffn_dim % (32 * tp_size) ||
        cfg->vocab_size % tp_size)
      return fail(SQ_ERR_CONFIG, "model_create: heads, kv heads, FFN blocks and vocabulary must divide by tp_size");
  }
  int ndev = 0;
  SQ_CUDA(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return fail(SQ_ERR_ARG, "model_create: no such device");
  auto m = std::make_unique<sq_model>();
  m->cfg = *cfg;
  m->lc = *cfg;
  m->lc.n_heads = cfg->n_heads / tp_size;
  m->lc.n_kv_heads = cfg->n_kv_heads / tp_size;
  m->lc.ffn_dim = cfg->ffn_dim / tp_size;
  m->lc.vocab_size = cfg->vocab_size / tp_size;
  m->vocab0 = tp_rank * m->lc.vocab_size;
  m->device = device;
  m->acts = acts == SQ_ACTS_Q8 ? SQ_ACTS_Q8 : SQ_ACTS_F32;
  m->tp_rank = tp_rank;
  m->tp_size = tp_size;
  if (tp_size > 1) {
    SQ_CUDA(cudaSetDevice(device));
    if ((st = nccl_comm_init(nccl_id, tp_rank, tp_size, &m->nccl))) return st;
    if ((st = tp_allreduce_create(m.get()))) return st;  // collective, like the NCCL init
  }
  *out = m.release();
  return SQ_OK;
}

extern "C" int sq_model_create(const sq_llama_config *cfg, int device, int acts, sq_model **out) {
  return model_create(cfg, device, acts, 0, 1, nullptr, out);
}

extern "C" int sq_model_create_tp(const sq_llama_config *cfg, int device, int acts, int tp_rank, int tp_size,
                                  const void *nccl_id, sq_model **out) {
  return model_create(cfg, device, acts, tp_rank, tp_size, nccl_id, out);
}

extern "C" int sq_model_upload_tensor(sq_model *m, const char *name, int ggml_type, const uint64_t *dims,
                                      int n_dims, const void *host_data, size_t nbytes) {
  if (!m || !name || !dims || !host_data) return fail(SQ_ERR_ARG, "upload_tensor: null pointer");
  if (m->finalized) return fail(SQ_ERR_ARG, "upload_tensor: model already finalized");
  if (n_dims <= 0 || n_dims > 4) return fail(SQ_ERR_SHAPE, std::string("upload_tensor: bad rank for ") + name);
  uint64_t numel = 1;
  for (int i = 0; i < n_dims; i++) numel *= dims[i];
  const size_t need = tensor_nbytes(ggml_type, numel);
  if (!need) return fail(SQ_ERR_INVALID_TYPE, std::string("upload_tensor: unsupported type for ") + name);
  if (need != nbytes) return fail(SQ_ERR_SHAPE, std::string("upload_tensor: byte size mismatch for ") + name);
  SQ_CUDA(cudaSetDevice(m->device));
  DevTensor t;
  t.type = ggml_type;
  t.dims.assign(dims, dims + n_dims);
  t.nbytes = nbytes;
  std::vector<uint8_t> shard;
  if (m->tp_size > 1) {  // this rank's shard, still in the native block layout
    uint64_t sd[4];
    size_t sb = 0;
    int st = sq_tp_shard_tensor(name, ggml_type, dims, n_dims, m->tp_rank, m->tp_size, host_data, nbytes, nullptr, 0,
                                sd, &sb);
    if (st) return st;
    shard.resize(sb);
    if ((st = sq_tp_shard_tensor(name, ggml_type, dims, n_dims, m->tp_rank, m->tp_size, host_data, nbytes,
                                 shard.data(), sb, sd, &sb)))
      return st;
    t.dims.assign(sd, sd + n_dims);
    t.nbytes = sb;
    host_data = shard.data();
  }
  SQ_CUDA(cudaMalloc(&t.ptr, (t.nbytes + 255) / 256 * 256));  // native block layout, 256-byte aligned
  SQ_CUDA(cudaMemcpy(t.ptr, host_data, t.nbytes, cudaMemcpyHostToDevice));
  auto it = m->tensors.find(name);
  if (it != m->tensors.end()) cudaFree(it->second.ptr);
  m->tensors[name] = t;
  return SQ_OK;
}

static int need_tensor(sq_model *m, const std::string &name, int type, std::vector<uint64_t> dims,
                       const DevTensor **out) {
  auto it = m->tensors.find(name);
  if (it == m->tensors.end()) return fail(SQ_ERR_CONFIG, "missing tensor " + name);  // weights.rs:51-56
  if (type >= 0 && it->second.type != type) return fail(SQ_ERR_INVALID_TYPE, "wrong type for tensor " + name);
  if (it->second.dims != dims) return fail(SQ_ERR_SHAPE, "wrong shape for tensor " + name);
  *out = &it->second;
  return SQ_OK;
}

extern "C" int sq_model_finalize(sq_model *m) {
  if (!m) return fail(SQ_ERR_ARG, "finalize: null model");
  if (m->finalized) return SQ_OK;
  const sq_llama_config &c = m->lc;  // this rank's shard of the projections
  const uint64_t E = c.embed_dim, Q = (uint64_t)c.n_heads * c.head_dim, KVd = (uint64_t)c.n_kv_heads * c.head_dim,
                 F = c.ffn_dim, V = c.vocab_size, Vall = m->cfg.vocab_size;
  const int wt = c.weight_type;
  m->layers.resize(c.n_blocks);
  const DevTensor *t;
  int st;
  for (int i = 0; i < c.n_blocks; i++) {
    auto nm = [&](const char *s) { return "blk." + std::to_string(i) + "." + s; };
    auto &L = m->layers[i];
    if ((st = need_tensor(m, nm("attn_norm.weight"), SQ_F32, {E}, &t))) return st;
    L.attn_norm = (const float *)t->ptr;
    if ((st = need_tensor(m, nm("ffn_norm.weight"), SQ_F32, {E}, &t))) return st;
    L.ffn_norm = (const float *)t->ptr;
    if ((st = need_tensor(m, nm("attn_q.weight"), wt, {E, Q}, &t))) return st;
    L.q = t->ptr;
    if ((st = need_tensor(m, nm("attn_k.weight"), wt, {E, KVd}, &t))) return st;
    L.k = t->ptr;
    if ((st = need_tensor(m, nm("attn_v.weight"), wt, {E, KVd}, &t))) return st;
    L.v = t->ptr;
    if ((st = need_tensor(m, nm("attn_output.weight"), wt, {Q, E}, &t))) return st;
    L.o = t->ptr;
    if ((st = need_tensor(m, nm("ffn_gate.weight"), wt, {E, F}, &t))) return st;
    L.gate = t->ptr;
    if ((st = need_tensor(m, nm("ffn_up.weight"), wt, {E, F}, &t))) return st;
    L.up = t->ptr;
    if ((st = need_tensor(m, nm("ffn_down.weight"), wt, {F, E}, &t))) return st;
    L.down = t->ptr;
  }
  if ((st = need_tensor(m, "token_embd.weight", -1, {E, Vall}, &t))) return st;  // replicated
  if (!is_weight_type(t->type)) return fail(SQ_ERR_INVALID_TYPE, "token_embd.weight: unsupported type");
  m->embd = t->ptr;
  m->embd_type = t->type;
  if ((st = need_tensor(m, "output_norm.weight", SQ_F32, {E}, &t))) return st;
  m->out_norm = (const float *)t->ptr;
  if (m->tensors.count("output.weight")) {
    if ((st = need_tensor(m, "output.weight", -1, {E, V}, &t))) return st;
    if (!is_weight_type(t->type)) return fail(SQ_ERR_INVALID_TYPE, "output.weight: unsupported type");
    m->out_w = t->ptr;
    m->out_type = t->type;
  } else {  // tied LM head, weights.rs:87-89 (this rank's vocabulary rows of token_embd)
    m->out_w = (const uint8_t *)m->embd + tensor_nbytes(m->embd_type, (uint64_t)m->vocab0 * E);
    m->out_type = m->embd_type;
  }
  rope_inv_freq(c, m->inv_freq);
  SQ_CUDA(cudaSetDevice(m->device));
  SQ_CUDA(cudaMalloc(&m->d_inv_freq, m->inv_freq.size() * sizeof(float)));
  SQ_CUDA(cudaMemcpy(m->d_inv_freq, m->inv_freq.data(), m->inv_freq.size() * sizeof(float), cudaMemcpyHostToDevice));
  m->finalized = true;
  return SQ_OK;
}

static int load_gguf(const char *path, int device, int acts, int tp_rank, int tp_size, const void *nccl_id,
                     sq_model **out) {
  if (!path || !out) return fail(SQ_ERR_ARG, "load_gguf: null pointer");
  *out = nullptr;
  GgufFile g;
  int st = g.open(path);
  if (st) return st;
  // LlamaConfig::from_gguf, config.rs:29-73
  sq_llama_config c{};
  uint32_t u;
  float f;
  auto req_u32 = [&](const char *k, int *dst) -> int {
    if (!g.u32(k, &u)) return fail(SQ_ERR_CONFIG, std::string("missing or non-U32 metadata ") + k);
    *dst = (int)u;
    return SQ_OK;
  };
  if ((st = req_u32("llama.block_count", &c.n_blocks))) return st;
  if ((st = req_u32("llama.embedding_length", &c.embed_dim))) return st;
  if ((st = req_u32("llama.feed_forward_length", &c.ffn_dim))) return st;
  if ((st = req_u32("llama.attention.head_count", &c.n_heads))) return st;
  if ((st = req_u32("llama.attention.head_count_kv", &c.n_kv_heads))) return st;
  c.head_dim = g.u32("llama.rope.dimension_count", &u) ? (int)u : (c.n_heads ? c.embed_dim / c.n_heads : 0);
  if (!g.f32("llama.rope.freq_base", &c.rope_base)) return fail(SQ_ERR_CONFIG, "missing llama.rope.freq_base");
  if (!g.f32("llama.attention.layer_norm_rms_epsilon", &c.rms_eps))
    return fail(SQ_ERR_CONFIG, "missing llama.attention.layer_norm_rms_epsilon");
  if ((st = req_u32("llama.context_length", &c.context_length))) return st;
  if (!g.u32("tokenizer.ggml.bos_token_id", &c.bos_token_id)) return fail(SQ_ERR_CONFIG, "missing bos id");
  if (!g.u32("tokenizer.ggml.eos_token_id", &c.eos_token_id)) return fail(SQ_ERR_CONFIG, "missing eos id");
  if (g.u32("llama.vocab_size", &u)) {
    c.vocab_size = (int)u;
  } else {
    auto it = g.kv.find("tokenizer.ggml.tokens");
    if (it == g.kv.end() || it->second.type != GT_ARR)
      return fail(SQ_ERR_CONFIG, "missing llama.vocab_size / tokenizer.ggml.tokens");
    c.vocab_size = (int)it->second.arr_len;
  }
  c.rope_factor = g.f32("llama.rope.scaling.factor", &f) ? f : 32.0f;
  c.rope_low_freq = g.f32("llama.rope.scaling.low_freq_factor", &f) ? f : 1.0f;
  c.rope_high_freq = g.f32("llama.rope.scaling.high_freq_factor", &f) ? f : 4.0f;
  c.rope_orig_ctx = g.u32("llama.rope.scaling.original_context_length", &u) ? (float)u : 8192.0f;
  auto q = g.tensors.find("blk.0.attn_q.weight");
  if (q == g.tensors.end()) return fail(SQ_ERR_CONFIG, "missing tensor blk.0.attn_q.weight");
  c.weight_type = q->second.type;

  sq_model *m = nullptr;
  if ((st = model_create(&c, device, acts, tp_rank, tp_size, nccl_id, &m))) return st;
  for (auto &kv : g.tensors) {
    const std::string &name = kv.first;
    const TInfo &t = kv.second;
    const bool wanted = name.rfind("blk.", 0) == 0 || name == "token_embd.weight" || name == "output_norm.weight" ||
                        name == "output.weight";
    if (!wanted) continue;
    uint64_t numel = 1;
    for (auto d : t.dims) numel *= d;
    size_t nb = tensor_nbytes(t.type, numel);
    if (!nb) {
      sq_model_free(m);
      return fail(SQ_ERR_INVALID_TYPE, "unsupported tensor type for " + name);  // gguf_tensor_info.rs:52-65
    }
    if (g.data_off + t.offset + nb > g.len) {
      sq_model_free(m);
      return fail(SQ_ERR_IO, "tensor data past end of file: " + name);
    }
    st = sq_model_upload_tensor(m, name.c_str(), t.type, t.dims.data(), (int)t.dims.size(),
                                (const uint8_t *)g.map + g.data_off + t.offset, nb);
    if (st) {
      sq_model_free(m);
      return st;
    }
  }
  if ((st = sq_model_finalize(m))) {
    sq_model_free(m);
    return st;
  }
  *out = m;
  return SQ_OK;
}

extern "C" int sq_model_load_gguf(const char *path, int device, int acts, sq_model **out) {
  return load_gguf(path, device, acts, 0, 1, nullptr, out);
}

extern "C" int sq_model_load_gguf_tp(const char *path, int device, int acts, int tp_rank, int tp_size,
                                     const void *nccl_id, sq_model **out) {
  return load_gguf(path, device, acts, tp_rank, tp_size, nccl_id, out);
}

extern "C" int sq_model_config(const sq_model *m, sq_llama_config *out) {
  if (!m || !out) return fail(SQ_ERR_ARG, "model_config: null pointer");
  *out = m->cfg;
  return SQ_OK;
}

extern "C" void sq_model_free(sq_model *m) { delete m; }

// ------------------------------------------------------------------------------------
// context
// ------------------------------------------------------------------------------------
sq_ctx::~sq_ctx() {
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(m->device);
  if (stream) cudaStreamSynchronize(stream);
  if (step_graph) cudaGraphExecDestroy(step_graph);  // before the buffers (and any NCCL communicator) it uses
  decode_release(this);
  cudaFree(d_out_ids);
  if (h_ids) cudaFreeHost(h_ids);
  if (h_status) cudaFreeHost(h_status);
  for (void *p : allocs) cudaFree(p);
  if (stream) cudaStreamDestroy(stream);
  cudaSetDevice(prev);
}

template <class T>
static cudaError_t ctx_alloc(sq_ctx *c, T **p, size_t n) {
  cudaError_t e = cudaMalloc((void **)p, n * sizeof(T) + 256);
  if (e == cudaSuccess) c->allocs.push_back((void *)*p);
  return e;
}

extern "C" int sq_ctx_create(sq_model *m, int max_ctx, sq_ctx **out) {
  if (!m || !out) return fail(SQ_ERR_ARG, "ctx_create: null pointer");
  if (!m->finalized) return fail(SQ_ERR_ARG, "ctx_create: model not finalized");
  *out = nullptr;
  const sq_llama_config &c = m->lc;  // this rank's heads, KV heads, FFN rows and vocabulary rows
  if (max_ctx <= 0) max_ctx = c.context_length > 0 && c.context_length < 8192 ? c.context_length : 8192;
  SQ_CUDA(cudaSetDevice(m->device));
  auto x = std::make_unique<sq_ctx>();
  x->m = m;
  x->max_ctx = max_ctx;
  SQ_CUDA(cudaStreamCreateWithFlags(&x->stream, cudaStreamNonBlocking));
  const int E = c.embed_dim, Q = c.n_heads * c.head_dim, KVd = c.n_kv_heads * c.head_dim, F = c.ffn_dim;
  const size_t kv_elems = (size_t)c.n_blocks * c.n_kv_heads * max_ctx * c.head_dim;
  SQ_CUDA(ctx_alloc(x.get(), &x->kc, kv_elems));
  SQ_CUDA(ctx_alloc(x.get(), &x->vc, kv_elems));
  // Prefill is processed in chunks of this many rows (SQB200_PREFILL_ROWS overrides
  // the default of 2048): the larger the chunk, the more output tiles per GEMM.
  int rows_cap = 2048;
  if (const char *v = getenv("SQB200_PREFILL_ROWS")) rows_cap = std::max(1, atoi(v));
  const int R = x->ws_rows = std::max(1, std::min(rows_cap, max_ctx));
  SQ_CUDA(ctx_alloc(x.get(), &x->hidden, (size_t)R * E));
  SQ_CUDA(ctx_alloc(x.get(), &x->normed, (size_t)R * E));
  SQ_CUDA(ctx_alloc(x.get(), &x->q, (size_t)R * Q));
  SQ_CUDA(ctx_alloc(x.get(), &x->k, (size_t)R * KVd));
  SQ_CUDA(ctx_alloc(x.get(), &x->v, (size_t)R * KVd));
  SQ_CUDA(ctx_alloc(x.get(), &x->attn, (size_t)R * Q));
  SQ_CUDA(ctx_alloc(x.get(), &x->attn_out, (size_t)R * E));
  SQ_CUDA(ctx_alloc(x.get(), &x->gate, (size_t)R * F));
  SQ_CUDA(ctx_alloc(x.get(), &x->up, (size_t)R * F));
  SQ_CUDA(ctx_alloc(x.get(), &x->act, (size_t)R * F));
  SQ_CUDA(ctx_alloc(x.get(), &x->ffn_out, (size_t)R * E));
  SQ_CUDA(ctx_alloc(x.get(), &x->logits, (size_t)c.vocab_size));
  const int widest = std::max(std::max(E, F), Q);
  SQ_CUDA(ctx_alloc(x.get(), (uint8_t **)&x->xq, (size_t)R * (widest / QK) * Q8_BYTES));
  x->gemm_ws_floats = (size_t)4 * R * widest;
  SQ_CUDA(ctx_alloc(x.get(), &x->gemm_ws, x->gemm_ws_floats));
  x->sdpa_part_floats = sdpa_max_partials_floats(c.head_dim);
  SQ_CUDA(ctx_alloc(x.get(), &x->sdpa_part, x->sdpa_part_floats));
  SQ_CUDA(ctx_alloc(x.get(), &x->sdpa_cnt, (size_t)SDPA_MAX_ROW_SPLITS));
  SQ_CUDA(cudaMemset(x->sdpa_cnt, 0, (size_t)SDPA_MAX_ROW_SPLITS * sizeof(int)));
  SQ_CUDA(ctx_alloc(x.get(), (uint8_t **)&x->argmax_part, (size_t)argmax_partials(c.vocab_size) * 32));
  SQ_CUDA(ctx_alloc(x.get(), &x->d_argmax, 1));
  SQ_CUDA(ctx_alloc(x.get(), &x->d_gpos, 1));
  if (m->tp_size > 1) {
    SQ_CUDA(ctx_alloc(x.get(), &x->logits_full, (size_t)m->cfg.vocab_size));
    SQ_CUDA(ctx_alloc(x.get(), (uint8_t **)&x->arg_local, argmax_state_bytes()));
    SQ_CUDA(ctx_alloc(x.get(), (uint8_t **)&x->arg_all, argmax_state_bytes() * m->tp_size));
  }
  SQ_CUDA(ctx_alloc(x.get(), &x->d_tokens, (size_t)R));
  SQ_CUDA(ctx_alloc(x.get(), &x->d_status, 8));
  SQ_CUDA(cudaHostAlloc((void **)&x->h_ids, (size_t)max_ctx * sizeof(uint32_t), cudaHostAllocDefault));
  SQ_CUDA(cudaHostAlloc((void **)&x->h_status, 8 * sizeof(unsigned long long), cudaHostAllocDefault));
  // RoPE table from the C library's sinf/cosf of pos * inv_freq[j] (rope.rs:25-26)
  const int half = c.head_dim / 2;
  std::vector<float> ct((size_t)max_ctx * half), stb((size_t)max_ctx * half);
  for (int p = 0; p < max_ctx; p++)
    for (int j = 0; j < half; j++) {
      const float theta = (float)p * m->inv_freq[j];
      ct[(size_t)p * half + j] = cosf(theta);
      stb[(size_t)p * half + j] = sinf(theta);
    }
  SQ_CUDA(ctx_alloc(x.get(), &x->d_cos, ct.size()));
  SQ_CUDA(ctx_alloc(x.get(), &x->d_sin, stb.size()));
  SQ_CUDA(cudaMemcpy(x->d_cos, ct.data(), ct.size() * 4, cudaMemcpyHostToDevice));
  SQ_CUDA(cudaMemcpy(x->d_sin, stb.data(), stb.size() * 4, cudaMemcpyHostToDevice));
  int st = decode_prepare(x.get());
  if (st) return st;
  *out = x.release();
  return SQ_OK;
}

extern "C" void sq_ctx_free(sq_ctx *c) { delete c; }

extern "C" int sq_ctx_reset(sq_ctx *c) {
  if (!c) return fail(SQ_ERR_ARG, "ctx_reset: null context");
  c->seq_len = 0;
  c->have_logits = false;
  return SQ_OK;
}

extern "C" int sq_ctx_seq_len(const sq_ctx *c, int *out) {
  if (!c || !out) return fail(SQ_ERR_ARG, "ctx_seq_len: null pointer");
  *out = c->seq_len;
  return SQ_OK;
}

extern "C" void *sq_ctx_stream(sq_ctx *c) { return c ? (void *)c->stream : nullptr; }

namespace sq {

// The one-row matvecs of layer l (decode through the op level): q/k/v and gate/up
// as one launch each, the norms, SiLU.mul (the gate/up epilogue) and (single GPU)
// residual adds folded in.
// Returns whether the streaming matvec takes all four.
static bool layer_matvecs(const sq_ctx *c, int l, MvArgs &qkv, MvArgs &o, MvArgs &gu, MvArgs &dn) {
  const sq_model *m = c->m;
  const sq_llama_config &cf = m->lc;
  const auto &L = m->layers[l];
  const int E = cf.embed_dim, Q = cf.n_heads * cf.head_dim, KVd = cf.n_kv_heads * cf.head_dim, F = cf.ffn_dim;
  const bool tp = m->tp_size > 1;
  qkv = MvArgs{}, o = MvArgs{}, gu = MvArgs{}, dn = MvArgs{};
  qkv.x = c->hidden, qkv.norm_w = L.attn_norm, qkv.eps = cf.rms_eps, qkv.in_dim = E, qkv.n = 3;
  qkv.w[0] = (const uint8_t *)L.q, qkv.w[1] = (const uint8_t *)L.k, qkv.w[2] = (const uint8_t *)L.v;
  qkv.out_dim[0] = Q, qkv.out_dim[1] = KVd, qkv.out_dim[2] = KVd;
  qkv.y[0] = c->q, qkv.y[1] = c->k, qkv.y[2] = c->v;
  o.x = c->attn, o.in_dim = Q, o.n = 1, o.w[0] = (const uint8_t *)L.o, o.out_dim[0] = E;
  o.y[0] = tp ? c->attn_out : c->hidden, o.res[0] = tp ? nullptr : c->hidden;
  gu.x = c->hidden, gu.norm_w = L.ffn_norm, gu.eps = cf.rms_eps, gu.in_dim = E, gu.n = 2;
  gu.w[0] = (const uint8_t *)L.gate, gu.w[1] = (const uint8_t *)L.up, gu.out_dim[0] = F, gu.out_dim[1] = F;
  gu.y[0] = c->gate, gu.y[1] = c->act, gu.gate_act = 1;  // SiLU(gate) * up formed in the epilogue
  dn.x = c->act, dn.in_dim = F, dn.n = 1, dn.w[0] = (const uint8_t *)L.down, dn.out_dim[0] = E;
  dn.y[0] = tp ? c->ffn_out : c->hidden, dn.res[0] = tp ? nullptr : c->hidden;
  const int wt = cf.weight_type;
  const bool aq = m->acts == SQ_ACTS_Q8 && wt != SQ_BF16;
  return !aq && matvec_fused_ok(qkv, wt) && matvec_fused_ok(o, wt) && matvec_fused_ok(gu, wt) &&
         matvec_fused_ok(dn, wt);
}

// The LM head of row `row` with the final norm folded in; whether the streaming
// matvec takes it.
static bool lm_matvec(const sq_ctx *c, int row, MvArgs &lm) {
  const sq_model *m = c->m;
  const sq_llama_config &cf = m->lc;
  const int E = cf.embed_dim;
  lm = MvArgs{};
  lm.x = c->hidden + (size_t)row * E, lm.norm_w = m->out_norm, lm.eps = cf.rms_eps, lm.in_dim = E, lm.n = 1;
  lm.w[0] = (const uint8_t *)m->out_w, lm.out_dim[0] = cf.vocab_size, lm.y[0] = c->logits;
  const bool lm_q8 = m->acts == SQ_ACTS_Q8 && m->out_type != SQ_BF16;
  return !lm_q8 && matvec_fused_ok(lm, m->out_type);
}

}  // namespace sq

// Kernels of ours one decode step launches (NCCL's not counted): the op-level
// sequence of forward_rows for one row plus the position counter, or the
// persistent decode kernel.
extern "C" int sq_ctx_launches_per_token(const sq_ctx *c, int *out) {
  if (!c || !out) return fail(SQ_ERR_ARG, "launches_per_token: null pointer");
  if (decode_available(c)) {
    *out = 1;
    return SQ_OK;
  }
  const sq_llama_config &cf = c->m->lc;
  const bool tp = c->m->tp_size > 1;
  const int aq = c->m->acts == SQ_ACTS_Q8 && cf.weight_type != SQ_BF16;
  int n = 1;  // embedding
  for (int l = 0; l < cf.n_blocks; l++) {
    sq::MvArgs a, b, g, d;
    // fused: qkv, rope+append, attention, o, gate/up, down (+ two residual adds after
    // the all-reduces); otherwise norm, q, k, v, rope+append, attention, o, add, norm,
    // gate, up, silu_mul, down, add (+ two activation quantizations)
    n += sq::layer_matvecs(c, l, a, b, g, d) ? 6 + (tp ? 2 : 0) : 14 + 2 * aq;
  }
  sq::MvArgs lm;
  n += sq::lm_matvec(c, 0, lm) ? 1 : 2;  // LM head (+ the final norm)
  n += 2;                                // argmax: partials and final (shards: state and fold)
  n += 1;                                // the device position counter
  *out = n;
  return SQ_OK;
}

namespace sq {

// One prefill chunk of n rows at position c->seq_len through every layer
// (layers.rs:81-109), then the LM head on the last row when `last`.
static int forward_rows(sq_ctx *c, const uint32_t *d_ids, int n, bool last, const int *pos_dev = nullptr) {
  const sq_model *m = c->m;
  const sq_llama_config &cf = m->lc;  // this rank's shard (the whole model when tp_size == 1)
  cudaStream_t s = c->stream;
  const int E = cf.embed_dim, Q = cf.n_heads * cf.head_dim, KVd = cf.n_kv_heads * cf.head_dim, F = cf.ffn_dim;
  const int wt = cf.weight_type;
  const int aq = m->acts == SQ_ACTS_Q8 && wt != SQ_BF16;
  const int pos = c->seq_len;
  const size_t layer_kv = (size_t)cf.n_kv_heads * c->max_ctx * cf.head_dim;
  const bool tp = m->tp_size > 1;
#define TRY(x)                                                  \
  do {                                                          \
    const cudaError_t e_ = (x);                                 \
    if (e_ != cudaSuccess) return cuda_fail(e_, "forward");     \
  } while (0)
#define TRY_ST(x)              \
  do {                         \
    const int st_ = (x);       \
    if (st_) return st_;       \
  } while (0)
  TRY(launch_embed(s, d_ids, n, m->embd, m->embd_type, E, m->cfg.vocab_size, c->hidden));  // replicated table
  float *ws = c->gemm_ws;
  const size_t wsf = c->gemm_ws_floats;
  // tensor-core layers on one GPU defer each residual add (elementwise_add.rs:47-61)
  // into the next RMSNorm's pass over the hidden rows (one read and write fewer)
  const float *pending = nullptr;
  for (int l = 0; l < cf.n_blocks; l++) {
    const auto &L = m->layers[l];
    float *kc = c->kc + l * layer_kv, *vc = c->vc + l * layer_kv;
    // Tensor-core layer: the normalised inputs and SiLU.mul go straight to the GEMMs'
    // bf16 terms (written once, shared by q/k/v and by gate/up); only the attention
    // output is split by a separate pass.
    const bool tcl = !aq && gemm_tc_enabled() && n >= 2 && rms_norm_terms_ok(c->hidden, L.attn_norm, E) &&
                     gemm_tc_supported(n, E, ws, L.q, wt, ws, wsf) && gemm_tc_supported(n, E, ws, L.k, wt, ws, wsf) &&
                     gemm_tc_supported(n, E, ws, L.v, wt, ws, wsf) && gemm_tc_supported(n, Q, ws, L.o, wt, ws, wsf) &&
                     gemm_tc_supported(n, E, ws, L.gate, wt, ws, wsf) && gemm_tc_supported(n, E, ws, L.up, wt, ws, wsf) &&
                     gemm_tc_supported(n, F, ws, L.down, wt, ws, wsf);
    // One-row layer (decode through the op level): the streaming matvec with the norm,
    // SiLU.mul and residual add folded in, q/k/v and gate/up as one launch each.
    MvArgs qkv, o, gu, dn;
    const bool fused = layer_matvecs(c, l, qkv, o, gu, dn) && n == 1;
    // the one-row step's kernels start while their predecessor finishes (each waits
    // for it before touching activations)
    const bool pdl = fused && pdl_enabled();
    if (pending && !tcl) {  // a deferred residual add that this layer's norm does not take
      TRY(launch_add(s, c->hidden, pending, (size_t)n * E));
      pending = nullptr;
    }
    if (fused) {
      TRY(launch_matvec_fused(s, qkv, wt, pdl));
    } else if (tcl) {
      if (pending) TRY(launch_add_rms_norm_terms(s, c->hidden, pending, L.attn_norm, ws, n, E, cf.rms_eps));
      else TRY(launch_rms_norm_terms(s, c->hidden, L.attn_norm, ws, n, E, cf.rms_eps));
      pending = nullptr;
      const void *wqkv[3] = {L.q, L.k, L.v};
      const int nqkv[3] = {Q, KVd, KVd};
      float *yqkv[3] = {c->q, c->k, c->v};
      TRY(launch_gemm_tc_terms_multi(s, n, E, 3, wqkv, wt, nqkv, yqkv, ws, wsf));
    } else {
      TRY(launch_rms_norm(s, c->hidden, L.attn_norm, c->normed, n, E, cf.rms_eps));
      if (aq) TRY(launch_quantize_q8_0(s, c->normed, (size_t)n * E, c->xq));  // shared quantization
      TRY(launch_linear(s, aq ? nullptr : c->normed, n, E, L.q, wt, Q, c->q, aq, c->xq, ws, wsf));
      TRY(launch_linear(s, aq ? nullptr : c->normed, n, E, L.k, wt, KVd, c->k, aq, c->xq, ws, wsf));
      TRY(launch_linear(s, aq ? nullptr : c->normed, n, E, L.v, wt, KVd, c->v, aq, c->xq, ws, wsf));
    }
    // pos_dev: positions come from the device counter (a captured decode step); the
    // attention then keeps the split count of the longest context
    TRY(launch_rope_append(s, c->q, c->k, c->v, kc, vc, n, Q, KVd, cf.head_dim, pos, c->max_ctx, c->d_cos, c->d_sin,
                           pos_dev, pdl));
    const long long khs = (long long)c->max_ctx * cf.head_dim;
    if (!pos_dev && attn_tc_supported(n, pos + n, cf.n_heads, cf.n_kv_heads, cf.head_dim, cf.head_dim, khs, c->q, kc,
                                      vc, c->gemm_ws_floats * sizeof(float))) {
      // tensor cores; the GEMM workspace is free between the projections
      TRY(launch_attn_tc(s, c->q, kc, vc, c->attn, n, pos + n, cf.n_heads, cf.n_kv_heads, cf.head_dim, cf.head_dim,
                         khs, c->gemm_ws, c->gemm_ws_floats * sizeof(float)));
    } else {
      const int ns = pos_dev ? sdpa_num_splits(n, c->max_ctx, cf.n_heads) : sdpa_num_splits(n, pos + n, cf.n_heads);
      TRY(launch_sdpa(s, c->q, kc, vc, c->attn, n, pos + n, cf.n_heads, cf.n_kv_heads, cf.head_dim, cf.head_dim, khs,
                      ns, c->sdpa_part, pos_dev, c->sdpa_cnt, pdl));
    }
    if (fused) {
      TRY(launch_matvec_fused(s, o, wt, pdl));  // single GPU: hidden += O.attn in the epilogue
    } else if (tcl) {
      TRY(launch_split_terms(s, c->attn, n, Q, ws));
      TRY(launch_gemm_tc_terms(s, n, Q, L.o, wt, E, c->attn_out, ws, wsf));
    } else {
      TRY(launch_linear(s, c->attn, n, Q, L.o, wt, E, c->attn_out, aq, c->xq, ws, wsf));
    }
    // row-parallel O: sum the shards, then the residual add (one peer-memory kernel for a decode row)
    if (tp && n == 1 && m->ar) {
      TRY(launch_allreduce_add(s, m->ar, c->hidden, c->attn_out, pdl));
    } else {
      if (tp) TRY_ST(nccl_all_reduce_sum(m->nccl, c->attn_out, (size_t)n * E, s));
      if (tcl && !tp) pending = c->attn_out;  // added by the FFN norm below
      else if (!fused || tp) TRY(launch_add(s, c->hidden, c->attn_out, (size_t)n * E));
    }
    if (fused) {
      TRY(launch_matvec_fused(s, gu, wt, pdl));
      TRY(launch_matvec_fused(s, dn, wt, pdl));
    } else if (tcl) {
      if (pending) TRY(launch_add_rms_norm_terms(s, c->hidden, pending, L.ffn_norm, ws, n, E, cf.rms_eps));
      else TRY(launch_rms_norm_terms(s, c->hidden, L.ffn_norm, ws, n, E, cf.rms_eps));
      pending = nullptr;
      const void *wgu[2] = {L.gate, L.up};
      const int ngu[2] = {F, F};
      float *ygu[2] = {c->gate, c->up};
      TRY(launch_gemm_tc_terms_multi(s, n, E, 2, wgu, wt, ngu, ygu, ws, wsf));
      TRY(launch_silu_mul_terms(s, c->gate, c->up, ws, (size_t)n * F));
      TRY(launch_gemm_tc_terms(s, n, F, L.down, wt, E, c->ffn_out, ws, wsf));
    } else {
      TRY(launch_rms_norm(s, c->hidden, L.ffn_norm, c->normed, n, E, cf.rms_eps));
      if (aq) TRY(launch_quantize_q8_0(s, c->normed, (size_t)n * E, c->xq));
      TRY(launch_linear(s, aq ? nullptr : c->normed, n, E, L.gate, wt, F, c->gate, aq, c->xq, ws, wsf));
      TRY(launch_linear(s, aq ? nullptr : c->normed, n, E, L.up, wt, F, c->up, aq, c->xq, ws, wsf));
      TRY(launch_silu_mul(s, c->gate, c->up, c->act, (size_t)n * F));
      TRY(launch_linear(s, c->act, n, F, L.down, wt, E, c->ffn_out, aq, c->xq, ws, wsf));
    }
    if (tp && n == 1 && m->ar) {  // row-parallel down, likewise
      TRY(launch_allreduce_add(s, m->ar, c->hidden, c->ffn_out, pdl));
    } else {
      if (tp) TRY_ST(nccl_all_reduce_sum(m->nccl, c->ffn_out, (size_t)n * E, s));
      if (tcl && !tp) pending = c->ffn_out;  // added by the next layer's attention norm
      else if (!fused || tp) TRY(launch_add(s, c->hidden, c->ffn_out, (size_t)n * E));
    }
  }
  if (pending) TRY(launch_add(s, c->hidden, pending, (size_t)n * E));  // the last layer's
  c->seq_len += n;
  if (last) {
    // final norm of the last row only: rows are normalized independently (model.rs:72-87)
    MvArgs lm;
    const bool lm_q8 = m->acts == SQ_ACTS_Q8 && m->out_type != SQ_BF16;
    if (lm_matvec(c, n - 1, lm)) {
      TRY(launch_matvec_fused(s, lm, m->out_type, n == 1 && pdl_enabled()));  // the norm folded into the LM head
    } else {
      TRY(launch_rms_norm(s, c->hidden + (size_t)(n - 1) * E, m->out_norm, c->normed, 1, E, cf.rms_eps));
      TRY(launch_linear(s, c->normed, 1, E, m->out_w, m->out_type, cf.vocab_size, c->logits, lm_q8, c->xq,
                        c->gemm_ws, c->gemm_ws_floats));
    }
    if (!tp) {
      TRY(launch_argmax(s, c->logits, cf.vocab_size, c->argmax_part, c->d_argmax));
    } else {  // greedy over the vocabulary shards: per-rank states, folded in rank (= index) order
      TRY(launch_argmax_state(s, c->logits, cf.vocab_size, m->vocab0, c->argmax_part, c->arg_local));
      TRY_ST(nccl_all_gather_bytes(m->nccl, c->arg_local, c->arg_all, argmax_state_bytes(), s));
      TRY(launch_argmax_fold(s, c->arg_all, m->tp_size, c->d_argmax));
    }
  }
#undef TRY
#undef TRY_ST
  return SQ_OK;
}

// One decode step of the op-level sequence (no persistent kernel: tensor-parallel
// contexts, shapes it does not take) from the token id in c->d_tokens. The first
// step runs eagerly; the second is captured into a CUDA graph - every kernel, and
// the NCCL calls of a tensor-parallel context, with positions read from the device
// counter c->d_gpos and a final kernel advancing it - and every later step is one
// graph launch. A capture that fails leaves the context on eager launches.
static int step_one(sq_ctx *c) {
  cudaStream_t s = c->stream;
  if (c->gpos != c->seq_len) {  // prefill or reset moved the host's count
    const cudaError_t e = launch_set_int(s, c->d_gpos, c->seq_len);
    if (e != cudaSuccess) return cuda_fail(e, "decode position");
    c->gpos = c->seq_len;
  }
  if (!c->step_graph && !c->graph_failed && c->eager_steps >= 1) {
    cudaGraph_t g = nullptr;
    int st = SQ_OK;
    cudaError_t e = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
    if (e == cudaSuccess) {
      const int saved = c->seq_len;
      st = forward_rows(c, c->d_tokens, 1, true, c->d_gpos);
      c->seq_len = saved;  // nothing ran during the capture
      if (!st) e = launch_add_int(s, c->d_gpos, 1);
      const cudaError_t e2 = cudaStreamEndCapture(s, &g);
      if (e == cudaSuccess) e = e2;
    }
    if (!st && e == cudaSuccess && g) e = cudaGraphInstantiate(&c->step_graph, g, 0);
    if (g) cudaGraphDestroy(g);
    if (st || e != cudaSuccess || !c->step_graph) {
      c->graph_failed = true;
      c->step_graph = nullptr;
      cudaGetLastError();  // clear the capture's error; eager launches from here on
    }
  }
  if (c->step_graph) {
    const cudaError_t e = cudaGraphLaunch(c->step_graph, s);
    if (e != cudaSuccess) return cuda_fail(e, "decode step graph");
    c->seq_len += 1;
    c->gpos = c->seq_len;
    return SQ_OK;
  }
  c->eager_steps++;
  const int st = forward_rows(c, c->d_tokens, 1, true);
  c->gpos = -1;  // the device counter did not advance
  return st;
}

// Model::forward for ids already on the device (prefill in chunks; decode of one
// token through the persistent decode kernel when it is available).
int forward_device(sq_ctx *c, const uint32_t *d_ids, int n) {
  if (n == 1 && decode_available(c)) return decode_launch(c, const_cast<uint32_t *>(d_ids), nullptr, 0);
  for (int r0 = 0; r0 < n; r0 += c->ws_rows) {
    const int rows = std::min(c->ws_rows, n - r0);
    const int st = forward_rows(c, d_ids + r0, rows, r0 + rows == n);
    if (st) return st;
  }
  return SQ_OK;
}

}  // namespace sq

static int check_ids(sq_ctx *c, const uint32_t *ids, size_t n) {
  if (!ids) return fail(SQ_ERR_ARG, "forward: null ids");
  if (n == 0) return fail(SQ_ERR_EMPTY, "forward: no token ids");  // model.rs:57-61
  if ((size_t)c->seq_len + n > (size_t)c->max_ctx) return fail(SQ_ERR_CAPACITY, "forward: KV cache full");
  for (size_t i = 0; i < n; i++)
    if (ids[i] >= (uint32_t)c->m->cfg.vocab_size) return fail(SQ_ERR_SHAPE, "forward: token id out of range");
  return SQ_OK;
}

// The end of a model-level call: one launch gathers the argmax and every bounded-wait
// error word the call's kernels may have set (decode kernel, streaming matvec,
// tensor-core kernels, peer all-reduce) into one buffer, one copy brings it to pinned
// host memory, one stream sync. Only when a word is set do the per-kernel status
// reads (which clear the words and name the kernel) run.
static int finish_call(sq_ctx *c, const char *what, long long *id) {
  const unsigned *ar_err = c->m->ar ? tp_allreduce_err_ptr(c->m->ar) : nullptr;
  SQ_CUDA(launch_collect_status(c->stream, c->d_argmax, decode_err_ptr(c), mv_err_ptr(), tc_err_ptr(), ar_err,
                                c->d_status));
  SQ_CUDA(cudaMemcpyAsync(c->h_status, c->d_status, 5 * sizeof(unsigned long long), cudaMemcpyDeviceToHost,
                          c->stream));
  SQ_CUDA(cudaStreamSynchronize(c->stream));
  const unsigned long long *hs = c->h_status;
  if (hs[1] || decode_check_always(c)) {
    const int st = decode_check(c);
    if (st) return st;
  }
  if (hs[2] || hs[3]) {
    const int st = device_wait_status(true, what);
    if (st) return st;
  }
  if (hs[4] && tp_allreduce_status(c->m->ar, true))
    return fail(SQ_ERR_TIMEOUT, std::string(what) +
                                    ": a peer's partial sum did not arrive within the tensor-parallel all-reduce's limit");
  if (id) *id = (long long)hs[0];
  return SQ_OK;
}

extern "C" int sq_forward(sq_ctx *c, const uint32_t *ids, size_t n, uint32_t *out_argmax) {
  if (!c) return fail(SQ_ERR_ARG, "forward: null context");
  int st = check_ids(c, ids, n);
  if (st) return st;
  SQ_CUDA(cudaSetDevice(c->m->device));
  memcpy(c->h_ids, ids, n * sizeof(uint32_t));  // pinned staging (the previous call's copies have finished)
  for (size_t r0 = 0; r0 < n; r0 += c->ws_rows) {
    const int rows = (int)std::min((size_t)c->ws_rows, n - r0);
    SQ_CUDA(cudaMemcpyAsync(c->d_tokens, c->h_ids + r0, rows * sizeof(uint32_t), cudaMemcpyHostToDevice, c->stream));
    if (rows == 1 && r0 == 0 && decode_available(c)) {
      st = decode_launch(c, c->d_tokens, nullptr, 0);
    } else if (n == 1) {
      st = step_one(c);
    } else {
      st = forward_rows(c, c->d_tokens, rows, r0 + rows == n);
    }
    if (st) return st;
  }
  c->have_logits = true;
  long long id = 0;
  st = finish_call(c, "forward", &id);
  if (st) return st;
  if (out_argmax) *out_argmax = (uint32_t)id;
  return SQ_OK;
}

extern "C" int sq_ctx_logits(sq_ctx *c, float *out, size_t n) {
  if (!c || !out) return fail(SQ_ERR_ARG, "ctx_logits: null pointer");
  if (n != (size_t)c->m->cfg.vocab_size) return fail(SQ_ERR_SHAPE, "ctx_logits: buffer must hold vocab_size floats");
  if (!c->have_logits) return fail(SQ_ERR_EMPTY, "ctx_logits: no forward pass yet");
  SQ_CUDA(cudaSetDevice(c->m->device));
  const float *src = c->logits;
  if (c->m->tp_size > 1) {  // vocabulary shards gathered in rank order: every rank of the group calls this
    const int st = nccl_all_gather_bytes(c->m->nccl, c->logits, c->logits_full,
                                         (size_t)c->m->lc.vocab_size * sizeof(float), c->stream);
    if (st) return st;
    src = c->logits_full;
  }
  SQ_CUDA(cudaMemcpyAsync(out, src, n * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
  SQ_CUDA(cudaStreamSynchronize(c->stream));
  return SQ_OK;
}

extern "C" int sq_generate(sq_ctx *c, const uint32_t *prompt, size_t n_prompt, int max_tokens, int ignore_eos,
                           uint32_t *out_ids, float *step_ms, int *n_out) {
  if (!c || !out_ids || !n_out) return fail(SQ_ERR_ARG, "generate: null pointer");
  *n_out = 0;
  std::vector<uint32_t> input(prompt, prompt + n_prompt);
  for (int step = 1; step <= max_tokens; step++) {  // text_generator.rs:61-97
    auto t0 = std::chrono::steady_clock::now();
    uint32_t next = 0;
    int st = sq_forward(c, input.data(), input.size(), &next);
    if (st) return st;
    auto t1 = std::chrono::steady_clock::now();
    if (step_ms) step_ms[step - 1] = std::chrono::duration<float, std::milli>(t1 - t0).count();
    if (next == c->m->cfg.eos_token_id && !ignore_eos) break;
    out_ids[(*n_out)++] = next;
    input.assign(1, next);
  }
  return SQ_OK;
}

extern "C" int sq_decode_steps(sq_ctx *c, int n_steps, uint32_t *out_ids) {
  if (!c || !out_ids) return fail(SQ_ERR_ARG, "decode_steps: null pointer");
  if (n_steps <= 0) return SQ_OK;
  if (c->seq_len == 0) return fail(SQ_ERR_EMPTY, "decode_steps: context holds no position yet");
  if ((size_t)c->seq_len + n_steps > (size_t)c->max_ctx) return fail(SQ_ERR_CAPACITY, "decode_steps: KV cache full");
  SQ_CUDA(cudaSetDevice(c->m->device));
  if (n_steps > c->out_cap) {  // grow the context's id buffer (kept across calls)
    SQ_CUDA(cudaStreamSynchronize(c->stream));
    cudaFree(c->d_out_ids);
    c->d_out_ids = nullptr;
    c->out_cap = 0;
    SQ_CUDA(cudaMalloc((void **)&c->d_out_ids, (size_t)n_steps * sizeof(uint32_t)));
    c->out_cap = n_steps;
  }
  uint32_t *d_out = c->d_out_ids;
  // the previous forward's argmax is the first input
  cudaError_t e = launch_feedback(c->stream, c->d_argmax, c->d_tokens, nullptr, 0);
  int st = e == cudaSuccess ? SQ_OK : cuda_fail(e, "decode_steps");
  for (int i = 0; i < n_steps && !st; i++) {
    if (decode_available(c)) {
      st = decode_launch(c, c->d_tokens, d_out, i);
    } else {
      st = step_one(c);
      if (!st) {
        e = launch_feedback(c->stream, c->d_argmax, c->d_tokens, d_out, i);
        st = e == cudaSuccess ? SQ_OK : cuda_fail(e, "decode_steps");
      }
    }
  }
  if (!st) {
    cudaError_t e2 = cudaMemcpyAsync(c->h_ids, d_out, n_steps * sizeof(uint32_t), cudaMemcpyDeviceToHost, c->stream);
    if (e2 != cudaSuccess) st = cuda_fail(e2, "decode_steps copy");
  }
  if (!st) st = finish_call(c, "decode_steps", nullptr);  // synchronizes the stream
  if (st) {
    cudaStreamSynchronize(c->stream);  // nothing of this call is left running
    decode_check(c);                   // and the decode kernel's counters are reset
  } else {
    memcpy(out_ids, c->h_ids, n_steps * sizeof(uint32_t));
  }
  c->have_logits = true;
  return st;
}
