// allreduce.cu — one-shot all-reduce over NVLink peer memory for the tensor-parallel
// decode step, fused with the residual add that follows it.
//
// The reference runs on one CPU; in the tensor-parallel 8B configuration the two
// row-parallel projections of every layer (O, layers.rs:57, and down, layers.rs:76)
// leave each rank a partial sum of the hidden vector, which must be summed over the
// ranks before the residual adds (layers.rs:96 and :106). For one decode row that
// is 4096 floats (16 KB): NCCL's ring/tree all-reduce is latency-bound there. This
// kernel does it in one pass and adds the sum to the residual:
//
//   - every rank owns a mailbox in its own HBM: data [2][world][E] floats and flags
//     [2][world][nb] words (two slots, used alternately by consecutive all-reduces);
//   - CTA c of the kernel owns elements [c E/nb, (c+1) E/nb): it stores this rank's
//     partial for them into slot s, row `rank`, of EVERY rank's mailbox (plain
//     stores through the peer mappings, over NVLink), then, after a barrier, thread r
//     writes the sequence number into rank r's flag [s][rank][c] with a system-scope
//     release store;
//   - thread r then polls its own mailbox's flag [s][r][c] (acquire, bounded by a
//     clock limit) until rank r's data are there, and the CTA sums the world rows in
//     rank order - the same order on every rank, so every rank gets the same bits -
//     and adds them to its residual.
//
// Sequence numbers come from per-CTA counters in device memory (epoch[c]), so a
// captured CUDA graph replays correctly. A rank can be at most one all-reduce ahead
// of any other (it cannot finish all-reduce k+1 without everyone's partial k+1,
// which each rank writes only after finishing k), so two slots suffice.
//
// No TMA, no bulk copy and no multicast touches peer memory: the peer traffic is
// plain 16-byte stores. Every wait gives up after about a second, sets an error word
// (tp_allreduce_status) and lets the CTA finish.
#include <cuda_runtime.h>
#include <stdlib.h>
#include <string.h>

#include <string>
#include <vector>

#include "../host/model.h"
#include "common.cuh"
#include "ops.cuh"
#include "status.h"

namespace sq {

constexpr int AR_THREADS = 128;
constexpr int AR_MAX_WORLD = 8;
constexpr long long AR_WAIT_LIMIT = 2000000000LL;  // ~1 s of SM clocks

struct TpAllReduce {
  int world = 0, rank = 0, E = 0, nb = 0;
  void *local = nullptr;               // this rank's mailbox (cudaMalloc)
  std::vector<void *> mapped;          // base of every rank's mailbox in this process (peer mappings)
  float **d_data = nullptr;            // device array: data base of each rank's mailbox
  unsigned **d_flags = nullptr;        // device array: flag base of each rank's mailbox
  unsigned *epoch = nullptr, *err = nullptr;  // this rank's per-CTA sequence counters and error word
  // Failure-detection tests only (SQ_TEST_WITHHOLD_PARTIAL=k, read when the model is
  // created): the k-th all-reduce this rank launches (or captures) stores its partial
  // but not its flags, so the other ranks' waits for it expire. 0 = off.
  unsigned withhold = 0, launches = 0;
  // the persistent decode kernel's exchange area in every rank's mailbox (after the
  // all-reduce's data and flags): [2][world][E] tagged words for the O / down
  // partials, then [world][3] for the ranks' argmax states
  std::vector<unsigned long long *> dec_box;
  size_t bytes = 0;
};

// Bytes of a mailbox: the all-reduce's data and flags, then the decode kernel's area.
static size_t mailbox_bytes(int world, int E, int nb, size_t *data_b, size_t *flag_b, size_t *dec_b) {
  auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
  *data_b = al((size_t)2 * world * E * sizeof(float));
  *flag_b = al((size_t)2 * world * nb * sizeof(unsigned));
  *dec_b = al(((size_t)2 * world * E + (size_t)world * 3) * sizeof(unsigned long long));
  return *data_b + *flag_b + *dec_b;
}

namespace {

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ float4 ldcg4(const float *p) { return __ldcg(reinterpret_cast<const float4 *>(p)); }

__global__ void __launch_bounds__(AR_THREADS) k_allreduce_add(float *hidden, const float *part, float *const *data,
                                                              unsigned *const *flags, unsigned *epoch, unsigned *err,
                                                              int rank, int world, int E, int nb, int withhold) {
  const int c = blockIdx.x, tid = threadIdx.x;
  const int chunk = E / nb, e0 = c * chunk;
  pdl_wait();     // the partial comes from the kernel before (programmatic launch)
  pdl_trigger();  // the next kernel may start streaming its weights meanwhile
  __shared__ unsigned s_seq;
  if (tid == 0) s_seq = epoch[c] + 1u;
  __syncthreads();
  const unsigned seq = s_seq;
  const int slot = (int)(seq & 1u);
  // 1. this rank's partial into row `rank` of slot `slot` of every mailbox
  const size_t row = ((size_t)slot * world + rank) * E + e0;
  for (int i = tid; i < chunk / 4; i += AR_THREADS) {
    const float4 v = ldcg4(part + e0 + 4 * i);
    for (int r = 0; r < world; r++) *reinterpret_cast<float4 *>(data[r] + row + 4 * i) = v;
  }
  __syncthreads();  // every thread's stores precede the releases below
  if (tid < world && !withhold) st_release_sys(flags[tid] + ((size_t)slot * world + rank) * nb + c, seq);
  // 2. wait for every rank's row in this rank's own mailbox
  if (tid < world) {
    const unsigned *f = flags[rank] + ((size_t)slot * world + tid) * nb + c;
    const long long t0 = clock64();
    for (unsigned it = 0; ld_acquire_sys(f) != seq; it++) {
      if ((it & 63u) == 63u) {
        if (*(volatile unsigned *)err) break;
        if (clock64() - t0 > AR_WAIT_LIMIT) {
          atomicExch(err, 1u);
          break;
        }
      }
    }
  }
  __syncthreads();
  // 3. the sum in rank order (identical on every rank), added to the residual
  const float *mine = data[rank] + (size_t)slot * world * E + e0;
  for (int i = tid; i < chunk / 4; i += AR_THREADS) {
    float4 s = ldcg4(mine + 4 * i);
    for (int r = 1; r < world; r++) {
      const float4 v = ldcg4(mine + (size_t)r * E + 4 * i);
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
    float4 *h = reinterpret_cast<float4 *>(hidden + e0) + i;
    float4 hv = *h;
    hv.x += s.x;
    hv.y += s.y;
    hv.z += s.z;
    hv.w += s.w;
    *h = hv;
  }
  if (tid == 0) epoch[c] = seq;
}

size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

}  // namespace

// Collective over the model's NCCL group: every rank calls it in the same order. On
// success m->ar is set; when a rank cannot map its peers' memory (no peer access),
// every rank keeps the NCCL all-reduce (m->ar stays null) and SQ_OK is returned.
int tp_allreduce_create(sq_model *m) {
  const int world = m->tp_size, rank = m->tp_rank, E = m->cfg.embed_dim;
  if (world < 2 || world > AR_MAX_WORLD || E % 512) return SQ_OK;
  if (const char *v = getenv("SQB200_TP_ALLREDUCE"))
    if (strcmp(v, "nccl") == 0) return SQ_OK;
  SQ_CUDA(cudaSetDevice(m->device));
  auto *ar = new TpAllReduce();
  ar->world = world;
  ar->rank = rank;
  ar->E = E;
  ar->nb = E >= 4096 ? 8 : E / 512;
  if (const char *v = getenv("SQ_TEST_WITHHOLD_PARTIAL")) ar->withhold = (unsigned)strtoul(v, nullptr, 10);
  size_t data_b = 0, flag_b = 0, dec_b = 0;
  const size_t bytes = mailbox_bytes(world, E, ar->nb, &data_b, &flag_b, &dec_b);
  ar->bytes = bytes;
  int ok = 1;
  std::string why;
  cudaIpcMemHandle_t mine{};
  if (cudaMalloc(&ar->local, bytes) != cudaSuccess || cudaMemset(ar->local, 0, bytes) != cudaSuccess ||
      cudaMalloc((void **)&ar->epoch, align256(ar->nb * sizeof(unsigned)) + 256) != cudaSuccess ||
      cudaMemset(ar->epoch, 0, align256(ar->nb * sizeof(unsigned)) + 256) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess || cudaIpcGetMemHandle(&mine, ar->local) != cudaSuccess) {
    ok = 0;
    why = "mailbox allocation or IPC handle";
    cudaGetLastError();
  }
  ar->err = (unsigned *)((uint8_t *)ar->epoch + align256(ar->nb * sizeof(unsigned)));
  // every rank's handle and status, gathered through NCCL (the mailboxes are zeroed
  // before any rank can learn a handle, so no peer writes into an unzeroed mailbox)
  struct Entry {
    cudaIpcMemHandle_t h;
    int ok;
    int pad[15];
  };
  Entry me{};
  me.h = mine;
  me.ok = ok;
  Entry *d_all = nullptr;
  std::vector<Entry> all(world);
  int st = SQ_OK;
  if (cudaMalloc((void **)&d_all, world * sizeof(Entry)) != cudaSuccess) {
    delete ar;
    return fail(SQ_ERR_CUDA, "tp all-reduce: handle buffer");
  }
  cudaMemcpy(d_all + rank, &me, sizeof(Entry), cudaMemcpyHostToDevice);
  st = nccl_all_gather_bytes(m->nccl, d_all + rank, d_all, sizeof(Entry), 0);
  if (!st && cudaStreamSynchronize(0) != cudaSuccess) st = fail(SQ_ERR_CUDA, "tp all-reduce: handle exchange");
  if (!st) cudaMemcpy(all.data(), d_all, world * sizeof(Entry), cudaMemcpyDeviceToHost);
  cudaFree(d_all);
  if (st) {
    cudaFree(ar->local);
    cudaFree(ar->epoch);
    delete ar;
    return st;
  }
  ar->mapped.assign(world, nullptr);
  ar->mapped[rank] = ar->local;
  int mapped_ok = 1;
  for (int r = 0; r < world; r++) mapped_ok &= all[r].ok;
  for (int r = 0; r < world && mapped_ok; r++) {
    if (r == rank) continue;
    if (cudaIpcOpenMemHandle(&ar->mapped[r], all[r].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      mapped_ok = 0;
      ar->mapped[r] = nullptr;
    }
  }
  // all ranks agree: the peer path only if every rank mapped every peer
  int *d_flag = nullptr;
  int agree = mapped_ok;
  if (cudaMalloc((void **)&d_flag, sizeof(int)) == cudaSuccess) {
    cudaMemcpy(d_flag, &agree, sizeof(int), cudaMemcpyHostToDevice);
    st = nccl_all_reduce_min_int(m->nccl, d_flag, 0);
    if (!st && cudaStreamSynchronize(0) == cudaSuccess) cudaMemcpy(&agree, d_flag, sizeof(int), cudaMemcpyDeviceToHost);
    else agree = 0;
    cudaFree(d_flag);
  } else {
    agree = 0;
  }
  if (!agree || st) {
    tp_allreduce_release(ar);
    return st;
  }
  std::vector<float *> data(world);
  std::vector<unsigned *> flags(world);
  for (int r = 0; r < world; r++) {
    data[r] = (float *)ar->mapped[r];
    flags[r] = (unsigned *)((uint8_t *)ar->mapped[r] + data_b);
    ar->dec_box.push_back((unsigned long long *)((uint8_t *)ar->mapped[r] + data_b + flag_b));
  }
  if (cudaMalloc((void **)&ar->d_data, world * sizeof(float *)) != cudaSuccess ||
      cudaMalloc((void **)&ar->d_flags, world * sizeof(unsigned *)) != cudaSuccess ||
      cudaMemcpy(ar->d_data, data.data(), world * sizeof(float *), cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(ar->d_flags, flags.data(), world * sizeof(unsigned *), cudaMemcpyHostToDevice) != cudaSuccess) {
    tp_allreduce_release(ar);
    return fail(SQ_ERR_CUDA, "tp all-reduce: pointer tables");
  }
  m->ar = ar;
  return SQ_OK;
}

void tp_allreduce_release(TpAllReduce *ar) {
  if (!ar) return;
  for (int r = 0; r < (int)ar->mapped.size(); r++)
    if (r != ar->rank && ar->mapped[r]) cudaIpcCloseMemHandle(ar->mapped[r]);
  cudaFree(ar->local);
  cudaFree(ar->epoch);
  cudaFree(ar->d_data);
  cudaFree(ar->d_flags);
  delete ar;
}

cudaError_t launch_allreduce_add(cudaStream_t s, TpAllReduce *ar, float *hidden, const float *part, bool pdl) {
  const int withhold = ar->withhold && ++ar->launches == ar->withhold;
  return launch_ex(k_allreduce_add, dim3(ar->nb), dim3(AR_THREADS), 0, s, pdl, hidden, part,
                   (float *const *)ar->d_data, (unsigned *const *)ar->d_flags, ar->epoch, ar->err, ar->rank, ar->world,
                   ar->E, ar->nb, withhold);
}

// Collective re-synchronization after a timeout: a barrier (every rank's last
// all-reduce kernel has finished writing into the mailboxes), each rank zeroes its
// own mailbox flags, sequence counters and error word, a second barrier (no rank
// writes into a mailbox before its owner has zeroed it).
int tp_allreduce_recover(sq_model *m) {
  TpAllReduce *ar = m->ar;
  if (!ar) return SQ_OK;
  SQ_CUDA(cudaSetDevice(m->device));
  SQ_CUDA(cudaDeviceSynchronize());
  int *d = nullptr;
  SQ_CUDA(cudaMalloc((void **)&d, sizeof(int)));
  int st = nccl_all_reduce_min_int(m->nccl, d, 0);
  cudaError_t e = st ? cudaSuccess : cudaStreamSynchronize(0);
  if (!st && e == cudaSuccess) e = cudaMemset(ar->local, 0, ar->bytes);
  if (!st && e == cudaSuccess) e = cudaMemset(ar->epoch, 0, align256(ar->nb * sizeof(unsigned)) + 256);
  if (!st && e == cudaSuccess) e = cudaDeviceSynchronize();
  if (!st && e == cudaSuccess) st = nccl_all_reduce_min_int(m->nccl, d, 0);
  if (!st && e == cudaSuccess) e = cudaStreamSynchronize(0);
  cudaFree(d);
  if (st) return st;
  return e == cudaSuccess ? SQ_OK : cuda_fail(e, "tp_recover");
}

unsigned *tp_allreduce_err_ptr(const TpAllReduce *ar) { return ar ? ar->err : nullptr; }

int tp_decode_boxes(const TpAllReduce *ar, unsigned long long **boxes, int max) {
  if (!ar || (int)ar->dec_box.size() != ar->world || ar->world > max) return 0;
  for (int r = 0; r < ar->world; r++) boxes[r] = ar->dec_box[r];
  return ar->world;
}

unsigned tp_allreduce_status(const TpAllReduce *ar, bool clear) {
  if (!ar) return 0;
  unsigned v = 0;
  cudaMemcpy(&v, ar->err, sizeof(v), cudaMemcpyDeviceToHost);
  if (clear && v) cudaMemset(ar->err, 0, sizeof(unsigned));
  return v;
}

}  // namespace sq

extern "C" int sq_tp_recover(sq_model *m) {
  if (!m) return sq::fail(SQ_ERR_ARG, "tp_recover: null model");
  return sq::tp_allreduce_recover(m);
}
