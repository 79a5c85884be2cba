// argmax_noalloc.cu — sq_argmax_noalloc: the greedy argmax of sq_argmax with its
// per-chunk partial states kept in a fixed buffer of this library's static device
// memory instead of stream-ordered allocations. It launches the same two kernels
// as sq_argmax (k_argmax_partial, k_argmax_final via launch_argmax), so its result
// is the same index; only where the partials live differs.
#include <mutex>

#include "../../include/squirrel_cuda.h"
#include "common.cuh"
#include "ops.cuh"
#include "status.h"

namespace sq {

// One partial state per 4096-element chunk of the logits: SQ_ARGMAX_NOALLOC_MAX_N
// elements need 4096 states (96 KiB). Every state the final pass reads is written
// by the partial pass of the same call, so nothing needs clearing between calls.
constexpr int NOALLOC_ARGMAX_STATES = 4096;
static_assert(sizeof(ArgState) == 24, "the 96 KiB figure counts 24-byte states");
static __device__ __align__(256) ArgState g_argmax_states[NOALLOC_ARGMAX_STATES];

// Device address of g_argmax_states, looked up once per device with that device
// current (the first call on each device; later calls only read the table).
constexpr int NOALLOC_MAX_DEVICES = 64;
static void *g_states_addr[NOALLOC_MAX_DEVICES];
static std::mutex g_states_mu;

static int states_address(void **out) {
  int dev = 0;
  SQ_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return fail(SQ_ERR_ARG, "argmax_noalloc: device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_states_mu);
  if (!g_states_addr[dev]) SQ_CUDA(cudaGetSymbolAddress(&g_states_addr[dev], g_argmax_states));
  *out = g_states_addr[dev];
  return SQ_OK;
}

}  // namespace sq

extern "C" int sq_argmax_noalloc(void *stream, const float *logits, size_t n, int64_t *out_index) {
  using namespace sq;
  if (!logits || !out_index) return fail(SQ_ERR_ARG, "argmax_noalloc: null pointer");
  if (!n) return fail(SQ_ERR_EMPTY, "argmax_noalloc: empty logits");
  if (n > (size_t)SQ_ARGMAX_NOALLOC_MAX_N || argmax_partials(n) > NOALLOC_ARGMAX_STATES)
    return fail(SQ_ERR_ARG, "argmax_noalloc: n = " + std::to_string(n) + " exceeds the fixed scratch limit of " +
                                std::to_string((size_t)SQ_ARGMAX_NOALLOC_MAX_N) + " elements (use sq_argmax)");
  void *states = nullptr;
  const int st = states_address(&states);
  if (st != SQ_OK) return st;
  cudaError_t e = launch_argmax((cudaStream_t)stream, logits, n, states, (long long *)out_index);
  return e == cudaSuccess ? SQ_OK : cuda_fail(e, "sq_argmax_noalloc");
}
