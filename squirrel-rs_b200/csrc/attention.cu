// attention.cu — causal GQA attention for the op-level ABI and prefill
// (kernels/attention.rs:11-70 semantics: scores = (q.k) * 1/sqrt(hd) over keys
// 0..=offset+t, max-subtracted softmax, probability-weighted sum of V).
//
// One CTA per (query row t, head h, key split). Each of the 4 warps walks a
// strided subset of the split's keys, four consecutive keys at a time, with an
// online softmax (running max m, running sum l, accumulator a[d]); lanes own
// head_dim/32 dimensions each, so K
// and V rows are read coalesced. Warp states are merged in shared memory; with
// one split the CTA writes out = a * (1/l), otherwise it writes (m, l, a) and the
// splits are merged in split order: by k_sdpa_combine, or (with a counter per query
// row) by the row's last CTA to finish, which saves a launch per call.
#include <math.h>

#include "common.cuh"
#include "ops.cuh"

namespace sq {

constexpr int SDPA_WARPS = 4;
constexpr int SDPA_KPI = 4;  // keys a warp iteration
constexpr int SDPA_MAX_HD = 256;

// Merge the n_split partials (m, l, a[hd]) of one query row in split order
// (splits without keys carry l = 0 and are skipped); threads stride the dimensions.
__device__ __forceinline__ void combine_row(const float *pp, float *out_row, int n_split, int hd) {
  float M = -INFINITY;
  for (int i = 0; i < n_split; i++)
    if (__ldcg(pp + i * (hd + 2) + 1) > 0.f) M = fmaxf(M, __ldcg(pp + i * (hd + 2)));
  float L = 0.f;
  for (int i = 0; i < n_split; i++) {
    const float l = __ldcg(pp + i * (hd + 2) + 1);
    if (l > 0.f) L = fmaf(l, expf(__ldcg(pp + i * (hd + 2)) - M), L);
  }
  const float inv = 1.0f / L;
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float a = 0.f;
    for (int i = 0; i < n_split; i++) {
      const float l = __ldcg(pp + i * (hd + 2) + 1);
      if (l > 0.f) a = fmaf(__ldcg(pp + i * (hd + 2) + 2 + d), expf(__ldcg(pp + i * (hd + 2)) - M), a);
    }
    out_row[d] = a * inv;
  }
}

__global__ void k_sdpa_combine(const float *__restrict__ part, float *__restrict__ out, int n_split, int hd) {
  const int row = blockIdx.x;
  combine_row(part + (size_t)row * n_split * (hd + 2), out + (size_t)row * hd, n_split, hd);
}

template <int DPL>  // dims per lane = head_dim / 32
__global__ void __launch_bounds__(SDPA_WARPS * 32)
    k_sdpa(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
           float *__restrict__ out, float *__restrict__ part, int seq_q, int seq_k, int n_heads,
           int group, long long kps, long long khs, int split_len, float scale, const int *__restrict__ pos_dev,
           int *__restrict__ split_cnt) {
  const int hd = DPL * 32;
  pdl_wait();  // q and the cache come from earlier kernels
  pdl_trigger();
  if (pos_dev) {  // the keys end at the position the device holds (graph replay: no host values)
    seq_k = *pos_dev + seq_q;
    split_len = (seq_k + (int)gridDim.y - 1) / (int)gridDim.y;
  }
  const int row = blockIdx.x;  // t * n_heads + h
  const int split = blockIdx.y, n_split = gridDim.y;
  const int t = row / n_heads, h = row % n_heads, g = h / group;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int live = seq_k - seq_q + t + 1;
  const int k0 = split * split_len;
  const int k1 = min(live, k0 + split_len);

  float qv[DPL];
#pragma unroll
  for (int i = 0; i < DPL; i++) qv[i] = q[(size_t)row * hd + lane + 32 * i];

  float m = -INFINITY, l = 0.f, acc[DPL];
#pragma unroll
  for (int i = 0; i < DPL; i++) acc[i] = 0.f;

  const float *kb = k + g * khs, *vb = v + g * khs;
  // four consecutive keys a warp iteration: their loads, dots and reductions are
  // independent, so one key's latency hides behind the others'
  for (int s = k0 + SDPA_KPI * wid; s < k1; s += SDPA_KPI * SDPA_WARPS) {
    float d[SDPA_KPI], vv[SDPA_KPI][DPL];
#pragma unroll
    for (int j = 0; j < SDPA_KPI; j++) {
      d[j] = 0.f;
      if (s + j < k1) {
        const float *kr = kb + (size_t)(s + j) * kps, *vr = vb + (size_t)(s + j) * kps;
#pragma unroll
        for (int i = 0; i < DPL; i++) {
          d[j] = fmaf(qv[i], kr[lane + 32 * i], d[j]);
          vv[j][i] = vr[lane + 32 * i];
        }
      } else {
#pragma unroll
        for (int i = 0; i < DPL; i++) vv[j][i] = 0.f;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int j = 0; j < SDPA_KPI; j++) d[j] += __shfl_xor_sync(0xffffffffu, d[j], o);
    float sc[SDPA_KPI], mn = m;
#pragma unroll
    for (int j = 0; j < SDPA_KPI; j++) {
      sc[j] = s + j < k1 ? d[j] * scale : -INFINITY;
      mn = fmaxf(mn, sc[j]);
    }
    const float corr = expf(m - mn);  // 0 on the first keys (m = -inf); key s is always live
    float p[SDPA_KPI], ps = 0.f;
#pragma unroll
    for (int j = 0; j < SDPA_KPI; j++) {
      p[j] = expf(sc[j] - mn);  // 0 past the live keys
      ps += p[j];
    }
    l = l * corr + ps;
#pragma unroll
    for (int i = 0; i < DPL; i++) {
      float a = acc[i] * corr;
#pragma unroll
      for (int j = 0; j < SDPA_KPI; j++) a = fmaf(p[j], vv[j][i], a);
      acc[i] = a;
    }
    m = mn;
  }

  __shared__ float sm_m[SDPA_WARPS], sm_l[SDPA_WARPS];
  __shared__ float sm_a[SDPA_WARPS][SDPA_MAX_HD];
  if (lane == 0) {
    sm_m[wid] = m;
    sm_l[wid] = l;
  }
#pragma unroll
  for (int i = 0; i < DPL; i++) sm_a[wid][lane + 32 * i] = acc[i];
  __syncthreads();
  if (wid == 0) {
    float M = -INFINITY;
    for (int w = 0; w < SDPA_WARPS; w++) M = fmaxf(M, sm_m[w]);
    float L = 0.f, A[DPL];
#pragma unroll
    for (int i = 0; i < DPL; i++) A[i] = 0.f;
    for (int w = 0; w < SDPA_WARPS; w++) {
      const float f = (sm_l[w] > 0.f) ? expf(sm_m[w] - M) : 0.f;
      L = fmaf(sm_l[w], f, L);
#pragma unroll
      for (int i = 0; i < DPL; i++) A[i] = fmaf(sm_a[w][lane + 32 * i], f, A[i]);
    }
    if (n_split == 1) {
      const float inv = 1.0f / L;
#pragma unroll
      for (int i = 0; i < DPL; i++) out[(size_t)row * hd + lane + 32 * i] = A[i] * inv;
    } else {
      float *pp = part + ((size_t)row * n_split + split) * (hd + 2);
      if (lane == 0) {
        pp[0] = M;
        pp[1] = L;
      }
#pragma unroll
      for (int i = 0; i < DPL; i++) pp[2 + lane + 32 * i] = A[i];
    }
  }
  if (n_split > 1 && split_cnt) {  // the row's last CTA to finish merges the splits
    __shared__ int last;
    __threadfence();  // this CTA's partials are visible before its arrival is counted
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(split_cnt + row, 1) == n_split - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    combine_row(part + (size_t)row * n_split * (hd + 2), out + (size_t)row * hd, n_split, hd);
    if (threadIdx.x == 0) split_cnt[row] = 0;  // ready for the next call
  }
}

// Splits per query row: enough CTAs to fill the GPU when there are few rows, and
// never more than SDPA_MAX_ROW_SPLITS (row, split) pairs in total, so one scratch
// buffer of sdpa_max_partials_floats(head_dim) floats serves every call.
int sdpa_num_splits(int seq_q, int seq_k, int n_heads) {
  const long long rows = (long long)seq_q * n_heads;
  if (rows >= 2 * 148) return 1;
  int ns = (seq_k + 31) / 32;  // at least 32 keys a split (two iterations of the CTA's warps)
  const int want = (int)((4 * 148 + rows - 1) / rows);
  if (ns > want) ns = want;
  if (ns > 64) ns = 64;
  if ((long long)ns * rows > SDPA_MAX_ROW_SPLITS) ns = (int)(SDPA_MAX_ROW_SPLITS / rows);
  return ns < 1 ? 1 : ns;
}

size_t sdpa_partials_floats(int seq_q, int n_heads, int head_dim, int n_split) {
  return (size_t)seq_q * n_heads * n_split * (head_dim + 2);
}

size_t sdpa_max_partials_floats(int head_dim) { return (size_t)SDPA_MAX_ROW_SPLITS * (head_dim + 2); }

cudaError_t launch_sdpa(cudaStream_t s, const float *q, const float *k, const float *v, float *out, int seq_q,
                        int seq_k, int n_heads, int n_kv_heads, int head_dim, long long kps, long long khs,
                        int n_split, float *part, const int *pos_dev, int *split_cnt, bool pdl) {
  const int group = n_heads / n_kv_heads;
  const float scale = 1.0f / sqrtf((float)head_dim);  // attention.rs:37
  const int split_len = (seq_k + n_split - 1) / n_split;
  dim3 grid(seq_q * n_heads, n_split);
  cudaError_t e = cudaSuccess;
  switch (head_dim / 32) {
    case 1: e = launch_ex(k_sdpa<1>, grid, dim3(SDPA_WARPS * 32), 0, s, pdl, q, k, v, out, part, seq_q, seq_k, n_heads, group, kps, khs, split_len, scale, pos_dev, split_cnt); break;
    case 2: e = launch_ex(k_sdpa<2>, grid, dim3(SDPA_WARPS * 32), 0, s, pdl, q, k, v, out, part, seq_q, seq_k, n_heads, group, kps, khs, split_len, scale, pos_dev, split_cnt); break;
    case 3: e = launch_ex(k_sdpa<3>, grid, dim3(SDPA_WARPS * 32), 0, s, pdl, q, k, v, out, part, seq_q, seq_k, n_heads, group, kps, khs, split_len, scale, pos_dev, split_cnt); break;
    case 4: e = launch_ex(k_sdpa<4>, grid, dim3(SDPA_WARPS * 32), 0, s, pdl, q, k, v, out, part, seq_q, seq_k, n_heads, group, kps, khs, split_len, scale, pos_dev, split_cnt); break;
    case 5: e = launch_ex(k_sdpa<5>, grid, dim3(SDPA_WARPS * 32), 0, s, pdl, q, k, v, out, part, seq_q, seq_k, n_heads, group, kps, khs, split_len, scale, pos_dev, split_cnt); break;
    case 6: e = launch_ex(k_sdpa<6>, grid, dim3(SDPA_WARPS * 32), 0, s, pdl, q, k, v, out, part, seq_q, seq_k, n_heads, group, kps, khs, split_len, scale, pos_dev, split_cnt); break;
    case 7: e = launch_ex(k_sdpa<7>, grid, dim3(SDPA_WARPS * 32), 0, s, pdl, q, k, v, out, part, seq_q, seq_k, n_heads, group, kps, khs, split_len, scale, pos_dev, split_cnt); break;
    default: e = launch_ex(k_sdpa<8>, grid, dim3(SDPA_WARPS * 32), 0, s, pdl, q, k, v, out, part, seq_q, seq_k, n_heads, group, kps, khs, split_len, scale, pos_dev, split_cnt); break;
  }
  if (e != cudaSuccess) return e;
  if (n_split > 1 && !split_cnt) k_sdpa_combine<<<seq_q * n_heads, 64, 0, s>>>(part, out, n_split, head_dim);
  return cudaGetLastError();
}

}  // namespace sq
