/*
 * oracle.c — CPU restatement of squirrel-rs's Llama token loop (test
 * infrastructure only; see oracle.h for scope, build flags and parity status).
 * Each function names the reference file:line whose arithmetic it follows. The
 * summation order of every output value is the reference's; threads only split
 * independent output rows, as rayon does in the reference.
 */
#define _GNU_SOURCE
#include "oracle.h"

#include <fcntl.h>
#include <math.h>
#include <omp.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

/* ------------------------------------------------------------------------- */
/* half / bf16                                                                */
/* ------------------------------------------------------------------------- */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* half::f16::to_f32: exact widening. */
float or_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    if (exp == 0) {
        float v = ldexpf((float)man, -24);
        return sign ? -v : v;
    }
    if (exp == 31) return u2f(sign | 0x7F800000u | (man << 13));
    return u2f(sign | ((exp + 112u) << 23) | (man << 13));
}

/* half::f16::from_f32: IEEE-754 round-to-nearest-even narrowing. */
uint16_t or_f32_to_f16(float f) {
    uint32_t x = f2u(f);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t exp = (x >> 23) & 0xFFu, man = x & 0x7FFFFFu;
    if (exp == 0xFF) return man ? (uint16_t)(sign | 0x7E00u | (man >> 13)) : (uint16_t)(sign | 0x7C00u);
    int e = (int)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return sign;
        uint32_t full = man | 0x800000u;
        int shift = 14 - e;
        uint32_t m = full >> shift, rem = full & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (m & 1u))) m++;
        return (uint16_t)(sign | m);
    }
    uint32_t m = man >> 13, rem = man & 0x1FFFu;
    uint32_t h = (uint32_t)sign | ((uint32_t)e << 10) | m;
    if (rem > 0x1000u || (rem == 0x1000u && (m & 1u))) h++;
    return (uint16_t)h;
}

float or_bf16_to_f32(uint16_t b) { return u2f((uint32_t)b << 16); }

static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

size_t or_block_bytes(int type) {
    switch (type) {
    case OR_Q8_0: return 34;
    case OR_Q4_0: return 18;
    case OR_BF16: return 64;
    case OR_F32: return 128;
    default: return 0;
    }
}

/* ------------------------------------------------------------------------- */
/* block dequant / quant / dots  (src/kernels/dot_prod.rs)                    */
/* ------------------------------------------------------------------------- */

void or_dequantize(int type, const uint8_t *blocks, size_t nblocks, float *out) {
    for (size_t b = 0; b < nblocks; b++) {
        const uint8_t *blk = blocks + b * or_block_bytes(type);
        float *o = out + b * 32;
        if (type == OR_Q8_0) { /* dot_prod.rs:409-414 */
            float s = or_f16_to_f32(rd16(blk));
            for (int i = 0; i < 32; i++) o[i] = s * (float)(int8_t)blk[2 + i];
        } else if (type == OR_Q4_0) { /* dot_prod.rs:440-446 */
            float s = or_f16_to_f32(rd16(blk));
            for (int j = 0; j < 16; j++) {
                uint8_t byte = blk[2 + j];
                o[j] = s * (float)((int)(byte & 0x0F) - 8);
                o[j + 16] = s * (float)((int)(byte >> 4) - 8);
            }
        } else if (type == OR_BF16) { /* dot_prod.rs:524-528 */
            for (int i = 0; i < 32; i++) o[i] = or_bf16_to_f32(rd16(blk + 2 * i));
        } else if (type == OR_F32) {
            memcpy(o, blk, 128);
        }
    }
}

/* quantize_row_q8_0_scalar, dot_prod.rs:21-31. */
void or_quantize_row_q8_0(const float *src, size_t n, uint8_t *out) {
    for (size_t b = 0; b < n / 32; b++) {
        const float *chunk = src + b * 32;
        uint8_t *blk = out + b * 34;
        float amax = 0.0f;
        for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(chunk[i]));
        float scale = amax / 127.0f;
        float inv = scale > 0.0f ? 1.0f / scale : 0.0f;
        uint16_t d = or_f32_to_f16(scale);
        blk[0] = (uint8_t)(d & 0xFF);
        blk[1] = (uint8_t)(d >> 8);
        for (int i = 0; i < 32; i++) {
            float r = roundf(chunk[i] * inv); /* ties away from zero, as f32::round */
            int8_t q;
            if (isnan(r)) q = 0; /* `NaN as i8` is 0 */
            else q = (int8_t)(r < -127.0f ? -127.0f : (r > 127.0f ? 127.0f : r));
            blk[2 + i] = (uint8_t)q;
        }
    }
}

/* dot_f32_q8_0_fallback, dot_prod.rs:86-96. */
float or_dot_f32_q8_0(const float *a, const uint8_t *b, size_t nblocks) {
    float acc = 0.0f;
    for (size_t k = 0; k < nblocks; k++) {
        const uint8_t *blk = b + k * 34;
        const float *ch = a + k * 32;
        float block_acc = 0.0f;
        for (int i = 0; i < 32; i++) block_acc += ch[i] * (float)(int8_t)blk[2 + i];
        acc += block_acc * or_f16_to_f32(rd16(blk));
    }
    return acc;
}

/* dot_f32_q4_0_fallback, dot_prod.rs:255-270. */
float or_dot_f32_q4_0(const float *a, const uint8_t *b, size_t nblocks) {
    float acc = 0.0f;
    for (size_t k = 0; k < nblocks; k++) {
        const uint8_t *blk = b + k * 18;
        const float *ch = a + k * 32;
        float block_acc = 0.0f;
        for (int j = 0; j < 16; j++) {
            uint8_t byte = blk[2 + j];
            int lo = (int)(byte & 0x0F) - 8, hi = (int)(byte >> 4) - 8;
            block_acc += ch[j] * (float)lo + ch[j + 16] * (float)hi;
        }
        acc += block_acc * or_f16_to_f32(rd16(blk));
    }
    return acc;
}

/* dot_f32_bf16_fallback, dot_prod.rs:464-472: one running sum over the row. */
float or_dot_f32_bf16(const float *a, const uint8_t *b, size_t nblocks) {
    float acc = 0.0f;
    for (size_t k = 0; k < nblocks; k++) {
        const uint8_t *blk = b + k * 64;
        for (int i = 0; i < 32; i++) acc += a[k * 32 + i] * or_bf16_to_f32(rd16(blk + 2 * i));
    }
    return acc;
}

/* dot_q8_0_q8_0_scalar, dot_prod.rs:378-388. */
float or_dot_q8_0_q8_0(const uint8_t *a, const uint8_t *b, size_t nblocks) {
    float total = 0.0f;
    for (size_t k = 0; k < nblocks; k++) {
        const uint8_t *ba = a + k * 34, *bb = b + k * 34;
        int32_t isum = 0;
        for (int i = 0; i < 32; i++) isum += (int32_t)(int8_t)ba[2 + i] * (int32_t)(int8_t)bb[2 + i];
        total += (float)isum * or_f16_to_f32(rd16(ba)) * or_f16_to_f32(rd16(bb));
    }
    return total;
}

/* dot_q8_0_q4_0_scalar, dot_prod.rs:391-403. */
float or_dot_q8_0_q4_0(const uint8_t *a, const uint8_t *b, size_t nblocks) {
    float total = 0.0f;
    for (size_t k = 0; k < nblocks; k++) {
        const uint8_t *ba = a + k * 34, *bb = b + k * 18;
        int32_t isum = 0;
        for (int j = 0; j < 16; j++) {
            uint8_t byte = bb[2 + j];
            int lo = (int)(byte & 0x0F) - 8, hi = (int)(byte >> 4) - 8;
            isum += (int32_t)(int8_t)ba[2 + j] * lo + (int32_t)(int8_t)ba[2 + j + 16] * hi;
        }
        total += (float)isum * or_f16_to_f32(rd16(ba)) * or_f16_to_f32(rd16(bb));
    }
    return total;
}

/* dot_f32_f32, dot_prod.rs:540-549. */
float or_dot_f32_f32(const float *a, const float *b, size_t n) {
    float acc = 0.0f;
    for (size_t i = 0; i < n; i++) acc += a[i] * b[i];
    return acc;
}

/* Eight activation rows against one weight row at once, for prefill (m > 1). Lane j
 * of every vector belongs to row j alone and takes exactly the operations of the
 * single-row function above in the same order (f32 mul, then add; -ffp-contract=off
 * keeps them unfused), so each output is bit-identical to or_dot_f32_*; the lanes
 * only let eight independent sums run side by side. `at` is the row block
 * transposed: at[i * 8 + j] = row j, element i. */
#define OR_RB 8
typedef float or_v8 __attribute__((vector_size(32)));

static inline or_v8 v8_splat(float x) { return (or_v8){x, x, x, x, x, x, x, x}; }

static or_v8 dot8_f32_q8_0(const or_v8 *at, const uint8_t *b, size_t nblocks) {
    or_v8 acc = v8_splat(0.0f);
    for (size_t k = 0; k < nblocks; k++) {
        const uint8_t *blk = b + k * 34;
        const or_v8 *ch = at + k * 32;
        or_v8 block_acc = v8_splat(0.0f);
        for (int i = 0; i < 32; i++) block_acc = block_acc + ch[i] * v8_splat((float)(int8_t)blk[2 + i]);
        acc = acc + block_acc * v8_splat(or_f16_to_f32(rd16(blk)));
    }
    return acc;
}

static or_v8 dot8_f32_q4_0(const or_v8 *at, const uint8_t *b, size_t nblocks) {
    or_v8 acc = v8_splat(0.0f);
    for (size_t k = 0; k < nblocks; k++) {
        const uint8_t *blk = b + k * 18;
        const or_v8 *ch = at + k * 32;
        or_v8 block_acc = v8_splat(0.0f);
        for (int j = 0; j < 16; j++) {
            uint8_t byte = blk[2 + j];
            int lo = (int)(byte & 0x0F) - 8, hi = (int)(byte >> 4) - 8;
            block_acc = block_acc + (ch[j] * v8_splat((float)lo) + ch[j + 16] * v8_splat((float)hi));
        }
        acc = acc + block_acc * v8_splat(or_f16_to_f32(rd16(blk)));
    }
    return acc;
}

static or_v8 dot8_f32_bf16(const or_v8 *at, const uint8_t *b, size_t nblocks) {
    or_v8 acc = v8_splat(0.0f);
    for (size_t k = 0; k < nblocks; k++) {
        const uint8_t *blk = b + k * 64;
        for (int i = 0; i < 32; i++) acc = acc + at[k * 32 + i] * v8_splat(or_bf16_to_f32(rd16(blk + 2 * i)));
    }
    return acc;
}

/* ------------------------------------------------------------------------- */
/* linear  (ops/linear.rs:26-168, kernels/matmul.rs:28-171)                    */
/* ------------------------------------------------------------------------- */

int or_linear(const float *in, int m, int in_dim, const uint8_t *w, int type, int out_dim,
              float *out, int acts_q8, int nthreads) {
    size_t bb = or_block_bytes(type);
    if (bb == 0 || type == OR_F32) return OR_INVALID_TYPE;
    if (m <= 0 || in_dim <= 0 || out_dim <= 0 || in_dim % 32) return OR_SHAPE;
    int bpr = in_dim / 32;
    int int_acts = acts_q8 && (type == OR_Q8_0 || type == OR_Q4_0);
    uint8_t *aq = NULL;
    if (int_acts) { /* quantize the whole [m, in] input once, linear.rs:127 / matmul.rs:91-98 */
        aq = (uint8_t *)malloc((size_t)m * bpr * 34);
        or_quantize_row_q8_0(in, (size_t)m * in_dim, aq);
    }
    if (nthreads <= 0) nthreads = 1;
    if (!int_acts && m > 1) {
        /* prefill: blocks of OR_RB rows against each weight row (outputs identical to
         * the row-outermost loop of matmul.rs:34, which only orders independent sums) */
        or_v8 *at = (or_v8 *)aligned_alloc(32, sizeof(or_v8) * (size_t)in_dim);
        for (int r0 = 0; r0 < m; r0 += OR_RB) {
            int nr = m - r0 < OR_RB ? m - r0 : OR_RB;
            for (int i = 0; i < in_dim; i++)
                for (int j = 0; j < OR_RB; j++) at[i][j] = j < nr ? in[(size_t)(r0 + j) * in_dim + i] : 0.0f;
#pragma omp parallel for num_threads(nthreads) schedule(static)
            for (int n = 0; n < out_dim; n++) {
                const uint8_t *wr = w + (size_t)n * bpr * bb;
                or_v8 v = type == OR_Q8_0 ? dot8_f32_q8_0(at, wr, bpr)
                                          : (type == OR_Q4_0 ? dot8_f32_q4_0(at, wr, bpr) : dot8_f32_bf16(at, wr, bpr));
                for (int j = 0; j < nr; j++) out[(size_t)(r0 + j) * out_dim + n] = v[j];
            }
        }
        free(at);
        return OR_OK;
    }
    for (int r = 0; r < m; r++) { /* fused_bridge_rows: row loop outermost, matmul.rs:34 */
        const float *a = in + (size_t)r * in_dim;
#pragma omp parallel for num_threads(nthreads) schedule(static)
        for (int n = 0; n < out_dim; n++) {
            const uint8_t *wr = w + (size_t)n * bpr * bb;
            float v;
            if (int_acts)
                v = type == OR_Q8_0 ? or_dot_q8_0_q8_0(aq + (size_t)r * bpr * 34, wr, bpr)
                                    : or_dot_q8_0_q4_0(aq + (size_t)r * bpr * 34, wr, bpr);
            else if (type == OR_Q8_0) v = or_dot_f32_q8_0(a, wr, bpr);
            else if (type == OR_Q4_0) v = or_dot_f32_q4_0(a, wr, bpr);
            else v = or_dot_f32_bf16(a, wr, bpr);
            out[(size_t)r * out_dim + n] = v;
        }
    }
    free(aq);
    return OR_OK;
}

/* ------------------------------------------------------------------------- */
/* norm / rope / softmax / attention / activations                            */
/* ------------------------------------------------------------------------- */

/* rms_norm_f32_into, kernels/rms_norm.rs:40-56 (per row, ops/rms_norm.rs:13-43). */
int or_rms_norm(const float *in, const float *w, float *out, int rows, int dim, float eps) {
    if (dim <= 0) return OR_SHAPE;
    for (int r = 0; r < rows; r++) {
        const float *x = in + (size_t)r * dim;
        float *y = out + (size_t)r * dim;
        float ss = 0.0f;
        for (int i = 0; i < dim; i++) ss += x[i] * x[i];
        float mean = ss / (float)dim;
        float rms = sqrtf(mean + eps);
        for (int i = 0; i < dim; i++) y[i] = (x[i] * w[i]) / rms;
    }
    return OR_OK;
}

/* rms_norm_f32_inplace, kernels/rms_norm.rs:63-74. */
int or_rms_norm_inplace(float *x, const float *w, int rows, int dim, float eps) {
    return or_rms_norm(x, w, x, rows, dim, eps); /* the squared sum completes before any write */
}

/* rope_f32_interleaved, kernels/rope.rs:7-36, per row (ops/rope.rs:6-32). */
int or_rope_rows(float *x, int seq, int row_dim, int base_pos, const float *inv_freq, int half) {
    int head_dim = 2 * half;
    if (head_dim == 0 || seq <= 0 || row_dim % head_dim) return OR_SHAPE;
    for (int r = 0; r < seq; r++) {
        float pos = (float)(base_pos + r);
        for (int h = 0; h < row_dim / head_dim; h++) {
            float *head = x + (size_t)r * row_dim + (size_t)h * head_dim;
            for (int j = 0; j < half; j++) {
                float theta = pos * inv_freq[j];
                float s = sinf(theta), c = cosf(theta);
                float a = head[2 * j], b = head[2 * j + 1];
                head[2 * j] = a * c - b * s;
                head[2 * j + 1] = a * s + b * c;
            }
        }
    }
    return OR_OK;
}

/* softmax_f32, kernels/softmax.rs:4-27. */
int or_softmax(const float *a, float *out, int n) {
    if (n <= 0) return OR_EMPTY;
    float mx = -INFINITY;
    for (int i = 0; i < n; i++) mx = fmaxf(mx, a[i]);
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        out[i] = expf(a[i] - mx);
        sum += out[i];
    }
    float inv = 1.0f / sum;
    for (int i = 0; i < n; i++) out[i] *= inv;
    return OR_OK;
}

/* sdpa_f32, kernels/attention.rs:11-70. */
int or_sdpa(const float *q, const float *k, const float *v, float *out, int seq_q, int seq_k,
            int n_heads, int n_kv_heads, int head_dim, int nthreads) {
    if (n_kv_heads <= 0 || n_heads % n_kv_heads) return OR_SHAPE;
    if (seq_k < seq_q || seq_q <= 0 || head_dim <= 0) return OR_SHAPE;
    int offset = seq_k - seq_q;
    int group = n_heads / n_kv_heads;
    float scale = 1.0f / sqrtf((float)head_dim);
    if (nthreads <= 0) nthreads = 1;
#pragma omp parallel num_threads(nthreads)
    {
        float *scores = (float *)malloc((size_t)seq_k * sizeof(float));
        float *probs = (float *)malloc((size_t)seq_k * sizeof(float));
#pragma omp for schedule(static)
        for (int idx = 0; idx < seq_q * n_heads; idx++) {
            int t = idx / n_heads, h = idx % n_heads, kvh = h / group;
            int live = offset + t + 1;
            const float *qr = q + ((size_t)t * n_heads + h) * head_dim;
            for (int s = 0; s < live; s++)
                scores[s] = or_dot_f32_f32(qr, k + ((size_t)s * n_kv_heads + kvh) * head_dim, head_dim) * scale;
            or_softmax(scores, probs, live);
            float *o = out + (size_t)idx * head_dim;
            for (int d = 0; d < head_dim; d++) o[d] = 0.0f;
            for (int s = 0; s < live; s++) {
                const float *vr = v + ((size_t)s * n_kv_heads + kvh) * head_dim;
                float p = probs[s];
                for (int d = 0; d < head_dim; d++) o[d] += p * vr[d];
            }
        }
        free(scores);
        free(probs);
    }
    return OR_OK;
}

/* sigmoid_f32, kernels/sigmoid.rs:2-9. */
float or_sigmoid(float x) {
    if (x >= 0.0f) return 1.0f / (1.0f + expf(-x));
    float z = expf(x);
    return z / (1.0f + z);
}

/* silu_f32, kernels/silu.rs:4-8. */
void or_silu(float *x, int n) {
    for (int i = 0; i < n; i++) x[i] = x[i] * or_sigmoid(x[i]);
}

/* elementwise_mul_f32, kernels/elementwise_mul.rs:3-17. */
int or_mul(const float *a, const float *b, float *out, int n) {
    for (int i = 0; i < n; i++) out[i] = a[i] * b[i];
    return OR_OK;
}

/* elementwise_add_f32_inplace, kernels/elementwise_add.rs:47-61. */
int or_add_inplace(float *a, const float *b, int n) {
    for (int i = 0; i < n; i++) a[i] += b[i];
    return OR_OK;
}

/* GreedySampler::sample, samplers/greedy.rs:6-15. Iterator::max_by keeps the
 * running best only when it compares Greater than the next item; NaN compares
 * Equal, so the later item wins (ties and NaN resolve to the later index). */
int64_t or_greedy(const float *logits, size_t n) {
    if (n == 0) return -1;
    size_t best = 0;
    for (size_t i = 1; i < n; i++) {
        float a = logits[best], b = logits[i];
        if (!(a > b)) best = i; /* Greater keeps a; Less / Equal / unordered take b */
    }
    return (int64_t)best;
}

/* embed, ops/embedding.rs:10-52. */
int or_embed(const uint32_t *tokens, int n, const uint8_t *w, int type, int embed_dim, int vocab,
             float *out) {
    size_t bb = or_block_bytes(type);
    if (bb == 0 || type == OR_F32) return OR_INVALID_TYPE;
    if (embed_dim % 32) return OR_SHAPE;
    int bpt = embed_dim / 32;
    for (int t = 0; t < n; t++) {
        if ((int)tokens[t] >= vocab) return OR_SHAPE; /* the reference would panic on the slice */
        or_dequantize(type, w + (size_t)tokens[t] * bpt * bb, bpt, out + (size_t)t * embed_dim);
    }
    return OR_OK;
}

/* compute_rope_inv_freq, models/llama/config.rs:83-127. */
void or_rope_inv_freq(int head_dim, float base, float factor, float low, float high,
                      float orig_ctx, float *out) {
    int half = head_dim / 2;
    float inv_head_dim = 1.0f / (float)head_dim;
    for (int j = 0; j < half; j++) out[j] = powf(base, -2.0f * (float)j * inv_head_dim);
    const float two_pi = 6.28318548202514648438f; /* std::f32::consts::TAU */
    float low_wl = orig_ctx / low, high_wl = orig_ctx / high;
    for (int j = 0; j < half; j++) {
        float f = out[j];
        float wavelen = two_pi / f;
        if (wavelen > low_wl) {
            out[j] = f / factor;
        } else if (wavelen >= high_wl) {
            float smooth = (orig_ctx / wavelen - low) / (high - low);
            out[j] = (1.0f - smooth) * (f / factor) + smooth * f;
        }
    }
}

/* ------------------------------------------------------------------------- */
/* GGUF reader  (the file_parser module of the reference)                     */
/* ------------------------------------------------------------------------- */

typedef struct {
    char name[96];
    int type;
    int ndims;
    uint64_t dims[4];
    uint64_t offset;
} or_tinfo;

typedef struct {
    const uint8_t *p, *end;
    int bad;
} rd_t;

static uint64_t rd_u(rd_t *r, int n) {
    if (r->p + n > r->end) { r->bad = 1; return 0; }
    uint64_t v = 0;
    for (int i = 0; i < n; i++) v |= (uint64_t)r->p[i] << (8 * i);
    r->p += n;
    return v;
}

/* Key lookup results (gguf_metadata_value.rs:49-80 types). */
typedef struct { int found, type; uint64_t u; float f; uint64_t arr_len; } kv_t;

enum { GT_U8 = 0, GT_I8, GT_U16, GT_I16, GT_U32, GT_I32, GT_F32, GT_BOOL, GT_STR, GT_ARR, GT_U64, GT_I64, GT_F64 };

static void skip_value(rd_t *r, int type, kv_t *kv, int depth) {
    static const int sz[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (type < 0 || type > 12) { r->bad = 1; return; }
    if (type == GT_STR) {
        uint64_t n = rd_u(r, 8);
        if (r->p + n > r->end) { r->bad = 1; return; }
        r->p += n;
    } else if (type == GT_ARR) {
        int at = (int)rd_u(r, 4);
        uint64_t n = rd_u(r, 8);
        if (kv && depth == 0) kv->arr_len = n;
        for (uint64_t i = 0; i < n && !r->bad; i++) skip_value(r, at, NULL, depth + 1);
    } else {
        uint64_t v = rd_u(r, sz[type]);
        if (kv && depth == 0) {
            kv->u = v;
            if (type == GT_F32) { uint32_t w = (uint32_t)v; memcpy(&kv->f, &w, 4); }
        }
    }
}

struct or_model {
    void *map;
    size_t map_len;
    or_config cfg;
    float *inv_freq;
    int acts_q8;
    const uint8_t *embd;
    int embd_type;
    const uint8_t *out_w;
    int out_type;
    const float *out_norm;
    struct {
        const float *attn_norm, *ffn_norm;
        const uint8_t *q, *k, *v, *o, *gate, *up, *down;
    } *blk;
};

struct or_ctx {
    const or_model *m;
    int seq_len, cap;
    float **k, **v; /* per layer [cap][kv_dim] */
    float *logits;
};

#define NKEYS 19
static const char *KEYS[NKEYS] = {
    "llama.block_count", "llama.embedding_length", "llama.feed_forward_length",
    "llama.attention.head_count", "llama.attention.head_count_kv", "llama.rope.dimension_count",
    "llama.rope.freq_base", "llama.attention.layer_norm_rms_epsilon", "llama.context_length",
    "tokenizer.ggml.bos_token_id", "tokenizer.ggml.eos_token_id", "llama.vocab_size",
    "tokenizer.ggml.tokens", "llama.rope.scaling.factor", "llama.rope.scaling.low_freq_factor",
    "llama.rope.scaling.high_freq_factor", "llama.rope.scaling.original_context_length",
    "general.alignment", "general.architecture"};

static int need_u32(const kv_t *kv, uint32_t *out) {
    if (!kv->found || kv->type != GT_U32) return 0;
    *out = (uint32_t)kv->u;
    return 1;
}
static int need_f32(const kv_t *kv, float *out) {
    if (!kv->found || kv->type != GT_F32) return 0;
    *out = kv->f;
    return 1;
}

or_model *or_model_load(const char *path, int acts_q8, int *status) {
    int st = OR_IO;
    int fd = open(path, O_RDONLY);
    if (fd < 0) { if (status) *status = OR_IO; return NULL; }
    struct stat sb;
    fstat(fd, &sb);
    void *map = mmap(NULL, (size_t)sb.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) { if (status) *status = OR_IO; return NULL; }
    rd_t r = {(const uint8_t *)map, (const uint8_t *)map + sb.st_size, 0};
    /* gguf_header.rs:13-24 (the magic is read, not checked) */
    rd_u(&r, 4);
    rd_u(&r, 4);
    uint64_t n_tensors = rd_u(&r, 8), n_kv = rd_u(&r, 8);
    kv_t kvs[NKEYS];
    memset(kvs, 0, sizeof kvs);
    for (uint64_t i = 0; i < n_kv && !r.bad; i++) {
        uint64_t klen = rd_u(&r, 8);
        if (r.p + klen > r.end) { r.bad = 1; break; }
        const char *key = (const char *)r.p;
        r.p += klen;
        int type = (int)rd_u(&r, 4);
        kv_t *hit = NULL;
        for (int k = 0; k < NKEYS; k++)
            if (strlen(KEYS[k]) == klen && !memcmp(KEYS[k], key, klen)) hit = &kvs[k];
        if (hit) { hit->found = 1; hit->type = type; }
        skip_value(&r, type, hit, 0);
    }
    or_tinfo *ti = (or_tinfo *)calloc(n_tensors ? n_tensors : 1, sizeof(or_tinfo));
    for (uint64_t i = 0; i < n_tensors && !r.bad; i++) { /* gguf_tensor_info.rs:25-50 */
        uint64_t nlen = rd_u(&r, 8);
        if (r.p + nlen > r.end || nlen >= sizeof ti[i].name) { r.bad = 1; break; }
        memcpy(ti[i].name, r.p, nlen);
        r.p += nlen;
        ti[i].ndims = (int)rd_u(&r, 4);
        if (ti[i].ndims > 4) { r.bad = 1; break; }
        for (int d = 0; d < ti[i].ndims; d++) ti[i].dims[d] = rd_u(&r, 8);
        ti[i].type = (int)rd_u(&r, 4);
        ti[i].offset = rd_u(&r, 8);
    }
    or_model *m = NULL;
    if (r.bad) goto fail;
    /* gguf_file.rs:44-46: data starts at the next multiple of a hard-coded 32 */
    uint64_t pos = (uint64_t)(r.p - (const uint8_t *)map);
    uint64_t data_off = (pos + 31) & ~(uint64_t)31;

    m = (or_model *)calloc(1, sizeof(or_model));
    m->map = map;
    m->map_len = (size_t)sb.st_size;
    m->acts_q8 = acts_q8;
    or_config *c = &m->cfg;
    uint32_t u;
    float f;
    st = OR_SHAPE;
    /* config.rs:29-73 */
#define REQ_U32(i, field) do { if (!need_u32(&kvs[i], &u)) goto fail; field = (int)u; } while (0)
#define REQ_F32(i, field) do { if (!need_f32(&kvs[i], &f)) goto fail; field = f; } while (0)
    REQ_U32(0, c->n_blocks);
    REQ_U32(1, c->embed_dim);
    REQ_U32(2, c->ffn_dim);
    REQ_U32(3, c->n_heads);
    REQ_U32(4, c->n_kv_heads);
    c->head_dim = need_u32(&kvs[5], &u) ? (int)u : c->embed_dim / c->n_heads;
    REQ_F32(6, c->rope_base);
    REQ_F32(7, c->rms_eps);
    REQ_U32(8, c->context_length);
    if (!need_u32(&kvs[9], &c->bos_token_id)) goto fail;
    if (!need_u32(&kvs[10], &c->eos_token_id)) goto fail;
#undef REQ_U32
#undef REQ_F32
    if (need_u32(&kvs[11], &u)) c->vocab_size = (int)u;
    else if (kvs[12].found && kvs[12].type == GT_ARR) c->vocab_size = (int)kvs[12].arr_len;
    else goto fail;
    float factor = 32.0f, low = 1.0f, high = 4.0f, orig = 8192.0f;
    need_f32(&kvs[13], &factor);
    need_f32(&kvs[14], &low);
    need_f32(&kvs[15], &high);
    if (need_u32(&kvs[16], &u)) orig = (float)u;
    m->inv_freq = (float *)malloc(sizeof(float) * (size_t)(c->head_dim / 2 > 0 ? c->head_dim / 2 : 1));
    or_rope_inv_freq(c->head_dim, c->rope_base, factor, low, high, orig, m->inv_freq);

    /* weights.rs:50-97 */
#define FIND(nm, out_ptr, out_type)                                                       \
    do {                                                                                  \
        int _f = 0;                                                                       \
        for (uint64_t _i = 0; _i < n_tensors; _i++)                                       \
            if (!strcmp(ti[_i].name, nm)) {                                               \
                out_ptr = (const void *)((const uint8_t *)map + data_off + ti[_i].offset); \
                out_type = ti[_i].type;                                                   \
                _f = 1;                                                                   \
                break;                                                                    \
            }                                                                             \
        if (!_f) goto fail;                                                               \
    } while (0)
    m->blk = calloc((size_t)c->n_blocks, sizeof *m->blk);
    char nm[96];
    const void *p;
    int t;
    st = OR_INVALID_TYPE;
    for (int i = 0; i < c->n_blocks; i++) {
        snprintf(nm, sizeof nm, "blk.%d.attn_norm.weight", i); FIND(nm, p, t); if (t != OR_F32) goto fail; m->blk[i].attn_norm = p;
        snprintf(nm, sizeof nm, "blk.%d.ffn_norm.weight", i); FIND(nm, p, t); if (t != OR_F32) goto fail; m->blk[i].ffn_norm = p;
        snprintf(nm, sizeof nm, "blk.%d.attn_q.weight", i); FIND(nm, p, t); m->blk[i].q = p; if (i == 0) c->weight_type = t;
        snprintf(nm, sizeof nm, "blk.%d.attn_k.weight", i); FIND(nm, p, t); m->blk[i].k = p;
        snprintf(nm, sizeof nm, "blk.%d.attn_v.weight", i); FIND(nm, p, t); m->blk[i].v = p;
        snprintf(nm, sizeof nm, "blk.%d.attn_output.weight", i); FIND(nm, p, t); m->blk[i].o = p;
        snprintf(nm, sizeof nm, "blk.%d.ffn_gate.weight", i); FIND(nm, p, t); m->blk[i].gate = p;
        snprintf(nm, sizeof nm, "blk.%d.ffn_up.weight", i); FIND(nm, p, t); m->blk[i].up = p;
        snprintf(nm, sizeof nm, "blk.%d.ffn_down.weight", i); FIND(nm, p, t); m->blk[i].down = p;
    }
    FIND("token_embd.weight", p, t); m->embd = p; m->embd_type = t;
    FIND("output_norm.weight", p, t); if (t != OR_F32) goto fail; m->out_norm = p;
    {
        int found = 0;
        for (uint64_t i = 0; i < n_tensors; i++)
            if (!strcmp(ti[i].name, "output.weight")) {
                m->out_w = (const uint8_t *)map + data_off + ti[i].offset;
                m->out_type = ti[i].type;
                found = 1;
            }
        if (!found) { m->out_w = m->embd; m->out_type = m->embd_type; } /* tied, weights.rs:89 */
    }
#undef FIND
    free(ti);
    if (status) *status = OR_OK;
    return m;
fail:
    free(ti);
    if (m) { free(m->inv_freq); free(m->blk); free(m); }
    munmap(map, (size_t)sb.st_size);
    if (status) *status = st;
    return NULL;
}

void or_model_free(or_model *m) {
    if (!m) return;
    munmap(m->map, m->map_len);
    free(m->inv_freq);
    free(m->blk);
    free(m);
}

void or_model_config(const or_model *m, or_config *out) { *out = m->cfg; }
const float *or_model_inv_freq(const or_model *m) { return m->inv_freq; }

or_ctx *or_ctx_new(const or_model *m) {
    or_ctx *c = (or_ctx *)calloc(1, sizeof(or_ctx));
    c->m = m;
    c->k = (float **)calloc((size_t)m->cfg.n_blocks, sizeof(float *));
    c->v = (float **)calloc((size_t)m->cfg.n_blocks, sizeof(float *));
    c->logits = (float *)calloc((size_t)m->cfg.vocab_size, sizeof(float));
    return c;
}

void or_ctx_free(or_ctx *c) {
    if (!c) return;
    for (int l = 0; l < c->m->cfg.n_blocks; l++) { free(c->k[l]); free(c->v[l]); }
    free(c->k);
    free(c->v);
    free(c->logits);
    free(c);
}

void or_ctx_reset(or_ctx *c) { c->seq_len = 0; } /* kv_cache.rs:72-78 keeps capacity */
int or_ctx_seq_len(const or_ctx *c) { return c->seq_len; }
const float *or_ctx_logits(const or_ctx *c) { return c->logits; }

static void ctx_reserve(or_ctx *c, int need) {
    if (need <= c->cap) return;
    int cap = c->cap ? c->cap : 64;
    while (cap < need) cap *= 2;
    size_t kvd = (size_t)c->m->cfg.n_kv_heads * c->m->cfg.head_dim;
    for (int l = 0; l < c->m->cfg.n_blocks; l++) {
        c->k[l] = (float *)realloc(c->k[l], (size_t)cap * kvd * sizeof(float));
        c->v[l] = (float *)realloc(c->v[l], (size_t)cap * kvd * sizeof(float));
    }
    c->cap = cap;
}

/* Llama3_2::forward, models/llama/model.rs:45-97, with layers::block (layers.rs:81-109). */
int or_forward(const or_model *m, or_ctx *c, const uint32_t *ids, int n, int nthreads) {
    const or_config *cf = &m->cfg;
    if (n <= 0) return OR_EMPTY;
    int E = cf->embed_dim, Q = cf->n_heads * cf->head_dim, KV = cf->n_kv_heads * cf->head_dim,
        F = cf->ffn_dim, wt = cf->weight_type, aq = m->acts_q8;
    float *hidden = malloc(sizeof(float) * (size_t)n * E), *normed = malloc(sizeof(float) * (size_t)n * E);
    float *q = malloc(sizeof(float) * (size_t)n * Q), *k = malloc(sizeof(float) * (size_t)n * KV),
          *v = malloc(sizeof(float) * (size_t)n * KV), *attn = malloc(sizeof(float) * (size_t)n * Q),
          *attn_out = malloc(sizeof(float) * (size_t)n * E), *gate = malloc(sizeof(float) * (size_t)n * F),
          *up = malloc(sizeof(float) * (size_t)n * F), *act = malloc(sizeof(float) * (size_t)n * F),
          *ffn_out = malloc(sizeof(float) * (size_t)n * E);
    int st = or_embed(ids, n, m->embd, m->embd_type, E, cf->vocab_size, hidden);
    int position = c->seq_len;
    ctx_reserve(c, position + n);
    for (int l = 0; l < cf->n_blocks && st == OR_OK; l++) {
        or_rms_norm(hidden, m->blk[l].attn_norm, normed, n, E, cf->rms_eps);
        /* linear_shared(normed -> q, k, v): x86 runs linear() per weight (linear.rs:160-166);
         * the aarch64 branch quantizes once — identical bytes either way. */
        or_linear(normed, n, E, m->blk[l].q, wt, Q, q, aq, nthreads);
        or_linear(normed, n, E, m->blk[l].k, wt, KV, k, aq, nthreads);
        or_linear(normed, n, E, m->blk[l].v, wt, KV, v, aq, nthreads);
        or_rope_rows(q, n, Q, position, m->inv_freq, cf->head_dim / 2);
        or_rope_rows(k, n, KV, position, m->inv_freq, cf->head_dim / 2);
        memcpy(c->k[l] + (size_t)position * KV, k, sizeof(float) * (size_t)n * KV); /* kv_cache.rs:38-53 */
        memcpy(c->v[l] + (size_t)position * KV, v, sizeof(float) * (size_t)n * KV);
        st = or_sdpa(q, c->k[l], c->v[l], attn, n, position + n, cf->n_heads, cf->n_kv_heads,
                     cf->head_dim, nthreads);
        or_linear(attn, n, Q, m->blk[l].o, wt, E, attn_out, aq, nthreads);
        or_add_inplace(hidden, attn_out, n * E);
        or_rms_norm(hidden, m->blk[l].ffn_norm, normed, n, E, cf->rms_eps);
        or_linear(normed, n, E, m->blk[l].gate, wt, F, gate, aq, nthreads);
        or_linear(normed, n, E, m->blk[l].up, wt, F, up, aq, nthreads);
        or_silu(gate, n * F);
        or_mul(gate, up, act, n * F);
        or_linear(act, n, F, m->blk[l].down, wt, E, ffn_out, aq, nthreads);
        or_add_inplace(hidden, ffn_out, n * E);
    }
    if (st == OR_OK) {
        c->seq_len += n; /* cache.advance, model.rs:70 */
        or_rms_norm_inplace(hidden, m->out_norm, n, E, cf->rms_eps);
        st = or_linear(hidden + (size_t)(n - 1) * E, 1, E, m->out_w, m->out_type, cf->vocab_size,
                       c->logits, aq, nthreads);
    }
    free(hidden); free(normed); free(q); free(k); free(v); free(attn); free(attn_out);
    free(gate); free(up); free(act); free(ffn_out);
    return st;
}

static double now_ms(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1e3 + ts.tv_nsec / 1e6;
}

/* TextTokenGenerator::generate, text_generator.rs:58-97 (token ids only). */
int or_generate(const or_model *m, const uint32_t *prompt, int n_prompt, int max_tokens,
                int ignore_eos, uint32_t *out_ids, double *step_ms, float *logits_out,
                int nthreads) {
    or_ctx *c = or_ctx_new(m);
    uint32_t *input = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)(n_prompt > 0 ? n_prompt : 1));
    memcpy(input, prompt, sizeof(uint32_t) * (size_t)n_prompt);
    int n_in = n_prompt, produced = 0;
    for (int step = 1; step <= max_tokens; step++) {
        double t0 = now_ms();
        int st = or_forward(m, c, input, n_in, nthreads);
        if (st != OR_OK) { produced = -st; break; }
        uint32_t next = (uint32_t)or_greedy(c->logits, (size_t)m->cfg.vocab_size);
        double t1 = now_ms();
        if (step_ms) step_ms[step - 1] = t1 - t0;
        if (logits_out)
            memcpy(logits_out + (size_t)(step - 1) * m->cfg.vocab_size, c->logits,
                   sizeof(float) * (size_t)m->cfg.vocab_size);
        if (next == m->cfg.eos_token_id && !ignore_eos) break;
        out_ids[produced++] = next;
        input[0] = next;
        n_in = 1;
    }
    free(input);
    or_ctx_free(c);
    return produced;
}
