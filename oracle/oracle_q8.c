/*
 * oracle_q8.c -- CPU restatement of the lluda-inference Qwen3 path with Q8_0 linears.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA library, never the product. It is
 * loaded by tests/, __graft_entry__.smoke() and bench.py (cpu_baseline and the reference
 * arm) and nothing else.
 *
 * Build: see oracle/Makefile (gcc -O2 -ffp-contract=off, no fast-math). Floating-point
 * operations are written in the reference's order; a multiply followed by an add is never
 * contracted into an FMA, because Rust does not contract either.
 *
 * File:line citations are paths inside the reference project (crate lluda-inference).
 */
#include "oracle_q8.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ====================================================================================== */
/* scalar conversions                                                                     */
/* ====================================================================================== */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* bf16.rs:112-131: bits + (0x7FFF + ((bits >> 16) & 1)), then the top 16 bits (wrapping). */
uint16_t orc_f32_to_bf16(float f) {
    uint32_t bits = f2u(f);
    uint32_t bias = 0x7FFFu + ((bits >> 16) & 1u);
    return (uint16_t)((bits + bias) >> 16);
}

/* bf16.rs:136-142: shift left by 16, exact. */
float orc_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

/* IEEE 754 binary32 -> binary16, round to nearest, ties to even. Written from the format
 * definition: normal results round the 23-bit fraction to 10 bits; results below 2^-14
 * become subnormal multiples of 2^-24; |x| >= 65520 overflows to infinity. */
uint16_t orc_f32_to_f16(float f) {
    uint32_t x = f2u(f);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return sign | (ax > 0x7F800000u ? 0x7E00u : 0x7C00u);
    if (ax >= 0x477FF000u) return sign | 0x7C00u;          /* >= 65520 -> inf           */
    if (ax < 0x33000000u) return sign;                       /* <= 2^-25 -> +-0 (tie even) */
    uint32_t e = ax >> 23;
    uint32_t mant = (ax & 0x7FFFFFu) | 0x800000u;
    if (e < 113u) {                                          /* subnormal binary16 result */
        uint32_t s = 126u - e;                               /* 14..24                     */
        uint32_t r = (mant + ((1u << (s - 1)) - 1u) + ((mant >> s) & 1u)) >> s;
        return sign | (uint16_t)r;                           /* r == 1024 is the min normal */
    }
    uint32_t h = ((e - 112u) << 10) + ((ax & 0x7FFFFFu) >> 13);
    uint32_t rem = ax & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return sign | (uint16_t)h;
}

float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    if (e == 0x1Fu) return u2f(sign | 0x7F800000u | (m << 13));
    if (e == 0) {
        if (m == 0) return u2f(sign);
        /* subnormal: m * 2^-24, exact in f32 */
        float v = (float)m * 5.9604644775390625e-08f;
        return sign ? -v : v;
    }
    return u2f(sign | ((e + 112u) << 23) | (m << 13));
}

void orc_f32_to_bf16_array(const float* x, int64_t n, uint16_t* out) {
    for (int64_t i = 0; i < n; i++) out[i] = orc_f32_to_bf16(x[i]);
}
void orc_bf16_to_f32_array(const uint16_t* x, int64_t n, float* out) {
    for (int64_t i = 0; i < n; i++) out[i] = orc_bf16_to_f32(x[i]);
}

/* ====================================================================================== */
/* seeded generators                                                                      */
/* ====================================================================================== */

/* SplitMix64 (Steele, Lea, Flood 2014), the published 64-bit mixing function. */
uint64_t orc_splitmix64(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static inline uint64_t gen_key(uint64_t seed, uint64_t tensor_id) {
    return orc_splitmix64(seed ^ (tensor_id * 0xD1B54A32D192ED03ull));
}

/* sqrt(3)/65536 * std: the Irwin-Hall sum of four uniforms on [0, 65535] has standard
 * deviation 65536/sqrt(3) (to 1e-9 relative). */
float orc_gen_scale(double std_dev) { return (float)(std_dev * 1.7320508075688772 / 65536.0); }

static inline float gen_value(uint64_t key, uint64_t idx, float scale) {
    uint64_t h = orc_splitmix64(key + idx);
    int32_t s = (int32_t)(h & 0xFFFFu) + (int32_t)((h >> 16) & 0xFFFFu) +
                (int32_t)((h >> 32) & 0xFFFFu) + (int32_t)((h >> 48) & 0xFFFFu) - 131070;
    return (float)s * scale;   /* |s| < 2^24: exact conversion; one IEEE multiply */
}

void orc_gen_bf16(uint64_t seed, uint64_t tensor_id, int64_t offset, int64_t count,
                  float scale, uint16_t* out) {
    uint64_t key = gen_key(seed, tensor_id);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < count; i++)
        out[i] = orc_f32_to_bf16(gen_value(key, (uint64_t)(offset + i), scale));
}

void orc_gen_tokens(uint64_t seed, uint64_t stream, int64_t count, int64_t vocab, int32_t* out) {
    uint64_t key = gen_key(seed, 0x70C0000000000000ull ^ stream);
    for (int64_t i = 0; i < count; i++)
        out[i] = (int32_t)(orc_splitmix64(key + (uint64_t)i) % (uint64_t)vocab);
}

/* ====================================================================================== */
/* Q8_0                                                                                    */
/* ====================================================================================== */

/* One block, GGML quantize_row_q8_0_ref: amax = max|x| (MAX macro order), d = amax/127,
 * id = d ? 1/d : 0, q = roundf(x*id) (half away from zero), d stored as fp16 RNE. The clamp
 * to [-127,127] never triggers for finite input (|x*id| <= 127*(1+2^-24)^3); it is kept as
 * the format's documented range. */
static void q8_block(const float* x, int8_t* qs, uint16_t* d) {
    float amax = 0.0f;
    for (int j = 0; j < ORC_QK; j++) {
        float v = fabsf(x[j]);
        amax = amax > v ? amax : v;
    }
    float dd = amax / 127.0f;
    float id = dd != 0.0f ? 1.0f / dd : 0.0f;
    *d = orc_f32_to_f16(dd);
    for (int j = 0; j < ORC_QK; j++) {
        float x0 = x[j] * id;
        float r = roundf(x0);
        if (r > 127.0f) r = 127.0f;
        if (r < -127.0f) r = -127.0f;
        qs[j] = (int8_t)r;
    }
}

void orc_q8_0_quantize_f32(const float* x, int64_t rows, int64_t k, int8_t* qs, uint16_t* d) {
    int64_t nb = k / ORC_QK;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++)
        for (int64_t b = 0; b < nb; b++)
            q8_block(x + r * k + b * ORC_QK, qs + r * k + b * ORC_QK, d + r * nb + b);
}

void orc_q8_0_quantize_bf16(const uint16_t* x, int64_t rows, int64_t k, int8_t* qs, uint16_t* d) {
    int64_t nb = k / ORC_QK;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        float tmp[ORC_QK];
        for (int64_t b = 0; b < nb; b++) {
            for (int j = 0; j < ORC_QK; j++) tmp[j] = orc_bf16_to_f32(x[r * k + b * ORC_QK + j]);
            q8_block(tmp, qs + r * k + b * ORC_QK, d + r * nb + b);
        }
    }
}

void orc_q8_0_pack_blocks(const int8_t* qs, const uint16_t* d, int64_t rows, int64_t k, uint8_t* blocks) {
    int64_t nb = k / ORC_QK;
    for (int64_t r = 0; r < rows; r++)
        for (int64_t b = 0; b < nb; b++) {
            uint8_t* o = blocks + (r * nb + b) * 34;
            uint16_t dv = d[r * nb + b];
            o[0] = (uint8_t)(dv & 0xFF);
            o[1] = (uint8_t)(dv >> 8);
            memcpy(o + 2, qs + r * k + b * ORC_QK, ORC_QK);
        }
}

void orc_q8_0_unpack_blocks(const uint8_t* blocks, int64_t rows, int64_t k, int8_t* qs, uint16_t* d) {
    int64_t nb = k / ORC_QK;
    for (int64_t r = 0; r < rows; r++)
        for (int64_t b = 0; b < nb; b++) {
            const uint8_t* o = blocks + (r * nb + b) * 34;
            d[r * nb + b] = (uint16_t)(o[0] | (o[1] << 8));
            memcpy(qs + r * k + b * ORC_QK, o + 2, ORC_QK);
        }
}

/* GGML ggml_vec_dot_q8_0_q8_0 (scalar path): sumf += sumi * (d_w * d_x), blocks ascending. */
void orc_q8_0_matmul(const int8_t* xq, const uint16_t* xd, int64_t m,
                     const int8_t* wq, const uint16_t* wd, int64_t n, int64_t k,
                     float* y, float* abs_terms) {
    int64_t nb = k / ORC_QK;
#pragma omp parallel for schedule(static) collapse(2)
    for (int64_t i = 0; i < m; i++) {
        for (int64_t j = 0; j < n; j++) {
            const int8_t* a = xq + i * k;
            const int8_t* w = wq + j * k;
            float acc = 0.0f, accabs = 0.0f;
            for (int64_t b = 0; b < nb; b++) {
                int32_t s = 0;
                for (int t = 0; t < ORC_QK; t++) s += (int32_t)a[b * ORC_QK + t] * (int32_t)w[b * ORC_QK + t];
                float sc = orc_f16_to_f32(wd[j * nb + b]) * orc_f16_to_f32(xd[i * nb + b]);
                float term = (float)s * sc;
                acc = acc + term;
                accabs = accabs + fabsf(term);
            }
            y[i * n + j] = acc;
            if (abs_terms) abs_terms[i * n + j] = accabs;
        }
    }
}

void orc_q8_0_linear_f32(const float* x, int64_t m, int64_t k,
                         const int8_t* wq, const uint16_t* wd, int64_t n, float* y) {
    int8_t* xq = (int8_t*)malloc((size_t)(m * k));
    uint16_t* xd = (uint16_t*)malloc((size_t)(m * (k / ORC_QK)) * 2);
    orc_q8_0_quantize_f32(x, m, k, xq, xd);
    orc_q8_0_matmul(xq, xd, m, wq, wd, n, k, y, NULL);
    free(xq); free(xd);
}

void orc_q8_0_linear_bf16(const uint16_t* x, int64_t m, int64_t k,
                          const int8_t* wq, const uint16_t* wd, int64_t n, float* y) {
    int8_t* xq = (int8_t*)malloc((size_t)(m * k));
    uint16_t* xd = (uint16_t*)malloc((size_t)(m * (k / ORC_QK)) * 2);
    orc_q8_0_quantize_bf16(x, m, k, xq, xd);
    orc_q8_0_matmul(xq, xd, m, wq, wd, n, k, y, NULL);
    free(xq); free(xd);
}

/* tensor.rs:2716-2753: C[i,j] = sum_k A[i,k]*B[k,j], k ascending, one f32 accumulator. */
void orc_matmul_2d(const float* a, int64_t m, int64_t k, const float* b, int64_t n, float* c) {
    for (int64_t i = 0; i < m; i++)
        for (int64_t j = 0; j < n; j++) {
            float sum = 0.0f;
            for (int64_t t = 0; t < k; t++) { float p = a[i * k + t] * b[t * n + j]; sum = sum + p; }
            c[i * n + j] = sum;
        }
}

/* ====================================================================================== */
/* small ops                                                                              */
/* ====================================================================================== */

/* rms_norm.rs:144-176 on bf16 data: f32 sum of squares in order, inv = 1/sqrt(mean + eps),
 * out = bf16((x * inv) * w). */
/* Noise probe for the tests (never set by a reference path): 1 sums the squares in reverse
 * order, a reordering as legitimate as the reference's own, so that oracle-vs-oracle gives the
 * model's sensitivity to f32 summation order. */
static int g_sum_order_reversed = 0;
void orc_set_sum_order(int reversed) { g_sum_order_reversed = reversed; }

static void rmsnorm_row_bf16(const uint16_t* x, int64_t dim, const uint16_t* w, float eps, uint16_t* out) {
    float sum_sq = 0.0f;
    if (g_sum_order_reversed) {
        for (int64_t i = dim - 1; i >= 0; i--) { float v = orc_bf16_to_f32(x[i]); float p = v * v; sum_sq = sum_sq + p; }
    } else {
        for (int64_t i = 0; i < dim; i++) { float v = orc_bf16_to_f32(x[i]); float p = v * v; sum_sq = sum_sq + p; }
    }
    float mean_sq = sum_sq / (float)dim;
    float inv_rms = 1.0f / sqrtf(mean_sq + eps);
    for (int64_t i = 0; i < dim; i++) {
        float v = orc_bf16_to_f32(x[i]);
        float t = v * inv_rms;
        float nrm = t * orc_bf16_to_f32(w[i]);
        out[i] = orc_f32_to_bf16(nrm);
    }
}

void orc_rmsnorm_bf16(const uint16_t* x, int64_t rows, int64_t dim, const uint16_t* w, float eps, uint16_t* out) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) rmsnorm_row_bf16(x + r * dim, dim, w, eps, out + r * dim);
}

/* rms_norm.rs:144: an F32 input is first rounded to BF16 (to_vec_bf16). */
void orc_rmsnorm_f32(const float* x, int64_t rows, int64_t dim, const uint16_t* w, float eps, uint16_t* out) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        uint16_t* tmp = (uint16_t*)malloc((size_t)dim * 2);
        for (int64_t i = 0; i < dim; i++) tmp[i] = orc_f32_to_bf16(x[r * dim + i]);
        rmsnorm_row_bf16(tmp, dim, w, eps, out + r * dim);
        free(tmp);
    }
}

/* rope.rs:77-128: rope_dim = head_dim/2, inv_freq[i] = 1/theta^(2i/rope_dim) for
 * i < rope_dim/2, entries 2i and 2i+1 of each row both hold angle pos*inv_freq[i]; cos and
 * sin are evaluated in f64 and stored as f32. */
void orc_rope_tables(int64_t head_dim, int64_t max_pos, double theta, float* cos_t, float* sin_t) {
    int64_t rope_dim = head_dim / 2, half = rope_dim / 2;
    double* inv_freq = (double*)malloc(sizeof(double) * (size_t)half);
    for (int64_t i = 0; i < half; i++) inv_freq[i] = 1.0 / pow(theta, (double)(2 * i) / (double)rope_dim);
    for (int64_t p = 0; p < max_pos; p++)
        for (int64_t i = 0; i < half; i++) {
            double fr = (double)p * inv_freq[i];
            float c = (float)cos(fr), s = (float)sin(fr);
            cos_t[p * rope_dim + 2 * i] = c; cos_t[p * rope_dim + 2 * i + 1] = c;
            sin_t[p * rope_dim + 2 * i] = s; sin_t[p * rope_dim + 2 * i + 1] = s;
        }
    free(inv_freq);
}

/* rope.rs:245-303: for pair p < rope_dim/2, dims (2p, 2p+1) rotate against
 * (rope_dim+2p, rope_dim+2p+1) with the table entry at column 2p. */
void orc_rope_apply(float* x, int64_t bh, int64_t seq, int64_t head_dim, int64_t offset,
                    const float* cos_t, const float* sin_t) {
    int64_t rope_dim = head_dim / 2;
    for (int64_t h = 0; h < bh; h++)
        for (int64_t l = 0; l < seq; l++) {
            float* r = x + (h * seq + l) * head_dim;
            const float* ct = cos_t + (offset + l) * rope_dim;
            const float* st = sin_t + (offset + l) * rope_dim;
            for (int64_t p = 0; p < rope_dim / 2; p++) {
                int64_t d0 = 2 * p, d1 = 2 * p + 1;
                float x10 = r[d0], x11 = r[d1], x20 = r[rope_dim + d0], x21 = r[rope_dim + d1];
                float c = ct[d0], s = st[d0];
                float a, b;
                a = x10 * c; b = x20 * s; r[d0] = a - b;
                a = x11 * c; b = x21 * s; r[d1] = a - b;
                a = x20 * c; b = x10 * s; r[rope_dim + d0] = a + b;
                a = x21 * c; b = x11 * s; r[rope_dim + d1] = a + b;
            }
        }
}

/* tensor.rs:1977-1986 (F32 branch): x / (1 + exp(-x)) */
float orc_silu(float x) { float e = expf(-x); float den = 1.0f + e; return x / den; }

/* tensor.rs:2451-2482 with Rust's Iterator::max_by: the later element wins unless the current
 * best compares Greater; NaN compares Equal. */
int64_t orc_argmax(const float* x, int64_t n) {
    int64_t best = 0;
    for (int64_t i = 1; i < n; i++)
        if (!(x[best] > x[i])) best = i;
    return best;
}

/* tensor.rs:1913-1934: max (from -inf), subtract, exp, sum in order, divide. */
void orc_softmax(float* x, int64_t n) {
    float mx = -INFINITY;
    for (int64_t i = 0; i < n; i++) if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (int64_t i = 0; i < n; i++) { x[i] = expf(x[i] - mx); sum = sum + x[i]; }
    for (int64_t i = 0; i < n; i++) x[i] = x[i] / sum;
}

/* attention.rs:368-394 for one query row: scores = (q . k_j) * (1/sqrt(d)), masked entries
 * j > causal_limit get -inf added (causal_mask.rs:143-150), softmax, out = sum_j p_j v_j. */
void orc_attend_row(const float* q, const float* k, const float* v, int64_t ctx, int64_t ld,
                    int64_t d, int masked, int64_t causal_limit, float* scratch, float* out) {
    float scale = 1.0f / sqrtf((float)d);
    for (int64_t j = 0; j < ctx; j++) {
        float s = 0.0f;
        for (int64_t t = 0; t < d; t++) { float p = q[t] * k[j * ld + t]; s = s + p; }
        s = s * scale;
        if (masked) s = s + (j > causal_limit ? -INFINITY : 0.0f);
        scratch[j] = s;
    }
    orc_softmax(scratch, ctx);
    for (int64_t t = 0; t < d; t++) {
        float acc = 0.0f;
        for (int64_t j = 0; j < ctx; j++) { float p = scratch[j] * v[j * ld + t]; acc = acc + p; }
        out[t] = acc;
    }
}

/* ====================================================================================== */
/* Qwen3 model                                                                            */
/* ====================================================================================== */

/* Tensor ids of the seeded generator; the CUDA library uses the same numbering. */
enum { K_Q = 0, K_K, K_V, K_O, K_GATE, K_UP, K_DOWN, K_QNORM, K_KNORM, K_INNORM, K_POSTNORM, K_ROUTER };
#define TID_LAYER(l, kind) (((uint64_t)(l) << 8) | (uint64_t)(kind))
/* expert weights: kind 0 gate, 1 up, 2 down */
#define TID_EXPERT(l, e, kind) ((1ull << 40) | ((uint64_t)(l) << 20) | ((uint64_t)(e) << 4) | (uint64_t)(kind))
#define TID_EMBED 0x7FFF0001ull
#define TID_LMHEAD 0x7FFF0002ull
#define TID_FINALNORM 0x7FFF0003ull

typedef struct { int64_t n, k; int8_t* qs; uint16_t* d; } qw_t;

typedef struct {
    qw_t q, k, v, o, gate, up, down;
    uint16_t *q_norm, *k_norm, *in_norm, *post_norm;
    qw_t router;             /* MoE: [E][H] */
    qw_t *eg, *eu, *ed;      /* MoE: per-expert gate [moe_inter][H], up, down [H][moe_inter] */
} layer_t;

struct orc_model {
    orc_qwen3_config c;
    int64_t nl, ctx_max;
    uint16_t* embed;         /* [vocab][hidden] bf16 */
    uint16_t* final_norm;
    qw_t lm_head;
    layer_t* L;
    float *kc, *vc;          /* [nl][n_kv][ctx_max][head_dim] */
    float *cos_t, *sin_t;
};

static void make_linear(qw_t* w, uint64_t seed, uint64_t tid, int64_t n, int64_t k, float scale) {
    w->n = n; w->k = k;
    w->qs = (int8_t*)malloc((size_t)(n * k));
    w->d = (uint16_t*)malloc((size_t)(n * (k / ORC_QK)) * 2);
    int64_t chunk = 256;
    uint16_t* tmp = (uint16_t*)malloc((size_t)(chunk * k) * 2);
    for (int64_t r = 0; r < n; r += chunk) {
        int64_t rows = (n - r) < chunk ? (n - r) : chunk;
        orc_gen_bf16(seed, tid, r * k, rows * k, scale, tmp);
        orc_q8_0_quantize_bf16(tmp, rows, k, w->qs + r * k, w->d + r * (k / ORC_QK));
    }
    free(tmp);
}

static uint16_t* make_norm(const orc_qwen3_config* c, uint64_t seed, uint64_t tid, int64_t dim) {
    uint16_t* w = (uint16_t*)malloc((size_t)dim * 2);
    if (c->norm_std == 0.0f) {
        for (int64_t i = 0; i < dim; i++) w[i] = 0x3F80;      /* 1.0 */
    } else {
        uint64_t key = gen_key(seed, tid);
        float sc = orc_gen_scale(c->norm_std);
        for (int64_t i = 0; i < dim; i++) w[i] = orc_f32_to_bf16(1.0f + gen_value(key, (uint64_t)i, sc));
    }
    return w;
}

orc_model* orc_qwen3_create(const orc_qwen3_config* cfg, uint64_t seed, int64_t layers_limit, int64_t ctx_max) {
    orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
    m->c = *cfg;
    m->nl = (layers_limit > 0 && layers_limit < cfg->layers) ? layers_limit : cfg->layers;
    m->ctx_max = ctx_max;
    const orc_qwen3_config* c = cfg;
    float sc = orc_gen_scale(c->init_std);
    int64_t H = c->hidden, D = c->head_dim;
    m->embed = (uint16_t*)malloc((size_t)(c->vocab * H) * 2);
    orc_gen_bf16(seed, TID_EMBED, 0, c->vocab * H, sc, m->embed);
    m->final_norm = make_norm(c, seed, TID_FINALNORM, H);
    if (c->tied) {
        m->lm_head.n = c->vocab; m->lm_head.k = H;
        m->lm_head.qs = (int8_t*)malloc((size_t)(c->vocab * H));
        m->lm_head.d = (uint16_t*)malloc((size_t)(c->vocab * (H / ORC_QK)) * 2);
        orc_q8_0_quantize_bf16(m->embed, c->vocab, H, m->lm_head.qs, m->lm_head.d);
    } else {
        make_linear(&m->lm_head, seed, TID_LMHEAD, c->vocab, H, sc);
    }
    m->L = (layer_t*)calloc((size_t)m->nl, sizeof(layer_t));
    for (int64_t l = 0; l < m->nl; l++) {
        layer_t* ly = &m->L[l];
        make_linear(&ly->q, seed, TID_LAYER(l, K_Q), c->n_heads * D, H, sc);
        make_linear(&ly->k, seed, TID_LAYER(l, K_K), c->n_kv_heads * D, H, sc);
        make_linear(&ly->v, seed, TID_LAYER(l, K_V), c->n_kv_heads * D, H, sc);
        make_linear(&ly->o, seed, TID_LAYER(l, K_O), H, c->n_heads * D, sc);
        if (c->n_experts > 0) {
            int64_t E = c->n_experts, I = c->moe_inter;
            make_linear(&ly->router, seed, TID_LAYER(l, K_ROUTER), E, H, sc);
            ly->eg = (qw_t*)calloc((size_t)E, sizeof(qw_t));
            ly->eu = (qw_t*)calloc((size_t)E, sizeof(qw_t));
            ly->ed = (qw_t*)calloc((size_t)E, sizeof(qw_t));
            for (int64_t e = 0; e < E; e++) {
                make_linear(&ly->eg[e], seed, TID_EXPERT(l, e, 0), I, H, sc);
                make_linear(&ly->eu[e], seed, TID_EXPERT(l, e, 1), I, H, sc);
                make_linear(&ly->ed[e], seed, TID_EXPERT(l, e, 2), H, I, sc);
            }
        } else {
            make_linear(&ly->gate, seed, TID_LAYER(l, K_GATE), c->inter, H, sc);
            make_linear(&ly->up, seed, TID_LAYER(l, K_UP), c->inter, H, sc);
            make_linear(&ly->down, seed, TID_LAYER(l, K_DOWN), H, c->inter, sc);
        }
        ly->q_norm = make_norm(c, seed, TID_LAYER(l, K_QNORM), D);
        ly->k_norm = make_norm(c, seed, TID_LAYER(l, K_KNORM), D);
        ly->in_norm = make_norm(c, seed, TID_LAYER(l, K_INNORM), H);
        ly->post_norm = make_norm(c, seed, TID_LAYER(l, K_POSTNORM), H);
    }
    size_t kv = (size_t)(m->nl * c->n_kv_heads * ctx_max * D);
    m->kc = (float*)calloc(kv, sizeof(float));
    m->vc = (float*)calloc(kv, sizeof(float));
    int64_t rope_rows = ctx_max;   /* only positions < ctx_max are ever looked up */
    m->cos_t = (float*)malloc(sizeof(float) * (size_t)(rope_rows * D / 2));
    m->sin_t = (float*)malloc(sizeof(float) * (size_t)(rope_rows * D / 2));
    orc_rope_tables(D, rope_rows, c->theta, m->cos_t, m->sin_t);
    return m;
}

static void free_lin(qw_t* w) { free(w->qs); free(w->d); }

void orc_qwen3_destroy(orc_model* m) {
    if (!m) return;
    for (int64_t l = 0; l < m->nl; l++) {
        layer_t* ly = &m->L[l];
        free_lin(&ly->q); free_lin(&ly->k); free_lin(&ly->v); free_lin(&ly->o);
        free_lin(&ly->gate); free_lin(&ly->up); free_lin(&ly->down);
        free(ly->q_norm); free(ly->k_norm); free(ly->in_norm); free(ly->post_norm);
        if (ly->eg) {
            for (int64_t e = 0; e < m->c.n_experts; e++) {
                free_lin(&ly->eg[e]); free_lin(&ly->eu[e]); free_lin(&ly->ed[e]);
            }
            free(ly->eg); free(ly->eu); free(ly->ed);
            free_lin(&ly->router);
        }
    }
    free(m->L); free(m->embed); free(m->final_norm); free_lin(&m->lm_head);
    free(m->kc); free(m->vc); free(m->cos_t); free(m->sin_t);
    free(m);
}

void orc_qwen3_clear(orc_model* m) {
    size_t kv = (size_t)(m->nl * m->c.n_kv_heads * m->ctx_max * m->c.head_dim);
    memset(m->kc, 0, kv * sizeof(float));
    memset(m->vc, 0, kv * sizeof(float));
}

int64_t orc_qwen3_layers(const orc_model* m) { return m->nl; }
const uint16_t* orc_qwen3_embed(const orc_model* m) { return m->embed; }

int64_t orc_qwen3_linear(const orc_model* m, int64_t layer, int kind, const int8_t** qs,
                         const uint16_t** d, int64_t* k) {
    const qw_t* w = NULL;
    if (layer < 0) {
        if (kind == 7) w = &m->lm_head;
    } else if (layer < m->nl) {
        const layer_t* ly = &m->L[layer];
        const qw_t* all[7] = {&ly->q, &ly->k, &ly->v, &ly->o, &ly->gate, &ly->up, &ly->down};
        if (kind >= 0 && kind < 7) w = all[kind];
    }
    if (!w || !w->qs) return -1;
    *qs = w->qs; *d = w->d; *k = w->k;
    return w->n;
}

int64_t orc_qwen3_expert(const orc_model* m, int64_t layer, int64_t expert, int kind, const int8_t** qs,
                         const uint16_t** d, int64_t* k) {
    if (layer < 0 || layer >= m->nl || m->c.n_experts <= 0) return -1;
    const layer_t* ly = &m->L[layer];
    const qw_t* w = NULL;
    if (kind == 10) w = &ly->router;
    else if (expert >= 0 && expert < m->c.n_experts) {
        if (kind == 11) w = &ly->eg[expert];
        else if (kind == 12) w = &ly->eu[expert];
        else if (kind == 13) w = &ly->ed[expert];
    }
    if (!w || !w->qs) return -1;
    *qs = w->qs; *d = w->d; *k = w->k;
    return w->n;
}

void orc_moe_forward(const uint16_t* xn, int64_t rows, int64_t H, int64_t E, int64_t top_k, int64_t inter,
                     int norm_topk, const int8_t* rq, const uint16_t* rd, const int8_t* const* gq,
                     const uint16_t* const* gd, const int8_t* const* uq, const uint16_t* const* ud,
                     const int8_t* const* dq, const uint16_t* const* dd, float* out, int32_t* ids,
                     float* weights) {
    float* logits = (float*)malloc(sizeof(float) * (size_t)(rows * E));
    orc_q8_0_linear_bf16(xn, rows, H, rq, rd, E, logits);
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t t = 0; t < rows; t++) {
        const float* lg = logits + t * E;
        float* p = (float*)malloc(sizeof(float) * (size_t)E);
        int32_t* sel = (int32_t*)malloc(sizeof(int32_t) * (size_t)top_k);
        float* w = (float*)malloc(sizeof(float) * (size_t)top_k);
        char* used = (char*)calloc((size_t)E, 1);
        float* g = (float*)malloc(sizeof(float) * (size_t)inter);
        float* u = (float*)malloc(sizeof(float) * (size_t)inter);
        float* y = (float*)malloc(sizeof(float) * (size_t)H);
        float* acc = (float*)calloc((size_t)H, sizeof(float));
        memcpy(p, lg, sizeof(float) * (size_t)E);
        orc_softmax(p, E);
        /* top-k by logit; on equal logits the lower expert index first */
        for (int64_t j = 0; j < top_k; j++) {
            int64_t best = -1;
            for (int64_t e = 0; e < E; e++)
                if (!used[e] && (best < 0 || lg[e] > lg[best])) best = e;
            used[best] = 1;
            sel[j] = (int32_t)best;
            w[j] = p[best];
        }
        if (norm_topk) {
            float s = 0.0f;
            for (int64_t j = 0; j < top_k; j++) s = s + w[j];
            for (int64_t j = 0; j < top_k; j++) w[j] = w[j] / s;
        }
        if (ids) for (int64_t j = 0; j < top_k; j++) ids[t * top_k + j] = sel[j];
        if (weights) for (int64_t j = 0; j < top_k; j++) weights[t * top_k + j] = w[j];
        /* experts in ascending index (the index_add order of the sparse block) */
        for (int64_t e = 0; e < E; e++) {
            if (!used[e]) continue;
            float we = 0.0f;
            for (int64_t j = 0; j < top_k; j++) if (sel[j] == e) we = w[j];
            orc_q8_0_linear_bf16(xn + t * H, 1, H, gq[e], gd[e], inter, g);
            orc_q8_0_linear_bf16(xn + t * H, 1, H, uq[e], ud[e], inter, u);
            for (int64_t i = 0; i < inter; i++) { float s = orc_silu(g[i]); g[i] = s * u[i]; }
            orc_q8_0_linear_f32(g, 1, inter, dq[e], dd[e], H, y);
            for (int64_t i = 0; i < H; i++) acc[i] = acc[i] + we * y[i];
        }
        memcpy(out + t * H, acc, sizeof(float) * (size_t)H);
        free(p); free(sel); free(w); free(used); free(g); free(u); free(y); free(acc);
    }
    free(logits);
}

static void lin_bf16(const qw_t* w, const uint16_t* x, int64_t rows, float* y) {
    orc_q8_0_linear_bf16(x, rows, w->k, w->qs, w->d, w->n, y);
}
static void lin_f32(const qw_t* w, const float* x, int64_t rows, float* y) {
    orc_q8_0_linear_f32(x, rows, w->k, w->qs, w->d, w->n, y);
}

/* DecoderLayer::forward (transformer.rs:180-204) with Attention::forward
 * (attention.rs:318-403) and MLP::forward (mlp.rs:151-164); x is [L][H] f32 in place. */
static void layer_forward(orc_model* m, int64_t li, float* x, int64_t L, int64_t offset) {
    const orc_qwen3_config* c = &m->c;
    layer_t* ly = &m->L[li];
    int64_t H = c->hidden, D = c->head_dim, Hq = c->n_heads, Hk = c->n_kv_heads, I = c->inter;
    int64_t groups = Hq / Hk, ctx = offset + L;
    uint16_t* xn = (uint16_t*)malloc((size_t)(L * H) * 2);
    float* q = (float*)malloc(sizeof(float) * (size_t)(L * Hq * D));
    float* k = (float*)malloc(sizeof(float) * (size_t)(L * Hk * D));
    float* v = (float*)malloc(sizeof(float) * (size_t)(L * Hk * D));
    orc_rmsnorm_f32(x, L, H, ly->in_norm, c->eps, xn);
    lin_bf16(&ly->q, xn, L, q);
    lin_bf16(&ly->k, xn, L, k);
    lin_bf16(&ly->v, xn, L, v);
    /* [L][Hx][D] -> per-head [Hx][L][D], per-head RMSNorm, RoPE (attention.rs:337-361) */
    float* qh = (float*)malloc(sizeof(float) * (size_t)(Hq * L * D));
    float* kh = (float*)malloc(sizeof(float) * (size_t)(Hk * L * D));
    uint16_t* tb = (uint16_t*)malloc((size_t)D * 2);
    for (int64_t h = 0; h < Hq; h++)
        for (int64_t l = 0; l < L; l++) {
            orc_rmsnorm_f32(q + (l * Hq + h) * D, 1, D, ly->q_norm, c->eps, tb);
            for (int64_t t = 0; t < D; t++) qh[(h * L + l) * D + t] = orc_bf16_to_f32(tb[t]);
        }
    for (int64_t h = 0; h < Hk; h++)
        for (int64_t l = 0; l < L; l++) {
            orc_rmsnorm_f32(k + (l * Hk + h) * D, 1, D, ly->k_norm, c->eps, tb);
            for (int64_t t = 0; t < D; t++) kh[(h * L + l) * D + t] = orc_bf16_to_f32(tb[t]);
        }
    free(tb);
    orc_rope_apply(qh, Hq, L, D, offset, m->cos_t, m->sin_t);
    orc_rope_apply(kh, Hk, L, D, offset, m->cos_t, m->sin_t);
    /* KvCache::append (attention.rs:507-559): cat along the sequence axis */
    float* kc = m->kc + li * Hk * m->ctx_max * D;
    float* vc = m->vc + li * Hk * m->ctx_max * D;
    for (int64_t h = 0; h < Hk; h++)
        for (int64_t l = 0; l < L; l++)
            for (int64_t t = 0; t < D; t++) {
                kc[(h * m->ctx_max + offset + l) * D + t] = kh[(h * L + l) * D + t];
                vc[(h * m->ctx_max + offset + l) * D + t] = v[(l * Hk + h) * D + t];
            }
    /* attention per (head, row); output [L][Hq*D] (attention.rs:396-399) */
    float* att = (float*)malloc(sizeof(float) * (size_t)(L * Hq * D));
#pragma omp parallel for schedule(static) collapse(2)
    for (int64_t h = 0; h < Hq; h++)
        for (int64_t l = 0; l < L; l++) {
            float* scratch = (float*)malloc(sizeof(float) * (size_t)ctx);
            int64_t kvh = h / groups;  /* repeat_kv (attention.rs:426-456) */
            orc_attend_row(qh + (h * L + l) * D, kc + kvh * m->ctx_max * D, vc + kvh * m->ctx_max * D,
                           ctx, D, D, L > 1, offset + l, scratch, att + (l * Hq + h) * D);
            free(scratch);
        }
    float* o = (float*)malloc(sizeof(float) * (size_t)(L * H));
    lin_f32(&ly->o, att, L, o);
    for (int64_t i = 0; i < L * H; i++) x[i] = x[i] + o[i];
    /* MLP */
    orc_rmsnorm_f32(x, L, H, ly->post_norm, c->eps, xn);
    if (c->n_experts > 0) {
        int64_t E = c->n_experts;
        const int8_t** gq = (const int8_t**)malloc(sizeof(void*) * (size_t)E * 6);
        const uint16_t** gd = (const uint16_t**)(gq + E);
        const int8_t** uq = (const int8_t**)(gq + 2 * E);
        const uint16_t** ud = (const uint16_t**)(gq + 3 * E);
        const int8_t** dq = (const int8_t**)(gq + 4 * E);
        const uint16_t** dd = (const uint16_t**)(gq + 5 * E);
        for (int64_t e = 0; e < E; e++) {
            gq[e] = ly->eg[e].qs; gd[e] = ly->eg[e].d;
            uq[e] = ly->eu[e].qs; ud[e] = ly->eu[e].d;
            dq[e] = ly->ed[e].qs; dd[e] = ly->ed[e].d;
        }
        orc_moe_forward(xn, L, H, E, c->top_k, c->moe_inter, c->norm_topk, ly->router.qs, ly->router.d,
                        gq, gd, uq, ud, dq, dd, o, NULL, NULL);
        free((void*)gq);
        for (int64_t i = 0; i < L * H; i++) x[i] = x[i] + o[i];
        free(xn); free(q); free(k); free(v); free(qh); free(kh); free(att); free(o);
        return;
    }
    float* g = (float*)malloc(sizeof(float) * (size_t)(L * I));
    float* u = (float*)malloc(sizeof(float) * (size_t)(L * I));
    lin_bf16(&ly->gate, xn, L, g);
    lin_bf16(&ly->up, xn, L, u);
    for (int64_t i = 0; i < L * I; i++) { float s = orc_silu(g[i]); g[i] = s * u[i]; }
    lin_f32(&ly->down, g, L, o);
    for (int64_t i = 0; i < L * H; i++) x[i] = x[i] + o[i];
    free(xn); free(q); free(k); free(v); free(qh); free(kh); free(att); free(o); free(g); free(u);
}

int orc_qwen3_forward(orc_model* m, const int32_t* ids, int64_t L, int64_t offset, float* logits) {
    const orc_qwen3_config* c = &m->c;
    int64_t H = c->hidden;
    if (L <= 0 || offset + L > m->ctx_max) return -1;
    for (int64_t i = 0; i < L; i++) if (ids[i] < 0 || ids[i] >= c->vocab) return -1;
    float* x = (float*)malloc(sizeof(float) * (size_t)(L * H));
    /* Embedding::forward (embedding.rs:105-153): BF16 rows; widened exactly */
    for (int64_t i = 0; i < L; i++)
        for (int64_t t = 0; t < H; t++) x[i * H + t] = orc_bf16_to_f32(m->embed[(int64_t)ids[i] * H + t]);
    for (int64_t l = 0; l < m->nl; l++) layer_forward(m, l, x, L, offset);
    /* final norm, last row, LM head (model.rs:194, :357-369) */
    uint16_t* xn = (uint16_t*)malloc((size_t)H * 2);
    orc_rmsnorm_f32(x + (L - 1) * H, 1, H, m->final_norm, c->eps, xn);
    lin_bf16(&m->lm_head, xn, 1, logits);
    free(xn); free(x);
    return 0;
}

int orc_qwen3_generate(orc_model* m, const int32_t* prompt, int64_t L, int64_t new_tokens,
                       int32_t* out_tokens, float* last_logits) {
    int64_t V = m->c.vocab;
    float* logits = (float*)malloc(sizeof(float) * (size_t)V);
    orc_qwen3_clear(m);
    if (orc_qwen3_forward(m, prompt, L, 0, logits)) { free(logits); return -1; }
    int32_t next = (int32_t)orc_argmax(logits, V);
    out_tokens[0] = next;
    for (int64_t i = 1; i < new_tokens; i++) {
        if (orc_qwen3_forward(m, &next, 1, L + i - 1, logits)) { free(logits); return -1; }
        next = (int32_t)orc_argmax(logits, V);
        out_tokens[i] = next;
    }
    if (last_logits) memcpy(last_logits, logits, sizeof(float) * (size_t)V);
    free(logits);
    return 0;
}

/* ---- sampling (generate.rs) ----------------------------------------------------------
 * Every strategy of the reference picks a token deterministically ("Phase 0"):
 *   sample_greedy (generate.rs:153-175): argmax, ties -> the last index (orc_argmax);
 *   sample_temperature (:190-210): T == 1 (within 1e-6) -> greedy, else greedy over
 *     x * (1/T) (mul_scalar, tensor.rs:1515-1519);
 *   sample_top_k (:228-257): a stable sort by value descending, the first element: the
 *     maximum, ties -> the first index (temperature unused);
 *   sample_top_p (:274-326): p == 1 -> sample_temperature; else s = x / T when T != 1,
 *     probabilities exp(s - max) / sum (sum in index order), a stable sort by probability
 *     descending, the first element: ties -> the first index;
 *   apply_repetition_penalty (:374-411): for every generated token in order (repeats
 *     included), x > 0 -> x / penalty, x < 0 -> x * penalty;
 *   sample_with_config (:687-705): penalty, then greedy when T == 0 or (T == 1 and k == 0
 *     and p == 1), else top-k when k > 0, else top-p when p != 1, else temperature.
 * Logits are assumed finite (the reference's partial_cmp makes NaN order unspecified). */
static int64_t argmax_first(const float* x, int64_t n) {
    int64_t best = 0;
    for (int64_t i = 1; i < n; i++)
        if (x[i] > x[best]) best = i;
    return best;
}

/* exp as the reference's f32::exp (libm expf), or correctly rounded (exp in double, rounded
 * once to f32) -- the device's choice for top-p, see orc_sample_ex */
static float exp_f32(float x, int cr) { return cr ? (float)exp((double)x) : expf(x); }

int32_t orc_sample(const float* logits, int64_t V, const int32_t* generated, int64_t n_generated,
                   float temperature, int64_t top_k, float top_p, float penalty) {
    return orc_sample_ex(logits, V, generated, n_generated, temperature, top_k, top_p, penalty, 0);
}

int32_t orc_sample_ex(const float* logits, int64_t V, const int32_t* generated, int64_t n_generated,
                      float temperature, int64_t top_k, float top_p, float penalty, int cr_exp) {
    float* x = (float*)malloc(sizeof(float) * (size_t)V);
    memcpy(x, logits, sizeof(float) * (size_t)V);
    if (!(fabsf(penalty - 1.0f) < 1e-6f) && n_generated > 0) {
        for (int64_t i = 0; i < n_generated; i++) {
            const int64_t t = (int64_t)(uint32_t)generated[i];
            if (t < V) {
                const float v = x[t];
                if (v > 0.0f) x[t] = v / penalty;
                else if (v < 0.0f) x[t] = v * penalty;
            }
        }
    }
    int64_t tok;
    const int temp_one = fabsf(temperature - 1.0f) < 1e-6f;
    const int p_one = fabsf(top_p - 1.0f) < 1e-6f;
    if (temperature == 0.0f || (temp_one && top_k == 0 && p_one)) {
        tok = orc_argmax(x, V);
    } else if (top_k > 0) {
        tok = argmax_first(x, V);
    } else if (!p_one) {
        if (!temp_one)
            for (int64_t i = 0; i < V; i++) x[i] = x[i] / temperature;
        float mx = x[0];
        for (int64_t i = 1; i < V; i++)
            if (!(mx > x[i])) mx = x[i];
        float sum = 0.0f;
        for (int64_t i = 0; i < V; i++) sum = sum + exp_f32(x[i] - mx, cr_exp);
        for (int64_t i = 0; i < V; i++) x[i] = exp_f32(x[i] - mx, cr_exp) / sum;
        tok = argmax_first(x, V);
    } else {
        const float inv = 1.0f / temperature;
        for (int64_t i = 0; i < V; i++) x[i] = x[i] * inv;
        tok = orc_argmax(x, V);
    }
    free(x);
    return (int32_t)tok;
}

/* generate (generate.rs:611-661) with a sampling configuration: the first token from the
 * prompt's logits with no history, then one token per step with the history of every token
 * generated so far (the prompt is not part of it); EOS is not checked. */
int orc_qwen3_generate_cfg(orc_model* m, const int32_t* prompt, int64_t L, int64_t new_tokens,
                           float temperature, int64_t top_k, float top_p, float penalty,
                           int32_t* out_tokens, float* last_logits) {
    int64_t V = m->c.vocab;
    float* logits = (float*)malloc(sizeof(float) * (size_t)V);
    orc_qwen3_clear(m);
    if (orc_qwen3_forward(m, prompt, L, 0, logits)) { free(logits); return -1; }
    int32_t next = orc_sample(logits, V, out_tokens, 0, temperature, top_k, top_p, penalty);
    out_tokens[0] = next;
    for (int64_t i = 1; i < new_tokens; i++) {
        if (orc_qwen3_forward(m, &next, 1, L + i - 1, logits)) { free(logits); return -1; }
        next = orc_sample(logits, V, out_tokens, i, temperature, top_k, top_p, penalty);
        out_tokens[i] = next;
    }
    if (last_logits) memcpy(last_logits, logits, sizeof(float) * (size_t)V);
    free(logits);
    return 0;
}

void orc_set_threads(int n) {
#ifdef _OPENMP
    omp_set_num_threads(n > 0 ? n : 1);
#else
    (void)n;
#endif
}
int orc_get_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
