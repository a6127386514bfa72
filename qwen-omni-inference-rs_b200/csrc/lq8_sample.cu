// lq8_sample.cu -- the reference's token choice on the device: sample_with_config
// (generate.rs:687-705) after apply_repetition_penalty (generate.rs:374-411), for rows of
// logits.
//
// Every strategy of the reference picks its token deterministically:
//   greedy (generate.rs:153-175)       argmax of x, ties -> the last index
//   temperature (:190-210)             argmax of x * (1/T) (f32 reciprocal), ties -> last
//   top-k (:228-257)                   first element of a stable descending sort: argmax of
//                                      x, ties -> the first index (T unused)
//   top-p (:274-326)                   s = x / T (T != 1), p_i = exp(s_i - max) / sum, the
//                                      first element of a stable descending sort of p
// and the penalty divides a positive logit by the penalty and multiplies a negative one, once
// per generated occurrence, in order. One CTA per row: the penalized row is written to a
// scratch copy (each distinct history token handled by the thread of its first occurrence,
// which applies its occurrences in order), then a block reduction of 64-bit keys (orderable
// value bits above the index, or its complement for ties to the first index) picks the token.
// Top-p: tokens whose exp(s - max) rounds to 1 share the maximum probability; a token whose
// exp(s - max) lies within 2^-22 below 1 may round to the same probability, which depends on
// the sum, so only then one thread forms the sum in index order (rare: two scaled logits
// within ~2.4e-7 of each other at the maximum). Top-p's exponentials are correctly rounded
// (exp in double, rounded once to f32); the reference's libm expf rounds a few inputs the
// other way, which can change the sum's last bit and so the choice in such a near-tie.
#include "lq8_async.cuh"
#include "lq8_internal.cuh"

#include <cmath>

namespace lq {

enum { SM_GREEDY = 0, SM_TEMP = 1, SM_TOPK = 2, SM_TOPP = 3 };
constexpr int SM_THREADS = 1024;

struct SampleParams {
    const float* logits;  // [rows][ld]
    int64_t ld;
    int V;
    const int32_t* gen;   // generated tokens [rows][gen_ld]
    int64_t gen_ld;
    int n_host;           // tokens generated so far; < 0: *pos - *gen_base + 1 (decode step)
    const int32_t* pos;
    const int32_t* gen_base;
    int mode;
    float inv_t;          // temperature: fl(1/T)
    float t;              // top-p: the divisor T
    int divide;           // top-p: T != 1
    float penalty;
    int use_penalty;
    float* scratch;       // [rows][V]
    int32_t* out;         // [rows]
    int32_t* gen_out;     // optional: the chosen token appended at gen[row][n]
};

__device__ __forceinline__ uint32_t order_bits(float v) {
    if (v == 0.0f) v = 0.0f;  // -0 == +0
    uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ unsigned long long block_max_u64(unsigned long long k, unsigned long long* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long x = __shfl_xor_sync(0xffffffffu, k, o);
        k = x > k ? x : k;
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = k;
    __syncthreads();
    k = 0ull;
    if (threadIdx.x < (blockDim.x >> 5)) k = red[threadIdx.x];
    if (warp == 0) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long x = __shfl_xor_sync(0xffffffffu, k, o);
            k = x > k ? x : k;
        }
        if (lane == 0) red[0] = k;
    }
    __syncthreads();
    return red[0];
}

// exp rounded once to f32 from a double-precision exp
__device__ __forceinline__ float exp_cr(float x) { return __double2float_rn(exp((double)x)); }

__device__ __forceinline__ float sm_value(const SampleParams& p, float v) {
    if (p.mode == SM_TEMP) return __fmul_rn(v, p.inv_t);
    if (p.mode == SM_TOPP && p.divide) return __fdiv_rn(v, p.t);
    return v;
}

__global__ void __launch_bounds__(SM_THREADS) sample_kernel(const SampleParams p) {
    __shared__ unsigned long long red[32];
    __shared__ int near_any;
    pdl_wait();
    pdl_trigger();
    const int row = blockIdx.x, tid = threadIdx.x, V = p.V;
    if (tid == 0) near_any = 0;  // ordered before its other uses by the reductions' barriers
    const float* l = p.logits + (int64_t)row * p.ld;
    int n = p.n_host;
    if (n < 0) n = *p.pos - *p.gen_base + 1;
    n = max(0, min(n, (int)p.gen_ld));
    const int32_t* gen = p.gen ? p.gen + (int64_t)row * p.gen_ld : nullptr;
    const float* src = l;
    if (p.use_penalty && n > 0 && gen) {
        float* x = p.scratch + (int64_t)row * V;
        for (int i = tid; i < V; i += blockDim.x) x[i] = l[i];
        __syncthreads();
        for (int h = tid; h < n; h += blockDim.x) {
            const uint32_t t = (uint32_t)gen[h];
            if (t >= (uint32_t)V) continue;
            bool first = true;
            for (int j = 0; j < h && first; j++) first = (uint32_t)gen[j] != t;
            if (!first) continue;
            float v = l[t];
            for (int j = h; j < n; j++)
                if ((uint32_t)gen[j] == t) {
                    if (v > 0.0f) v = __fdiv_rn(v, p.penalty);
                    else if (v < 0.0f) v = __fmul_rn(v, p.penalty);
                }
            x[t] = v;
        }
        __syncthreads();
        src = x;
    }
    const bool ties_first = p.mode == SM_TOPK || p.mode == SM_TOPP;
    unsigned long long key = 0ull;
    for (int i = tid; i < V; i += blockDim.x) {
        const unsigned long long k = ((unsigned long long)order_bits(sm_value(p, src[i])) << 32) |
                                     (ties_first ? (unsigned long long)(0xFFFFFFFFu - (uint32_t)i)
                                                 : (unsigned long long)(uint32_t)i);
        key = k > key ? k : key;
    }
    key = block_max_u64(key, red);
    int win = ties_first ? (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull)) : (int)(uint32_t)(key & 0xFFFFFFFFull);
    if (p.mode == SM_TOPP) {
        // tokens whose exp(s - max) rounds to 1 tie with the maximum's probability (the lowest
        // index wins); flag tokens just below 1, whose probability may round to the same value
        const float smax = sm_value(p, src[win]);
        unsigned long long lo = 0ull;  // complement-coded minimum index with exp == 1
        bool near = false;
        for (int i = tid; i < V; i += blockDim.x) {
            const float e = exp_cr(__fsub_rn(sm_value(p, src[i]), smax));
            if (e == 1.0f) lo = max(lo, (unsigned long long)(0xFFFFFFFFu - (uint32_t)i));
            else if (e >= 1.0f - 2.384185791015625e-7f) near = true;  // 1 - 2^-22
        }
        if (near) near_any = 1;
        lo = block_max_u64(lo, red);
        win = (int)(0xFFFFFFFFu - (uint32_t)lo);
        if (near_any && tid == 0) {
            // the probabilities themselves decide: sum in index order, then compare
            float sum = 0.0f;
            for (int i = 0; i < V; i++) sum = __fadd_rn(sum, exp_cr(__fsub_rn(sm_value(p, src[i]), smax)));
            const float pmax = __fdiv_rn(1.0f, sum);
            for (int i = 0; i < V; i++) {
                const float e = exp_cr(__fsub_rn(sm_value(p, src[i]), smax));
                if (__fdiv_rn(e, sum) == pmax) {
                    win = i;
                    break;
                }
            }
        }
    }
    if (tid == 0) {
        p.out[row] = win;
        if (p.gen_out && n < p.gen_ld) p.gen_out[(int64_t)row * p.gen_ld + n] = win;
    }
}

// the configuration's strategy (sample_with_config's dispatch, generate.rs:691-704)
static int sample_mode(const lq_sampling& c) {
    const bool t_one = std::fabs(c.temperature - 1.0f) < 1e-6f, p_one = std::fabs(c.top_p - 1.0f) < 1e-6f;
    if (c.temperature == 0.0f || (t_one && c.top_k == 0 && p_one)) return SM_GREEDY;
    if (c.top_k > 0) return SM_TOPK;
    if (!p_one) return SM_TOPP;
    return SM_TEMP;
}

bool sampling_is_greedy(const lq_sampling& c) {
    return sample_mode(c) == SM_GREEDY && !(std::fabs(c.repetition_penalty - 1.0f) >= 1e-6f);
}

int check_sampling(lq_ctx* ctx, const lq_sampling* c) {
    // GenerationConfig::new (generate.rs:93-126)
    LQ_REQUIRE(ctx, c, "sampling: NULL configuration");
    LQ_REQUIRE(ctx, std::isfinite(c->temperature) && c->temperature >= 0.0f, "sampling: temperature must be >= 0.0, got %g",
               (double)c->temperature);
    LQ_REQUIRE(ctx, c->top_p >= 0.0f && c->top_p <= 1.0f, "sampling: top_p must be in [0.0, 1.0], got %g",
               (double)c->top_p);
    LQ_REQUIRE(ctx, std::isfinite(c->repetition_penalty) && c->repetition_penalty >= 1.0f,
               "sampling: repetition_penalty must be >= 1.0, got %g", (double)c->repetition_penalty);
    LQ_REQUIRE(ctx, c->top_k >= 0, "sampling: top_k must be >= 0, got %d", (int)c->top_k);
    return LQ_OK;
}

size_t sample_scratch_bytes(int64_t rows, int64_t V) { return (size_t)(rows * V) * 4; }

int launch_sample(lq_ctx* ctx, const float* logits, int64_t rows, int64_t V, int64_t ld, const int32_t* gen,
                  int64_t gen_ld, int n_host, const int32_t* pos, const int32_t* gen_base, const lq_sampling& c,
                  float* scratch, int32_t* out, int32_t* gen_out) {
    if (rows == 0) return LQ_OK;
    SampleParams p = {};
    p.logits = logits;
    p.ld = ld;
    p.V = (int)V;
    p.gen = gen;
    p.gen_ld = gen_ld;
    p.n_host = n_host;
    p.pos = pos;
    p.gen_base = gen_base;
    p.mode = sample_mode(c);
    p.inv_t = c.temperature != 0.0f ? 1.0f / c.temperature : 0.0f;
    p.t = c.temperature;
    p.divide = std::fabs(c.temperature - 1.0f) > 1e-6f;
    p.penalty = c.repetition_penalty;
    p.use_penalty = !(std::fabs(c.repetition_penalty - 1.0f) < 1e-6f);
    p.scratch = scratch;
    p.out = out;
    p.gen_out = gen_out;
    return launch_kernel(ctx, sample_kernel, dim3((unsigned)rows), dim3(SM_THREADS), 0, "sample", p);
}

}  // namespace lq

extern "C" int lq_sample(lq_ctx* ctx, const float* logits, int64_t rows, int64_t vocab, int64_t ld,
                         const int32_t* generated, int64_t gen_ld, int64_t n_generated, const lq_sampling* cfg,
                         int32_t* out) {
    LQ_ENTRY(ctx, "lq_sample");
    int rc = lq::check_sampling(ctx, cfg);
    if (rc) return rc;
    LQ_REQUIRE(ctx, rows >= 0 && vocab > 0 && vocab < (1ll << 31) && ld >= vocab, "lq_sample: bad shape");
    LQ_REQUIRE(ctx, n_generated >= 0 && n_generated <= gen_ld && gen_ld < (1ll << 31),
               "lq_sample: n_generated %lld outside [0, gen_ld]", (long long)n_generated);
    if (rows == 0) return LQ_OK;
    LQ_REQUIRE(ctx, logits && out && (generated || n_generated == 0), "lq_sample: NULL pointer");
    float* scratch = nullptr;
    if (!(std::fabs(cfg->repetition_penalty - 1.0f) < 1e-6f) && n_generated > 0) {
        rc = lq::ensure_scratch(ctx, lq::sample_scratch_bytes(rows, vocab));
        if (rc) return rc;
        scratch = static_cast<float*>(ctx->scratch);
    }
    return lq::launch_sample(ctx, logits, rows, vocab, ld, generated, gen_ld, (int)n_generated, nullptr, nullptr, *cfg,
                             scratch, out, nullptr);
}
