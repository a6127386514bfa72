// lq8_ops.cu -- the small Qwen3 ops that keep activations in HBM, fused with the Q8_0
// quantization of their output where the next op is a Q8_0 linear. The row math lives in
// lq8_fused.cuh and is shared with the fused prologues of the decode kernels.
#include "lq8_async.cuh"
#include "lq8_fused.cuh"
#include "lq8_internal.cuh"

#include <cmath>
#include <vector>

namespace lq {

__device__ __forceinline__ void set_err(int* flag, int code, int value) {
    if (flag && atomicCAS(flag, 0, code) == 0) flag[1] = value;
}

constexpr int NORM_THREADS = 256;

// =========================================================================================
// RMSNorm (rms_norm.rs:144-176) + optional Q8_0 quantization of the bf16 output; one CTA
// of 256 threads per row (the same row function as the fused GEMV prologue).
// =========================================================================================
template <typename T>
__global__ void __launch_bounds__(NORM_THREADS)
rmsnorm_kernel(const T* __restrict__ x, int dim, const uint16_t* __restrict__ w, float eps,
               uint16_t* __restrict__ out, int8_t* __restrict__ xq, uint16_t* __restrict__ xd) {
    __shared__ float red[32];
    pdl_trigger();  // early: the next kernel (a weight stream) may start; it waits for us in pdl_wait
    // the norm weights do not depend on the preceding kernel: bring them into L2 while it ends
    for (int b = threadIdx.x * 64; b < dim; b += NORM_THREADS * 64)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(w + b));
    pdl_wait();
    const int64_t row = blockIdx.x;
    rms_row<T, NORM_THREADS, 0, 8>(x + row * dim, dim, w, eps, threadIdx.x, red, out ? out + row * dim : nullptr,
                                xq ? xq + row * dim : nullptr, xq ? xd + row * (dim >> 5) : nullptr);
}

int launch_rmsnorm(lq_ctx* ctx, const void* x, lq_dtype dt, int64_t rows, int64_t dim,
                   const uint16_t* w, float eps, uint16_t* out, int8_t* xq, uint16_t* xd) {
    if (rows == 0) return LQ_OK;
    const dim3 grid((unsigned)rows);
    if (dt == LQ_DTYPE_F32)
        return launch_kernel(ctx, rmsnorm_kernel<float>, grid, dim3(NORM_THREADS), 0, "rmsnorm", (const float*)x,
                             (int)dim, w, eps, out, xq, xd);
    return launch_kernel(ctx, rmsnorm_kernel<uint16_t>, grid, dim3(NORM_THREADS), 0, "rmsnorm",
                         (const uint16_t*)x, (int)dim, w, eps, out, xq, xd);
}

// =========================================================================================
// per-head q/k RMSNorm + RoPE + KV-cache append (attention.rs:337-364, rope.rs:245-303).
// One warp per (token row, head). Heads [0,Hq) are q, [Hq,Hq+Hkv) k, [Hq+Hkv, Hq+2Hkv) v.
// =========================================================================================
__global__ void __launch_bounds__(256)
qk_norm_rope_kv_kernel(const float* __restrict__ qkv, int B, int L, int Hq, int Hkv,
                       const uint16_t* __restrict__ qn, const uint16_t* __restrict__ kn, float eps,
                       const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                       int pos0, const int32_t* __restrict__ pos0_dev, float* __restrict__ q_out,
                       float* __restrict__ kc, float* __restrict__ vc, int ctx_max, int* err) {
    constexpr int D = 128, RD = 64;
    pdl_trigger();  // early: the next kernel (a weight stream) may start; it waits for us in pdl_wait
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int heads = Hq + 2 * Hkv;
    if (item >= (int64_t)B * L * heads) return;
    const int h = (int)(item % heads);
    const int64_t row = item / heads;  // b*L + l
    const int b = (int)(row / L), l = (int)(row % L);
    const int p0 = pos0_dev ? *pos0_dev : pos0;
    const int pos = p0 + l;
    if (pos < 0 || pos >= ctx_max) {
        if (lane == 0) set_err(err, 1, pos);
        return;
    }
    const float* src = qkv + row * (int64_t)heads * D + (int64_t)h * D;
    if (h >= Hq + Hkv) {  // v: KvCache::append of the projection output (f32)
        const int kvh = h - Hq - Hkv;
        float* dst = vc + (((int64_t)b * Hkv + kvh) * ctx_max + pos) * D;
        const int d0 = 2 * lane;
        *reinterpret_cast<float2*>(dst + d0) = *reinterpret_cast<const float2*>(src + d0);
        *reinterpret_cast<float2*>(dst + RD + d0) = *reinterpret_cast<const float2*>(src + RD + d0);
        return;
    }
    float* dst = h < Hq ? q_out + (((int64_t)b * Hq + h) * L + l) * D
                        : kc + (((int64_t)b * Hkv + (h - Hq)) * ctx_max + pos) * D;
    head_norm_rope(src, h < Hq ? qn : kn, eps, cos_t + (int64_t)pos * RD, sin_t + (int64_t)pos * RD, lane, dst);
}

int launch_qk_norm_rope_kv(lq_ctx* ctx, const float* qkv, int64_t B, int64_t L, int64_t Hq,
                           int64_t Hkv, int64_t D, const uint16_t* qn, const uint16_t* kn,
                           float eps, const float* cos_t, const float* sin_t, int64_t pos0,
                           const int32_t* pos0_dev, float* q_out, float* kc, float* vc,
                           int64_t ctx_max) {
    (void)D;
    const int64_t items = B * L * (Hq + 2 * Hkv);
    if (items == 0) return LQ_OK;
    return launch_kernel(ctx, qk_norm_rope_kv_kernel, dim3(ceil_div(items, 8)), dim3(256), 0, "qk_norm_rope_kv",
                         qkv, (int)B, (int)L, (int)Hq, (int)Hkv, qn, kn, eps, cos_t, sin_t, (int)pos0, pos0_dev,
                         q_out, kc, vc, (int)ctx_max, ctx->err_flag);
}

// =========================================================================================
// SiLU(gate) * up + Q8_0, one CTA of 256 threads per row (the same row function as the fused
// down-projection prologue)
// =========================================================================================
__global__ void __launch_bounds__(256)
silu_mul_kernel(const float* __restrict__ gu, int inter, float* __restrict__ h, int8_t* __restrict__ xq,
                uint16_t* __restrict__ xd) {
    pdl_trigger();  // early: the next kernel (a weight stream) may start; it waits for us in pdl_wait
    pdl_wait();
    // CTA (row, 1024-column chunk): one pass of the row function over its chunk (each 8-lane
    // group quantizes one 32-element block, so the chunking does not change a value)
    const int64_t row = blockIdx.x;
    const int c0 = blockIdx.y * 1024, n = min(1024, inter - c0);
    const float* g = gu + row * 2 * inter + c0;
    const int e = threadIdx.x * 4;
    const bool valid = e < n;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (valid) {
        const float4 gg = *reinterpret_cast<const float4*>(g + e);
        const float4 uu = *reinterpret_cast<const float4*>(g + inter + e);
        v[0] = swiglu(gg.x, uu.x);
        v[1] = swiglu(gg.y, uu.y);
        v[2] = swiglu(gg.z, uu.z);
        v[3] = swiglu(gg.w, uu.w);
        if (h) *reinterpret_cast<float4*>(h + row * inter + c0 + e) = make_float4(v[0], v[1], v[2], v[3]);
    }
    if (xq) {
        const int64_t o = row * inter + c0 + e;
        const uint32_t q = quant_group8(v, threadIdx.x & 7, valid ? xd + (o >> 5) : nullptr);
        if (valid) *reinterpret_cast<uint32_t*>(xq + o) = q;
    }
}

int launch_silu_mul(lq_ctx* ctx, const float* gu, int64_t m, int64_t inter, float* h, int8_t* xq,
                    uint16_t* xd) {
    if (m == 0) return LQ_OK;
    return launch_kernel(ctx, silu_mul_kernel, dim3((unsigned)m, (unsigned)ceil_div(inter, 1024)), dim3(256), 0,
                         "silu_mul", gu, (int)inter, h, xq, xd);
}

// =========================================================================================
// embedding gather (embedding.rs:105-153), bf16 rows widened exactly to f32
// =========================================================================================
__global__ void embedding_kernel(const uint16_t* __restrict__ table, int64_t vocab, int hidden,
                                 const int32_t* __restrict__ ids, int64_t n, float* __restrict__ out,
                                 int* err) {
    pdl_wait();
    pdl_trigger();
    const int64_t row = blockIdx.x;
    if (row >= n) return;
    const int32_t id = ids[row];
    const bool ok = id >= 0 && id < vocab;
    if (!ok && threadIdx.x == 0) set_err(err, 2, id);
    for (int c = threadIdx.x * 4; c < hidden; c += blockDim.x * 4) {
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        if (ok) {
            const uint2 t = *reinterpret_cast<const uint2*>(table + (int64_t)id * hidden + c);
            o = make_float4(bf16_to_f32((uint16_t)(t.x & 0xFFFF)), bf16_to_f32((uint16_t)(t.x >> 16)),
                            bf16_to_f32((uint16_t)(t.y & 0xFFFF)), bf16_to_f32((uint16_t)(t.y >> 16)));
        }
        *reinterpret_cast<float4*>(out + row * hidden + c) = o;
    }
}

int launch_embedding(lq_ctx* ctx, const uint16_t* table, int64_t vocab, int64_t hidden,
                     const int32_t* ids, int64_t n, float* out) {
    if (n == 0) return LQ_OK;
    return launch_kernel(ctx, embedding_kernel, dim3((unsigned)n), dim3(256), 0, "embedding", table, vocab,
                         (int)hidden, ids, n, out, ctx->err_flag);
}

// =========================================================================================
// argmax (tensor.rs:2451-2482): max value, ties -> highest index
// =========================================================================================
__global__ void __launch_bounds__(1024)
argmax_kernel(const float* __restrict__ x, int64_t n, int32_t* __restrict__ out) {
    __shared__ unsigned long long red[32];
    pdl_wait();
    pdl_trigger();
    const float* xr = x + (int64_t)blockIdx.x * n;
    unsigned long long best = 0ull;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const unsigned long long k = argmax_key(xr[i], (int)i);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
        best = v > best ? v : best;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x < 32) {
        best = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0ull;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
            best = v > best ? v : best;
        }
        if (threadIdx.x == 0) out[blockIdx.x] = (int32_t)(uint32_t)(best & 0xFFFFFFFFull);
    }
}

// next token ids from the LM head's fused argmax keys (out may be NULL when a sampler chose
// them); clears the keys for the next step, appends each row's token to its generated-token
// history gen[row][n] (n = n_host, or *pos_counter - *gen_base + 1 when n_host < 0) and then
// advances the device position of the decode graph. One block, so the position is read by
// every thread before it is advanced.
__global__ void argmax_finalize_kernel(unsigned long long* keys, int64_t rows, int32_t* out, int32_t* pos_counter,
                                       int32_t* gen, int64_t gen_ld, int n_host, const int32_t* gen_base) {
    pdl_wait();
    pdl_trigger();
    int n = n_host;
    if (gen && n < 0) n = *pos_counter - *gen_base + 1;
    for (int64_t i = threadIdx.x; i < rows; i += blockDim.x) {
        const int32_t t = (int32_t)(uint32_t)(keys[i] & 0xFFFFFFFFull);
        if (out) out[i] = t;
        if (gen && n >= 0 && n < gen_ld) gen[i * gen_ld + n] = t;
        keys[i] = 0ull;
    }
    __syncthreads();
    if (threadIdx.x == 0 && pos_counter) *pos_counter += 1;
}

int launch_argmax_finalize(lq_ctx* ctx, unsigned long long* keys, int64_t rows, int32_t* out,
                           int32_t* pos_counter, int32_t* gen, int64_t gen_ld, int n_host, const int32_t* gen_base) {
    const int threads = (int)std::min<int64_t>(1024, std::max<int64_t>(32, (rows + 31) / 32 * 32));
    return launch_kernel(ctx, argmax_finalize_kernel, dim3(1), dim3(threads), 0, "argmax_finalize", keys, rows, out,
                         pos_counter, gen, gen_ld, n_host, gen_base);
}

__global__ void add_kernel(const float* a, const float* b, int64_t n, float* out) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = __fadd_rn(a[i], b[i]);
}

__global__ void keys_offset_kernel(unsigned long long* keys, int64_t n, long long offset) {
    pdl_wait();  // the keys are the preceding LM-head kernel's
    pdl_trigger();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n && keys[i]) keys[i] += (unsigned long long)offset;
}

int launch_keys_offset(lq_ctx* ctx, unsigned long long* keys, int64_t n, int64_t offset) {
    if (n <= 0 || offset == 0) return LQ_OK;
    return launch_kernel(ctx, keys_offset_kernel, dim3((unsigned)ceil_div(n, 128)), dim3(128), 0, "keys_offset", keys, n,
                         (long long)offset);
}

}  // namespace lq

// =========================================================================================
// C ABI
// =========================================================================================
extern "C" {

int lq_rmsnorm(lq_ctx* ctx, const void* x, lq_dtype dt, int64_t rows, int64_t dim,
               const uint16_t* w, float eps, uint16_t* out, int8_t* xq, uint16_t* xd) {
    LQ_ENTRY(ctx, "lq_rmsnorm");
    LQ_REQUIRE(ctx, dt == LQ_DTYPE_F32 || dt == LQ_DTYPE_BF16, "lq_rmsnorm: dtype must be F32 or BF16");
    LQ_REQUIRE(ctx, rows >= 0 && dim > 0 && dim % 4 == 0, "lq_rmsnorm: dim=%lld must be a positive multiple of 4",
               (long long)dim);
    LQ_REQUIRE(ctx, !xq || dim % 32 == 0, "lq_rmsnorm: Q8_0 output needs dim %% 32 == 0");
    LQ_REQUIRE(ctx, (xq == nullptr) == (xd == nullptr), "lq_rmsnorm: xq and xd go together");
    LQ_REQUIRE(ctx, rows < (1ll << 31), "lq_rmsnorm: too many rows");
    if (rows == 0) return LQ_OK;
    LQ_REQUIRE(ctx, x && w && (out || xq), "lq_rmsnorm: NULL pointer");
    return lq::launch_rmsnorm(ctx, x, dt, rows, dim, w, eps, out, xq, xd);
}

int lq_rope_tables(lq_ctx* ctx, int64_t head_dim, int64_t max_pos, double theta, float* cos_dev,
                   float* sin_dev) {
    LQ_ENTRY(ctx, "lq_rope_tables");
    LQ_REQUIRE(ctx, head_dim > 0 && head_dim % 4 == 0 && max_pos > 0,
               "lq_rope_tables: head_dim must be a multiple of 4 (rope.rs:77-83 requires even)");
    LQ_REQUIRE(ctx, cos_dev && sin_dev, "lq_rope_tables: NULL pointer");
    // rope.rs:89-117, evaluated in double on the host exactly like the reference
    const int64_t rd = head_dim / 2, half = rd / 2;
    std::vector<double> inv(half);
    for (int64_t i = 0; i < half; i++) inv[i] = 1.0 / std::pow(theta, (double)(2 * i) / (double)rd);
    std::vector<float> c((size_t)(max_pos * rd)), s((size_t)(max_pos * rd));
    for (int64_t p = 0; p < max_pos; p++)
        for (int64_t i = 0; i < half; i++) {
            const double fr = (double)p * inv[i];
            const float cv = (float)std::cos(fr), sv = (float)std::sin(fr);
            c[p * rd + 2 * i] = cv; c[p * rd + 2 * i + 1] = cv;
            s[p * rd + 2 * i] = sv; s[p * rd + 2 * i + 1] = sv;
        }
    LQ_CUDA(ctx, cudaMemcpyAsync(cos_dev, c.data(), c.size() * 4, cudaMemcpyHostToDevice, ctx->stream));
    LQ_CUDA(ctx, cudaMemcpyAsync(sin_dev, s.data(), s.size() * 4, cudaMemcpyHostToDevice, ctx->stream));
    LQ_CUDA(ctx, cudaStreamSynchronize(ctx->stream));  // host vectors go out of scope
    return LQ_OK;
}

int lq_qk_norm_rope_kv(lq_ctx* ctx, const float* qkv, int64_t B, int64_t L, int64_t Hq, int64_t Hkv,
                       int64_t D, const uint16_t* qn, const uint16_t* kn, float eps, const float* cos_t,
                       const float* sin_t, int64_t pos0, const int32_t* pos0_dev, float* q_out, float* kc,
                       float* vc, int64_t ctx_max) {
    LQ_ENTRY(ctx, "lq_qk_norm_rope_kv");
    LQ_REQUIRE(ctx, D == 128, "lq_qk_norm_rope_kv: head_dim %lld unsupported (Qwen3 uses 128)", (long long)D);
    LQ_REQUIRE(ctx, B >= 0 && L >= 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0, "lq_qk_norm_rope_kv: bad head counts");
    LQ_REQUIRE(ctx, pos0_dev || (pos0 >= 0 && pos0 + L <= ctx_max),
               "lq_qk_norm_rope_kv: positions [%lld, %lld) exceed ctx_max %lld", (long long)pos0,
               (long long)(pos0 + L), (long long)ctx_max);
    if (B == 0 || L == 0) return LQ_OK;
    LQ_REQUIRE(ctx, qkv && qn && kn && cos_t && sin_t && q_out && kc && vc, "lq_qk_norm_rope_kv: NULL pointer");
    return lq::launch_qk_norm_rope_kv(ctx, qkv, B, L, Hq, Hkv, D, qn, kn, eps, cos_t, sin_t, pos0, pos0_dev, q_out,
                                      kc, vc, ctx_max);
}

int lq_silu_mul(lq_ctx* ctx, const float* gu, int64_t m, int64_t inter, float* h, int8_t* xq, uint16_t* xd) {
    LQ_ENTRY(ctx, "lq_silu_mul");
    LQ_REQUIRE(ctx, m >= 0 && inter > 0 && inter % 32 == 0, "lq_silu_mul: inter must be a multiple of 32");
    LQ_REQUIRE(ctx, m < (1ll << 31), "lq_silu_mul: too many rows");
    LQ_REQUIRE(ctx, (xq == nullptr) == (xd == nullptr), "lq_silu_mul: xq and xd go together");
    if (m == 0) return LQ_OK;
    LQ_REQUIRE(ctx, gu && (h || xq), "lq_silu_mul: NULL pointer");
    return lq::launch_silu_mul(ctx, gu, m, inter, h, xq, xd);
}

int lq_add(lq_ctx* ctx, const float* a, const float* b, int64_t n, float* out) {
    LQ_ENTRY(ctx, "lq_add");
    LQ_REQUIRE(ctx, n >= 0, "lq_add: negative size");
    if (n == 0) return LQ_OK;
    LQ_REQUIRE(ctx, a && b && out, "lq_add: NULL pointer");
    const int grid = (int)std::min<int64_t>((n + 255) / 256, (int64_t)ctx->sm_count * 16);
    return lq::launch_kernel(ctx, lq::add_kernel, dim3(grid), dim3(256), 0, "add", a, b, n, out);
}

int lq_embedding(lq_ctx* ctx, const uint16_t* table, int64_t vocab, int64_t hidden, const int32_t* ids, int64_t n,
                 float* out) {
    LQ_ENTRY(ctx, "lq_embedding");
    LQ_REQUIRE(ctx, vocab > 0 && hidden > 0 && hidden % 4 == 0 && n >= 0, "lq_embedding: bad shape");
    if (n == 0) return LQ_OK;
    LQ_REQUIRE(ctx, table && ids && out, "lq_embedding: NULL pointer");
    int rc = lq::launch_embedding(ctx, table, vocab, hidden, ids, n, out);
    if (rc) return rc;
    return lq::consume_device_error(ctx, "lq_embedding (token id out of range)");
}

int lq_argmax(lq_ctx* ctx, const float* x, int64_t rows, int64_t n, int32_t* out) {
    LQ_ENTRY(ctx, "lq_argmax");
    LQ_REQUIRE(ctx, rows >= 0 && n > 0 && n < (1ll << 31), "lq_argmax: bad shape");
    if (rows == 0) return LQ_OK;
    LQ_REQUIRE(ctx, x && out, "lq_argmax: NULL pointer");
    return lq::launch_kernel(ctx, lq::argmax_kernel, dim3((unsigned)rows), dim3(1024), 0, "argmax", x, n, out);
}

}  // extern "C"
