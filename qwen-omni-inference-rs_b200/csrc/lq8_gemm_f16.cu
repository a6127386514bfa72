// lq8_gemm_f16.cu -- prefill Q8_0 GEMM through fp16 operands on the tcgen05 tensor cores.
//
// The exact prefill GEMM (lq8_gemm_tc.cu) issues one MMA per Q8_0 block and is bound by its
// per-block scale epilogue (three FP operations per output per block). This variant takes the
// scales out of the K loop: the weight blocks are dequantized once per call into fp16
// (w = fp16(q * d): the product q * d is exact in f32, one rounding), the activation rows into
// fp16 scaled by a power of two per row (x = fp16(q * d * 2^-e), e > 0 only when a row's
// largest value would leave the fp16 range; the epilogue multiplies by 2^e exactly), and one
// tcgen05.mma.kind::f16 chain accumulates the whole K in f32 in TMEM. Each operand carries at
// most 2^-11 relative rounding, so |y - exact| <= 2^-10 * sum_k |w_k x_k| plus the f32
// accumulation error and the fp16 subnormal range; the tests hold the kernel to that bound.
//
// Tile: 128 weight rows (MMA M) x 256 tokens (MMA N); K in stages of 64 fp16 (128-byte rows,
// 128-byte swizzle by TMA): 16 KB of weights + 32 KB of tokens per stage, 4 stages; the f32
// accumulator takes 256 TMEM columns. Warps 0-7: epilogue (warp w reads TMEM lanes 32*(w%4)..
// and token columns 128*(w/4)..); warp 8: TMA producer; warp 9: TMEM allocator and MMA issuer
// (one lane). The CTAs sharing a weight tile are adjacent in launch order (token tile
// fastest), so a weight tile is read from HBM once and from L2 by the others. Every wait is
// bounded; a timeout sets the context's error flag and the CTA goes to its teardown (TMEM is
// always released).
//
// TMA loads here read only this GPU's memory and use no multicast.
#include <cuda_fp16.h>

#include "lq8_async.cuh"
#include "lq8_internal.cuh"
#include "lq8_tma.cuh"

namespace lq {

constexpr int F16_BM = 128;                        // weight rows per CTA (MMA M)
constexpr int F16_BN = 256;                        // tokens per CTA (MMA N)
constexpr int F16_BK = 64;                         // K elements per stage: one 128-byte row
constexpr int F16_STAGES = 4;
constexpr int F16_EPI_WARPS = 8;
constexpr int F16_THREADS = (F16_EPI_WARPS + 2) * 32;
constexpr int F16_A = F16_BM * 128;                // weight tile bytes per stage
constexpr int F16_B = F16_BN * 128;                // token tile bytes per stage
constexpr int F16_STAGE = F16_A + F16_B;
constexpr int F16_SMEM = F16_STAGES * F16_STAGE + 1024 /*barriers*/ + 1024 /*alignment*/;
constexpr int F16_TMEM_COLS = F16_BN;              // f32 accumulator columns

struct F16Bars {
    uint64_t full[F16_STAGES];
    uint64_t empty[F16_STAGES];
    uint64_t mma_done;
    uint32_t tmem_base;
    int abort;
};

// K-major, 128-byte swizzled operand tile (rows of 128 B, 8-row groups 1024 B apart)
__device__ __forceinline__ uint64_t f16_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);  // start address (16-byte units)
    d |= (uint64_t)1 << 16;                   // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;         // stride byte offset: 8 rows x 128 B
    d |= (uint64_t)1 << 46;                   // descriptor version (sm100)
    d |= (uint64_t)2 << 61;                   // 128-byte swizzle
    return d;
}

// kind::f16 instruction descriptor: D f32, A and B fp16, both K-major, M x N
__host__ __device__ constexpr uint32_t f16_idesc() {
    return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(F16_BN >> 3) << 17) | ((uint32_t)(F16_BM >> 4) << 24);
}

__device__ __forceinline__ bool f16_wait(uint64_t* bar, unsigned parity) {
    return mbar_wait_ns(bar, parity, 2000000000ull);
}
__device__ __forceinline__ void f16_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void f16_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// four int8 (one u32) -> two half2, exact: each byte b becomes the fp16 1024 + (b ^ 0x80),
// from which 1152 is subtracted
__device__ __forceinline__ void i8x4_to_h2x2(uint32_t v, __half2& lo, __half2& hi) {
    const uint32_t u = v ^ 0x80808080u;
    const uint32_t a = __byte_perm(u, 0x64646464u, 0x7170 /* bytes 0,1 */);
    const uint32_t b = __byte_perm(u, 0x64646464u, 0x7372 /* bytes 2,3 */);
    const __half2 bias = __half2half2(__ushort_as_half((uint16_t)0x6480));  // 1152
    lo = __hsub2(*reinterpret_cast<const __half2*>(&a), bias);
    hi = __hsub2(*reinterpret_cast<const __half2*>(&b), bias);
}

// w16[n][k] = fp16(q * d), one thread per 32-element block
__global__ void __launch_bounds__(256) dequant_w_f16_kernel(const int8_t* __restrict__ qs,
                                                            const uint16_t* __restrict__ d, int64_t nblocks,
                                                            __half* __restrict__ out, int* err) {
    pdl_wait();  // the previous prefill GEMM may still read the buffer written here
    pdl_trigger();
    for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < nblocks;
         b += (int64_t)gridDim.x * blockDim.x) {
        const int4* src = reinterpret_cast<const int4*>(qs + b * 32);
        const int4 v0 = src[0], v1 = src[1];
        const __half dh = __ushort_as_half(d[b]);
        if (fabsf(__half2float(dh)) * 127.0f > 65504.0f) atomicCAS(err, 0, 80);  // outside fp16
        const __half2 d2 = __half2half2(dh);
        const uint32_t w[8] = {(uint32_t)v0.x, (uint32_t)v0.y, (uint32_t)v0.z, (uint32_t)v0.w,
                               (uint32_t)v1.x, (uint32_t)v1.y, (uint32_t)v1.z, (uint32_t)v1.w};
        uint4 o[4];
        uint32_t* op = reinterpret_cast<uint32_t*>(o);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            __half2 lo, hi;
            i8x4_to_h2x2(w[i], lo, hi);
            lo = __hmul2(lo, d2);  // exact fp16 integer times fp16 scale, rounded once
            hi = __hmul2(hi, d2);
            op[2 * i] = *reinterpret_cast<uint32_t*>(&lo);
            op[2 * i + 1] = *reinterpret_cast<uint32_t*>(&hi);
        }
        uint4* dst = reinterpret_cast<uint4*>(out + b * 32);
#pragma unroll
        for (int i = 0; i < 4; i++) dst[i] = o[i];
    }
}

// x16[m][k] = fp16(q * d * 2^-e[m]) with e[m] >= 0 the least exponent keeping the row's
// largest |q * d| (<= 127 * max d) inside the fp16 range; rowscale[m] = 2^e[m]. One CTA per row.
__global__ void __launch_bounds__(256) dequant_x_f16_kernel(const int8_t* __restrict__ xq,
                                                            const uint16_t* __restrict__ xd, int K,
                                                            __half* __restrict__ out, float* __restrict__ rowscale) {
    __shared__ float red[8];
    pdl_wait();
    pdl_trigger();
    const int64_t m = blockIdx.x;
    const int nb = K / 32, tid = threadIdx.x;
    float dmax = 0.0f;
    for (int b = tid; b < nb; b += blockDim.x) dmax = fmaxf(dmax, fabsf(h2f(xd[m * nb + b])));
    dmax = warp_max(dmax);
    if ((tid & 31) == 0) red[tid >> 5] = dmax;
    __syncthreads();
    dmax = red[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); i++) dmax = fmaxf(dmax, red[i]);
    int e = 0;
    while (127.0f * dmax * ldexpf(1.0f, -e) > 32768.0f) e++;
    const float inv = ldexpf(1.0f, -e);
    if (tid == 0) rowscale[m] = ldexpf(1.0f, e);
    for (int b = tid; b < nb; b += blockDim.x) {
        const int4* src = reinterpret_cast<const int4*>(xq + m * K + (int64_t)b * 32);
        const int4 v0 = src[0], v1 = src[1];
        const float dd = __fmul_rn(h2f(xd[m * nb + b]), inv);  // a power-of-two scaling: exact
        const signed char* q0 = reinterpret_cast<const signed char*>(&v0);
        const signed char* q1 = reinterpret_cast<const signed char*>(&v1);
        uint4 o[4];
        __half* oh = reinterpret_cast<__half*>(o);
#pragma unroll
        for (int i = 0; i < 16; i++) {
            oh[i] = __float2half_rn(__fmul_rn((float)q0[i], dd));  // q * d exact in f32, rounded once
            oh[16 + i] = __float2half_rn(__fmul_rn((float)q1[i], dd));
        }
        uint4* dst = reinterpret_cast<uint4*>(out + m * K + (int64_t)b * 32);
#pragma unroll
        for (int i = 0; i < 4; i++) dst[i] = o[i];
    }
}

struct F16Params {
    int N, K, M, ldy;
    const float* resid;
    const float* rowscale;
    float* y;
    int* err;
};

__global__ void __launch_bounds__(F16_THREADS, 1)
q8_gemm_f16_kernel(const __grid_constant__ CUtensorMap mw, const __grid_constant__ CUtensorMap mx, F16Params p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_addr(smem_raw);
    uint8_t* sm = smem_raw + (((raw + 1023) & ~1023u) - raw);  // 1024-aligned for the swizzle atoms
    F16Bars& B = *reinterpret_cast<F16Bars*>(sm + F16_STAGES * F16_STAGE);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * F16_BN, n0 = blockIdx.y * F16_BM;
    const int nstages = p.K / F16_BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < F16_STAGES; s++) {
            mbar_init(&B.full[s], 1);
            mbar_init(&B.empty[s], 1);
        }
        mbar_init(&B.mma_done, 1);
        mbar_fence_init();
    }
    if (warp == F16_EPI_WARPS + 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&B.tmem_base)),
                     "n"(F16_TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    f16_fence_before();
    __syncthreads();
    f16_fence_after();
    const uint32_t tmem = B.tmem_base;
    pdl_wait();  // the fp16 operands come from the dequantization kernels
    pdl_trigger();
    // a CTA that finds the error flag set (an earlier CTA timed out) does no work
    if (threadIdx.x == 0) B.abort = *reinterpret_cast<volatile int*>(p.err);
    __syncthreads();
    bool ok = B.abort == 0;

    if (warp == F16_EPI_WARPS) {
        // ------------------------------ TMA producer ------------------------------
        if (lane == 0) {
            tma_prefetch_map(&mw);
            tma_prefetch_map(&mx);
            int issued = 0;
            for (int ks = 0; ks < nstages && ok; ks++) {
                const int s = ks % F16_STAGES;
                const unsigned ph = (unsigned)(ks / F16_STAGES) & 1u;
                if (!f16_wait(&B.empty[s], ph ^ 1u)) { atomicCAS(p.err, 0, 81); ok = false; break; }
                issued = ks + 1;
                uint8_t* st = sm + s * F16_STAGE;
                mbar_expect_tx(&B.full[s], (unsigned)F16_STAGE);
                tma_load_2d(st, &mw, ks * F16_BK, n0, &B.full[s]);
                tma_load_2d(st + F16_A, &mx, ks * F16_BK, m0, &B.full[s]);
            }
            // no copy may still be landing when the CTA exits: wait (bounded) for the last ones
            for (int ks = issued > F16_STAGES ? issued - F16_STAGES : 0; ks < issued; ks++)
                f16_wait(&B.full[ks % F16_STAGES], (unsigned)(ks / F16_STAGES) & 1u);
        }
    } else if (warp == F16_EPI_WARPS + 1) {
        // ------------------------------ MMA issuer ------------------------------
        if (lane == 0) {
            constexpr uint32_t idesc = f16_idesc();
            for (int ks = 0; ks < nstages && ok; ks++) {
                const int s = ks % F16_STAGES;
                if (!f16_wait(&B.full[s], (unsigned)(ks / F16_STAGES) & 1u)) { atomicCAS(p.err, 0, 82); ok = false; break; }
                f16_fence_after();
                const uint32_t st = smem_addr(sm + s * F16_STAGE);
#pragma unroll
                for (int j = 0; j < F16_BK / 16; j++) {  // MMA K = 16 fp16 = 32 bytes of each 128-byte row
                    const uint64_t adesc = f16_desc_sw128(st + j * 32), bdesc = f16_desc_sw128(st + F16_A + j * 32);
                    const uint32_t acc = (ks > 0 || j > 0) ? 1u : 0u;
                    asm volatile(
                        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}\n" ::"r"(tmem),
                        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(0));
                }
                // the stage's operands may be overwritten once these MMAs have completed
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 smem_addr(&B.empty[s]))
                             : "memory");
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_addr(&B.mma_done))
                         : "memory");
            if (!f16_wait(&B.mma_done, 0)) atomicCAS(p.err, 0, 83);
        }
    } else {
        // ------------------------------ epilogue ------------------------------
        const int q = warp & 3;   // TMEM lane quarter: weight rows 32q .. 32q+31
        const int h = warp >> 2;  // token columns 128h .. 128h+127
        const int n = n0 + q * 32 + lane;
        if (ok) {
            // one lane per warp polls the accumulator's completion (the GEMM's whole duration)
            bool done = true;
            if (lane == 0) done = f16_wait(&B.mma_done, 0);
            if (!__shfl_sync(0xffffffffu, done, 0)) {
                if (lane == 0) atomicCAS(p.err, 0, 84);
                ok = false;
            }
        }
        if (ok) {
            f16_fence_after();
#pragma unroll 1
            for (int c0 = 0; c0 < 128; c0 += 16) {
                uint32_t r[16];
                const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * 128 + c0);
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
                    "[%16];"
                    : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                      "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                      "=r"(r[15])
                    : "r"(taddr));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (n < p.N) {
#pragma unroll
                    for (int i = 0; i < 16; i++) {
                        const int m = m0 + h * 128 + c0 + i;
                        if (m < p.M) {
                            const size_t o = (size_t)m * p.ldy + n;
                            const float v = __fmul_rn(__uint_as_float(r[i]), p.rowscale[m]);
                            p.y[o] = p.resid ? __fadd_rn(p.resid[o], v) : v;
                        }
                    }
                }
            }
        }
    }
    f16_fence_before();
    __syncthreads();
    f16_fence_after();
    if (warp == F16_EPI_WARPS + 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(F16_TMEM_COLS));
}

static bool gemm_f16_qualifies(const lq_q8_tensor* w, int64_t m) {
    return m >= 128 && w->k % F16_BK == 0 && w->k >= F16_BK && w->n >= 1 && w->n < (1ll << 31) &&
           (uintptr_t)w->qs % 16 == 0 && getenv("LQ_PREFILL_EXACT") == nullptr;
}

int launch_gemm_f16(lq_ctx* ctx, const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd, int64_t m, float* y,
                    const float* resid, int64_t ldy) {
    if (!gemm_f16_qualifies(w, m) || (uintptr_t)xq % 16) return LQ_ERR_UNSUPPORTED;
    const int64_t N = w->n, K = w->k;
    auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
    const size_t wb = al((size_t)N * K * 2), xb = al((size_t)m * K * 2), sb = al((size_t)m * 4);
    int rc = ensure_wide(ctx, wb + xb + sb);
    if (rc) return rc;
    __half* w16 = reinterpret_cast<__half*>(ctx->wide);
    __half* x16 = reinterpret_cast<__half*>((uint8_t*)ctx->wide + wb);
    float* rowscale = reinterpret_cast<float*>((uint8_t*)ctx->wide + wb + xb);
    const int64_t nblocks = N * (K / 32);
    const int dq_grid = (int)std::min<int64_t>(ceil_div(nblocks, 256), 16ll * ctx->sm_count);
    rc = launch_kernel(ctx, dequant_w_f16_kernel, dim3((unsigned)dq_grid), dim3(256), 0, "dequant_w_f16", w->qs, w->d,
                       nblocks, w16, ctx->err_flag);
    if (rc) return rc;
    rc = launch_kernel(ctx, dequant_x_f16_kernel, dim3((unsigned)m), dim3(256), 0, "dequant_x_f16", xq, xd, (int)K, x16,
                       rowscale);
    if (rc) return rc;
    CUtensorMap mw, mx;
    if ((rc = make_tensor_map_2d(ctx, &mw, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, w16, (uint64_t)K, (uint64_t)N,
                                 (uint64_t)K * 2, F16_BK, F16_BM, CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    if ((rc = make_tensor_map_2d(ctx, &mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x16, (uint64_t)K, (uint64_t)m,
                                 (uint64_t)K * 2, F16_BK, F16_BN, CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    if ((rc = ensure_func_smem(ctx, (const void*)q8_gemm_f16_kernel, F16_SMEM))) return rc;
    F16Params p;
    p.N = (int)N;
    p.K = (int)K;
    p.M = (int)m;
    p.ldy = (int)ldy;
    p.resid = resid;
    p.rowscale = rowscale;
    p.y = y;
    p.err = ctx->err_flag;
    const dim3 grid((unsigned)ceil_div(m, F16_BN), (unsigned)ceil_div(N, F16_BM));
    return launch_kernel(ctx, q8_gemm_f16_kernel, grid, dim3(F16_THREADS), (size_t)F16_SMEM, "q8_gemm_f16", mw, mx, p);
}

int launch_q8_matmul_prefill(lq_ctx* ctx, const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd, int64_t m,
                             float* y, const float* resid, int64_t ldy) {
    const int rc = launch_gemm_f16(ctx, w, xq, xd, m, y, resid, ldy);
    if (rc != LQ_ERR_UNSUPPORTED) return rc;
    return launch_q8_matmul(ctx, w, xq, xd, m, y, resid, ldy, nullptr);
}

}  // namespace lq

extern "C" int lq_q8_0_matmul_prefill(lq_ctx* ctx, const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd,
                                      int64_t m, float* y, const float* resid, int64_t ldy) {
    LQ_ENTRY(ctx, "lq_q8_0_matmul_prefill");
    LQ_REQUIRE(ctx, w && w->qs && w->d && w->n > 0 && w->k > 0 && w->k % 32 == 0,
               "lq_q8_0_matmul_prefill: bad Q8_0 tensor");
    LQ_REQUIRE(ctx, m >= 0 && m < (1 << 24), "lq_q8_0_matmul_prefill: m=%lld out of range", (long long)m);
    if (ldy == 0) ldy = w->n;
    LQ_REQUIRE(ctx, ldy >= w->n, "lq_q8_0_matmul_prefill: ldy < n");
    if (m == 0) return LQ_OK;
    LQ_REQUIRE(ctx, xq && xd && y, "lq_q8_0_matmul_prefill: NULL pointer");
    return lq::launch_q8_matmul_prefill(ctx, w, xq, xd, m, y, resid, ldy);
}
