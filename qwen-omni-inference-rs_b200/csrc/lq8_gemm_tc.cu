// lq8_gemm_tc.cu -- prefill Q8_0 x Q8_0 GEMM on the 5th-generation tensor cores (tcgen05).
//
// y[m][n] = sum_b sumi_b(m, n) * (d_w[n][b] * d_x[m][b]) for M >= 64 tokens.
//
// One MMA per Q8_0 block: tcgen05.mma.kind::i8 with K = 32 computes the exact int32 block
// dot products of a 128-row weight tile (MMA M) by a 64-token tile (MMA N) into a fresh TMEM
// accumulator. The per-block scales differ per (row, block) and per (token, block), so the
// block results cannot be summed inside TMEM; 16 epilogue warps read every block's int32 tile
// from TMEM (tcgen05.ld) and add (float)sumi * (d_w * d_x) to f32 registers in ascending
// block order -- the oracle's order, so results are bit-identical to it. The epilogue is the
// bound (3 FP operations per output per block against one MMA per block): it converts the
// int32 sums exactly without the conversion unit and multiplies f32 pairs (f32x2, each lane
// rounded like the scalar operation); the accumulating adds are scalar.
//
// Roles (18 warps): warps 0-15 epilogue (warp w reads TMEM lanes 32*(w%4).. and token columns
// 16*(w/4)..), warp 16 TMA producer, warp 17 TMEM allocator + MMA issuer (one elected lane).
// Shared-memory stages of 256 bytes of K (8 blocks): weights 2 x [128 x 128 B] and tokens
// 2 x [64 x 128 B], 128-byte swizzled by TMA, plus the stage's fp16 scales. A stage is freed
// when its MMAs have completed (tcgen05.commit) and the epilogue has used its scales. TMEM
// holds 8 block accumulators of 64 columns (the whole 512 columns), so the MMA runs up to 8
// blocks ahead of the epilogue. Every wait is bounded; a timeout sets the context's error
// flag and the CTA skips to its teardown (TMEM is always released).
//
// TMA loads here read only this GPU's memory and use no multicast.
#include "lq8_async.cuh"
#include "lq8_internal.cuh"
#include "lq8_tma.cuh"

namespace lq {

constexpr int TC_BM = 128;            // weight rows per CTA (MMA M)
constexpr int TC_BN = 64;             // tokens per CTA (MMA N)
constexpr int TC_KS = 256;            // K bytes per stage (8 Q8_0 blocks)
constexpr int TC_STAGES = 4;
constexpr int TC_BUFS = 8;            // TMEM block accumulators (64 columns each)
constexpr int TC_EPI_WARPS = 16;
constexpr int TC_EW = TC_BN / (TC_EPI_WARPS / 4);  // tokens per epilogue warp
constexpr int TC_THREADS = (TC_EPI_WARPS + 2) * 32;
constexpr int TC_A_SUB = TC_BM * 128;  // bytes of one 128-byte-wide weight sub-tile
constexpr int TC_B_SUB = TC_BN * 128;
constexpr int TC_STAGE = 2 * TC_A_SUB + 2 * TC_B_SUB + TC_BM * 16 + TC_BN * 16;  // 52224
constexpr int TC_SMEM = TC_STAGES * TC_STAGE + 1024 /*barriers*/ + TC_EPI_WARPS * 8 * TC_EW * 4 /*f32 token scales*/ +
                        1024 /*alignment*/;

struct TcBars {
    uint64_t full[TC_STAGES];
    uint64_t empty[TC_STAGES];
    uint64_t tfull[TC_BUFS];
    uint64_t tempty[TC_BUFS];
    uint64_t mma_done;
    uint32_t tmem_base;
    int abort;
};


// K-major, 128-byte swizzled operand tile: rows of 128 B, 8-row groups 1024 B apart
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);          // start address (16-byte units)
    d |= (uint64_t)1 << 16;                           // leading byte offset (unused: 1)
    d |= (uint64_t)(1024 >> 4) << 32;                 // stride byte offset: 8 rows x 128 B
    d |= (uint64_t)1 << 46;                           // descriptor version (sm100)
    d |= (uint64_t)2 << 61;                           // layout: 128-byte swizzle
    return d;
}

// kind::i8 instruction descriptor: D s32, A and B signed 8-bit, both K-major, M x N
__host__ __device__ constexpr uint32_t tc_idesc() {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TC_BN >> 3) << 17) | ((uint32_t)(TC_BM >> 4) << 24);
}

// every wait in this kernel is legitimately microseconds long; 2 s means a lost copy or MMA
__device__ __forceinline__ bool tc_wait(uint64_t* bar, unsigned parity) {
    return mbar_wait_ns(bar, parity, 2000000000ull);
}

// f32 pair multiply, each lane rounded to nearest like __fmul_rn. The accumulation stays
// scalar (__fadd_rn): an f32x2 multiply feeding an f32x2 add is contracted into an f32x2 FMA
// by the code generator even with explicit .rn and -fmad=false, which would change the
// rounding of acc + sumi * scale; a packed multiply feeding scalar adds measured bit-exact.
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
    float2 d;
    asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
        " mul.rn.f32x2 rd, ra, rb;\n mov.b64 {%0, %1}, rd;\n}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
    float2 d;
    asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
        " add.rn.f32x2 rd, ra, rb;\n mov.b64 {%0, %1}, rd;\n}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

struct TcParams {
    int N, K, M, ldy;
    const float* resid;
    float* y;
    int* err;
};

__global__ void __launch_bounds__(TC_THREADS, 1)
q8_gemm_tc_kernel(const __grid_constant__ CUtensorMap mw, const __grid_constant__ CUtensorMap mx,
                  const __grid_constant__ CUtensorMap mdw, const __grid_constant__ CUtensorMap mdx, TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_addr(smem_raw);
    uint8_t* sm = smem_raw + (((raw + 1023) & ~1023u) - raw);  // 1024-aligned for the swizzle atoms
    TcBars& B = *reinterpret_cast<TcBars*>(sm + TC_STAGES * TC_STAGE);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * TC_BM, m0 = blockIdx.y * TC_BN;
    const int nstages = p.K / TC_KS;
    constexpr uint32_t kStageTx = TC_STAGE;

    if (threadIdx.x == 0) {
        for (int s = 0; s < TC_STAGES; s++) {
            mbar_init(&B.full[s], 1);
            mbar_init(&B.empty[s], 1 + TC_EPI_WARPS);
        }
        for (int b = 0; b < TC_BUFS; b++) {
            mbar_init(&B.tfull[b], 1);
            mbar_init(&B.tempty[b], TC_EPI_WARPS);
        }
        mbar_init(&B.mma_done, 1);
        mbar_fence_init();
    }
    if (warp == TC_EPI_WARPS + 1) {  // allocate all 512 TMEM columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_addr(&B.tmem_base)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = B.tmem_base;
    pdl_wait();
    pdl_trigger();
    // a CTA that finds the error flag set (an earlier CTA timed out) does no work, so a
    // failing launch ends after one wave of timeouts instead of one per wave
    if (threadIdx.x == 0) B.abort = *reinterpret_cast<volatile int*>(p.err);
    __syncthreads();
    bool ok = B.abort == 0;

    if (warp == TC_EPI_WARPS) {
        // ------------------------------ TMA producer ------------------------------
        if (lane == 0) {
            int issued = 0;
            for (int ks = 0; ks < nstages && ok; ks++) {
                const int s = ks % TC_STAGES;
                const unsigned ph = (unsigned)(ks / TC_STAGES) & 1u;
                if (!tc_wait(&B.empty[s], ph ^ 1u)) { atomicCAS(p.err, 0, 11); ok = false; break; }
                issued = ks + 1;
                uint8_t* st = sm + s * TC_STAGE;
                mbar_expect_tx(&B.full[s], kStageTx);
                const int kb = ks * TC_KS;
                tma_load_2d(st, &mw, kb, n0, &B.full[s]);
                tma_load_2d(st + TC_A_SUB, &mw, kb + 128, n0, &B.full[s]);
                tma_load_2d(st + 2 * TC_A_SUB, &mx, kb, m0, &B.full[s]);
                tma_load_2d(st + 2 * TC_A_SUB + TC_B_SUB, &mx, kb + 128, m0, &B.full[s]);
                tma_load_2d(st + 2 * TC_A_SUB + 2 * TC_B_SUB, &mdw, ks * 8, n0, &B.full[s]);
                tma_load_2d(st + 2 * TC_A_SUB + 2 * TC_B_SUB + TC_BM * 16, &mdx, ks * 8, m0, &B.full[s]);
            }
            // no copy may still be landing in shared memory when the CTA exits: wait (bounded)
            // for the last stages issued; each slot has completed at most one phase past them
            for (int ks = issued > TC_STAGES ? issued - TC_STAGES : 0; ks < issued; ks++)
                tc_wait(&B.full[ks % TC_STAGES], (unsigned)(ks / TC_STAGES) & 1u);
        }
    } else if (warp == TC_EPI_WARPS + 1) {
        // ------------------------------ MMA issuer ------------------------------
        if (lane == 0) {
            constexpr uint32_t idesc = tc_idesc();
            for (int ks = 0; ks < nstages && ok; ks++) {
                const int s = ks % TC_STAGES;
                if (!tc_wait(&B.full[s], (unsigned)(ks / TC_STAGES) & 1u)) { atomicCAS(p.err, 0, 12); ok = false; break; }
                tc_fence_after();
                const uint32_t st = smem_addr(sm + s * TC_STAGE);
                for (int j = 0; j < 8 && ok; j++) {
                    const int g = ks * 8 + j;  // global block index
                    const int buf = g % TC_BUFS;
                    if (!tc_wait(&B.tempty[buf], ((unsigned)(g / TC_BUFS) & 1u) ^ 1u)) {
                        atomicCAS(p.err, 0, 13);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = st + (j >> 2) * TC_A_SUB + (j & 3) * 32;
                    const uint32_t b_addr = st + 2 * TC_A_SUB + (j >> 2) * TC_B_SUB + (j & 3) * 32;
                    const uint64_t adesc = umma_desc_sw128(a_addr), bdesc = umma_desc_sw128(b_addr);
                    const uint32_t dtm = tmem + (uint32_t)(buf * TC_BN);
                    asm volatile(
                        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}\n" ::"r"(dtm),
                        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(0), "r"(0));
                    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                     smem_addr(&B.tfull[buf]))
                                 : "memory");
                }
                // the stage's operands may be overwritten once these MMAs have completed
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 smem_addr(&B.empty[s]))
                             : "memory");
            }
            // every MMA issued has completed before TMEM is released
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_addr(&B.mma_done))
                         : "memory");
            if (!tc_wait(&B.mma_done, 0)) atomicCAS(p.err, 0, 16);
        }
    } else {
        // ------------------------------ epilogue ------------------------------
        const int q = warp & 3;   // TMEM lane quarter: weight rows 32q .. 32q+31
        const int h = warp >> 2;  // token slice: columns TC_EW*h .. +TC_EW-1
        const int row = q * 32 + lane;
        float* dxf = reinterpret_cast<float*>(sm + TC_STAGES * TC_STAGE + 1024) + warp * (8 * TC_EW);
        float2 acc[TC_EW / 2];
#pragma unroll
        for (int c = 0; c < TC_EW / 2; c++) acc[c] = make_float2(0.0f, 0.0f);
        for (int ks = 0; ks < nstages && ok; ks++) {
            const int s = ks % TC_STAGES;
            if (!__all_sync(0xffffffffu, tc_wait(&B.full[s], (unsigned)(ks / TC_STAGES) & 1u))) {
                if (lane == 0) atomicCAS(p.err, 0, 14);
                ok = false;
                break;
            }
            const uint16_t* sdw = reinterpret_cast<const uint16_t*>(sm + s * TC_STAGE + 2 * TC_A_SUB + 2 * TC_B_SUB);
            const uint16_t* sdx = sdw + TC_BM * 8;
            // this warp's token scales of the stage as f32, [block][token]
            for (int e = lane; e < 8 * TC_EW; e += 32) {
                const int jj = e / TC_EW, tok = e % TC_EW;
                dxf[e] = h2f(sdx[(h * TC_EW + tok) * 8 + jj]);
            }
            __syncwarp();
            for (int j = 0; j < 8; j++) {
                const int g = ks * 8 + j;
                const int buf = g % TC_BUFS;
                if (!__all_sync(0xffffffffu, tc_wait(&B.tfull[buf], (unsigned)(g / TC_BUFS) & 1u))) {
                    if (lane == 0) atomicCAS(p.err, 0, 15);
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint32_t r[TC_EW];
                const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * TC_BN + h * TC_EW);
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
                    "[%16];"
                    : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                      "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                      "=r"(r[15])
                    : "r"(taddr));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&B.tempty[buf]);  // the accumulator is in registers now
                const float dw = h2f(sdw[row * 8 + j]);
                const float2 dw2 = make_float2(dw, dw);
                const float4* dx4 = reinterpret_cast<const float4*>(dxf + j * TC_EW);
#pragma unroll
                for (int c = 0; c < TC_EW / 4; c++) {
                    const float4 x = dx4[c];
                    // exact int -> float: |sumi| <= 32*127*127 < 2^22, so 1.5*2^23 + sumi is an
                    // exactly representable float whose bit pattern is the integer sum
                    const float2 s01 = add2_rn(make_float2(__int_as_float((int)r[4 * c] + 0x4B400000),
                                                              __int_as_float((int)r[4 * c + 1] + 0x4B400000)),
                                                  make_float2(-12582912.0f, -12582912.0f));
                    const float2 s23 = add2_rn(make_float2(__int_as_float((int)r[4 * c + 2] + 0x4B400000),
                                                              __int_as_float((int)r[4 * c + 3] + 0x4B400000)),
                                                  make_float2(-12582912.0f, -12582912.0f));
                    const float2 sc01 = mul2_rn(dw2, make_float2(x.x, x.y));
                    const float2 sc23 = mul2_rn(dw2, make_float2(x.z, x.w));
                    const float2 p01 = mul2_rn(s01, sc01), p23 = mul2_rn(s23, sc23);
                    acc[2 * c].x = __fadd_rn(acc[2 * c].x, p01.x);
                    acc[2 * c].y = __fadd_rn(acc[2 * c].y, p01.y);
                    acc[2 * c + 1].x = __fadd_rn(acc[2 * c + 1].x, p23.x);
                    acc[2 * c + 1].y = __fadd_rn(acc[2 * c + 1].y, p23.y);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&B.empty[s]);  // this stage's scales are used
        }
        if (ok) {
            const int n = n0 + row;
            if (n < p.N) {
#pragma unroll
                for (int c = 0; c < TC_EW; c++) {
                    const int m = m0 + h * TC_EW + c;
                    const float a = (c & 1) ? acc[c / 2].y : acc[c / 2].x;
                    if (m < p.M) {
                        const size_t o = (size_t)m * p.ldy + n;
                        p.y[o] = p.resid ? __fadd_rn(p.resid[o], a) : a;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == TC_EPI_WARPS + 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
}

// ---------------------------------------------------------------------------------------
// host side: tensor maps through the driver entry point (no -lcuda link)
// ---------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn(lq_ctx* ctx) {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
        else
            set_error(ctx, LQ_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
    }
    return fn;
}

int make_tensor_map_2d(lq_ctx* ctx, CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
                    uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                    CUtensorMapSwizzle swz) {
    EncodeTiledFn fn = encode_fn(ctx);
    if (!fn) return LQ_ERR_CUDA;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(ctx, LQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return LQ_OK;
}

bool gemm_tc_supported(int64_t m, int64_t K, const void* wq, const void* xq, const void* wd, const void* xd) {
    if (m < TC_BN || K % TC_KS != 0) return false;
    // TMA: 16-byte aligned bases (row strides K and K/16 bytes are multiples of 16 here)
    for (const void* ptr : {wq, xq, wd, xd})
        if ((uintptr_t)ptr % 16) return false;
    return getenv("LQ_NO_TCGEN05") == nullptr;
}

int launch_gemm_tc(lq_ctx* ctx, const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd, int64_t m, float* y,
                   const float* resid, int64_t ldy) {
    const int64_t N = w->n, K = w->k, nb = K / 32;
    CUtensorMap mw, mx, mdw, mdx;
    int rc;
    if ((rc = make_tensor_map_2d(ctx, &mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->qs, K, N, K, 128, TC_BM,
                       CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    if ((rc = make_tensor_map_2d(ctx, &mx, CU_TENSOR_MAP_DATA_TYPE_UINT8, xq, K, m, K, 128, TC_BN, CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    if ((rc = make_tensor_map_2d(ctx, &mdw, CU_TENSOR_MAP_DATA_TYPE_UINT16, w->d, nb, N, nb * 2, 8, TC_BM,
                       CU_TENSOR_MAP_SWIZZLE_NONE)))
        return rc;
    if ((rc = make_tensor_map_2d(ctx, &mdx, CU_TENSOR_MAP_DATA_TYPE_UINT16, xd, nb, m, nb * 2, 8, TC_BN,
                       CU_TENSOR_MAP_SWIZZLE_NONE)))
        return rc;
    if (const int rc = ensure_func_smem(ctx, (const void*)q8_gemm_tc_kernel, TC_SMEM)) return rc;
    TcParams p;
    p.N = (int)N;
    p.K = (int)K;
    p.M = (int)m;
    p.ldy = (int)ldy;
    p.resid = resid;
    p.y = y;
    p.err = ctx->err_flag;
    const dim3 grid(ceil_div(N, TC_BM), ceil_div(m, TC_BN));
    return launch_kernel(ctx, q8_gemm_tc_kernel, grid, dim3(TC_THREADS), (size_t)TC_SMEM, "q8_gemm_tc", mw, mx, mdw, mdx,
                         p);
}

}  // namespace lq
