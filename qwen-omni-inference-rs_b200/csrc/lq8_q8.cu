// lq8_q8.cu -- Q8_0 quantization, block packing and the Q8_0 x Q8_0 matmul kernels.
//
// Device layout of a Q8_0 tensor [n][k]: qs int8 [n][k] row-major and d fp16 [n][k/32]
// row-major. Both the decode GEMV and the GEMM read this one layout; weights are written
// once at load.
#include "lq8_internal.cuh"

#include <cmath>
#include "lq8_async.cuh"
#include "lq8_fused.cuh"
#include "lq8_tma.cuh"

namespace lq {

// =========================================================================================
// quantization: one 8-lane group per 32-element block, 4 elements per lane
// =========================================================================================
template <typename T>
__device__ __forceinline__ void load4(const T* p, float v[4]);
template <>
__device__ __forceinline__ void load4<float>(const float* p, float v[4]) {
    float4 t = *reinterpret_cast<const float4*>(p);
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
}
template <>
__device__ __forceinline__ void load4<uint16_t>(const uint16_t* p, float v[4]) {
    uint2 t = *reinterpret_cast<const uint2*>(p);
    v[0] = bf16_to_f32((uint16_t)(t.x & 0xFFFF)); v[1] = bf16_to_f32((uint16_t)(t.x >> 16));
    v[2] = bf16_to_f32((uint16_t)(t.y & 0xFFFF)); v[3] = bf16_to_f32((uint16_t)(t.y >> 16));
}

template <typename T>
__global__ void quantize_rows_kernel(const T* __restrict__ src, int64_t nblocks, int8_t* __restrict__ qs,
                                     uint16_t* __restrict__ d) {
    int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t blk = gid >> 3;
    int sub = threadIdx.x & 7;
    bool valid = blk < nblocks;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (valid) load4<T>(src + blk * QK + sub * 4, v);
    uint32_t q = quant_group8(v, sub, valid ? d + blk : nullptr);
    if (valid) reinterpret_cast<uint32_t*>(qs + blk * QK)[sub] = q;
}

int launch_quantize_rows(lq_ctx* ctx, const void* src, lq_dtype dt, int64_t rows, int64_t k,
                         int8_t* qs, uint16_t* d) {
    int64_t nblocks = rows * (k / QK);
    if (nblocks == 0) return LQ_OK;
    int64_t threads = nblocks * 8;
    int grid = (int)((threads + 255) / 256);
    if (dt == LQ_DTYPE_F32)
        quantize_rows_kernel<float><<<grid, 256, 0, ctx->stream>>>((const float*)src, nblocks, qs, d);
    else
        quantize_rows_kernel<uint16_t><<<grid, 256, 0, ctx->stream>>>((const uint16_t*)src, nblocks, qs, d);
    LQ_LAUNCH_CHECK(ctx, "quantize_rows");
    return LQ_OK;
}

// =========================================================================================
// GGML block packing: {fp16 d; int8 qs[32]} (34 bytes) <-> SoA
// =========================================================================================
__global__ void pack_blocks_kernel(const int8_t* __restrict__ qs, const uint16_t* __restrict__ d,
                                   int64_t nblocks, uint8_t* __restrict__ out) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // byte index in output
    if (i >= nblocks * 34) return;
    int64_t b = i / 34;
    int o = (int)(i - b * 34);
    uint8_t v;
    if (o < 2) v = (uint8_t)(d[b] >> (8 * o));
    else v = (uint8_t)qs[b * QK + (o - 2)];
    out[i] = v;
}

__global__ void unpack_blocks_kernel(const uint8_t* __restrict__ in, int64_t nblocks,
                                     int8_t* __restrict__ qs, uint16_t* __restrict__ d) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nblocks * 34) return;
    int64_t b = i / 34;
    int o = (int)(i - b * 34);
    if (o == 0) d[b] = (uint16_t)(in[i] | (in[i + 1] << 8));
    else if (o >= 2) qs[b * QK + (o - 2)] = (int8_t)in[i];
}

// =========================================================================================
// decode GEMV, M <= 4 tokens: CUDA-core dp4a. One warp owns R weight rows over all of K;
// lane l takes blocks l, l+32, ... (32 contiguous bytes each, two 128-bit streaming loads),
// so a warp reads 1 KiB contiguous per row per step. Per-lane partial sums are combined by a
// butterfly reduction. x (quantized activations) is read through L1.
// =========================================================================================
template <int M, int R, int U>
__global__ void __launch_bounds__(256)
q8_gemv_dp4a_kernel(const int8_t* __restrict__ wq, const uint16_t* __restrict__ wd, int N, int K,
                    const int8_t* __restrict__ xq, const uint16_t* __restrict__ xd,
                    const float* resid, float* y, int ldy, unsigned long long* argmax_keys) {
    const int lane = threadIdx.x & 31;
    const int row0 = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * R;
    const int nb = K >> 5;
    float acc[R][M];
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int m = 0; m < M; m++) acc[r][m] = 0.0f;
    const bool warp_active = row0 < N;
    if (warp_active) {
        const int8_t* wrow[R];
        const uint16_t* drow[R];
#pragma unroll
        for (int r = 0; r < R; r++) {
            int row = min(row0 + r, N - 1);
            wrow[r] = wq + (size_t)row * K;
            drow[r] = wd + (size_t)row * nb;
        }
        for (int b0 = 0; b0 < nb; b0 += 32 * U) {
            int4 w[U][R][2];
            uint16_t dw[U][R];
#pragma unroll
            for (int u = 0; u < U; u++) {
                int b = b0 + u * 32 + lane;
                if (b < nb) {
#pragma unroll
                    for (int r = 0; r < R; r++) {
                        w[u][r][0] = ld_stream_v4(wrow[r] + (size_t)b * QK);
                        w[u][r][1] = ld_stream_v4(wrow[r] + (size_t)b * QK + 16);
                        dw[u][r] = drow[r][b];
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                int b = b0 + u * 32 + lane;
                if (b < nb) {
#pragma unroll
                    for (int m = 0; m < M; m++) {
                        const int4* xp = reinterpret_cast<const int4*>(xq + (size_t)m * K + (size_t)b * QK);
                        int4 x0 = __ldg(xp), x1 = __ldg(xp + 1);
                        float dx = h2f(xd[(size_t)m * nb + b]);
#pragma unroll
                        for (int r = 0; r < R; r++) {
                            int s = 0;
                            s = __dp4a(w[u][r][0].x, x0.x, s); s = __dp4a(w[u][r][0].y, x0.y, s);
                            s = __dp4a(w[u][r][0].z, x0.z, s); s = __dp4a(w[u][r][0].w, x0.w, s);
                            s = __dp4a(w[u][r][1].x, x1.x, s); s = __dp4a(w[u][r][1].y, x1.y, s);
                            s = __dp4a(w[u][r][1].z, x1.z, s); s = __dp4a(w[u][r][1].w, x1.w, s);
                            float sc = __fmul_rn(h2f(dw[u][r]), dx);
                            acc[r][m] = __fadd_rn(acc[r][m], __fmul_rn((float)s, sc));
                        }
                    }
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int m = 0; m < M; m++) acc[r][m] = warp_sum(acc[r][m]);
    // lane i < R*M writes output (i / M, i % M)
    if (warp_active) {
#pragma unroll
        for (int r = 0; r < R; r++)
#pragma unroll
            for (int m = 0; m < M; m++) {
                if (lane == r * M + m && row0 + r < N) {
                    size_t o = (size_t)m * ldy + row0 + r;
                    float v = acc[r][m];
                    if (resid) v = __fadd_rn(resid[o], v);
                    y[o] = v;
                }
            }
    }
    if (argmax_keys) {
        // fused greedy argmax of the LM head: per-CTA max key in shared memory, then one
        // 64-bit atomicMax per token per CTA (ties resolve to the highest row index)
        __shared__ unsigned long long cta_keys[M];
        if (threadIdx.x < M) cta_keys[threadIdx.x] = 0ull;
        __syncthreads();
        if (warp_active && lane == 0) {
#pragma unroll
            for (int m = 0; m < M; m++) {
                unsigned long long key = 0ull;
#pragma unroll
                for (int r = 0; r < R; r++)
                    if (row0 + r < N) {
                        unsigned long long kk = argmax_key(acc[r][m], row0 + r);
                        key = kk > key ? kk : key;
                    }
                atomicMax(&cta_keys[m], key);
            }
        }
        __syncthreads();
        if (threadIdx.x < M && cta_keys[threadIdx.x]) atomicMax(argmax_keys + threadIdx.x, cta_keys[threadIdx.x]);
    }
}

// =========================================================================================
// Q8_0 GEMM on mma.sync m16n8k32 (s8 x s8 -> s32), one MMA = one Q8_0 block of K.
// Weights are the MMA "A" operand (16 rows), tokens the "B" operand (8 columns). Tiles are
// staged in shared memory with cp.async (BK = 64 bytes = 2 blocks per stage). Every output
// is owned by one thread, which adds the per-block terms (float)sumi * (d_w*d_x) in
// ascending block order with separately rounded multiply and add -- the oracle's order, so
// results are bit-identical to it.
// =========================================================================================
constexpr int GEMM_BK = 64;            // bytes of K per stage
constexpr int GEMM_LDS = GEMM_BK + 16; // padded smem row stride (conflict-free ldmatrix)
constexpr int GEMM_STAGES = 4;

template <int BW, int BX, int WW, int WX>
struct GemmCfg {
    static constexpr int THREADS = WW * WX * 32;
    static constexpr int TW = BW / WW;   // weight rows per warp
    static constexpr int TX = BX / WX;   // tokens per warp
    static constexpr int MI = TW / 16;   // m16 tiles per warp
    static constexpr int NJ = TX / 8;    // n8 tiles per warp
    static constexpr int W_BYTES = BW * GEMM_LDS;
    static constexpr int X_BYTES = BX * GEMM_LDS;
    static constexpr int WS_BYTES = BW * 2 * 2;  // 2 fp16 scales per row per stage
    static constexpr int XS_BYTES = BX * 2 * 2;
    static constexpr int STAGE = W_BYTES + X_BYTES + WS_BYTES + XS_BYTES;
    static constexpr int SMEM = STAGE * GEMM_STAGES;
};

template <int BW, int BX, int WW, int WX>
__global__ void __launch_bounds__(WW * WX * 32)
q8_gemm_mma_kernel(const int8_t* __restrict__ wq, const uint16_t* __restrict__ wd, int N, int K,
                   const int8_t* __restrict__ xq, const uint16_t* __restrict__ xd, int M,
                   const float* resid, float* y, int ldy, unsigned long long* argmax_keys, int kslice,
                   float* part) {
    using C = GemmCfg<BW, BX, WW, WX>;
    extern __shared__ __align__(128) uint8_t smem[];
    pdl_wait();
    pdl_trigger();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ww = warp % WW, wx = warp / WW;
    const int n0 = blockIdx.x * BW;  // weight row base
    const int m0 = blockIdx.y * BX;  // token base
    const int nb = K >> 5;
    // K-split (part != nullptr): this CTA covers K bytes [k_lo, k_hi) and writes its partial
    // sums to part[blockIdx.z][M][N]; a second kernel adds the slices in order
    const int k_lo = part ? blockIdx.z * kslice : 0;
    const int k_hi = part ? min(K, k_lo + kslice) : K;
    const int nstages_k = (k_hi - k_lo + GEMM_BK - 1) / GEMM_BK;

    auto stage_ptr = [&](int s) { return smem + s * C::STAGE; };

    auto load_stage = [&](int s, int kt) {
        uint8_t* base = stage_ptr(s);
        uint8_t* sw = base;
        uint8_t* sx = base + C::W_BYTES;
        uint16_t* sws = reinterpret_cast<uint16_t*>(base + C::W_BYTES + C::X_BYTES);
        uint16_t* sxs = reinterpret_cast<uint16_t*>(base + C::W_BYTES + C::X_BYTES + C::WS_BYTES);
        const int kb = k_lo + kt * GEMM_BK;  // byte offset in K
        // weights: BW rows x 4 chunks of 16 B
        for (int c = tid; c < BW * 4; c += C::THREADS) {
            int r = c >> 2, ch = c & 3;
            int row = n0 + r;
            int kk = kb + ch * 16;
            bool p = row < N && kk < k_hi;
            const int8_t* g = wq + (size_t)(p ? row : 0) * K + (p ? kk : 0);
            cp_async16(sw + r * GEMM_LDS + ch * 16, g, p);
        }
        for (int c = tid; c < BX * 4; c += C::THREADS) {
            int r = c >> 2, ch = c & 3;
            int tok = m0 + r;
            int kk = kb + ch * 16;
            bool p = tok < M && kk < k_hi;
            const int8_t* g = xq + (size_t)(p ? tok : 0) * K + (p ? kk : 0);
            cp_async16(sx + r * GEMM_LDS + ch * 16, g, p);
        }
        // scales: 2 blocks per row = 4 bytes; the 4-byte async copy needs an even block count
        // per row (so that row*nb + b is even); otherwise plain loads
        const int b = kb >> 5, bhi = k_hi >> 5;
        const bool even = (nb & 1) == 0 && b + 1 < bhi;
        for (int r = tid; r < BW; r += C::THREADS) {
            int row = n0 + r;
            if (row < N && even) {
                cp_async4(sws + r * 2, wd + (size_t)row * nb + b, true);
            } else {
                sws[r * 2] = (row < N && b < bhi) ? wd[(size_t)row * nb + b] : (uint16_t)0;
                sws[r * 2 + 1] = (row < N && b + 1 < bhi) ? wd[(size_t)row * nb + b + 1] : (uint16_t)0;
            }
        }
        for (int r = tid; r < BX; r += C::THREADS) {
            int tok = m0 + r;
            if (tok < M && even) {
                cp_async4(sxs + r * 2, xd + (size_t)tok * nb + b, true);
            } else {
                sxs[r * 2] = (tok < M && b < bhi) ? xd[(size_t)tok * nb + b] : (uint16_t)0;
                sxs[r * 2 + 1] = (tok < M && b + 1 < bhi) ? xd[(size_t)tok * nb + b + 1] : (uint16_t)0;
            }
        }
    };

    float acc[C::MI][C::NJ][4];
#pragma unroll
    for (int i = 0; i < C::MI; i++)
#pragma unroll
        for (int j = 0; j < C::NJ; j++)
#pragma unroll
            for (int e = 0; e < 4; e++) acc[i][j][e] = 0.0f;

#pragma unroll
    for (int s = 0; s < GEMM_STAGES - 1; s++) {
        if (s < nstages_k) load_stage(s, s);
        cp_async_commit();
    }

    const int g = lane >> 2, t = lane & 3;
    for (int kt = 0; kt < nstages_k; kt++) {
        cp_async_wait<GEMM_STAGES - 2>();
        __syncthreads();
        {
            int nk = kt + GEMM_STAGES - 1;
            if (nk < nstages_k) load_stage(nk % GEMM_STAGES, nk);
            cp_async_commit();
        }
        const uint8_t* base = stage_ptr(kt % GEMM_STAGES);
        const uint8_t* sw = base;
        const uint8_t* sx = base + C::W_BYTES;
        const uint16_t* sws = reinterpret_cast<const uint16_t*>(base + C::W_BYTES + C::X_BYTES);
        const uint16_t* sxs = reinterpret_cast<const uint16_t*>(base + C::W_BYTES + C::X_BYTES + C::WS_BYTES);
#pragma unroll
        for (int kb = 0; kb < 2; kb++) {
            uint32_t a[C::MI][4];
            uint32_t bf[C::NJ][2];
#pragma unroll
            for (int i = 0; i < C::MI; i++) {
                int r = ww * C::TW + i * 16 + (lane & 15);
                ldmatrix_x4(a[i], sw + r * GEMM_LDS + kb * 32 + (lane >> 4) * 16);
            }
#pragma unroll
            for (int j = 0; j < C::NJ; j++) {
                int r = wx * C::TX + j * 8 + (lane & 7);
                ldmatrix_x2(bf[j], sx + r * GEMM_LDS + kb * 32 + ((lane >> 3) & 1) * 16);
            }
            float dw[C::MI][2], dx[C::NJ][2];
#pragma unroll
            for (int i = 0; i < C::MI; i++) {
                int r = ww * C::TW + i * 16 + g;
                dw[i][0] = h2f(sws[r * 2 + kb]);
                dw[i][1] = h2f(sws[(r + 8) * 2 + kb]);
            }
#pragma unroll
            for (int j = 0; j < C::NJ; j++) {
                int r = wx * C::TX + j * 8 + 2 * t;
                dx[j][0] = h2f(sxs[r * 2 + kb]);
                dx[j][1] = h2f(sxs[(r + 1) * 2 + kb]);
            }
#pragma unroll
            for (int i = 0; i < C::MI; i++)
#pragma unroll
                for (int j = 0; j < C::NJ; j++) {
                    int c[4];
                    mma_s8(c, a[i], bf[j]);
                    acc[i][j][0] = __fadd_rn(acc[i][j][0], __fmul_rn((float)c[0], __fmul_rn(dw[i][0], dx[j][0])));
                    acc[i][j][1] = __fadd_rn(acc[i][j][1], __fmul_rn((float)c[1], __fmul_rn(dw[i][0], dx[j][1])));
                    acc[i][j][2] = __fadd_rn(acc[i][j][2], __fmul_rn((float)c[2], __fmul_rn(dw[i][1], dx[j][0])));
                    acc[i][j][3] = __fadd_rn(acc[i][j][3], __fmul_rn((float)c[3], __fmul_rn(dw[i][1], dx[j][1])));
                }
        }
    }
    cp_async_wait<0>();

    // epilogue: element e of tile (i,j): weight row n = 16i + g + 8*(e>>1), token 8j + 2t + (e&1)
#pragma unroll
    for (int i = 0; i < C::MI; i++)
#pragma unroll
        for (int j = 0; j < C::NJ; j++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                int n = n0 + ww * C::TW + i * 16 + g + 8 * (e >> 1);
                int m = m0 + wx * C::TX + j * 8 + 2 * t + (e & 1);
                if (n < N && m < M) {
                    if (part) {
                        part[((size_t)blockIdx.z * M + m) * N + n] = acc[i][j][e];
                        continue;
                    }
                    size_t o = (size_t)m * ldy + n;
                    float v = acc[i][j][e];
                    if (resid) v = __fadd_rn(resid[o], v);
                    y[o] = v;
                }
            }
    if (argmax_keys && !part) {
        // per token: max over this thread's rows, then over the 8 lanes sharing t, then over
        // the CTA in shared memory, then one global atomic per token per CTA
        __shared__ unsigned long long cta_keys[BX];
        for (int i = tid; i < BX; i += C::THREADS) cta_keys[i] = 0ull;
        __syncthreads();
#pragma unroll
        for (int j = 0; j < C::NJ; j++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                int m = m0 + wx * C::TX + j * 8 + 2 * t + h;
                unsigned long long key = 0ull;
#pragma unroll
                for (int i = 0; i < C::MI; i++)
#pragma unroll
                    for (int e2 = 0; e2 < 2; e2++) {
                        int n = n0 + ww * C::TW + i * 16 + g + 8 * e2;
                        if (n < N && m < M) {
                            unsigned long long kk = argmax_key(acc[i][j][e2 * 2 + h], n);
                            key = kk > key ? kk : key;
                        }
                    }
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) {
                    unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
                    key = other > key ? other : key;
                }
                if (g == 0 && m < M) atomicMax(&cta_keys[m - m0], key);
            }
        __syncthreads();
        for (int i = tid; i < BX; i += C::THREADS)
            if (m0 + i < M && cta_keys[i]) atomicMax(argmax_keys + m0 + i, cta_keys[i]);
    }
}

// K-split combine: y[m][n] = resid + sum over the slices in ascending order; the greedy
// argmax keys (if any) per token over the CTA's outputs
__global__ void gemm_split_reduce_kernel(const float* __restrict__ part, int splits, int M, int N, const float* resid,
                                         float* y, int ldy, unsigned long long* keys) {
    pdl_trigger();  // early: the next kernel (a weight stream) may start; it waits for us in pdl_wait
    pdl_wait();
    // one column per thread; the slices' values are loaded 8 at a time ahead of the adds
    const int m = blockIdx.y, n = blockIdx.x * blockDim.x + threadIdx.x;
    __shared__ unsigned long long ck;
    if (threadIdx.x == 0) ck = 0ull;
    __syncthreads();
    unsigned long long key = 0ull;
    if (n < N) {
        const float* pp = part + (size_t)m * N + n;
        const size_t stride = (size_t)M * N;
        float v = 0.0f;
        int s = 0;
        for (; s + 8 <= splits; s += 8) {
            float t[8];
#pragma unroll
            for (int i = 0; i < 8; i++) t[i] = pp[(size_t)(s + i) * stride];
#pragma unroll
            for (int i = 0; i < 8; i++) v = __fadd_rn(v, t[i]);
        }
        for (; s < splits; s++) v = __fadd_rn(v, pp[(size_t)s * stride]);
        const size_t o = (size_t)m * ldy + n;
        if (resid) v = __fadd_rn(resid[o], v);
        y[o] = v;
        if (keys) {
            const unsigned long long kk = argmax_key(v, n);
            key = kk > key ? kk : key;
        }
    }
    if (keys) {
        atomicMax(&ck, key);
        __syncthreads();
        if (threadIdx.x == 0 && ck) atomicMax(keys + m, ck);
    }
}

// splits of K (whole 64-byte stages) that give the grid about three waves of CTAs when the
// plain grid of a small-M (<= 64 tokens) GEMM is short of two; 1 = no split (bit-identical to
// the oracle; LQ_GEMM_NO_SPLIT=1 forces it)
static int gemm_splits(lq_ctx* ctx, int64_t tiles, int64_t K, int64_t m) {
    if (m > 64 || tiles >= 2 * ctx->sm_count || getenv("LQ_GEMM_NO_SPLIT")) return 1;
    int64_t s = (3 * (int64_t)ctx->sm_count + tiles - 1) / tiles;
    const int64_t kst = (K + GEMM_BK - 1) / GEMM_BK;
    s = std::min<int64_t>(s, std::max<int64_t>(1, kst / 4));  // at least 4 stages per slice
    return (int)std::max<int64_t>(1, std::min<int64_t>(s, 32));
}

static int split_slice(int64_t K, int splits) {
    const int64_t kst = (K + GEMM_BK - 1) / GEMM_BK;
    return (int)(((kst + splits - 1) / splits) * GEMM_BK);
}

// mirrors run_gemm's choice (128-row tiles; 16/32/64-token tiles for m <= 64)
static int gs_slices(lq_ctx* ctx, int64_t n, int64_t k, int64_t m);
// the skinny (5-8 token) GEMM's partial buffer for an (n, k) weight (0 if it does not apply)
static size_t sk_partial_bytes(lq_ctx* ctx, int64_t n, int64_t k);

size_t gemm_split_bytes(lq_ctx* ctx, int64_t n, int64_t k, int64_t m) {
    if (m <= 4 || m > 64) return 0;
    // the streamed GEMM's slices when the shape qualifies (its alignment is checked per call, so
    // the mma.sync GEMM's need counts too)
    size_t gs = 0;
    if (k % 256 == 0 && n % 64 == 0) {
        const int s0 = gs_slices(ctx, n, k, m);
        const int64_t chunks = k / 256, ks = ((chunks + s0 - 1) / s0) * 256;
        if (s0 > 1) gs = (size_t)((k + ks - 1) / ks) * m * n * 4;
    }
    // the skinny GEMM's partial buffer (its alignment too is checked per call)
    if (m <= 8) gs = std::max(gs, sk_partial_bytes(ctx, n, k));
    const int64_t bx = m <= 16 ? 16 : m <= 32 ? 32 : 64;
    const int splits0 = gemm_splits(ctx, (int64_t)ceil_div(n, 128) * ceil_div(m, bx), k, m);
    if (splits0 <= 1) return gs;
    const int splits = ceil_div(k, split_slice(k, splits0));
    return std::max(gs, (size_t)splits * m * n * 4);
}

// K-split partials: the caller's fixed buffer when given, else the context's split buffer
static int split_partials(lq_ctx* ctx, const SplitBuf* fixed, size_t bytes, float** out) {
    if (fixed) {
        if (bytes > fixed->bytes)
            return set_error(ctx, LQ_ERR_STATE, "K-split partials need %zu bytes; the fixed buffer holds %zu", bytes,
                             fixed->bytes);
        *out = fixed->p;
        return LQ_OK;
    }
    const int rc = ensure_split(ctx, bytes);
    if (rc) return rc;
    *out = reinterpret_cast<float*>(ctx->split);
    return LQ_OK;
}

template <int BW, int BX, int WW, int WX>
static int run_gemm(lq_ctx* ctx, const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd,
                    int64_t m, float* y, const float* resid, int64_t ldy,
                    unsigned long long* keys, const SplitBuf* fixed) {
    using C = GemmCfg<BW, BX, WW, WX>;
    if (const int rc = ensure_func_smem(ctx, (const void*)q8_gemm_mma_kernel<BW, BX, WW, WX>, C::SMEM)) return rc;
    const int64_t tiles = (int64_t)ceil_div(w->n, BW) * ceil_div(m, BX);
    int splits = gemm_splits(ctx, tiles, w->k, m);
    int kslice = 0;
    float* part = nullptr;
    if (splits > 1) {
        kslice = split_slice(w->k, splits);
        splits = ceil_div(w->k, kslice);
        const int rc = split_partials(ctx, fixed, (size_t)splits * m * w->n * 4, &part);
        if (rc) return rc;
    }
    dim3 grid(ceil_div(w->n, BW), ceil_div(m, BX), splits);
    int rc = launch_kernel(ctx, q8_gemm_mma_kernel<BW, BX, WW, WX>, grid, dim3(C::THREADS), C::SMEM, "q8_gemm_mma",
                           w->qs, w->d, (int)w->n, (int)w->k, xq, xd, (int)m, resid, y, (int)ldy, keys, kslice, part);
    if (rc || splits == 1) return rc;
    return launch_kernel(ctx, gemm_split_reduce_kernel, dim3((unsigned)ceil_div(w->n, 256), (unsigned)m), dim3(256), 0,
                         "gemm_split_reduce", (const float*)part, splits, (int)m, (int)w->n, resid, y, (int)ldy, keys);
}

template <int M, int R>
static int run_gemv(lq_ctx* ctx, const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd,
                    float* y, const float* resid, int64_t ldy, unsigned long long* keys) {
    constexpr int U = (R >= 4) ? 2 : 4;
    int warps = ceil_div(w->n, R);
    int grid = ceil_div(warps, 8);
    q8_gemv_dp4a_kernel<M, R, U><<<grid, 256, 0, ctx->stream>>>(
        w->qs, w->d, (int)w->n, (int)w->k, xq, xd, resid, y, (int)ldy, keys);
    LQ_LAUNCH_CHECK(ctx, "q8_gemv_dp4a");
    return LQ_OK;
}

template <int M>
static int gemv_rows(lq_ctx* ctx, const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd,
                     float* y, const float* resid, int64_t ldy, unsigned long long* keys) {
    // enough warps to fill the SMs at least twice over: 148 SMs x 16 warps
    int64_t target = (int64_t)ctx->sm_count * 32;
    if (w->n / 4 >= target) return run_gemv<M, 4>(ctx, w, xq, xd, y, resid, ldy, keys);
    if (w->n / 2 >= target) return run_gemv<M, 2>(ctx, w, xq, xd, y, resid, ldy, keys);
    return run_gemv<M, 1>(ctx, w, xq, xd, y, resid, ldy, keys);
}

// =========================================================================================
// Small-M Q8_0 GEMM, streamed (5 <= m <= 64 tokens): the MoE expert kernel's pipeline for a
// dense weight. Work item = (64 weight rows, K slice, pass of TOK = 16 or 32 tokens); one
// producer lane streams per 256-byte K-chunk the item's weight rows (two 32-row groups x two
// 128-byte boxes, 128-byte swizzle), their fp16 scales, the pass's TOK token rows of the
// quantized activations (two swizzled boxes; rows past m read as zeros) and the tokens'
// scales into a shared-memory ring (22 or 26 KiB per stage). Eight consumer warps each own 16
// weight rows (one m16 tile) and TOK/16 of the pass's n8 tiles; each m16n8k32 MMA is one Q8_0
// block, its int32 dots become floats by the 1.5*2^23 bias (the MMA accumulates onto it) and
// are scaled and added per (row, token) in ascending block order with separately rounded
// multiply and add: the oracle's order, bit-identical to it when K is not split. Passes of
// one row tile run back to back, so the later passes read the weights from L2. Too few row
// tiles for the SMs split K into slices whose partials gemm_split_reduce adds in order.
// =========================================================================================
constexpr int GS_KC = 256;
constexpr int GS_CONS = 8;
constexpr int GS_THREADS = (GS_CONS + 1) * 32;
constexpr int GS_STAGES = 4;
constexpr int GS_BOXW = 32 * 128;                   // one weight box: 32 rows x 128 bytes
constexpr int GS_W = 4 * GS_BOXW;                   // 16 KiB: [group][half][32][128]
constexpr int GS_WD = 64 * 16;                      // weight scales [64][8] fp16

// TOK tokens per pass: activation boxes [2][TOK][128 B], token scales [TOK][8] fp16; each
// consumer warp takes TOK / 16 of the pass's n8 tiles
template <int TOK>
struct GsCfg {
    static constexpr int BOXX = TOK * 128;
    static constexpr int X = 2 * BOXX;
    static constexpr int XD = TOK * 16;
    static constexpr int BYTES = GS_W + X + GS_WD + XD;  // bytes landing per stage
    static constexpr int STAGE = (BYTES + 1023) / 1024 * 1024;
    static constexpr size_t SMEM = (size_t)GS_STAGES * STAGE + 2 * GS_STAGES * 8 + 64 * 8 + 1024;
    static constexpr int NTW = TOK / 16;
};

struct GsParams {
    int N, K, M;
    int tiles, slices, passes, kslice;  // kslice: K bytes per slice (a multiple of 256)
    const float* resid;
    float* y;
    int ldy;
    float* part;                  // slices > 1: [slices][M][N]
    unsigned long long* keys;     // fused greedy argmax (slices == 1 only)
    int* err;
};

template <int TOK>
__global__ void __launch_bounds__(GS_THREADS, 2) q8_gemm_stream_kernel(const __grid_constant__ CUtensorMap mw,
                                                                       const __grid_constant__ CUtensorMap mwd,
                                                                       const __grid_constant__ CUtensorMap mx,
                                                                       const __grid_constant__ CUtensorMap mxd,
                                                                       const GsParams p) {
    using C = GsCfg<TOK>;
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const uint32_t raw = smem_addr(smem_raw);
    uint8_t* sm = smem_raw + (((raw + 1023) & ~1023u) - raw);  // swizzled boxes need 1024-byte alignment
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + (size_t)GS_STAGES * C::STAGE);
    uint64_t* empty = full + GS_STAGES;
    unsigned long long* ckeys = reinterpret_cast<unsigned long long*>(empty + GS_STAGES);  // [64]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < GS_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], GS_CONS);
        }
        mbar_fence_init();
    }
    if (threadIdx.x < 64) ckeys[threadIdx.x] = 0ull;
    __syncthreads();
    const long long items = (long long)p.tiles * p.slices * p.passes;
    const long long i0 = items * blockIdx.x / gridDim.x, i1 = items * (blockIdx.x + 1) / gridDim.x;

    if (warp == GS_CONS) {
        // ---------------- producer (one lane); weights may stream before pdl_wait ----------------
        if (lane != 0) return;
        int it = 0;
        // the activations come from the preceding kernel: until pdl_wait has returned, only the
        // weights of the first stages go out (the whole ring, while that kernel finishes), and
        // their activation boxes follow in one batch after the wait
        bool waited = false;
        int npend = 0;
        int pend_k[GS_STAGES], pend_p[GS_STAGES];
        auto load_x = [&](int s, int k, int ps) {
            uint8_t* st = sm + (size_t)s * C::STAGE;
            tma_load_2d(st + GS_W, &mx, k, ps * TOK, &full[s]);
            tma_load_2d(st + GS_W + C::BOXX, &mx, k + 128, ps * TOK, &full[s]);
            tma_load_2d(st + GS_W + C::X + GS_WD, &mxd, k / 32, ps * TOK, &full[s]);
        };
        auto flush = [&]() {
            pdl_wait();
            waited = true;
            for (int i = 0; i < npend; i++) load_x(i, pend_k[i], pend_p[i]);  // stages 0 .. npend-1
            npend = 0;
        };
        for (long long item = i0; item < i1; item++) {
            const int ps = (int)(item % p.passes);
            const int sl = (int)((item / p.passes) % p.slices);
            const int rt = (int)(item / ((long long)p.passes * p.slices));
            const int k0 = sl * p.kslice, k1 = min(p.K, k0 + p.kslice);
            for (int k = k0; k < k1; k += GS_KC, it++) {
                if (!waited && npend == GS_STAGES) flush();
                const int s = it % GS_STAGES;
                if (!mbar_wait(&empty[s], ((unsigned)(it / GS_STAGES) & 1u) ^ 1u)) {
                    atomicCAS(p.err, 0, 24);
                    if (!waited) pdl_wait();
                    return;
                }
                uint8_t* st = sm + (size_t)s * C::STAGE;
                mbar_expect_tx(&full[s], (unsigned)C::BYTES);
                for (int q = 0; q < 2; q++) {
                    const int row = rt * 64 + q * 32;
                    tma_load_2d(st + q * 2 * GS_BOXW, &mw, k, row, &full[s]);
                    tma_load_2d(st + q * 2 * GS_BOXW + GS_BOXW, &mw, k + 128, row, &full[s]);
                    tma_load_2d(st + GS_W + C::X + q * 32 * 16, &mwd, k / 32, row, &full[s]);
                }
                if (waited) {
                    load_x(s, k, ps);
                } else {
                    pend_k[npend] = k;
                    pend_p[npend] = ps;
                    npend++;
                }
            }
        }
        if (!waited) flush();
        return;
    }
    // ---------------- consumers ----------------
    pdl_wait();  // resid / y / keys belong to the preceding kernels
    pdl_trigger();
    constexpr int NTW = C::NTW;
    const int g = lane >> 2, t = lane & 3;
    const int mt = warp & 3, n0 = (warp >> 2) * NTW;  // m16 tile (16 weight rows), first n8 tile
    const int q = mt >> 1;
    const int ra = 16 * (mt & 1) + g;                  // rows ra and ra + 8 of group q
    const int a_off = q * 2 * GS_BOXW + ra * 128 + (t & 1) * 8;
    const int b_off = GS_W + (8 * n0 + g) * 128 + (t & 1) * 8;
    const int sc_off = GS_W + C::X + (q * 32 + ra) * 16;
    const int xd_off = GS_W + C::X + GS_WD + (8 * n0 + 2 * t) * 16;
    int it = 0;
    bool bad = false;
    for (long long item = i0; item < i1; item++) {
        const int ps = (int)(item % p.passes);
        const int sl = (int)((item / p.passes) % p.slices);
        const int rt = (int)(item / ((long long)p.passes * p.slices));
        const int k0 = sl * p.kslice, k1 = min(p.K, k0 + p.kslice);
        const int ntok = min(TOK, p.M - ps * TOK);
        const int nact = min(NTW, max(0, (ntok - 8 * n0 + 7) / 8));  // this warp's tiles holding tokens
        float acc[NTW][4];
#pragma unroll
        for (int i = 0; i < NTW; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
        for (int k = k0; k < k1; k += GS_KC, it++) {
            const int s = it % GS_STAGES;
            if (!bad) {
                bool ok = true;
                if (lane == 0) ok = mbar_wait(&full[s], (unsigned)(it / GS_STAGES) & 1u);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) {
                    if (lane == 0) atomicCAS(p.err, 0, 25);
                    bad = true;
                }
            }
            if (bad) continue;
            const uint8_t* st = sm + (size_t)s * C::STAGE;
            if (nact == 0) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
                continue;
            }
            // one n8 tile: the warp's whole slice of the stage into registers and the stage
            // released at once; two tiles: the token fragments are read block by block and
            // the stage released after the blocks (fewer live registers)
            constexpr bool EARLY = NTW == 1;
            uint2 wa[8], wb[8], xv[EARLY ? 8 : 1];
            uint4 ua[NTW], ub[NTW];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int ch = ((2 * (j & 3) + (t >> 1)) ^ g) << 4;
                wa[j] = *reinterpret_cast<const uint2*>(st + a_off + (j >> 2) * GS_BOXW + ch);
                wb[j] = *reinterpret_cast<const uint2*>(st + a_off + 8 * 128 + (j >> 2) * GS_BOXW + ch);
                if constexpr (EARLY) xv[j] = *reinterpret_cast<const uint2*>(st + b_off + (j >> 2) * C::BOXX + ch);
            }
            const uint4 sa = *reinterpret_cast<const uint4*>(st + sc_off);
            const uint4 sb = *reinterpret_cast<const uint4*>(st + sc_off + 8 * 16);
#pragma unroll
            for (int i = 0; i < NTW; i++) {
                ua[i] = *reinterpret_cast<const uint4*>(st + xd_off + i * 8 * 16);
                ub[i] = *reinterpret_cast<const uint4*>(st + xd_off + i * 8 * 16 + 16);
            }
            if constexpr (EARLY) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
            }
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const uint32_t a[4] = {wa[j].x, wb[j].x, wa[j].y, wb[j].y};
                const uint32_t wsa = j < 2 ? sa.x : j < 4 ? sa.y : j < 6 ? sa.z : sa.w;
                const uint32_t wsb = j < 2 ? sb.x : j < 4 ? sb.y : j < 6 ? sb.z : sb.w;
                const float dwa = h2f((uint16_t)((j & 1) ? (wsa >> 16) : (wsa & 0xFFFFu)));
                const float dwb = h2f((uint16_t)((j & 1) ? (wsb >> 16) : (wsb & 0xFFFFu)));
                const int ch = ((2 * (j & 3) + (t >> 1)) ^ g) << 4;
#pragma unroll
                for (int i = 0; i < NTW; i++) {
                    if (i >= nact) break;
                    const uint2 xj = EARLY ? xv[EARLY ? j : 0]
                                           : *reinterpret_cast<const uint2*>(st + b_off + i * 8 * 128 +
                                                                             (j >> 2) * C::BOXX + ch);
                    const uint32_t b[2] = {xj.x, xj.y};
                    int d[4];
                    mma_s8_bias(d, a, b, 0x4B400000);
                    const uint32_t wx0 = j < 2 ? ua[i].x : j < 4 ? ua[i].y : j < 6 ? ua[i].z : ua[i].w;
                    const uint32_t wx1 = j < 2 ? ub[i].x : j < 4 ? ub[i].y : j < 6 ? ub[i].z : ub[i].w;
                    const float dx0 = h2f((uint16_t)((j & 1) ? (wx0 >> 16) : (wx0 & 0xFFFFu)));
                    const float dx1 = h2f((uint16_t)((j & 1) ? (wx1 >> 16) : (wx1 & 0xFFFFu)));
                    // the MMA added the dots to 1.5 * 2^23: one subtraction gives (float)dot exactly
                    const float f0 = __fsub_rn(__int_as_float(d[0]), 12582912.0f);
                    const float f1 = __fsub_rn(__int_as_float(d[1]), 12582912.0f);
                    const float f2 = __fsub_rn(__int_as_float(d[2]), 12582912.0f);
                    const float f3 = __fsub_rn(__int_as_float(d[3]), 12582912.0f);
                    acc[i][0] = __fadd_rn(acc[i][0], __fmul_rn(f0, __fmul_rn(dwa, dx0)));
                    acc[i][1] = __fadd_rn(acc[i][1], __fmul_rn(f1, __fmul_rn(dwa, dx1)));
                    acc[i][2] = __fadd_rn(acc[i][2], __fmul_rn(f2, __fmul_rn(dwb, dx0)));
                    acc[i][3] = __fadd_rn(acc[i][3], __fmul_rn(f3, __fmul_rn(dwb, dx1)));
                }
            }
            if constexpr (!EARLY) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
            }
        }
        if (bad || nact == 0) continue;
        // epilogue: value v of tile i is (row ra + 8 (v >> 1) of group q, token 8 (n0 + i) + 2t + (v & 1))
#pragma unroll
        for (int i = 0; i < NTW; i++) {
            if (i >= nact) break;
            unsigned long long kk[2] = {0ull, 0ull};
#pragma unroll
            for (int v = 0; v < 4; v++) {
                const int tk = 8 * (n0 + i) + 2 * t + (v & 1);
                const int m = ps * TOK + tk;
                const int row = rt * 64 + q * 32 + ra + 8 * (v >> 1);
                if (tk < ntok) {
                    if (p.part) {
                        p.part[((size_t)sl * p.M + m) * p.N + row] = acc[i][v];
                    } else {
                        const size_t o = (size_t)m * p.ldy + row;
                        float val = acc[i][v];
                        if (p.resid) val = __fadd_rn(p.resid[o], val);
                        p.y[o] = val;
                        if (p.keys) {
                            const unsigned long long key = argmax_key(val, row);
                            kk[v & 1] = key > kk[v & 1] ? key : kk[v & 1];
                        }
                    }
                }
            }
            if (p.keys && !p.part) {
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    unsigned long long key = kk[h];
#pragma unroll
                    for (int o = 4; o < 32; o <<= 1) {
                        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
                        key = other > key ? other : key;
                    }
                    const int tk = 8 * (n0 + i) + 2 * t + h;
                    if (g == 0 && tk < ntok && key) atomicMax(&ckeys[ps * TOK + tk], key);
                }
            }
        }
    }
    if (p.keys && !p.part) {
        asm volatile("bar.sync 1, %0;" ::"n"(GS_CONS * 32));
        for (int i = threadIdx.x; i < p.M; i += GS_CONS * 32)
            if (ckeys[i]) atomicMax(p.keys + i, ckeys[i]);
    }
}

// tokens per pass of the streamed GEMM: 16 up to 16 tokens, else 32 (one or two passes)
static int gs_tok(int64_t m) { return m <= 16 ? 16 : 32; }

// K slices for the streamed GEMM: about four items per CTA (two CTAs per SM), so that the
// contiguous item ranges come out even, each slice at least 2 chunks of 256 bytes
static int gs_slices(lq_ctx* ctx, int64_t n, int64_t k, int64_t m) {
    const int64_t tok = gs_tok(m), tiles = n / 64, passes = (m + tok - 1) / tok;
    const int64_t items = tiles * passes, target = 8 * (int64_t)ctx->sm_count;
    if (items >= target || getenv("LQ_GEMM_NO_SPLIT")) return 1;
    int64_t s = (target + items - 1) / items;
    s = std::min<int64_t>(s, std::max<int64_t>(1, (k / GS_KC) / 2));
    return (int)std::max<int64_t>(1, std::min<int64_t>(s, 16));
}

static bool gs_supported(const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd, int64_t m) {
    return m >= 5 && m <= 64 && w->k % GS_KC == 0 && w->n % 64 == 0 && w->n < (1ll << 31) &&
           ((uintptr_t)w->qs % 16) == 0 && ((uintptr_t)w->d % 16) == 0 && ((uintptr_t)xq % 16) == 0 &&
           ((uintptr_t)xd % 16) == 0 && !getenv("LQ_NO_GEMM_STREAM");
}

template <int TOK>
static int launch_gemm_stream_t(lq_ctx* ctx, const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd,
                                int64_t m, float* y, const float* resid, int64_t ldy, unsigned long long* keys,
                                const SplitBuf* fixed) {
    using C = GsCfg<TOK>;
    GsParams p = {};
    p.N = (int)w->n;
    p.K = (int)w->k;
    p.M = (int)m;
    p.tiles = (int)(w->n / 64);
    p.passes = (int)((m + TOK - 1) / TOK);
    const int64_t chunks = w->k / GS_KC;
    int slices = gs_slices(ctx, w->n, w->k, m);
    p.kslice = (int)(((chunks + slices - 1) / slices) * GS_KC);
    p.slices = (int)((w->k + p.kslice - 1) / p.kslice);
    p.resid = resid;
    p.y = y;
    p.ldy = (int)ldy;
    p.keys = keys;
    p.err = ctx->err_flag;
    if (p.slices > 1) {
        const int rc = split_partials(ctx, fixed, (size_t)p.slices * m * w->n * 4, &p.part);
        if (rc) return rc;
    }
    CUtensorMap mw, mwd, mx, mxd;
    int rc = make_tensor_map_2d(ctx, &mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->qs, (uint64_t)w->k, (uint64_t)w->n,
                                (uint64_t)w->k, 128, 32, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!rc)
        rc = make_tensor_map_2d(ctx, &mwd, CU_TENSOR_MAP_DATA_TYPE_UINT16, w->d, (uint64_t)(w->k / 32),
                                (uint64_t)w->n, (uint64_t)(w->k / 32) * 2, 8, 32, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!rc)
        rc = make_tensor_map_2d(ctx, &mx, CU_TENSOR_MAP_DATA_TYPE_UINT8, xq, (uint64_t)w->k, (uint64_t)m,
                                (uint64_t)w->k, 128, TOK, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!rc)
        rc = make_tensor_map_2d(ctx, &mxd, CU_TENSOR_MAP_DATA_TYPE_UINT16, xd, (uint64_t)(w->k / 32), (uint64_t)m,
                                (uint64_t)(w->k / 32) * 2, 8, TOK, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    if ((rc = ensure_func_smem(ctx, (const void*)q8_gemm_stream_kernel<TOK>, C::SMEM))) return rc;
    const long long items = (long long)p.tiles * p.slices * p.passes;
    const int grid = (int)std::min<long long>(items, 2ll * ctx->sm_count);
    rc = launch_kernel(ctx, q8_gemm_stream_kernel<TOK>, dim3(grid), dim3(GS_THREADS), C::SMEM, "q8_gemm_stream", mw,
                       mwd, mx, mxd, p);
    if (rc || p.slices == 1) return rc;
    return launch_kernel(ctx, gemm_split_reduce_kernel, dim3((unsigned)ceil_div(w->n, 256), (unsigned)m), dim3(256), 0,
                         "gemm_split_reduce", (const float*)p.part, p.slices, (int)m, (int)w->n, resid, y, (int)ldy,
                         keys);
}

static int launch_gemm_stream(lq_ctx* ctx, const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd, int64_t m,
                              float* y, const float* resid, int64_t ldy, unsigned long long* keys,
                              const SplitBuf* fixed) {
    return gs_tok(m) == 16 ? launch_gemm_stream_t<16>(ctx, w, xq, xd, m, y, resid, ldy, keys, fixed)
                           : launch_gemm_stream_t<32>(ctx, w, xq, xd, m, y, resid, ldy, keys, fixed);
}

// =========================================================================================
// Skinny Q8_0 GEMM (5 <= m <= 8 tokens: decode batches), one CTA per SM, stream-K.
// A tile is 128 weight rows; a unit is one 256-byte K chunk of a tile (8 Q8_0 blocks). The
// tiles' units, in tile-major order, are dealt to the CTAs in equal contiguous ranges, so every
// SM streams the same number of weight bytes whatever the shape. One producer lane loads per
// unit the tile's two 128-byte column boxes (128 rows each, 128-byte swizzle), their fp16
// scales, the m token rows (8-row boxes; rows past m read as zeros) and the tokens' scales into
// a 6-stage ring of 37 KiB. Eight consumer warps each own 16 rows of the tile and all 8 tokens:
// one m16n8k32 MMA per Q8_0 block, its int32 dots turned into floats by the 1.5*2^23 bias the
// MMA accumulates onto, then scaled and added per (row, token) in ascending block order with
// separately rounded multiply and add (the oracle's order). A tile whose units all fall to one
// CTA is written directly: bit-identical to the oracle. A tile cut between CTAs leaves one
// partial sum per CTA in the partial buffer; the CTA that arrives last (a per-tile counter,
// indexed by the tile's first CTA and reset by that last CTA) adds them in CTA order and writes
// the tile, so the result is deterministic and within the regrouping bound. No CTA waits for
// another. LQ_GEMM_NO_SPLIT=1 deals whole tiles instead.
// =========================================================================================
constexpr int SK_ROWS = 128;
constexpr int SK_KC = 256;
constexpr int SK_CONS = 8;
constexpr int SK_THREADS = (SK_CONS + 1) * 32;
constexpr int SK_STAGES = 6;
constexpr int SK_WBOX = SK_ROWS * 128;                 // 128 rows x 128 bytes
constexpr int SK_XBOX = 8 * 128;                       // 8 token rows x 128 bytes
constexpr int SK_OFF_X = 2 * SK_WBOX;
constexpr int SK_OFF_WD = SK_OFF_X + 2 * SK_XBOX;      // weight scales [128][8] fp16
constexpr int SK_OFF_XD = SK_OFF_WD + SK_ROWS * 16;    // token scales [8][8] fp16
constexpr int SK_BYTES = SK_OFF_XD + 8 * 16;           // bytes landing per stage
constexpr int SK_STAGE = (SK_BYTES + 1023) / 1024 * 1024;
constexpr size_t SK_SMEM = (size_t)SK_STAGES * SK_STAGE + 1024 + 256;
static_assert(SK_SMEM <= 227 * 1024, "skinny GEMM ring exceeds the shared memory of one CTA");
static_assert(SK_OFF_X % 1024 == 0 && SK_XBOX % 1024 == 0, "swizzled boxes need 1024-byte alignment");

struct SkParams {
    int N, K, M;
    int tiles, chunks;            // 128-row tiles; 256-byte units per tile
    int whole;                    // 1: whole tiles per CTA (no split)
    int narrow;                   // 1: (units + 1) * grid < 2^32 (32-bit unit arithmetic)
    int early;                    // ring stages whose weights go out before pdl_wait (1..SK_STAGES)
    long long units;              // tiles * chunks
    const float* resid;
    float* y;
    int ldy;
    float4* part;                 // [grid][2 slots][256 consumer threads] partial sums
    unsigned* cnt;                // [grid] arrivals at the tile that starts in that CTA
    unsigned long long* keys;     // fused greedy argmax per token
    int* err;
};

// first unit of CTA b (32-bit division when units * grid fits 32 bits, as it does for every
// decode shape: it sits on the path to the first weight load)
__device__ __forceinline__ long long sk_start(const SkParams& p, int b) {
    if (p.narrow)
        return p.whole ? (long long)((unsigned)p.tiles * (unsigned)b / gridDim.x) * p.chunks
                       : (long long)((unsigned)p.units * (unsigned)b / gridDim.x);
    const long long G = gridDim.x;
    return p.whole ? (long long)p.tiles * b / G * p.chunks : p.units * b / G;
}
// the CTA whose range holds unit u (split mode)
__device__ __forceinline__ int sk_owner(const SkParams& p, long long u) {
    if (p.narrow) return (int)((((unsigned)u + 1u) * gridDim.x - 1u) / (unsigned)p.units);
    return (int)(((u + 1) * (long long)gridDim.x - 1) / p.units);
}
// tile of unit u
__device__ __forceinline__ int sk_tile(const SkParams& p, long long u) {
    return p.narrow ? (int)((unsigned)u / (unsigned)p.chunks) : (int)(u / p.chunks);
}

// ST ring stages, MINB CTAs per SM: (6, 1) by default; (3, 2) with LQ_SK_DUAL=1 (two CTAs per SM,
// sixteen consumer warps per SM, each CTA with a 3-stage ring)
template <int ST, int MINB>
__global__ void __launch_bounds__(SK_THREADS, MINB) q8_gemm_skinny_kernel(const __grid_constant__ CUtensorMap mw,
                                                                       const __grid_constant__ CUtensorMap mwd,
                                                                       const __grid_constant__ CUtensorMap mx,
                                                                       const __grid_constant__ CUtensorMap mxd,
                                                                       const SkParams p) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const uint32_t raw = smem_addr(smem_raw);
    uint8_t* sm = smem_raw + (((raw + 1023) & ~1023u) - raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + (size_t)ST * SK_STAGE);
    uint64_t* empty = full + ST;
    unsigned long long* ckeys = reinterpret_cast<unsigned long long*>(empty + ST);  // [8]
    int* last_flag = reinterpret_cast<int*>(ckeys + 8);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], SK_CONS);
        }
        mbar_fence_init();
    }
    if (threadIdx.x < 8) ckeys[threadIdx.x] = 0ull;
    __syncthreads();
    const int b = blockIdx.x;
    const long long u0 = sk_start(p, b), u1 = b + 1 == (int)gridDim.x ? p.units : sk_start(p, b + 1);

    if (warp == SK_CONS) {
        // ---------------- producer (one lane); weights may stream before pdl_wait ----------------
        if (lane != 0) return;
        tma_prefetch_map(&mw);
        tma_prefetch_map(&mwd);
        tma_prefetch_map(&mx);
        tma_prefetch_map(&mxd);
        int s = 0;
        unsigned ph = 0;
        // the activations come from the preceding kernel: until pdl_wait has returned, only the
        // weights of the first stages go out (the whole ring, while that kernel finishes), and
        // their activation boxes follow in one batch after the wait
        bool waited = false;
        int npend = 0;
        int pend_k[ST];
        auto load_x = [&](int stage, int k) {
            uint8_t* st = sm + (size_t)stage * SK_STAGE;
            tma_load_2d(st + SK_OFF_X, &mx, k, 0, &full[stage]);
            tma_load_2d(st + SK_OFF_X + SK_XBOX, &mx, k + 128, 0, &full[stage]);
            tma_load_2d(st + SK_OFF_XD, &mxd, k / 32, 0, &full[stage]);
        };
        auto flush = [&]() {
            pdl_wait();
            waited = true;
            for (int i = 0; i < npend; i++) load_x(i, pend_k[i]);  // stages 0 .. npend-1
            npend = 0;
        };
        for (long long u = u0; u < u1;) {
            const int t = sk_tile(p, u);
            const long long ts = (long long)t * p.chunks;
            const long long e = min(u1, ts + p.chunks);
            const int row = t * SK_ROWS;
            for (int c = (int)(u - ts); c < (int)(e - ts); c++) {
                if (!waited && npend == p.early) flush();
                if (!mbar_wait(&empty[s], ph ^ 1u)) {
                    atomicCAS(p.err, 0, 26);
                    if (!waited) pdl_wait();
                    return;
                }
                uint8_t* st = sm + (size_t)s * SK_STAGE;
                const int k = c * SK_KC;
                mbar_expect_tx(&full[s], (unsigned)SK_BYTES);
                tma_load_2d(st, &mw, k, row, &full[s]);
                tma_load_2d(st + SK_WBOX, &mw, k + 128, row, &full[s]);
                tma_load_2d(st + SK_OFF_WD, &mwd, k / 32, row, &full[s]);
                if (waited)
                    load_x(s, k);
                else
                    pend_k[npend++] = k;
                if (++s == ST) {
                    s = 0;
                    ph ^= 1u;
                }
            }
            u = e;
        }
        if (!waited) flush();
        return;
    }
    // ---------------- consumers ----------------
    pdl_wait();  // resid / y / keys / the partial buffer and counters belong to preceding kernels
    pdl_trigger();
    const int g = lane >> 2, t4 = lane & 3, tid = threadIdx.x;
    const int ra = 16 * warp + g;                        // rows ra and ra + 8 of the tile
    const int a_off = ra * 128 + (t4 & 1) * 8;
    const int b_off = SK_OFF_X + g * 128 + (t4 & 1) * 8;
    const int sc_off = SK_OFF_WD + ra * 16;
    const int xd_off = SK_OFF_XD + 2 * t4 * 16;
    int s = 0;
    unsigned ph = 0;
    bool bad = false;
    bool first_seg = true;
    for (long long u = u0; u < u1; first_seg = false) {
        const int t = sk_tile(p, u);
        const long long ts = (long long)t * p.chunks;
        const long long e = min(u1, ts + p.chunks);
        const int c0 = (int)(u - ts), c1 = (int)(e - ts);
        u = e;
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int c = c0; c < c1; c++) {
            const int cs = s;
            const unsigned cph = ph;
            if (++s == ST) {
                s = 0;
                ph ^= 1u;
            }
            if (bad) continue;
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&full[cs], cph);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                if (lane == 0) atomicCAS(p.err, 0, 27);
                bad = true;
                continue;
            }
            const uint8_t* st = sm + (size_t)cs * SK_STAGE;
            // the warp's whole slice of the stage into registers, then the stage is released
            uint2 wa[8], wb[8], xv[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int ch = ((2 * (j & 3) + (t4 >> 1)) ^ g) << 4;
                wa[j] = *reinterpret_cast<const uint2*>(st + (j >> 2) * SK_WBOX + a_off + ch);
                wb[j] = *reinterpret_cast<const uint2*>(st + (j >> 2) * SK_WBOX + a_off + 8 * 128 + ch);
                xv[j] = *reinterpret_cast<const uint2*>(st + b_off + (j >> 2) * SK_XBOX + ch);
            }
            const uint4 sa = *reinterpret_cast<const uint4*>(st + sc_off);
            const uint4 sb = *reinterpret_cast<const uint4*>(st + sc_off + 8 * 16);
            const uint4 ua = *reinterpret_cast<const uint4*>(st + xd_off);
            const uint4 ub = *reinterpret_cast<const uint4*>(st + xd_off + 16);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[cs]);
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const uint32_t a[4] = {wa[j].x, wb[j].x, wa[j].y, wb[j].y};
                const uint32_t bb[2] = {xv[j].x, xv[j].y};
                int d[4];
                mma_s8_bias(d, a, bb, 0x4B400000);
                const uint32_t wsa = j < 2 ? sa.x : j < 4 ? sa.y : j < 6 ? sa.z : sa.w;
                const uint32_t wsb = j < 2 ? sb.x : j < 4 ? sb.y : j < 6 ? sb.z : sb.w;
                const uint32_t wx0 = j < 2 ? ua.x : j < 4 ? ua.y : j < 6 ? ua.z : ua.w;
                const uint32_t wx1 = j < 2 ? ub.x : j < 4 ? ub.y : j < 6 ? ub.z : ub.w;
                const int sh = (j & 1) * 16;
                const float dwa = h2f((uint16_t)(wsa >> sh)), dwb = h2f((uint16_t)(wsb >> sh));
                const float dx0 = h2f((uint16_t)(wx0 >> sh)), dx1 = h2f((uint16_t)(wx1 >> sh));
                // the MMA added the dots to 1.5 * 2^23: one subtraction gives (float)dot exactly
                const float f0 = __fsub_rn(__int_as_float(d[0]), 12582912.0f);
                const float f1 = __fsub_rn(__int_as_float(d[1]), 12582912.0f);
                const float f2 = __fsub_rn(__int_as_float(d[2]), 12582912.0f);
                const float f3 = __fsub_rn(__int_as_float(d[3]), 12582912.0f);
                acc[0] = __fadd_rn(acc[0], __fmul_rn(f0, __fmul_rn(dwa, dx0)));
                acc[1] = __fadd_rn(acc[1], __fmul_rn(f1, __fmul_rn(dwa, dx1)));
                acc[2] = __fadd_rn(acc[2], __fmul_rn(f2, __fmul_rn(dwb, dx0)));
                acc[3] = __fadd_rn(acc[3], __fmul_rn(f3, __fmul_rn(dwb, dx1)));
            }
        }
        // ---- segment end: a whole tile is written; a cut tile goes through the partial buffer ----
        float v[4] = {acc[0], acc[1], acc[2], acc[3]};
        if (!(c0 == 0 && c1 == p.chunks)) {
            const int slot = first_seg ? 0 : 1;
            __stcg(p.part + ((size_t)b * 2 + slot) * (SK_CONS * 32) + tid, make_float4(v[0], v[1], v[2], v[3]));
            __threadfence();
            asm volatile("bar.sync 1, %0;" ::"n"(SK_CONS * 32));
            const int bf = sk_owner(p, ts), bl = sk_owner(p, ts + p.chunks - 1);
            if (tid == 0) {
                const unsigned old = atomicAdd(&p.cnt[bf], 1u);
                const int last = old == (unsigned)(bl - bf);
                if (last) p.cnt[bf] = 0u;  // every CTA of the tile has arrived: ready for the next launch
                *last_flag = last;
            }
            asm volatile("bar.sync 1, %0;" ::"n"(SK_CONS * 32));
            if (!*last_flag) continue;
            __threadfence();
            for (int q = bf; q <= bl; q++) {
                // the tile is the last range piece of its first CTA (slot 1 if that CTA began in
                // an earlier tile) and the first piece of every later CTA (slot 0)
                const int sl = (q == bf && sk_start(p, q) < ts) ? 1 : 0;
                float4 o;
                if (q == b) {
                    o = make_float4(acc[0], acc[1], acc[2], acc[3]);
                } else {
                    o = __ldcg(p.part + ((size_t)q * 2 + sl) * (SK_CONS * 32) + tid);
                }
                if (q == bf) {
                    v[0] = o.x, v[1] = o.y, v[2] = o.z, v[3] = o.w;
                } else {
                    v[0] = __fadd_rn(v[0], o.x), v[1] = __fadd_rn(v[1], o.y);
                    v[2] = __fadd_rn(v[2], o.z), v[3] = __fadd_rn(v[3], o.w);
                }
            }
        }
        if (bad) continue;
        // value i: row ra + 8 (i >> 1) of tile t, token 2 t4 + (i & 1)
        unsigned long long kk[2] = {0ull, 0ull};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int tk = 2 * t4 + (i & 1);
            const int row = t * SK_ROWS + ra + 8 * (i >> 1);
            if (tk < p.M && row < p.N) {
                const size_t o = (size_t)tk * p.ldy + row;
                float val = v[i];
                if (p.resid) val = __fadd_rn(p.resid[o], val);
                p.y[o] = val;
                if (p.keys) {
                    const unsigned long long key = argmax_key(val, row);
                    kk[i & 1] = key > kk[i & 1] ? key : kk[i & 1];
                }
            }
        }
        if (p.keys) {
#pragma unroll
            for (int h = 0; h < 2; h++) {
                unsigned long long key = kk[h];
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) {
                    const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
                    key = other > key ? other : key;
                }
                if (g == 0 && key) atomicMax(&ckeys[2 * t4 + h], key);
            }
        }
    }
    if (p.keys) {
        asm volatile("bar.sync 1, %0;" ::"n"(SK_CONS * 32));
        if (tid < p.M && ckeys[tid]) atomicMax(p.keys + tid, ckeys[tid]);
    }
}

static bool sk_supported(const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd, int64_t m) {
    return m >= 5 && m <= 8 && w->k % SK_KC == 0 && w->n % 8 == 0 && w->n < (1ll << 31) &&
           ((uintptr_t)w->qs % 16) == 0 && ((uintptr_t)w->d % 16) == 0 && ((uintptr_t)xq % 16) == 0 &&
           ((uintptr_t)xd % 16) == 0 && !getenv("LQ_NO_GEMM_SKINNY");
}

// CTAs of the skinny GEMM: one per SM, never more than the units (or tiles, unsplit)
// CTAs of the skinny GEMM: `per_sm` per SM, never more than the units (or tiles, unsplit)
static int sk_grid(lq_ctx* ctx, int64_t n, int64_t k, bool whole, int per_sm = 1) {
    const int64_t tiles = (n + SK_ROWS - 1) / SK_ROWS, units = tiles * (k / SK_KC);
    return (int)std::min<int64_t>(std::min<int64_t>((int64_t)per_sm * ctx->sm_count, kTileCounters),
                                  whole ? tiles : units);
}

// partial-sum bytes of either configuration (sized for two CTAs per SM)
static size_t sk_partial_bytes(lq_ctx* ctx, int64_t n, int64_t k) {
    if (k % SK_KC != 0 || n % 8 != 0) return 0;
    return (size_t)sk_grid(ctx, n, k, false, 2) * 2 * SK_CONS * 32 * sizeof(float4);
}

static int launch_gemm_skinny(lq_ctx* ctx, const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd, int64_t m,
                              float* y, const float* resid, int64_t ldy, unsigned long long* keys,
                              const SplitBuf* fixed) {
    SkParams p = {};
    p.N = (int)w->n;
    p.K = (int)w->k;
    p.M = (int)m;
    p.tiles = (int)((w->n + SK_ROWS - 1) / SK_ROWS);
    p.chunks = (int)(w->k / SK_KC);
    p.units = (long long)p.tiles * p.chunks;
    p.whole = getenv("LQ_GEMM_NO_SPLIT") ? 1 : 0;
    const bool dual = getenv("LQ_SK_DUAL") != nullptr;
    const int stages = dual ? 3 : SK_STAGES;
    const int grid = sk_grid(ctx, w->n, w->k, p.whole != 0, dual ? 2 : 1);
    p.narrow = (uint64_t)(p.units + 1) * (uint64_t)grid < (1ull << 32) ? 1 : 0;
    p.early = stages;
    if (const char* e = getenv("LQ_SK_EARLY")) p.early = std::max(1, std::min(stages, atoi(e)));
    p.resid = resid;
    p.y = y;
    p.ldy = (int)ldy;
    p.keys = keys;
    p.cnt = ctx->tile_cnt;
    p.err = ctx->err_flag;
    float* part = nullptr;
    int rc = split_partials(ctx, fixed, (size_t)grid * 2 * SK_CONS * 32 * sizeof(float4), &part);
    if (rc) return rc;
    p.part = reinterpret_cast<float4*>(part);
    CUtensorMap mw, mwd, mx, mxd;
    rc = make_tensor_map_2d(ctx, &mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->qs, (uint64_t)w->k, (uint64_t)w->n,
                            (uint64_t)w->k, 128, SK_ROWS, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!rc)
        rc = make_tensor_map_2d(ctx, &mwd, CU_TENSOR_MAP_DATA_TYPE_UINT16, w->d, (uint64_t)(w->k / 32),
                                (uint64_t)w->n, (uint64_t)(w->k / 32) * 2, 8, SK_ROWS, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!rc)
        rc = make_tensor_map_2d(ctx, &mx, CU_TENSOR_MAP_DATA_TYPE_UINT8, xq, (uint64_t)w->k, (uint64_t)m,
                                (uint64_t)w->k, 128, 8, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!rc)
        rc = make_tensor_map_2d(ctx, &mxd, CU_TENSOR_MAP_DATA_TYPE_UINT16, xd, (uint64_t)(w->k / 32), (uint64_t)m,
                                (uint64_t)(w->k / 32) * 2, 8, 8, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    if (dual) {
        const size_t smem = (size_t)3 * SK_STAGE + 1024 + 256;
        if ((rc = ensure_func_smem(ctx, (const void*)q8_gemm_skinny_kernel<3, 2>, smem))) return rc;
        return launch_kernel(ctx, q8_gemm_skinny_kernel<3, 2>, dim3(grid), dim3(SK_THREADS), smem, "q8_gemm_skinny",
                             mw, mwd, mx, mxd, p);
    }
    if ((rc = ensure_func_smem(ctx, (const void*)q8_gemm_skinny_kernel<SK_STAGES, 1>, SK_SMEM))) return rc;
    return launch_kernel(ctx, q8_gemm_skinny_kernel<SK_STAGES, 1>, dim3(grid), dim3(SK_THREADS), SK_SMEM,
                         "q8_gemm_skinny", mw, mwd, mx, mxd, p);
}

int launch_q8_matmul(lq_ctx* ctx, const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd,
                     int64_t m, float* y, const float* resid, int64_t ldy,
                     unsigned long long* keys, const SplitBuf* split) {
    if (m <= 0 || w->n <= 0) return LQ_OK;
    if (m <= 4 && gemv_stream_supported(w->k) && ((uintptr_t)xq % 16) == 0 && ((uintptr_t)xd % 16) == 0 &&
        gemv_stream_smem(m, w->k) <= 227 * 1024)
        return launch_gemv_stream(ctx, w, xq, xd, m, y, resid, ldy, keys);
    switch (m) {
        case 1: return gemv_rows<1>(ctx, w, xq, xd, y, resid, ldy, keys);
        case 2: return gemv_rows<2>(ctx, w, xq, xd, y, resid, ldy, keys);
        case 3: return gemv_rows<3>(ctx, w, xq, xd, y, resid, ldy, keys);
        case 4: return gemv_rows<4>(ctx, w, xq, xd, y, resid, ldy, keys);
        default: break;
    }
    if (!keys && m > 64 && gemm_tc_supported(m, w->k, w->qs, xq, w->d, xd))
        return launch_gemm_tc(ctx, w, xq, xd, m, y, resid, ldy);
    if (sk_supported(w, xq, xd, m)) return launch_gemm_skinny(ctx, w, xq, xd, m, y, resid, ldy, keys, split);
    if (gs_supported(w, xq, xd, m)) return launch_gemm_stream(ctx, w, xq, xd, m, y, resid, ldy, keys, split);
    if (m <= 16) return run_gemm<128, 16, 8, 1>(ctx, w, xq, xd, m, y, resid, ldy, keys, split);
    if (m <= 32) return run_gemm<128, 32, 8, 1>(ctx, w, xq, xd, m, y, resid, ldy, keys, split);
    if (m <= 64) return run_gemm<128, 64, 4, 2>(ctx, w, xq, xd, m, y, resid, ldy, keys, split);
    return run_gemm<128, 128, 4, 2>(ctx, w, xq, xd, m, y, resid, ldy, keys, split);
}

// =========================================================================================
// seeded generator fill
// =========================================================================================
__global__ void fill_bf16_kernel(uint64_t key, int64_t offset, int64_t count, float scale,
                                 uint16_t* __restrict__ out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = f32_to_bf16(gen_value(key, (uint64_t)(offset + i), scale));
}

// rows x cols slice of a [*][src_ld] generated tensor starting at (row0, col0)
__global__ void fill_bf16_2d_kernel(uint64_t key, int64_t rows, int64_t cols, int64_t src_ld, int64_t row0,
                                    int64_t col0, float scale, uint16_t* __restrict__ out) {
    const int64_t count = rows * cols;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / cols, c = i - (i / cols) * cols;
        out[i] = f32_to_bf16(gen_value(key, (uint64_t)((row0 + r) * src_ld + col0 + c), scale));
    }
}

__global__ void fill_norm_kernel(uint64_t key, int64_t count, float scale, int unit,
                                 uint16_t* __restrict__ out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = unit ? (uint16_t)0x3F80 : f32_to_bf16(__fadd_rn(1.0f, gen_value(key, (uint64_t)i, scale)));
}

int launch_fill_bf16(lq_ctx* ctx, uint64_t seed, uint64_t tid, int64_t offset, int64_t count,
                     float scale, uint16_t* out) {
    if (count <= 0) return LQ_OK;
    int grid = (int)std::min<int64_t>((count + 255) / 256, (int64_t)ctx->sm_count * 32);
    fill_bf16_kernel<<<grid, 256, 0, ctx->stream>>>(gen_key(seed, tid), offset, count, scale, out);
    LQ_LAUNCH_CHECK(ctx, "fill_bf16");
    return LQ_OK;
}

int launch_fill_bf16_2d(lq_ctx* ctx, uint64_t seed, uint64_t tid, int64_t rows, int64_t cols, int64_t src_ld,
                        int64_t row0, int64_t col0, float scale, uint16_t* out) {
    const int64_t count = rows * cols;
    if (count <= 0) return LQ_OK;
    int grid = (int)std::min<int64_t>((count + 255) / 256, (int64_t)ctx->sm_count * 32);
    fill_bf16_2d_kernel<<<grid, 256, 0, ctx->stream>>>(gen_key(seed, tid), rows, cols, src_ld, row0, col0, scale, out);
    LQ_LAUNCH_CHECK(ctx, "fill_bf16_2d");
    return LQ_OK;
}

int launch_fill_norm(lq_ctx* ctx, uint64_t seed, uint64_t tid, int64_t count, float norm_std,
                     uint16_t* out) {
    if (count <= 0) return LQ_OK;
    int grid = (int)std::min<int64_t>((count + 255) / 256, 1024);
    fill_norm_kernel<<<grid, 256, 0, ctx->stream>>>(gen_key(seed, tid), count, gen_scale(norm_std),
                                                    norm_std == 0.0f, out);
    LQ_LAUNCH_CHECK(ctx, "fill_norm");
    return LQ_OK;
}

}  // namespace lq

// =========================================================================================
// C ABI
// =========================================================================================
extern "C" {

static int check_q8_tensor(lq_ctx* ctx, const lq_q8_tensor* w, const char* what) {
    LQ_REQUIRE(ctx, w != nullptr, "%s: weight is NULL", what);
    LQ_REQUIRE(ctx, w->n > 0 && w->k > 0 && w->k % 32 == 0,
               "%s: weight shape [%lld, %lld] invalid (k must be a positive multiple of 32)",
               what, (long long)w->n, (long long)w->k);
    LQ_REQUIRE(ctx, w->n < (1ll << 31) && w->k < (1ll << 31) && w->n * w->k < (1ll << 40),
               "%s: weight too large", what);
    LQ_REQUIRE(ctx, w->qs && w->d, "%s: weight buffers are NULL", what);
    return LQ_OK;
}

int lq_q8_0_quantize(lq_ctx* ctx, const void* src, lq_dtype dt, int64_t rows, int64_t k,
                     int8_t* qs, uint16_t* d) {
    LQ_ENTRY(ctx, "lq_q8_0_quantize");
    LQ_REQUIRE(ctx, dt == LQ_DTYPE_F32 || dt == LQ_DTYPE_BF16,
               "lq_q8_0_quantize: source dtype must be F32 or BF16");
    LQ_REQUIRE(ctx, rows >= 0 && k >= 0 && k % 32 == 0,
               "lq_q8_0_quantize: k=%lld must be a multiple of 32", (long long)k);
    if (rows == 0 || k == 0) return LQ_OK;
    LQ_REQUIRE(ctx, src && qs && d, "lq_q8_0_quantize: NULL pointer");
    return lq::launch_quantize_rows(ctx, src, dt, rows, k, qs, d);
}

// GGML's quantize_row_q8_0_ref on the host, one block at a time: amax, d = amax/127 (IEEE f32
// divide), id = d ? 1/d : 0, q = round-half-away(x*id) (|x*id| <= 127 by construction, clamped
// anyway as the device does), d stored as fp16 (round to nearest even). bf16 inputs are widened
// exactly. Same bits as lq_q8_0_quantize.
int lq_q8_0_quantize_host(const void* src, lq_dtype dt, int64_t rows, int64_t k, int8_t* qs, uint16_t* d) {
    if (lq::fault_injected("lq_q8_0_quantize_host"))
        return lq::set_error(nullptr, LQ_ERR_INJECTED, "lq_q8_0_quantize_host: injected fault (LQ_FAULT)");
    if (dt != LQ_DTYPE_F32 && dt != LQ_DTYPE_BF16)
        return lq::set_error(nullptr, LQ_ERR_INVALID_ARG, "lq_q8_0_quantize_host: source dtype must be F32 or BF16");
    if (rows < 0 || k < 0 || k % 32 != 0)
        return lq::set_error(nullptr, LQ_ERR_INVALID_ARG, "lq_q8_0_quantize_host: k=%lld must be a multiple of 32",
                             (long long)k);
    if (rows == 0 || k == 0) return LQ_OK;
    if (!src || !qs || !d) return lq::set_error(nullptr, LQ_ERR_INVALID_ARG, "lq_q8_0_quantize_host: NULL pointer");
    const float* sf = static_cast<const float*>(src);
    const uint16_t* sb = static_cast<const uint16_t*>(src);
    const int64_t nb = k / 32;
    for (int64_t r = 0; r < rows; r++)
        for (int64_t b = 0; b < nb; b++) {
            const int64_t e0 = r * k + b * 32;
            float x[32];
            float amax = 0.0f;
            for (int i = 0; i < 32; i++) {
                x[i] = dt == LQ_DTYPE_F32 ? sf[e0 + i] : lq::bf16_to_f32(sb[e0 + i]);
                amax = std::max(amax, std::fabs(x[i]));
            }
            const float dd = amax / 127.0f;
            const float id = dd != 0.0f ? 1.0f / dd : 0.0f;
            for (int i = 0; i < 32; i++) {
                float q = std::round(x[i] * id);
                q = std::min(std::max(q, -127.0f), 127.0f);
                qs[e0 + i] = (int8_t)(int)q;
            }
            const __half h = __float2half_rn(dd);
            uint16_t hb;
            memcpy(&hb, &h, 2);
            d[r * nb + b] = hb;
        }
    return LQ_OK;
}

int lq_q8_0_pack_blocks(lq_ctx* ctx, const int8_t* qs, const uint16_t* d, int64_t rows, int64_t k,
                        uint8_t* blocks) {
    LQ_ENTRY(ctx, "lq_q8_0_pack_blocks");
    LQ_REQUIRE(ctx, rows >= 0 && k >= 0 && k % 32 == 0, "lq_q8_0_pack_blocks: k must be a multiple of 32");
    int64_t nb = rows * (k / 32);
    if (nb == 0) return LQ_OK;
    LQ_REQUIRE(ctx, qs && d && blocks, "lq_q8_0_pack_blocks: NULL pointer");
    int64_t bytes = nb * 34;
    lq::pack_blocks_kernel<<<(int)((bytes + 255) / 256), 256, 0, ctx->stream>>>(qs, d, nb, blocks);
    LQ_LAUNCH_CHECK(ctx, "pack_blocks");
    return LQ_OK;
}

int lq_q8_0_unpack_blocks(lq_ctx* ctx, const uint8_t* blocks, int64_t rows, int64_t k, int8_t* qs,
                          uint16_t* d) {
    LQ_ENTRY(ctx, "lq_q8_0_unpack_blocks");
    LQ_REQUIRE(ctx, rows >= 0 && k >= 0 && k % 32 == 0, "lq_q8_0_unpack_blocks: k must be a multiple of 32");
    int64_t nb = rows * (k / 32);
    if (nb == 0) return LQ_OK;
    LQ_REQUIRE(ctx, qs && d && blocks, "lq_q8_0_unpack_blocks: NULL pointer");
    int64_t bytes = nb * 34;
    lq::unpack_blocks_kernel<<<(int)((bytes + 255) / 256), 256, 0, ctx->stream>>>(blocks, nb, qs, d);
    LQ_LAUNCH_CHECK(ctx, "unpack_blocks");
    return LQ_OK;
}

int lq_q8_0_matmul(lq_ctx* ctx, const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd,
                   int64_t m, float* y, const float* resid, int64_t ldy) {
    LQ_ENTRY(ctx, "lq_q8_0_matmul");
    int rc = check_q8_tensor(ctx, w, "lq_q8_0_matmul");
    if (rc) return rc;
    LQ_REQUIRE(ctx, m >= 0 && m < (1 << 24), "lq_q8_0_matmul: m=%lld out of range", (long long)m);
    if (ldy == 0) ldy = w->n;
    LQ_REQUIRE(ctx, ldy >= w->n, "lq_q8_0_matmul: ldy < n");
    if (m == 0) return LQ_OK;
    LQ_REQUIRE(ctx, xq && xd && y, "lq_q8_0_matmul: NULL pointer");
    return lq::launch_q8_matmul(ctx, w, xq, xd, m, y, resid, ldy, nullptr);
}

int lq_q8_0_linear(lq_ctx* ctx, const lq_q8_tensor* w, const void* x, lq_dtype dt, int64_t m,
                   float* y) {
    LQ_ENTRY(ctx, "lq_q8_0_linear");
    int rc = check_q8_tensor(ctx, w, "lq_q8_0_linear");
    if (rc) return rc;
    LQ_REQUIRE(ctx, dt == LQ_DTYPE_F32 || dt == LQ_DTYPE_BF16, "lq_q8_0_linear: x dtype must be F32 or BF16");
    LQ_REQUIRE(ctx, m >= 0 && m < (1 << 24), "lq_q8_0_linear: m=%lld out of range", (long long)m);
    if (m == 0) return LQ_OK;
    LQ_REQUIRE(ctx, x && y, "lq_q8_0_linear: NULL pointer");
    size_t qbytes = (size_t)(m * w->k);
    size_t off = (qbytes + 255) & ~(size_t)255;
    size_t dbytes = (size_t)(m * (w->k / 32)) * 2;
    rc = lq::ensure_scratch(ctx, off + dbytes);
    if (rc) return rc;
    int8_t* xq = (int8_t*)ctx->scratch;
    uint16_t* xd = (uint16_t*)((uint8_t*)ctx->scratch + off);
    rc = lq::launch_quantize_rows(ctx, x, dt, m, w->k, xq, xd);
    if (rc) return rc;
    return lq::launch_q8_matmul(ctx, w, xq, xd, m, y, nullptr, w->n, nullptr);
}

int lq_fill_bf16(lq_ctx* ctx, uint64_t seed, uint64_t tid, int64_t offset, int64_t count, double std_dev,
                 uint16_t* out) {
    LQ_ENTRY(ctx, "lq_fill_bf16");
    LQ_REQUIRE(ctx, count >= 0 && offset >= 0, "lq_fill_bf16: negative size");
    if (count == 0) return LQ_OK;
    LQ_REQUIRE(ctx, out != nullptr, "lq_fill_bf16: NULL pointer");
    return lq::launch_fill_bf16(ctx, seed, tid, offset, count, lq::gen_scale(std_dev), out);
}

}  // extern "C"

// =========================================================================================
// lq_q8_0_linear_noalloc: lq_q8_0_linear for callers that must not allocate device memory.
//
// lq_q8_0_linear quantizes x into context scratch that it grows with cudaMalloc (and frees
// the old buffer with cudaFree) when a call needs more, and the small-M GEMM it dispatches to
// keeps its K-split partial sums in a second context buffer grown the same way. Some callers
// cannot allow that: a decode loop with a latency budget (both calls may synchronise the whole
// device), or a host that has handed all device memory to its own pool and forbids
// allocations behind its back. This variant keeps both in one fixed array in the library's
// device image instead, so it allocates nothing. The array is 4 MiB on every GPU that loads
// the library, held until the process exits. A call needs, each part rounded up to 256 bytes:
// m*k bytes of quantized rows, m*(k/32)*2 bytes of their scales, and for 5..64 rows on a
// weight with few row tiles the GEMM's K-split partials (slices*m*n*4 bytes, the amount
// lq::gemm_split_bytes reports); calls that need more than the array fail with
// LQ_ERR_INVALID_ARG. The kernels and their order are lq_q8_0_linear's, so the output is
// bit-identical to it.
// =========================================================================================
#include <mutex>

namespace {
constexpr size_t kNoAllocScratchBytes = (size_t)4 << 20;
// host code only ever uses the device address obtained from cudaGetSymbolAddress below; the
// name itself is a host-side stand-in
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
constexpr int kMaxDevices = 128;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};

// device address of the fixed scratch on ctx->device, looked up once per device with that
// device current
int noalloc_scratch(lq_ctx* ctx, void** out) {
    if (ctx->device < 0 || ctx->device >= kMaxDevices)
        return lq::set_error(ctx, LQ_ERR_UNSUPPORTED, "lq_q8_0_linear_noalloc: device %d", ctx->device);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[ctx->device]) {
        int prev = 0;
        LQ_CUDA(ctx, cudaGetDevice(&prev));
        if (prev != ctx->device) LQ_CUDA(ctx, cudaSetDevice(ctx->device));
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (prev != ctx->device) cudaSetDevice(prev);
        if (e != cudaSuccess) return lq::check_cuda(ctx, e, "cudaGetSymbolAddress(g_noalloc_scratch)");
        g_noalloc_addr[ctx->device] = p;
    }
    *out = g_noalloc_addr[ctx->device];
    return LQ_OK;
}

inline size_t al256(size_t b) { return (b + 255) & ~(size_t)255; }
}  // namespace

extern "C" int lq_q8_0_linear_noalloc(lq_ctx* ctx, const lq_q8_tensor* w, const void* x, lq_dtype dt, int64_t m,
                                      float* y) {
    LQ_ENTRY(ctx, "lq_q8_0_linear_noalloc");
    int rc = check_q8_tensor(ctx, w, "lq_q8_0_linear_noalloc");
    if (rc) return rc;
    LQ_REQUIRE(ctx, dt == LQ_DTYPE_F32 || dt == LQ_DTYPE_BF16,
               "lq_q8_0_linear_noalloc: x dtype must be F32 or BF16");
    LQ_REQUIRE(ctx, m >= 0 && m < (1 << 24), "lq_q8_0_linear_noalloc: m=%lld out of range", (long long)m);
    if (m == 0) return LQ_OK;
    LQ_REQUIRE(ctx, x && y, "lq_q8_0_linear_noalloc: NULL pointer");
    const size_t q_bytes = al256((size_t)(m * w->k));
    const size_t d_bytes = al256((size_t)(m * (w->k / 32)) * 2);
    const size_t split_bytes = al256(lq::gemm_split_bytes(ctx, w->n, w->k, m));
    const size_t need = q_bytes + d_bytes + split_bytes;
    LQ_REQUIRE(ctx, need <= kNoAllocScratchBytes,
               "lq_q8_0_linear_noalloc: m=%lld, n=%lld, k=%lld needs %zu bytes of scratch; the fixed scratch holds "
               "%zu (use lq_q8_0_linear, or split the rows)",
               (long long)m, (long long)w->n, (long long)w->k, need, kNoAllocScratchBytes);
    void* scratch = nullptr;
    rc = noalloc_scratch(ctx, &scratch);
    if (rc) return rc;
    // every byte the matmul reads is written first in the same call (the quantized rows by the
    // quantization, each K-split partial by its slice before the reduce): nothing to clear
    int8_t* xq = (int8_t*)scratch;
    uint16_t* xd = (uint16_t*)((uint8_t*)scratch + q_bytes);
    lq::SplitBuf split = {reinterpret_cast<float*>((uint8_t*)scratch + q_bytes + d_bytes), split_bytes};
    rc = lq::launch_quantize_rows(ctx, x, dt, m, w->k, xq, xd);
    if (rc) return rc;
    return lq::launch_q8_matmul(ctx, w, xq, xd, m, y, nullptr, w->n, nullptr, &split);
}
