// lq8_gemv.cu -- decode GEMV for M <= 4 tokens: y[m][n] = sum_b sumi_b * (d_w * d_x).
//
// HBM-bound: each launch streams N*K*34/32 bytes of Q8_0 weights once. The kernel is
// persistent (two CTAs per SM). In each CTA one producer warp streams weight tiles -- 8 rows
// x up to 2 KiB of K, plus their fp16 scales -- into a 4-stage shared-memory ring with 1-D
// bulk async copies (cp.async.bulk, completion counted on an mbarrier); 8 consumer warps take
// one row each, dp4a the int8 blocks against the activations (read through L1) and release
// the stage. So 2 x 4 x 17 KiB per SM are in flight at all times.
//
// The weights do not depend on earlier kernels, so the producer starts streaming before
// pdl_wait(): under programmatic dependent launch the first tiles arrive while the preceding
// kernel (a norm, attention) is still finishing. Consumers wait for it before reading x.
//
// Per output the block terms are accumulated per lane and combined by a butterfly over the
// warp, so the f32 summation order differs from the oracle's sequential order (bounded
// reordering error).
#include "lq8_async.cuh"
#include "lq8_internal.cuh"

namespace lq {

constexpr int GV_ROWS = 8;        // weight rows per tile (one per consumer warp)
constexpr int GV_KC = 2048;       // K bytes per tile
constexpr int GV_STAGES = 4;
constexpr int GV_CONSUMERS = 8;
constexpr int GV_THREADS = (GV_CONSUMERS + 1) * 32;
constexpr int GV_CTAS_PER_SM = 2;

struct GvSmem {
    int8_t w[GV_STAGES][GV_ROWS * GV_KC];
    uint16_t d[GV_STAGES][GV_ROWS * GV_KC / 32];
    uint64_t full[GV_STAGES];
    uint64_t empty[GV_STAGES];
    unsigned long long keys[4];
};

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(GV_CONSUMERS * 32)); }

template <int M>
__global__ void __launch_bounds__(GV_THREADS)
q8_gemv_stream_kernel(const int8_t* __restrict__ wq, const uint16_t* __restrict__ wd, int N, int K,
                      const int8_t* __restrict__ xq, const uint16_t* __restrict__ xd, const float* resid,
                      float* y, int ldy, unsigned long long* argmax_keys, int* err) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    GvSmem& S = *reinterpret_cast<GvSmem*>(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = K >> 5;
    const int kc = K < GV_KC ? K : GV_KC;          // chunk bytes (row stride inside a stage)
    const int nchunks = (K + kc - 1) / kc;
    const int nrg = (N + GV_ROWS - 1) / GV_ROWS;

    if (threadIdx.x == 0) {
        for (int s = 0; s < GV_STAGES; s++) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], GV_CONSUMERS);
        }
        mbar_fence_init();
    }
    if (threadIdx.x < 4) S.keys[threadIdx.x] = 0ull;
    __syncthreads();

    if (warp == GV_CONSUMERS) {
        // ---------------- producer: weights only, so it may run ahead of pdl_wait ----------
        if (lane == 0) {
            int it = 0;
            for (int rg = blockIdx.x; rg < nrg; rg += gridDim.x) {
                const int r0 = rg * GV_ROWS;
                const int rows = min(GV_ROWS, N - r0);
                for (int c = 0; c < nchunks; c++, it++) {
                    const int s = it % GV_STAGES;
                    const unsigned ph = (unsigned)(it / GV_STAGES) & 1u;
                    if (!mbar_wait(&S.empty[s], ph ^ 1u)) {
                        atomicCAS(err, 0, 3);
                        return;
                    }
                    const int k0 = c * kc;
                    const int sz = min(kc, K - k0);
                    const unsigned bytes = (unsigned)(rows * sz + rows * (sz / 32) * 2);
                    mbar_expect_tx(&S.full[s], bytes);
                    if (sz == K) {  // whole rows: the tile is contiguous in HBM
                        bulk_g2s(S.w[s], wq + (size_t)r0 * K, (unsigned)(rows * K), &S.full[s]);
                        bulk_g2s(S.d[s], wd + (size_t)r0 * nb, (unsigned)(rows * nb * 2), &S.full[s]);
                    } else {
                        for (int r = 0; r < rows; r++) {
                            bulk_g2s(S.w[s] + r * kc, wq + (size_t)(r0 + r) * K + k0, (unsigned)sz, &S.full[s]);
                            bulk_g2s(S.d[s] + r * (kc / 32), wd + (size_t)(r0 + r) * nb + k0 / 32,
                                     (unsigned)(sz / 16), &S.full[s]);
                        }
                    }
                }
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    pdl_wait();     // x and y belong to the preceding kernels
    pdl_trigger();
    float acc[M];
#pragma unroll
    for (int m = 0; m < M; m++) acc[m] = 0.0f;
    int it = 0;
    bool ok = true;
    for (int rg = blockIdx.x; rg < nrg && ok; rg += gridDim.x) {
        const int r0 = rg * GV_ROWS;
        const int rows = min(GV_ROWS, N - r0);
        for (int c = 0; c < nchunks; c++, it++) {
            const int s = it % GV_STAGES;
            const unsigned ph = (unsigned)(it / GV_STAGES) & 1u;
            if (!mbar_wait(&S.full[s], ph)) {
                if (lane == 0) atomicCAS(err, 0, 4);
                ok = false;
                break;
            }
            const int k0 = c * kc;
            const int sz = min(kc, K - k0);
            if (warp < rows) {
                const int8_t* wrow = S.w[s] + warp * kc;
                const uint16_t* drow = S.d[s] + warp * (kc / 32);
                const int nbc = sz >> 5;
                for (int b = lane; b < nbc; b += 32) {
                    const int4 w0 = *reinterpret_cast<const int4*>(wrow + b * 32);
                    const int4 w1 = *reinterpret_cast<const int4*>(wrow + b * 32 + 16);
                    const float dw = h2f(drow[b]);
                    const int gb = (k0 >> 5) + b;
#pragma unroll
                    for (int m = 0; m < M; m++) {
                        const int4* xp = reinterpret_cast<const int4*>(xq + (size_t)m * K + (size_t)gb * 32);
                        const int4 x0 = __ldg(xp), x1 = __ldg(xp + 1);
                        int sum = 0;
                        sum = __dp4a(w0.x, x0.x, sum); sum = __dp4a(w0.y, x0.y, sum);
                        sum = __dp4a(w0.z, x0.z, sum); sum = __dp4a(w0.w, x0.w, sum);
                        sum = __dp4a(w1.x, x1.x, sum); sum = __dp4a(w1.y, x1.y, sum);
                        sum = __dp4a(w1.z, x1.z, sum); sum = __dp4a(w1.w, x1.w, sum);
                        const float sc = __fmul_rn(dw, h2f(xd[(size_t)m * nb + gb]));
                        acc[m] = __fadd_rn(acc[m], __fmul_rn((float)sum, sc));
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.empty[s]);
            if (c == nchunks - 1) {
                const int row = r0 + warp;
#pragma unroll
                for (int m = 0; m < M; m++) {
                    const float v = warp_sum(acc[m]);
                    acc[m] = 0.0f;
                    if (warp < rows) {
                        if (lane == m) {
                            const size_t o = (size_t)m * ldy + row;
                            y[o] = resid ? __fadd_rn(resid[o], v) : v;
                        }
                        if (argmax_keys && lane == 0) atomicMax(&S.keys[m], argmax_key(v, row));
                    }
                }
            }
        }
    }
    if (argmax_keys) {
        consumer_sync();
        if (threadIdx.x < M && S.keys[threadIdx.x]) atomicMax(argmax_keys + threadIdx.x, S.keys[threadIdx.x]);
    }
}

bool gemv_stream_supported(int64_t K) { return K % 256 == 0; }

template <int M>
static int run_stream(lq_ctx* ctx, const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd, float* y,
                      const float* resid, int64_t ldy, unsigned long long* keys) {
    static bool attr = false;
    if (!attr) {
        LQ_CUDA(ctx, cudaFuncSetAttribute(q8_gemv_stream_kernel<M>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)sizeof(GvSmem)));
        attr = true;
    }
    const int nrg = ceil_div(w->n, GV_ROWS);
    const int grid = std::min(nrg, ctx->sm_count * GV_CTAS_PER_SM);
    return launch_kernel(ctx, q8_gemv_stream_kernel<M>, dim3(grid), dim3(GV_THREADS), sizeof(GvSmem),
                         "q8_gemv_stream", w->qs, w->d, (int)w->n, (int)w->k, xq, xd, resid, y, (int)ldy, keys,
                         ctx->err_flag);
}

int launch_gemv_stream(lq_ctx* ctx, const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd, int64_t m,
                       float* y, const float* resid, int64_t ldy, unsigned long long* keys) {
    switch (m) {
        case 1: return run_stream<1>(ctx, w, xq, xd, y, resid, ldy, keys);
        case 2: return run_stream<2>(ctx, w, xq, xd, y, resid, ldy, keys);
        case 3: return run_stream<3>(ctx, w, xq, xd, y, resid, ldy, keys);
        case 4: return run_stream<4>(ctx, w, xq, xd, y, resid, ldy, keys);
        default: return set_error(ctx, LQ_ERR_INVALID_ARG, "gemv_stream: m=%lld > 4", (long long)m);
    }
}

}  // namespace lq
