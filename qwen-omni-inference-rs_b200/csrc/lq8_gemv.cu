// lq8_gemv.cu -- decode GEMV for M <= 4 tokens: y[m][n] = sum_b sumi_b * (d_w * d_x), with
// the op that produces its input fused in as a prologue.
//
// HBM-bound: each launch streams N*K*34/32 bytes of Q8_0 weights once. The kernel is
// persistent. In each CTA one producer warp streams weight tiles -- 8 rows x up to 2 KiB of K
// plus their fp16 scales, 17 KiB -- into a STAGES-deep shared-memory ring with 1-D bulk async
// copies (cp.async.bulk, completion counted on an mbarrier); 8 consumer warps take one row
// each, move their slice of the stage into registers, release the stage at once, and dp4a
// the int8 blocks against the activations held in shared memory.
//
// The weights do not depend on earlier kernels, so the producer starts streaming before
// pdl_wait(): under programmatic dependent launch the first tiles land while the preceding
// kernel finishes. Meanwhile the consumers build the Q8_0 activations in shared memory:
//   PRO_COPY  copy pre-quantized activations (xq, xd)
//   PRO_NORM  RMSNorm of the f32 residual rows + Q8_0 (input/post-attention/final norm)
//   PRO_QUANT Q8_0 of f32 rows (the MLP's h = silu(gate)*up for the down projection)
// with the same row functions as the standalone kernels (bit-identical). Epilogue: y, or
// y = residual + acc (y may alias the residual), and/or the LM head's fused greedy argmax;
// or, for the fused gate|up weight, h = silu(gate) * up (each CTA walks gate rows and the
// matching up rows as one unit).
//
// Stage layout (bytes): weights [8][cw] then scales [8][cw/32] fp16, cw = the chunk width.
//
// Per output the block terms are accumulated per lane and combined by a butterfly over the
// warp, so the f32 summation order differs from the oracle's sequential order (bounded
// reordering error).
#include "lq8_async.cuh"
#include "lq8_fused.cuh"
#include "lq8_internal.cuh"

#include <cstdlib>

namespace lq {

constexpr int GV_ROWS = 8;        // weight rows per tile (one per consumer warp)
constexpr int GV_KC = 2048;       // K bytes per tile
constexpr int GV_STAGE_BYTES = GV_ROWS * GV_KC + GV_ROWS * (GV_KC / 32) * 2;  // 17 KiB
constexpr int GV_CONSUMERS = 8;
constexpr int GV_CTHREADS = GV_CONSUMERS * 32;
constexpr int GV_THREADS = GV_CTHREADS + 32;
constexpr size_t GV_SMEM_MAX = 227 * 1024;

enum { PRO_COPY = 0, PRO_NORM = 1, PRO_QUANT = 2 };

struct GvParams {
    const int8_t* wq;
    const uint16_t* wd;
    int N, K;
    const int8_t* xq;          // PRO_COPY: [M][K]
    const uint16_t* xd;        // PRO_COPY: [M][K/32]
    const float* xf;           // PRO_NORM, PRO_QUANT: f32 rows [M][K]
    const uint16_t* nw;        // PRO_NORM: norm weight [K] (bf16)
    float eps;
    const float* resid;        // optional: y = resid + acc
    float* y;
    int ldy;
    unsigned long long* keys;  // optional: fused argmax keys [M]
    int* err;
    int early;                 // consumers release a stage before computing on it
};

template <int STAGES>
struct GvSmem {
    uint8_t stage[STAGES][GV_STAGE_BYTES];
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    unsigned long long keys[4];
    float red[32];
    // followed by the activations: xs int8 [M][K], xds fp16 [M][K/32]
};

__device__ __forceinline__ void consumer_sync() { group_sync<GV_CTHREADS, 1>(); }

template <int M>
__device__ __forceinline__ void dot_block(const int4 w0, const int4 w1, float dw, const int8_t* xs,
                                          const uint16_t* xds, int K, int nb, int gb, float acc[M]) {
#pragma unroll
    for (int m = 0; m < M; m++) {
        // lanes 4-7 of each quarter-warp take the block's second half first: the 16-byte
        // reads of a quarter-warp then cover all 32 banks once (blocks are 32 bytes apart)
        const int sw = (threadIdx.x >> 2) & 1;
        const int4* xp = reinterpret_cast<const int4*>(xs + (size_t)m * K + (size_t)gb * 32);
        const int4 xa = xp[sw], xb = xp[sw ^ 1];
        const int4 x0 = sw ? xb : xa, x1 = sw ? xa : xb;
        int sum = 0;
        sum = __dp4a(w0.x, x0.x, sum); sum = __dp4a(w0.y, x0.y, sum);
        sum = __dp4a(w0.z, x0.z, sum); sum = __dp4a(w0.w, x0.w, sum);
        sum = __dp4a(w1.x, x1.x, sum); sum = __dp4a(w1.y, x1.y, sum);
        sum = __dp4a(w1.z, x1.z, sum); sum = __dp4a(w1.w, x1.w, sum);
        const float sc = __fmul_rn(dw, h2f(xds[(size_t)m * nb + gb]));
        acc[m] = __fadd_rn(acc[m], __fmul_rn((float)sum, sc));
    }
}

// SWI: the weight is the fused [gate; up] matrix (N = 2I rows). Work unit u takes the gate
// rows 8u..8u+7 and then the up rows I+8u..; the epilogue writes h = silu(gate) * up [M][I].
template <int M, int PRO, int STAGES, bool SWI>
__global__ void __launch_bounds__(GV_THREADS) q8_gemv_stream_kernel(const GvParams p) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    using Smem = GvSmem<STAGES>;
    Smem& S = *reinterpret_cast<Smem*>(smem_raw);
    int8_t* xs = reinterpret_cast<int8_t*>(smem_raw + sizeof(Smem));
    const int K = p.K, N = p.N;
    const int nb = K >> 5;
    uint16_t* xds = reinterpret_cast<uint16_t*>(xs + (size_t)M * K);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kc = K < GV_KC ? K : GV_KC;
    const int nchunks = (K + kc - 1) / kc;
    constexpr int HALVES = SWI ? 2 : 1;
    const int nout = SWI ? N / 2 : N;  // rows of the output
    const int nrg = (nout + GV_ROWS - 1) / GV_ROWS;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
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
            for (int rg = blockIdx.x; rg < nrg; rg += gridDim.x)
            for (int half = 0; half < HALVES; half++) {
                const int r0 = half * nout + rg * GV_ROWS;
                const int rows = min(GV_ROWS, nout - rg * GV_ROWS);
                for (int c = 0; c < nchunks; c++, it++) {
                    const int s = it % STAGES;
                    const unsigned ph = (unsigned)(it / STAGES) & 1u;
                    if (!mbar_wait(&S.empty[s], ph ^ 1u)) {
                        atomicCAS(p.err, 0, 3);
                        return;
                    }
                    const int k0 = c * kc;
                    const int cw = min(kc, K - k0);
                    uint8_t* st = S.stage[s];
                    mbar_expect_tx(&S.full[s], (unsigned)(rows * cw + rows * (cw / 16)));
                    if (cw == K) {  // whole rows: weights and scales each one contiguous run
                        bulk_g2s(st, p.wq + (size_t)r0 * K, (unsigned)(rows * K), &S.full[s]);
                        bulk_g2s(st + GV_ROWS * cw, p.wd + (size_t)r0 * nb, (unsigned)(rows * nb * 2), &S.full[s]);
                    } else {
                        for (int r = 0; r < rows; r++) {
                            bulk_g2s(st + r * cw, p.wq + (size_t)(r0 + r) * K + k0, (unsigned)cw, &S.full[s]);
                            bulk_g2s(st + GV_ROWS * cw + r * (cw / 16), p.wd + (size_t)(r0 + r) * nb + k0 / 32,
                                     (unsigned)(cw / 16), &S.full[s]);
                        }
                    }
                }
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    const int tid = threadIdx.x;
    pdl_wait();     // the activations and y belong to the preceding kernels
    pdl_trigger();
    if constexpr (PRO == PRO_COPY) {
        const int4* src = reinterpret_cast<const int4*>(p.xq);
        int4* dst = reinterpret_cast<int4*>(xs);
        for (int i = tid; i < M * K / 16; i += GV_CTHREADS) dst[i] = __ldg(src + i);
        const int4* srcd = reinterpret_cast<const int4*>(p.xd);
        int4* dstd = reinterpret_cast<int4*>(xds);
        for (int i = tid; i < M * nb * 2 / 16; i += GV_CTHREADS) dstd[i] = __ldg(srcd + i);
    } else if constexpr (PRO == PRO_NORM) {
#pragma unroll 1
        for (int m = 0; m < M; m++)
            rms_row<float, GV_CTHREADS, 1>(p.xf + (size_t)m * K, K, p.nw, p.eps, tid, S.red, nullptr,
                                           xs + (size_t)m * K, xds + (size_t)m * nb);
    } else {
#pragma unroll 1
        for (int m = 0; m < M; m++)
            quant_row<GV_CTHREADS>(p.xf + (size_t)m * K, K, tid, xs + (size_t)m * K, xds + (size_t)m * nb);
    }
    consumer_sync();

    float acc[M], gate[M];
#pragma unroll
    for (int m = 0; m < M; m++) acc[m] = gate[m] = 0.0f;
    int it = 0;
    bool ok = true;
    for (int rg = blockIdx.x; rg < nrg && ok; rg += gridDim.x)
    for (int half = 0; half < HALVES && ok; half++) {
        const int r0 = rg * GV_ROWS;  // output row base
        const int rows = min(GV_ROWS, nout - r0);
        // the residual this lane adds (lane m: token m), read now so that its round trip
        // overlaps the row's chunks
        float res = 0.0f;
        if (!SWI && p.resid && lane < M && warp < rows) res = p.resid[(size_t)lane * p.ldy + r0 + warp];
        for (int c = 0; c < nchunks; c++, it++) {
            const int s = it % STAGES;
            const unsigned ph = (unsigned)(it / STAGES) & 1u;
            if (!mbar_wait(&S.full[s], ph)) {
                if (lane == 0) atomicCAS(p.err, 0, 4);
                ok = false;
                break;
            }
            const int k0 = c * kc;
            const int cw = min(kc, K - k0);
            const int nbc = cw >> 5;  // <= 64: at most two blocks per lane
            const int8_t* wrow = reinterpret_cast<const int8_t*>(S.stage[s]) + warp * cw;
            const uint16_t* drow = reinterpret_cast<const uint16_t*>(S.stage[s] + GV_ROWS * cw) + warp * (cw / 32);
            const bool mine = warp < rows;
            if (p.early) {
                // move this warp's slice into registers, release the stage, then compute
                int4 w[2][2];
                float dw[2];
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const int b = lane + 32 * j;
                    if (mine && b < nbc) {
                        const int sw = (lane >> 2) & 1;  // conflict-free order, as in dot_block
                        const int4 wa = *reinterpret_cast<const int4*>(wrow + b * 32 + sw * 16);
                        const int4 wb = *reinterpret_cast<const int4*>(wrow + b * 32 + (sw ^ 1) * 16);
                        w[j][0] = sw ? wb : wa;
                        w[j][1] = sw ? wa : wb;
                        dw[j] = h2f(drow[b]);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.empty[s]);
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const int b = lane + 32 * j;
                    if (mine && b < nbc) dot_block<M>(w[j][0], w[j][1], dw[j], xs, xds, K, nb, (k0 >> 5) + b, acc);
                }
            } else {
                if (mine)
                    for (int b = lane; b < nbc; b += 32)
                        dot_block<M>(*reinterpret_cast<const int4*>(wrow + b * 32),
                                     *reinterpret_cast<const int4*>(wrow + b * 32 + 16), h2f(drow[b]), xs, xds, K,
                                     nb, (k0 >> 5) + b, acc);
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.empty[s]);
            }
            if (c == nchunks - 1) {
                const int row = r0 + warp;
#pragma unroll
                for (int m = 0; m < M; m++) {
                    const float v = warp_sum(acc[m]);
                    acc[m] = 0.0f;
                    if (SWI && half == 0) {
                        gate[m] = v;  // kept until the matching up row is done
                    } else if (mine) {
                        if (lane == m) {
                            const size_t o = (size_t)m * p.ldy + row;
                            if (SWI) p.y[o] = swiglu(gate[m], v);
                            else p.y[o] = p.resid ? __fadd_rn(res, v) : v;
                        }
                        if (!SWI && p.keys && lane == 0) atomicMax(&S.keys[m], argmax_key(v, row));
                    }
                }
            }
        }
    }
    if (p.keys) {
        consumer_sync();
        if (tid < M && S.keys[tid]) atomicMax(p.keys + tid, S.keys[tid]);
    }
}

// ---- launch configuration ----
// Measured on B200 (M = 1): throughput follows the stage bytes in flight per SM and the
// number of producing CTAs per SM: 3 CTAs x 4 stages (204 KiB) reached 5.7 TB/s on a
// 24576x4096 matrix and 6.7 TB/s on 151936x4096, against 3.5 TB/s for 1 CTA x 8 stages.
// So each launch picks, among the compiled stage counts, the (CTAs, stages) with the most
// stage bytes per SM that fit in shared memory, preferring more CTAs.
// LQ_GV="stages,ctas_per_sm,early" forces a configuration (tuning experiments).
struct GvTuning {
    int stages = 0, ctas = 0, early = 1;  // 0: automatic
};

static GvTuning gv_tuning() {
    static GvTuning t = [] {
        GvTuning v;
        if (const char* s = getenv("LQ_GV")) {
            int a = 0, b = 0, c = 0;
            if (sscanf(s, "%d,%d,%d", &a, &b, &c) == 3) {
                if (a == 3 || a == 4) v.stages = a;
                if (b >= 1 && b <= 4) v.ctas = b;
                v.early = c ? 1 : 0;
            }
        }
        return v;
    }();
    return t;
}

static size_t stage_smem(int stages, int64_t m, int64_t K);

// (stages, ctas per SM) for an M x K activation footprint
static void gv_pick(int64_t m, int64_t K, int* stages, int* ctas) {
    const GvTuning t = gv_tuning();
    if (t.stages && t.ctas) {
        *stages = t.stages;
        *ctas = t.ctas;
        return;
    }
    // 4 stages per CTA (3 was measurably worse at K = 12288: 4.3 vs 5.1 TB/s), as many CTAs
    // (up to 3) as shared memory holds; 3 stages only when even one 4-stage CTA does not fit
    int c = 3;
    while (c > 1 && (size_t)c * (stage_smem(4, m, K) + 1024) > GV_SMEM_MAX + 1024) c--;
    *stages = stage_smem(4, m, K) <= GV_SMEM_MAX ? 4 : 3;
    *ctas = c;
}

bool gemv_stream_supported(int64_t K) { return K % 256 == 0; }

static size_t stage_smem(int stages, int64_t m, int64_t K) {
    size_t base = 0;
    switch (stages) {
        case 3: base = sizeof(GvSmem<3>); break;
        default: base = sizeof(GvSmem<4>); break;
    }
    return base + (size_t)(m * K) + (size_t)(m * (K / 32)) * 2;
}

// the smallest configuration must fit for the kernel to run at all
size_t gemv_stream_smem(int64_t m, int64_t K) { return stage_smem(3, m, K); }

template <int M, int PRO, int STAGES, bool SWI>
static int run_stream(lq_ctx* ctx, GvParams p, int ctas) {
    const size_t smem = stage_smem(STAGES, M, p.K);
    if (smem > GV_SMEM_MAX) return set_error(ctx, LQ_ERR_UNSUPPORTED, "gemv: K=%d too large for M=%d", p.K, M);
    auto kern = q8_gemv_stream_kernel<M, PRO, STAGES, SWI>;
    if (const int rc = ensure_func_smem(ctx, (const void*)kern, GV_SMEM_MAX)) return rc;
    // never more CTAs per SM than can be resident together (registers, threads, smem): a
    // persistent grid that spills into a second wave would serialise
    int resident = 0;
    LQ_CUDA(ctx, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, kern, GV_THREADS, smem));
    const int nrg = ceil_div(SWI ? p.N / 2 : p.N, GV_ROWS);
    const int grid = std::min(nrg, ctx->sm_count * std::max(1, std::min(ctas, resident)));
    return launch_kernel(ctx, kern, dim3(grid), dim3(GV_THREADS), smem, "q8_gemv_stream", p);
}

template <int M, int PRO, bool SWI>
static int run_stream_s(lq_ctx* ctx, const GvParams& p) {
    int stages = 4, ctas = 2;
    gv_pick(M, p.K, &stages, &ctas);
    switch (stages) {
        case 3: return run_stream<M, PRO, 3, SWI>(ctx, p, ctas);
        default: return run_stream<M, PRO, 4, SWI>(ctx, p, ctas);
    }
}

template <int PRO, bool SWI = false>
static int run_stream_m(lq_ctx* ctx, int64_t m, const GvParams& p) {
    switch (m) {
        case 1: return run_stream_s<1, PRO, SWI>(ctx, p);
        case 2: return run_stream_s<2, PRO, SWI>(ctx, p);
        case 3: return run_stream_s<3, PRO, SWI>(ctx, p);
        case 4: return run_stream_s<4, PRO, SWI>(ctx, p);
        default: return set_error(ctx, LQ_ERR_INVALID_ARG, "gemv_stream: m=%lld > 4", (long long)m);
    }
}

static GvParams base_params(lq_ctx* ctx, const lq_q8_tensor* w, float* y, const float* resid, int64_t ldy,
                            unsigned long long* keys) {
    GvParams p = {};
    p.wq = w->qs;
    p.wd = w->d;
    p.N = (int)w->n;
    p.K = (int)w->k;
    p.resid = resid;
    p.y = y;
    p.ldy = (int)ldy;
    p.keys = keys;
    p.err = ctx->err_flag;
    p.early = gv_tuning().early;
    return p;
}

int launch_gemv_stream(lq_ctx* ctx, const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd, int64_t m,
                       float* y, const float* resid, int64_t ldy, unsigned long long* keys) {
    GvParams p = base_params(ctx, w, y, resid, ldy, keys);
    p.xq = xq;
    p.xd = xd;
    return run_stream_m<PRO_COPY>(ctx, m, p);
}

int launch_gemv_norm(lq_ctx* ctx, const lq_q8_tensor* w, const float* x, const uint16_t* norm_w, float eps,
                     int64_t m, float* y, const float* resid, int64_t ldy, unsigned long long* keys) {
    GvParams p = base_params(ctx, w, y, resid, ldy, keys);
    p.xf = x;
    p.nw = norm_w;
    p.eps = eps;
    return run_stream_m<PRO_NORM>(ctx, m, p);
}

int launch_gemv_norm_swiglu(lq_ctx* ctx, const lq_q8_tensor* w, const float* x, const uint16_t* norm_w, float eps,
                            int64_t m, float* h, int64_t ldh) {
    GvParams p = base_params(ctx, w, h, nullptr, ldh, nullptr);
    p.xf = x;
    p.nw = norm_w;
    p.eps = eps;
    return run_stream_m<PRO_NORM, true>(ctx, m, p);
}

int launch_gemv_quant(lq_ctx* ctx, const lq_q8_tensor* w, const float* x, int64_t m, float* y, const float* resid,
                      int64_t ldy) {
    GvParams p = base_params(ctx, w, y, resid, ldy, nullptr);
    p.xf = x;
    return run_stream_m<PRO_QUANT>(ctx, m, p);
}

}  // namespace lq
