// lq8_moe.cu -- Qwen3-MoE sparse MLP on Q8_0 experts (router, top-k, grouped expert GEMVs,
// combine). The reference has no MoE code; the convention follows the Qwen3-MoE sparse block:
//   logits = x . R^T (Q8_0, blocks ascending, bit-identical to the oracle);
//   p = softmax(logits) (f32); the top_k experts by logit, ties to the lower expert index;
//   w_j = p[e_j], renormalised by their sum (selection order) when norm_topk;
//   y_e = down_e . (silu(gate_e . x) * (up_e . x)), h quantized to Q8_0 per 32-block;
//   out[t] = residual[t] + sum over the token's experts in ascending index of w_e * y_e[t].
//
// All counts live in device memory, so the whole layer is one fixed sequence of launches
// (CUDA-graph capturable):
//   moe_route     one CTA per token: logits (a thread per expert, sequential over blocks),
//                 softmax, top-k, weights; also the token's experts in ascending order.
//   moe_dispatch  one CTA: per-expert pair lists in token order (warp ballots, deterministic),
//                 offsets, the list of active experts, each pair's slot for the combine.
//   moe_expert    persistent grouped GEMV over work items (active expert, tile of 256 weight
//                 rows): a thread owns a weight row (gate/up: the row pair r, I+r) and up to 8
//                 tokens of the expert at a time, accumulating blocks in ascending order
//                 (bit-identical per output to the oracle's Q8_0 dot). The gate/up pass fuses
//                 SiLU * up and the Q8_0 quantization of h (a warp's 32 rows are one block).
//   moe_combine   per token: residual + sum_e w_e * y_e in ascending expert order.
#include "lq8_async.cuh"
#include "lq8_internal.cuh"

namespace lq {

constexpr int MOE_MAX_E = 512;
constexpr int MOE_MAX_K = 16;
constexpr int MOE_TG = 8;          // tokens per pass of a work item
constexpr int MOE_ROWS = 256;      // weight rows per work item (one per thread)

__device__ __forceinline__ int dot32(const int4 a0, const int4 a1, const int4 b0, const int4 b1) {
    int s = 0;
    s = __dp4a(a0.x, b0.x, s);
    s = __dp4a(a0.y, b0.y, s);
    s = __dp4a(a0.z, b0.z, s);
    s = __dp4a(a0.w, b0.w, s);
    s = __dp4a(a1.x, b1.x, s);
    s = __dp4a(a1.y, b1.y, s);
    s = __dp4a(a1.z, b1.z, s);
    s = __dp4a(a1.w, b1.w, s);
    return s;
}

// ---------------------------------------------------------------------------------------
// route: one CTA (max(E, 128) threads, multiple of 32) per token
// ---------------------------------------------------------------------------------------
__global__ void moe_route_kernel(const int8_t* __restrict__ xq, const uint16_t* __restrict__ xd, int H,
                                 const int8_t* __restrict__ rq, const uint16_t* __restrict__ rd, int E, int top_k,
                                 int norm_topk, int32_t* __restrict__ ids, float* __restrict__ wts,
                                 int32_t* __restrict__ ids_sorted, float* __restrict__ w_sorted) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const int nb = H / 32;
    int8_t* sx = reinterpret_cast<int8_t*>(smem_raw);                       // [H]
    float* sdx = reinterpret_cast<float*>(smem_raw + H);                     // [nb]
    float* lg = sdx + nb;                                                    // [E]
    float* pe = lg + E;                                                      // [E]
    __shared__ int sel[MOE_MAX_K];
    __shared__ float selw[MOE_MAX_K];
    const int t = blockIdx.x, tid = threadIdx.x;
    pdl_wait();
    pdl_trigger();
    for (int i = tid * 16; i < H; i += blockDim.x * 16)
        *reinterpret_cast<int4*>(sx + i) = *reinterpret_cast<const int4*>(xq + (size_t)t * H + i);
    for (int b = tid; b < nb; b += blockDim.x) sdx[b] = h2f(xd[(size_t)t * nb + b]);
    __syncthreads();
    for (int e = tid; e < E; e += blockDim.x) {
        const int8_t* wr = rq + (size_t)e * H;
        const uint16_t* wd = rd + (size_t)e * nb;
        float acc = 0.0f;
        for (int b = 0; b < nb; b++) {
            const int4 w0 = __ldg(reinterpret_cast<const int4*>(wr + b * 32));
            const int4 w1 = __ldg(reinterpret_cast<const int4*>(wr + b * 32 + 16));
            const int4 x0 = *reinterpret_cast<const int4*>(sx + b * 32);
            const int4 x1 = *reinterpret_cast<const int4*>(sx + b * 32 + 16);
            const int s = dot32(w0, w1, x0, x1);
            acc = __fadd_rn(acc, __fmul_rn((float)s, __fmul_rn(h2f(wd[b]), sdx[b])));
        }
        lg[e] = acc;
    }
    __syncthreads();
    if (tid == 0) {
        // softmax (max, exp(l - max), sum ascending, divide), then top-k by logit
        float mx = -INFINITY;
        for (int e = 0; e < E; e++) mx = fmaxf(mx, lg[e]);
        float sum = 0.0f;
        for (int e = 0; e < E; e++) {
            pe[e] = expf(__fsub_rn(lg[e], mx));
            sum = __fadd_rn(sum, pe[e]);
        }
        for (int e = 0; e < E; e++) pe[e] = __fdiv_rn(pe[e], sum);
        unsigned used[MOE_MAX_E / 32];
        for (int i = 0; i < MOE_MAX_E / 32; i++) used[i] = 0u;
        for (int j = 0; j < top_k; j++) {
            int best = -1;
            for (int e = 0; e < E; e++)
                if (!((used[e >> 5] >> (e & 31)) & 1u) && (best < 0 || lg[e] > lg[best])) best = e;
            used[best >> 5] |= 1u << (best & 31);
            sel[j] = best;
            selw[j] = pe[best];
        }
        if (norm_topk) {
            float s = 0.0f;
            for (int j = 0; j < top_k; j++) s = __fadd_rn(s, selw[j]);
            for (int j = 0; j < top_k; j++) selw[j] = __fdiv_rn(selw[j], s);
        }
        for (int j = 0; j < top_k; j++) {
            ids[(size_t)t * top_k + j] = sel[j];
            wts[(size_t)t * top_k + j] = selw[j];
        }
        // ascending expert order for the combine
        int jj = 0;
        for (int e = 0; e < E && jj < top_k; e++)
            if ((used[e >> 5] >> (e & 31)) & 1u) {
                float we = 0.0f;
                for (int j = 0; j < top_k; j++)
                    if (sel[j] == e) we = selw[j];
                ids_sorted[(size_t)t * top_k + jj] = e;
                w_sorted[(size_t)t * top_k + jj] = we;
                jj++;
            }
    }
}

// ---------------------------------------------------------------------------------------
// dispatch: one CTA of 1024 threads (32 warps); warp w handles experts w, w+32, ...
// ---------------------------------------------------------------------------------------
struct MoeLists {
    int32_t* counts;       // [E]
    int32_t* offsets;      // [E+1]
    int32_t* active;       // [E] active expert ids (ascending), then n_active at active[E]
    int32_t* pair_token;   // [rows*k] token of each pair, grouped by expert, tokens ascending
    int32_t* pair_slot;    // [rows][k] pair index of the token's jj-th expert (ascending expert)
};

__global__ void __launch_bounds__(1024) moe_dispatch_kernel(const int32_t* __restrict__ ids_sorted, int rows, int E,
                                                            int top_k, MoeLists L) {
    __shared__ int cnt[MOE_MAX_E];
    __shared__ int off[MOE_MAX_E + 1];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_wait();
    pdl_trigger();
    // pass 1: counts
    for (int e = warp; e < E; e += 32) {
        int c = 0;
        for (int t0 = 0; t0 < rows; t0 += 32) {
            const int t = t0 + lane;
            bool has = false;
            if (t < rows)
                for (int j = 0; j < top_k; j++) has |= ids_sorted[(size_t)t * top_k + j] == e;
            c += __popc(__ballot_sync(0xffffffffu, has));
        }
        if (lane == 0) cnt[e] = c;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int s = 0, na = 0;
        for (int e = 0; e < E; e++) {
            off[e] = s;
            s += cnt[e];
            if (cnt[e] > 0) L.active[na++] = e;
        }
        off[E] = s;
        L.active[E] = na;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        L.counts[e] = cnt[e];
        L.offsets[e] = off[e];
    }
    if (threadIdx.x == 0) L.offsets[E] = off[E];
    // pass 2: fill in token order
    for (int e = warp; e < E; e += 32) {
        int pos = off[e];
        for (int t0 = 0; t0 < rows; t0 += 32) {
            const int t = t0 + lane;
            int jj = -1;
            if (t < rows)
                for (int j = 0; j < top_k; j++)
                    if (ids_sorted[(size_t)t * top_k + j] == e) jj = j;
            const unsigned m = __ballot_sync(0xffffffffu, jj >= 0);
            if (jj >= 0) {
                const int p = pos + __popc(m & ((1u << lane) - 1u));
                L.pair_token[p] = t;
                L.pair_slot[(size_t)t * top_k + jj] = p;
            }
            pos += __popc(m);
        }
    }
}

// ---------------------------------------------------------------------------------------
// grouped expert GEMV
// ---------------------------------------------------------------------------------------
struct MoeExpertParams {
    const int8_t* wq;        // stacked expert weights [E * rows_per_expert][K]
    const uint16_t* wd;
    int rows_per_expert;     // gate/up: 2I (a thread computes rows r and I + r); down: H
    int out_rows;            // gate/up: I; down: H
    int K;
    int gate_up;             // 1: SiLU * up epilogue + Q8_0 output; 0: f32 output per pair
    const int8_t* xq;        // activations: gate/up [rows][K] by token; down [pairs][K] by pair
    const uint16_t* xd;
    const int32_t* pair_token;
    const int32_t* offsets;
    const int32_t* counts;
    const int32_t* active;   // [E] + n_active at [E]
    int E;
    int8_t* hq;              // gate/up output [pairs][I]
    uint16_t* hd;
    float* y;                // down output [pairs][H]
};

__global__ void __launch_bounds__(MOE_ROWS) moe_expert_kernel(const MoeExpertParams p) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const int K = p.K, nb = K / 32;
    int8_t* sx = reinterpret_cast<int8_t*>(smem_raw);                          // [MOE_TG][K]
    float* sdx = reinterpret_cast<float*>(smem_raw + (size_t)MOE_TG * K);      // [MOE_TG][nb]
    const int tid = threadIdx.x, lane = tid & 31;
    pdl_wait();
    pdl_trigger();
    const int n_active = p.active[p.E];
    const int tiles = (p.out_rows + MOE_ROWS - 1) / MOE_ROWS;
    const int items = n_active * tiles;
    for (int it = blockIdx.x; it < items; it += gridDim.x) {
        const int e = p.active[it / tiles];
        const int r = (it % tiles) * MOE_ROWS + tid;
        const bool row_ok = r < p.out_rows;
        const int cnt = p.counts[e], p0 = p.offsets[e];
        const size_t wrow0 = (size_t)e * p.rows_per_expert + (row_ok ? r : 0);
        const int8_t* w0 = p.wq + wrow0 * K;
        const uint16_t* d0 = p.wd + wrow0 * nb;
        const int8_t* w1 = w0 + (size_t)p.out_rows * K;          // up row (gate/up only)
        const uint16_t* d1 = d0 + (size_t)p.out_rows * nb;
        for (int g0 = 0; g0 < cnt; g0 += MOE_TG) {
            const int ng = min(MOE_TG, cnt - g0);
            __syncthreads();  // the previous group's activations are no longer read
            for (int i = tid; i < ng * (K / 16); i += MOE_ROWS) {
                const int tk = i / (K / 16), c = (i % (K / 16)) * 16;
                const int src = p.gate_up ? p.pair_token[p0 + g0 + tk] : p0 + g0 + tk;
                cp_async16(sx + (size_t)tk * K + c, p.xq + (size_t)src * K + c, true);
            }
            cp_async_commit();
            for (int i = tid; i < ng * nb; i += MOE_ROWS) {
                const int tk = i / nb, b = i % nb;
                const int src = p.gate_up ? p.pair_token[p0 + g0 + tk] : p0 + g0 + tk;
                sdx[tk * nb + b] = h2f(p.xd[(size_t)src * nb + b]);
            }
            cp_async_wait<0>();
            __syncthreads();
            float acc0[MOE_TG], acc1[MOE_TG];
#pragma unroll
            for (int j = 0; j < MOE_TG; j++) acc0[j] = acc1[j] = 0.0f;
            if (row_ok) {
#pragma unroll 2
                for (int b = 0; b < nb; b++) {
                    const int4 a0 = __ldcs(reinterpret_cast<const int4*>(w0 + b * 32));
                    const int4 a1 = __ldcs(reinterpret_cast<const int4*>(w0 + b * 32 + 16));
                    const float dw0 = h2f(__ldg(d0 + b));
                    int4 c0 = make_int4(0, 0, 0, 0), c1 = c0;
                    float dw1 = 0.0f;
                    if (p.gate_up) {
                        c0 = __ldcs(reinterpret_cast<const int4*>(w1 + b * 32));
                        c1 = __ldcs(reinterpret_cast<const int4*>(w1 + b * 32 + 16));
                        dw1 = h2f(__ldg(d1 + b));
                    }
#pragma unroll
                    for (int j = 0; j < MOE_TG; j++) {
                        if (j < ng) {
                            const int4 x0 = *reinterpret_cast<const int4*>(sx + (size_t)j * K + b * 32);
                            const int4 x1 = *reinterpret_cast<const int4*>(sx + (size_t)j * K + b * 32 + 16);
                            const float dx = sdx[j * nb + b];
                            acc0[j] = __fadd_rn(acc0[j], __fmul_rn((float)dot32(a0, a1, x0, x1), __fmul_rn(dw0, dx)));
                            if (p.gate_up)
                                acc1[j] = __fadd_rn(acc1[j],
                                                    __fmul_rn((float)dot32(c0, c1, x0, x1), __fmul_rn(dw1, dx)));
                        }
                    }
                }
            }
            // epilogue per token of the group
#pragma unroll
            for (int j = 0; j < MOE_TG; j++) {
                if (j < ng) {
                    const int pr = p0 + g0 + j;
                    if (p.gate_up) {
                        // h = silu(g) * u, quantized per 32 rows (this warp's rows form one block)
                        const float s = acc0[j] / (1.0f + expf(-acc0[j]));
                        const float h = row_ok ? __fmul_rn(s, acc1[j]) : 0.0f;
                        const float amax = warp_max(fabsf(h));
                        float d, id;
                        q8_scale(amax, d, id);
                        if (row_ok) {
                            p.hq[(size_t)pr * p.out_rows + r] = (int8_t)q8_quant(h, id);
                            if (lane == 0) p.hd[(size_t)pr * (p.out_rows / 32) + r / 32] = f2h(d);
                        }
                    } else if (row_ok) {
                        p.y[(size_t)pr * p.out_rows + r] = acc0[j];
                    }
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------------------
// combine: out[t][c] = resid[t][c] + sum_jj w_sorted[t][jj] * y[pair_slot[t][jj]][c]
// ---------------------------------------------------------------------------------------
__global__ void moe_combine_kernel(const float* __restrict__ y, const int32_t* __restrict__ pair_slot,
                                   const float* __restrict__ w_sorted, int top_k, int H, const float* resid,
                                   float* out) {
    const int t = blockIdx.x;
    pdl_wait();
    pdl_trigger();
    for (int c = threadIdx.x; c < H; c += blockDim.x) {
        float acc = 0.0f;
        for (int jj = 0; jj < top_k; jj++) {
            const int pr = pair_slot[(size_t)t * top_k + jj];
            acc = __fadd_rn(acc, __fmul_rn(w_sorted[(size_t)t * top_k + jj], y[(size_t)pr * H + c]));
        }
        const size_t o = (size_t)t * H + c;
        out[o] = resid ? __fadd_rn(resid[o], acc) : acc;
    }
}

// ---------------------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------------------
static size_t al256(size_t b) { return (b + 255) & ~(size_t)255; }

size_t moe_scratch_bytes(int64_t rows, int64_t E, int64_t top_k, int64_t H, int64_t inter) {
    const int64_t P = rows * top_k;
    return al256((size_t)P * 4) * 4 /*ids, wts, ids_sorted, w_sorted*/ + al256((size_t)E * 4) /*counts*/ +
           al256((size_t)(E + 1) * 4) * 2 /*active, offsets*/ + al256((size_t)P * 4) * 2 + al256((size_t)P * inter) +
           al256((size_t)P * (inter / 32) * 2) + al256((size_t)P * H * 4);
}

int launch_moe(lq_ctx* ctx, const lq_q8_tensor* router, const lq_q8_tensor* gate_up, const lq_q8_tensor* down,
               int64_t E, int64_t inter, int64_t top_k, int norm_topk, const int8_t* xq, const uint16_t* xd,
               int64_t rows, int64_t H, float* out, const float* resid, void* scratch, int32_t* ids_out,
               float* w_out) {
    if (rows <= 0) return LQ_OK;
    const int64_t P = rows * top_k;
    uint8_t* s = (uint8_t*)scratch;
    auto take = [&](size_t bytes) { uint8_t* q = s; s += al256(bytes); return q; };
    int32_t* ids = (int32_t*)take((size_t)P * 4);
    float* wts = (float*)take((size_t)P * 4);
    int32_t* ids_sorted = (int32_t*)take((size_t)P * 4);
    float* w_sorted = (float*)take((size_t)P * 4);
    MoeLists L;
    L.counts = (int32_t*)take((size_t)E * 4);
    L.active = (int32_t*)take((size_t)(E + 1) * 4);
    L.offsets = (int32_t*)take((size_t)(E + 1) * 4);
    L.pair_token = (int32_t*)take((size_t)P * 4);
    L.pair_slot = (int32_t*)take((size_t)P * 4);
    int8_t* hq = (int8_t*)take((size_t)P * inter);
    uint16_t* hd = (uint16_t*)take((size_t)P * (inter / 32) * 2);
    float* y = (float*)take((size_t)P * H * 4);

    const int route_threads = (int)std::max<int64_t>(128, ((E + 31) / 32) * 32);
    const size_t route_smem = (size_t)H + (size_t)(H / 32) * 4 + (size_t)E * 8;
    int rc = launch_kernel(ctx, moe_route_kernel, dim3((unsigned)rows), dim3(route_threads), route_smem, "moe_route",
                           xq, xd, (int)H, router->qs, router->d, (int)E, (int)top_k, norm_topk,
                           ids_out ? ids_out : ids, w_out ? w_out : wts, ids_sorted, w_sorted);
    if (rc) return rc;
    rc = launch_kernel(ctx, moe_dispatch_kernel, dim3(1), dim3(1024), 0, "moe_dispatch", (const int32_t*)ids_sorted,
                       (int)rows, (int)E, (int)top_k, L);
    if (rc) return rc;
    MoeExpertParams p = {};
    p.E = (int)E;
    p.pair_token = L.pair_token;
    p.offsets = L.offsets;
    p.counts = L.counts;
    p.active = L.active;
    const int grid = ctx->sm_count * 2;
    // gate/up -> h (Q8_0)
    p.wq = gate_up->qs;
    p.wd = gate_up->d;
    p.rows_per_expert = (int)(2 * inter);
    p.out_rows = (int)inter;
    p.K = (int)H;
    p.gate_up = 1;
    p.xq = xq;
    p.xd = xd;
    p.hq = hq;
    p.hd = hd;
    size_t smem = (size_t)MOE_TG * H + (size_t)MOE_TG * (H / 32) * 4;
    static bool attr[64] = {};
    if (ctx->device < 0 || ctx->device >= 64 || !attr[ctx->device]) {
        LQ_CUDA(ctx, cudaFuncSetAttribute(moe_expert_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        if (ctx->device >= 0 && ctx->device < 64) attr[ctx->device] = true;
    }
    rc = launch_kernel(ctx, moe_expert_kernel, dim3(grid), dim3(MOE_ROWS), smem, "moe_gate_up", p);
    if (rc) return rc;
    // down -> y (f32 per pair)
    p.wq = down->qs;
    p.wd = down->d;
    p.rows_per_expert = (int)H;
    p.out_rows = (int)H;
    p.K = (int)inter;
    p.gate_up = 0;
    p.xq = hq;
    p.xd = hd;
    p.y = y;
    smem = (size_t)MOE_TG * inter + (size_t)MOE_TG * (inter / 32) * 4;
    rc = launch_kernel(ctx, moe_expert_kernel, dim3(grid), dim3(MOE_ROWS), smem, "moe_down", p);
    if (rc) return rc;
    return launch_kernel(ctx, moe_combine_kernel, dim3((unsigned)rows), dim3(256), 0, "moe_combine", (const float*)y,
                         (const int32_t*)L.pair_slot, (const float*)w_sorted, (int)top_k, (int)H, resid, out);
}

}  // namespace lq

extern "C" int lq_moe_forward(lq_ctx* ctx, const lq_q8_tensor* router, const lq_moe_experts* experts,
                              const int8_t* xq, const uint16_t* xd, int64_t rows, int64_t top_k, int norm_topk,
                              float* out, const float* residual, int32_t* ids_out, float* weights_out) {
    LQ_ENTRY(ctx, "lq_moe_forward");
    LQ_REQUIRE(ctx, router && experts, "lq_moe_forward: NULL weights");
    const int64_t E = experts->n_experts, I = experts->inter, H = experts->hidden;
    LQ_REQUIRE(ctx, E > 0 && E <= lq::MOE_MAX_E && top_k > 0 && top_k <= lq::MOE_MAX_K && top_k <= E,
               "lq_moe_forward: need 0 < top_k <= min(E, %d) and E <= %d", lq::MOE_MAX_K, lq::MOE_MAX_E);
    LQ_REQUIRE(ctx, H > 0 && H % 32 == 0 && I > 0 && I % 32 == 0 && H % 16 == 0,
               "lq_moe_forward: hidden and inter must be multiples of 32");
    LQ_REQUIRE(ctx, router->n == E && router->k == H, "lq_moe_forward: router must be [E][hidden]");
    LQ_REQUIRE(ctx, experts->gate_up.n == E * 2 * I && experts->gate_up.k == H,
               "lq_moe_forward: gate_up must be [E*2*inter][hidden]");
    LQ_REQUIRE(ctx, experts->down.n == E * H && experts->down.k == I, "lq_moe_forward: down must be [E*hidden][inter]");
    LQ_REQUIRE(ctx, (size_t)8 * H + (size_t)8 * (H / 32) * 4 <= 200 * 1024 && (size_t)8 * I <= 200 * 1024,
               "lq_moe_forward: hidden/inter too large for the expert kernel");
    LQ_REQUIRE(ctx, rows >= 0 && rows * top_k < (1ll << 31), "lq_moe_forward: bad rows");
    if (rows == 0) return LQ_OK;
    LQ_REQUIRE(ctx, xq && xd && out, "lq_moe_forward: NULL activation");
    const int rc = lq::ensure_scratch(ctx, lq::moe_scratch_bytes(rows, E, top_k, H, I));
    if (rc) return rc;
    return lq::launch_moe(ctx, router, &experts->gate_up, &experts->down, E, I, top_k, norm_topk, xq, xd, rows, H, out,
                          residual, ctx->scratch, ids_out, weights_out);
}
