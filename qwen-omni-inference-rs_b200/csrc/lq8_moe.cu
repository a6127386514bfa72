// lq8_moe.cu -- Qwen3-MoE sparse MLP on Q8_0 experts (router, top-k, grouped expert GEMVs,
// combine). The reference has no MoE code; the convention follows the Qwen3-MoE sparse block:
//   logits = x . R^T (Q8_0, blocks ascending: bit-identical to the oracle, so the same experts
//   are chosen);
//   p = softmax(logits) (f32); the top_k experts by logit, ties to the lower expert index;
//   w_j = p[e_j], renormalised by their sum (selection order) when norm_topk;
//   y_e = down_e . (silu(gate_e . x) * (up_e . x)), h quantized to Q8_0 per 32-block;
//   out[t] = residual[t] + sum over the token's experts in ascending index of w_e * y_e[t].
//
// All counts live in device memory, so the whole layer is one fixed sequence of launches
// (CUDA-graph capturable):
//   moe_route     one CTA per token: logits (a warp per expert, block terms in parallel, summed
//                 in ascending block order),
//                 softmax, top-k, weights; also the token's experts in ascending order.
//   moe_dispatch  one CTA: per-expert pair lists in token order (warp ballots, deterministic),
//                 offsets, the list of active experts, each pair's slot for the combine.
//   moe_mma       persistent grouped GEMV on the int8 tensor cores streaming the touched
//                 experts' weights through a shared-memory ring (see below); the gate/up pass
//                 fuses SiLU * up and the Q8_0 quantization of h.
//   moe_combine   per token: residual + sum_e w_e * y_e in ascending expert order.
#include "lq8_async.cuh"
#include "lq8_fused.cuh"
#include "lq8_internal.cuh"
#include "lq8_tma.cuh"

#include <cstdlib>

namespace lq {

constexpr int MOE_MAX_E = 512;
constexpr int MOE_MAX_K = 16;

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
// route: one CTA per token (min(1024, max(128, 8E)) threads)
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) moe_route_kernel(const int8_t* __restrict__ xq, const uint16_t* __restrict__ xd, int H,
                                 const int8_t* __restrict__ rq, const uint16_t* __restrict__ rd, int E, int top_k,
                                 int norm_topk, int32_t* __restrict__ ids, float* __restrict__ wts,
                                 int32_t* __restrict__ ids_sorted, float* __restrict__ w_sorted) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const int nb = H / 32;
    int8_t* sx = reinterpret_cast<int8_t*>(smem_raw);                       // [H]
    float* sdx = reinterpret_cast<float*>(smem_raw + H);                     // [nb]
    float* lg = sdx + nb;                                                    // [E]
    float* pe = lg + E;                                                      // [E], then terms
    __shared__ int sel[MOE_MAX_K];
    __shared__ float selw[MOE_MAX_K];
    const int t = blockIdx.x, tid = threadIdx.x;
    pdl_wait();
    pdl_trigger();
    for (int i = tid * 16; i < H; i += blockDim.x * 16)
        *reinterpret_cast<int4*>(sx + i) = *reinterpret_cast<const int4*>(xq + (size_t)t * H + i);
    for (int b = tid; b < nb; b += blockDim.x) sdx[b] = h2f(xd[(size_t)t * nb + b]);
    __syncthreads();
    // logits: warp w takes experts 4w..4w+3 (then 4 (w + nwarps) ...). Lanes form the block
    // terms (int dot, scale product) of all four experts with every load of a pass in flight
    // at once; then lane q adds expert q's terms in ascending block order (the oracle's sum).
    const int warp = tid >> 5, lane = tid & 31, nwarps = blockDim.x >> 5;
    const int ts = nb + 1;                              // padded term row (conflict-free sums)
    float* terms = pe + E + (size_t)warp * 4 * ts;      // [4][nb + 1]
    for (int e0 = 4 * warp; e0 < E; e0 += 4 * nwarps) {
        for (int b0 = 0; b0 < nb; b0 += 32) {
            int4 w[4][1][2];
            float dw[4][1];
#pragma unroll
            for (int q = 0; q < 4; q++)
#pragma unroll
                for (int i = 0; i < 1; i++) {
                    const int e = e0 + q, b = b0 + lane + 32 * i;
                    w[q][i][0] = w[q][i][1] = make_int4(0, 0, 0, 0);
                    dw[q][i] = 0.0f;
                    if (e < E && b < nb) {
                        const int8_t* wr = rq + (size_t)e * H + (size_t)b * 32;
                        w[q][i][0] = __ldg(reinterpret_cast<const int4*>(wr));
                        w[q][i][1] = __ldg(reinterpret_cast<const int4*>(wr + 16));
                        dw[q][i] = h2f(__ldg(rd + (size_t)e * nb + b));
                    }
                }
#pragma unroll
            for (int i = 0; i < 1; i++) {
                const int b = b0 + lane + 32 * i;
                if (b < nb) {
                    const int4 x0 = *reinterpret_cast<const int4*>(sx + b * 32);
                    const int4 x1 = *reinterpret_cast<const int4*>(sx + b * 32 + 16);
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        if (e0 + q < E)
                            terms[q * ts + b] = __fmul_rn((float)dot32(w[q][i][0], w[q][i][1], x0, x1),
                                                          __fmul_rn(dw[q][i], sdx[b]));
                }
            }
        }
        __syncwarp();
        if (lane < 4 && e0 + lane < E) {
            float acc = 0.0f;
            for (int b = 0; b < nb; b++) acc = __fadd_rn(acc, terms[lane * ts + b]);
            lg[e0 + lane] = acc;
        }
        __syncwarp();
    }
    __syncthreads();
    if (warp != 0) return;
    // softmax: max (warp), exp in parallel, sum in ascending expert order (lane 0), divide
    float mx = -INFINITY;
    for (int e = lane; e < E; e += 32) mx = fmaxf(mx, lg[e]);
    mx = warp_max(mx);
    for (int e = lane; e < E; e += 32) pe[e] = expf(__fsub_rn(lg[e], mx));
    __syncwarp();
    float sum = 0.0f;
    if (lane == 0)
        for (int e = 0; e < E; e++) sum = __fadd_rn(sum, pe[e]);
    sum = __shfl_sync(0xffffffffu, sum, 0);
    for (int e = lane; e < E; e += 32) pe[e] = __fdiv_rn(pe[e], sum);
    __syncwarp();
    // top-k by logit, ties to the lower expert index: k rounds of a warp argmax
    unsigned used = 0u;  // bit i: expert lane + 32 i taken (E <= 512 -> 16 bits)
    for (int j = 0; j < top_k; j++) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int i = 0, e = lane; e < E; i++, e += 32)
            if (!((used >> i) & 1u) && (lg[e] > bv || bi == 0x7fffffff)) { bv = lg[e]; bi = e; }
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != 0x7fffffff && (bi == 0x7fffffff || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
        }
        if ((bi & 31) == lane) used |= 1u << (bi >> 5);
        if (lane == 0) { sel[j] = bi; selw[j] = pe[bi]; }
    }
    __syncwarp();
    if (lane == 0) {
        if (norm_topk) {
            float s = 0.0f;
            for (int j = 0; j < top_k; j++) s = __fadd_rn(s, selw[j]);
            for (int j = 0; j < top_k; j++) selw[j] = __fdiv_rn(selw[j], s);
        }
        int se[MOE_MAX_K];
        float sw[MOE_MAX_K];
        for (int j = 0; j < top_k; j++) {
            ids[(size_t)t * top_k + j] = sel[j];
            wts[(size_t)t * top_k + j] = selw[j];
            // insertion into ascending expert order (for the combine)
            int q = j;
            while (q > 0 && se[q - 1] > sel[j]) { se[q] = se[q - 1]; sw[q] = sw[q - 1]; q--; }
            se[q] = sel[j];
            sw[q] = selw[j];
        }
        for (int j = 0; j < top_k; j++) {
            ids_sorted[(size_t)t * top_k + j] = se[j];
            w_sorted[(size_t)t * top_k + j] = sw[j];
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
    int32_t* cum;          // [E+1] passes of the active experts before active index a (prefix)
};

// (expert parallelism: only experts [e_lo, e_hi) get lists; the other pairs keep slot -1)
// Counts by shared-memory atomics, offsets and the active list by block-wide scans, then one
// warp walks the pairs 32 at a time in pair order (= token order within every expert): a
// pair's place is its expert's offset + the pairs already placed + its rank among the
// warp's lanes holding the same expert.
__global__ void __launch_bounds__(1024) moe_dispatch_kernel(const int32_t* __restrict__ ids_g, int rows, int E,
                                                            int top_k, MoeLists L, int e_lo, int e_hi, int tok) {
    __shared__ int cnt[MOE_MAX_E];
    __shared__ int off[MOE_MAX_E];
    __shared__ int placed[MOE_MAX_E];
    __shared__ int wsum[32], wact[32], wpas[32];
    extern __shared__ int ids_s[];  // [rows][top_k] staged from global
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int P = rows * top_k;
    for (int e = tid; e < E; e += blockDim.x) {
        cnt[e] = 0;
        placed[e] = 0;
    }
    pdl_wait();
    pdl_trigger();
    __syncthreads();
    for (int i = tid; i < P; i += blockDim.x) {
        const int e = ids_g[i];
        ids_s[i] = e;
        if (e >= e_lo && e < e_hi) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    // exclusive scans of the counts, of the active flags and of the experts' passes of `tok`
    // tokens (E <= 1024: one pass)
    const int c = tid < E ? cnt[tid] : 0, a = c > 0, pc = (c + tok - 1) / tok;
    int cs = c, as = a, ps = pc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, cs, o), z = __shfl_up_sync(0xffffffffu, as, o);
        const int w = __shfl_up_sync(0xffffffffu, ps, o);
        if (lane >= o) {
            cs += y;
            as += z;
            ps += w;
        }
    }
    if (lane == 31) {
        wsum[warp] = cs;
        wact[warp] = as;
        wpas[warp] = ps;
    }
    __syncthreads();
    if (warp == 0) {
        int ws = wsum[lane], wa = wact[lane], wp = wpas[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, ws, o), z = __shfl_up_sync(0xffffffffu, wa, o);
            const int w = __shfl_up_sync(0xffffffffu, wp, o);
            if (lane >= o) {
                ws += y;
                wa += z;
                wp += w;
            }
        }
        wsum[lane] = ws - wsum[lane];  // exclusive
        wact[lane] = wa - wact[lane];
        wpas[lane] = wp - wpas[lane];
        if (lane == 31) {
            L.offsets[E] = ws;
            L.active[E] = wa;
            L.cum[wa] = wp;
        }
    }
    __syncthreads();
    if (tid < E) {
        const int ex = wsum[warp] + cs - c;
        off[tid] = ex;
        L.offsets[tid] = ex;
        L.counts[tid] = c;
        if (a) {
            L.active[wact[warp] + as - 1] = tid;
            L.cum[wact[warp] + as - 1] = wpas[warp] + ps - pc;
        }
    }
    __syncthreads();
    if (warp != 0) return;
    for (int i0 = 0; i0 < P; i0 += 32) {
        const int i = i0 + lane;
        const int e = i < P ? ids_s[i] : -1;
        const bool loc = e >= e_lo && e < e_hi;
        const unsigned peers = __match_any_sync(0xffffffffu, loc ? e : -1 - lane);
        const unsigned below = peers & ((1u << lane) - 1u);
        if (loc) {
            const int pos = off[e] + placed[e] + __popc(below);
            L.pair_token[pos] = i / top_k;
            L.pair_slot[i] = pos;
        } else if (i < P) {
            L.pair_slot[i] = -1;
        }
        __syncwarp();
        if (loc && below == 0) placed[e] += __popc(peers);
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------------------
// grouped expert GEMV on the int8 tensor cores (mma.sync m16n8k32, s8 x s8 -> s32)
//
// Work unit = (active expert, a tile of output rows, a pass of up to TOK of the expert's
// tokens): gate/up streams 32 gate rows and the 32 matching up rows (32 rows of h), down
// streams 64 rows of the down projection -- 64 weight rows either way. Units are ordered by
// expert, tile, pass (the dispatch writes each active expert's pass count as a prefix), and
// each CTA takes an equal contiguous range of them: consecutive units mostly share the
// expert, so its activations stay in shared memory, and an expert with many tokens spreads
// over more CTAs (with routing skewed towards a few experts, item ranges would leave the
// CTAs holding them last). Passes of one tile follow each other, so the later passes read
// the weights from L2. One producer lane streams the unit's rows in K-chunks of 256 bytes (8
// Q8_0 blocks) into a shared-memory ring with 2-D TMA loads: per 32-row group two
// 128-byte-wide boxes (128-byte swizzle) and one box of the chunk's fp16 scales, 17 KiB per
// stage. Consumer warp w owns stage rows 16w..16w+15 (one m16 tile) and the pass's tokens as
// one or two n8 tiles. One MMA covers one Q8_0 block of 16 rows x 8
// tokens; its int32 dots are scaled per block and added to f32 accumulators that each thread
// keeps for fixed (row, token) pairs, in ascending block order with separately rounded
// multiply and add: the oracle's order, so every output is bit-identical to it.
//
// The MMA's 32 k positions are a permutation of the block's bytes: thread t of a quad holds
// bytes 8t..8t+3 of its rows (and tokens) in the register the MMA reads as k = 4t..4t+3 and
// bytes 8t+4..8t+7 in the one read as k = 16+4t..16+4t+3. A and B use the same permutation,
// so the integer dot is unchanged, and each operand is a single 8-byte shared load (2
// wavefronts per warp: the swizzle spreads the weight rows, a 16-byte pad the token rows).
//
// Epilogue: gate/up -> the gate and up accumulators meet in shared memory, then
// h = silu(g) * u is quantized to Q8_0 (the item's 32 rows are one block of h); down -> y
// [pair][row] f32.
// ---------------------------------------------------------------------------------------
constexpr int ME_KC = 256;                            // K bytes per stage
constexpr int ME_GRP = 32;                            // rows per group (one TMA box tall)
constexpr int ME_BOX = ME_GRP * 128;                  // one 128-byte-wide box (4 KiB)
constexpr int ME_W_BYTES = 2 * ME_GRP * ME_KC;        // two groups: 16 KiB of weights
constexpr int ME_STAGE = ME_W_BYTES + 2 * ME_GRP * 16;  // + fp16 scales [64 rows][8]: 17 KiB
constexpr int ME_CONSUMERS = 4;
constexpr int ME_THREADS = (ME_CONSUMERS + 1) * 32;
constexpr int ME_MAX_STAGES = 8;
constexpr int ME_TOK = 16;                            // most tokens per pass (two n8 tiles)
constexpr int ME_XCH = 33;                            // row stride (floats) of the gate/up exchange
static_assert(ME_STAGE % 1024 == 0, "swizzled boxes need 1024-byte aligned stages");

struct MoeExpertParams {
    int rows_per_expert;     // gate/up: 2I (gate rows then up rows); down: H
    int out_rows;            // gate/up: I; down: H
    int K;                   // multiple of 256
    int stages;
    const int8_t* xq;        // activations: gate/up [rows][K] by token; down [pairs][K] by pair
    const uint16_t* xd;
    const int32_t* pair_token;
    const int32_t* offsets;
    const int32_t* counts;
    const int32_t* active;   // [E] + n_active at [E]
    const int32_t* cum;      // [n_active + 1] pass prefix over the active experts
    int E;
    int e_base;              // first expert held in the weight stack (expert parallelism)
    int8_t* hq;              // gate/up output [pairs][I]
    uint16_t* hd;
    float* y;                // down output [pairs][H]
    int* err;
};

// shared memory after the stages: barriers, the gate/up exchange, the pass's tokens
__host__ __device__ constexpr size_t me_fixed_bytes(bool gu, int K, int tok) {
    return (size_t)2 * ME_MAX_STAGES * 8 + (gu ? (size_t)2 * tok * ME_XCH * 4 : 0) +
           (size_t)tok * (K + 16) + (size_t)(K / 32) * tok * 4 + (size_t)(MOE_MAX_E + 4) * 4;
}

__device__ __forceinline__ float h2f_bits(uint32_t w, int hi) {
    return h2f((uint16_t)(hi ? (w >> 16) : (w & 0xFFFFu)));
}

// One stage's 8 blocks for NT n8 tiles: A pieces wa/wb (rows ra, ra + 8) and their scales
// sa/sb (8 fp16 each) in registers; xb -> this thread's 8 bytes of token g's first block
// (n-tile stride xstride), db -> the f32 scales of tokens 2t, 2t+1 of the first block.
template <int NT>
__device__ __forceinline__ void me_blocks(float2 (&acc)[2][2], const uint2 (&wa)[8], const uint2 (&wb)[8],
                                          const uint4 sa, const uint4 sb, const int8_t* xb, int xstride,
                                          const float* db, int tok) {
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const uint32_t a[4] = {wa[j].x, wb[j].x, wa[j].y, wb[j].y};
        const uint32_t wsa = j < 2 ? sa.x : j < 4 ? sa.y : j < 6 ? sa.z : sa.w;
        const uint32_t wsb = j < 2 ? sb.x : j < 4 ? sb.y : j < 6 ? sb.z : sb.w;
        const float dwa = h2f_bits(wsa, j & 1), dwb = h2f_bits(wsb, j & 1);
#pragma unroll
        for (int n = 0; n < NT; n++) {
            const uint2 xv = *reinterpret_cast<const uint2*>(xb + n * xstride + j * 32);
            const uint32_t b[2] = {xv.x, xv.y};
            // the MMA adds the dots to 0x4B400000 (1.5 * 2^23 as a float): |dot| <= 32*127*127 <
            // 2^22, so the bits read as a float are 1.5 * 2^23 + dot exactly, and one subtraction
            // gives (float)dot -- no int-to-float conversions
            int d[4];
            mma_s8_bias(d, a, b, 0x4B400000);
            const float2 dx = *reinterpret_cast<const float2*>(db + j * tok + 8 * n);
            const float f0 = __fsub_rn(__int_as_float(d[0]), 12582912.0f);
            const float f1 = __fsub_rn(__int_as_float(d[1]), 12582912.0f);
            const float f2 = __fsub_rn(__int_as_float(d[2]), 12582912.0f);
            const float f3 = __fsub_rn(__int_as_float(d[3]), 12582912.0f);
            acc[n][0].x = __fadd_rn(acc[n][0].x, __fmul_rn(f0, __fmul_rn(dwa, dx.x)));
            acc[n][0].y = __fadd_rn(acc[n][0].y, __fmul_rn(f1, __fmul_rn(dwa, dx.y)));
            acc[n][1].x = __fadd_rn(acc[n][1].x, __fmul_rn(f2, __fmul_rn(dwb, dx.x)));
            acc[n][1].y = __fadd_rn(acc[n][1].y, __fmul_rn(f3, __fmul_rn(dwb, dx.y)));
        }
    }
}

// TOK: tokens per pass (8: one n8 tile, a smaller activation buffer and three CTAs per SM,
// for batches that give experts a few tokens each; 16: two tiles, for larger batches).
// Measured at batch 64 (30B-A3B): the layer 143 us with 8, 162 us with 16.
template <bool GU, int TOK>
__global__ void __launch_bounds__(ME_THREADS, 2) moe_mma_kernel(const __grid_constant__ CUtensorMap mw,
                                                             const __grid_constant__ CUtensorMap md,
                                                             const MoeExpertParams p) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const uint32_t raw = smem_addr(smem_raw);
    uint8_t* sm = smem_raw + (((raw + 1023) & ~1023u) - raw);  // swizzled boxes need 1024-byte alignment
    const int K = p.K, nb = K / 32, nchunks = K / ME_KC, S = p.stages, XS = K + 16;
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + (size_t)S * ME_STAGE);
    uint64_t* empty = full + ME_MAX_STAGES;
    float* xch = reinterpret_cast<float*>(empty + ME_MAX_STAGES);                 // [2][TOK][ME_XCH]
    int8_t* xs = reinterpret_cast<int8_t*>(xch + (GU ? 2 * TOK * ME_XCH : 0));  // [TOK][K + 16]
    float* xdf = reinterpret_cast<float*>(xs + (size_t)TOK * XS);               // [nb][TOK]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], ME_CONSUMERS);
        }
        mbar_fence_init();
    }
    pdl_wait();
    pdl_trigger();
    // work units (active expert, row tile, pass of TOK tokens), ordered by expert, then tile,
    // then pass; each CTA takes an equal contiguous range, so an expert with many tokens
    // (several passes) spreads over more CTAs. The pass prefix is staged in shared memory.
    int* scum = reinterpret_cast<int*>(xdf + (size_t)nb * TOK);  // [n_active + 1]
    const int n_active = p.active[p.E];
    for (int i = threadIdx.x; i <= n_active; i += ME_THREADS) scum[i] = p.cum[i];
    __syncthreads();
    const int item_rows = GU ? ME_GRP : 2 * ME_GRP;  // output rows per item
    const int tiles = p.out_rows / item_rows;
    const long long U = (long long)scum[n_active] * tiles;
    const long long u0 = U * blockIdx.x / gridDim.x, u1 = U * (blockIdx.x + 1) / gridDim.x;
    int a0 = 0;  // the active expert holding unit u0: the last a with cum[a] * tiles <= u0
    if (u0 < u1) {
        int hi = n_active - 1;
        while (a0 < hi) {
            const int mid = (a0 + hi + 1) >> 1;
            if ((long long)scum[mid] * tiles <= u0) a0 = mid;
            else hi = mid - 1;
        }
    }

    if (warp == ME_CONSUMERS) {
        // ---------------- producer (one lane) ----------------
        if (lane != 0) return;
        int it = 0;
        int a = a0, cur_a = -1, e = 0;
        for (long long u = u0; u < u1; u++) {
            while (u >= (long long)scum[a + 1] * tiles) a++;
            if (a != cur_a) {
                cur_a = a;
                e = p.active[a];
            }
            const int np = scum[a + 1] - scum[a];
            const int r0 = (int)((u - (long long)scum[a] * tiles) / np) * item_rows;
            const int base = (e - p.e_base) * p.rows_per_expert;
            for (int c = 0; c < nchunks; c++, it++) {
                    const int s = it % S;
                    if (!mbar_wait(&empty[s], ((unsigned)(it / S) & 1u) ^ 1u)) {
                        atomicCAS(p.err, 0, 21);
                        return;
                    }
                    uint8_t* st = sm + (size_t)s * ME_STAGE;
                    mbar_expect_tx(&full[s], (unsigned)ME_STAGE);
                    for (int q = 0; q < 2; q++) {
                        const int row = base + (GU ? q * p.out_rows + r0 : r0 + q * ME_GRP);
                        tma_load_2d(st + q * 2 * ME_BOX, &mw, c * ME_KC, row, &full[s]);
                        tma_load_2d(st + q * 2 * ME_BOX + ME_BOX, &mw, c * ME_KC + 128, row, &full[s]);
                        tma_load_2d(st + ME_W_BYTES + q * ME_GRP * 16, &md, c * 8, row, &full[s]);
                    }
                }
        }
        return;
    }
    // ---------------- consumers ----------------
    const int g = lane >> 2, t = lane & 3;
    const int q = warp >> 1;                    // group: gate/up -> 0 gate, 1 up; down -> rows 32q..
    const int ra = 16 * (warp & 1) + g;         // rows ra and ra + 8 of the group
    // byte offsets in a stage: the two 8-byte A pieces of block j (swizzle key g = ra & 7)
    const int a_row = q * 2 * ME_BOX + ra * 128 + (t & 1) * 8;
    const int sc_off = ME_W_BYTES + q * ME_GRP * 16 + ra * 16;
    int it = 0, cur_e = -1, cur_g0 = -1;
    bool bad = false;
    int a = a0, cur_a = -1, e = 0, cnt = 0, p0 = 0;
    for (long long u = u0; u < u1; u++) {
        while (u >= (long long)scum[a + 1] * tiles) a++;
        if (a != cur_a) {
            cur_a = a;
            e = p.active[a];
            cnt = p.counts[e];
            p0 = p.offsets[e];
        }
        const int np = scum[a + 1] - scum[a];
        const long long v = u - (long long)scum[a] * tiles;
        const int r0 = (int)(v / np) * item_rows;
        {
            const int g0 = (int)(v % np) * TOK;
            const int ng = min(TOK, cnt - g0);
            if (e != cur_e || g0 != cur_g0) {
                group_sync<ME_CONSUMERS * 32, 1>();  // nobody still reads the previous tokens
                for (int i = threadIdx.x; i < ng * (K / 16); i += ME_CONSUMERS * 32) {
                    const int tk = i / (K / 16), c16 = (i % (K / 16)) * 16;
                    const int src = GU ? p.pair_token[p0 + g0 + tk] : p0 + g0 + tk;
                    cp_async16(xs + (size_t)tk * XS + c16, p.xq + (size_t)src * K + c16, true);
                }
                cp_async_commit();
                for (int i = threadIdx.x; i < ng * nb; i += ME_CONSUMERS * 32) {
                    const int tk = i / nb, b = i % nb;
                    const int src = GU ? p.pair_token[p0 + g0 + tk] : p0 + g0 + tk;
                    xdf[b * TOK + tk] = h2f(p.xd[(size_t)src * nb + b]);
                }
                cp_async_wait<0>();
                group_sync<ME_CONSUMERS * 32, 1>();
                cur_e = e;
                cur_g0 = g0;
            }
            const bool two = ng > 8;  // second n8 tile (warp-uniform)
            float2 acc[2][2];  // [n-tile][row ra, ra + 8] x tokens (2t, 2t + 1)
#pragma unroll
            for (int n = 0; n < 2; n++) acc[n][0] = acc[n][1] = make_float2(0.0f, 0.0f);
            for (int c = 0; c < nchunks; c++, it++) {
                const int s = it % S;
                if (!bad) {
                    bool ok = true;
                    if (lane == 0) ok = mbar_wait(&full[s], (unsigned)(it / S) & 1u);
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    if (!ok) {
                        if (lane == 0) atomicCAS(p.err, 0, 22);
                        bad = true;
                    }
                }
                if (bad) continue;
                const uint8_t* st = sm + (size_t)s * ME_STAGE;
                // this warp's slice of the stage into registers, then release the stage
                uint2 wa[8], wb[8];
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int ch = ((2 * (j & 3) + (t >> 1)) ^ g) << 4;
                    wa[j] = *reinterpret_cast<const uint2*>(st + a_row + (j >> 2) * ME_BOX + ch);
                    wb[j] = *reinterpret_cast<const uint2*>(st + a_row + 8 * 128 + (j >> 2) * ME_BOX + ch);
                }
                const uint4 sa = *reinterpret_cast<const uint4*>(st + sc_off);
                const uint4 sb = *reinterpret_cast<const uint4*>(st + sc_off + 8 * 16);
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
                // straight-line code for the chunk's 8 blocks (the n8-tile count is decided
                // once, outside), so loads and MMAs of different blocks can overlap
                const int8_t* xb = xs + (size_t)g * XS + c * ME_KC + 8 * t;
                const float* db = xdf + c * 8 * TOK + 2 * t;
                if (TOK > 8 && two) me_blocks<2>(acc, wa, wb, sa, sb, xb, 8 * XS, db, TOK);
                else me_blocks<1>(acc, wa, wb, sa, sb, xb, 8 * XS, db, TOK);
            }
            // epilogue: value v of n-tile n is (row ra + 8 (v >> 1), token 8n + 2t + (v & 1))
            if (GU) {
#pragma unroll
                for (int n = 0; n < TOK / 8; n++)
#pragma unroll
                    for (int v = 0; v < 4; v++)
                        xch[(q * TOK + 8 * n + 2 * t + (v & 1)) * ME_XCH + ra + 8 * (v >> 1)] =
                            (v & 1) ? acc[n][v >> 1].y : acc[n][v >> 1].x;
                group_sync<ME_CONSUMERS * 32, 1>();
                if (!bad)
                    for (int tk = warp; tk < ng; tk += ME_CONSUMERS) {
                        const float gv = xch[tk * ME_XCH + lane], uv = xch[(TOK + tk) * ME_XCH + lane];
                        const float h = __fmul_rn(gv / (1.0f + expf(-gv)), uv);
                        const float amax = warp_max(fabsf(h));
                        float d, id;
                        q8_scale(amax, d, id);
                        const int pr = p0 + g0 + tk;
                        p.hq[(size_t)pr * p.out_rows + r0 + lane] = (int8_t)q8_quant(h, id);
                        if (lane == 0) p.hd[(size_t)pr * (p.out_rows / 32) + r0 / 32] = f2h(d);
                    }
                group_sync<ME_CONSUMERS * 32, 1>();  // the exchange is rewritten by the next item
            } else if (!bad) {
                const int row = r0 + 32 * q + ra;
#pragma unroll
                for (int n = 0; n < TOK / 8; n++)
#pragma unroll
                    for (int v = 0; v < 4; v++) {
                        const int tk = 8 * n + 2 * t + (v & 1);
                        if (tk < ng)
                            p.y[(size_t)(p0 + g0 + tk) * p.out_rows + row + 8 * (v >> 1)] =
                                (v & 1) ? acc[n][v >> 1].y : acc[n][v >> 1].x;
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
    // grid (H / 1024 column blocks, tokens); thread -> 4 columns, all the token's pairs in flight
    __shared__ int sp[MOE_MAX_K];
    __shared__ float sw[MOE_MAX_K];
    const int t = blockIdx.y;
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x < top_k) {
        sp[threadIdx.x] = pair_slot[(size_t)t * top_k + threadIdx.x];
        sw[threadIdx.x] = w_sorted[(size_t)t * top_k + threadIdx.x];
    }
    __syncthreads();
    const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (c >= H) return;
    // every pair's row loaded before the ordered adds
    float4 v[MOE_MAX_K];
#pragma unroll
    for (int jj = 0; jj < MOE_MAX_K; jj++)
        if (jj < top_k && sp[jj] >= 0) v[jj] = *reinterpret_cast<const float4*>(y + (size_t)sp[jj] * H + c);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int jj = 0; jj < MOE_MAX_K; jj++) {
        if (jj >= top_k || sp[jj] < 0) continue;  // past top-k, or an expert of another rank
        const float w = sw[jj];
        acc.x = __fadd_rn(acc.x, __fmul_rn(w, v[jj].x));
        acc.y = __fadd_rn(acc.y, __fmul_rn(w, v[jj].y));
        acc.z = __fadd_rn(acc.z, __fmul_rn(w, v[jj].z));
        acc.w = __fadd_rn(acc.w, __fmul_rn(w, v[jj].w));
    }
    const size_t o = (size_t)t * H + c;
    if (resid) {
        const float4 r = *reinterpret_cast<const float4*>(resid + o);
        acc.x = __fadd_rn(r.x, acc.x);
        acc.y = __fadd_rn(r.y, acc.y);
        acc.z = __fadd_rn(r.z, acc.z);
        acc.w = __fadd_rn(r.w, acc.w);
    }
    *reinterpret_cast<float4*>(out + o) = acc;
}

// ---------------------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------------------
static size_t al256(size_t b) { return (b + 255) & ~(size_t)255; }

template <bool GU, int TOK>
static int launch_moe_stream(lq_ctx* ctx, MoeExpertParams p, const int8_t* wq, const uint16_t* wd,
                             int64_t total_rows) {
    // the most CTAs per SM (3, 2, 1: 228 KB of shared memory per SM, 1 KB reserved per CTA)
    // whose rings still hold three stages each
    const size_t fixed = me_fixed_bytes(GU, p.K, TOK) + 1024 /*alignment*/;
    const size_t solo_budget = 227 * 1024;
    int per_sm = 1, stages = 0;
    for (int n = 3; n >= 1; n--) {
        const size_t budget = n == 1 ? solo_budget : (228 * 1024) / n - 1024;
        stages = budget > fixed ? (int)((budget - fixed) / ME_STAGE) : 0;
        per_sm = n;
        if (stages >= 3) break;
    }
    stages = std::min(stages, ME_MAX_STAGES);
    if (stages < 2) return set_error(ctx, LQ_ERR_UNSUPPORTED, "moe: K=%d leaves no room for the weight ring", p.K);
    p.stages = stages;
    CUtensorMap mw, md;
    int rc = make_tensor_map_2d(ctx, &mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, wq, (uint64_t)p.K, (uint64_t)total_rows,
                                (uint64_t)p.K, 128, ME_GRP, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tensor_map_2d(ctx, &md, CU_TENSOR_MAP_DATA_TYPE_UINT16, wd, (uint64_t)(p.K / 32), (uint64_t)total_rows,
                            (uint64_t)(p.K / 32) * 2, 8, ME_GRP, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    const size_t smem = (size_t)stages * ME_STAGE + fixed;
    if (const int rc = ensure_func_smem(ctx, (const void*)moe_mma_kernel<GU, TOK>, solo_budget)) return rc;
    int occ = 1;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, moe_mma_kernel<GU, TOK>, ME_THREADS, smem);
    per_sm = std::max(1, std::min(per_sm, occ));
    return launch_kernel(ctx, moe_mma_kernel<GU, TOK>, dim3(ctx->sm_count * per_sm), dim3(ME_THREADS), smem,
                         GU ? "moe_gate_up" : "moe_down", mw, md, p);
}

size_t moe_scratch_bytes(int64_t rows, int64_t E, int64_t top_k, int64_t H, int64_t inter) {
    const int64_t P = rows * top_k;
    return al256((size_t)P * 4) * 4 /*ids, wts, ids_sorted, w_sorted*/ + al256((size_t)E * 4) /*counts*/ +
           al256((size_t)(E + 1) * 4) * 3 /*active, offsets, cum*/ + al256((size_t)P * 4) * 2 /*pair lists*/ +
           al256((size_t)P * inter) + al256((size_t)P * (inter / 32) * 2) /*h as Q8_0*/ +
           al256((size_t)P * H * 4) /*y*/;
}

int launch_moe(lq_ctx* ctx, const lq_q8_tensor* router, const lq_q8_tensor* gate_up, const lq_q8_tensor* down,
               int64_t E, int64_t inter, int64_t top_k, int norm_topk, const int8_t* xq, const uint16_t* xd,
               int64_t rows, int64_t H, float* out, const float* resid, void* scratch, int32_t* ids_out,
               float* w_out, int64_t e_lo, int64_t e_hi) {
    if (e_hi <= e_lo) {
        e_lo = 0;
        e_hi = E;
    }
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
    L.cum = (int32_t*)take((size_t)(E + 1) * 4);
    int8_t* hq = (int8_t*)take((size_t)P * inter);
    uint16_t* hd = (uint16_t*)take((size_t)P * (inter / 32) * 2);
    float* y = (float*)take((size_t)P * H * 4);

    const int route_threads = (int)std::min<int64_t>(1024, std::max<int64_t>(128, E * 8));
    const size_t route_smem = (size_t)H + (size_t)(H / 32) * 4 + (size_t)E * 8 +
                              (size_t)(route_threads / 32) * 4 * (size_t)(H / 32 + 1) * 4;
    if (route_smem > 48 * 1024) {
        if (const int rc = ensure_func_smem(ctx, (const void*)moe_route_kernel, 200 * 1024)) return rc;
    }
    int rc = launch_kernel(ctx, moe_route_kernel, dim3((unsigned)rows), dim3(route_threads), route_smem, "moe_route",
                           xq, xd, (int)H, router->qs, router->d, (int)E, (int)top_k, norm_topk,
                           ids_out ? ids_out : ids, w_out ? w_out : wts, ids_sorted, w_sorted);
    if (rc) return rc;
    const size_t disp_smem = (size_t)rows * top_k * 4;
    if (disp_smem > 48 * 1024) {
        if (const int rc = ensure_func_smem(ctx, (const void*)moe_dispatch_kernel, 200 * 1024)) return rc;
    }
    // 8 tokens per pass while experts get a few tokens each on average (most single-pass),
    // else 16
    const bool small = rows * top_k <= 6 * std::max<int64_t>(1, e_hi - e_lo);
    rc = launch_kernel(ctx, moe_dispatch_kernel, dim3(1), dim3(1024), disp_smem, "moe_dispatch",
                       (const int32_t*)ids_sorted, (int)rows, (int)E, (int)top_k, L, (int)e_lo, (int)e_hi,
                       small ? 8 : 16);
    if (rc) return rc;
    MoeExpertParams p = {};
    p.E = (int)E;
    p.pair_token = L.pair_token;
    p.offsets = L.offsets;
    p.counts = L.counts;
    p.active = L.active;
    p.cum = L.cum;
    p.err = ctx->err_flag;
    p.e_base = (int)e_lo;
    // gate/up -> h = silu(g) * u as Q8_0 per pair
    p.rows_per_expert = (int)(2 * inter);
    p.out_rows = (int)inter;
    p.K = (int)H;
    p.xq = xq;
    p.xd = xd;
    p.hq = hq;
    p.hd = hd;
    rc = small ? launch_moe_stream<true, 8>(ctx, p, gate_up->qs, gate_up->d, gate_up->n)
               : launch_moe_stream<true, 16>(ctx, p, gate_up->qs, gate_up->d, gate_up->n);
    if (rc) return rc;
    // down -> y (f32 per pair)
    p.rows_per_expert = (int)H;
    p.out_rows = (int)H;
    p.K = (int)inter;
    p.xq = hq;
    p.xd = hd;
    p.y = y;
    rc = small ? launch_moe_stream<false, 8>(ctx, p, down->qs, down->d, down->n)
               : launch_moe_stream<false, 16>(ctx, p, down->qs, down->d, down->n);
    if (rc) return rc;
    return launch_kernel(ctx, moe_combine_kernel, dim3((unsigned)ceil_div(H, 1024), (unsigned)rows), dim3(256), 0,
                         "moe_combine", (const float*)y,
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
    LQ_REQUIRE(ctx, H > 0 && H % 256 == 0 && H <= 8192 && I > 0 && I % 256 == 0 && I <= 8192,
               "lq_moe_forward: hidden and inter must be multiples of 256 (at most 8192)");
    LQ_REQUIRE(ctx, router->n == E && router->k == H, "lq_moe_forward: router must be [E][hidden]");
    LQ_REQUIRE(ctx, experts->gate_up.n == E * 2 * I && experts->gate_up.k == H,
               "lq_moe_forward: gate_up must be [E*2*inter][hidden]");
    LQ_REQUIRE(ctx, experts->down.n == E * H && experts->down.k == I, "lq_moe_forward: down must be [E*hidden][inter]");
    LQ_REQUIRE(ctx, rows >= 0 && rows * top_k <= 49152, "lq_moe_forward: rows * top_k must be at most 49152");
    if (rows == 0) return LQ_OK;
    LQ_REQUIRE(ctx, xq && xd && out, "lq_moe_forward: NULL activation");
    LQ_REQUIRE(ctx, ((uintptr_t)out & 15) == 0 && ((uintptr_t)residual & 15) == 0,
               "lq_moe_forward: out and residual must be 16-byte aligned");
    const int rc = lq::ensure_scratch(ctx, lq::moe_scratch_bytes(rows, E, top_k, H, I));
    if (rc) return rc;
    return lq::launch_moe(ctx, router, &experts->gate_up, &experts->down, E, I, top_k, norm_topk, xq, xd, rows, H, out,
                          residual, ctx->scratch, ids_out, weights_out, 0, E);
}

extern "C" int lq_moe_forward_ep(lq_ctx* ctx, lq_comm* comm, const lq_q8_tensor* router, const lq_moe_experts* local,
                                 int64_t first_expert, const int8_t* xq, const uint16_t* xd, int64_t rows,
                                 int64_t top_k, int norm_topk, float* out, const float* residual) {
    LQ_ENTRY(ctx, "lq_moe_forward_ep");
    LQ_REQUIRE(ctx, comm && lq::comm_ctx(comm) == ctx, "lq_moe_forward_ep: communicator of another context");
    LQ_REQUIRE(ctx, router && local, "lq_moe_forward_ep: NULL weights");
    const int64_t E = router->n, El = local->n_experts, I = local->inter, H = local->hidden;
    LQ_REQUIRE(ctx, E > 0 && E <= lq::MOE_MAX_E && top_k > 0 && top_k <= lq::MOE_MAX_K && top_k <= E,
               "lq_moe_forward_ep: need 0 < top_k <= min(E, %d) and E <= %d", lq::MOE_MAX_K, lq::MOE_MAX_E);
    LQ_REQUIRE(ctx, El > 0 && first_expert >= 0 && first_expert + El <= E,
               "lq_moe_forward_ep: local experts [%lld, %lld) outside [0, %lld)", (long long)first_expert,
               (long long)(first_expert + El), (long long)E);
    LQ_REQUIRE(ctx, H > 0 && H % 256 == 0 && H <= 8192 && I > 0 && I % 256 == 0 && I <= 8192 && router->k == H,
               "lq_moe_forward_ep: hidden and inter must be multiples of 256 (at most 8192)");
    LQ_REQUIRE(ctx, local->gate_up.n == El * 2 * I && local->gate_up.k == H && local->down.n == El * H &&
                        local->down.k == I,
               "lq_moe_forward_ep: local expert stacks must be [El*2*inter][hidden] and [El*hidden][inter]");
    LQ_REQUIRE(ctx, rows >= 0 && rows * top_k <= 49152, "lq_moe_forward_ep: rows * top_k must be at most 49152");
    if (rows == 0) return LQ_OK;
    LQ_REQUIRE(ctx, xq && xd && out, "lq_moe_forward_ep: NULL activation");
    LQ_REQUIRE(ctx, ((uintptr_t)out & 15) == 0 && ((uintptr_t)residual & 15) == 0,
               "lq_moe_forward_ep: out and residual must be 16-byte aligned");
    int rc = lq::ensure_scratch(ctx, lq::moe_scratch_bytes(rows, E, top_k, H, I));
    if (rc) return rc;
    // this rank's experts, the residual on rank 0 only, then the sum over ranks
    rc = lq::launch_moe(ctx, router, &local->gate_up, &local->down, E, I, top_k, norm_topk, xq, xd, rows, H, out,
                        lq::comm_rank(comm) == 0 ? residual : nullptr, ctx->scratch, nullptr, nullptr, first_expert,
                        first_expert + El);
    if (rc) return rc;
    return lq::comm_allreduce_sum_f32(comm, out, out, rows * H);
}
