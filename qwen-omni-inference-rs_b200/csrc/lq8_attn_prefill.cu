// lq8_attn_prefill.cu -- causal GQA attention for prefill (L query positions per sequence) over
// the f32 KV cache: softmax((q.k^T) * 1/sqrt(128) + causal mask) . v  (attention.rs:366-399,
// repeat_kv attention.rs:426-456, mask causal_mask.rs:104-164, softmax tensor.rs:1913-1934).
//
// A CTA owns one sequence, one kv head and a tile of 128 (query position, query head) rows:
// the G = Hq/Hkv heads sharing the kv head times TQ = 128/G consecutive positions, so every K/V
// chunk staged in shared memory serves all of them. It walks the causally visible keys in
// chunks of 64 with an online softmax (running max m, running sum l, output rescaled by
// exp(m_old - m_new)); f32 throughout, scores and P.V on the CUDA cores with fused
// multiply-adds. The result equals the reference's full-row softmax up to f32 rounding.
//
// Thread (256 per CTA) t owns rows r_i = t/8 + 32 i (i < 4); in the score phase keys
// k_j = t%8 + 8 j (j < 8), in the P.V phase dims 4 (t%8 + 8 j) .. +3 (j < 4). The row owners
// coincide, so each thread keeps m and l of its rows in registers. Q, K, P rows are padded to
// conflict-free strides. K of chunk c+1 loads during c's softmax and P.V, V of c+1 during
// c+1's scores (cp.async groups).
#include "lq8_async.cuh"
#include "lq8_internal.cuh"

namespace lq {

constexpr int PF_ROWS = 128;          // (position, head) rows per CTA
constexpr int PF_C = 64;              // keys per chunk
constexpr int PF_D = 128;
constexpr int PF_QS = PF_D + 4;       // padded row strides (floats)
constexpr int PF_PS = PF_C + 4;
constexpr int PF_THREADS = 256;

struct PfSmem {
    float q[PF_ROWS][PF_QS];   // query rows; holds the output rows at the end
    float k[PF_C][PF_QS];
    float v[PF_C][PF_D];
    float p[PF_ROWS][PF_PS];
};

struct PfParams {
    const float* q;   // [B][Hq][L][D]
    const float* kc;  // [B][Hkv][ctx_max][D]
    const float* vc;
    int Hq, Hkv, L, G, TQ, pos0, ctx_max, ntiles;
    const int32_t* pos0_dev;
    float* out;       // [B*L][Hq*D] or NULL
    int8_t* xq;       // Q8_0 of out, or NULL
    uint16_t* xd;
};

__device__ __forceinline__ void pf_quant_warp32(float v, int lane, int8_t* q_out, uint16_t* d_out) {
    const float amax = warp_max(fabsf(v));
    float d, id;
    q8_scale(amax, d, id);
    q_out[lane] = (int8_t)q8_quant(v, id);
    if (lane == 0) *d_out = f2h(d);
}

__global__ void __launch_bounds__(PF_THREADS, 1) attn_prefill_kernel(const PfParams p) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    PfSmem& S = *reinterpret_cast<PfSmem*>(smem_raw);
    const int t = threadIdx.x, rg = t >> 3, kg = t & 7;
    const int G = p.G, TQ = p.TQ, L = p.L, D = PF_D;
    const int tile = p.ntiles - 1 - (int)blockIdx.x;  // longest (latest) tiles first
    const int kvh = blockIdx.y, b = blockIdx.z;
    const int l0 = tile * TQ;
    const int nq = min(TQ, L - l0);  // valid positions in this tile
    pdl_wait();
    pdl_trigger();
    const int pos0 = p.pos0_dev ? *p.pos0_dev : p.pos0;
    const int limit = pos0 + l0 + nq - 1;  // last key any row of the tile sees
    if (limit >= p.ctx_max) return;        // rejected on the host for host positions
    const int nchunks = limit / PF_C + 1;
    const float* kbase = p.kc + ((int64_t)b * p.Hkv + kvh) * (int64_t)p.ctx_max * D;
    const float* vbase = p.vc + ((int64_t)b * p.Hkv + kvh) * (int64_t)p.ctx_max * D;

    // query rows r = g*TQ + lq (zero rows past the sequence end)
    for (int i = t; i < PF_ROWS * (D / 4); i += PF_THREADS) {
        const int r = i / (D / 4), c = (i % (D / 4)) * 4;
        const int g = r / TQ, lq = r - (r / TQ) * TQ;
        const bool ok = lq < nq;
        const float* src = p.q + (((int64_t)b * p.Hq + kvh * G + g) * L + (ok ? l0 + lq : 0)) * D + c;
        cp_async16(&S.q[r][c], src, ok);
    }
    auto load_k = [&](int c) {
        for (int i = t; i < PF_C * (D / 4); i += PF_THREADS) {
            const int r = i / (D / 4), cc = (i % (D / 4)) * 4;
            const int key = c * PF_C + r;
            cp_async16(&S.k[r][cc], kbase + (int64_t)(key <= limit ? key : 0) * D + cc, key <= limit);
        }
    };
    auto load_v = [&](int c) {
        for (int i = t; i < PF_C * (D / 4); i += PF_THREADS) {
            const int r = i / (D / 4), cc = (i % (D / 4)) * 4;
            const int key = c * PF_C + r;
            cp_async16(&S.v[r][cc], vbase + (int64_t)(key <= limit ? key : 0) * D + cc, key <= limit);
        }
    };
    load_k(0);
    cp_async_commit();
    load_v(0);
    cp_async_commit();

    // the causal limit of each of this thread's rows
    int qpos[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int r = rg + 32 * i;
        qpos[i] = pos0 + l0 + (r - (r / TQ) * TQ);
    }
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)D));
    float m[4], l[4];
    float4 o[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        m[i] = -INFINITY;
        l[i] = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; j++) o[i][j] = make_float4(0.f, 0.f, 0.f, 0.f);
    }

    for (int c = 0; c < nchunks; c++) {
        cp_async_wait<1>();  // Q and K_c have landed (V_c may still be in flight)
        __syncthreads();
        float s[4][8];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 8; j++) s[i][j] = 0.0f;
#pragma unroll 2
        for (int d4 = 0; d4 < D / 4; d4++) {
            float4 qv[4], kv[8];
#pragma unroll
            for (int i = 0; i < 4; i++) qv[i] = *reinterpret_cast<const float4*>(&S.q[rg + 32 * i][4 * d4]);
#pragma unroll
            for (int j = 0; j < 8; j++) kv[j] = *reinterpret_cast<const float4*>(&S.k[kg + 8 * j][4 * d4]);
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    s[i][j] = fmaf(qv[i].x, kv[j].x, s[i][j]);
                    s[i][j] = fmaf(qv[i].y, kv[j].y, s[i][j]);
                    s[i][j] = fmaf(qv[i].z, kv[j].z, s[i][j]);
                    s[i][j] = fmaf(qv[i].w, kv[j].w, s[i][j]);
                }
        }
        __syncthreads();  // K_c fully read
        if (c + 1 < nchunks) load_k(c + 1);
        cp_async_commit();
        // online softmax over this chunk; the 8 lanes sharing rg hold a row's 64 keys
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float cmax = -INFINITY;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int key = c * PF_C + kg + 8 * j;
                s[i][j] = key <= qpos[i] ? __fmul_rn(s[i][j], scale) : -INFINITY;
                cmax = fmaxf(cmax, s[i][j]);
            }
            cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 1));
            cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 2));
            cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 4));
            const float mn = fmaxf(m[i], cmax);  // finite: key 0 of chunk 0 is visible to every row
            const float alpha = expf(m[i] - mn);
            float rs = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const float e = expf(s[i][j] - mn);
                S.p[rg + 32 * i][kg + 8 * j] = e;
                rs += e;
            }
            rs += __shfl_xor_sync(0xffffffffu, rs, 1);
            rs += __shfl_xor_sync(0xffffffffu, rs, 2);
            rs += __shfl_xor_sync(0xffffffffu, rs, 4);
            l[i] = fmaf(l[i], alpha, rs);
            m[i] = mn;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                o[i][j].x *= alpha;
                o[i][j].y *= alpha;
                o[i][j].z *= alpha;
                o[i][j].w *= alpha;
            }
        }
        cp_async_wait<1>();  // V_c has landed (K_{c+1} may still be in flight)
        __syncthreads();
#pragma unroll 2
        for (int kk = 0; kk < PF_C; kk += 4) {
            float4 pv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) pv[i] = *reinterpret_cast<const float4*>(&S.p[rg + 32 * i][kk]);
#pragma unroll
            for (int u = 0; u < 4; u++) {
                float4 vv[4];
#pragma unroll
                for (int j = 0; j < 4; j++) vv[j] = *reinterpret_cast<const float4*>(&S.v[kk + u][4 * (kg + 8 * j)]);
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float pu = u == 0 ? pv[i].x : u == 1 ? pv[i].y : u == 2 ? pv[i].z : pv[i].w;
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        o[i][j].x = fmaf(pu, vv[j].x, o[i][j].x);
                        o[i][j].y = fmaf(pu, vv[j].y, o[i][j].y);
                        o[i][j].z = fmaf(pu, vv[j].z, o[i][j].z);
                        o[i][j].w = fmaf(pu, vv[j].w, o[i][j].w);
                    }
                }
            }
        }
        __syncthreads();  // V_c and P fully read
        if (c + 1 < nchunks) load_v(c + 1);
        cp_async_commit();
    }
    cp_async_wait<0>();

    // normalise into the (now free) query rows, then write f32 and/or Q8_0 row slices
#pragma unroll
    for (int i = 0; i < 4; i++) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            float4 v = o[i][j];
            v.x = __fdiv_rn(v.x, l[i]);
            v.y = __fdiv_rn(v.y, l[i]);
            v.z = __fdiv_rn(v.z, l[i]);
            v.w = __fdiv_rn(v.w, l[i]);
            *reinterpret_cast<float4*>(&S.q[rg + 32 * i][4 * (kg + 8 * j)]) = v;
        }
    }
    __syncthreads();
    const int warp = t >> 5, lane = t & 31;
    for (int r = warp; r < PF_ROWS; r += PF_THREADS / 32) {
        const int g = r / TQ, lq = r - (r / TQ) * TQ;
        if (lq >= nq) continue;
        const int64_t row = (int64_t)b * L + l0 + lq;
        const int64_t e0 = row * p.Hq * D + (int64_t)(kvh * G + g) * D;
#pragma unroll
        for (int blk = 0; blk < D / 32; blk++) {
            const float v = S.q[r][blk * 32 + lane];
            const int64_t e = e0 + blk * 32 + lane;
            if (p.out) p.out[e] = v;
            if (p.xq) pf_quant_warp32(v, lane, p.xq + (e - lane), p.xd + (e >> 5));
        }
    }
}

bool attention_prefill_supported(int64_t L, int64_t Hq, int64_t Hkv) {
    const int64_t G = Hq / Hkv;
    return L >= 16 && (G == 1 || G == 2 || G == 4 || G == 8) && getenv("LQ_ATTN_CHUNKED") == nullptr;
}

int launch_attention_prefill(lq_ctx* ctx, const float* q, const float* kc, const float* vc, int64_t B, int64_t Hq,
                             int64_t Hkv, int64_t L, int64_t pos0, const int32_t* pos0_dev, int64_t ctx_max,
                             float* out, int8_t* xq, uint16_t* xd) {
    PfParams p = {};
    p.q = q;
    p.kc = kc;
    p.vc = vc;
    p.Hq = (int)Hq;
    p.Hkv = (int)Hkv;
    p.L = (int)L;
    p.G = (int)(Hq / Hkv);
    p.TQ = PF_ROWS / p.G;
    p.pos0 = (int)pos0;
    p.pos0_dev = pos0_dev;
    p.ctx_max = (int)ctx_max;
    p.ntiles = ceil_div(L, p.TQ);
    p.out = out;
    p.xq = xq;
    p.xd = xd;
    if (const int rc = ensure_func_smem(ctx, (const void*)attn_prefill_kernel, sizeof(PfSmem))) return rc;
    const dim3 grid((unsigned)p.ntiles, (unsigned)Hkv, (unsigned)B);
    return launch_kernel(ctx, attn_prefill_kernel, grid, dim3(PF_THREADS), sizeof(PfSmem), "attn_prefill", p);
}

}  // namespace lq
