// lq8_attention.cu -- GQA attention over the f32 KV cache (attention.rs:366-399, repeat_kv
// attention.rs:426-456, causal mask causal_mask.rs:104-164), split over key positions.
//
// A CTA owns (one query row, one kv head, one chunk of ATT_C positions) and all G = Hq/Hkv
// query heads that share the kv head. It stages the chunk's K and V rows into shared memory
// with every 16-byte async copy in flight at once (rows of earlier positions before pdl_wait,
// since earlier steps wrote them), computes the G score rows (each score a 128-term dot in
// dimension order, then the scale), a chunk softmax (max, exp, sum) and the chunk's P.V.
// Fused decode variant: the last CTA of a (row, kv head) to finish -- found with an atomic
// counter -- merges the chunks (rescaling by exp(m_s - M)) and writes the [Hq*D] output row
// in f32 and/or Q8_0 for o_proj. Unfused variant: a merge kernel follows.
//
// The decode variant (FUSED) also performs the step before it: from the fused q|k|v
// projection row it computes the G query heads' RMSNorm + RoPE into shared memory, and the
// CTA whose chunk holds the new position computes that position's k (RMSNorm + RoPE) and v,
// uses them from shared memory and appends them to the caches.
#include <type_traits>

#include "lq8_async.cuh"
#include "lq8_fused.cuh"
#include "lq8_internal.cuh"

namespace lq {

constexpr int ATT_C = 64;           // key positions per chunk
constexpr int ATT_D = 128;          // head_dim
constexpr int ATT_KS = ATT_D + 4;   // padded K row stride in floats: conflict-free float4 reads
constexpr int ATT_G = 8;            // max query heads per kv head
constexpr int ATT_THREADS = 128;
constexpr int ATT_SLICE = 256;      // query rows per launch (bounds the partials)
constexpr int ATT_MAX_SPLITS = 128; // chunks per row: contexts up to 8192 positions
constexpr int ATT_MAX_KV = 64;
// scratch: [counters: fixed ATT_SLICE*ATT_MAX_KV ints][part_ml][part_o]. The counter region
// has the same place and size for every call, so launches with different row counts sharing
// one scratch never overlap counters with another launch's partials.
constexpr size_t ATT_COUNTER_BYTES = (size_t)ATT_SLICE * ATT_MAX_KV * 4;

constexpr int ATT_CM_FLOATS = ATT_G * ATT_MAX_SPLITS;  // merge weights [G][ATT_MAX_SPLITS]

struct AttSmem {
    float ks[ATT_C][ATT_KS];
    float vs[ATT_C][ATT_D];
    float qs[ATT_G][ATT_D];
    float ps[ATT_G][ATT_C];
    float ml[ATT_G][2];
    float cl[ATT_G];                  // combine: total denominator
    int last;
};

// The unfused variant (query rows from a q tensor: short prefills) has its own layout: q heads
// with the second half of the dims shifted by 4 floats (so that the two halves of a warp read q
// with one broadcast wavefront), scores by position (so that P.V reads a position's 8
// probabilities with two broadcast loads). Both variants keep the merge weights
// exp(m_s - M) in the last 4 KiB of the V staging area (free once the chunk's P.V is done),
// which keeps each struct small enough for three CTAs per SM.
struct AttSmemR {
    float ks[ATT_C][ATT_KS];
    float vs[ATT_C][ATT_D];
    float qp[ATT_G][ATT_KS];
    float pt[ATT_C][ATT_G];
    float ml[ATT_G][2];
    float cl[ATT_G];
    int last;
};

struct AttParams {
    const float* q;        // [B][Hq][L][D] (unfused)
    const float* qkv;      // [B][(Hq+2Hkv)*D] (fused decode)
    const uint16_t* qn;
    const uint16_t* kn;
    float eps;
    const float* cos_t;
    const float* sin_t;
    float* kc;             // [B][Hkv][ctx_max][D]
    float* vc;
    int Hq, Hkv, L, pos0;
    const int32_t* pos0_dev;
    int ctx_max, row0, nsplit;
    float* part_o;
    float* part_ml;
    int* counters;
    float* out;
    int8_t* xq;
    uint16_t* xd;
    int rows;              // query rows of the launch (streamed decode kernel)
    int ring;              // 1: chunk partials of the ring kernel (ranges of 32-position sub-chunks)
    int* err;
};

// two-lane fused multiply-add (sm_100 packed f32x2): (a.x*b.x + c.x, a.y*b.y + c.y), through the
// compiler's builtin so that the operand pairs stay where the register allocator puts them
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

__device__ __forceinline__ void quant_warp32(float v, int lane, int8_t* q_out, uint16_t* d_out) {
    float amax = warp_max(fabsf(v));
    float d, id;
    q8_scale(amax, d, id);
    q_out[lane] = (int8_t)q8_quant(v, id);
    if (lane == 0) *d_out = f2h(d);
}

__device__ __forceinline__ float* att_cm(AttSmem& S) { return &S.vs[0][0] + ATT_C * ATT_D - ATT_CM_FLOATS; }
__device__ __forceinline__ float* att_cm(AttSmemR& S) { return &S.vs[0][0] + ATT_C * ATT_D - ATT_CM_FLOATS; }

// Unfused chunk: scores (thread -> position tid/2 and one 64-dim half, all GN heads; the halves
// meet by a shuffle), per-head chunk softmax, P.V (thread -> dim, all heads), partials out.
// S: AttSmemR, or a view with the same members (ks, vs, qp, pt, ml) over one ring stage; BAR:
// 0 = __syncthreads, else the named barrier of the ATT_THREADS computing threads
template <int GN, int BAR = 0, typename SM>
__device__ __forceinline__ void attn_chunk_fma(SM& S, int G, int cnt, float scale, int tid,
                                               const AttParams& p, int64_t hbase, int nsplit) {
    const int lane = tid & 31, warp = tid >> 5;
    {
        const int pp = tid >> 1, hf = tid & 1;
        float s[GN];
        float2 s2[GN];  // even and odd dims apart (two-lane fused multiply-add)
#pragma unroll
        for (int g = 0; g < GN; g++) s2[g] = make_float2(0.0f, 0.0f);
        if (pp < cnt) {
            const float* kr = &S.ks[pp][hf * (ATT_D / 2)];
            const float* qr = &S.qp[0][hf * (ATT_D / 2 + 4)];
#pragma unroll 4
            for (int d4 = 0; d4 < ATT_D / 8; d4++) {
                const float4 k4 = *reinterpret_cast<const float4*>(kr + 4 * d4);
#pragma unroll
                for (int g = 0; g < GN; g++) {
                    if (g < G) {
                        const float4 q4 = *reinterpret_cast<const float4*>(qr + g * ATT_KS + 4 * d4);
                        s2[g] = fma2(make_float2(q4.x, q4.y), make_float2(k4.x, k4.y), s2[g]);
                        s2[g] = fma2(make_float2(q4.z, q4.w), make_float2(k4.z, k4.w), s2[g]);
                    }
                }
            }
        }
#pragma unroll
        for (int g = 0; g < GN; g++) {
            s[g] = __fadd_rn(s2[g].x, s2[g].y);
            s[g] = __fadd_rn(s[g], __shfl_xor_sync(0xffffffffu, s[g], 1));
        }
        // half 0 stores heads 0..3, half 1 heads 4..7
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int g = 4 * hf + i;
            float v = 0.0f;
            if (i < GN) v = s[i < GN ? i : 0];
            if (GN > 4 && hf) v = s[4 + i < GN ? 4 + i : 0];
            if (g < G) S.pt[pp][g] = pp < cnt ? __fmul_rn(v, scale) : -INFINITY;
        }
    }
    group_sync<ATT_THREADS, BAR>();
    for (int g = warp; g < G; g += ATT_THREADS / 32) {
        const float a = S.pt[lane][g], c = S.pt[lane + 32][g];
        const float m = warp_max(fmaxf(a, c));
        const float ea = expf(__fsub_rn(a, m)), ec = expf(__fsub_rn(c, m));
        S.pt[lane][g] = ea;
        S.pt[lane + 32][g] = ec;
        const float sum = warp_sum(__fadd_rn(ea, ec));
        if (lane == 0) { S.ml[g][0] = m; S.ml[g][1] = sum; }
    }
    group_sync<ATT_THREADS, BAR>();
    {
        const int d = tid;
        float acc[GN];
        constexpr int GP = (GN + 1) / 2;  // head pairs (two-lane fused multiply-add)
        float2 a2[GP];
#pragma unroll
        for (int i = 0; i < GP; i++) a2[i] = make_float2(0.0f, 0.0f);
#pragma unroll 4
        for (int j = 0; j < cnt; j++) {
            const float vv = S.vs[j][d];
            const float2 v2 = make_float2(vv, vv);
            const float4 pa = *reinterpret_cast<const float4*>(&S.pt[j][0]);
            a2[0] = fma2(make_float2(pa.x, pa.y), v2, a2[0]);
            if constexpr (GN > 2) a2[1] = fma2(make_float2(pa.z, pa.w), v2, a2[1]);
            if constexpr (GN > 4) {
                const float4 pb = *reinterpret_cast<const float4*>(&S.pt[j][4]);
                a2[2] = fma2(make_float2(pb.x, pb.y), v2, a2[2]);
                a2[3] = fma2(make_float2(pb.z, pb.w), v2, a2[3]);
            }
        }
#pragma unroll
        for (int g = 0; g < GN; g++) acc[g] = (g & 1) ? a2[g >> 1].y : a2[g >> 1].x;
#pragma unroll
        for (int g = 0; g < GN; g++)
            if (g < G) p.part_o[(hbase + (int64_t)g * nsplit) * ATT_D + d] = acc[g];
        if (tid < G) {
            p.part_ml[(hbase + (int64_t)tid * nsplit) * 2] = S.ml[tid][0];
            p.part_ml[(hbase + (int64_t)tid * nsplit) * 2 + 1] = S.ml[tid][1];
        }
    }
}

// FUSED: the decode step's fused variant: each score one fused multiply-add chain over the 128
// dimensions in order, each P.V output one chain over the positions in order (the persistent
// decode kernel computes the same chains, bit for bit). Unfused: GT query heads per kv head
// (0: any G <= 8), two-lane packed multiply-adds and each score's two 64-dim halves added at
// the end.
template <bool FUSED, int GT>
__global__ void __launch_bounds__(ATT_THREADS) attn_chunk_kernel(const AttParams p) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    using Smem = typename std::conditional<FUSED, AttSmem, AttSmemR>::type;
    Smem& S = *reinterpret_cast<Smem*>(smem_raw);
    const int Hq = p.Hq, Hkv = p.Hkv, L = p.L, ctx_max = p.ctx_max, nsplit = p.nsplit;
    const int G = GT ? GT : Hq / Hkv;
    const int split = blockIdx.x, kvh = blockIdx.y, lrow = blockIdx.z;
    const int row = p.row0 + lrow;  // b*L + l
    const int b = row / L, l = row - (row / L) * L;
    const int p0 = p.pos0_dev ? *p.pos0_dev : p.pos0;  // written by an earlier step: safe before pdl_wait
    const int limit = p0 + l;  // last visible position
    if (limit < 0 || limit >= ctx_max) return;
    const int n_active = min(limit / ATT_C + 1, nsplit);
    if (split >= n_active) return;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int j0 = split * ATT_C;
    const int cnt = min(ATT_C, limit + 1 - j0);
    float* kbase = p.kc + ((int64_t)b * Hkv + kvh) * (int64_t)ctx_max * ATT_D + (int64_t)j0 * ATT_D;
    float* vbase = p.vc + ((int64_t)b * Hkv + kvh) * (int64_t)ctx_max * ATT_D + (int64_t)j0 * ATT_D;
    // every 16-byte piece of the chunk's K and V rows in flight at once. Rows of positions
    // before p0 were appended by earlier steps and are read before pdl_wait(); the rows of
    // this launch's positions are produced by the preceding kernel (or, fused, right here).
    const int fresh = p0 - j0;  // chunk rows r >= fresh belong to this launch
    for (int i = tid; i < cnt * (ATT_D / 4); i += ATT_THREADS) {
        const int r = i / (ATT_D / 4), c = (i % (ATT_D / 4)) * 4;
        if (r < fresh) {
            cp_async16(&S.ks[r][c], kbase + (int64_t)r * ATT_D + c, true);
            cp_async16(&S.vs[r][c], vbase + (int64_t)r * ATT_D + c, true);
        }
    }
    pdl_wait();
    pdl_trigger();
    if constexpr (FUSED) {
        // q heads: per-head RMSNorm + RoPE at position p0 (decode: L == 1)
        const int heads = Hq + 2 * Hkv;
        const float* qrow = p.qkv + (int64_t)b * heads * ATT_D;
        const float* cs = p.cos_t + (int64_t)p0 * (ATT_D / 2);
        const float* sn = p.sin_t + (int64_t)p0 * (ATT_D / 2);
        for (int g = warp; g < G; g += ATT_THREADS / 32)
            head_norm_rope(qrow + (int64_t)(kvh * G + g) * ATT_D, p.qn, p.eps, cs, sn, lane, S.qs[g]);
        if (fresh >= 0 && fresh < cnt) {
            // this chunk holds the new position: compute its k and v, use and append them
            if (warp == 0) {
                head_norm_rope(qrow + (int64_t)(Hq + kvh) * ATT_D, p.kn, p.eps, cs, sn, lane, S.ks[fresh]);
                __syncwarp();
                const float4 kk = *reinterpret_cast<const float4*>(&S.ks[fresh][lane * 4]);
                *reinterpret_cast<float4*>(kbase + (int64_t)fresh * ATT_D + lane * 4) = kk;
            } else if (warp == 1) {
                const float4 vv =
                    *reinterpret_cast<const float4*>(qrow + (int64_t)(Hq + Hkv + kvh) * ATT_D + lane * 4);
                *reinterpret_cast<float4*>(&S.vs[fresh][lane * 4]) = vv;
                *reinterpret_cast<float4*>(vbase + (int64_t)fresh * ATT_D + lane * 4) = vv;
            }
        }
        cp_async_commit();
    } else {
        for (int i = tid; i < cnt * (ATT_D / 4); i += ATT_THREADS) {
            const int r = i / (ATT_D / 4), c = (i % (ATT_D / 4)) * 4;
            if (r >= fresh) {
                cp_async16(&S.ks[r][c], kbase + (int64_t)r * ATT_D + c, true);
                cp_async16(&S.vs[r][c], vbase + (int64_t)r * ATT_D + c, true);
            }
        }
        cp_async_commit();
        for (int i = tid; i < G * ATT_D; i += ATT_THREADS) {
            const int g = i / ATT_D, d = i % ATT_D;
            S.qp[g][d + (d >= ATT_D / 2 ? 4 : 0)] = p.q[(((int64_t)b * Hq + kvh * G + g) * L + l) * ATT_D + d];
        }
    }
    cp_async_wait<0>();
    __syncthreads();

    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)ATT_D));
    if constexpr (!FUSED) {
        attn_chunk_fma<GT ? GT : ATT_G>(S, G, cnt, scale, tid, p, ((int64_t)lrow * Hq + (int64_t)kvh * G) * nsplit + split,
                                        nsplit);
    } else {
    // scores: thread -> (position pp, heads half, half+2, ...); one multiply-add chain over d
    {
        const int pp = tid % ATT_C, half = tid / ATT_C;
        float s[ATT_G / 2];
#pragma unroll
        for (int i = 0; i < ATT_G / 2; i++) s[i] = 0.0f;
        if (pp < cnt) {
#pragma unroll 8
            for (int d4 = 0; d4 < ATT_D / 4; d4++) {
                const float4 k4 = *reinterpret_cast<const float4*>(&S.ks[pp][4 * d4]);
#pragma unroll
                for (int i = 0; i < ATT_G / 2; i++) {
                    const int g = half + 2 * i;
                    if (g < G) {
                        const float4 q4 = *reinterpret_cast<const float4*>(&S.qs[g][4 * d4]);
                        s[i] = fmaf(q4.x, k4.x, s[i]);
                        s[i] = fmaf(q4.y, k4.y, s[i]);
                        s[i] = fmaf(q4.z, k4.z, s[i]);
                        s[i] = fmaf(q4.w, k4.w, s[i]);
                    }
                }
            }
        }
#pragma unroll
        for (int i = 0; i < ATT_G / 2; i++) {
            const int g = half + 2 * i;
            if (g < G) S.ps[g][pp] = pp < cnt ? __fmul_rn(s[i], scale) : -INFINITY;
        }
    }
    __syncthreads();
    // chunk softmax per head: max, exp(s - max), sum
    for (int g = warp; g < G; g += ATT_THREADS / 32) {
        const float a = S.ps[g][lane], c = S.ps[g][lane + 32];
        const float m = warp_max(fmaxf(a, c));
        const float ea = expf(__fsub_rn(a, m)), ec = expf(__fsub_rn(c, m));
        S.ps[g][lane] = ea;
        S.ps[g][lane + 32] = ec;
        const float sum = warp_sum(__fadd_rn(ea, ec));
        if (lane == 0) { S.ml[g][0] = m; S.ml[g][1] = sum; }
    }
    __syncthreads();
    // chunk P.V: thread = dim
    {
        const int d = tid;
        float acc[ATT_G];
#pragma unroll
        for (int g = 0; g < ATT_G; g++) acc[g] = 0.0f;
        for (int j = 0; j < cnt; j++) {
            const float vv = S.vs[j][d];
#pragma unroll
            for (int g = 0; g < ATT_G; g++)
                if (g < G) acc[g] = fmaf(S.ps[g][j], vv, acc[g]);
        }
        const int64_t hbase = ((int64_t)lrow * Hq + (int64_t)kvh * G) * nsplit + split;
#pragma unroll
        for (int g = 0; g < ATT_G; g++)
            if (g < G) p.part_o[(hbase + (int64_t)g * nsplit) * ATT_D + d] = acc[g];
        if (tid < G) {
            p.part_ml[(hbase + (int64_t)tid * nsplit) * 2] = S.ml[tid][0];
            p.part_ml[(hbase + (int64_t)tid * nsplit) * 2 + 1] = S.ml[tid][1];
        }
    }
    }
    // unfused: attn_merge_kernel, launched next, merges the chunks
    if constexpr (!FUSED) return;
    // the last chunk CTA of this (row, kv head) merges the chunks
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const int prev = atomicAdd(&p.counters[lrow * Hkv + kvh], 1);
        S.last = (prev == n_active - 1);
    }
    __syncthreads();
    if (!S.last) return;
    __threadfence();
    const int64_t hbase0 = ((int64_t)lrow * Hq + (int64_t)kvh * G) * nsplit;
    // bring each head's chunk partials into shared memory (the free K/V staging area, two head
    // buffers) with all 16-byte copies of a head in flight at once, the next head's copies
    // overlapping the current head's sum: one L2 round trip per head instead of a chain of
    // dependent loads
    float* po = &S.ks[0][0];
    float* cm = att_cm(S);  // [G][ATT_MAX_SPLITS]
    const size_t head_floats = (size_t)n_active * ATT_D;
    const bool staged = 2 * head_floats * 4 <= sizeof(S.ks) + sizeof(S.vs) - ATT_CM_FLOATS * 4;
    auto stage_head = [&](int g) {
        float* dst = po + (size_t)(g & 1) * head_floats;
        for (int i = tid; i < n_active * (ATT_D / 4); i += ATT_THREADS) {
            const int s = i / (ATT_D / 4), c = (i % (ATT_D / 4)) * 4;
            cp_async16(dst + (size_t)s * ATT_D + c, p.part_o + (hbase0 + (int64_t)g * nsplit + s) * ATT_D + c, true);
        }
        cp_async_commit();
    };
    if (staged) {
        stage_head(0);
        if (G > 1) stage_head(1);
    }
    for (int g = warp; g < G; g += ATT_THREADS / 32) {
        float m = -INFINITY;
        for (int s = lane; s < n_active; s += 32)
            m = fmaxf(m, ld_cg(&p.part_ml[(hbase0 + (int64_t)g * nsplit + s) * 2]));
        m = warp_max(m);
        float lsum = 0.0f;
        for (int s = lane; s < n_active; s += 32) {
            const float w = expf(__fsub_rn(ld_cg(&p.part_ml[(hbase0 + (int64_t)g * nsplit + s) * 2]), m));
            cm[g * ATT_MAX_SPLITS + s] = w;
            lsum = __fadd_rn(lsum, __fmul_rn(w, ld_cg(&p.part_ml[(hbase0 + (int64_t)g * nsplit + s) * 2 + 1])));
        }
        lsum = warp_sum(lsum);
        if (lane == 0) S.cl[g] = lsum;
    }
    __syncthreads();
    const int d = tid;
    for (int g = 0; g < G; g++) {
        float o = 0.0f;
        if (staged) {
            if (g + 1 < G) cp_async_wait<1>();
            else cp_async_wait<0>();
            __syncthreads();
            const float* pg = po + (size_t)(g & 1) * head_floats + d;
            for (int s = 0; s < n_active; s++)
                o = __fadd_rn(o, __fmul_rn(cm[g * ATT_MAX_SPLITS + s], pg[(size_t)s * ATT_D]));
            __syncthreads();  // this buffer is refilled next
            if (g + 2 < G) stage_head(g + 2);
        } else {
#pragma unroll 8
            for (int s = 0; s < n_active; s++)
                o = __fadd_rn(o, __fmul_rn(cm[g * ATT_MAX_SPLITS + s],
                                           ld_cg(&p.part_o[(hbase0 + (int64_t)g * nsplit + s) * ATT_D + d])));
        }
        o = __fdiv_rn(o, S.cl[g]);
        const int64_t e = (int64_t)row * Hq * ATT_D + (int64_t)(kvh * G + g) * ATT_D + d;
        if (p.out) p.out[e] = o;
        if (p.xq) quant_warp32(o, lane, p.xq + (e - lane), p.xd + (e >> 5));
    }
    if (tid == 0) p.counters[lrow * Hkv + kvh] = 0;  // ready for the next launch
}

// =========================================================================================
// Unfused chunk kernel (query rows from a q tensor: batched decode rows and short prefills).
// A fixed number of CTAs per (query row, kv head) -- nsplit, about three CTAs per SM over all
// pairs -- each owns a contiguous range of the visible positions, cut into 32-position
// sub-chunks that stream through a two-stage ring in shared memory: a sub-chunk's K rows (one
// bulk copy per row, into padded slots) and V rows (one bulk copy) land on the stage's two
// mbarriers while the other stage is computed, so one CTA's copies and arithmetic overlap and
// its fixed costs (position read, barrier set-up, query load) are paid once per range. The rows
// written before this step are requested before pdl_wait, the rows of this launch's positions
// after it. Per sub-chunk: scores (thread -> (position, 64-dim half, 2 heads), two-lane packed
// multiply-adds; the halves added through shared memory, then the scale), an online softmax
// per head (one warp per head: running max m and sum l, the P.V sums rescaled by
// exp(m_old - m_new)) and P.V (thread -> (dimension, 4 heads)). Out: one partial (o, m, l) per
// (head, range) for attn_merge_kernel (ring mode). 256 threads, three CTAs per SM.
// =========================================================================================
constexpr int ATB_THREADS = 256;
constexpr int ATB_QS = ATT_D + 12;  // q row stride: halves 4 floats apart (one broadcast wavefront)
constexpr int ATB_P = 32;           // positions per sub-chunk
constexpr int ATB_CTAS_PER_SM = 3;

struct AttSmemB {
    float ks[2][ATB_P][ATT_KS];       // K rows, padded: conflict-free float4 reads by position
    float vs[2][ATB_P][ATT_D];
    float qp[ATT_G][ATB_QS];          // query heads
    float sp[2][ATB_P][ATT_G];        // partial scores of the two dim halves
    float pt[ATB_P][ATT_G];           // probabilities of the current sub-chunk
    float al[ATT_G];                  // rescale of the running P.V sums
    float kn[ATT_D], vn[ATT_D];       // QKV: the new position's k (normalised, rotated) and v
    uint64_t kbar[2], vbar[2];        // per stage: K rows, V rows
    int fail;
};

// sub-chunks of 32 positions per CTA range (ring mode), from the number to attend
__device__ __forceinline__ int ring_per(int nsub, int nsplit) { return (nsub + nsplit - 1) / nsplit; }

// QKV (decode rows, L == 1, device position): the kernel also does the step before it, from the
// fused q|k|v projection rows: the G query heads' RMSNorm + RoPE into shared memory, and, in the
// CTA whose range holds the new position, that position's k (RMSNorm + RoPE) and v, used from
// shared memory and appended to the caches. Every cache row it copies then predates this step,
// so all its copies go out before pdl_wait.
template <int GT, bool QKV>
__global__ void __launch_bounds__(ATB_THREADS, ATB_CTAS_PER_SM) attn_chunk_bulk_kernel(const AttParams p) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    AttSmemB& S = *reinterpret_cast<AttSmemB*>(smem_raw);
    const int Hq = p.Hq, Hkv = p.Hkv, L = p.L, ctx_max = p.ctx_max, nsplit = p.nsplit;
    const int G = GT ? GT : Hq / Hkv;
    const int split = blockIdx.x, kvh = blockIdx.y, lrow = blockIdx.z;
    const int row = p.row0 + lrow;  // b*L + l
    const int b = row / L, l = row - (row / L) * L;
    const int p0 = p.pos0_dev ? *p.pos0_dev : p.pos0;  // written by an earlier step: safe before pdl_wait
    const int limit = p0 + l;  // last visible position
    if (limit < 0 || limit >= ctx_max) return;
    const int nsub = limit / ATB_P + 1;
    const int per = ring_per(nsub, nsplit);
    const int j0 = split * per, j1 = min(nsub, j0 + per);
    if (j0 >= j1) return;
    const int nj = j1 - j0;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t slab = ((int64_t)b * Hkv + kvh) * (int64_t)ctx_max * ATT_D;
    float* kbase = p.kc + slab;
    float* vbase = p.vc + slab;
    auto cnt_of = [&](int j) { return min(ATB_P, limit + 1 - ATB_P * j); };
    // rows copied from the caches: QKV leaves out the new position (computed here)
    auto copied_of = [&](int j) { return cnt_of(j) - (QKV && ATB_P * j + cnt_of(j) - 1 >= p0 ? 1 : 0); };
    if (tid == 0) {
        for (int i = 0; i < 2; i++) {
            mbar_init(&S.kbar[i], 1);
            mbar_init(&S.vbar[i], 1);
        }
        mbar_fence_init();
        for (int i = 0; i < 2 && i < nj; i++) {
            mbar_expect_tx(&S.kbar[i], (unsigned)(copied_of(j0 + i) * ATT_D * 4));
            mbar_expect_tx(&S.vbar[i], (unsigned)(copied_of(j0 + i) * ATT_D * 4));
        }
        S.fail = 0;
    }
    __syncthreads();
    // copies of sub-chunk j into stage st: K row r by thread r, V rows by thread 64 + st; rows of
    // positions before p0 (earlier steps) when pass 0, from p0 on (this launch's) when pass 1, all
    // when pass 2 (QKV: never the row of p0)
    auto issue = [&](int j, int st, int pass) {
        const int c = cnt_of(j), base = ATB_P * j;
        if (tid < c) {
            const bool pre = base + tid < p0;
            if ((pass == 2 || (pass == 0) == pre) && !(QKV && base + tid >= p0))
                bulk_g2s(&S.ks[st][tid][0], kbase + (int64_t)(base + tid) * ATT_D, ATT_D * 4, &S.kbar[st]);
        }
        if (tid == 64 + st) {
            const int r0 = pass == 1 ? max(base, p0) : base;
            const int r1 = (pass == 0 || QKV) ? min(base + c, p0) : base + c;
            if (r1 > r0)
                bulk_g2s(&S.vs[st][r0 - base][0], vbase + (int64_t)r0 * ATT_D, (unsigned)((r1 - r0) * ATT_D * 4),
                         &S.vbar[st]);
        }
    };
    for (int i = 0; i < 2 && i < nj; i++) issue(j0 + i, i, 0);
    pdl_wait();
    pdl_trigger();
    if constexpr (QKV) {
        // q heads: per-head RMSNorm + RoPE at position p0 (the second half 4 floats further on)
        const int heads = Hq + 2 * Hkv;
        const float* qrow = p.qkv + (int64_t)b * heads * ATT_D;
        const float* cs = p.cos_t + (int64_t)p0 * (ATT_D / 2);
        const float* sn = p.sin_t + (int64_t)p0 * (ATT_D / 2);
        if (warp < G) head_norm_rope(qrow + (int64_t)(kvh * G + warp) * ATT_D, p.qn, p.eps, cs, sn, lane, S.qp[warp],
                                     ATT_D / 2 + 4);
        if (j1 == nsub) {  // this range holds the new position: its k and v, appended to the caches
            if (warp == 0) {
                head_norm_rope(qrow + (int64_t)(Hq + kvh) * ATT_D, p.kn, p.eps, cs, sn, lane, S.kn);
                __syncwarp();
                *reinterpret_cast<float4*>(kbase + (int64_t)p0 * ATT_D + 4 * lane) =
                    *reinterpret_cast<const float4*>(&S.kn[4 * lane]);
            } else if (warp == 1) {
                const float4 vv = *reinterpret_cast<const float4*>(qrow + (int64_t)(Hq + Hkv + kvh) * ATT_D + 4 * lane);
                *reinterpret_cast<float4*>(&S.vn[4 * lane]) = vv;
                *reinterpret_cast<float4*>(vbase + (int64_t)p0 * ATT_D + 4 * lane) = vv;
            }
        }
    } else {
        for (int i = 0; i < 2 && i < nj; i++) issue(j0 + i, i, 1);
        // query heads (the second half of each row 4 floats further on)
        for (int i = tid; i < G * ATT_D; i += ATB_THREADS) {
            const int g = i / ATT_D, d = i % ATT_D;
            S.qp[g][d + (d >= ATT_D / 2 ? 4 : 0)] = p.q[(((int64_t)b * Hq + kvh * G + g) * L + l) * ATT_D + d];
        }
    }
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)ATT_D));
    float m_run = -INFINITY, l_run = 0.0f;  // warp g < G: head g's running max and sum
    float2 a2[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
    const int sd = tid & (ATT_D - 1), sgh = tid >> 7;  // P.V: dimension, heads 4 sgh .. 4 sgh + 3
    // bounded waits by thread 0; after a failure the kernel still waits (briefly) for every copy it
    // issued and finishes on whatever landed, so no copy outlives the CTA; the error is reported
    auto wait_bar = [&](uint64_t* bar, unsigned par) {
        if (tid == 0 && !mbar_wait_sleep(bar, par, S.fail ? 1000000ull : 2000000000ull)) {
            if (!S.fail && p.err) atomicCAS(p.err, 0, 72);
            S.fail = 1;
        }
    };
#pragma unroll 1
    for (int i = 0; i < nj; i++) {
        const int st = i & 1, j = j0 + i, ch = cnt_of(j);
        const unsigned par = (unsigned)(i >> 1) & 1u;
        wait_bar(&S.kbar[st], par);
        __syncthreads();
        {
            const int pp = lane, hf = warp & 1, gq = warp >> 1;  // position, dim half, heads 2gq, 2gq+1
            float2 s2[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
            if (pp < ch && 2 * gq < G) {
                const float* kr = (QKV && ATB_P * j + pp == p0) ? &S.kn[hf * (ATT_D / 2)] : &S.ks[st][pp][hf * (ATT_D / 2)];
                const float* qr = &S.qp[2 * gq][hf * (ATT_D / 2 + 4)];
#pragma unroll 4
                for (int d4 = 0; d4 < ATT_D / 8; d4++) {
                    const float4 k4 = *reinterpret_cast<const float4*>(kr + 4 * d4);
#pragma unroll
                    for (int e = 0; e < 2; e++) {
                        if (2 * gq + e < G) {
                            const float4 q4 = *reinterpret_cast<const float4*>(qr + e * ATB_QS + 4 * d4);
                            s2[e] = fma2(make_float2(q4.x, q4.y), make_float2(k4.x, k4.y), s2[e]);
                            s2[e] = fma2(make_float2(q4.z, q4.w), make_float2(k4.z, k4.w), s2[e]);
                        }
                    }
                }
            }
#pragma unroll
            for (int e = 0; e < 2; e++)
                if (2 * gq + e < G) S.sp[hf][pp][2 * gq + e] = __fadd_rn(s2[e].x, s2[e].y);
        }
        __syncthreads();
        if (warp < G) {
            const int g = warp;
            const float sv = lane < ch ? __fmul_rn(__fadd_rn(S.sp[0][lane][g], S.sp[1][lane][g]), scale) : -INFINITY;
            const float mn = fmaxf(m_run, warp_max(sv));
            const float pv = expf(__fsub_rn(sv, mn));
            const float ps = warp_sum(pv);
            const float a = expf(__fsub_rn(m_run, mn));  // 0 on the first sub-chunk (m_run = -inf)
            S.pt[lane][g] = pv;
            if (lane == 0) S.al[g] = a;
            l_run = __fadd_rn(__fmul_rn(l_run, a), ps);
            m_run = mn;
        }
        wait_bar(&S.vbar[st], par);
        __syncthreads();
        if (4 * sgh < G) {
            const float4 al4 = *reinterpret_cast<const float4*>(&S.al[4 * sgh]);
            a2[0] = make_float2(__fmul_rn(a2[0].x, al4.x), __fmul_rn(a2[0].y, al4.y));
            a2[1] = make_float2(__fmul_rn(a2[1].x, al4.z), __fmul_rn(a2[1].y, al4.w));
#pragma unroll 4
            for (int r = 0; r < ch; r++) {
                const float vv = (QKV && ATB_P * j + r == p0) ? S.vn[sd] : S.vs[st][r][sd];
                const float2 v2 = make_float2(vv, vv);
                const float4 pr = *reinterpret_cast<const float4*>(&S.pt[r][4 * sgh]);
                a2[0] = fma2(make_float2(pr.x, pr.y), v2, a2[0]);
                a2[1] = fma2(make_float2(pr.z, pr.w), v2, a2[1]);
            }
        }
        const bool refill = i + 2 < nj;
        if (refill && tid == 0) {
            mbar_expect_tx(&S.kbar[st], (unsigned)(copied_of(j + 2) * ATT_D * 4));
            mbar_expect_tx(&S.vbar[st], (unsigned)(copied_of(j + 2) * ATT_D * 4));
        }
        __syncthreads();  // stage st, pt, al and sp are free again
        if (refill) issue(j + 2, st, 2);
    }
    const int64_t hbase = ((int64_t)lrow * Hq + (int64_t)kvh * G) * nsplit + split;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int g = 4 * sgh + i;
        if (g < G) p.part_o[(hbase + (int64_t)g * nsplit) * ATT_D + sd] = (i & 1) ? a2[i >> 1].y : a2[i >> 1].x;
    }
    if (warp < G && lane == 0) {
        p.part_ml[(hbase + (int64_t)warp * nsplit) * 2] = m_run;
        p.part_ml[(hbase + (int64_t)warp * nsplit) * 2 + 1] = l_run;
    }
}

// =========================================================================================
// The ring kernel's arithmetic on the tensor cores (the default for batched decode rows; the
// f32 FMA kernel above with LQ_ATT_FMA=1). Same ranges, two-stage ring, copies, online softmax
// and partials; scores and P.V are `mma.sync.m16n8k8` TF32 products with f32 accumulation, each
// f32 operand split as x = big + small (big = tf32(x), small = tf32(x - big)) and every product
// formed as small·big + big·small + big·big, so it keeps ~22 bits of each operand (the dropped
// small·small term is below 2^-22 of the product; the attention tolerance is 2e-5 of the row's
// max). Scores: S^T[position][head] = K·q^T, warp w owns 16 positions (w & 1) and 32 dims
// (w >> 1): 4 k-steps whose K fragments come by ldmatrix from the padded K rows and whose q
// fragments sit in registers for the whole range; the four dim groups' partial scores meet in
// shared memory. P.V: O^T[dim][head] = V^T·P^T, warp w owns 16 dims, 4 k-steps of 8 positions;
// the accumulators stay in registers across the range, rescaled by exp(m_old - m_new). V rows
// arrive one bulk copy per row into slots of 136 floats, so the transposed fragment loads hit
// 32 different banks.
// =========================================================================================
constexpr int ATM_VS = ATT_D + 8;   // V row stride (floats)

struct AttSmemM {
    float ks[2][ATB_P][ATT_KS];       // K rows (stride 132: ldmatrix rows in 8 bank groups)
    float vs[2][ATB_P][ATM_VS];       // V rows
    union {
        float qs[ATT_G][ATT_KS];      // query heads (read once into registers)
        float sp[4][ATB_P][ATT_G + 1]; // the four dim groups' partial scores (padded)
    } u;
    float pt[ATT_G][ATB_P + 4];       // probabilities, [head][position]
    float al[ATT_G];                  // rescale of the running P.V sums
    float kn[ATT_D], vn[ATT_D];       // QKV: the new position's k (normalised, rotated) and v
    uint64_t kbar[2], vbar[2];
    int fail;
};

static_assert((sizeof(AttSmemM) + 1024) * ATB_CTAS_PER_SM <= 228 * 1024, "three MMA ring CTAs must fit one SM");
static_assert((sizeof(AttSmemB) + 1024) * ATB_CTAS_PER_SM <= 228 * 1024, "three FMA ring CTAs must fit one SM");

__device__ __forceinline__ uint32_t tf32_big(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}
// x = big + small (both tf32): big = x with its low 13 mantissa bits cleared (exact), small =
// the remainder (exact in f32, at most 2^-10 |x|) rounded to tf32: |x - big - small| <= 2^-22 |x|
__device__ __forceinline__ void tf32_split(float x, uint32_t& big, uint32_t& small) {
    big = __float_as_uint(x) & 0xFFFFE000u;
    small = tf32_big(__fsub_rn(x, __uint_as_float(big)));
}
// D += A(16x8 tf32, row) * B(8x8 tf32, col), f32 accumulate
__device__ __forceinline__ void mma_tf32(float d[4], const uint32_t a[4], const uint32_t b[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
// D += A*B with both operands split: small*big + big*small + big*big
__device__ __forceinline__ void mma_tf32x3(float d[4], const uint32_t ab[4], const uint32_t as[4], const uint32_t bb[2],
                                           const uint32_t bs[2]) {
    mma_tf32(d, as, bb);
    mma_tf32(d, ab, bs);
    mma_tf32(d, ab, bb);
}

template <int GT, bool QKV>
__global__ void __launch_bounds__(ATB_THREADS, ATB_CTAS_PER_SM) attn_chunk_mma_kernel(const AttParams p) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    AttSmemM& S = *reinterpret_cast<AttSmemM*>(smem_raw);
    const int Hq = p.Hq, Hkv = p.Hkv, L = p.L, ctx_max = p.ctx_max, nsplit = p.nsplit;
    const int G = GT ? GT : Hq / Hkv;
    const int split = blockIdx.x, kvh = blockIdx.y, lrow = blockIdx.z;
    const int row = p.row0 + lrow;  // b*L + l
    const int b = row / L, l = row - (row / L) * L;
    const int p0 = p.pos0_dev ? *p.pos0_dev : p.pos0;  // written by an earlier step: safe before pdl_wait
    const int limit = p0 + l;  // last visible position
    if (limit < 0 || limit >= ctx_max) return;
    const int nsub = limit / ATB_P + 1;
    const int per = ring_per(nsub, nsplit);
    const int j0 = split * per, j1 = min(nsub, j0 + per);
    if (j0 >= j1) return;
    const int nj = j1 - j0;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;  // fragment row group, thread in group
    const int64_t slab = ((int64_t)b * Hkv + kvh) * (int64_t)ctx_max * ATT_D;
    float* kbase = p.kc + slab;
    float* vbase = p.vc + slab;
    auto cnt_of = [&](int j) { return min(ATB_P, limit + 1 - ATB_P * j); };
    auto copied_of = [&](int j) { return cnt_of(j) - (QKV && ATB_P * j + cnt_of(j) - 1 >= p0 ? 1 : 0); };
    if (tid == 0) {
        for (int i = 0; i < 2; i++) {
            mbar_init(&S.kbar[i], 1);
            mbar_init(&S.vbar[i], 1);
        }
        mbar_fence_init();
        for (int i = 0; i < 2 && i < nj; i++) {
            mbar_expect_tx(&S.kbar[i], (unsigned)(copied_of(j0 + i) * ATT_D * 4));
            mbar_expect_tx(&S.vbar[i], (unsigned)(copied_of(j0 + i) * ATT_D * 4));
        }
        S.fail = 0;
    }
    __syncthreads();
    // copies of sub-chunk j into stage st: K row r by thread r, V row r by thread 64 + r; rows of
    // positions before p0 when pass 0, from p0 on when pass 1, all when pass 2 (QKV: never p0's)
    auto issue = [&](int j, int st, int pass) {
        const int c = cnt_of(j), base = ATB_P * j;
        const int r = tid & 63;
        if (r < c && tid < 128) {
            const bool pre = base + r < p0;
            if ((pass == 2 || (pass == 0) == pre) && !(QKV && base + r >= p0)) {
                if (tid < 64)
                    bulk_g2s(&S.ks[st][r][0], kbase + (int64_t)(base + r) * ATT_D, ATT_D * 4, &S.kbar[st]);
                else
                    bulk_g2s(&S.vs[st][r][0], vbase + (int64_t)(base + r) * ATT_D, ATT_D * 4, &S.vbar[st]);
            }
        }
    };
    for (int i = 0; i < 2 && i < nj; i++) issue(j0 + i, i, 0);
    pdl_wait();
    pdl_trigger();
    if constexpr (QKV) {
        const int heads = Hq + 2 * Hkv;
        const float* qrow = p.qkv + (int64_t)b * heads * ATT_D;
        const float* cs = p.cos_t + (int64_t)p0 * (ATT_D / 2);
        const float* sn = p.sin_t + (int64_t)p0 * (ATT_D / 2);
        if (warp < G) head_norm_rope(qrow + (int64_t)(kvh * G + warp) * ATT_D, p.qn, p.eps, cs, sn, lane, S.u.qs[warp]);
        if (j1 == nsub) {  // this range holds the new position: its k and v, appended to the caches
            if (warp == 0) {
                head_norm_rope(qrow + (int64_t)(Hq + kvh) * ATT_D, p.kn, p.eps, cs, sn, lane, S.kn);
                __syncwarp();
                *reinterpret_cast<float4*>(kbase + (int64_t)p0 * ATT_D + 4 * lane) =
                    *reinterpret_cast<const float4*>(&S.kn[4 * lane]);
            } else if (warp == 1) {
                const float4 vv = *reinterpret_cast<const float4*>(qrow + (int64_t)(Hq + Hkv + kvh) * ATT_D + 4 * lane);
                *reinterpret_cast<float4*>(&S.vn[4 * lane]) = vv;
                *reinterpret_cast<float4*>(vbase + (int64_t)p0 * ATT_D + 4 * lane) = vv;
            }
        }
    } else {
        for (int i = 0; i < 2 && i < nj; i++) issue(j0 + i, i, 1);
        for (int i = tid; i < G * ATT_D; i += ATB_THREADS) {
            const int hh = i / ATT_D, d = i % ATT_D;
            S.u.qs[hh][d] = p.q[(((int64_t)b * Hq + kvh * G + hh) * L + l) * ATT_D + d];
        }
    }
    __syncthreads();
    // this warp's q fragments for its four k-steps (B[k][n] = q[head n][dim k]; heads >= G are 0)
    const int mt = warp & 1, kg = warp >> 1;  // scores: positions 16 mt .., dims 32 kg ..
    uint32_t qb[4][2], qsm[4][2];
#pragma unroll
    for (int ks = 0; ks < 4; ks++) {
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const float v = g < G ? S.u.qs[g][32 * kg + 8 * ks + t + 4 * h] : 0.0f;
            tf32_split(v, qb[ks][h], qsm[ks][h]);
        }
    }
    __syncthreads();  // q is in registers: the union now holds partial scores
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)ATT_D));
    float m_run = -INFINITY, l_run = 0.0f;  // warp h < G: head h's running max and sum
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // O^T rows (dims) 16 warp + g, + 8; cols (heads) 2t, 2t+1
    auto wait_bar = [&](uint64_t* bar, unsigned par) {
        if (tid == 0 && !mbar_wait_sleep(bar, par, S.fail ? 1000000ull : 2000000000ull)) {
            if (!S.fail && p.err) atomicCAS(p.err, 0, 74);
            S.fail = 1;
        }
    };
    const int lr = 16 * mt + (lane & 7) + 8 * ((lane >> 3) & 1);  // the K row this lane addresses
#pragma unroll 1
    for (int i = 0; i < nj; i++) {
        const int st = i & 1, j = j0 + i, ch = cnt_of(j);
        const unsigned par = (unsigned)(i >> 1) & 1u;
        const int fr = (QKV && p0 >= ATB_P * j && p0 < ATB_P * j + ATB_P) ? p0 - ATB_P * j : -1;  // new row
        wait_bar(&S.kbar[st], par);
        __syncthreads();
        {
            float c[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            const float* krow = (lr == fr) ? S.kn : &S.ks[st][lr][0];
#pragma unroll
            for (int ks = 0; ks < 4; ks++) {
                uint32_t a[4], ab[4], as[4];
                ldmatrix_x4(a, krow + 32 * kg + 8 * ks + 4 * (lane >> 4));
#pragma unroll
                for (int e = 0; e < 4; e++) tf32_split(__uint_as_float(a[e]), ab[e], as[e]);
                mma_tf32x3(c, ab, as, qb[ks], qsm[ks]);
            }
            S.u.sp[kg][16 * mt + g][2 * t] = c[0];
            S.u.sp[kg][16 * mt + g][2 * t + 1] = c[1];
            S.u.sp[kg][16 * mt + g + 8][2 * t] = c[2];
            S.u.sp[kg][16 * mt + g + 8][2 * t + 1] = c[3];
        }
        __syncthreads();
        if (warp < G) {
            const int h = warp;
            float sv = -INFINITY;
            if (lane < ch) {
                const float s01 = __fadd_rn(S.u.sp[0][lane][h], S.u.sp[1][lane][h]);
                const float s23 = __fadd_rn(S.u.sp[2][lane][h], S.u.sp[3][lane][h]);
                sv = __fmul_rn(__fadd_rn(s01, s23), scale);
            }
            const float mn = fmaxf(m_run, warp_max(sv));
            const float pv = expf(__fsub_rn(sv, mn));
            const float ps = warp_sum(pv);
            const float a = expf(__fsub_rn(m_run, mn));  // 0 on the first sub-chunk (m_run = -inf)
            S.pt[h][lane] = pv;
            if (lane == 0) S.al[h] = a;
            l_run = __fadd_rn(__fmul_rn(l_run, a), ps);
            m_run = mn;
        }
        wait_bar(&S.vbar[st], par);
        __syncthreads();
        {
            // rescale the running sums of heads 2t, 2t+1 (heads >= G are never written)
            const float s0 = 2 * t < G ? S.al[2 * t] : 0.0f, s1 = 2 * t + 1 < G ? S.al[2 * t + 1] : 0.0f;
            acc[0] = __fmul_rn(acc[0], s0);
            acc[1] = __fmul_rn(acc[1], s1);
            acc[2] = __fmul_rn(acc[2], s0);
            acc[3] = __fmul_rn(acc[3], s1);
            const int d0 = 16 * warp + g;
#pragma unroll
            for (int ks = 0; ks < 4; ks++) {
                const int k0 = 8 * ks;
                if (k0 < ch) {  // uniform
                    const int r0 = k0 + t, r1 = k0 + t + 4;
                    float va[4];
                    if (k0 + 8 <= ch && fr < 0) {  // uniform: a full k-step of cache rows
                        va[0] = S.vs[st][r0][d0];
                        va[1] = S.vs[st][r0][d0 + 8];
                        va[2] = S.vs[st][r1][d0];
                        va[3] = S.vs[st][r1][d0 + 8];
                    } else {
                        auto vget = [&](int r, int d) -> float {
                            if (r >= ch) return 0.0f;
                            return r == fr ? S.vn[d] : S.vs[st][r][d];
                        };
                        va[0] = vget(r0, d0);
                        va[1] = vget(r0, d0 + 8);
                        va[2] = vget(r1, d0);
                        va[3] = vget(r1, d0 + 8);
                    }
                    uint32_t ab[4], as[4], bb[2], bs[2];
#pragma unroll
                    for (int e = 0; e < 4; e++) tf32_split(va[e], ab[e], as[e]);
                    tf32_split(g < G ? S.pt[g][r0] : 0.0f, bb[0], bs[0]);
                    tf32_split(g < G ? S.pt[g][r1] : 0.0f, bb[1], bs[1]);
                    mma_tf32x3(acc, ab, as, bb, bs);
                }
            }
        }
        const bool refill = i + 2 < nj;
        if (refill && tid == 0) {
            mbar_expect_tx(&S.kbar[st], (unsigned)(copied_of(j + 2) * ATT_D * 4));
            mbar_expect_tx(&S.vbar[st], (unsigned)(copied_of(j + 2) * ATT_D * 4));
        }
        __syncthreads();  // stage st, pt, al and the partial scores are free again
        if (refill) issue(j + 2, st, 2);
    }
    const int64_t hbase = ((int64_t)lrow * Hq + (int64_t)kvh * G) * nsplit + split;
    const int d0 = 16 * warp + g;
#pragma unroll
    for (int e = 0; e < 4; e++) {
        const int h = 2 * t + (e & 1), d = d0 + 8 * (e >> 1);
        if (h < G) p.part_o[(hbase + (int64_t)h * nsplit) * ATT_D + d] = acc[e];
    }
    if (warp < G && lane == 0) {
        p.part_ml[(hbase + (int64_t)warp * nsplit) * 2] = m_run;
        p.part_ml[(hbase + (int64_t)warp * nsplit) * 2 + 1] = l_run;
    }
}

// the unfused path's merge: one CTA per (kv head, query row, query head) rescales that head's
// chunk partials by exp(m_s - M), adds them in chunk order and divides by the summed
// denominators (the same arithmetic as the fused kernel's last-CTA merge). A kernel of its own,
// so that the chunk CTAs end without a fence and an atomic; one head per CTA, so that a batch
// of decode rows spreads its G * Hkv * rows merges over every SM.
__global__ void __launch_bounds__(ATT_D) attn_merge_kernel(const AttParams p) {
    __shared__ float cm[ATT_MAX_SPLITS];
    __shared__ float cl;
    const int Hq = p.Hq, Hkv = p.Hkv, L = p.L, nsplit = p.nsplit, G = Hq / Hkv;
    const int kvh = blockIdx.x, lrow = blockIdx.y, g = blockIdx.z;
    const int row = p.row0 + lrow, l = row % L;
    pdl_trigger();  // early: the next kernel (a weight stream) may start; it waits for us in pdl_wait
    pdl_wait();
    const int p0 = p.pos0_dev ? *p.pos0_dev : p.pos0;
    const int limit = p0 + l;
    if (limit < 0 || limit >= p.ctx_max) return;
    int n_active = min(limit / ATT_C + 1, nsplit);
    if (p.ring) {
        const int nsub = limit / ATB_P + 1;
        n_active = (nsub + ring_per(nsub, nsplit) - 1) / ring_per(nsub, nsplit);
    }
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t hb = ((int64_t)lrow * Hq + (int64_t)kvh * G + g) * nsplit;
    if (warp == 0) {
        const float* ml = p.part_ml + hb * 2;
        float m = -INFINITY;
        for (int s = lane; s < n_active; s += 32) m = fmaxf(m, ml[2 * s]);
        m = warp_max(m);
        float lsum = 0.0f;
        for (int s = lane; s < n_active; s += 32) {
            const float w = expf(__fsub_rn(ml[2 * s], m));
            cm[s] = w;
            lsum = __fadd_rn(lsum, __fmul_rn(w, ml[2 * s + 1]));
        }
        lsum = warp_sum(lsum);
        if (lane == 0) cl = lsum;
    }
    __syncthreads();
    const int d = tid;
    const float* po = p.part_o + hb * ATT_D + d;
    float o = 0.0f;
    // the chunks' values loaded 16 at a time ahead of the ordered adds
    int s = 0;
    for (; s + 16 <= n_active; s += 16) {
        float t[16];
#pragma unroll
        for (int i = 0; i < 16; i++) t[i] = po[(int64_t)(s + i) * ATT_D];
#pragma unroll
        for (int i = 0; i < 16; i++) o = __fadd_rn(o, __fmul_rn(cm[s + i], t[i]));
    }
    for (; s < n_active; s++) o = __fadd_rn(o, __fmul_rn(cm[s], po[(int64_t)s * ATT_D]));
    o = __fdiv_rn(o, cl);
    const int64_t e = (int64_t)row * Hq * ATT_D + (int64_t)(kvh * G + g) * ATT_D + d;
    if (p.out) p.out[e] = o;
    if (p.xq) quant_warp32(o, lane, p.xq + (e - lane), p.xd + (e >> 5));
}

// =========================================================================================
// Batched decode attention, streamed (one query row per sequence, L == 1, G <= 8 query heads per
// kv head). The 32-position chunks of all (row, kv head) pairs are dealt in equal contiguous
// ranges to one CTA per SM. A producer warp fills a 5-stage ring with bulk copies (each K row
// into its padded slot, the chunk's V rows in one copy, the pair's G query heads); eight
// consumer warps compute a chunk while the next ones land: scores (one thread per (position,
// head): four interleaved multiply-add chains over the 128 dimensions, added pairwise, then the
// scale), an online softmax per head over the CTA's chunks of the pair (running max and
// denominator; the P.V accumulators rescaled by exp(m_old - m_new)) and P.V (one thread per
// (dimension, 4 heads)). At the end of its chunks of a pair a CTA leaves (m, l, o) in the
// partial buffer; the CTA that completes the pair's chunk count (an atomic per pair, reset by
// that CTA) merges the pieces in CTA order (weights exp(m_c - M)) and writes the output row
// (f32 and/or Q8_0). The key/value stream never waits on the arithmetic, and no merge kernel
// follows.
// =========================================================================================
constexpr int AV_P = 32;                      // positions per chunk (one per producer lane)
constexpr int AV_STAGES = 5;
constexpr int AV_CONS = 256;                  // eight consumer warps
constexpr int AV_THREADS = AV_CONS + 32;      // + the producer warp

struct AvStage {
    float ks[AV_P][ATT_KS];
    float vs[AV_P][ATT_D];
    float qs[ATT_G][ATT_KS];
};
struct AvSmem {
    AvStage st[AV_STAGES];
    float pt[AV_P][ATT_G];                    // scores, then probabilities
    float mr[ATT_G], lr[ATT_G], al[ATT_G];    // running max and denominator; this chunk's rescale
    uint64_t full[AV_STAGES];
    uint64_t empty[AV_STAGES];
    int last;
};

// partial pieces: CTA b's j-th pair at slot b * jmax + j: o [G][D] unnormalised, (m, l) [G][2]
struct AvRange {
    long long units, u0, u1;
    int nch;
};

template <int GT>
__global__ void __launch_bounds__(AV_THREADS, 1) attn_decode_stream_kernel(const AttParams p) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    AvSmem& S = *reinterpret_cast<AvSmem*>(smem_raw);
    const int Hq = p.Hq, Hkv = p.Hkv, ctx_max = p.ctx_max, jmax = p.nsplit;
    const int G = GT ? GT : Hq / Hkv;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < AV_STAGES; i++) {
            mbar_init(&S.full[i], 1);
            mbar_init(&S.empty[i], 1);
        }
        mbar_fence_init();
    }
    if (tid < ATT_G) {
        S.mr[tid] = -INFINITY;
        S.lr[tid] = 0.0f;
    }
    __syncthreads();
    const int p0 = p.pos0_dev ? *p.pos0_dev : p.pos0;  // written by an earlier step: safe before pdl_wait
    if (p0 < 0 || p0 >= ctx_max) return;
    const int nch = p0 / AV_P + 1;
    const long long units = (long long)p.rows * Hkv * nch, GG = gridDim.x;
    const long long u0 = units * blockIdx.x / GG, u1 = units * (blockIdx.x + 1) / GG;

    if (warp == AV_CONS / 32) {
        // ---------------- producer warp ----------------
        pdl_wait();  // the query rows and this step's K/V rows come from the preceding kernel
        int s = 0;
        unsigned ph = 0;
        for (long long u = u0; u < u1; u++) {
            const int pair = (int)(u / nch), c = (int)(u - (long long)pair * nch);
            const int lrow = pair / Hkv, kvh = pair - lrow * Hkv;
            const int b = p.row0 + lrow;
            const int j0 = c * AV_P, cnt = min(AV_P, p0 + 1 - j0);
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&S.empty[s], ph ^ 1u);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                if (lane == 0 && p.err) atomicCAS(p.err, 0, 70);
                return;
            }
            AvStage& T = S.st[s];
            if (lane == 0) mbar_expect_tx(&S.full[s], (unsigned)((2 * cnt + G) * ATT_D * 4));
            __syncwarp();
            const int64_t kv0 = (((int64_t)b * Hkv + kvh) * ctx_max + j0) * ATT_D;
            if (lane < cnt) bulk_g2s(&T.ks[lane][0], p.kc + kv0 + (int64_t)lane * ATT_D, ATT_D * 4, &S.full[s]);
            if (lane == 0) bulk_g2s(&T.vs[0][0], p.vc + kv0, (unsigned)(cnt * ATT_D * 4), &S.full[s]);
            if (lane < G)  // q rows [B][Hq][1][D]
                bulk_g2s(&T.qs[lane][0], p.q + ((int64_t)b * Hq + kvh * G + lane) * ATT_D, ATT_D * 4, &S.full[s]);
            if (++s == AV_STAGES) {
                s = 0;
                ph ^= 1u;
            }
        }
        return;
    }
    // ---------------- consumers: 256 threads, named barrier 1 ----------------
    pdl_wait();  // the partial buffer and counters of the previous launch are done with
    pdl_trigger();
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)ATT_D));
    const int sp = tid >> 3, sg = tid & 7;             // score: (position, head)
    const int d = tid & (ATT_D - 1), h0 = 4 * (tid >> 7);  // P.V: dimension d, heads h0..h0+3
    const long long first_pair = u0 / nch;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int s = 0, done = 0;
    unsigned ph = 0;
    bool bad = false;
    for (long long u = u0; u < u1; u++) {
        const int pair = (int)(u / nch), c = (int)(u - (long long)pair * nch);
        const int cnt = min(AV_P, p0 + 1 - c * AV_P);
        const int cs = s;
        const unsigned cph = ph;
        if (++s == AV_STAGES) {
            s = 0;
            ph ^= 1u;
        }
        if (!bad) {
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&S.full[cs], cph);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                if (lane == 0 && p.err) atomicCAS(p.err, 0, 71);
                bad = true;  // keeps computing (on whatever is there) so that the barriers still meet
            }
        }
        const AvStage& T = S.st[cs];
        {
            float sc = -INFINITY;
            if (sp < cnt && sg < G) {
                const float* kr = T.ks[sp];
                const float* qr = T.qs[sg];
                float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
#pragma unroll 8
                for (int d4 = 0; d4 < ATT_D / 4; d4++) {
                    const float4 k4 = *reinterpret_cast<const float4*>(kr + 4 * d4);
                    const float4 q4 = *reinterpret_cast<const float4*>(qr + 4 * d4);
                    a0 = fmaf(q4.x, k4.x, a0);
                    a1 = fmaf(q4.y, k4.y, a1);
                    a2 = fmaf(q4.z, k4.z, a2);
                    a3 = fmaf(q4.w, k4.w, a3);
                }
                sc = __fmul_rn(__fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3)), scale);
            }
            S.pt[sp][sg] = sc;
        }
        group_sync<AV_CONS, 1>();
        if (warp < G) {
            // online softmax of head g over this chunk: lane = position
            const int g = warp;
            const float sv = S.pt[lane][g];
            const float mo = S.mr[g];
            const float mn = fmaxf(mo, warp_max(sv));
            const float pv = expf(__fsub_rn(sv, mn));
            const float ps = warp_sum(pv);
            S.pt[lane][g] = pv;
            if (lane == 0) {
                const float a = expf(__fsub_rn(mo, mn));  // 0 on the pair's first chunk (mo = -inf)
                S.al[g] = a;
                S.lr[g] = __fadd_rn(__fmul_rn(S.lr[g], a), ps);
                S.mr[g] = mn;
            }
        }
        group_sync<AV_CONS, 1>();
        {
#pragma unroll
            for (int i = 0; i < 4; i++) acc[i] = h0 + i < G ? __fmul_rn(acc[i], S.al[h0 + i]) : 0.0f;
            for (int j = 0; j < cnt; j++) {
                const float vv = T.vs[j][d];
                const float4 pj = *reinterpret_cast<const float4*>(&S.pt[j][h0]);
                acc[0] = fmaf(pj.x, vv, acc[0]);
                acc[1] = fmaf(pj.y, vv, acc[1]);
                acc[2] = fmaf(pj.z, vv, acc[2]);
                acc[3] = fmaf(pj.w, vv, acc[3]);
            }
        }
        group_sync<AV_CONS, 1>();  // the stage and pt are free again
        if (tid == 0) mbar_arrive(&S.empty[cs]);
        done++;
        if (c != nch - 1 && u + 1 != u1) continue;
        // ---- this CTA's piece of the pair: (m, l, o) out; the CTA completing the count merges ----
        {
            const size_t slot = (size_t)blockIdx.x * jmax + (size_t)(pair - first_pair);
            float* po = p.part_o + slot * G * ATT_D;
#pragma unroll
            for (int i = 0; i < 4; i++)
                if (h0 + i < G) __stcg(po + (h0 + i) * ATT_D + d, acc[i]);
            if (tid < G) {
                __stcg(p.part_ml + (slot * G + tid) * 2, S.mr[tid]);
                __stcg(p.part_ml + (slot * G + tid) * 2 + 1, S.lr[tid]);
            }
        }
        __threadfence();
        group_sync<AV_CONS, 1>();
        int* cnt_p = p.counters + pair;
        if (tid == 0) {
            const int prev = atomicAdd(cnt_p, done);
            S.last = prev + done == nch;
        }
        group_sync<AV_CONS, 1>();
        if (tid < ATT_G) {  // running state of the next pair (read after the next scores barrier)
            S.mr[tid] = -INFINITY;
            S.lr[tid] = 0.0f;
        }
        acc[0] = acc[1] = acc[2] = acc[3] = 0.0f;
        done = 0;
        if (!S.last) continue;
        __threadfence();
        // contributors: the CTAs whose ranges hold the pair's first and last chunks, and those between
        const long long pu0 = (long long)pair * nch;
        const int bf = (int)(((pu0 + 1) * GG - 1) / units), bl = (int)(((pu0 + nch) * GG - 1) / units);
        const int lrow = pair / Hkv, kvh = pair - lrow * Hkv;
        const int64_t row = p.row0 + lrow;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int h = h0 + i;
            if (h >= G) break;  // uniform per warp
            float M = -INFINITY;
            for (int q = bf; q <= bl; q++) {
                const size_t sl = (size_t)q * jmax + (size_t)(pair - units * q / GG / nch);
                M = fmaxf(M, __ldcg(p.part_ml + (sl * G + h) * 2));
            }
            float Ls = 0.0f, O = 0.0f;
            for (int q = bf; q <= bl; q++) {
                const size_t sl = (size_t)q * jmax + (size_t)(pair - units * q / GG / nch);
                const float w = expf(__fsub_rn(__ldcg(p.part_ml + (sl * G + h) * 2), M));
                Ls = __fadd_rn(Ls, __fmul_rn(w, __ldcg(p.part_ml + (sl * G + h) * 2 + 1)));
                O = __fadd_rn(O, __fmul_rn(w, __ldcg(p.part_o + (sl * G + h) * ATT_D + d)));
            }
            const float o = __fdiv_rn(O, Ls);
            const int64_t e = row * Hq * ATT_D + (int64_t)(kvh * G + h) * ATT_D + d;
            if (p.out) p.out[e] = o;
            if (p.xq) quant_warp32(o, lane, p.xq + (e - lane), p.xd + (e >> 5));
        }
        if (tid == 0) *cnt_p = 0;  // ready for the next launch
    }
}

// partial-buffer slots per CTA: the most (row, kv head) pairs one CTA's range can touch
static int av_jmax(int64_t pairs, int grid) { return (int)((pairs + grid - 1) / grid + 1); }

static size_t av_scratch_bytes(int64_t pairs, int grid, int G) {
    const size_t slots = (size_t)grid * av_jmax(pairs, grid);
    return ATT_COUNTER_BYTES + ((slots * G * 2 * 4 + 255) & ~(size_t)255) + slots * G * ATT_D * 4;
}

template <int GT>
static int launch_decode_stream(lq_ctx* ctx, AttParams p, int64_t rows, void* scratch, bool zero_counters) {
    const int grid = ctx->sm_count, G = p.Hq / p.Hkv;
    const int64_t pairs = rows * p.Hkv;
    const size_t slots = (size_t)grid * av_jmax(pairs, grid);
    p.counters = (int*)scratch;
    p.part_ml = (float*)((uint8_t*)scratch + ATT_COUNTER_BYTES);
    p.part_o = (float*)((uint8_t*)scratch + ATT_COUNTER_BYTES + ((slots * G * 2 * 4 + 255) & ~(size_t)255));
    p.nsplit = av_jmax(pairs, grid);  // the kernel's partial slots per CTA
    p.row0 = 0;
    p.rows = (int)rows;
    p.err = ctx->err_flag;
    if (const int rc = ensure_func_smem(ctx, (const void*)attn_decode_stream_kernel<GT>, sizeof(AvSmem))) return rc;
    if (zero_counters) LQ_CUDA(ctx, cudaMemsetAsync(p.counters, 0, (size_t)pairs * 4, ctx->stream));
    return launch_kernel(ctx, attn_decode_stream_kernel<GT>, dim3((unsigned)grid), dim3(AV_THREADS), sizeof(AvSmem),
                         "attn_decode_stream", p);
}

int attention_max_ctx() { return ATT_C * ATT_MAX_SPLITS; }

size_t attention_scratch_bytes(int64_t rows, int64_t Hq, int64_t ctx_max, int64_t D) {
    (void)D;
    const int64_t slice = std::min<int64_t>(rows, ATT_SLICE);
    const int64_t nsplit = (ctx_max + ATT_C - 1) / ATT_C;
    const size_t ml = ((size_t)(slice * Hq * nsplit * 2) * 4 + 255) & ~(size_t)255;
    return ATT_COUNTER_BYTES + ml + (size_t)(slice * Hq * nsplit * ATT_D) * 4;
}

template <bool FUSED, int GT, bool QKV = false>
static int launch_chunks(lq_ctx* ctx, AttParams p, int64_t rows, void* scratch, bool zero_counters) {
    using Smem = typename std::conditional<FUSED, AttSmem, AttSmemR>::type;
    const int64_t slice = std::min<int64_t>(rows, ATT_SLICE);
    p.counters = (int*)scratch;
    p.part_ml = (float*)((uint8_t*)scratch + ATT_COUNTER_BYTES);
    const size_t ml = ((size_t)(slice * p.Hq * p.nsplit * 2) * 4 + 255) & ~(size_t)255;
    p.part_o = (float*)((uint8_t*)scratch + ATT_COUNTER_BYTES + ml);
    {
        const int rc = ensure_func_smem(ctx, (const void*)attn_chunk_kernel<FUSED, GT>, sizeof(Smem));
        if (rc) return rc;
    }
    if (zero_counters)
        LQ_CUDA(ctx, cudaMemsetAsync(p.counters, 0, (size_t)(slice * p.Hkv) * 4, ctx->stream));
    // unfused: the ring kernel (LQ_ATT_CP=1: the cp.async chunk kernel), nsplit CTAs per (row,
    // kv head): about ATB_CTAS_PER_SM per SM over the pairs of a slice, at most the 64-position
    // chunks the scratch holds
    const bool bulk = QKV || (!FUSED && getenv("LQ_ATT_CP") == nullptr);
    // the ring's arithmetic on the tensor cores (3xTF32), or on the CUDA cores (LQ_ATT_FMA=1)
    const bool mma = bulk && getenv("LQ_ATT_FMA") == nullptr;
    p.err = ctx->err_flag;
    if (bulk) {
        const int rc = mma ? ensure_func_smem(ctx, (const void*)attn_chunk_mma_kernel<GT, QKV>, sizeof(AttSmemM))
                           : ensure_func_smem(ctx, (const void*)attn_chunk_bulk_kernel<GT, QKV>, sizeof(AttSmemB));
        if (rc) return rc;
        const int64_t pairs = std::max<int64_t>(1, slice * p.Hkv);
        const int64_t want = ((int64_t)ATB_CTAS_PER_SM * ctx->sm_count + pairs - 1) / pairs;
        p.nsplit = (int)std::max<int64_t>(1, std::min<int64_t>(want, p.nsplit));
        p.ring = 1;
    }
    for (int64_t r0 = 0; r0 < rows; r0 += slice) {
        const int64_t n = std::min(slice, rows - r0);
        p.row0 = (int)r0;
        const dim3 grid(p.nsplit, (unsigned)p.Hkv, (unsigned)n);
        int rc = mma ? launch_kernel(ctx, attn_chunk_mma_kernel<GT, QKV>, grid, dim3(ATB_THREADS), sizeof(AttSmemM),
                                     "attn_chunk_mma", p)
                 : bulk ? launch_kernel(ctx, attn_chunk_bulk_kernel<GT, QKV>, grid, dim3(ATB_THREADS), sizeof(AttSmemB),
                                      "attn_chunk_bulk", p)
                      : launch_kernel(ctx, attn_chunk_kernel<FUSED, GT>, grid, dim3(ATT_THREADS), sizeof(Smem),
                                      "attn_chunk", p);
        if (rc) return rc;
        if (!FUSED) {
            rc = launch_kernel(ctx, attn_merge_kernel, dim3((unsigned)p.Hkv, (unsigned)n, (unsigned)(p.Hq / p.Hkv)),
                               dim3(ATT_D), 0,
                               "attn_merge", p);
            if (rc) return rc;
        }
    }
    return LQ_OK;
}

int launch_attention(lq_ctx* ctx, const float* q, const float* kc, const float* vc, int64_t B,
                     int64_t Hq, int64_t Hkv, int64_t L, int64_t pos0, const int32_t* pos0_dev,
                     int64_t ctx_max, int64_t D, float* out, int8_t* xq, uint16_t* xd,
                     void* scratch, bool zero_counters) {
    (void)D;
    const int64_t rows = B * L;
    if (rows == 0) return LQ_OK;
    if (attention_prefill_supported(L, Hq, Hkv))
        return launch_attention_prefill(ctx, q, kc, vc, B, Hq, Hkv, L, pos0, pos0_dev, ctx_max, out, xq, xd);
    AttParams p = {};
    p.q = q;
    p.kc = const_cast<float*>(kc);
    p.vc = const_cast<float*>(vc);
    p.Hq = (int)Hq;
    p.Hkv = (int)Hkv;
    p.L = (int)L;
    p.pos0 = (int)pos0;
    p.pos0_dev = pos0_dev;
    p.ctx_max = (int)ctx_max;
    // with a host-known position only the chunks up to pos0+L are launched; with a device
    // position (CUDA-graph decode) the grid covers ctx_max and idle chunks exit at once
    const int64_t span = pos0_dev ? ctx_max : std::min<int64_t>(ctx_max, pos0 + L);
    p.nsplit = ceil_div(span, ATT_C);
    p.out = out;
    p.xq = xq;
    p.xd = xd;
    if (L == 1 && rows <= ATT_SLICE && getenv("LQ_ATT_STREAM") != nullptr &&
        av_scratch_bytes(rows * Hkv, ctx->sm_count, (int)(Hq / Hkv)) <= attention_scratch_bytes(rows, Hq, ctx_max, D)) {
        // decode rows, LQ_ATT_STREAM=1: the streamed kernel (slower than one CTA per 64-key
        // chunk + the merge kernel at 32B batch 8 today)
        switch (Hq / Hkv) {
            case 8: return launch_decode_stream<8>(ctx, p, rows, scratch, zero_counters);
            case 4: return launch_decode_stream<4>(ctx, p, rows, scratch, zero_counters);
            case 2: return launch_decode_stream<2>(ctx, p, rows, scratch, zero_counters);
            case 1: return launch_decode_stream<1>(ctx, p, rows, scratch, zero_counters);
            default: return launch_decode_stream<0>(ctx, p, rows, scratch, zero_counters);
        }
    }
    switch (Hq / Hkv) {
        case 8: return launch_chunks<false, 8>(ctx, p, rows, scratch, zero_counters);
        case 4: return launch_chunks<false, 4>(ctx, p, rows, scratch, zero_counters);
        case 2: return launch_chunks<false, 2>(ctx, p, rows, scratch, zero_counters);
        case 1: return launch_chunks<false, 1>(ctx, p, rows, scratch, zero_counters);
        default: return launch_chunks<false, 0>(ctx, p, rows, scratch, zero_counters);
    }
}

int launch_attention_decode_fused(lq_ctx* ctx, const float* qkv, const uint16_t* qn, const uint16_t* kn,
                                  float eps, const float* cos_t, const float* sin_t, float* kc, float* vc,
                                  int64_t B, int64_t Hq, int64_t Hkv, const int32_t* pos_dev, int64_t ctx_max,
                                  int8_t* xq, uint16_t* xd, void* scratch) {
    if (B == 0) return LQ_OK;
    AttParams p = {};
    p.qkv = qkv;
    p.qn = qn;
    p.kn = kn;
    p.eps = eps;
    p.cos_t = cos_t;
    p.sin_t = sin_t;
    p.kc = kc;
    p.vc = vc;
    p.Hq = (int)Hq;
    p.Hkv = (int)Hkv;
    p.L = 1;
    p.pos0_dev = pos_dev;
    p.ctx_max = (int)ctx_max;
    p.nsplit = ceil_div(ctx_max, ATT_C);
    p.xq = xq;
    p.xd = xd;
    return launch_chunks<true, 0>(ctx, p, B, scratch, false);
}

// Batched decode rows (L == 1, device position) straight from the fused q|k|v projection: q/k
// RMSNorm + RoPE, the KV append and attention in the ring kernel, then the merge kernel.
int launch_attention_decode_qkv(lq_ctx* ctx, const float* qkv, const uint16_t* qn, const uint16_t* kn, float eps,
                                const float* cos_t, const float* sin_t, float* kc, float* vc, int64_t B, int64_t Hq,
                                int64_t Hkv, const int32_t* pos_dev, int64_t ctx_max, int8_t* xq, uint16_t* xd,
                                void* scratch) {
    if (B == 0) return LQ_OK;
    AttParams p = {};
    p.qkv = qkv;
    p.qn = qn;
    p.kn = kn;
    p.eps = eps;
    p.cos_t = cos_t;
    p.sin_t = sin_t;
    p.kc = kc;
    p.vc = vc;
    p.Hq = (int)Hq;
    p.Hkv = (int)Hkv;
    p.L = 1;
    p.pos0_dev = pos_dev;
    p.ctx_max = (int)ctx_max;
    p.nsplit = ceil_div(ctx_max, ATT_C);
    p.xq = xq;
    p.xd = xd;
    switch (Hq / Hkv) {
        case 8: return launch_chunks<false, 8, true>(ctx, p, B, scratch, false);
        case 4: return launch_chunks<false, 4, true>(ctx, p, B, scratch, false);
        case 2: return launch_chunks<false, 2, true>(ctx, p, B, scratch, false);
        case 1: return launch_chunks<false, 1, true>(ctx, p, B, scratch, false);
        default: return launch_chunks<false, 0, true>(ctx, p, B, scratch, false);
    }
}

}  // namespace lq

extern "C" int lq_attention(lq_ctx* ctx, const float* q, const float* kc, const float* vc, int64_t B, int64_t Hq,
                            int64_t Hkv, int64_t L, int64_t pos0, const int32_t* pos0_dev, int64_t ctx_max,
                            int64_t D, float* out, int8_t* xq, uint16_t* xd) {
    LQ_ENTRY(ctx, "lq_attention");
    LQ_REQUIRE(ctx, D == 128, "lq_attention: head_dim %lld unsupported (Qwen3 uses 128)", (long long)D);
    LQ_REQUIRE(ctx, Hq > 0 && Hkv > 0 && Hq % Hkv == 0 && Hq / Hkv <= 8 && Hkv <= lq::ATT_MAX_KV,
               "lq_attention: need Hq %% Hkv == 0, Hq/Hkv <= 8 and at most %d kv heads", lq::ATT_MAX_KV);
    LQ_REQUIRE(ctx, B >= 0 && L >= 0 && B * L < (1ll << 31), "lq_attention: bad B/L");
    LQ_REQUIRE(ctx, pos0_dev || (pos0 >= 0 && pos0 + L <= ctx_max), "lq_attention: positions exceed ctx_max");
    LQ_REQUIRE(ctx, ctx_max <= lq::attention_max_ctx(), "lq_attention: ctx_max %lld exceeds %d",
               (long long)ctx_max, lq::attention_max_ctx());
    LQ_REQUIRE(ctx, (xq == nullptr) == (xd == nullptr), "lq_attention: xq and xd go together");
    if (B == 0 || L == 0) return LQ_OK;
    LQ_REQUIRE(ctx, q && kc && vc && (out || xq), "lq_attention: NULL pointer");
    const size_t need = lq::attention_scratch_bytes(B * L, Hq, ctx_max, D);
    const int rc = lq::ensure_scratch(ctx, need);
    if (rc) return rc;
    return lq::launch_attention(ctx, q, kc, vc, B, Hq, Hkv, L, pos0, pos0_dev, ctx_max, D, out, xq, xd,
                                ctx->scratch, true);
}
