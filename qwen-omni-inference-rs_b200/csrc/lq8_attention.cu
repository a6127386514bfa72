// lq8_attention.cu -- GQA attention over the f32 KV cache (attention.rs:366-399, repeat_kv
// attention.rs:426-456, causal mask causal_mask.rs:104-164), split over key positions.
//
// A CTA owns (one query row, one kv head, one chunk of ATT_C positions) and all G = Hq/Hkv
// query heads that share the kv head. It stages the chunk's K and V rows into shared memory
// with every 16-byte async copy in flight at once, computes the G score rows (each score is
// the reference's sequential 128-term dot product, then the scale), a chunk softmax
// (max, exp, sum) and the chunk's P.V. The last CTA of a (row, kv head) to finish -- found
// with an atomic counter -- merges the chunks (rescaling by exp(m_s - M)) and writes the
// [Hq*D] output row in f32 and/or Q8_0 for o_proj. One launch, no combine kernel.
#include "lq8_async.cuh"
#include "lq8_internal.cuh"

namespace lq {

constexpr int ATT_C = 64;           // key positions per chunk
constexpr int ATT_D = 128;          // head_dim
constexpr int ATT_KS = ATT_D + 4;   // padded K row stride in floats: conflict-free float4 reads
constexpr int ATT_G = 8;            // max query heads per kv head
constexpr int ATT_THREADS = 128;
constexpr int ATT_SLICE = 256;      // query rows per launch (bounds the partials)
constexpr int ATT_MAX_SPLITS = 128; // chunks per row: contexts up to 8192 positions

struct AttSmem {
    float ks[ATT_C][ATT_KS];
    float vs[ATT_C][ATT_D];
    float qs[ATT_G][ATT_D];
    float ps[ATT_G][ATT_C];
    float ml[ATT_G][2];
    float cm[ATT_G][ATT_MAX_SPLITS];  // combine: per-chunk weights exp(m_s - M)
    float cl[ATT_G];       // combine: total denominator
    int last;
};

__device__ __forceinline__ void quant_warp32(float v, int lane, int8_t* q_out, uint16_t* d_out) {
    float amax = warp_max(fabsf(v));
    float d, id;
    q8_scale(amax, d, id);
    q_out[lane] = (int8_t)q8_quant(v, id);
    if (lane == 0) *d_out = f2h(d);
}

__global__ void __launch_bounds__(ATT_THREADS)
attn_chunk_kernel(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
                  int Hq, int Hkv, int L, int pos0, const int32_t* __restrict__ pos0_dev, int ctx_max,
                  int row0, int nsplit, float* __restrict__ part_o, float* __restrict__ part_ml,
                  int* __restrict__ counters, float* __restrict__ out, int8_t* __restrict__ xq,
                  uint16_t* __restrict__ xd) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    AttSmem& S = *reinterpret_cast<AttSmem*>(smem_raw);
    const int G = Hq / Hkv;
    const int split = blockIdx.x, kvh = blockIdx.y, lrow = blockIdx.z;
    const int row = row0 + lrow;  // b*L + l
    const int b = row / L, l = row - (row / L) * L;
    const int p0 = pos0_dev ? *pos0_dev : pos0;
    const int limit = p0 + l;  // last visible position
    if (limit < 0 || limit >= ctx_max) return;
    const int n_active = min(limit / ATT_C + 1, nsplit);
    if (split >= n_active) return;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int j0 = split * ATT_C;
    const int cnt = min(ATT_C, limit + 1 - j0);
    const float* kbase = kc + ((int64_t)b * Hkv + kvh) * (int64_t)ctx_max * ATT_D + (int64_t)j0 * ATT_D;
    const float* vbase = vc + ((int64_t)b * Hkv + kvh) * (int64_t)ctx_max * ATT_D + (int64_t)j0 * ATT_D;
    // every 16-byte piece of the chunk's K and V rows in flight at once. Rows of positions
    // before p0 were appended by earlier steps and are read before pdl_wait(); the rows of
    // this launch's positions are written by the preceding kernel and are read after it.
    const int fresh = p0 - j0;  // chunk rows r >= fresh belong to this launch
    for (int i = tid; i < cnt * (ATT_D / 4); i += ATT_THREADS) {
        int r = i / (ATT_D / 4), c = (i % (ATT_D / 4)) * 4;
        if (r < fresh) {
            cp_async16(&S.ks[r][c], kbase + (int64_t)r * ATT_D + c, true);
            cp_async16(&S.vs[r][c], vbase + (int64_t)r * ATT_D + c, true);
        }
    }
    pdl_wait();
    pdl_trigger();
    for (int i = tid; i < cnt * (ATT_D / 4); i += ATT_THREADS) {
        int r = i / (ATT_D / 4), c = (i % (ATT_D / 4)) * 4;
        if (r >= fresh) {
            cp_async16(&S.ks[r][c], kbase + (int64_t)r * ATT_D + c, true);
            cp_async16(&S.vs[r][c], vbase + (int64_t)r * ATT_D + c, true);
        }
    }
    cp_async_commit();
    for (int i = tid; i < G * ATT_D; i += ATT_THREADS) {
        int g = i / ATT_D, d = i % ATT_D;
        S.qs[g][d] = q[(((int64_t)b * Hq + kvh * G + g) * L + l) * ATT_D + d];
    }
    cp_async_wait<0>();
    __syncthreads();

    // scores: thread -> (position p, heads half, half+2, ...); sequential 128-term dot
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)ATT_D));
    {
        const int p = tid % ATT_C, half = tid / ATT_C;
        float s[ATT_G / 2];
#pragma unroll
        for (int i = 0; i < ATT_G / 2; i++) s[i] = 0.0f;
        if (p < cnt) {
#pragma unroll 8
            for (int d4 = 0; d4 < ATT_D / 4; d4++) {
                float4 k4 = *reinterpret_cast<const float4*>(&S.ks[p][4 * d4]);
#pragma unroll
                for (int i = 0; i < ATT_G / 2; i++) {
                    int g = half + 2 * i;
                    if (g < G) {
                        float4 q4 = *reinterpret_cast<const float4*>(&S.qs[g][4 * d4]);
                        s[i] = __fadd_rn(s[i], __fmul_rn(q4.x, k4.x));
                        s[i] = __fadd_rn(s[i], __fmul_rn(q4.y, k4.y));
                        s[i] = __fadd_rn(s[i], __fmul_rn(q4.z, k4.z));
                        s[i] = __fadd_rn(s[i], __fmul_rn(q4.w, k4.w));
                    }
                }
            }
        }
#pragma unroll
        for (int i = 0; i < ATT_G / 2; i++) {
            int g = half + 2 * i;
            if (g < G) S.ps[g][p] = p < cnt ? __fmul_rn(s[i], scale) : -INFINITY;
        }
    }
    __syncthreads();
    // chunk softmax per head: max, exp(s - max), sum
    for (int g = warp; g < G; g += ATT_THREADS / 32) {
        float a = S.ps[g][lane], c = S.ps[g][lane + 32];
        float m = warp_max(fmaxf(a, c));
        float ea = expf(__fsub_rn(a, m)), ec = expf(__fsub_rn(c, m));
        S.ps[g][lane] = ea;
        S.ps[g][lane + 32] = ec;
        float sum = warp_sum(__fadd_rn(ea, ec));
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
            float vv = S.vs[j][d];
#pragma unroll
            for (int g = 0; g < ATT_G; g++)
                if (g < G) acc[g] = __fadd_rn(acc[g], __fmul_rn(S.ps[g][j], vv));
        }
        const int64_t hbase = ((int64_t)lrow * Hq + (int64_t)kvh * G) * nsplit + split;
#pragma unroll
        for (int g = 0; g < ATT_G; g++)
            if (g < G) part_o[(hbase + (int64_t)g * nsplit) * ATT_D + d] = acc[g];
        if (tid < G) {
            part_ml[(hbase + (int64_t)tid * nsplit) * 2] = S.ml[tid][0];
            part_ml[(hbase + (int64_t)tid * nsplit) * 2 + 1] = S.ml[tid][1];
        }
    }
    // the last chunk CTA of this (row, kv head) merges the chunks
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        int prev = atomicAdd(&counters[lrow * Hkv + kvh], 1);
        S.last = (prev == n_active - 1);
    }
    __syncthreads();
    if (!S.last) return;
    __threadfence();
    const int64_t hbase0 = ((int64_t)lrow * Hq + (int64_t)kvh * G) * nsplit;
    for (int g = warp; g < G; g += ATT_THREADS / 32) {
        float m = -INFINITY;
        for (int s = lane; s < n_active; s += 32) m = fmaxf(m, ld_cg(&part_ml[(hbase0 + (int64_t)g * nsplit + s) * 2]));
        m = warp_max(m);
        float lsum = 0.0f;
        for (int s = lane; s < n_active; s += 32) {
            float w = expf(__fsub_rn(ld_cg(&part_ml[(hbase0 + (int64_t)g * nsplit + s) * 2]), m));
            S.cm[g][s] = w;
            lsum = __fadd_rn(lsum, __fmul_rn(w, ld_cg(&part_ml[(hbase0 + (int64_t)g * nsplit + s) * 2 + 1])));
        }
        lsum = warp_sum(lsum);
        if (lane == 0) S.cl[g] = lsum;
    }
    __syncthreads();
    const int d = tid;
    for (int g = 0; g < G; g++) {
        float o = 0.0f;
#pragma unroll 8
        for (int s = 0; s < n_active; s++)
            o = __fadd_rn(o, __fmul_rn(S.cm[g][s], ld_cg(&part_o[(hbase0 + (int64_t)g * nsplit + s) * ATT_D + d])));
        o = __fdiv_rn(o, S.cl[g]);
        const int64_t e = (int64_t)row * Hq * ATT_D + (int64_t)(kvh * G + g) * ATT_D + d;
        if (out) out[e] = o;
        if (xq) quant_warp32(o, lane, xq + (e - lane), xd + (e >> 5));
    }
    if (tid == 0) counters[lrow * Hkv + kvh] = 0;  // ready for the next launch
}

int attention_max_ctx() { return ATT_C * ATT_MAX_SPLITS; }

static int attn_nsplit(int64_t ctx_max, int64_t pos0, int64_t L, bool dev_pos) {
    int64_t span = dev_pos ? ctx_max : std::min<int64_t>(ctx_max, pos0 + L);
    return ceil_div(span, ATT_C);
}

// scratch: [counters: fixed ATT_SLICE*ATT_MAX_KV ints][part_ml slice*Hq*nsplit*2]
// [part_o slice*Hq*nsplit*D]. The counter region has the same place and size for every call,
// so launches with different row counts sharing one scratch never overlap counters with
// another launch's partials.
constexpr int ATT_MAX_KV = 64;
constexpr size_t ATT_COUNTER_BYTES = (size_t)ATT_SLICE * ATT_MAX_KV * 4;

size_t attention_scratch_bytes(int64_t rows, int64_t Hq, int64_t ctx_max, int64_t D) {
    (void)D;
    int64_t slice = std::min<int64_t>(rows, ATT_SLICE);
    int64_t nsplit = (ctx_max + ATT_C - 1) / ATT_C;
    size_t ml = ((size_t)(slice * Hq * nsplit * 2) * 4 + 255) & ~(size_t)255;
    return ATT_COUNTER_BYTES + ml + (size_t)(slice * Hq * nsplit * ATT_D) * 4;
}

int launch_attention(lq_ctx* ctx, const float* q, const float* kc, const float* vc, int64_t B,
                     int64_t Hq, int64_t Hkv, int64_t L, int64_t pos0, const int32_t* pos0_dev,
                     int64_t ctx_max, int64_t D, float* out, int8_t* xq, uint16_t* xd,
                     void* scratch, bool zero_counters) {
    (void)D;
    const int64_t rows = B * L;
    if (rows == 0) return LQ_OK;
    const int nsplit = attn_nsplit(ctx_max, pos0, L, pos0_dev != nullptr);
    const int64_t slice = std::min<int64_t>(rows, ATT_SLICE);
    int* counters = (int*)scratch;
    float* part_ml = (float*)((uint8_t*)scratch + ATT_COUNTER_BYTES);
    size_t ml = ((size_t)(slice * Hq * nsplit * 2) * 4 + 255) & ~(size_t)255;
    float* part_o = (float*)((uint8_t*)scratch + ATT_COUNTER_BYTES + ml);
    static bool attr = false;
    if (!attr) {
        LQ_CUDA(ctx, cudaFuncSetAttribute(attn_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)sizeof(AttSmem)));
        attr = true;
    }
    if (zero_counters) LQ_CUDA(ctx, cudaMemsetAsync(counters, 0, (size_t)(slice * Hkv) * 4, ctx->stream));
    for (int64_t r0 = 0; r0 < rows; r0 += slice) {
        int64_t n = std::min(slice, rows - r0);
        dim3 grid(nsplit, (unsigned)Hkv, (unsigned)n);
        int rc = launch_kernel(ctx, attn_chunk_kernel, grid, dim3(ATT_THREADS), sizeof(AttSmem), "attn_chunk", q,
                               kc, vc, (int)Hq, (int)Hkv, (int)L, (int)pos0, pos0_dev, (int)ctx_max, (int)r0,
                               nsplit, part_o, part_ml, counters, out, xq, xd);
        if (rc) return rc;
    }
    return LQ_OK;
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
    size_t need = lq::attention_scratch_bytes(B * L, Hq, ctx_max, D);
    int rc = lq::ensure_scratch(ctx, need);
    if (rc) return rc;
    return lq::launch_attention(ctx, q, kc, vc, B, Hq, Hkv, L, pos0, pos0_dev, ctx_max, D, out, xq, xd,
                                ctx->scratch, true);
}
