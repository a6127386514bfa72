// lq8_fused.cuh -- device functions shared by the standalone op kernels and the fused
// prologues of the decode kernels, so both produce bit-identical results.
#pragma once

#include "lq8_internal.cuh"

namespace lq {

// Quantize 4 values held by each lane of an aligned 8-lane group (one Q8_0 block of 32);
// returns the packed int8x4; lane 0 of the group stores the fp16 scale when d_out != NULL.
// Every lane of the warp must call it (shuffles over the full mask).
__device__ __forceinline__ uint32_t quant_group8(const float v[4], int sub, uint16_t* d_out) {
    float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
    float d, id;
    q8_scale(amax, d, id);
    if (sub == 0 && d_out) *d_out = f2h(d);
    uint32_t q0 = (uint32_t)(q8_quant(v[0], id) & 0xFF), q1 = (uint32_t)(q8_quant(v[1], id) & 0xFF);
    uint32_t q2 = (uint32_t)(q8_quant(v[2], id) & 0xFF), q3 = (uint32_t)(q8_quant(v[3], id) & 0xFF);
    return q0 | (q1 << 8) | (q2 << 16) | (q3 << 24);
}

// SiLU(gate) * up of one element (mlp.rs:153-160; silu = x/(1+exp(-x)), tensor.rs:1977-1986)
__device__ __forceinline__ float swiglu(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

// barrier over the THREADS threads running a row function: __syncthreads() when BAR == 0,
// else the named barrier BAR (a sub-group of the CTA, e.g. the consumer warps)
template <int THREADS, int BAR>
__device__ __forceinline__ void group_sync() {
    if constexpr (BAR == 0) __syncthreads();
    else asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(THREADS));
}

template <typename T>
__device__ __forceinline__ void load4_any(const T* p, float v[4]);
template <>
__device__ __forceinline__ void load4_any<float>(const float* p, float v[4]) {
    float4 t = *reinterpret_cast<const float4*>(p);
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
}
template <>
__device__ __forceinline__ void load4_any<uint16_t>(const uint16_t* p, float v[4]) {
    uint2 t = *reinterpret_cast<const uint2*>(p);
    v[0] = bf16_to_f32((uint16_t)(t.x & 0xFFFF)); v[1] = bf16_to_f32((uint16_t)(t.x >> 16));
    v[2] = bf16_to_f32((uint16_t)(t.y & 0xFFFF)); v[3] = bf16_to_f32((uint16_t)(t.y >> 16));
}

// RmsNorm::forward of one row (rms_norm.rs:144-176) by THREADS threads (tid in [0,THREADS)):
// the input is rounded to bf16; each thread sums the squares of its elements (4 consecutive
// per 4*THREADS-wide pass, in pass order), a warp butterfly and a cross-warp sum in warp order
// give the total; inv = 1/sqrt(sum/dim + eps); out = bf16((x*inv)*w). Optional outputs: the
// bf16 row and/or its Q8_0 quantization (xq [dim], xd [dim/32]). red: >= 32 floats of smem.
template <typename T, int THREADS, int BAR, int RC = 0>
__device__ __forceinline__ void rms_row(const T* __restrict__ xr, int dim, const uint16_t* __restrict__ w,
                                        float eps, int tid, float* red, uint16_t* out, int8_t* xq,
                                        uint16_t* xd) {
    // RC > 0: rows of up to RC * THREADS * 4 elements stay in registers between the two passes
    // (all their loads issued at once); otherwise (and for longer rows) the second pass reads the
    // row again. The sum of squares runs in the same order either way.
    float cache[RC > 0 ? RC : 1][4];
    uint2 wcache[RC > 0 ? RC : 1];  // the norm weights too: their loads overlap the reduction
    const bool cached = RC > 0 && dim <= RC * THREADS * 4;
#pragma unroll
    for (int c = 0; c < RC; c++) {
        const int e = c * THREADS * 4 + tid * 4;
        if (cached && e < dim) {
            load4_any<T>(xr + e, cache[c]);
            wcache[c] = *reinterpret_cast<const uint2*>(w + e);
        }
    }
    float ss = 0.0f;
    for (int base = 0; base < dim; base += THREADS * 4) {
        const int e = base + tid * 4;
        if (e < dim) {
            float v[4];
            if (cached) {
#pragma unroll
                for (int c = 0; c < RC; c++)
                    if (c * THREADS * 4 == base) v[0] = cache[c][0], v[1] = cache[c][1], v[2] = cache[c][2], v[3] = cache[c][3];
            } else {
                load4_any<T>(xr + e, v);
            }
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float r = round_bf16(v[i]);
                ss = __fadd_rn(ss, __fmul_rn(r, r));
            }
        }
    }
    ss = warp_sum(ss);
    const int lane = tid & 31, warp = tid >> 5;
    if (lane == 0) red[warp] = ss;
    group_sync<THREADS, BAR>();
    float tot = lane < THREADS / 32 ? red[lane] : 0.0f;
    tot = warp_sum(tot);
    group_sync<THREADS, BAR>();  // red may be reused right after
    const float mean = __fdiv_rn(tot, (float)dim);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    for (int base = 0; base < dim; base += THREADS * 4) {
        const int e = base + tid * 4;
        const bool valid = e < dim;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (valid) {
            if (cached) {
#pragma unroll
                for (int c = 0; c < RC; c++)
                    if (c * THREADS * 4 == base) v[0] = cache[c][0], v[1] = cache[c][1], v[2] = cache[c][2], v[3] = cache[c][3];
            } else {
                load4_any<T>(xr + e, v);
            }
            uint2 wt;
            if (cached) {
#pragma unroll
                for (int c = 0; c < RC; c++)
                    if (c * THREADS * 4 == base) wt = wcache[c];
            } else {
                wt = *reinterpret_cast<const uint2*>(w + e);
            }
            const float wv[4] = {bf16_to_f32((uint16_t)(wt.x & 0xFFFF)), bf16_to_f32((uint16_t)(wt.x >> 16)),
                                 bf16_to_f32((uint16_t)(wt.y & 0xFFFF)), bf16_to_f32((uint16_t)(wt.y >> 16))};
            uint16_t o[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float r = round_bf16(v[i]);
                o[i] = f32_to_bf16(__fmul_rn(__fmul_rn(r, inv), wv[i]));
                v[i] = bf16_to_f32(o[i]);
            }
            if (out) {
                uint2 ov;
                ov.x = (uint32_t)o[0] | ((uint32_t)o[1] << 16);
                ov.y = (uint32_t)o[2] | ((uint32_t)o[3] << 16);
                *reinterpret_cast<uint2*>(out + e) = ov;
            }
        }
        if (xq) {  // uniform: every lane joins the group shuffles
            const uint32_t q = quant_group8(v, tid & 7, valid ? xd + (e >> 5) : nullptr);
            if (valid) *reinterpret_cast<uint32_t*>(xq + e) = q;
        }
    }
}

// SiLU(gate) * up of one row (mlp.rs:153-160; silu x/(1+exp(-x)) tensor.rs:1977-1986, mul f32)
// from gu [2*inter] (gate first), by THREADS threads; writes h f32 and/or Q8_0.
template <int THREADS>
__device__ __forceinline__ void silu_row(const float* __restrict__ gu, int inter, int tid, float* h, int8_t* xq,
                                         uint16_t* xd) {
    for (int base = 0; base < inter; base += THREADS * 4) {
        const int e = base + tid * 4;
        const bool valid = e < inter;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (valid) {
            const float4 g = *reinterpret_cast<const float4*>(gu + e);
            const float4 u = *reinterpret_cast<const float4*>(gu + inter + e);
            const float gg[4] = {g.x, g.y, g.z, g.w}, uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int i = 0; i < 4; i++) v[i] = swiglu(gg[i], uu[i]);
            if (h) *reinterpret_cast<float4*>(h + e) = make_float4(v[0], v[1], v[2], v[3]);
        }
        if (xq) {
            const uint32_t q = quant_group8(v, tid & 7, valid ? xd + (e >> 5) : nullptr);
            if (valid) *reinterpret_cast<uint32_t*>(xq + e) = q;
        }
    }
}

// Q8_0 quantization of one f32 row (dim % 32 == 0) by THREADS threads, 4 elements a lane,
// one 8-lane group per 32-element block (the same grouping as the producing row functions).
template <int THREADS>
__device__ __forceinline__ void quant_row(const float* __restrict__ x, int dim, int tid, int8_t* xq, uint16_t* xd) {
    for (int base = 0; base < dim; base += THREADS * 4) {
        const int e = base + tid * 4;
        const bool valid = e < dim;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (valid) {
            const float4 t = *reinterpret_cast<const float4*>(x + e);
            v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
        }
        const uint32_t q = quant_group8(v, tid & 7, valid ? xd + (e >> 5) : nullptr);
        if (valid) *reinterpret_cast<uint32_t*>(xq + e) = q;
    }
}

// Per-head RMSNorm + RoPE of one 128-dim q or k head vector by one warp (attention.rs:350-361,
// rope.rs:245-303): lane p holds dims (2p, 2p+1) and (64+2p, 64+2p+1) -- one rotation pair
// set, so the rotation is lane-local. src: the f32 projection output of the head; out gets
// the rotated f32 vector, its dims 64..127 starting at out + hi_off.
__device__ __forceinline__ void head_norm_rope(const float* __restrict__ src, const uint16_t* __restrict__ nw,
                                               float eps, const float* __restrict__ cos_row,
                                               const float* __restrict__ sin_row, int lane, float* out,
                                               int hi_off = 64) {
    constexpr int D = 128, RD = 64;
    const int d0 = 2 * lane;
    const float2 a = *reinterpret_cast<const float2*>(src + d0);
    const float2 c = *reinterpret_cast<const float2*>(src + RD + d0);
    float v[4] = {round_bf16(a.x), round_bf16(a.y), round_bf16(c.x), round_bf16(c.y)};
    float ss = __fadd_rn(__fadd_rn(__fmul_rn(v[0], v[0]), __fmul_rn(v[1], v[1])),
                         __fadd_rn(__fmul_rn(v[2], v[2]), __fmul_rn(v[3], v[3])));
    ss = warp_sum(ss);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), eps)));
    const int dims[4] = {d0, d0 + 1, RD + d0, RD + d0 + 1};
#pragma unroll
    for (int i = 0; i < 4; i++) v[i] = round_bf16(__fmul_rn(__fmul_rn(v[i], inv), bf16_to_f32(nw[dims[i]])));
    const float cs = cos_row[d0], sn = sin_row[d0];
    const float r0 = __fsub_rn(__fmul_rn(v[0], cs), __fmul_rn(v[2], sn));
    const float r1 = __fsub_rn(__fmul_rn(v[1], cs), __fmul_rn(v[3], sn));
    const float r2 = __fadd_rn(__fmul_rn(v[2], cs), __fmul_rn(v[0], sn));
    const float r3 = __fadd_rn(__fmul_rn(v[3], cs), __fmul_rn(v[1], sn));
    *reinterpret_cast<float2*>(out + d0) = make_float2(r0, r1);
    *reinterpret_cast<float2*>(out + hi_off + d0) = make_float2(r2, r3);  // the second half (dims 64..)
}

}  // namespace lq
