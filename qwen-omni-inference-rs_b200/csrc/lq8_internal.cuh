// lq8_internal.cuh -- shared host/device helpers of liblq8 (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/lq8.h"

// ------------------------------------------------------------------------------------------
// context
// ------------------------------------------------------------------------------------------
constexpr int kTileCounters = 1024;

struct lq_ctx {
    int device = 0;
    int sm_count = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    std::string last_error;
    // scratch owned by the context (activation quantization of lq_q8_0_linear, attention
    // partials); grown with cudaMalloc on demand, freed at lq_destroy
    void* scratch = nullptr;
    size_t scratch_bytes = 0;
    // K-split partial sums of the small-M GEMM (separate from scratch, which may hold that
    // GEMM's activations); reserved ahead by models so that graph capture never allocates
    void* split = nullptr;
    size_t split_bytes = 0;
    // fp16 operands of the prefill GEMM (weights and activations dequantized from Q8_0); grown
    // on demand outside graph capture
    void* wide = nullptr;
    size_t wide_bytes = 0;
    int* err_flag = nullptr;      // device int[4]: kernels report bad inputs here
    // device unsigned[kTileCounters], zero between launches: arrivals of the CTAs that share a
    // GEMM tile (the skinny GEMM's stream-K combine; the last CTA resets its counter)
    unsigned* tile_cnt = nullptr;
    // launch kernels with programmatic stream serialization (PDL): every kernel of the library
    // calls pdl_wait() before it touches data written by earlier kernels
    bool pdl = true;
};

namespace lq {

int set_error(lq_ctx* ctx, int code, const char* fmt, ...);
int check_cuda(lq_ctx* ctx, cudaError_t e, const char* what);
// host-side fault injection: LQ_FAULT=<entry point name> makes that entry fail
bool fault_injected(const char* entry);
// grow ctx scratch to at least `bytes`; returns LQ_OK or an error
int ensure_scratch(lq_ctx* ctx, size_t bytes);
// grows ctx->split (an error while the stream is capturing a graph)
int ensure_split(lq_ctx* ctx, size_t bytes);
// grows ctx->wide (an error while the stream is capturing a graph)
int ensure_wide(lq_ctx* ctx, size_t bytes);
// partial-sum bytes the M x (N, K) Q8_0 GEMM needs when it splits K (0: no split)
size_t gemm_split_bytes(lq_ctx* ctx, int64_t n, int64_t k, int64_t m);
// read + clear the device error flag (synchronises the stream)
int consume_device_error(lq_ctx* ctx, const char* what);
// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) for `func` on ctx->device, once per
// (function, device) and again only when a launch needs more than was set before
int ensure_func_smem(lq_ctx* ctx, const void* func, size_t bytes);

}  // namespace lq

#define LQ_ENTRY(ctx, name)                                                                 \
    do {                                                                                    \
        if (!(ctx)) return LQ_ERR_INVALID_ARG;                                              \
        if (lq::fault_injected(name))                                                       \
            return lq::set_error((ctx), LQ_ERR_INJECTED, "%s: injected fault (LQ_FAULT)", name); \
    } while (0)

#define LQ_REQUIRE(ctx, cond, ...)                                                          \
    do {                                                                                    \
        if (!(cond)) return lq::set_error((ctx), LQ_ERR_INVALID_ARG, __VA_ARGS__);          \
    } while (0)

#define LQ_CUDA(ctx, expr)                                                                  \
    do {                                                                                    \
        cudaError_t e__ = (expr);                                                           \
        if (e__ != cudaSuccess) return lq::check_cuda((ctx), e__, #expr);                   \
    } while (0)

#define LQ_LAUNCH_CHECK(ctx, what) LQ_CUDA(ctx, cudaGetLastError())

// ------------------------------------------------------------------------------------------
// device helpers
// ------------------------------------------------------------------------------------------
namespace lq {

constexpr int QK = 32;

// bf16.rs:112-131: f32 -> bf16 with bias 0x7FFF + lsb (wrapping 32-bit add)
__host__ __device__ __forceinline__ uint16_t f32_to_bf16(float f) {
#ifdef __CUDA_ARCH__
    uint32_t bits = __float_as_uint(f);
#else
    uint32_t bits;
    memcpy(&bits, &f, 4);
#endif
    return (uint16_t)((bits + 0x7FFFu + ((bits >> 16) & 1u)) >> 16);
}
__host__ __device__ __forceinline__ float bf16_to_f32(uint16_t h) {
#ifdef __CUDA_ARCH__
    return __uint_as_float((uint32_t)h << 16);
#else
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
#endif
}
// round an f32 to the nearest bf16 value, kept in f32
__device__ __forceinline__ float round_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

// GGML Q8_0 scale for a block whose max |x| is amax: d = amax/127, id = d ? 1/d : 0
__device__ __forceinline__ void q8_scale(float amax, float& d, float& id) {
    d = __fdiv_rn(amax, 127.0f);
    id = d != 0.0f ? __frcp_rn(d) : 0.0f;
}
// q = clamp(roundf(x*id), -127, 127) as int
__device__ __forceinline__ int q8_quant(float x, float id) {
    float r = roundf(__fmul_rn(x, id));
    r = fminf(fmaxf(r, -127.0f), 127.0f);
    return (int)r;
}

// streaming 128-bit load that does not allocate in L1
__device__ __forceinline__ int4 ld_stream_v4(const void* p) {
    int4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.s32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// orderable key of an f32 for "max value, ties -> highest index" 64-bit atomicMax
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    if (v == 0.0f) v = 0.0f;  // -0 and +0 compare equal in the reference
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(uint32_t)idx;
}

// SplitMix64 and the Irwin-Hall(4) generator shared with the CPU oracle
__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__host__ __device__ __forceinline__ uint64_t gen_key(uint64_t seed, uint64_t tensor_id) {
    return splitmix64(seed ^ (tensor_id * 0xD1B54A32D192ED03ull));
}
inline float gen_scale(double std_dev) { return (float)(std_dev * 1.7320508075688772 / 65536.0); }
__device__ __forceinline__ float gen_value(uint64_t key, uint64_t idx, float scale) {
    uint64_t h = splitmix64(key + idx);
    int32_t s = (int32_t)(h & 0xFFFFu) + (int32_t)((h >> 16) & 0xFFFFu) +
                (int32_t)((h >> 32) & 0xFFFFu) + (int32_t)((h >> 48) & 0xFFFFu) - 131070;
    return __fmul_rn((float)s, scale);
}

inline int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

// Launch on the context's stream; with ctx->pdl the launch may overlap the tail of the
// preceding kernel (programmatic dependent launch), which the kernel orders with pdl_wait().
template <typename... KArgs, typename... Args>
inline int launch_kernel(lq_ctx* ctx, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                         const char* what, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = ctx->pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ((KArgs)args)...);
    if (e != cudaSuccess) return check_cuda(ctx, e, what);
    return LQ_OK;
}

}  // namespace lq

// kernels launched across translation units
namespace lq {
int launch_quantize_rows(lq_ctx* ctx, const void* src, lq_dtype dt, int64_t rows, int64_t k,
                         int8_t* qs, uint16_t* d);
// a caller-owned buffer for the K-split partial sums of the small-M GEMM: when given, the
// matmul uses it instead of growing ctx->split (and fails with LQ_ERR_STATE if it is short)
struct SplitBuf {
    float* p;
    size_t bytes;
};
int launch_q8_matmul(lq_ctx* ctx, const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd,
                     int64_t m, float* y, const float* resid, int64_t ldy,
                     unsigned long long* argmax_keys, const SplitBuf* split = nullptr);
bool gemv_stream_supported(int64_t K);
// prefill GEMM on tcgen05 (m >= 64 tokens, K % 256 == 0, 16-byte aligned operands)
bool gemm_tc_supported(int64_t m, int64_t K, const void* wq, const void* xq, const void* wd, const void* xd);
// prefill GEMM through fp16 operands (m >= 128 rows, K % 64 == 0): weights and activations
// dequantized from Q8_0 into ctx->wide, one fp16 tcgen05 GEMM with f32 accumulation. Returns
// LQ_ERR_UNSUPPORTED (nothing launched) when the shape does not qualify.
int launch_gemm_f16(lq_ctx* ctx, const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd, int64_t m, float* y,
                    const float* resid, int64_t ldy);
// the prefill projections: launch_gemm_f16 when it qualifies (LQ_PREFILL_EXACT=1 turns it off),
// else launch_q8_matmul
int launch_q8_matmul_prefill(lq_ctx* ctx, const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd, int64_t m,
                             float* y, const float* resid, int64_t ldy);
int launch_gemm_tc(lq_ctx* ctx, const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd, int64_t m, float* y,
                   const float* resid, int64_t ldy);
size_t gemv_stream_smem(int64_t m, int64_t K);
// decode GEMV (m <= 4, K % 256 == 0) on pre-quantized activations
int launch_gemv_stream(lq_ctx* ctx, const lq_q8_tensor* w, const int8_t* xq, const uint16_t* xd, int64_t m,
                       float* y, const float* resid, int64_t ldy, unsigned long long* keys);
// decode GEMV whose prologue is RMSNorm + Q8_0 of the f32 rows x [m][K]
int launch_gemv_norm(lq_ctx* ctx, const lq_q8_tensor* w, const float* x, const uint16_t* norm_w, float eps,
                     int64_t m, float* y, const float* resid, int64_t ldy, unsigned long long* keys);
// decode GEMV of the fused [gate; up] weight (2I rows) with the RMSNorm prologue and the
// SwiGLU epilogue: h [m][I] (row stride ldh) = silu(x.gate^T) * (x.up^T)
int launch_gemv_norm_swiglu(lq_ctx* ctx, const lq_q8_tensor* w, const float* x, const uint16_t* norm_w, float eps,
                            int64_t m, float* h, int64_t ldh);
// decode GEMV whose prologue is the Q8_0 quantization of the f32 rows x [m][K]
int launch_gemv_quant(lq_ctx* ctx, const lq_q8_tensor* w, const float* x, int64_t m, float* y, const float* resid,
                      int64_t ldy);
// decode attention (L = 1) with q/k RMSNorm, RoPE and the KV-cache append fused in; reads the
// fused q|k|v projection rows qkv [B][(Hq+2Hkv)*128]
int launch_attention_decode_fused(lq_ctx* ctx, const float* qkv, const uint16_t* qn, const uint16_t* kn,
                                  float eps, const float* cos_t, const float* sin_t, float* kc, float* vc,
                                  int64_t B, int64_t Hq, int64_t Hkv, const int32_t* pos_dev, int64_t ctx_max,
                                  int8_t* xq, uint16_t* xd, void* scratch);
// the same steps for batched decode rows through the ring chunk kernel and the merge kernel
int launch_attention_decode_qkv(lq_ctx* ctx, const float* qkv, const uint16_t* qn, const uint16_t* kn, float eps,
                                const float* cos_t, const float* sin_t, float* kc, float* vc, int64_t B, int64_t Hq,
                                int64_t Hkv, const int32_t* pos_dev, int64_t ctx_max, int8_t* xq, uint16_t* xd,
                                void* scratch);
int launch_fill_bf16(lq_ctx* ctx, uint64_t seed, uint64_t tid, int64_t offset, int64_t count,
                     float scale, uint16_t* out);
// rows x cols slice, at (row0, col0), of the generated tensor `tid` whose rows are src_ld long
int launch_fill_bf16_2d(lq_ctx* ctx, uint64_t seed, uint64_t tid, int64_t rows, int64_t cols, int64_t src_ld,
                        int64_t row0, int64_t col0, float scale, uint16_t* out);
int launch_fill_norm(lq_ctx* ctx, uint64_t seed, uint64_t tid, int64_t count, float norm_std,
                     uint16_t* out);
// out: tokens from the keys (NULL: keep what a sampler wrote); gen: generated-token history
// [rows][gen_ld] appended at n (n_host, or *pos_counter - *gen_base + 1 when n_host < 0)
int launch_argmax_finalize(lq_ctx* ctx, unsigned long long* keys, int64_t rows, int32_t* out,
                           int32_t* pos_counter, int32_t* gen = nullptr, int64_t gen_ld = 0, int n_host = 0,
                           const int32_t* gen_base = nullptr);
// prefill attention (L >= 16 query positions per sequence): tiles of 128 (position, head) rows
bool attention_prefill_supported(int64_t L, int64_t Hq, int64_t Hkv);
int launch_attention_prefill(lq_ctx* ctx, const float* q, const float* kc, const float* vc, int64_t B, int64_t Hq,
                             int64_t Hkv, int64_t L, int64_t pos0, const int32_t* pos0_dev, int64_t ctx_max,
                             float* out, int8_t* xq, uint16_t* xd);
// tensor-parallel collectives on the communicator's context stream (lq8_comm.cu)
int comm_allreduce_sum_f32(lq_comm* c, const float* send, float* recv, int64_t count);
int comm_allreduce_max_u64(lq_comm* c, unsigned long long* buf, int64_t count);
int comm_allgather_f32(lq_comm* c, const float* send, float* recv, int64_t count);
int comm_rank(const lq_comm* c);
// one-shot all-reduce of up to ALLREDUCE_ROWS rows over CUDA-IPC exchange regions (every rank's
// region mapped by every rank; layout from allreduce_layout, zeroed before first use):
// x [rows][H] = sum over ranks of part (rank order); replaces the NCCL all-reduce of decode rows
constexpr int ALLREDUCE_ROWS = 8;
constexpr int ALLREDUCE_CTAS = 32;
constexpr int ALLREDUCE_MAX_TP = 8;
struct AllreduceRegions {
    void* region[ALLREDUCE_MAX_TP];
    int tp, rank;
};
size_t allreduce_layout(int64_t H, int tp, size_t* flags_off, size_t* done_off, size_t* norm_off = nullptr);
int launch_xchg_allreduce(lq_ctx* ctx, const AllreduceRegions& ar, const float* part, int64_t rows, int64_t H,
                          float* x);
// the same all-reduce fused with the RMSNorm (bf16 weights w) + Q8_0 quantization of the summed
// rows into xq/xd: rows <= ALLREDUCE_ROWS, H % 1024 == 0; opt-in (LQ_AR_NORM=1): slower than
// the all-reduce kernel followed by the RMSNorm kernel at 32B tp2 batch 8 (933.5 vs 984.5 tok/s)
bool xchg_allreduce_norm_supported(int64_t rows, int64_t H);
int launch_xchg_allreduce_norm(lq_ctx* ctx, const AllreduceRegions& ar, const float* part, int64_t rows, int64_t H,
                               float* x, const uint16_t* w, float eps, int8_t* xq, uint16_t* xd);
int comm_world(const lq_comm* c);
lq_ctx* comm_ctx(const lq_comm* c);
// add `offset` to the index half of the non-zero argmax keys (a vocabulary shard's base)
int launch_keys_offset(lq_ctx* ctx, unsigned long long* keys, int64_t n, int64_t offset);
// Qwen3-MoE sparse MLP (router, top-k, grouped expert GEMVs, combine); scratch from
// moe_scratch_bytes for `rows` tokens
size_t moe_scratch_bytes(int64_t rows, int64_t E, int64_t top_k, int64_t H, int64_t inter);
int launch_moe(lq_ctx* ctx, const lq_q8_tensor* router, const lq_q8_tensor* gate_up, const lq_q8_tensor* down,
               int64_t E, int64_t inter, int64_t top_k, int norm_topk, const int8_t* xq, const uint16_t* xd,
               int64_t rows, int64_t H, float* out, const float* resid, void* scratch, int32_t* ids_out,
               float* w_out, int64_t e_lo, int64_t e_hi);  // experts [e_lo, e_hi) only (e_hi <= e_lo: all)
size_t attention_scratch_bytes(int64_t rows, int64_t n_heads, int64_t ctx_max, int64_t head_dim);
int attention_max_ctx();
// scratch starts with per-(row, kv head) counters that must be zero before the first launch;
// every launch leaves them zero again (zero_counters re-clears them for shared scratch)
int launch_attention(lq_ctx* ctx, const float* q, const float* kc, const float* vc, int64_t B,
                     int64_t Hq, int64_t Hkv, int64_t L, int64_t pos0, const int32_t* pos0_dev,
                     int64_t ctx_max, int64_t D, float* out, int8_t* xq, uint16_t* xd,
                     void* scratch, bool zero_counters);
int launch_rmsnorm(lq_ctx* ctx, const void* x, lq_dtype dt, int64_t rows, int64_t dim,
                   const uint16_t* w, float eps, uint16_t* out, int8_t* xq, uint16_t* xd);
int launch_qk_norm_rope_kv(lq_ctx* ctx, const float* qkv, int64_t B, int64_t L, int64_t Hq,
                           int64_t Hkv, int64_t D, const uint16_t* qn, const uint16_t* kn,
                           float eps, const float* cos_t, const float* sin_t, int64_t pos0,
                           const int32_t* pos0_dev, float* q_out, float* kc, float* vc,
                           int64_t ctx_max);
int launch_silu_mul(lq_ctx* ctx, const float* gu, int64_t m, int64_t inter, float* h, int8_t* xq,
                    uint16_t* xd);
int launch_embedding(lq_ctx* ctx, const uint16_t* table, int64_t vocab, int64_t hidden,
                     const int32_t* ids, int64_t n, float* out);

// the whole dense decode step as one persistent kernel (lq8_decode.cu)
struct PdHostLayer {
    const lq_q8_tensor *qkv, *o, *gate_up, *down;
    const uint16_t *in_norm, *post_norm, *q_norm, *k_norm;
    float *kc, *vc;
};
struct PdLaunch {
    const void* desc;  // decode_persist_desc_bytes, written by decode_persist_write_desc
    int64_t n_layers, m, H, Hq, Hkv, I, V, ctx_max;
    float eps;
    const uint16_t* final_norm;
    const float *cos_t, *sin_t;
    const int32_t* pos_dev;
    float* x;          // [m][H] residual stream (embedded input rows)
    float* qkv;        // [m][(Hq+2Hkv)*128]
    int8_t* att_q;     // [m][Hq*128]
    uint16_t* att_d;   // [m][Hq*4]
    int8_t* hq;        // [m][I] Q8_0 of SiLU(gate)*up (may share att_q's buffer)
    uint16_t* hd;      // [m][I/32]
    float* part;       // decode_persist_part_bytes
    float* logits;     // [m][V]
    unsigned long long* keys;
    unsigned* counters;  // decode_persist_counter_bytes, zeroed by the launch
    // tensor parallelism (tp > 1): every rank's exchange region (decode_persist_xchg_layout),
    // indexed by rank, own included; zero-initialised on every rank before the first step
    int tp = 1, rank = 0;
    int64_t vbase = 0;     // first vocabulary row of this rank's LM-head shard
    int64_t keys_n = 0;    // argmax keys the region holds (the model's max batch)
    void* xchg[8] = {};
};
// the per-rank exchange region of the tensor-parallel persistent step: partial sums
// [2][tp][H/16][8][16] f32 at 0, counters [sm_count + 1] u32 at *flags_off, argmax keys
// [max(8, keys_n)] u64 at *keys_off, step counts [2] u32 at *seq_off; returns the total bytes
size_t decode_persist_xchg_layout(int64_t H, int tp, int sm_count, int64_t keys_n, size_t* flags_off,
                                  size_t* keys_off, size_t* seq_off);
bool decode_persist_supported(lq_ctx* ctx, int64_t m, int64_t H, int64_t Hq, int64_t Hkv, int64_t I,
                              int64_t ctx_max);
size_t decode_persist_desc_bytes(int64_t n_layers);
size_t decode_persist_part_bytes(int64_t m, int64_t Hq);
size_t decode_persist_counter_bytes(int64_t m, int64_t Hkv, int64_t n_layers);
int decode_persist_write_desc(lq_ctx* ctx, void* dev, const PdHostLayer* layers, int64_t n_layers,
                              const lq_q8_tensor* lm_head);
int launch_decode_persist(lq_ctx* ctx, const PdLaunch& a);
// token choice of the reference's generate loop (lq8_sample.cu); n_host < 0: the number of
// generated tokens is *pos - *gen_base + 1 (a decode step of the graph)
int check_sampling(lq_ctx* ctx, const lq_sampling* c);
bool sampling_is_greedy(const lq_sampling& c);
size_t sample_scratch_bytes(int64_t rows, int64_t V);
int launch_sample(lq_ctx* ctx, const float* logits, int64_t rows, int64_t V, int64_t ld, const int32_t* gen,
                  int64_t gen_ld, int n_host, const int32_t* pos, const int32_t* gen_base, const lq_sampling& c,
                  float* scratch, int32_t* out, int32_t* gen_out);
}  // namespace lq
