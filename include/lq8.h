/*
 * lq8.h -- C ABI of the B200 (sm_100a) Q8_0 linear path for Qwen3 (liblq8.so).
 *
 * This is the drop-in boundary for the lluda-inference crate. Each entry point names the
 * reference interface it replaces (paths inside the reference project, crate
 * lluda-inference). The reference binds nothing like this today; the Rust crate lluda-cuda-sys
 * (rust/lluda-cuda-sys in this repository) carries the matching `extern "C"` block.
 *
 * Conventions
 *  - Every function returns an int status: LQ_OK (0) or a negative lq_status. Nothing aborts
 *    the process; lq_last_error() holds the message of the last failure on that context
 *    (lq_last_error(NULL) gives the last failure of lq_init on this thread). Like the
 *    reference's Result<T, LludaError> (error.rs:17-99) with GPU failures mapped to
 *    LludaError::Msg and no fallback (GPU_DESIGN_PRINCIPLES.md:3-21).
 *  - Pointers named *_dev are device pointers; *_host are host pointers. All device work
 *    is asynchronous on the context's stream unless the name ends in _sync or the
 *    function takes host buffers (those synchronise before returning).
 *  - A context is used by one host thread at a time.
 *  - Q8_0 tensors are stored on the device as SoA: qs int8 [rows][k] and d fp16 bits
 *    [rows][k/32]. lq_q8_0_pack_blocks / unpack_blocks convert to and from the GGML
 *    34-byte block {fp16 d; int8 qs[32]}.
 */
#ifndef LQ8_H
#define LQ8_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define LQ8_ABI_VERSION 3

typedef enum {
    LQ_OK = 0,
    LQ_ERR_INVALID_ARG = -1,
    LQ_ERR_CUDA = -2,
    LQ_ERR_OOM = -3,
    LQ_ERR_UNSUPPORTED = -4,
    LQ_ERR_INJECTED = -5,   /* host-side fault injection: LQ_FAULT=<function name> */
    LQ_ERR_STATE = -6,
    LQ_ERR_NCCL = -7,
    LQ_ERR_TIMEOUT = -8
} lq_status;

typedef enum {
    LQ_DTYPE_F32 = 0,
    LQ_DTYPE_BF16 = 1,
    LQ_DTYPE_F16 = 2,
    LQ_DTYPE_I8 = 3,
    LQ_DTYPE_I32 = 4
} lq_dtype;

typedef struct lq_ctx lq_ctx;
typedef struct lq_model lq_model;

/* Device-resident Q8_0 tensor (the reference's planned QTensor), rows = out_features. */
typedef struct {
    int64_t n;        /* rows (out_features)                  */
    int64_t k;        /* columns (in_features), multiple of 32 */
    int8_t* qs;       /* device [n][k]                         */
    uint16_t* d;      /* device [n][k/32] fp16 bits            */
} lq_q8_tensor;

/* ---------------------------------------------------------------------------------------
 * Context. Replaces the wgpu OnceLock context gpu::get_context (gpu/mod.rs:129-178); a
 * failed init returns an error instead of panicking.
 * ------------------------------------------------------------------------------------- */
int lq_abi_version(void);
int lq_init(int device, lq_ctx** out);
int lq_destroy(lq_ctx* ctx);
const char* lq_last_error(const lq_ctx* ctx);
int lq_set_stream(lq_ctx* ctx, void* cuda_stream);   /* NULL = the context's own stream */
void* lq_get_stream(lq_ctx* ctx);
int lq_synchronize(lq_ctx* ctx);
int lq_device_info(lq_ctx* ctx, int* sm_count, int* cc_major, int* cc_minor, size_t* total_mem);

/* ---------------------------------------------------------------------------------------
 * Device memory. Replaces GpuTensorBuffer upload/download (gpu/buffer.rs:19-300) and
 * Tensor::to_gpu / to_cpu (tensor.rs:2947-3066).
 * ------------------------------------------------------------------------------------- */
int lq_malloc(lq_ctx* ctx, size_t bytes, void** out_dev);
int lq_free(lq_ctx* ctx, void* dev);
int lq_memcpy_h2d(lq_ctx* ctx, void* dst_dev, const void* src_host, size_t bytes);
int lq_memcpy_d2h(lq_ctx* ctx, void* dst_host, const void* src_dev, size_t bytes);
int lq_memset(lq_ctx* ctx, void* dst_dev, int value, size_t bytes);

/* ---------------------------------------------------------------------------------------
 * Q8_0 format (no reference source: README.md:24,32 plan it; GGML Q8_0 block layout from
 * docs/architecture/arch-2026-01-31-qwen3-omni-q8-rust.md:36-38,278).
 * ------------------------------------------------------------------------------------- */
/* Quantize rows [rows][k] of f32 or bf16 into SoA Q8_0 (bit-exact with the GGML rule). The
 * planned Tensor::quantize_q8_0() / QTensor constructor. */
int lq_q8_0_quantize(lq_ctx* ctx, const void* src_dev, lq_dtype src_dtype, int64_t rows,
                     int64_t k, int8_t* qs_dev, uint16_t* d_dev);
/* Host mirror of lq_q8_0_quantize (same bits): src_host [rows][k] f32 or bf16 into qs_host
 * [rows][k] and d_host [rows][k/32]. Needs no context and no GPU (the planned
 * Tensor::quantize_q8_0() on the CPU side of the crate, e.g. for checkpoint packing);
 * failures are reported through lq_last_error(NULL). */
int lq_q8_0_quantize_host(const void* src_host, lq_dtype src_dtype, int64_t rows, int64_t k,
                          int8_t* qs_host, uint16_t* d_host);
int lq_q8_0_pack_blocks(lq_ctx* ctx, const int8_t* qs_dev, const uint16_t* d_dev, int64_t rows,
                        int64_t k, uint8_t* blocks_dev);
int lq_q8_0_unpack_blocks(lq_ctx* ctx, const uint8_t* blocks_dev, int64_t rows, int64_t k,
                          int8_t* qs_dev, uint16_t* d_dev);
/* Q8_0 x Q8_0 matmul: y[m][n] (+)= sum_b sumi_b * (d_w * d_x), activations already
 * quantized. Replaces Tensor::matmul (tensor.rs:804-817) for a Q8_0 right-hand side.
 * residual_dev may be NULL; when given, y = residual + x.W^T (y may alias residual). ldy is
 * the row stride of y and residual in elements (0 = n). */
int lq_q8_0_matmul(lq_ctx* ctx, const lq_q8_tensor* w, const int8_t* xq_dev,
                   const uint16_t* xd_dev, int64_t m, float* y_dev, const float* residual_dev,
                   int64_t ldy);
/* The same product for prefill rows (m >= 128, k % 64 == 0), computed through fp16 operands:
 * the weight blocks dequantized once per call to fp16(q * d), the activation rows to
 * fp16(q * d * 2^-e) with a per-row power of two that keeps them in range, one fp16
 * tensor-core GEMM with f32 accumulation over the whole K. Within 2^-10 * sum_k |w_k x_k| of
 * lq_q8_0_matmul (which is exact) and several times faster at prefill sizes; other shapes
 * take lq_q8_0_matmul. Allocates the fp16 operands in the context on first use. Same
 * arguments as lq_q8_0_matmul. */
int lq_q8_0_matmul_prefill(lq_ctx* ctx, const lq_q8_tensor* w, const int8_t* xq_dev,
                           const uint16_t* xd_dev, int64_t m, float* y_dev, const float* residual_dev,
                           int64_t ldy);
/* Linear::forward (attention.rs:101-136) with a Q8_0 weight: x [m][k] f32 or bf16 is
 * quantized into the context's scratch, then multiplied; y [m][n] f32. */
int lq_q8_0_linear(lq_ctx* ctx, const lq_q8_tensor* w, const void* x_dev, lq_dtype x_dtype,
                   int64_t m, float* y_dev);
/* lq_q8_0_linear that allocates no device memory. It has no counterpart in the reference.
 * lq_q8_0_linear grows its scratch (the quantized rows, and the K-split partial sums of the
 * 5..64-row GEMM) with cudaMalloc/cudaFree, which some callers cannot allow: a latency-bound
 * decode loop (both calls can synchronise the whole device), or a host whose device memory
 * all belongs to its own pool allocator. This variant keeps all of it in a fixed 4 MiB array
 * inside the library's device image instead (present on every GPU that loads liblq8, until
 * process exit). A call needs, each part rounded up to 256 bytes, m*k bytes of quantized rows,
 * 2*m*(k/32) bytes of scales and, for 5..64 rows on a weight with few 64-row tiles, the K-split
 * partials (slices*m*n*4 bytes); calls that need more than 4 MiB fail with LQ_ERR_INVALID_ARG.
 * The first call on a device looks the array's address up (cudaGetSymbolAddress). All calls
 * on a device share the one array, so calls that overlap on the GPU (different streams or
 * contexts of the same device) race; each call writes every scratch byte before it reads it,
 * so nothing needs clearing between calls. The kernels are lq_q8_0_linear's: the output is
 * bit-identical to it. */
int lq_q8_0_linear_noalloc(lq_ctx* ctx, const lq_q8_tensor* w, const void* x_dev,
                           lq_dtype x_dtype, int64_t m, float* y_dev);

/* ---------------------------------------------------------------------------------------
 * Small ops that keep activations on the device.
 * ------------------------------------------------------------------------------------- */
/* RmsNorm::forward (rms_norm.rs:123-177): input rounded to bf16, bf16 output. Either output
 * may be NULL: out_bf16_dev [rows][dim], and/or the Q8_0 quantization of that output
 * (xq_dev [rows][dim], xd_dev [rows][dim/32]) that the next Linear consumes. */
int lq_rmsnorm(lq_ctx* ctx, const void* x_dev, lq_dtype x_dtype, int64_t rows, int64_t dim,
               const uint16_t* w_bf16_dev, float eps, uint16_t* out_bf16_dev,
               int8_t* xq_dev, uint16_t* xd_dev);
/* RotaryEmbedding::new (rope.rs:77-128): cos/sin [max_pos][head_dim/2] f32, built in f64 on
 * the host exactly as the reference does, then uploaded. */
int lq_rope_tables(lq_ctx* ctx, int64_t head_dim, int64_t max_pos, double theta,
                   float* cos_dev, float* sin_dev);
/* Attention::forward steps 2-5 (attention.rs:333-364): from the fused projection output
 * qkv [B*L][(Hq+2*Hkv)*D] (row b*L+l), per-head q/k RMSNorm, RoPE at positions pos0+l
 * (rope.rs:167-303), q to q_out [B][Hq][L][D], k and v appended to the caches
 * [B][Hkv][ctx_max][D] (KvCache::append, attention.rs:507-559). pos0_dev (device int32)
 * overrides pos0 when not NULL. */
int lq_qk_norm_rope_kv(lq_ctx* ctx, const float* qkv_dev, int64_t B, int64_t L,
                       int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
                       const uint16_t* q_norm_dev, const uint16_t* k_norm_dev, float eps,
                       const float* cos_dev, const float* sin_dev, int64_t pos0,
                       const int32_t* pos0_dev, float* q_out_dev, float* k_cache_dev,
                       float* v_cache_dev, int64_t ctx_max);
/* Attention::forward steps 6-9 (attention.rs:366-399) with repeat_kv folded in: q
 * [B][Hq][L][D] against cache positions [0, pos0+L) with the causal mask when L > 1
 * (causal_mask.rs:104-164). Output rows [B*L][Hq*D]: f32 to out_dev and/or Q8_0 to
 * xq_dev/xd_dev (either may be NULL). */
int lq_attention(lq_ctx* ctx, const float* q_dev, const float* k_cache_dev,
                 const float* v_cache_dev, int64_t B, int64_t n_heads, int64_t n_kv_heads,
                 int64_t L, int64_t pos0, const int32_t* pos0_dev, int64_t ctx_max,
                 int64_t head_dim, float* out_dev, int8_t* xq_dev, uint16_t* xd_dev);
/* MLP::forward middle (mlp.rs:153-160, tensor.rs:1955-1990): h = silu(gate) * up from the
 * fused gate/up projection gu [m][2*inter] (gate columns first). h f32 and/or Q8_0. */
int lq_silu_mul(lq_ctx* ctx, const float* gu_dev, int64_t m, int64_t inter, float* h_dev,
                int8_t* xq_dev, uint16_t* xd_dev);
/* Tensor::add (tensor.rs:1236-1290), f32: out = a + b (out may alias a). */
int lq_add(lq_ctx* ctx, const float* a_dev, const float* b_dev, int64_t n, float* out_dev);
/* Embedding::forward (embedding.rs:105-153): bf16 rows widened to f32 [n][hidden]. Ids out
 * of range are an error checked on the device; the first bad id is reported. */
int lq_embedding(lq_ctx* ctx, const uint16_t* table_dev, int64_t vocab, int64_t hidden,
                 const int32_t* ids_dev, int64_t n, float* out_dev);
/* sample_greedy / argmax_last_dim (generate.rs:153-174, tensor.rs:2451-2482): per row,
 * index of the maximum, ties -> highest index. */
int lq_argmax(lq_ctx* ctx, const float* x_dev, int64_t rows, int64_t n, int32_t* out_dev);
/* Token choice of the reference's generate loop (generate.rs:687-705 sample_with_config after
 * :374-411 apply_repetition_penalty): temperature 0 -> greedy (ties -> last index);
 * top_k > 0 -> the largest logit (ties -> first index); top_p < 1 -> the largest probability
 * of softmax(x / T) (ties -> first index); else the largest x * (1/T) (ties -> last). The
 * penalty (>= 1) divides positive and multiplies negative logits of generated tokens, once per
 * occurrence. Validated like GenerationConfig::new (generate.rs:93-126). */
typedef struct lq_sampling {
    float temperature;         /* >= 0; 0: greedy */
    int32_t top_k;             /* >= 0; 0: off */
    float top_p;               /* [0, 1]; 1: off */
    float repetition_penalty;  /* >= 1; 1: off */
} lq_sampling;
/* rows of logits [rows][ld] (device), generated tokens [rows][gen_ld] (device; the first
 * n_generated of each row count), out_dev [rows] (device) */
int lq_sample(lq_ctx* ctx, const float* logits_dev, int64_t rows, int64_t vocab, int64_t ld,
              const int32_t* generated_dev, int64_t gen_ld, int64_t n_generated, const lq_sampling* cfg,
              int32_t* out_dev);
/* Integer-exact seeded generator (bf16 values approximating N(0, std^2)); the CPU oracle
 * implements the same function. */
int lq_fill_bf16(lq_ctx* ctx, uint64_t seed, uint64_t tensor_id, int64_t offset, int64_t count,
                 double std_dev, uint16_t* out_dev);

/* ---------------------------------------------------------------------------------------
 * Tensor parallelism over NCCL (one process per GPU; the reference is single-device).
 * NCCL is opened at run time (libnccl.so.2). Rank 0 creates the id, the host hands it to the
 * other ranks (e.g. torch.distributed), every rank calls lq_comm_init on its own context.
 * Collectives run on the context's stream.
 * ------------------------------------------------------------------------------------- */
#define LQ_COMM_ID_BYTES 128
typedef struct lq_comm lq_comm;
int lq_comm_unique_id(lq_ctx* ctx, uint8_t* id_out /* [LQ_COMM_ID_BYTES] */);
int lq_comm_init(lq_ctx* ctx, const uint8_t* id, int rank, int world, lq_comm** out);
int lq_comm_destroy(lq_comm* comm);
int lq_comm_rank(lq_comm* comm, int* rank, int* world);
/* in-place sum over the ranks of buf_dev [count] f32 */
int lq_comm_allreduce_f32(lq_comm* comm, float* buf_dev, int64_t count);
/* Row-parallel Linear (o_proj / down_proj under TP): w is this rank's K-slice [n][k/world]
 * (whole Q8_0 blocks), x this rank's Q8_0 slice [m][k/world]; y [m][n] f32 = residual
 * (may be NULL, may equal y) + the sum over ranks of x_r . w_r^T. */
int lq_q8_0_matmul_allreduce(lq_ctx* ctx, lq_comm* comm, const lq_q8_tensor* w, const int8_t* xq_dev,
                             const uint16_t* xd_dev, int64_t m, float* y_dev, const float* residual_dev);

/* ---------------------------------------------------------------------------------------
 * Mixture of experts (Qwen3-MoE sparse MLP). The reference has no MoE code (its architecture
 * notes plan one); this follows the Qwen3-MoE sparse block so that a MoE checkpoint's layer
 * is one call: router logits x.R^T (Q8_0), softmax, top_k experts by logit (ties -> lower
 * expert index), weights renormalised over the top_k when norm_topk, expert SwiGLU on Q8_0
 * weights, contributions added in ascending expert index.
 * ------------------------------------------------------------------------------------- */
typedef struct {
    int64_t n_experts, inter, hidden;
    lq_q8_tensor gate_up;   /* [n_experts * 2 * inter][hidden]: expert e's gate rows, then up rows */
    lq_q8_tensor down;      /* [n_experts * hidden][inter] */
} lq_moe_experts;

/* out [rows][hidden] f32 = residual (may be NULL; may equal out) + sum_e w_e * expert_e(x),
 * x given as Q8_0 rows (xq_dev [rows][hidden], xd_dev [rows][hidden/32], e.g. from lq_rmsnorm).
 * ids_out / weights_out [rows][top_k] (selection order; device, may be NULL). Uses the
 * context scratch. */
int lq_moe_forward(lq_ctx* ctx, const lq_q8_tensor* router, const lq_moe_experts* experts,
                   const int8_t* xq_dev, const uint16_t* xd_dev, int64_t rows, int64_t top_k,
                   int norm_topk, float* out_dev, const float* residual_dev, int32_t* ids_out_dev,
                   float* weights_out_dev);

/* Expert-parallel MoE layer (each rank holds experts [first_expert, first_expert + n_experts)
 * of `local`; the router is replicated): out = residual + sum over ALL experts, the same on
 * every rank (this rank's experts, then a sum all-reduce over comm). */
int lq_moe_forward_ep(lq_ctx* ctx, lq_comm* comm, const lq_q8_tensor* router, const lq_moe_experts* local,
                      int64_t first_expert, const int8_t* xq_dev, const uint16_t* xd_dev, int64_t rows,
                      int64_t top_k, int norm_topk, float* out_dev, const float* residual_dev);

/* ---------------------------------------------------------------------------------------
 * Qwen3 model runner (Qwen3ForCausalLM, model.rs:273-372; generate.rs:611-661).
 * ------------------------------------------------------------------------------------- */
typedef struct {
    int64_t hidden, layers, n_heads, n_kv_heads, head_dim, inter, vocab, max_pos;
    int32_t tied;       /* tie_word_embeddings */
    float eps;
    double theta;
    float init_std;     /* random-init weights ~ N(0, init_std) (seeded generator) */
    float norm_std;     /* 0 -> norm weights 1.0 */
    /* Qwen3-MoE: n_experts > 0 replaces every layer's MLP by the sparse block (lq_moe_forward)
     * with top_k experts of moe_inter; inter is then unused. */
    int64_t n_experts, top_k, moe_inter;
    int32_t norm_topk;  /* renormalise the top-k routing weights */
    int32_t pad_;
} lq_qwen3_config;

/* Builds the model with seeded random-init weights, all linears Q8_0 (Qwen3ForCausalLM::load,
 * model.rs:273-302; the weights come from the generator instead of safetensors). KV caches
 * for max_batch sequences of ctx_max positions. */
int lq_qwen3_create(lq_ctx* ctx, const lq_qwen3_config* cfg, uint64_t seed, int64_t max_batch,
                    int64_t ctx_max, lq_model** out);
/* Tensor-parallel shard of the same model on this rank of comm: q/k/v and gate/up split by
 * output rows (heads, intermediate), o and down by K (whole Q8_0 blocks) followed by a sum
 * all-reduce, the LM head by vocabulary rows with a global greedy argmax (ties -> highest
 * index). Needs n_heads, n_kv_heads, inter/32 and vocab divisible by the world size and an
 * untied LM head. For a MoE config the split is expert-parallel instead: attention, router
 * and LM head replicated, n_experts / world experts per rank, one sum all-reduce per MoE
 * layer. Every rank makes the same calls with the same ids. */
int lq_qwen3_create_tp(lq_ctx* ctx, const lq_qwen3_config* cfg, uint64_t seed, int64_t max_batch,
                       int64_t ctx_max, lq_comm* comm, lq_model** out);
int lq_qwen3_destroy(lq_model* model);
/* clear_kv_cache (model.rs:396) */
int lq_qwen3_reset(lq_model* model);
/* Prefill B sequences of L tokens (ids_host [B][L]) from position 0; next_host [B] gets the
 * greedy next token; logits_host [B][vocab] (may be NULL) the last-row logits. */
int lq_qwen3_prefill(lq_model* model, const int32_t* ids_host, int64_t B, int64_t L,
                     int32_t* next_host, float* logits_host);
/* One decode step (Qwen3ForCausalLM::forward with L=1 + sample_greedy): ids_host [B] in,
 * next_host [B] out, logits_host [B][vocab] optional. Replays a CUDA graph. */
int lq_qwen3_decode_step(lq_model* model, const int32_t* ids_host, int32_t* next_host,
                         float* logits_host);
/* Device-resident decode: consumes the model's current token buffer, writes the next tokens
 * back into it; no host copies, no synchronisation. n_steps steps. */
int lq_qwen3_decode_device(lq_model* model, int64_t n_steps);
/* Batch size (1..max_batch) of the decode graph; the default is max_batch. */
int lq_qwen3_set_batch(lq_model* model, int64_t B);
/* Token choice for the following prefill and decode steps (see lq_sampling; default greedy).
 * The device keeps each sequence's generated tokens (reset by every prefill) for the
 * repetition penalty. Non-greedy choices need the whole vocabulary on the rank (not under
 * tensor parallelism). */
int lq_qwen3_set_sampling(lq_model* model, const lq_sampling* cfg);
/* The device token buffer [max_batch] int32 used by lq_qwen3_decode_device. */
int lq_qwen3_token_buffer(lq_model* model, int32_t** tokens_dev);
int lq_qwen3_position(lq_model* model, int64_t* pos);
/* Access to a layer's Q8_0 linear (kind: 0 q,1 k,2 v,3 o,4 gate,5 up,6 down, 8 fused q/k/v,
 * 9 fused gate/up; layer -1 with kind 7 = lm_head). Returned pointers alias the model's
 * device buffers. */
int lq_qwen3_linear(lq_model* model, int64_t layer, int kind, lq_q8_tensor* out);
/* Bytes of Q8_0 weights streamed per decode step (for rooflines). */
int lq_qwen3_weight_bytes(lq_model* model, int64_t* bytes);
/* Access to a bf16 parameter: kind 20 input norm, 21 post-attention norm, 22 q norm, 23 k norm
 * of a layer; layer -1 with kind 24 final norm, 25 embedding table [vocab][hidden]. *dev_out
 * aliases the model's buffer (load a checkpoint by writing into it); *count = elements. */
int lq_qwen3_tensor(lq_model* model, int64_t layer, int kind, uint16_t** dev_out, int64_t* count);
/* MoE weights of a layer: kind 10 router (expert ignored), 11 gate, 12 up, 13 down of
 * `expert` (views into the stacked expert tensors). */
int lq_qwen3_expert(lq_model* model, int64_t layer, int64_t expert, int kind, lq_q8_tensor* out);
/* Kernel launches in one decode step (kernel nodes of the captured CUDA graph; 0 before the
 * first decode step or lq_qwen3_set_batch). */
int lq_qwen3_graph_kernels(lq_model* model, int64_t* n);

#ifdef __cplusplus
}
#endif

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#endif
