/*
 * oracle_q8.h -- CPU restatement of lluda-inference's Qwen3 forward path with the
 * Q8_0 linear layers, used ONLY as the checker for the CUDA library.
 *
 * TEST INFRASTRUCTURE. Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * reference arm may load this code. The product library (liblq8.so) never links or calls it.
 *
 * Every function names the reference file:line it restates (paths inside the reference
 * project, crate `lluda-inference`). The Q8_0 block format has no source in the reference
 * (it is a roadmap item, README.md:24,32); it follows the published GGML Q8_0 algorithm
 * (quantize_row_q8_0_ref / ggml_vec_dot_q8_0_q8_0 in ggml-quants.c), pinned here against
 * gguf-py 0.19.0 `gguf.quants.Q8_0`, which states bit-exactness with that C code.
 */
#ifndef ORACLE_Q8_H
#define ORACLE_Q8_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_QK 32  /* elements per Q8_0 block */

/* ---- scalar conversions ------------------------------------------------------------ */
uint16_t orc_f32_to_bf16(float f);          /* bf16.rs:112-131 (bias 0x7FFF + lsb, RNE)     */
float    orc_bf16_to_f32(uint16_t h);        /* bf16.rs:136-142 (exact shift)                 */
uint16_t orc_f32_to_f16(float f);            /* IEEE binary16, round to nearest even          */
float    orc_f16_to_f32(uint16_t h);         /* exact                                         */
void orc_f32_to_bf16_array(const float* x, int64_t n, uint16_t* out);
void orc_bf16_to_f32_array(const uint16_t* x, int64_t n, float* out);

/* ---- seeded integer-exact generators (identical bits on CPU and GPU) ---------------- */
uint64_t orc_splitmix64(uint64_t x);
/* bf16 values approximating N(0, std^2): Irwin-Hall sum of four 16-bit uniforms, scaled by
 * one IEEE f32 multiply and rounded RNE to bf16. `scale` = std / 37837.2266... as f32. */
void orc_gen_bf16(uint64_t seed, uint64_t tensor_id, int64_t offset, int64_t count,
                  float scale, uint16_t* out);
/* token ids uniform in [0, vocab) */
void orc_gen_tokens(uint64_t seed, uint64_t stream, int64_t count, int64_t vocab, int32_t* out);
float orc_gen_scale(double std_dev);

/* ---- Q8_0 (A6-A8) -------------------------------------------------------------------- */
/* quantize rows of x[rows][k] (k % 32 == 0) into SoA qs[rows][k] + d[rows][k/32] (fp16 bits) */
void orc_q8_0_quantize_f32(const float* x, int64_t rows, int64_t k, int8_t* qs, uint16_t* d);
void orc_q8_0_quantize_bf16(const uint16_t* x, int64_t rows, int64_t k, int8_t* qs, uint16_t* d);
/* GGML AoS blocks {fp16 d; int8 qs[32]} (34 bytes) <-> SoA */
void orc_q8_0_pack_blocks(const int8_t* qs, const uint16_t* d, int64_t rows, int64_t k, uint8_t* blocks);
void orc_q8_0_unpack_blocks(const uint8_t* blocks, int64_t rows, int64_t k, int8_t* qs, uint16_t* d);
/* y[m][n] = sum_b (float)sumi_b * (dw[n][b] * dx[m][b]), b ascending, one f32 accumulator.
 * abs_terms (optional) receives sum_b |term_b| per output, used to bound reorder error. */
void orc_q8_0_matmul(const int8_t* xq, const uint16_t* xd, int64_t m,
                     const int8_t* wq, const uint16_t* wd, int64_t n, int64_t k,
                     float* y, float* abs_terms);
/* Linear::forward with a Q8_0 weight: quantize each row of x, then orc_q8_0_matmul. */
void orc_q8_0_linear_f32(const float* x, int64_t m, int64_t k,
                         const int8_t* wq, const uint16_t* wd, int64_t n, float* y);
void orc_q8_0_linear_bf16(const uint16_t* x, int64_t m, int64_t k,
                          const int8_t* wq, const uint16_t* wd, int64_t n, float* y);

/* ---- dense reference matmul (tensor.rs:2716-2753), used for the reference's known answers */
void orc_matmul_2d(const float* a, int64_t m, int64_t k, const float* b, int64_t n, float* c);

/* ---- small ops ------------------------------------------------------------------------ */
/* RMSNorm (rms_norm.rs:123-177): x rounded to bf16, f32 sum of squares, bf16 output */
void orc_rmsnorm_f32(const float* x, int64_t rows, int64_t dim, const uint16_t* w, float eps, uint16_t* out);
void orc_rmsnorm_bf16(const uint16_t* x, int64_t rows, int64_t dim, const uint16_t* w, float eps, uint16_t* out);
/* RoPE tables (rope.rs:77-128): cos/sin [max_pos][head_dim/2] in f32 from f64 */
void orc_rope_tables(int64_t head_dim, int64_t max_pos, double theta, float* cos_t, float* sin_t);
/* apply_rope_to_tensor (rope.rs:245-303) in place on x[bh][seq][head_dim], positions offset.. */
void orc_rope_apply(float* x, int64_t bh, int64_t seq, int64_t head_dim, int64_t offset,
                    const float* cos_t, const float* sin_t);
float orc_silu(float x);                     /* tensor.rs:1955-1990 */
/* argmax over n values, ties -> last index (tensor.rs:2451-2482, Rust max_by) */
int64_t orc_argmax(const float* x, int64_t n);
/* softmax over n values (tensor.rs:1913-1934) */
void orc_softmax(float* x, int64_t n);
/* attention for one (q head, query row): q[D], K/V rows [ctx][D] (stride ld), scores scaled,
 * positions > causal_limit masked with -inf when masked != 0 (attention.rs:368-394). */
void orc_attend_row(const float* q, const float* k, const float* v, int64_t ctx, int64_t ld,
                    int64_t d, int masked, int64_t causal_limit, float* scratch, float* out);

/* ---- Qwen3 model (model.rs, transformer.rs, attention.rs, mlp.rs) -------------------- */
typedef struct {
    int64_t hidden, layers, n_heads, n_kv_heads, head_dim, inter, vocab, max_pos;
    int32_t tied;           /* tie_word_embeddings */
    float eps;
    double theta;
    float init_std;         /* weights ~ N(0, init_std) (integer-exact generator) */
    float norm_std;         /* 0 -> norm weights 1.0; else 1 + N(0,norm_std) */
    /* Mixture of experts (Qwen3-MoE); n_experts == 0 -> dense MLP. Not in the reference:
     * the spec is the Qwen3-MoE sparse block restated in orc_moe_forward below. */
    int64_t n_experts, top_k, moe_inter;
    int32_t norm_topk;      /* renormalise the top-k routing weights to sum 1 */
    int32_t pad_;
} orc_qwen3_config;

typedef struct orc_model orc_model;
/* Builds the model from the seeded generator. layers_limit>0 truncates the stack (CPU sample). */
orc_model* orc_qwen3_create(const orc_qwen3_config* cfg, uint64_t seed, int64_t layers_limit,
                            int64_t ctx_max);
void orc_qwen3_destroy(orc_model* m);
void orc_qwen3_clear(orc_model* m);
/* Qwen3ForCausalLM::forward (model.rs:345-372): ids[L] at offset -> logits[vocab] of last row */
int orc_qwen3_forward(orc_model* m, const int32_t* ids, int64_t L, int64_t offset, float* logits);
/* generate() restricted to greedy decoding (generate.rs:611-661) */
int orc_qwen3_generate(orc_model* m, const int32_t* prompt, int64_t L, int64_t new_tokens,
                       int32_t* out_tokens, float* last_logits);
/* Mixture-of-experts MLP of one layer (Qwen3-MoE convention; the reference has no MoE code):
 * xn [rows][H] bf16 (post_attention_layernorm output), router R [E][H] Q8_0;
 *   logits[e] = Q8_0 dot (the Linear rule, blocks ascending);
 *   p = softmax(logits) in f32 (max, exp, sum ascending, divide);
 *   the top_k experts by logit (ties -> lower expert index), in that order;
 *   w_j = p[e_j], and with norm_topk w_j = w_j / (w_0 + ... + w_{k-1}) (sum in selection order);
 *   expert e: h = silu(gate_e . xn) * (up_e . xn) (f32), y_e = down_e . h (h quantized per row);
 *   out[t] = sum over the selected experts in ascending expert index of w_e * y_e[t] (f32).
 * Writes out [rows][H]; ids/weights [rows][top_k] (selection order) when not NULL. */
void orc_moe_forward(const uint16_t* xn, int64_t rows, int64_t H, int64_t E, int64_t top_k, int64_t inter,
                     int norm_topk, const int8_t* rq, const uint16_t* rd, const int8_t* const* gq,
                     const uint16_t* const* gd, const int8_t* const* uq, const uint16_t* const* ud,
                     const int8_t* const* dq, const uint16_t* const* dd, float* out, int32_t* ids,
                     float* weights);
/* Accessors used by the tests to hand the identical weights to the GPU */
int64_t orc_qwen3_layers(const orc_model* m);
const uint16_t* orc_qwen3_embed(const orc_model* m);      /* [vocab][hidden] bf16 */
/* Q8_0 weight of a layer's linear (kind 0 q,1 k,2 v,3 o,4 gate,5 up,6 down; layer -1 kind 7
 * = lm_head): returns rows, fills *qs / *d with the oracle's buffers. -1 if out of range. */
int64_t orc_qwen3_linear(const orc_model* m, int64_t layer, int kind, const int8_t** qs,
                         const uint16_t** d, int64_t* k);
/* MoE weights: kind 10 router (expert ignored), 11 expert gate, 12 expert up, 13 expert down. */
int64_t orc_qwen3_expert(const orc_model* m, int64_t layer, int64_t expert, int kind, const int8_t** qs,
                         const uint16_t** d, int64_t* k);
/* sample_with_config (generate.rs:687-705) after apply_repetition_penalty (:374-411) for one
 * row of logits; generated = the tokens generated so far (repeats count) */
int32_t orc_sample(const float* logits, int64_t V, const int32_t* generated, int64_t n_generated,
                   float temperature, int64_t top_k, float top_p, float penalty);
/* the same with cr_exp != 0: top-p's exponentials correctly rounded instead of libm's expf
 * (they differ in the last bit for a few inputs; only near-ties at the maximum can see it) */
int32_t orc_sample_ex(const float* logits, int64_t V, const int32_t* generated, int64_t n_generated,
                      float temperature, int64_t top_k, float top_p, float penalty, int cr_exp);
/* generate (generate.rs:611-661) with a sampling configuration */
int orc_qwen3_generate_cfg(orc_model* m, const int32_t* prompt, int64_t L, int64_t new_tokens,
                           float temperature, int64_t top_k, float top_p, float penalty,
                           int32_t* out_tokens, float* last_logits);
void orc_set_threads(int n);
/* test-only noise probe: 1 = RMSNorm sums of squares in reverse order (0 = the reference's) */
void orc_set_sum_order(int reversed);
int orc_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
