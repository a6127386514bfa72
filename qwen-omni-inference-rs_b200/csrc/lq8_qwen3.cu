// lq8_qwen3.cu -- Qwen3ForCausalLM runner on the Q8_0 kernels (model.rs:273-372,
// transformer.rs:180-204, attention.rs:318-403, mlp.rs:151-164, generate.rs:611-661).
//
// Weights are random-init from the seeded generator shared with the CPU oracle, quantized to
// Q8_0 on the device once at creation. q/k/v share one fused [Nq+2Nk][H] Q8_0 buffer and
// gate/up one [2I][H] buffer (rows are independent, so fusing changes no result), so one
// decode layer streams four weight matrices. The decode step (L = 1) is captured once per
// batch size into a CUDA graph that reads the position and the input tokens from device
// memory and writes the next tokens back in place.
#include "lq8_internal.cuh"

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <vector>

namespace {

enum { K_Q = 0, K_K, K_V, K_O, K_GATE, K_UP, K_DOWN, K_QNORM, K_KNORM, K_INNORM, K_POSTNORM, K_ROUTER };
inline uint64_t tid_layer(int64_t l, int kind) { return ((uint64_t)l << 8) | (uint64_t)kind; }
// expert weights: kind 0 gate, 1 up, 2 down
inline uint64_t tid_expert(int64_t l, int64_t e, int kind) {
    return (1ull << 40) | ((uint64_t)l << 20) | ((uint64_t)e << 4) | (uint64_t)kind;
}
constexpr uint64_t TID_EMBED = 0x7FFF0001ull;
constexpr uint64_t TID_LMHEAD = 0x7FFF0002ull;
constexpr uint64_t TID_FINALNORM = 0x7FFF0003ull;

struct Layer {
    lq_q8_tensor qkv{}, o{}, gate_up{}, down{};
    uint16_t *q_norm = nullptr, *k_norm = nullptr, *in_norm = nullptr, *post_norm = nullptr;
    // MoE: router [E][H], experts stacked: gate/up [E*2I][H] (per expert gate rows then up
    // rows), down [E*H][I]
    lq_q8_tensor router{}, moe_gate_up{}, moe_down{};
};

}  // namespace

struct lq_model {
    lq_ctx* ctx = nullptr;
    lq_qwen3_config c{};
    int64_t max_batch = 0, ctx_max = 0, rows_cap = 0;
    int64_t Nq = 0, Nk = 0, Nqkv = 0, Hqd = 0;
    std::vector<Layer> layers;
    uint16_t* embed = nullptr;
    uint16_t* final_norm = nullptr;
    lq_q8_tensor lm_head{};
    bool lm_head_owned = true;
    float *kc = nullptr, *vc = nullptr;  // [layers][max_batch][Hkv][ctx_max][D]
    float *cos_t = nullptr, *sin_t = nullptr;
    // activations, sized for rows_cap rows
    float* x = nullptr;        // residual stream [rows][H]
    float* x_last = nullptr;   // last rows of each sequence [max_batch][H]
    int8_t* xq = nullptr;      // quantized activation [rows][max(H, Hq*D, I)]
    uint16_t* xd = nullptr;
    float* qkv = nullptr;      // [rows][Nqkv]
    float* q_rot = nullptr;    // [rows][Hq*D]
    float* gu = nullptr;       // [rows][2I]
    float* logits = nullptr;   // [max_batch][V]
    void* att_scratch = nullptr;
    size_t att_scratch_bytes = 0;
    void* moe_scratch = nullptr;         // MoE layers: route/dispatch/expert buffers for rows_cap
    bool moe = false;
    // tensor parallelism: this rank's shard sizes (the whole model when tp == 1)
    lq_comm* comm = nullptr;
    int tp = 1, rank = 0;
    bool ep = false;             // MoE under a communicator: experts split, the rest replicated
    int64_t E_l = 0, e_lo = 0;   // this rank's experts [e_lo, e_lo + E_l)
    int64_t Hq_l = 0, Hkv_l = 0, I_l = 0, V_l = 0, vocab_off = 0;
    float* part = nullptr;       // row-parallel partial sums [rows][H] (tp > 1)
    float* logits_all = nullptr; // gathered logits [tp][max_batch][V_l] (tp > 1)
    unsigned long long* keys = nullptr;  // argmax keys [max_batch]
    int32_t* tokens = nullptr;           // [rows_cap]
    int32_t* pos_dev = nullptr;
    int64_t pos = 0;
    cudaGraphExec_t exec = nullptr;
    int64_t graph_batch = 0;
    int64_t graph_kernels = 0;   // kernel nodes in the decode graph
    bool fused_decode = false;   // the decode GEMVs can take every K of this model
    // the whole decode step as one persistent kernel (dense, one GPU, batch <= persist_batch)
    bool persist = false;
    int64_t persist_batch = 0;
    void* pd_desc = nullptr;         // per-layer tensor maps and pointers
    float* pd_part = nullptr;        // attention chunk partials
    unsigned* pd_counters = nullptr; // grid barrier + chunk counters
    // token choice (generate.rs sample_with_config); greedy keeps the LM head's fused argmax
    lq_sampling samp{0.0f, 0, 1.0f, 1.0f};
    int32_t* gen = nullptr;          // generated tokens [max_batch][ctx_max] (the penalty's history)
    int32_t* gen_base = nullptr;     // device position of the first decode step after prefill
    float* samp_scratch = nullptr;   // [max_batch][vocab] penalized logits
    std::vector<void*> allocs;
    // tensor-parallel persistent step: every rank's exchange region (own: allocated here,
    // peers': opened from their CUDA IPC handles)
    void* xchg[8] = {};
    std::vector<void*> ipc_open;
    // tensor parallelism, decode rows (<= 8) of the per-layer path: the one-shot all-reduce over
    // every rank's CUDA-IPC region instead of NCCL (LQ_TP_NCCL=1 keeps NCCL)
    bool ar_ok = false;
    lq::AllreduceRegions ar{};
};

namespace {

int dalloc(lq_model* m, void** p, size_t bytes) {
    if (bytes == 0) bytes = 256;
    cudaError_t e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) return lq::check_cuda(m->ctx, e, "cudaMalloc (model)");
    m->allocs.push_back(*p);
    return LQ_OK;
}
template <typename T>
int dalloc_t(lq_model* m, T** p, size_t count) {
    return dalloc(m, reinterpret_cast<void**>(p), count * sizeof(T));
}

int alloc_q8(lq_model* m, lq_q8_tensor* t, int64_t n, int64_t k) {
    t->n = n;
    t->k = k;
    int rc = dalloc_t(m, &t->qs, (size_t)(n * k));
    if (rc) return rc;
    return dalloc_t(m, &t->d, (size_t)(n * (k / 32)));
}

// view of rows [r0, r0+n) of a Q8_0 tensor
lq_q8_tensor rows_view(const lq_q8_tensor& t, int64_t r0, int64_t n) {
    lq_q8_tensor v;
    v.n = n;
    v.k = t.k;
    v.qs = t.qs + r0 * t.k;
    v.d = t.d + r0 * (t.k / 32);
    return v;
}

// generate bf16 weights for tensor id `tid` (rows [src_r0, src_r0+n) of a [*][k] tensor) and
// quantize into rows [r0, r0+n) of dst
int gen_linear(lq_model* m, uint16_t* tmp, size_t tmp_elems, uint64_t seed, uint64_t tid,
               const lq_q8_tensor& dst, int64_t r0, int64_t n, int64_t src_r0 = 0) {
    float sc = lq::gen_scale(m->c.init_std);
    int64_t k = dst.k;
    int64_t chunk_rows = std::max<int64_t>(1, (int64_t)(tmp_elems / (size_t)k));
    for (int64_t r = 0; r < n; r += chunk_rows) {
        int64_t rows = std::min(chunk_rows, n - r);
        int rc = lq::launch_fill_bf16(m->ctx, seed, tid, (src_r0 + r) * k, rows * k, sc, tmp);
        if (rc) return rc;
        rc = lq::launch_quantize_rows(m->ctx, tmp, LQ_DTYPE_BF16, rows, k, dst.qs + (r0 + r) * k,
                                      dst.d + (r0 + r) * (k / 32));
        if (rc) return rc;
    }
    return LQ_OK;
}

// row-parallel output (dense TP's o/down, EP's MoE layer): y = x + partial on rank 0, the
// partial elsewhere, the sum over ranks into x
inline bool split_out(const lq_model* m, bool moe_layer) { return m->tp > 1 && (m->ep == moe_layer); }
inline float* rp_out(lq_model* m, bool moe_layer = false) { return split_out(m, moe_layer) ? m->part : m->x; }
inline const float* rp_resid(lq_model* m, bool moe_layer = false) {
    return (split_out(m, moe_layer) && m->rank != 0) ? nullptr : m->x;
}
inline int rp_reduce(lq_model* m, int64_t rows, bool moe_layer = false) {
    if (!split_out(m, moe_layer)) return LQ_OK;
    if (m->ar_ok && rows <= lq::ALLREDUCE_ROWS)
        return lq::launch_xchg_allreduce(m->ctx, m->ar, m->part, rows, m->c.hidden, m->x);
    return lq::comm_allreduce_sum_f32(m->comm, m->part, m->x, rows * m->c.hidden);
}
// dense row-parallel output followed by an RMSNorm with weights w: the sum over ranks, the norm
// and the Q8_0 quantization into xq/xd in one kernel over the exchange regions when it applies
// (*normed then true), else the plain reduction (the caller normalises)
inline int rp_reduce_norm(lq_model* m, int64_t rows, const uint16_t* w, bool* normed) {
    *normed = false;
    if (split_out(m, false) && m->ar_ok && lq::xchg_allreduce_norm_supported(rows, m->c.hidden)) {
        *normed = true;
        return lq::launch_xchg_allreduce_norm(m->ctx, m->ar, m->part, rows, m->c.hidden, m->x, w, m->c.eps, m->xq,
                                              m->xd);
    }
    return rp_reduce(m, rows);
}
// greedy argmax over the vocabulary shards (dense TP): global indices, max over ranks
inline int lm_keys_reduce(lq_model* m, int64_t B) {
    if (m->tp == 1 || m->ep) return LQ_OK;
    int rc = lq::launch_keys_offset(m->ctx, m->keys, B, m->vocab_off);
    if (rc) return rc;
    return lq::comm_allreduce_max_u64(m->comm, m->keys, B);
}

// post_attention_layernorm -> Q8_0, sparse MoE MLP, residual (in place on m->x); under EP
// this rank's experts and a sum all-reduce
int moe_mlp(lq_model* m, const Layer& ly, int64_t rows) {
    const lq_qwen3_config& c = m->c;
    int rc = lq::launch_rmsnorm(m->ctx, m->x, LQ_DTYPE_F32, rows, c.hidden, ly.post_norm, c.eps, nullptr, m->xq,
                                m->xd);
    if (rc) return rc;
    rc = lq::launch_moe(m->ctx, &ly.router, &ly.moe_gate_up, &ly.moe_down, c.n_experts, c.moe_inter, c.top_k,
                        c.norm_topk, m->xq, m->xd, rows, c.hidden, rp_out(m, true), rp_resid(m, true), m->moe_scratch,
                        nullptr, nullptr, m->e_lo, m->e_lo + m->E_l);
    if (rc) return rc;
    return rp_reduce(m, rows, true);
}

// columns [col0, col0 + dst.k) of every row of the [dst.n][src_k] tensor `tid` (a K-slice for
// a row-parallel shard; col0 and dst.k are whole Q8_0 blocks, so the blocks are the full
// tensor's blocks)
int gen_linear_cols(lq_model* m, uint16_t* tmp, size_t tmp_elems, uint64_t seed, uint64_t tid, const lq_q8_tensor& dst,
                    int64_t src_k, int64_t col0) {
    float sc = lq::gen_scale(m->c.init_std);
    const int64_t k = dst.k, n = dst.n;
    int64_t chunk_rows = std::max<int64_t>(1, (int64_t)(tmp_elems / (size_t)k));
    for (int64_t r = 0; r < n; r += chunk_rows) {
        int64_t rows = std::min(chunk_rows, n - r);
        int rc = lq::launch_fill_bf16_2d(m->ctx, seed, tid, rows, k, src_k, r, col0, sc, tmp);
        if (rc) return rc;
        rc = lq::launch_quantize_rows(m->ctx, tmp, LQ_DTYPE_BF16, rows, k, dst.qs + r * k, dst.d + r * (k / 32));
        if (rc) return rc;
    }
    return LQ_OK;
}

void destroy_graph(lq_model* m) {
    if (m->exec) cudaGraphExecDestroy(m->exec);
    m->exec = nullptr;
    m->graph_batch = 0;
}

// One forward pass over B sequences of L new tokens each at positions [pos0, pos0+L)
// (pos_dev overrides pos0 when set). tokens [B*L] must already be in m->tokens. Writes the
// greedy next token of each sequence to m->tokens[0..B) and the last-row logits to m->logits.
// the next token of each row from the last-row logits: the LM head's fused argmax keys when
// the configuration is greedy, else the sampler over m->logits; both append the token to the
// generated-token history (index 0 after a prefill, else position - gen_base + 1) and advance
// the device position when asked
int finish_tokens(lq_model* m, int64_t B, const int32_t* pos_dev, bool bump_pos) {
    lq_ctx* ctx = m->ctx;
    const int n_host = pos_dev ? -1 : 0;
    if (lq::sampling_is_greedy(m->samp))
        return lq::launch_argmax_finalize(ctx, m->keys, B, m->tokens, bump_pos ? m->pos_dev : nullptr, m->gen,
                                          m->ctx_max, n_host, m->gen_base);
    int rc = lq::launch_sample(ctx, m->logits, B, m->c.vocab, m->V_l, m->gen, m->ctx_max, n_host, m->pos_dev,
                               m->gen_base, m->samp, m->samp_scratch, m->tokens, m->gen);
    if (rc) return rc;
    return lq::launch_argmax_finalize(ctx, m->keys, B, nullptr, bump_pos ? m->pos_dev : nullptr);
}

int forward(lq_model* m, int64_t B, int64_t L, int64_t pos0, const int32_t* pos_dev, bool bump_pos) {
    lq_ctx* ctx = m->ctx;
    const lq_qwen3_config& c = m->c;
    const int64_t H = c.hidden, D = c.head_dim, Hq = m->Hq_l, Hkv = m->Hkv_l, I = m->I_l;
    const int64_t rows = B * L;
    int rc;
#define RC(expr) do { rc = (expr); if (rc) return rc; } while (0)
    RC(lq::launch_embedding(ctx, m->embed, c.vocab, H, m->tokens, rows, m->x));
    const size_t kv_layer = (size_t)(m->max_batch * Hkv * m->ctx_max * D);
    if (L == 1 && pos_dev && m->persist && B <= m->persist_batch) {
        // decode, one persistent kernel for every layer and the LM head
        lq::PdLaunch a = {};
        a.desc = m->pd_desc;
        a.n_layers = c.layers;
        a.m = B;
        a.H = H;
        a.Hq = Hq;
        a.Hkv = Hkv;
        a.I = I;
        a.V = m->V_l;
        a.ctx_max = m->ctx_max;
        a.eps = c.eps;
        a.final_norm = m->final_norm;
        a.cos_t = m->cos_t;
        a.sin_t = m->sin_t;
        a.pos_dev = pos_dev;
        a.x = m->x;
        a.qkv = m->qkv;
        a.att_q = m->xq;
        a.att_d = m->xd;
        a.hq = m->xq;  // the attention output is consumed (o) before h is written (gate|up)
        a.hd = m->xd;
        a.part = m->pd_part;
        a.logits = m->logits;
        a.keys = m->keys;
        a.counters = m->pd_counters;
        a.tp = m->tp;
        a.rank = m->rank;
        a.vbase = m->vocab_off;
        a.keys_n = m->max_batch;
        for (int t = 0; t < m->tp && t < 8; t++) a.xchg[t] = m->xchg[t];
        RC(lq::launch_decode_persist(ctx, a));
        RC(finish_tokens(m, B, pos_dev, bump_pos));
        return LQ_OK;
    }
    if (L == 1 && pos_dev && m->fused_decode && B <= 4) {
        // decode, five kernels per layer: [norm -> q|k|v] [q/k norm, RoPE, KV append,
        // attention -> Q8_0] [o + residual] [norm -> gate|up -> SiLU*up] [down + residual]
        for (size_t li = 0; li < m->layers.size(); li++) {
            Layer& ly = m->layers[li];
            float* kc = m->kc + li * kv_layer;
            float* vc = m->vc + li * kv_layer;
            RC(lq::launch_gemv_norm(ctx, &ly.qkv, m->x, ly.in_norm, c.eps, B, m->qkv, nullptr, m->Nqkv, nullptr));
            RC(lq::launch_attention_decode_fused(ctx, m->qkv, ly.q_norm, ly.k_norm, c.eps, m->cos_t, m->sin_t, kc, vc,
                                                 B, Hq, Hkv, pos_dev, m->ctx_max, m->xq, m->xd, m->att_scratch));
            RC(lq::launch_gemv_stream(ctx, &ly.o, m->xq, m->xd, B, rp_out(m), rp_resid(m), H, nullptr));
            RC(rp_reduce(m, B));
            if (m->moe) {
                RC(moe_mlp(m, ly, B));
                continue;
            }
            RC(lq::launch_gemv_norm_swiglu(ctx, &ly.gate_up, m->x, ly.post_norm, c.eps, B, m->gu, I));
            RC(lq::launch_gemv_quant(ctx, &ly.down, m->gu, B, rp_out(m), rp_resid(m), H));
            RC(rp_reduce(m, B));
        }
        RC(lq::launch_gemv_norm(ctx, &m->lm_head, m->x, m->final_norm, c.eps, B, m->logits, nullptr, m->V_l,
                                m->keys));
        RC(lm_keys_reduce(m, B));
        RC(finish_tokens(m, B, pos_dev, bump_pos));
        return LQ_OK;
    }
    // decode steps with a device position (graph replays) of more rows than the fused GEMV path
    // takes: the separate q/k-norm + RoPE + KV append, chunk and merge kernels; LQ_ATT_FUSED=1
    // takes the fused attention kernel instead (one launch, its last chunk CTA merging; slower
    // at 32B batch 8 today: 11.31 against 11.21 ms per step)
    const bool fused_att = L == 1 && pos_dev && m->fused_decode && B <= 256 && getenv("LQ_ATT_FUSED") != nullptr;
    // decode rows with a device position: the ring attention kernel takes the q|k|v rows
    // directly (LQ_ATT_QKV_OFF=1 or LQ_ATT_CP=1: the separate q/k norm + RoPE + append kernel)
    const bool qkv_att = L == 1 && pos_dev && B <= 256 && !fused_att && getenv("LQ_UNFUSED") == nullptr &&
                         getenv("LQ_ATT_QKV_OFF") == nullptr && getenv("LQ_ATT_CP") == nullptr;
    bool normed = false;  // xq/xd already hold the next norm's output (fused with the TP all-reduce)
    for (size_t li = 0; li < m->layers.size(); li++) {
        Layer& ly = m->layers[li];
        float* kc = m->kc + li * kv_layer;
        float* vc = m->vc + li * kv_layer;
        // input_layernorm -> Q8_0
        if (!normed) RC(lq::launch_rmsnorm(ctx, m->x, LQ_DTYPE_F32, rows, H, ly.in_norm, c.eps, nullptr, m->xq, m->xd));
        normed = false;
        // fused q/k/v projection
        RC(lq::launch_q8_matmul_prefill(ctx, &ly.qkv, m->xq, m->xd, rows, m->qkv, nullptr, m->Nqkv));
        if (fused_att) {
            // batched decode: q/k norm, RoPE, KV append, attention and the chunk merge -> Q8_0
            // rows in one kernel (the chunks' last CTA merges)
            RC(lq::launch_attention_decode_fused(ctx, m->qkv, ly.q_norm, ly.k_norm, c.eps, m->cos_t, m->sin_t, kc,
                                                 vc, B, Hq, Hkv, pos_dev, m->ctx_max, m->xq, m->xd, m->att_scratch));
        } else if (qkv_att) {
            // batched decode: q/k norm, RoPE and the KV append inside the ring attention kernel
            RC(lq::launch_attention_decode_qkv(ctx, m->qkv, ly.q_norm, ly.k_norm, c.eps, m->cos_t, m->sin_t, kc, vc,
                                               B, Hq, Hkv, pos_dev, m->ctx_max, m->xq, m->xd, m->att_scratch));
        } else {
        RC(lq::launch_qk_norm_rope_kv(ctx, m->qkv, B, L, Hq, Hkv, D, ly.q_norm, ly.k_norm, c.eps, m->cos_t,
                                      m->sin_t, pos0, pos_dev, m->q_rot, kc, vc, m->ctx_max));
        // attention -> Q8_0 rows [rows][Hq*D]
        if (L == 1) {
            RC(lq::launch_attention(ctx, m->q_rot, kc, vc, B, Hq, Hkv, 1, pos0, pos_dev, m->ctx_max, D, nullptr,
                                    m->xq, m->xd, m->att_scratch, false));
        } else {
            // one sequence at a time keeps the split-K partials within att_scratch
            for (int64_t b = 0; b < B; b++) {
                RC(lq::launch_attention(ctx, m->q_rot + b * L * Hq * D, kc + b * Hkv * m->ctx_max * D,
                                        vc + b * Hkv * m->ctx_max * D, 1, Hq, Hkv, L, pos0, pos_dev, m->ctx_max,
                                        D, nullptr, m->xq + b * L * m->Hqd, m->xd + b * L * (m->Hqd / 32),
                                        m->att_scratch, false));
            }
        }
        }
        // o_proj + residual (transformer.rs:194)
        RC(lq::launch_q8_matmul_prefill(ctx, &ly.o, m->xq, m->xd, rows, rp_out(m), rp_resid(m), H));
        if (m->moe) {
            RC(rp_reduce(m, rows));
            RC(moe_mlp(m, ly, rows));
            continue;
        }
        // (TP: the all-reduce of the o partial sums with post_attention_layernorm -> Q8_0)
        RC(rp_reduce_norm(m, rows, ly.post_norm, &normed));
        // post_attention_layernorm -> Q8_0, gate/up, silu*up -> Q8_0, down + residual
        if (!normed) RC(lq::launch_rmsnorm(ctx, m->x, LQ_DTYPE_F32, rows, H, ly.post_norm, c.eps, nullptr, m->xq, m->xd));
        normed = false;  // consumed: xq / xd now feed gate|up
        RC(lq::launch_q8_matmul_prefill(ctx, &ly.gate_up, m->xq, m->xd, rows, m->gu, nullptr, 2 * I));
        RC(lq::launch_silu_mul(ctx, m->gu, rows, I, nullptr, m->xq, m->xd));
        // (TP: the all-reduce of the down partial sums with the next input norm, or with the final
        // norm when every row is the last of its sequence)
        const bool last = li + 1 == m->layers.size();
        const uint16_t* next_norm = last ? m->final_norm : m->layers[li + 1].in_norm;
        RC(lq::launch_q8_matmul_prefill(ctx, &ly.down, m->xq, m->xd, rows, rp_out(m), rp_resid(m), H));
        if (!last || L == 1)
            RC(rp_reduce_norm(m, rows, next_norm, &normed));
        else
            RC(rp_reduce(m, rows));
    }
    // final norm on the last row of each sequence (model.rs:194, :357-358)
    const float* xlast = m->x;
    if (L > 1) {
        LQ_CUDA(ctx, cudaMemcpy2DAsync(m->x_last, H * sizeof(float), m->x + (L - 1) * H, L * H * sizeof(float),
                                       H * sizeof(float), B, cudaMemcpyDeviceToDevice, ctx->stream));
        xlast = m->x_last;
    }
    if (!normed) RC(lq::launch_rmsnorm(ctx, xlast, LQ_DTYPE_F32, B, H, m->final_norm, c.eps, nullptr, m->xq, m->xd));
    // LM head with the greedy argmax fused into its epilogue
    RC(lq::launch_q8_matmul(ctx, &m->lm_head, m->xq, m->xd, B, m->logits, nullptr, m->V_l, m->keys));
    RC(lm_keys_reduce(m, B));
    RC(finish_tokens(m, B, pos_dev, bump_pos));
#undef RC
    return LQ_OK;
}

int build_graph(lq_model* m, int64_t B) {
    lq_ctx* ctx = m->ctx;
    destroy_graph(m);
    cudaGraph_t g = nullptr;
    LQ_CUDA(ctx, cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
    int rc = forward(m, B, 1, 0, m->pos_dev, true);
    cudaError_t e = cudaStreamEndCapture(ctx->stream, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return lq::check_cuda(ctx, e, "cudaStreamEndCapture");
    size_t nn = 0;
    cudaGraphGetNodes(g, nullptr, &nn);
    std::vector<cudaGraphNode_t> nodes(nn);
    if (nn) cudaGraphGetNodes(g, nodes.data(), &nn);
    m->graph_kernels = 0;
    for (auto nd : nodes) {
        cudaGraphNodeType t;
        if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) m->graph_kernels++;
    }
    e = cudaGraphInstantiate(&m->exec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return lq::check_cuda(ctx, e, "cudaGraphInstantiate");
    m->graph_batch = B;
    return LQ_OK;
}

}  // namespace

extern "C" {

int lq_qwen3_destroy(lq_model* m) {
    if (!m) return LQ_ERR_INVALID_ARG;
    cudaSetDevice(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    destroy_graph(m);
    for (void* p : m->ipc_open) cudaIpcCloseMemHandle(p);
    for (void* p : m->allocs) cudaFree(p);
    delete m;
    return LQ_OK;
}

// the persistent step's device descriptor: per layer the tensor maps of its four matrices, its
// norm weights and its KV-cache slices (rewritten when the caches move)
static int write_persist_desc(lq_model* m) {
    const int64_t D = m->c.head_dim;
    std::vector<lq::PdHostLayer> hl(m->layers.size());
    const size_t kv_layer = (size_t)(m->max_batch * m->Hkv_l * m->ctx_max * D);
    for (size_t l = 0; l < m->layers.size(); l++) {
        const Layer& ly = m->layers[l];
        hl[l] = {&ly.qkv, &ly.o, &ly.gate_up, &ly.down, ly.in_norm, ly.post_norm, ly.q_norm, ly.k_norm,
                 m->kc + l * kv_layer, m->vc + l * kv_layer};
    }
    return lq::decode_persist_write_desc(m->ctx, m->pd_desc, hl.data(), m->c.layers, &m->lm_head);
}

// replace a tracked allocation (the old one is freed)
static void swap_alloc(lq_model* m, void* old_p, void* new_p) {
    for (auto& p : m->allocs)
        if (p == old_p) p = new_p;
    cudaFree(old_p);
}

// KvCache::append grows the reference's cache without a fixed limit (attention.rs:463-592):
// when a prefill or decode step needs more than ctx_max positions, the caches (and the RoPE
// tables, the generated-token history and the attention scratch, all sized by it) move to
// buffers of max(need, 2 ctx_max) positions, up to max_pos and the attention's limit; the
// positions written so far are copied, the decode graph is rebuilt at the next step and the
// persistent step's descriptors are rewritten. Every rank of a tensor-parallel group grows at
// the same call (they make the same calls).
static int grow_context(lq_model* m, int64_t need) {
    if (need <= m->ctx_max) return LQ_OK;
    lq_ctx* ctx = m->ctx;
    const lq_qwen3_config& c = m->c;
    int64_t limit = lq::attention_max_ctx();
    if (c.max_pos > 0) limit = std::min<int64_t>(limit, c.max_pos);
    if (need > limit)
        return lq::set_error(ctx, LQ_ERR_INVALID_ARG, "context of %lld positions exceeds the limit %lld (max_pos, "
                             "attention chunks)", (long long)need, (long long)limit);
    const int64_t old = m->ctx_max, nc = std::min(limit, std::max(need, 2 * old));
    const int64_t D = c.head_dim, rows = c.layers * m->max_batch * m->Hkv_l;
    const int64_t att_rows = std::max<int64_t>(m->max_batch, std::min<int64_t>(m->rows_cap, nc));
    const size_t att_bytes = lq::attention_scratch_bytes(att_rows, m->Hq_l, nc, D);
    LQ_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    void* nb[6] = {};
    const size_t sizes[6] = {(size_t)(rows * nc * D) * 4, (size_t)(rows * nc * D) * 4, (size_t)(nc * D / 2) * 4,
                             (size_t)(nc * D / 2) * 4, (size_t)(m->max_batch * nc) * 4, att_bytes};
    for (int i = 0; i < 6; i++) {
        const cudaError_t e = cudaMalloc(&nb[i], sizes[i]);
        if (e != cudaSuccess) {
            for (int j = 0; j < i; j++) cudaFree(nb[j]);
            return lq::check_cuda(ctx, e, "cudaMalloc (growing the context)");
        }
    }
    float *kc = (float*)nb[0], *vc = (float*)nb[1], *cs = (float*)nb[2], *sn = (float*)nb[3];
    int32_t* gen = (int32_t*)nb[4];
    const size_t ob = (size_t)(old * D) * 4, nbytes = (size_t)(nc * D) * 4;
    LQ_CUDA(ctx, cudaMemcpy2DAsync(kc, nbytes, m->kc, ob, ob, (size_t)rows, cudaMemcpyDeviceToDevice, ctx->stream));
    LQ_CUDA(ctx, cudaMemcpy2DAsync(vc, nbytes, m->vc, ob, ob, (size_t)rows, cudaMemcpyDeviceToDevice, ctx->stream));
    LQ_CUDA(ctx, cudaMemcpy2DAsync(gen, (size_t)nc * 4, m->gen, (size_t)old * 4, (size_t)old * 4, (size_t)m->max_batch,
                                   cudaMemcpyDeviceToDevice, ctx->stream));
    LQ_CUDA(ctx, cudaMemsetAsync(nb[5], 0, att_bytes, ctx->stream));  // chunk counters start at zero
    int rc = lq_rope_tables(ctx, D, nc, c.theta, cs, sn);
    if (rc) return rc;
    LQ_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    destroy_graph(m);
    swap_alloc(m, m->kc, kc);
    swap_alloc(m, m->vc, vc);
    swap_alloc(m, m->cos_t, cs);
    swap_alloc(m, m->sin_t, sn);
    swap_alloc(m, m->gen, gen);
    swap_alloc(m, m->att_scratch, nb[5]);
    m->kc = kc;
    m->vc = vc;
    m->cos_t = cs;
    m->sin_t = sn;
    m->gen = gen;
    m->att_scratch = nb[5];
    m->att_scratch_bytes = att_bytes;
    m->ctx_max = nc;
    // the persistent step reads the caches through its descriptors (its attention takes the same
    // context limit as the growth)
    if (m->persist) return write_persist_desc(m);
    return LQ_OK;
}

// Tensor parallelism, persistent decode step: allocate this rank's exchange region (zeroed),
// then one all-gather of (CUDA IPC handle, persistent batch, SM count, willingness) over the
// communicator; if every rank is willing with the same batch and SM count (the same units fall
// to the same CTA index everywhere), open the peers' regions. A second all-gather confirms that
// every rank opened them, so all ranks decide alike (*want).
static int tp_exchange_setup(lq_model* m, int64_t pb, bool* want) {
    lq_ctx* ctx = m->ctx;
    const int T = m->tp, rank = m->rank;
    constexpr int W = 48;  // words per rank in the hand-over: two IPC handles (16 words each), then metadata
    static_assert(sizeof(cudaIpcMemHandle_t) <= 16 * 4, "IPC handle does not fit the hand-over");
    size_t fo = 0, ko = 0, so = 0, afo = 0, ado = 0;
    const size_t bytes = lq::decode_persist_xchg_layout(m->c.hidden, T, ctx->sm_count, m->max_batch, &fo, &ko, &so);
    const size_t abytes = lq::allreduce_layout(m->c.hidden, T, &afo, &ado);
    int rc = dalloc(m, &m->xchg[rank], bytes);
    if (!rc) rc = dalloc(m, &m->ar.region[rank], abytes);
    if (rc) return rc;
    LQ_CUDA(ctx, cudaMemsetAsync(m->xchg[rank], 0, bytes, ctx->stream));
    LQ_CUDA(ctx, cudaMemsetAsync(m->ar.region[rank], 0, abytes, ctx->stream));
    uint32_t mine[W] = {};
    cudaIpcMemHandle_t h, ha;
    bool ipc = true;
    if (cudaIpcGetMemHandle(&h, m->xchg[rank]) != cudaSuccess || cudaIpcGetMemHandle(&ha, m->ar.region[rank]) != cudaSuccess) {
        cudaGetLastError();
        ipc = false;
    }
    memcpy(mine, &h, sizeof h);
    memcpy(mine + 16, &ha, sizeof ha);
    mine[40] = (uint32_t)pb;
    mine[41] = (uint32_t)ctx->sm_count;
    mine[42] = *want ? 1u : 0u;
    mine[43] = ipc ? 1u : 0u;
    float* dev = nullptr;
    rc = dalloc(m, reinterpret_cast<void**>(&dev), (size_t)(T + 1) * W * 4);
    if (rc) return rc;
    std::vector<uint32_t> all((size_t)T * W);
    LQ_CUDA(ctx, cudaMemcpyAsync(dev, mine, W * 4, cudaMemcpyHostToDevice, ctx->stream));
    rc = lq::comm_allgather_f32(m->comm, dev, dev + W, W);  // bytes are moved, not added
    if (rc) return rc;
    LQ_CUDA(ctx, cudaMemcpyAsync(all.data(), dev + W, (size_t)T * W * 4, cudaMemcpyDeviceToHost, ctx->stream));
    LQ_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    bool ok = true;   // every rank can share its regions
    bool pers = true;  // ... and takes the persistent step with the same batch and SM count
    for (int t = 0; t < T; t++) {
        const uint32_t* r = all.data() + (size_t)t * W;
        ok = ok && r[43] == 1u;
        pers = pers && r[40] == (uint32_t)pb && r[41] == (uint32_t)ctx->sm_count && r[42] == 1u;
    }
    for (int t = 0; t < T && ok; t++) {
        if (t == rank) continue;
        for (int k = 0; k < 2 && ok; k++) {
            cudaIpcMemHandle_t ph;
            memcpy(&ph, all.data() + (size_t)t * W + 16 * k, sizeof ph);
            void* p = nullptr;
            if (cudaIpcOpenMemHandle(&p, ph, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                cudaGetLastError();
                ok = false;
                break;
            }
            m->ipc_open.push_back(p);
            (k == 0 ? m->xchg[t] : m->ar.region[t]) = p;
        }
    }
    // every rank opened every peer's regions, or none uses them
    uint32_t flag[W] = {};
    flag[0] = ok ? 1u : 0u;
    LQ_CUDA(ctx, cudaMemcpyAsync(dev, flag, W * 4, cudaMemcpyHostToDevice, ctx->stream));
    rc = lq::comm_allgather_f32(m->comm, dev, dev + W, W);
    if (rc) return rc;
    LQ_CUDA(ctx, cudaMemcpyAsync(all.data(), dev + W, (size_t)T * W * 4, cudaMemcpyDeviceToHost, ctx->stream));
    LQ_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    for (int t = 0; t < T; t++) ok = ok && all[(size_t)t * W] == 1u;
    *want = ok && pers;
    if (*want) m->keys = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(m->xchg[rank]) + ko);
    m->ar.tp = T;
    m->ar.rank = rank;
    m->ar_ok = ok && T <= lq::ALLREDUCE_MAX_TP && getenv("LQ_TP_NCCL") == nullptr;
    return LQ_OK;
}

static int create_model(lq_ctx* ctx, const lq_qwen3_config* cfg, uint64_t seed, int64_t max_batch, int64_t ctx_max,
                        lq_comm* comm, lq_model** out) {
    LQ_REQUIRE(ctx, cfg && out, "lq_qwen3_create: NULL argument");
    *out = nullptr;
    const int T = lq::comm_world(comm), rank = lq::comm_rank(comm);
    const lq_qwen3_config& c = *cfg;
    LQ_REQUIRE(ctx, c.head_dim == 128, "lq_qwen3_create: head_dim must be 128");
    const bool moe = c.n_experts > 0;
    LQ_REQUIRE(ctx, c.hidden > 0 && c.hidden % 32 == 0 && (moe || (c.inter % 32 == 0 && c.inter > 0)),
               "lq_qwen3_create: hidden and intermediate sizes must be multiples of 32");
    LQ_REQUIRE(ctx, !moe || (c.top_k > 0 && c.top_k <= 16 && c.top_k <= c.n_experts && c.n_experts <= 512 &&
                             c.moe_inter > 0 && c.moe_inter % 256 == 0 && c.moe_inter <= 8192 &&
                             c.hidden % 256 == 0 && c.hidden <= 8192),
               "lq_qwen3_create: MoE needs 0 < top_k <= min(16, n_experts), n_experts <= 512, hidden and "
               "moe_inter multiples of 256 (at most 8192)");
    LQ_REQUIRE(ctx, c.n_heads > 0 && c.n_kv_heads > 0 && c.n_heads % c.n_kv_heads == 0 &&
                        c.n_heads / c.n_kv_heads <= 8,
               "lq_qwen3_create: need n_heads %% n_kv_heads == 0 and at most 8 q heads per kv head");
    LQ_REQUIRE(ctx, c.layers > 0 && c.vocab > 0 && max_batch > 0 && ctx_max > 0, "lq_qwen3_create: bad sizes");
    LQ_REQUIRE(ctx, c.max_pos <= 0 || ctx_max <= c.max_pos, "lq_qwen3_create: ctx_max exceeds max_pos");
    LQ_REQUIRE(ctx, ctx_max <= lq::attention_max_ctx(), "lq_qwen3_create: ctx_max %lld exceeds %d",
               (long long)ctx_max, lq::attention_max_ctx());
    LQ_REQUIRE(ctx, !comm || lq::comm_ctx(comm) == ctx, "lq_qwen3_create_tp: communicator of another context");
    LQ_REQUIRE(ctx, T == 1 || moe || (!c.tied && c.n_heads % T == 0 && c.n_kv_heads % T == 0 &&
                                       c.inter % (32 * T) == 0 && c.vocab % T == 0),
               "lq_qwen3_create_tp: %d ranks need a dense untied model with n_heads, n_kv_heads, inter/32 and "
               "vocab divisible by the world size", T);
    LQ_REQUIRE(ctx, T == 1 || !moe || c.n_experts % T == 0,
               "lq_qwen3_create_tp: expert parallelism needs n_experts divisible by the world size (%d)", T);

    lq_model* m = new lq_model();
    m->comm = comm;
    m->tp = T;
    m->rank = rank;
    m->ctx = ctx;
    m->c = c;
    m->max_batch = max_batch;
    m->ctx_max = ctx_max;
    m->moe = moe;
    // this rank's shard (the whole model when T == 1; MoE under T > 1: experts only)
    const bool ep = moe && T > 1;
    const int Ta = ep ? 1 : T;  // the attention / dense-MLP / vocabulary split
    const int64_t H = c.hidden, D = c.head_dim, Hq = c.n_heads / Ta, Hkv = c.n_kv_heads / Ta, V = c.vocab;
    const int64_t I = moe ? c.moe_inter : c.inter / T, E = moe ? c.n_experts : 0, Vl = V / Ta;
    const int64_t El = moe ? E / T : 0;
    m->ep = ep;
    m->E_l = El;
    m->e_lo = (int64_t)rank * El;
    m->Hq_l = Hq;
    m->Hkv_l = Hkv;
    m->I_l = I;
    m->V_l = Vl;
    m->vocab_off = ep ? 0 : (int64_t)rank * Vl;
    const int rank_a = ep ? 0 : rank;  // shard index of the attention / vocabulary split
    m->Nq = Hq * D;
    m->Nk = Hkv * D;
    m->Nqkv = m->Nq + 2 * m->Nk;
    m->Hqd = Hq * D;
    // rows per forward pass: whole sequences, at most 8192 rows (or one sequence)
    // (MoE: 2048, which bounds the per-pair expert outputs rows * top_k * hidden)
    const int64_t pass_rows = moe ? 2048 : 8192;
    m->rows_cap = std::max<int64_t>(max_batch, std::min<int64_t>(max_batch * ctx_max, std::max<int64_t>(pass_rows, ctx_max)));
    int rc = LQ_OK;
    auto fail = [&](int code) { lq_qwen3_destroy(m); return code; };
#define RC(expr) do { rc = (expr); if (rc) return fail(rc); } while (0)
    // weights
    m->layers.resize((size_t)c.layers);
    for (auto& ly : m->layers) {
        RC(alloc_q8(m, &ly.qkv, m->Nqkv, H));
        RC(alloc_q8(m, &ly.o, H, m->Hqd));
        if (moe) {
            RC(alloc_q8(m, &ly.router, E, H));
            RC(alloc_q8(m, &ly.moe_gate_up, El * 2 * I, H));
            RC(alloc_q8(m, &ly.moe_down, El * H, I));
        } else {
            RC(alloc_q8(m, &ly.gate_up, 2 * I, H));
            RC(alloc_q8(m, &ly.down, H, I));
        }
        RC(dalloc_t(m, &ly.q_norm, (size_t)D));
        RC(dalloc_t(m, &ly.k_norm, (size_t)D));
        RC(dalloc_t(m, &ly.in_norm, (size_t)H));
        RC(dalloc_t(m, &ly.post_norm, (size_t)H));
    }
    RC(dalloc_t(m, &m->embed, (size_t)(V * H)));
    RC(dalloc_t(m, &m->final_norm, (size_t)H));
    RC(alloc_q8(m, &m->lm_head, Vl, H));
    // generation scratch: the largest single weight, capped at 64 Mi elements
    size_t tmp_elems = (size_t)std::min<int64_t>(std::max({I * H, m->Nq * H, H * m->Hqd}), 64ll << 20);
    uint16_t* tmp = nullptr;
    RC(dalloc_t(m, &tmp, tmp_elems));
    const float sc = lq::gen_scale(c.init_std);
    for (int64_t l = 0; l < c.layers; l++) {
        Layer& ly = m->layers[(size_t)l];
        // column-parallel q/k/v: this rank's heads; row-parallel o: its heads' K columns
        RC(gen_linear(m, tmp, tmp_elems, seed, tid_layer(l, K_Q), ly.qkv, 0, m->Nq, rank_a * m->Nq));
        RC(gen_linear(m, tmp, tmp_elems, seed, tid_layer(l, K_K), ly.qkv, m->Nq, m->Nk, rank_a * m->Nk));
        RC(gen_linear(m, tmp, tmp_elems, seed, tid_layer(l, K_V), ly.qkv, m->Nq + m->Nk, m->Nk, rank_a * m->Nk));
        if (Ta > 1) RC(gen_linear_cols(m, tmp, tmp_elems, seed, tid_layer(l, K_O), ly.o, c.n_heads * D, rank * m->Hqd));
        else RC(gen_linear(m, tmp, tmp_elems, seed, tid_layer(l, K_O), ly.o, 0, H));
        if (moe) {
            RC(gen_linear(m, tmp, tmp_elems, seed, tid_layer(l, K_ROUTER), ly.router, 0, E));
            for (int64_t j = 0; j < El; j++) {  // local slot j holds expert e_lo + j
                const int64_t e = m->e_lo + j;
                RC(gen_linear(m, tmp, tmp_elems, seed, tid_expert(l, e, 0), ly.moe_gate_up, j * 2 * I, I));
                RC(gen_linear(m, tmp, tmp_elems, seed, tid_expert(l, e, 1), ly.moe_gate_up, j * 2 * I + I, I));
                RC(gen_linear(m, tmp, tmp_elems, seed, tid_expert(l, e, 2), ly.moe_down, j * H, H));
            }
        } else {
            RC(gen_linear(m, tmp, tmp_elems, seed, tid_layer(l, K_GATE), ly.gate_up, 0, I, rank * I));
            RC(gen_linear(m, tmp, tmp_elems, seed, tid_layer(l, K_UP), ly.gate_up, I, I, rank * I));
            if (T > 1) RC(gen_linear_cols(m, tmp, tmp_elems, seed, tid_layer(l, K_DOWN), ly.down, c.inter, rank * I));
            else RC(gen_linear(m, tmp, tmp_elems, seed, tid_layer(l, K_DOWN), ly.down, 0, H));
        }
        RC(lq::launch_fill_norm(ctx, seed, tid_layer(l, K_QNORM), D, c.norm_std, ly.q_norm));
        RC(lq::launch_fill_norm(ctx, seed, tid_layer(l, K_KNORM), D, c.norm_std, ly.k_norm));
        RC(lq::launch_fill_norm(ctx, seed, tid_layer(l, K_INNORM), H, c.norm_std, ly.in_norm));
        RC(lq::launch_fill_norm(ctx, seed, tid_layer(l, K_POSTNORM), H, c.norm_std, ly.post_norm));
    }
    RC(lq::launch_fill_bf16(ctx, seed, TID_EMBED, 0, V * H, sc, m->embed));
    RC(lq::launch_fill_norm(ctx, seed, TID_FINALNORM, H, c.norm_std, m->final_norm));
    if (c.tied) {
        // tied embeddings: the LM head is the Q8_0 quantization of the bf16 table
        RC(lq::launch_quantize_rows(ctx, m->embed, LQ_DTYPE_BF16, V, H, m->lm_head.qs, m->lm_head.d));
    } else {
        RC(gen_linear(m, tmp, tmp_elems, seed, TID_LMHEAD, m->lm_head, 0, Vl, rank_a * Vl));
    }
    // caches and activations
    size_t kv = (size_t)(c.layers * max_batch * Hkv * ctx_max * D);
    RC(dalloc_t(m, &m->kc, kv));
    RC(dalloc_t(m, &m->vc, kv));
    RC(dalloc_t(m, &m->cos_t, (size_t)(ctx_max * D / 2)));
    RC(dalloc_t(m, &m->sin_t, (size_t)(ctx_max * D / 2)));
    RC(lq_rope_tables(ctx, D, ctx_max, c.theta, m->cos_t, m->sin_t));
    const int64_t R = m->rows_cap;
    const int64_t kmax = std::max({H, m->Hqd, I});
    RC(dalloc_t(m, &m->x, (size_t)(R * H)));
    RC(dalloc_t(m, &m->x_last, (size_t)(max_batch * H)));
    RC(dalloc_t(m, &m->xq, (size_t)(R * kmax)));
    RC(dalloc_t(m, &m->xd, (size_t)(R * kmax / 32)));
    RC(dalloc_t(m, &m->qkv, (size_t)(R * m->Nqkv)));
    RC(dalloc_t(m, &m->q_rot, (size_t)(R * m->Hqd)));
    RC(dalloc_t(m, &m->gu, (size_t)(R * 2 * I)));
    RC(dalloc_t(m, &m->logits, (size_t)(max_batch * Vl)));
    if (T > 1) RC(dalloc_t(m, &m->part, (size_t)(R * H)));
    if (Ta > 1) RC(dalloc_t(m, &m->logits_all, (size_t)(T * max_batch * Vl)));
    RC(dalloc_t(m, &m->keys, (size_t)max_batch));
    RC(dalloc_t(m, &m->tokens, (size_t)R));
    RC(dalloc_t(m, &m->gen, (size_t)(max_batch * ctx_max)));
    RC(dalloc_t(m, &m->gen_base, 1));
    RC(dalloc_t(m, &m->pos_dev, 1));
    // attention partials: decode (max_batch rows) or one prefill sequence (<= R rows)
    int64_t att_rows = std::max<int64_t>(max_batch, std::min<int64_t>(R, ctx_max));
    m->att_scratch_bytes = lq::attention_scratch_bytes(att_rows, Hq, ctx_max, D);
    RC(dalloc(m, &m->att_scratch, m->att_scratch_bytes));
    if (moe) RC(dalloc(m, &m->moe_scratch, lq::moe_scratch_bytes(R, E, c.top_k, H, I)));
    LQ_CUDA(ctx, cudaMemsetAsync(m->att_scratch, 0, m->att_scratch_bytes, ctx->stream));  // chunk counters
    {
        // the small-M GEMM's K-split partials, reserved now: graph capture cannot allocate
        size_t need = 0;
        const int64_t shapes[5][2] = {{m->Nqkv, H}, {H, m->Hqd}, {2 * I, H}, {H, I}, {Vl, H}};
        for (int64_t rows = 5; rows <= std::min<int64_t>(R, 64); rows++)
            for (const auto& sh : shapes) need = std::max(need, lq::gemm_split_bytes(ctx, sh[0], sh[1], rows));
        if (need) RC(lq::ensure_split(ctx, need));
    }
    LQ_CUDA(ctx, cudaMemsetAsync(m->keys, 0, (size_t)max_batch * 8, ctx->stream));
    LQ_CUDA(ctx, cudaMemsetAsync(m->pos_dev, 0, 4, ctx->stream));
    LQ_CUDA(ctx, cudaMemsetAsync(m->kc, 0, kv * 4, ctx->stream));
    LQ_CUDA(ctx, cudaMemsetAsync(m->vc, 0, kv * 4, ctx->stream));
    LQ_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
#undef RC
    {
        // the fused decode path needs every matmul K on the streaming GEMV (K % 256 == 0,
        // 4 tokens of activations in shared memory); LQ_UNFUSED=1 forces the separate kernels
        bool ok = getenv("LQ_UNFUSED") == nullptr;
        for (int64_t k : {H, m->Hqd, moe ? H : I})
            ok = ok && lq::gemv_stream_supported(k) && lq::gemv_stream_smem(4, k) <= 227 * 1024;
        m->fused_decode = ok;
    }
    {
        // the persistent decode step (dense models, one GPU or tensor-parallel ranks that
        // exchange the o/down partial sums inside the kernel); LQ_NO_PERSIST=1 keeps the
        // per-layer kernels, LQ_TP_NCCL=1 the per-layer kernels with NCCL all-reduces under TP.
        // The largest batch whose activations leave room for the weight ring: up to 4 by default
        // (the dp4a consumers, bit-identical to the per-layer path); LQ_PERSIST_MAX_BATCH=8 also
        // takes batches of 5-8 (tensor-core consumers; slower than the per-layer kernels today).
        int64_t pmax = 4;
        if (const char* e = getenv("LQ_PERSIST_MAX_BATCH")) pmax = std::max<int64_t>(1, std::min<int64_t>(8, atoll(e)));
        int64_t pb = std::min<int64_t>(max_batch, pmax);
        while (pb > 0 && !lq::decode_persist_supported(ctx, pb, H, Hq, Hkv, I, ctx_max)) pb--;
        bool want = !moe && m->fused_decode && pb > 0 && (T == 1 || getenv("LQ_TP_NCCL") == nullptr);
        if (T > 8) want = false;
        if (!moe && T > 1 && T <= 8) {
            // every rank must take the same path: agree on it, and share the exchange regions
            int xrc = tp_exchange_setup(m, pb, &want);
            if (xrc) {
                lq_qwen3_destroy(m);
                return xrc;
            }
        }
        if (want) {
            int prc = dalloc(m, &m->pd_desc, lq::decode_persist_desc_bytes(c.layers));
            if (!prc) prc = dalloc(m, reinterpret_cast<void**>(&m->pd_part), lq::decode_persist_part_bytes(pb, Hq));
            if (!prc)
                prc = dalloc(m, reinterpret_cast<void**>(&m->pd_counters), lq::decode_persist_counter_bytes(pb, Hkv, c.layers));
            if (!prc) prc = write_persist_desc(m);
            if (prc) {
                lq_qwen3_destroy(m);
                return prc;
            }
            m->persist = true;
            m->persist_batch = pb;
        }
    }
    *out = m;
    return LQ_OK;
}

int lq_qwen3_create(lq_ctx* ctx, const lq_qwen3_config* cfg, uint64_t seed, int64_t max_batch, int64_t ctx_max,
                    lq_model** out) {
    LQ_ENTRY(ctx, "lq_qwen3_create");
    return create_model(ctx, cfg, seed, max_batch, ctx_max, nullptr, out);
}

int lq_qwen3_create_tp(lq_ctx* ctx, const lq_qwen3_config* cfg, uint64_t seed, int64_t max_batch, int64_t ctx_max,
                       lq_comm* comm, lq_model** out) {
    LQ_ENTRY(ctx, "lq_qwen3_create_tp");
    LQ_REQUIRE(ctx, comm, "lq_qwen3_create_tp: NULL communicator");
    return create_model(ctx, cfg, seed, max_batch, ctx_max, comm, out);
}

// copy the last-row logits [nb][vocab] to the host, gathering the vocabulary shards (a
// collective under TP: every rank calls it)
static int logits_to_host(lq_model* m, int64_t nb, float* host) {
    lq_ctx* ctx = m->ctx;
    const int64_t V = m->c.vocab, Vl = m->V_l;
    if (m->tp == 1 || m->ep) {
        LQ_CUDA(ctx, cudaMemcpyAsync(host, m->logits, (size_t)(nb * V) * 4, cudaMemcpyDeviceToHost, ctx->stream));
        return LQ_OK;
    }
    int rc = lq::comm_allgather_f32(m->comm, m->logits, m->logits_all, nb * Vl);
    if (rc) return rc;
    for (int t = 0; t < m->tp; t++)
        LQ_CUDA(ctx, cudaMemcpy2DAsync(host + (size_t)t * Vl, (size_t)V * 4, m->logits_all + (size_t)t * nb * Vl,
                                       (size_t)Vl * 4, (size_t)Vl * 4, (size_t)nb, cudaMemcpyDeviceToHost, ctx->stream));
    return LQ_OK;
}

int lq_qwen3_reset(lq_model* m) {
    if (!m) return LQ_ERR_INVALID_ARG;
    LQ_ENTRY(m->ctx, "lq_qwen3_reset");
    m->pos = 0;
    LQ_CUDA(m->ctx, cudaMemsetAsync(m->pos_dev, 0, 4, m->ctx->stream));
    return LQ_OK;
}

int lq_qwen3_prefill(lq_model* m, const int32_t* ids, int64_t B, int64_t L, int32_t* next, float* logits) {
    if (!m) return LQ_ERR_INVALID_ARG;
    lq_ctx* ctx = m->ctx;
    LQ_ENTRY(ctx, "lq_qwen3_prefill");
    LQ_REQUIRE(ctx, ids && next, "lq_qwen3_prefill: NULL argument");
    LQ_REQUIRE(ctx, B > 0 && B <= m->max_batch && L > 0, "lq_qwen3_prefill: B=%lld (max %lld), L=%lld",
               (long long)B, (long long)m->max_batch, (long long)L);
    LQ_REQUIRE(ctx, L <= m->rows_cap, "lq_qwen3_prefill: L=%lld exceeds the %lld rows of one pass", (long long)L,
               (long long)m->rows_cap);
    if (int rc = grow_context(m, L)) return rc;
    for (int64_t i = 0; i < B * L; i++)
        LQ_REQUIRE(ctx, ids[i] >= 0 && ids[i] < m->c.vocab, "lq_qwen3_prefill: token id %d out of range", ids[i]);
    // whole sequences per pass; the KV caches of sequence b live at batch slot b
    int64_t per_pass = std::max<int64_t>(1, m->rows_cap / L);
    const int64_t H = m->c.hidden, D = m->c.head_dim, Hkv = m->Hkv_l;
    for (int64_t b0 = 0; b0 < B; b0 += per_pass) {
        int64_t nb = std::min(per_pass, B - b0);
        LQ_CUDA(ctx, cudaMemcpyAsync(m->tokens, ids + b0 * L, (size_t)(nb * L) * 4, cudaMemcpyHostToDevice,
                                     ctx->stream));
        // point the per-layer cache views at slot b0 by running forward on shifted caches
        // (the cache layout is [layer][batch][Hkv][ctx][D]; a pass over sequences
        // [b0, b0+nb) uses batch offsets b0.. inside each layer)
        float* kc_save = m->kc;
        float* vc_save = m->vc;
        int32_t* gen_save = m->gen;
        m->kc = kc_save + b0 * Hkv * m->ctx_max * D;
        m->vc = vc_save + b0 * Hkv * m->ctx_max * D;
        m->gen = gen_save + b0 * m->ctx_max;
        int rc = forward(m, nb, L, 0, nullptr, false);
        m->kc = kc_save;
        m->vc = vc_save;
        m->gen = gen_save;
        if (rc) return rc;
        LQ_CUDA(ctx, cudaMemcpyAsync(next + b0, m->tokens, (size_t)nb * 4, cudaMemcpyDeviceToHost, ctx->stream));
        if (logits) {
            rc = logits_to_host(m, nb, logits + b0 * m->c.vocab);
            if (rc) return rc;
        }
    }
    (void)H;
    m->pos = L;
    int32_t p = (int32_t)L;
    LQ_CUDA(ctx, cudaMemcpyAsync(m->pos_dev, &p, 4, cudaMemcpyHostToDevice, ctx->stream));
    // the first decode step (position L) samples with one generated token in the history
    LQ_CUDA(ctx, cudaMemcpyAsync(m->gen_base, &p, 4, cudaMemcpyHostToDevice, ctx->stream));
    LQ_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    return lq::consume_device_error(ctx, "lq_qwen3_prefill");
}

static int decode_prepare(lq_model* m, int64_t B) {
    if (m->exec && m->graph_batch == B) return LQ_OK;
    return build_graph(m, B);
}

int lq_qwen3_decode_step(lq_model* m, const int32_t* ids, int32_t* next, float* logits) {
    if (!m) return LQ_ERR_INVALID_ARG;
    lq_ctx* ctx = m->ctx;
    LQ_ENTRY(ctx, "lq_qwen3_decode_step");
    LQ_REQUIRE(ctx, ids && next, "lq_qwen3_decode_step: NULL argument");
    const int64_t B = m->graph_batch ? m->graph_batch : m->max_batch;
    if (int rc = grow_context(m, m->pos + 1)) return rc;
    for (int64_t i = 0; i < B; i++)
        LQ_REQUIRE(ctx, ids[i] >= 0 && ids[i] < m->c.vocab, "lq_qwen3_decode_step: token id %d out of range", ids[i]);
    int rc = decode_prepare(m, B);
    if (rc) return rc;
    LQ_CUDA(ctx, cudaMemcpyAsync(m->tokens, ids, (size_t)B * 4, cudaMemcpyHostToDevice, ctx->stream));
    LQ_CUDA(ctx, cudaGraphLaunch(m->exec, ctx->stream));
    LQ_CUDA(ctx, cudaMemcpyAsync(next, m->tokens, (size_t)B * 4, cudaMemcpyDeviceToHost, ctx->stream));
    if (logits) {
        rc = logits_to_host(m, B, logits);
        if (rc) return rc;
    }
    // synchronises; a kernel that gave up waiting (a stalled copy or grid barrier) reports here
    rc = lq::consume_device_error(ctx, "lq_qwen3_decode_step");
    if (rc) return rc;
    m->pos += 1;
    return LQ_OK;
}

int lq_qwen3_decode_device(lq_model* m, int64_t n_steps) {
    if (!m) return LQ_ERR_INVALID_ARG;
    lq_ctx* ctx = m->ctx;
    LQ_ENTRY(ctx, "lq_qwen3_decode_device");
    const int64_t B = m->graph_batch ? m->graph_batch : m->max_batch;
    LQ_REQUIRE(ctx, n_steps >= 0, "lq_qwen3_decode_device: n_steps=%lld", (long long)n_steps);
    if (int rc = grow_context(m, m->pos + n_steps)) return rc;
    int rc = decode_prepare(m, B);
    if (rc) return rc;
    for (int64_t s = 0; s < n_steps; s++) LQ_CUDA(ctx, cudaGraphLaunch(m->exec, ctx->stream));
    m->pos += n_steps;
    return LQ_OK;
}

int lq_qwen3_set_batch(lq_model* m, int64_t B) {
    if (!m) return LQ_ERR_INVALID_ARG;
    LQ_ENTRY(m->ctx, "lq_qwen3_set_batch");
    LQ_REQUIRE(m->ctx, B > 0 && B <= m->max_batch, "lq_qwen3_set_batch: B=%lld out of range", (long long)B);
    return decode_prepare(m, B);
}

int lq_qwen3_token_buffer(lq_model* m, int32_t** tokens) {
    if (!m || !tokens) return LQ_ERR_INVALID_ARG;
    *tokens = m->tokens;
    return LQ_OK;
}

int lq_qwen3_position(lq_model* m, int64_t* pos) {
    if (!m || !pos) return LQ_ERR_INVALID_ARG;
    *pos = m->pos;
    return LQ_OK;
}

int lq_qwen3_linear(lq_model* m, int64_t layer, int kind, lq_q8_tensor* out) {
    if (!m || !out) return LQ_ERR_INVALID_ARG;
    lq_ctx* ctx = m->ctx;
    if (layer < 0) {
        LQ_REQUIRE(ctx, kind == 7, "lq_qwen3_linear: layer -1 needs kind 7 (lm_head)");
        *out = m->lm_head;
        return LQ_OK;
    }
    LQ_REQUIRE(ctx, layer < (int64_t)m->layers.size(), "lq_qwen3_linear: layer out of range");
    LQ_REQUIRE(ctx, !m->moe || (kind != K_GATE && kind != K_UP && kind != K_DOWN && kind != 9),
               "lq_qwen3_linear: a MoE model has no dense MLP (use lq_qwen3_expert)");
    const Layer& ly = m->layers[(size_t)layer];
    const int64_t I = m->I_l;
    switch (kind) {
        case K_Q: *out = rows_view(ly.qkv, 0, m->Nq); break;
        case K_K: *out = rows_view(ly.qkv, m->Nq, m->Nk); break;
        case K_V: *out = rows_view(ly.qkv, m->Nq + m->Nk, m->Nk); break;
        case K_O: *out = ly.o; break;
        case K_GATE: *out = rows_view(ly.gate_up, 0, I); break;
        case K_UP: *out = rows_view(ly.gate_up, I, I); break;
        case K_DOWN: *out = ly.down; break;
        case 8: *out = ly.qkv; break;       // fused q/k/v as streamed by the decode step
        case 9: *out = ly.gate_up; break;   // fused gate/up
        default: return lq::set_error(ctx, LQ_ERR_INVALID_ARG, "lq_qwen3_linear: kind %d", kind);
    }
    return LQ_OK;
}

int lq_qwen3_expert(lq_model* m, int64_t layer, int64_t expert, int kind, lq_q8_tensor* out) {
    if (!m || !out) return LQ_ERR_INVALID_ARG;
    lq_ctx* ctx = m->ctx;
    LQ_REQUIRE(ctx, m->moe, "lq_qwen3_expert: not a MoE model");
    LQ_REQUIRE(ctx, layer >= 0 && layer < (int64_t)m->layers.size(), "lq_qwen3_expert: layer out of range");
    const Layer& ly = m->layers[(size_t)layer];
    const int64_t I = m->c.moe_inter, H = m->c.hidden;
    if (kind == 10) {
        *out = ly.router;
        return LQ_OK;
    }
    LQ_REQUIRE(ctx, expert >= m->e_lo && expert < m->e_lo + m->E_l,
               "lq_qwen3_expert: expert %lld not held by this rank", (long long)expert);
    const int64_t j = expert - m->e_lo;
    switch (kind) {
        case 11: *out = rows_view(ly.moe_gate_up, j * 2 * I, I); break;
        case 12: *out = rows_view(ly.moe_gate_up, j * 2 * I + I, I); break;
        case 13: *out = rows_view(ly.moe_down, j * H, H); break;
        default: return lq::set_error(ctx, LQ_ERR_INVALID_ARG, "lq_qwen3_expert: kind %d", kind);
    }
    return LQ_OK;
}

int lq_qwen3_tensor(lq_model* m, int64_t layer, int kind, uint16_t** dev_out, int64_t* count) {
    if (!m || !dev_out || !count) return LQ_ERR_INVALID_ARG;
    lq_ctx* ctx = m->ctx;
    const int64_t H = m->c.hidden, D = m->c.head_dim;
    if (layer < 0) {
        switch (kind) {
            case 24: *dev_out = m->final_norm; *count = H; return LQ_OK;
            case 25: *dev_out = m->embed; *count = m->c.vocab * H; return LQ_OK;
            default: return lq::set_error(ctx, LQ_ERR_INVALID_ARG, "lq_qwen3_tensor: layer -1 needs kind 24 or 25");
        }
    }
    LQ_REQUIRE(ctx, layer < (int64_t)m->layers.size(), "lq_qwen3_tensor: layer out of range");
    const Layer& ly = m->layers[(size_t)layer];
    switch (kind) {
        case 20: *dev_out = ly.in_norm; *count = H; break;
        case 21: *dev_out = ly.post_norm; *count = H; break;
        case 22: *dev_out = ly.q_norm; *count = D; break;
        case 23: *dev_out = ly.k_norm; *count = D; break;
        default: return lq::set_error(ctx, LQ_ERR_INVALID_ARG, "lq_qwen3_tensor: kind %d", kind);
    }
    return LQ_OK;
}

int lq_qwen3_set_sampling(lq_model* m, const lq_sampling* cfg) {
    if (!m) return LQ_ERR_INVALID_ARG;
    lq_ctx* ctx = m->ctx;
    LQ_ENTRY(ctx, "lq_qwen3_set_sampling");
    int rc = lq::check_sampling(ctx, cfg);
    if (rc) return rc;
    if (!lq::sampling_is_greedy(*cfg)) {
        LQ_REQUIRE(ctx, m->V_l == m->c.vocab, "lq_qwen3_set_sampling: a vocabulary-sharded LM head (tensor parallel) "
                                              "supports greedy decoding only");
        if (!m->samp_scratch) {
            void* buf = nullptr;
            rc = dalloc(m, &buf, lq::sample_scratch_bytes(m->max_batch, m->c.vocab));
            if (rc) return rc;
            m->samp_scratch = static_cast<float*>(buf);
        }
    }
    m->samp = *cfg;
    destroy_graph(m);  // the decode graph holds the token-choice kernels
    return LQ_OK;
}

int lq_qwen3_graph_kernels(lq_model* m, int64_t* n) {
    if (!m || !n) return LQ_ERR_INVALID_ARG;
    *n = m->graph_kernels;
    return LQ_OK;
}

int lq_qwen3_weight_bytes(lq_model* m, int64_t* bytes) {
    if (!m || !bytes) return LQ_ERR_INVALID_ARG;
    auto q8b = [](const lq_q8_tensor& t) { return t.n * t.k + t.n * (t.k / 32) * 2; };
    int64_t s = q8b(m->lm_head);
    for (auto& ly : m->layers)
        s += q8b(ly.qkv) + q8b(ly.o) + q8b(ly.gate_up) + q8b(ly.down) + q8b(ly.router) + q8b(ly.moe_gate_up) +
             q8b(ly.moe_down);
    *bytes = s;
    return LQ_OK;
}

}  // extern "C"
