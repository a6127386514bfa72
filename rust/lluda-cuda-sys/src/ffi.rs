//! Raw declarations of every entry point in include/lq8.h (the C ABI of liblq8), with the
//! #[repr(C)] structs the ABI passes by pointer. Checked against the header by
//! tests/test_rust_ffi.py (names, argument order and types, struct fields).
//!
//! Conventions of the ABI: every function returns a status (0 = LQ_OK, negative = error
//! class, see LQ_ERR_*); lq_last_error(ctx) holds the message (lq_last_error(null) for
//! lq_init and the context-free host calls). Pointers named *_dev are device memory.
#![allow(non_camel_case_types)]

use std::os::raw::{c_char, c_int, c_void};

pub const LQ8_ABI_VERSION: c_int = 3;

pub const LQ_OK: c_int = 0;
pub const LQ_ERR_INVALID_ARG: c_int = -1;
pub const LQ_ERR_CUDA: c_int = -2;
pub const LQ_ERR_OOM: c_int = -3;
pub const LQ_ERR_UNSUPPORTED: c_int = -4;
pub const LQ_ERR_INJECTED: c_int = -5;
pub const LQ_ERR_STATE: c_int = -6;
pub const LQ_ERR_NCCL: c_int = -7;
pub const LQ_ERR_TIMEOUT: c_int = -8;

/// lq_dtype (a C enum, passed as int)
pub type LqDtype = c_int;
pub const LQ_DTYPE_F32: LqDtype = 0;
pub const LQ_DTYPE_BF16: LqDtype = 1;
pub const LQ_DTYPE_F16: LqDtype = 2;
pub const LQ_DTYPE_I8: LqDtype = 3;
pub const LQ_DTYPE_I32: LqDtype = 4;

pub const LQ_COMM_ID_BYTES: usize = 128;

/// Opaque context (one CUDA device, one stream).
#[repr(C)]
pub struct LqCtx {
    _opaque: [u8; 0],
}
/// Opaque Qwen3 model runner.
#[repr(C)]
pub struct LqModel {
    _opaque: [u8; 0],
}
/// Opaque NCCL communicator.
#[repr(C)]
pub struct LqComm {
    _opaque: [u8; 0],
}

/// lq_q8_tensor: a device Q8_0 tensor, SoA (qs int8 [n][k], d fp16 bits [n][k/32]).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct LqQ8Tensor {
    pub n: i64,
    pub k: i64,
    pub qs: *mut i8,
    pub d: *mut u16,
}

/// lq_sampling: GenerationConfig's knobs (generate.rs:38-64 of lluda-inference).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct LqSampling {
    pub temperature: f32,
    pub top_k: i32,
    pub top_p: f32,
    pub repetition_penalty: f32,
}

/// lq_moe_experts: stacked expert weights (gate|up [E*2I][H], down [E*H][I]).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct LqMoeExperts {
    pub n_experts: i64,
    pub inter: i64,
    pub hidden: i64,
    pub gate_up: LqQ8Tensor,
    pub down: LqQ8Tensor,
}

/// lq_qwen3_config: Qwen3 (and Qwen3-MoE) architecture of a model runner.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct LqQwen3Config {
    pub hidden: i64,
    pub layers: i64,
    pub n_heads: i64,
    pub n_kv_heads: i64,
    pub head_dim: i64,
    pub inter: i64,
    pub vocab: i64,
    pub max_pos: i64,
    pub tied: i32,
    pub eps: f32,
    pub theta: f64,
    pub init_std: f32,
    pub norm_std: f32,
    pub n_experts: i64,
    pub top_k: i64,
    pub moe_inter: i64,
    pub norm_topk: i32,
    pub pad_: i32,
}

extern "C" {
    pub fn lq_abi_version() -> c_int;
    pub fn lq_init(device: c_int, out: *mut *mut LqCtx) -> c_int;
    pub fn lq_destroy(ctx: *mut LqCtx) -> c_int;
    pub fn lq_last_error(ctx: *const LqCtx) -> *const c_char;
    pub fn lq_set_stream(ctx: *mut LqCtx, cuda_stream: *mut c_void) -> c_int;
    pub fn lq_get_stream(ctx: *mut LqCtx) -> *mut c_void;
    pub fn lq_synchronize(ctx: *mut LqCtx) -> c_int;
    pub fn lq_device_info(ctx: *mut LqCtx, sm_count: *mut c_int, cc_major: *mut c_int, cc_minor: *mut c_int, total_mem: *mut usize) -> c_int;
    pub fn lq_malloc(ctx: *mut LqCtx, bytes: usize, out_dev: *mut *mut c_void) -> c_int;
    pub fn lq_free(ctx: *mut LqCtx, dev: *mut c_void) -> c_int;
    pub fn lq_memcpy_h2d(ctx: *mut LqCtx, dst_dev: *mut c_void, src_host: *const c_void, bytes: usize) -> c_int;
    pub fn lq_memcpy_d2h(ctx: *mut LqCtx, dst_host: *mut c_void, src_dev: *const c_void, bytes: usize) -> c_int;
    pub fn lq_memset(ctx: *mut LqCtx, dst_dev: *mut c_void, value: c_int, bytes: usize) -> c_int;
    pub fn lq_q8_0_quantize(ctx: *mut LqCtx, src_dev: *const c_void, src_dtype: c_int, rows: i64, k: i64, qs_dev: *mut i8, d_dev: *mut u16) -> c_int;
    pub fn lq_q8_0_quantize_host(src_host: *const c_void, src_dtype: c_int, rows: i64, k: i64, qs_host: *mut i8, d_host: *mut u16) -> c_int;
    pub fn lq_q8_0_pack_blocks(ctx: *mut LqCtx, qs_dev: *const i8, d_dev: *const u16, rows: i64, k: i64, blocks_dev: *mut u8) -> c_int;
    pub fn lq_q8_0_unpack_blocks(ctx: *mut LqCtx, blocks_dev: *const u8, rows: i64, k: i64, qs_dev: *mut i8, d_dev: *mut u16) -> c_int;
    pub fn lq_q8_0_matmul(ctx: *mut LqCtx, w: *const LqQ8Tensor, xq_dev: *const i8, xd_dev: *const u16, m: i64, y_dev: *mut f32, residual_dev: *const f32, ldy: i64) -> c_int;
    pub fn lq_q8_0_matmul_prefill(ctx: *mut LqCtx, w: *const LqQ8Tensor, xq_dev: *const i8, xd_dev: *const u16, m: i64, y_dev: *mut f32, residual_dev: *const f32, ldy: i64) -> c_int;
    pub fn lq_q8_0_linear(ctx: *mut LqCtx, w: *const LqQ8Tensor, x_dev: *const c_void, x_dtype: c_int, m: i64, y_dev: *mut f32) -> c_int;
    pub fn lq_q8_0_linear_noalloc(ctx: *mut LqCtx, w: *const LqQ8Tensor, x_dev: *const c_void, x_dtype: c_int, m: i64, y_dev: *mut f32) -> c_int;
    pub fn lq_rmsnorm(ctx: *mut LqCtx, x_dev: *const c_void, x_dtype: c_int, rows: i64, dim: i64, w_bf16_dev: *const u16, eps: f32, out_bf16_dev: *mut u16, xq_dev: *mut i8, xd_dev: *mut u16) -> c_int;
    pub fn lq_rope_tables(ctx: *mut LqCtx, head_dim: i64, max_pos: i64, theta: f64, cos_dev: *mut f32, sin_dev: *mut f32) -> c_int;
    pub fn lq_qk_norm_rope_kv(ctx: *mut LqCtx, qkv_dev: *const f32, batch: i64, len: i64, n_heads: i64, n_kv_heads: i64, head_dim: i64, q_norm_dev: *const u16, k_norm_dev: *const u16, eps: f32, cos_dev: *const f32, sin_dev: *const f32, pos0: i64, pos0_dev: *const i32, q_out_dev: *mut f32, k_cache_dev: *mut f32, v_cache_dev: *mut f32, ctx_max: i64) -> c_int;
    pub fn lq_attention(ctx: *mut LqCtx, q_dev: *const f32, k_cache_dev: *const f32, v_cache_dev: *const f32, batch: i64, n_heads: i64, n_kv_heads: i64, len: i64, pos0: i64, pos0_dev: *const i32, ctx_max: i64, head_dim: i64, out_dev: *mut f32, xq_dev: *mut i8, xd_dev: *mut u16) -> c_int;
    pub fn lq_silu_mul(ctx: *mut LqCtx, gu_dev: *const f32, m: i64, inter: i64, h_dev: *mut f32, xq_dev: *mut i8, xd_dev: *mut u16) -> c_int;
    pub fn lq_add(ctx: *mut LqCtx, a_dev: *const f32, b_dev: *const f32, n: i64, out_dev: *mut f32) -> c_int;
    pub fn lq_embedding(ctx: *mut LqCtx, table_dev: *const u16, vocab: i64, hidden: i64, ids_dev: *const i32, n: i64, out_dev: *mut f32) -> c_int;
    pub fn lq_argmax(ctx: *mut LqCtx, x_dev: *const f32, rows: i64, n: i64, out_dev: *mut i32) -> c_int;
    pub fn lq_sample(ctx: *mut LqCtx, logits_dev: *const f32, rows: i64, vocab: i64, ld: i64, generated_dev: *const i32, gen_ld: i64, n_generated: i64, cfg: *const LqSampling, out_dev: *mut i32) -> c_int;
    pub fn lq_fill_bf16(ctx: *mut LqCtx, seed: u64, tensor_id: u64, offset: i64, count: i64, std_dev: f64, out_dev: *mut u16) -> c_int;
    pub fn lq_comm_unique_id(ctx: *mut LqCtx, id_out: *mut u8) -> c_int;
    pub fn lq_comm_init(ctx: *mut LqCtx, id: *const u8, rank: c_int, world: c_int, out: *mut *mut LqComm) -> c_int;
    pub fn lq_comm_destroy(comm: *mut LqComm) -> c_int;
    pub fn lq_comm_rank(comm: *mut LqComm, rank: *mut c_int, world: *mut c_int) -> c_int;
    pub fn lq_comm_allreduce_f32(comm: *mut LqComm, buf_dev: *mut f32, count: i64) -> c_int;
    pub fn lq_q8_0_matmul_allreduce(ctx: *mut LqCtx, comm: *mut LqComm, w: *const LqQ8Tensor, xq_dev: *const i8, xd_dev: *const u16, m: i64, y_dev: *mut f32, residual_dev: *const f32) -> c_int;
    pub fn lq_moe_forward(ctx: *mut LqCtx, router: *const LqQ8Tensor, experts: *const LqMoeExperts, xq_dev: *const i8, xd_dev: *const u16, rows: i64, top_k: i64, norm_topk: c_int, out_dev: *mut f32, residual_dev: *const f32, ids_out_dev: *mut i32, weights_out_dev: *mut f32) -> c_int;
    pub fn lq_moe_forward_ep(ctx: *mut LqCtx, comm: *mut LqComm, router: *const LqQ8Tensor, local: *const LqMoeExperts, first_expert: i64, xq_dev: *const i8, xd_dev: *const u16, rows: i64, top_k: i64, norm_topk: c_int, out_dev: *mut f32, residual_dev: *const f32) -> c_int;
    pub fn lq_qwen3_create(ctx: *mut LqCtx, cfg: *const LqQwen3Config, seed: u64, max_batch: i64, ctx_max: i64, out: *mut *mut LqModel) -> c_int;
    pub fn lq_qwen3_create_tp(ctx: *mut LqCtx, cfg: *const LqQwen3Config, seed: u64, max_batch: i64, ctx_max: i64, comm: *mut LqComm, out: *mut *mut LqModel) -> c_int;
    pub fn lq_qwen3_destroy(model: *mut LqModel) -> c_int;
    pub fn lq_qwen3_reset(model: *mut LqModel) -> c_int;
    pub fn lq_qwen3_prefill(model: *mut LqModel, ids_host: *const i32, batch: i64, len: i64, next_host: *mut i32, logits_host: *mut f32) -> c_int;
    pub fn lq_qwen3_decode_step(model: *mut LqModel, ids_host: *const i32, next_host: *mut i32, logits_host: *mut f32) -> c_int;
    pub fn lq_qwen3_decode_device(model: *mut LqModel, n_steps: i64) -> c_int;
    pub fn lq_qwen3_set_batch(model: *mut LqModel, batch: i64) -> c_int;
    pub fn lq_qwen3_set_sampling(model: *mut LqModel, cfg: *const LqSampling) -> c_int;
    pub fn lq_qwen3_token_buffer(model: *mut LqModel, tokens_dev: *mut *mut i32) -> c_int;
    pub fn lq_qwen3_position(model: *mut LqModel, pos: *mut i64) -> c_int;
    pub fn lq_qwen3_linear(model: *mut LqModel, layer: i64, kind: c_int, out: *mut LqQ8Tensor) -> c_int;
    pub fn lq_qwen3_weight_bytes(model: *mut LqModel, bytes: *mut i64) -> c_int;
    pub fn lq_qwen3_tensor(model: *mut LqModel, layer: i64, kind: c_int, dev_out: *mut *mut u16, count: *mut i64) -> c_int;
    pub fn lq_qwen3_expert(model: *mut LqModel, layer: i64, expert: i64, kind: c_int, out: *mut LqQ8Tensor) -> c_int;
    pub fn lq_qwen3_graph_kernels(model: *mut LqModel, n: *mut i64) -> c_int;
}
