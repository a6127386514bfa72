//! Q8_0 linear path for lluda-inference on B200 (liblq8 through lluda-cuda-sys).
//!
//! This file is source for the lluda-inference crate itself (it uses `crate::tensor`,
//! `crate::error` and `crate::bf16`): add it as `src/q8.rs`, declare `#[cfg(feature = "cuda")]
//! pub mod q8;` in `src/lib.rs`, and add the dependency and feature of Cargo.toml.fragment.
//! It is not compiled in this repository (no Rust toolchain on its machines).
//!
//! What it adds, at the switch point the reference already has (`Linear::forward`,
//! attention.rs:101-136, which calls `Tensor::matmul`, tensor.rs:804-817):
//! - `QTensor`: a weight packed into Q8_0 blocks once (GGML's rule, bit-exact with the
//!   device quantizer), kept on the host and uploaded once to the device;
//! - `Tensor::quantize_q8_0()`;
//! - `LinearWeight::{Dense, Q8_0}` and a `Linear` whose `forward` keeps the reference's
//!   contract (host tensor `[..., in]` in, host F32 tensor `[..., out]` out, `Result` errors)
//!   and routes Q8_0 weights to `lq_q8_0_linear` on the device. Dense weights keep the
//!   reference's `matmul` path unchanged.
//! - one process-wide device context behind a `Mutex` (as `gpu::get_context`, gpu/mod.rs:129,
//!   but an initialisation failure is an error instead of a panic).
//! GPU failures map to `LludaError::Msg` (error.rs:92) and there is no CPU fallback for a Q8_0
//! weight, following GPU_DESIGN_PRINCIPLES.md:3-21.
use std::os::raw::c_void;
use std::sync::{Mutex, OnceLock};

use lluda_cuda_sys as lq;

use crate::bf16::BF16;
use crate::error::{LludaError, Result};
use crate::tensor::{DType, Tensor};

fn gpu_err(e: lq::Error) -> LludaError {
    LludaError::Msg(e.to_string())
}

/// The device context every Q8_0 Linear uses (device 0, or LLUDA_CUDA_DEVICE).
fn context() -> Result<&'static Mutex<lq::Context>> {
    static CTX: OnceLock<std::result::Result<Mutex<lq::Context>, String>> = OnceLock::new();
    let slot = CTX.get_or_init(|| {
        let dev = std::env::var("LLUDA_CUDA_DEVICE").ok().and_then(|s| s.parse().ok()).unwrap_or(0);
        lq::Context::new(dev).map(Mutex::new).map_err(|e| e.to_string())
    });
    slot.as_ref().map_err(|m| LludaError::Msg(format!("CUDA context: {m}")))
}

/// A weight `[out_features, in_features]` in Q8_0: 32-element int8 blocks along the input
/// dimension, each with an fp16 scale (GGML's Q8_0), stored as two arrays (values, scales).
#[derive(Debug, Clone)]
pub struct QTensor {
    host: lq::Q8Host,
}

impl QTensor {
    /// Shape `[out_features, in_features]`.
    pub fn shape(&self) -> [usize; 2] {
        [self.host.n, self.host.k]
    }

    /// The int8 values `[n][k]` and fp16 scale bits `[n][k/32]`.
    pub fn blocks(&self) -> (&[i8], &[u16]) {
        (&self.host.qs, &self.host.d)
    }

    /// GGML's 34-byte blocks {fp16 d; int8 qs[32]}, row-major (the on-disk Q8_0 layout).
    pub fn to_ggml_blocks(&self) -> Vec<u8> {
        let nb = self.host.k / 32;
        let mut out = Vec::with_capacity(self.host.n * nb * 34);
        for r in 0..self.host.n {
            for b in 0..nb {
                out.extend_from_slice(&self.host.d[r * nb + b].to_le_bytes());
                let q = &self.host.qs[r * self.host.k + b * 32..r * self.host.k + b * 32 + 32];
                out.extend(q.iter().map(|&v| v as u8));
            }
        }
        out
    }
}

impl Tensor {
    /// Q8_0 packing of a 2-D F32 or BF16 tensor along its last dimension (a multiple of 32).
    /// BF16 values are widened exactly; the result is bit-identical to the device quantizer.
    pub fn quantize_q8_0(&self) -> Result<QTensor> {
        if self.ndim() != 2 || self.shape()[1] % 32 != 0 {
            return Err(LludaError::ShapeMismatch { expected: vec![0, 32], got: self.shape().to_vec() });
        }
        let (rows, k) = (self.shape()[0], self.shape()[1]);
        let host = match self.dtype() {
            DType::F32 => lq::quantize_q8_0_host(lq::HostRows::F32(&self.to_vec_f32()), rows, k),
            DType::BF16 => {
                let bits: Vec<u16> = self.to_vec_bf16().into_iter().map(BF16::to_bits).collect();
                lq::quantize_q8_0_host(lq::HostRows::BF16(&bits), rows, k)
            }
        }
        .map_err(gpu_err)?;
        Ok(QTensor { host })
    }
}

/// The weight of a Linear: the reference's dense tensor, or Q8_0 blocks resident on the device
/// (uploaded once, at construction).
pub enum LinearWeight {
    Dense(Tensor),
    Q8_0 { q: QTensor, dev: lq::Q8Device },
}

/// `attention::Linear` with a Q8_0 variant: replaces the struct of attention.rs:32-71 (same
/// constructor and `forward` contract).
pub struct Linear {
    pub(crate) weight: LinearWeight,
}

impl Linear {
    /// Dense weight `[out_features, in_features]`, as `attention::Linear::new`.
    pub fn new(weight: Tensor) -> Result<Self> {
        if weight.ndim() != 2 {
            return Err(LludaError::ShapeMismatch { expected: vec![0, 0], got: weight.shape().to_vec() });
        }
        Ok(Linear { weight: LinearWeight::Dense(weight) })
    }

    /// Q8_0 weight, uploaded to the device once.
    pub fn new_q8_0(q: QTensor) -> Result<Self> {
        // the context is process-wide and never dropped, so it outlives every device weight
        let ctx = context()?;
        let ctx = ctx.lock().map_err(|_| LludaError::Msg("CUDA context poisoned".into()))?;
        let dev = lq::Q8Device::upload(&ctx, &q.host).map_err(gpu_err)?;
        Ok(Linear { weight: LinearWeight::Q8_0 { q, dev } })
    }

    /// Packs a dense weight to Q8_0 and uploads it (the loader's path for the linears).
    pub fn from_dense_q8_0(weight: &Tensor) -> Result<Self> {
        Self::new_q8_0(weight.quantize_q8_0()?)
    }

    fn shape(&self) -> [usize; 2] {
        match &self.weight {
            LinearWeight::Dense(w) => [w.shape()[0], w.shape()[1]],
            LinearWeight::Q8_0 { q, .. } => q.shape(),
        }
    }

    /// `x @ weight.T` for x `[..., in_features]` -> `[..., out_features]` F32.
    pub fn forward(&self, x: &Tensor) -> Result<Tensor> {
        let [out_features, in_features] = self.shape();
        let in_shape = x.shape();
        if in_shape[in_shape.len() - 1] != in_features {
            return Err(LludaError::ShapeMismatch { expected: vec![in_features], got: vec![in_shape[in_shape.len() - 1]] });
        }
        let m: usize = in_shape[..in_shape.len() - 1].iter().product();
        let mut out_shape = in_shape[..in_shape.len() - 1].to_vec();
        out_shape.push(out_features);
        match &self.weight {
            LinearWeight::Dense(w) => {
                // the reference's path (attention.rs:101-136)
                let y = x.reshape(&[m, in_features])?.matmul(&w.transpose()?)?;
                y.reshape(&out_shape)
            }
            LinearWeight::Q8_0 { dev, .. } => {
                let ctx = context()?;
                let ctx = ctx.lock().map_err(|_| LludaError::Msg("CUDA context poisoned".into()))?;
                // the activations go up as they are (F32, or BF16 bits) and are quantized on the
                // device, fused with the matmul's input side
                let mut y_dev = ctx.alloc::<f32>(m * out_features).map_err(gpu_err)?;
                match x.dtype() {
                    DType::F32 => {
                        let xd = ctx.upload(&x.to_vec_f32()).map_err(gpu_err)?;
                        lq::linear(&ctx, dev, xd.as_ptr() as *const c_void, lq::ffi::LQ_DTYPE_F32, m, y_dev.as_mut_ptr())
                            .map_err(gpu_err)?;
                    }
                    DType::BF16 => {
                        let bits: Vec<u16> = x.to_vec_bf16().into_iter().map(BF16::to_bits).collect();
                        let xd = ctx.upload(&bits).map_err(gpu_err)?;
                        lq::linear(&ctx, dev, xd.as_ptr() as *const c_void, lq::ffi::LQ_DTYPE_BF16, m, y_dev.as_mut_ptr())
                            .map_err(gpu_err)?;
                    }
                }
                let y = y_dev.download().map_err(gpu_err)?;
                Tensor::new(y, out_shape)
            }
        }
    }
}
