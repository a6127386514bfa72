//! Safe wrappers over liblq8 (see `ffi` for the raw C ABI): a device context, owned device
//! buffers, Q8_0 tensors uploaded once, the host Q8_0 quantizer and the Q8_0 Linear.
//!
//! Errors carry the library's status code and message; nothing here falls back to the CPU.
//! A `Context` is used by one thread at a time (wrap it in a `Mutex` to share it, as
//! lluda-inference does with its GPU context).
pub mod ffi;

use std::ffi::CStr;
use std::fmt;
use std::os::raw::c_void;
use std::ptr;

/// A failed liblq8 call: its status (`ffi::LQ_ERR_*`) and `lq_last_error` message.
#[derive(Debug, Clone)]
pub struct Error {
    pub code: i32,
    pub message: String,
}

impl fmt::Display for Error {
    fn fmt(&self, f: &mut fmt::Formatter<'_>) -> fmt::Result {
        write!(f, "liblq8 status {}: {}", self.code, self.message)
    }
}

impl std::error::Error for Error {}

pub type Result<T> = std::result::Result<T, Error>;

fn last_error(ctx: *const ffi::LqCtx) -> String {
    unsafe {
        let p = ffi::lq_last_error(ctx);
        if p.is_null() {
            String::new()
        } else {
            CStr::from_ptr(p).to_string_lossy().into_owned()
        }
    }
}

fn check(ctx: *const ffi::LqCtx, rc: i32) -> Result<()> {
    if rc == ffi::LQ_OK {
        Ok(())
    } else {
        Err(Error { code: rc, message: last_error(ctx) })
    }
}

/// lq_ctx on one CUDA device; destroyed on drop.
pub struct Context {
    raw: *mut ffi::LqCtx,
}

// The context may move between threads; it is not shared without a lock.
unsafe impl Send for Context {}

impl Context {
    pub fn new(device: i32) -> Result<Self> {
        let mut raw = ptr::null_mut();
        check(ptr::null(), unsafe { ffi::lq_init(device, &mut raw) })?;
        Ok(Context { raw })
    }

    pub fn raw(&self) -> *mut ffi::LqCtx {
        self.raw
    }

    pub fn synchronize(&self) -> Result<()> {
        check(self.raw, unsafe { ffi::lq_synchronize(self.raw) })
    }

    /// Checks a status returned by a raw call on this context.
    pub fn check(&self, rc: i32) -> Result<()> {
        check(self.raw, rc)
    }

    pub fn alloc<T: Copy>(&self, len: usize) -> Result<DeviceBuffer<T>> {
        let mut p: *mut c_void = ptr::null_mut();
        self.check(unsafe { ffi::lq_malloc(self.raw, len * std::mem::size_of::<T>(), &mut p) })?;
        Ok(DeviceBuffer { ctx: self.raw, ptr: p as *mut T, len })
    }

    /// A device copy of `host` (synchronous with respect to the host slice).
    pub fn upload<T: Copy>(&self, host: &[T]) -> Result<DeviceBuffer<T>> {
        let buf = self.alloc::<T>(host.len())?;
        self.check(unsafe {
            ffi::lq_memcpy_h2d(self.raw, buf.ptr as *mut c_void, host.as_ptr() as *const c_void, std::mem::size_of_val(host))
        })?;
        self.synchronize()?;
        Ok(buf)
    }
}

impl Drop for Context {
    fn drop(&mut self) {
        unsafe {
            ffi::lq_destroy(self.raw);
        }
    }
}

/// Device memory allocated through a context; freed on drop. The context must outlive its
/// buffers (drop them first).
pub struct DeviceBuffer<T: Copy> {
    ctx: *mut ffi::LqCtx,
    ptr: *mut T,
    len: usize,
}

unsafe impl<T: Copy> Send for DeviceBuffer<T> {}

impl<T: Copy> DeviceBuffer<T> {
    pub fn as_ptr(&self) -> *const T {
        self.ptr
    }
    pub fn as_mut_ptr(&mut self) -> *mut T {
        self.ptr
    }
    pub fn len(&self) -> usize {
        self.len
    }
    pub fn is_empty(&self) -> bool {
        self.len == 0
    }
    /// Copies the buffer back to the host (waits for the context's stream).
    pub fn download(&self) -> Result<Vec<T>> {
        let mut v = Vec::<T>::with_capacity(self.len);
        check(self.ctx, unsafe {
            ffi::lq_memcpy_d2h(self.ctx, v.as_mut_ptr() as *mut c_void, self.ptr as *const c_void,
                               self.len * std::mem::size_of::<T>())
        })?;
        check(self.ctx, unsafe { ffi::lq_synchronize(self.ctx) })?;
        unsafe { v.set_len(self.len) };
        Ok(v)
    }
}

impl<T: Copy> Drop for DeviceBuffer<T> {
    fn drop(&mut self) {
        unsafe {
            ffi::lq_free(self.ctx, self.ptr as *mut c_void);
        }
    }
}

/// Q8_0 blocks on the host in the library's SoA layout: int8 values [n][k] and fp16 scale
/// bits [n][k/32] (GGML's 34-byte blocks split in two arrays).
#[derive(Clone, Debug)]
pub struct Q8Host {
    pub n: usize,
    pub k: usize,
    pub qs: Vec<i8>,
    pub d: Vec<u16>,
}

/// Host input of the quantizer.
pub enum HostRows<'a> {
    F32(&'a [f32]),
    /// bf16 bit patterns
    BF16(&'a [u16]),
}

/// GGML's Q8_0 rule on the host (lq_q8_0_quantize_host): the same bits as the device
/// quantizer. `rows` rows of `k` values, k a multiple of 32.
pub fn quantize_q8_0_host(src: HostRows<'_>, rows: usize, k: usize) -> Result<Q8Host> {
    let (ptr, len, dtype) = match src {
        HostRows::F32(s) => (s.as_ptr() as *const c_void, s.len(), ffi::LQ_DTYPE_F32),
        HostRows::BF16(s) => (s.as_ptr() as *const c_void, s.len(), ffi::LQ_DTYPE_BF16),
    };
    if len != rows * k {
        return Err(Error { code: ffi::LQ_ERR_INVALID_ARG, message: format!("{len} values for {rows} x {k}") });
    }
    let mut out = Q8Host { n: rows, k, qs: vec![0; rows * k], d: vec![0; rows * (k / 32)] };
    check(ptr::null(), unsafe {
        ffi::lq_q8_0_quantize_host(ptr, dtype, rows as i64, k as i64, out.qs.as_mut_ptr(), out.d.as_mut_ptr())
    })?;
    Ok(out)
}

/// A Q8_0 weight uploaded once (rows = out_features), usable by `linear`.
pub struct Q8Device {
    qs: DeviceBuffer<i8>,
    d: DeviceBuffer<u16>,
    pub n: usize,
    pub k: usize,
}

impl Q8Device {
    pub fn upload(ctx: &Context, w: &Q8Host) -> Result<Self> {
        Ok(Q8Device { qs: ctx.upload(&w.qs)?, d: ctx.upload(&w.d)?, n: w.n, k: w.k })
    }

    pub fn raw(&self) -> ffi::LqQ8Tensor {
        ffi::LqQ8Tensor { n: self.n as i64, k: self.k as i64, qs: self.qs.ptr, d: self.d.ptr }
    }
}

/// Linear::forward with a Q8_0 weight on device rows: x [m][k] (f32 or bf16 bits on the
/// device) -> y [m][n] f32 on the device; asynchronous on the context's stream.
pub fn linear(ctx: &Context, w: &Q8Device, x_dev: *const c_void, x_dtype: ffi::LqDtype, m: usize,
              y_dev: *mut f32) -> Result<()> {
    let t = w.raw();
    ctx.check(unsafe { ffi::lq_q8_0_linear(ctx.raw, &t, x_dev, x_dtype, m as i64, y_dev) })
}
