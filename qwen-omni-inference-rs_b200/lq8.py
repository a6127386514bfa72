"""Python binding of liblq8.so (the C ABI in include/lq8.h) over ctypes.

It mirrors the reference crate's surface for the Q8_0 path -- `QTensor` (the planned Q8_0
tensor), `Linear::new / Linear::forward` (attention.rs:32-136), the small layer ops, and
`Qwen3ForCausalLM` with greedy `generate` (model.rs:273-372, generate.rs:611-661) -- so tests
read like the reference's own. Device buffers are torch CUDA tensors (plumbing only); every
computation runs in liblq8.so. There is no fallback: if the library or a GPU is missing the
calls raise.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblq8.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "lq8.h")

LQ_OK = 0
STATUS = {0: "LQ_OK", -1: "LQ_ERR_INVALID_ARG", -2: "LQ_ERR_CUDA", -3: "LQ_ERR_OOM",
          -4: "LQ_ERR_UNSUPPORTED", -5: "LQ_ERR_INJECTED", -6: "LQ_ERR_STATE", -7: "LQ_ERR_NCCL",
          -8: "LQ_ERR_TIMEOUT"}
DTYPE_F32, DTYPE_BF16, DTYPE_F16, DTYPE_I8, DTYPE_I32 = 0, 1, 2, 3, 4
KIND = {"q": 0, "k": 1, "v": 2, "o": 3, "gate": 4, "up": 5, "down": 6, "lm_head": 7, "qkv": 8,
        "gate_up": 9}


class LQ8Error(RuntimeError):
    """A non-zero status from liblq8 (LludaError::Msg in the reference)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS.get(code, code)}: {msg}")
        self.code = code


class Q8Tensor(C.Structure):
    _fields_ = [("n", C.c_int64), ("k", C.c_int64), ("qs", C.c_void_p), ("d", C.c_void_p)]


class Qwen3Config(C.Structure):
    _fields_ = [
        ("hidden", C.c_int64), ("layers", C.c_int64), ("n_heads", C.c_int64),
        ("n_kv_heads", C.c_int64), ("head_dim", C.c_int64), ("inter", C.c_int64),
        ("vocab", C.c_int64), ("max_pos", C.c_int64), ("tied", C.c_int32),
        ("eps", C.c_float), ("theta", C.c_double), ("init_std", C.c_float),
        ("norm_std", C.c_float), ("n_experts", C.c_int64), ("top_k", C.c_int64),
        ("moe_inter", C.c_int64), ("norm_topk", C.c_int32), ("pad_", C.c_int32),
    ]


class Sampling(C.Structure):
    """lq_sampling: the reference's GenerationConfig knobs (generate.rs:38-64)."""
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int32), ("top_p", C.c_float),
                ("repetition_penalty", C.c_float)]


def sampling(temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0, repetition_penalty: float = 1.0):
    return Sampling(temperature, top_k, top_p, repetition_penalty)


class MoeExperts(C.Structure):
    """lq_moe_experts: stacked expert weights (gate/up [E*2I][H], down [E*H][I])."""
    _fields_ = [("n_experts", C.c_int64), ("inter", C.c_int64), ("hidden", C.c_int64),
                ("gate_up", Q8Tensor), ("down", Q8Tensor)]


# Qwen3 architectures of the benchmark configurations
QWEN3_0_6B = dict(hidden=1024, layers=28, n_heads=16, n_kv_heads=8, head_dim=128, inter=3072,
                  vocab=151936, max_pos=40960, tied=1, eps=1e-6, theta=1e6, init_std=0.02, norm_std=0.0)
QWEN3_8B = dict(hidden=4096, layers=36, n_heads=32, n_kv_heads=8, head_dim=128, inter=12288,
                vocab=151936, max_pos=40960, tied=0, eps=1e-6, theta=1e6, init_std=0.02, norm_std=0.0)
QWEN3_32B = dict(hidden=5120, layers=64, n_heads=64, n_kv_heads=8, head_dim=128, inter=25600,
                 vocab=151936, max_pos=40960, tied=0, eps=1e-6, theta=1e6, init_std=0.02, norm_std=0.0)
QWEN3_30B_A3B = dict(hidden=2048, layers=48, n_heads=32, n_kv_heads=4, head_dim=128, inter=0,
                     vocab=151936, max_pos=40960, tied=0, eps=1e-6, theta=1e6, init_std=0.02, norm_std=0.0,
                     n_experts=128, top_k=8, moe_inter=768, norm_topk=1)


def make_config(**kw) -> Qwen3Config:
    c = Qwen3Config()
    d = dict(QWEN3_0_6B)
    d.update(kw)
    for k, v in d.items():
        setattr(c, k, v)
    return c


_P = C.c_void_p
_I64 = C.c_int64
_lib = None

# name -> (restype, argtypes); the single source of the binding, checked against lq8.h
ABI_VERSION = 3   # LQ8_ABI_VERSION of the struct layouts below

SIGNATURES = {
    "lq_abi_version": (C.c_int, []),
    "lq_init": (C.c_int, [C.c_int, C.POINTER(_P)]),
    "lq_destroy": (C.c_int, [_P]),
    "lq_last_error": (C.c_char_p, [_P]),
    "lq_set_stream": (C.c_int, [_P, _P]),
    "lq_get_stream": (_P, [_P]),
    "lq_synchronize": (C.c_int, [_P]),
    "lq_device_info": (C.c_int, [_P, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int),
                                 C.POINTER(C.c_size_t)]),
    "lq_malloc": (C.c_int, [_P, C.c_size_t, C.POINTER(_P)]),
    "lq_free": (C.c_int, [_P, _P]),
    "lq_memcpy_h2d": (C.c_int, [_P, _P, _P, C.c_size_t]),
    "lq_memcpy_d2h": (C.c_int, [_P, _P, _P, C.c_size_t]),
    "lq_memset": (C.c_int, [_P, _P, C.c_int, C.c_size_t]),
    "lq_q8_0_quantize": (C.c_int, [_P, _P, C.c_int, _I64, _I64, _P, _P]),
    "lq_q8_0_pack_blocks": (C.c_int, [_P, _P, _P, _I64, _I64, _P]),
    "lq_q8_0_unpack_blocks": (C.c_int, [_P, _P, _I64, _I64, _P, _P]),
    "lq_q8_0_matmul": (C.c_int, [_P, C.POINTER(Q8Tensor), _P, _P, _I64, _P, _P, _I64]),
    "lq_q8_0_matmul_prefill": (C.c_int, [_P, C.POINTER(Q8Tensor), _P, _P, _I64, _P, _P, _I64]),
    "lq_q8_0_linear": (C.c_int, [_P, C.POINTER(Q8Tensor), _P, C.c_int, _I64, _P]),
    "lq_q8_0_linear_noalloc": (C.c_int, [_P, C.POINTER(Q8Tensor), _P, C.c_int, _I64, _P]),
    "lq_q8_0_quantize_host": (C.c_int, [_P, C.c_int, _I64, _I64, _P, _P]),
    "lq_rmsnorm": (C.c_int, [_P, _P, C.c_int, _I64, _I64, _P, C.c_float, _P, _P, _P]),
    "lq_rope_tables": (C.c_int, [_P, _I64, _I64, C.c_double, _P, _P]),
    "lq_qk_norm_rope_kv": (C.c_int, [_P, _P, _I64, _I64, _I64, _I64, _I64, _P, _P, C.c_float, _P, _P,
                                     _I64, _P, _P, _P, _P, _I64]),
    "lq_attention": (C.c_int, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _I64, _I64, _P, _P, _P]),
    "lq_silu_mul": (C.c_int, [_P, _P, _I64, _I64, _P, _P, _P]),
    "lq_add": (C.c_int, [_P, _P, _P, _I64, _P]),
    "lq_embedding": (C.c_int, [_P, _P, _I64, _I64, _P, _I64, _P]),
    "lq_argmax": (C.c_int, [_P, _P, _I64, _I64, _P]),
    "lq_fill_bf16": (C.c_int, [_P, C.c_uint64, C.c_uint64, _I64, _I64, C.c_double, _P]),
    "lq_qwen3_create": (C.c_int, [_P, C.POINTER(Qwen3Config), C.c_uint64, _I64, _I64, C.POINTER(_P)]),
    "lq_qwen3_create_tp": (C.c_int, [_P, C.POINTER(Qwen3Config), C.c_uint64, _I64, _I64, _P, C.POINTER(_P)]),
    "lq_comm_unique_id": (C.c_int, [_P, _P]),
    "lq_comm_init": (C.c_int, [_P, _P, C.c_int, C.c_int, C.POINTER(_P)]),
    "lq_comm_destroy": (C.c_int, [_P]),
    "lq_comm_rank": (C.c_int, [_P, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "lq_comm_allreduce_f32": (C.c_int, [_P, _P, _I64]),
    "lq_q8_0_matmul_allreduce": (C.c_int, [_P, _P, C.POINTER(Q8Tensor), _P, _P, _I64, _P, _P]),
    "lq_qwen3_destroy": (C.c_int, [_P]),
    "lq_qwen3_reset": (C.c_int, [_P]),
    "lq_qwen3_prefill": (C.c_int, [_P, _P, _I64, _I64, _P, _P]),
    "lq_qwen3_decode_step": (C.c_int, [_P, _P, _P, _P]),
    "lq_qwen3_decode_device": (C.c_int, [_P, _I64]),
    "lq_qwen3_set_batch": (C.c_int, [_P, _I64]),
    "lq_qwen3_token_buffer": (C.c_int, [_P, C.POINTER(_P)]),
    "lq_qwen3_position": (C.c_int, [_P, C.POINTER(_I64)]),
    "lq_qwen3_linear": (C.c_int, [_P, _I64, C.c_int, C.POINTER(Q8Tensor)]),
    "lq_qwen3_weight_bytes": (C.c_int, [_P, C.POINTER(_I64)]),
    "lq_qwen3_graph_kernels": (C.c_int, [_P, C.POINTER(_I64)]),
    "lq_qwen3_set_sampling": (C.c_int, [_P, C.POINTER(Sampling)]),
    "lq_qwen3_tensor": (C.c_int, [_P, _I64, C.c_int, C.POINTER(_P), C.POINTER(_I64)]),
    "lq_sample": (C.c_int, [_P, _P, _I64, _I64, _I64, _P, _I64, _I64, C.POINTER(Sampling), _P]),
    "lq_qwen3_expert": (C.c_int, [_P, _I64, _I64, C.c_int, C.POINTER(Q8Tensor)]),
    "lq_moe_forward": (C.c_int, [_P, C.POINTER(Q8Tensor), C.POINTER(MoeExperts), _P, _P, _I64, _I64, C.c_int,
                                 _P, _P, _P, _P]),
    "lq_moe_forward_ep": (C.c_int, [_P, _P, C.POINTER(Q8Tensor), C.POINTER(MoeExperts), _I64, _P, _P, _I64, _I64,
                                    C.c_int, _P, _P]),
}


def load():
    """Load liblq8.so (built in-tree by build.py). Raises if it is missing: no fallback."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"liblq8.so not built ({LIB_PATH}); run qwen-omni-inference-rs_b200/build.py")
        lib = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(lib, name)
            f.restype = res
            f.argtypes = args
        if lib.lq_abi_version() != ABI_VERSION:
            raise OSError(f"liblq8.so ABI {lib.lq_abi_version()} != binding ABI {ABI_VERSION}; rebuild")
        _lib = lib
    return _lib


def _ptr(t) -> int | None:
    if t is None:
        return None
    return t.data_ptr()


class Context:
    """lq_ctx on one CUDA device (gpu::get_context in the reference, but fallible)."""

    def __init__(self, device: int = 0, use_torch_stream: bool = True):
        lib = load()
        h = _P()
        rc = lib.lq_init(device, C.byref(h))
        if rc != LQ_OK:
            raise LQ8Error(rc, lib.lq_last_error(None).decode())
        self.h = h
        self.lib = lib
        self.device = device
        if use_torch_stream:
            # one stream for torch and the library keeps their work ordered; torch's legacy
            # default stream cannot be captured into a CUDA graph, so a dedicated stream is
            # made current for this thread
            import torch
            cur = torch.cuda.current_stream(device)
            if cur.cuda_stream == 0:
                cur = torch.cuda.Stream(device=device)
                torch.cuda.set_stream(cur)
            self._torch_stream = cur
            self.check(lib.lq_set_stream(h, cur.cuda_stream))

    def check(self, rc: int) -> None:
        if rc != LQ_OK:
            raise LQ8Error(rc, self.lib.lq_last_error(self.h).decode())

    def call(self, name: str, *args) -> None:
        self.check(getattr(self.lib, name)(self.h, *args))

    @property
    def stream(self) -> int:
        return self.lib.lq_get_stream(self.h) or 0

    def synchronize(self) -> None:
        self.check(self.lib.lq_synchronize(self.h))

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.lq_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass



@dataclass
class QTensor:
    """Q8_0 tensor on the device: qs int8 [n, k], d fp16 bits [n, k/32] (stored as int16)."""
    qs: "torch.Tensor"
    d: "torch.Tensor"

    @property
    def n(self) -> int:
        return self.qs.shape[0]

    @property
    def k(self) -> int:
        return self.qs.shape[1]

    def struct(self) -> Q8Tensor:
        return Q8Tensor(self.n, self.k, self.qs.data_ptr(), self.d.data_ptr())

    @staticmethod
    def quantize(ctx: Context, w) -> "QTensor":
        """Tensor::quantize_q8_0 of a 2-D f32 or bf16 CUDA tensor (bf16 may be given as int16 bits)."""
        import torch
        assert w.dim() == 2 and w.is_cuda and w.is_contiguous()
        n, k = w.shape
        qs = torch.empty((n, k), dtype=torch.int8, device=w.device)
        d = torch.empty((n, k // 32), dtype=torch.int16, device=w.device)
        dt = DTYPE_F32 if w.dtype == torch.float32 else DTYPE_BF16
        ctx.call("lq_q8_0_quantize", w.data_ptr(), dt, n, k, qs.data_ptr(), d.data_ptr())
        return QTensor(qs, d)

    @staticmethod
    def from_struct(t: Q8Tensor) -> "QTensor":
        """Copy a Q8_0 tensor owned elsewhere (e.g. a model's fused weight) into torch tensors."""
        qs = wrap_device(t.qs, (t.n, t.k), "|i1").clone()
        d = wrap_device(t.d, (t.n, t.k // 32), "<i2").clone()
        return QTensor(qs, d)


def wrap_device(ptr: int, shape, typestr: str):
    """A torch CUDA tensor viewing raw device memory (no ownership, no copy)."""
    import torch

    class _Arr:
        __cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                    "version": 3, "strides": None}
    return torch.as_tensor(_Arr(), device="cuda")


class Linear:
    """Linear layer with a Q8_0 weight [out, in] (attention.rs:32-136)."""

    def __init__(self, ctx: Context, weight: QTensor):
        if weight.qs.dim() != 2:
            raise ValueError("Linear::new: weight must be 2-D")
        self.ctx = ctx
        self.weight = weight

    def forward(self, x):
        """x [..., in] f32 or bf16 (torch.bfloat16) CUDA tensor -> [..., out] f32."""
        import torch
        if x.shape[-1] != self.weight.k:
            raise ValueError(f"ShapeMismatch: expected [{self.weight.k}], got [{x.shape[-1]}]")
        x2 = x.reshape(-1, self.weight.k).contiguous()
        m = x2.shape[0]
        y = torch.empty((m, self.weight.n), dtype=torch.float32, device=x.device)
        dt = DTYPE_F32 if x.dtype == torch.float32 else DTYPE_BF16
        w = self.weight.struct()
        self.ctx.call("lq_q8_0_linear", C.byref(w), x2.data_ptr(), dt, m, y.data_ptr())
        return y.reshape(*x.shape[:-1], self.weight.n)


def sample(ctx: Context, logits, generated=None, n_generated: int = 0, out=None, **cfg):
    """lq_sample: the reference's token choice (sample_with_config after the repetition
    penalty) for rows of device logits [rows][V] (torch CUDA tensor, f32); generated: device
    int32 [rows][gen_ld] of which the first n_generated per row count. Returns int32 [rows]."""
    import torch
    rows, V = logits.shape
    if out is None:
        out = torch.empty(rows, dtype=torch.int32, device=logits.device)
    sc = sampling(**cfg)
    gen_ld = generated.shape[1] if generated is not None else 0
    ctx.call("lq_sample", logits.data_ptr(), rows, V, logits.stride(0), _ptr(generated), gen_ld, n_generated,
             C.byref(sc), out.data_ptr())
    return out


def matmul_q8(ctx: Context, w: QTensor, xq, xd, residual=None, out=None):
    """Q8_0 x Q8_0 matmul with pre-quantized activations (optionally y = residual + x.W^T)."""
    import torch
    m = xq.shape[0]
    y = out if out is not None else torch.empty((m, w.n), dtype=torch.float32, device=xq.device)
    ws = w.struct()
    ctx.call("lq_q8_0_matmul", C.byref(ws), xq.data_ptr(), xd.data_ptr(), m, y.data_ptr(),
             _ptr(residual), y.shape[1])
    return y


COMM_ID_BYTES = 128


class Comm:
    """NCCL communicator of this rank (lq_comm_*). `from_process_group` makes rank 0's NCCL id
    and hands it to the other ranks over an initialised torch.distributed process group."""

    def __init__(self, ctx: Context, uid: bytes, rank: int, world: int):
        self.ctx = ctx
        buf = (C.c_uint8 * COMM_ID_BYTES).from_buffer_copy(uid)
        h = _P()
        ctx.check(ctx.lib.lq_comm_init(ctx.h, buf, rank, world, C.byref(h)))
        self.h = h
        self.rank, self.world = rank, world

    @staticmethod
    def unique_id(ctx: Context) -> bytes:
        buf = (C.c_uint8 * COMM_ID_BYTES)()
        ctx.check(ctx.lib.lq_comm_unique_id(ctx.h, buf))
        return bytes(buf)

    @classmethod
    def from_process_group(cls, ctx: Context) -> "Comm":
        import torch.distributed as dist
        rank, world = dist.get_rank(), dist.get_world_size()
        obj = [cls.unique_id(ctx) if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        return cls(ctx, obj[0], rank, world)

    def allreduce_(self, t) -> None:
        """In-place sum over the ranks of a contiguous f32 CUDA tensor."""
        self.ctx.check(self.ctx.lib.lq_comm_allreduce_f32(self.h, _ptr(t), t.numel()))

    def close(self):
        if getattr(self, "h", None):
            self.ctx.lib.lq_comm_destroy(self.h)
            self.h = None


class Qwen3ForCausalLM:
    """Qwen3 model runner with seeded random-init Q8_0 weights (model.rs:273-372). With `comm`
    this rank's tensor-parallel shard (every rank makes the same calls in the same order)."""

    def __init__(self, ctx: Context, cfg: Qwen3Config, seed: int, max_batch: int = 1, ctx_max: int = 64,
                 comm: "Comm | None" = None):
        self.ctx = ctx
        self.cfg = cfg
        self.max_batch = max_batch
        self.ctx_max = ctx_max
        self.comm = comm
        h = _P()
        if comm is None:
            ctx.check(ctx.lib.lq_qwen3_create(ctx.h, C.byref(cfg), seed, max_batch, ctx_max, C.byref(h)))
        else:
            ctx.check(ctx.lib.lq_qwen3_create_tp(ctx.h, C.byref(cfg), seed, max_batch, ctx_max, comm.h, C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            self.ctx.lib.lq_qwen3_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc):
        self.ctx.check(rc)

    def clear_kv_cache(self):
        self._check(self.ctx.lib.lq_qwen3_reset(self.h))

    def prefill(self, ids: np.ndarray, want_logits: bool = False):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        if ids.ndim == 1:
            ids = ids[None, :]
        B, L = ids.shape
        nxt = np.empty(B, dtype=np.int32)
        lg = np.empty((B, self.cfg.vocab), dtype=np.float32) if want_logits else None
        self._check(self.ctx.lib.lq_qwen3_prefill(self.h, ids.ctypes.data, B, L, nxt.ctypes.data,
                                                  lg.ctypes.data if lg is not None else None))
        return (nxt, lg) if want_logits else nxt

    def set_sampling(self, **cfg):
        """Token choice for the following steps (temperature, top_k, top_p,
        repetition_penalty; defaults greedy), as the reference's sample_with_config."""
        sc = sampling(**cfg)
        self._check(self.ctx.lib.lq_qwen3_set_sampling(self.h, C.byref(sc)))

    def set_batch(self, B: int):
        self._check(self.ctx.lib.lq_qwen3_set_batch(self.h, B))

    def decode_step(self, ids: np.ndarray, want_logits: bool = False):
        ids = np.ascontiguousarray(ids, dtype=np.int32).reshape(-1)
        nxt = np.empty_like(ids)
        lg = np.empty((ids.size, self.cfg.vocab), dtype=np.float32) if want_logits else None
        self._check(self.ctx.lib.lq_qwen3_decode_step(self.h, ids.ctypes.data, nxt.ctypes.data,
                                                      lg.ctypes.data if lg is not None else None))
        return (nxt, lg) if want_logits else nxt

    def decode_device(self, n_steps: int):
        self._check(self.ctx.lib.lq_qwen3_decode_device(self.h, n_steps))

    def token_buffer_ptr(self) -> int:
        p = _P()
        self._check(self.ctx.lib.lq_qwen3_token_buffer(self.h, C.byref(p)))
        return p.value

    def position(self) -> int:
        p = _I64()
        self._check(self.ctx.lib.lq_qwen3_position(self.h, C.byref(p)))
        return p.value

    def linear(self, layer: int, kind: str) -> Q8Tensor:
        t = Q8Tensor()
        self._check(self.ctx.lib.lq_qwen3_linear(self.h, layer, KIND[kind], C.byref(t)))
        return t

    def expert(self, layer: int, expert: int, kind: int) -> Q8Tensor:
        """MoE weight view: kind 10 router, 11 gate, 12 up, 13 down of `expert`."""
        t = Q8Tensor()
        self._check(self.ctx.lib.lq_qwen3_expert(self.h, layer, expert, kind, C.byref(t)))
        return t

    def tensor(self, layer: int, kind: str):
        """Device (pointer, count) of a bf16 parameter: 'in_norm', 'post_norm', 'q_norm',
        'k_norm' of a layer; layer -1: 'final_norm', 'embed'."""
        kid = {"in_norm": 20, "post_norm": 21, "q_norm": 22, "k_norm": 23, "final_norm": 24, "embed": 25}[kind]
        p, n = _P(), _I64()
        self._check(self.ctx.lib.lq_qwen3_tensor(self.h, layer, kid, C.byref(p), C.byref(n)))
        return p.value, n.value

    def graph_kernels(self) -> int:
        n = _I64()
        self._check(self.ctx.lib.lq_qwen3_graph_kernels(self.h, C.byref(n)))
        return n.value

    def weight_bytes(self) -> int:
        b = _I64()
        self._check(self.ctx.lib.lq_qwen3_weight_bytes(self.h, C.byref(b)))
        return b.value

    def generate(self, prompt: np.ndarray, max_new_tokens: int) -> np.ndarray:
        """Greedy generate (generate.rs:611-661) for a [B, L] or [L] prompt; EOS is not checked."""
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        if prompt.ndim == 1:
            prompt = prompt[None, :]
        self.clear_kv_cache()
        self.set_batch(prompt.shape[0])
        out = np.empty((prompt.shape[0], max_new_tokens), dtype=np.int32)
        nxt = self.prefill(prompt)
        out[:, 0] = nxt
        for i in range(1, max_new_tokens):
            nxt = self.decode_step(nxt)
            out[:, i] = nxt
        return out
