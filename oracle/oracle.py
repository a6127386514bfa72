"""ctypes wrapper of the CPU oracle (oracle/liboracle_q8.so).

TEST INFRASTRUCTURE ONLY. This module is the checker: tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / reference arm may import it; the product library never does.
The C sources cite the reference file:line each function restates.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle_q8.so")
_lib = None

QK = 32
VOCAB_QWEN3 = 151936


def build() -> str:
    """Compile the oracle with its Makefile (gcc); returns the .so path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = C.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


class Qwen3Config(C.Structure):
    _fields_ = [
        ("hidden", C.c_int64), ("layers", C.c_int64), ("n_heads", C.c_int64),
        ("n_kv_heads", C.c_int64), ("head_dim", C.c_int64), ("inter", C.c_int64),
        ("vocab", C.c_int64), ("max_pos", C.c_int64), ("tied", C.c_int32),
        ("eps", C.c_float), ("theta", C.c_double), ("init_std", C.c_float),
        ("norm_std", C.c_float), ("n_experts", C.c_int64), ("top_k", C.c_int64),
        ("moe_inter", C.c_int64), ("norm_topk", C.c_int32), ("pad_", C.c_int32),
    ]


_P = C.c_void_p
_I64 = C.c_int64


def _declare(L):
    L.orc_f32_to_bf16.restype = C.c_uint16
    L.orc_f32_to_bf16.argtypes = [C.c_float]
    L.orc_bf16_to_f32.restype = C.c_float
    L.orc_bf16_to_f32.argtypes = [C.c_uint16]
    L.orc_f32_to_f16.restype = C.c_uint16
    L.orc_f32_to_f16.argtypes = [C.c_float]
    L.orc_f16_to_f32.restype = C.c_float
    L.orc_f16_to_f32.argtypes = [C.c_uint16]
    L.orc_f32_to_bf16_array.argtypes = [_P, _I64, _P]
    L.orc_bf16_to_f32_array.argtypes = [_P, _I64, _P]
    L.orc_splitmix64.restype = C.c_uint64
    L.orc_splitmix64.argtypes = [C.c_uint64]
    L.orc_gen_bf16.argtypes = [C.c_uint64, C.c_uint64, _I64, _I64, C.c_float, _P]
    L.orc_gen_tokens.argtypes = [C.c_uint64, C.c_uint64, _I64, _I64, _P]
    L.orc_gen_scale.restype = C.c_float
    L.orc_gen_scale.argtypes = [C.c_double]
    L.orc_q8_0_quantize_f32.argtypes = [_P, _I64, _I64, _P, _P]
    L.orc_q8_0_quantize_bf16.argtypes = [_P, _I64, _I64, _P, _P]
    L.orc_q8_0_pack_blocks.argtypes = [_P, _P, _I64, _I64, _P]
    L.orc_q8_0_unpack_blocks.argtypes = [_P, _I64, _I64, _P, _P]
    L.orc_q8_0_matmul.argtypes = [_P, _P, _I64, _P, _P, _I64, _I64, _P, _P]
    L.orc_q8_0_linear_f32.argtypes = [_P, _I64, _I64, _P, _P, _I64, _P]
    L.orc_q8_0_linear_bf16.argtypes = [_P, _I64, _I64, _P, _P, _I64, _P]
    L.orc_matmul_2d.argtypes = [_P, _I64, _I64, _P, _I64, _P]
    L.orc_rmsnorm_f32.argtypes = [_P, _I64, _I64, _P, C.c_float, _P]
    L.orc_rmsnorm_bf16.argtypes = [_P, _I64, _I64, _P, C.c_float, _P]
    L.orc_rope_tables.argtypes = [_I64, _I64, C.c_double, _P, _P]
    L.orc_rope_apply.argtypes = [_P, _I64, _I64, _I64, _I64, _P, _P]
    L.orc_silu.restype = C.c_float
    L.orc_silu.argtypes = [C.c_float]
    L.orc_argmax.restype = _I64
    L.orc_argmax.argtypes = [_P, _I64]
    L.orc_softmax.argtypes = [_P, _I64]
    L.orc_attend_row.argtypes = [_P, _P, _P, _I64, _I64, _I64, C.c_int, _I64, _P, _P]
    L.orc_qwen3_create.restype = _P
    L.orc_sample.argtypes = [_P, _I64, _P, _I64, C.c_float, _I64, C.c_float, C.c_float]
    L.orc_sample.restype = C.c_int32
    L.orc_sample_ex.argtypes = [_P, _I64, _P, _I64, C.c_float, _I64, C.c_float, C.c_float, C.c_int]
    L.orc_sample_ex.restype = C.c_int32
    L.orc_qwen3_generate_cfg.argtypes = [_P, _P, _I64, _I64, C.c_float, _I64, C.c_float, C.c_float, _P, _P]
    L.orc_qwen3_generate_cfg.restype = C.c_int
    L.orc_qwen3_create.argtypes = [C.POINTER(Qwen3Config), C.c_uint64, _I64, _I64]
    L.orc_qwen3_destroy.argtypes = [_P]
    L.orc_qwen3_clear.argtypes = [_P]
    L.orc_qwen3_forward.restype = C.c_int
    L.orc_qwen3_forward.argtypes = [_P, _P, _I64, _I64, _P]
    L.orc_qwen3_generate.restype = C.c_int
    L.orc_qwen3_generate.argtypes = [_P, _P, _I64, _I64, _P, _P]
    L.orc_qwen3_layers.restype = _I64
    L.orc_qwen3_layers.argtypes = [_P]
    L.orc_qwen3_embed.restype = _P
    L.orc_qwen3_embed.argtypes = [_P]
    L.orc_qwen3_linear.restype = _I64
    L.orc_qwen3_linear.argtypes = [_P, _I64, C.c_int, C.POINTER(_P), C.POINTER(_P), C.POINTER(_I64)]
    L.orc_qwen3_expert.restype = _I64
    L.orc_qwen3_expert.argtypes = [_P, _I64, _I64, C.c_int, C.POINTER(_P), C.POINTER(_P), C.POINTER(_I64)]
    L.orc_moe_forward.argtypes = [_P, _I64, _I64, _I64, _I64, _I64, C.c_int, _P, _P, _P, _P, _P, _P, _P, _P,
                                  _P, _P, _P]
    L.orc_set_threads.argtypes = [C.c_int]
    L.orc_set_sum_order.argtypes = [C.c_int]
    L.orc_get_threads.restype = C.c_int


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


# ---------------------------------------------------------------------------- conversions
def f32_to_bf16(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_f32_to_bf16_array(_p(x), x.size, _p(out))
    return out


def bf16_to_f32(h) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    lib().orc_bf16_to_f32_array(_p(h), h.size, _p(out))
    return out


def f32_to_f16_bits(x: float) -> int:
    return int(lib().orc_f32_to_f16(float(x)))


def f16_bits_to_f32(h: int) -> float:
    return float(lib().orc_f16_to_f32(int(h)))


# ---------------------------------------------------------------------------- generators
def gen_scale(std: float) -> float:
    return float(lib().orc_gen_scale(std))


def gen_bf16(seed: int, tensor_id: int, count: int, std: float, offset: int = 0) -> np.ndarray:
    out = np.empty(count, dtype=np.uint16)
    lib().orc_gen_bf16(seed, tensor_id, offset, count, lib().orc_gen_scale(std), _p(out))
    return out


def gen_tokens(seed: int, stream: int, count: int, vocab: int) -> np.ndarray:
    out = np.empty(count, dtype=np.int32)
    lib().orc_gen_tokens(seed, stream, count, vocab, _p(out))
    return out


# ---------------------------------------------------------------------------- Q8_0
def q8_0_quantize(x: np.ndarray):
    """Rows of x (f32, or bf16 bit patterns as uint16) -> (qs int8 [rows,k], d uint16 [rows,k/32])."""
    x = np.ascontiguousarray(x)
    rows, k = x.shape
    qs = np.empty((rows, k), dtype=np.int8)
    d = np.empty((rows, k // QK), dtype=np.uint16)
    if x.dtype == np.float32:
        lib().orc_q8_0_quantize_f32(_p(x), rows, k, _p(qs), _p(d))
    elif x.dtype == np.uint16:
        lib().orc_q8_0_quantize_bf16(_p(x), rows, k, _p(qs), _p(d))
    else:
        raise TypeError(x.dtype)
    return qs, d


def q8_0_pack(qs: np.ndarray, d: np.ndarray) -> np.ndarray:
    rows, k = qs.shape
    out = np.empty((rows, (k // QK) * 34), dtype=np.uint8)
    lib().orc_q8_0_pack_blocks(_p(np.ascontiguousarray(qs)), _p(np.ascontiguousarray(d)), rows, k, _p(out))
    return out


def q8_0_unpack(blocks: np.ndarray, k: int):
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    rows = blocks.shape[0]
    qs = np.empty((rows, k), dtype=np.int8)
    d = np.empty((rows, k // QK), dtype=np.uint16)
    lib().orc_q8_0_unpack_blocks(_p(blocks), rows, k, _p(qs), _p(d))
    return qs, d


def q8_0_matmul(xq, xd, wq, wd, with_abs: bool = False):
    m, k = xq.shape
    n = wq.shape[0]
    y = np.empty((m, n), dtype=np.float32)
    a = np.empty((m, n), dtype=np.float32) if with_abs else None
    lib().orc_q8_0_matmul(_p(np.ascontiguousarray(xq)), _p(np.ascontiguousarray(xd)), m,
                          _p(np.ascontiguousarray(wq)), _p(np.ascontiguousarray(wd)), n, k,
                          _p(y), _p(a) if with_abs else None)
    return (y, a) if with_abs else y


def q8_0_linear(x: np.ndarray, wq: np.ndarray, wd: np.ndarray) -> np.ndarray:
    """Linear::forward with a Q8_0 weight; x f32 or bf16 bits (uint16)."""
    xq, xd = q8_0_quantize(x)
    return q8_0_matmul(xq, xd, wq, wd)


def matmul_2d(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), dtype=np.float32)
    lib().orc_matmul_2d(_p(a), m, k, _p(b), n, _p(c))
    return c


# ---------------------------------------------------------------------------- small ops
def rmsnorm(x: np.ndarray, w_bf16: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x)
    rows, dim = x.shape
    out = np.empty((rows, dim), dtype=np.uint16)
    w = np.ascontiguousarray(w_bf16, dtype=np.uint16)
    if x.dtype == np.float32:
        lib().orc_rmsnorm_f32(_p(x), rows, dim, _p(w), eps, _p(out))
    else:
        lib().orc_rmsnorm_bf16(_p(x), rows, dim, _p(w), eps, _p(out))
    return out


def rope_tables(head_dim: int, max_pos: int, theta: float):
    c = np.empty((max_pos, head_dim // 2), dtype=np.float32)
    s = np.empty((max_pos, head_dim // 2), dtype=np.float32)
    lib().orc_rope_tables(head_dim, max_pos, theta, _p(c), _p(s))
    return c, s


def rope_apply(x: np.ndarray, offset: int, cos_t, sin_t) -> np.ndarray:
    """x [BH, L, D] f32 -> rotated copy."""
    y = np.array(x, dtype=np.float32, copy=True, order="C")
    bh, seq, d = y.shape
    lib().orc_rope_apply(_p(y), bh, seq, d, offset, _p(cos_t), _p(sin_t))
    return y


def silu(x: float) -> float:
    return float(lib().orc_silu(float(x)))


def argmax(x: np.ndarray) -> int:
    x = np.ascontiguousarray(x, dtype=np.float32)
    return int(lib().orc_argmax(_p(x), x.size))


def softmax(x: np.ndarray) -> np.ndarray:
    y = np.array(x, dtype=np.float32, copy=True)
    lib().orc_softmax(_p(y), y.size)
    return y


def attend_row(q, k, v, masked=False, causal_limit=0):
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    ctx, d = k.shape
    scratch = np.empty(ctx, dtype=np.float32)
    out = np.empty(d, dtype=np.float32)
    lib().orc_attend_row(_p(q), _p(k), _p(v), ctx, d, d, int(masked), causal_limit, _p(scratch), _p(out))
    return out


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def set_sum_order(reversed_: bool) -> None:
    """Noise probe: RMSNorm sums of squares in reverse order (True) or the reference's order."""
    lib().orc_set_sum_order(1 if reversed_ else 0)


def get_threads() -> int:
    return int(lib().orc_get_threads())


# ---------------------------------------------------------------------------- model
def make_config(**kw) -> Qwen3Config:
    c = Qwen3Config()
    defaults = dict(hidden=1024, layers=28, n_heads=16, n_kv_heads=8, head_dim=128, inter=3072,
                    vocab=VOCAB_QWEN3, max_pos=40960, tied=1, eps=1e-6, theta=1e6,
                    init_std=0.02, norm_std=0.0, n_experts=0, top_k=0, moe_inter=0, norm_topk=0)
    defaults.update(kw)
    for k, v in defaults.items():
        setattr(c, k, v)
    return c


def sample(logits, generated=(), temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0,
           repetition_penalty: float = 1.0, exact_exp: bool = False) -> int:
    """sample_with_config (generate.rs:687-705) after apply_repetition_penalty (:374-411) for
    one row of logits (orc_sample); `generated` = the tokens generated so far. exact_exp:
    top-p's exponentials correctly rounded instead of libm's expf (orc_sample_ex)."""
    lg = np.ascontiguousarray(logits, dtype=np.float32).ravel()
    gen = np.ascontiguousarray(np.asarray(generated, dtype=np.int32).ravel())
    return int(lib().orc_sample_ex(_p(lg), lg.size, _p(gen) if gen.size else None, gen.size, temperature, top_k,
                                   top_p, repetition_penalty, 1 if exact_exp else 0))


class Qwen3Model:
    """Oracle Qwen3ForCausalLM with Q8_0 linears (model.rs:273-372)."""

    def __init__(self, cfg: Qwen3Config, seed: int, layers_limit: int = 0, ctx_max: int = 64):
        self.cfg = cfg
        self.ctx_max = ctx_max
        self._h = lib().orc_qwen3_create(C.byref(cfg), seed, layers_limit, ctx_max)
        if not self._h:
            raise RuntimeError("orc_qwen3_create failed")

    def close(self):
        if self._h:
            lib().orc_qwen3_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def clear(self):
        lib().orc_qwen3_clear(self._h)

    def forward(self, ids, offset: int) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        logits = np.empty(self.cfg.vocab, dtype=np.float32)
        rc = lib().orc_qwen3_forward(self._h, _p(ids), ids.size, offset, _p(logits))
        if rc:
            raise ValueError("orc_qwen3_forward: invalid ids or context overflow")
        return logits

    def linear(self, layer: int, kind: int):
        """(qs int8 [n,k], d uint16 [n,k/32]) copies of a Q8_0 weight (kind 7, layer -1 = lm_head)."""
        qs, d, k = C.c_void_p(), C.c_void_p(), C.c_int64()
        n = lib().orc_qwen3_linear(self._h, layer, kind, C.byref(qs), C.byref(d), C.byref(k))
        if n < 0:
            raise IndexError((layer, kind))
        q = np.ctypeslib.as_array(C.cast(qs, C.POINTER(C.c_int8)), shape=(n, k.value)).copy()
        dd = np.ctypeslib.as_array(C.cast(d, C.POINTER(C.c_uint16)), shape=(n, k.value // QK)).copy()
        return q, dd

    def expert(self, layer: int, expert: int, kind: int):
        """(qs, d) copies of a MoE weight: kind 10 router, 11 gate, 12 up, 13 down of `expert`."""
        qs, d, k = C.c_void_p(), C.c_void_p(), C.c_int64()
        n = lib().orc_qwen3_expert(self._h, layer, expert, kind, C.byref(qs), C.byref(d), C.byref(k))
        if n < 0:
            raise IndexError((layer, expert, kind))
        q = np.ctypeslib.as_array(C.cast(qs, C.POINTER(C.c_int8)), shape=(n, k.value)).copy()
        dd = np.ctypeslib.as_array(C.cast(d, C.POINTER(C.c_uint16)), shape=(n, k.value // QK)).copy()
        return q, dd

    def generate(self, prompt, new_tokens: int, sampling: dict | None = None):
        """Greedy generate, or with `sampling` = dict(temperature, top_k, top_p,
        repetition_penalty) the reference's sample_with_config at every step."""
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(new_tokens, dtype=np.int32)
        logits = np.empty(self.cfg.vocab, dtype=np.float32)
        if sampling is None:
            rc = lib().orc_qwen3_generate(self._h, _p(prompt), prompt.size, new_tokens, _p(out), _p(logits))
        else:
            sc = {"temperature": 0.0, "top_k": 0, "top_p": 1.0, "repetition_penalty": 1.0}
            sc.update(sampling)
            rc = lib().orc_qwen3_generate_cfg(self._h, _p(prompt), prompt.size, new_tokens, sc["temperature"],
                                              sc["top_k"], sc["top_p"], sc["repetition_penalty"], _p(out),
                                              _p(logits))
        if rc:
            raise ValueError("orc_qwen3_generate failed")
        return out, logits


# ---------------------------------------------------------------------------- MoE
def moe_forward(xn_bf16: np.ndarray, router, gate, up, down, top_k: int, norm_topk: bool = True):
    """Mixture-of-experts MLP of one layer (orc_moe_forward). xn_bf16 [rows][H] uint16;
    router = (qs [E][H], d); gate/up/down = lists of per-expert (qs, d). Returns
    (out [rows][H] f32, ids [rows][top_k] int32, weights [rows][top_k] f32)."""
    xn = np.ascontiguousarray(xn_bf16, dtype=np.uint16)
    rows, H = xn.shape
    E = router[0].shape[0]
    inter = gate[0][0].shape[0]
    keep = []

    def ptrs(lst, i):
        arr = (C.c_void_p * E)()
        for e in range(E):
            a = np.ascontiguousarray(lst[e][i])
            keep.append(a)
            arr[e] = a.ctypes.data
        keep.append(arr)
        return C.cast(arr, C.c_void_p)

    out = np.empty((rows, H), np.float32)
    ids = np.empty((rows, top_k), np.int32)
    w = np.empty((rows, top_k), np.float32)
    rq = np.ascontiguousarray(router[0])
    rd = np.ascontiguousarray(router[1])
    lib().orc_moe_forward(_p(xn), rows, H, E, top_k, inter, int(norm_topk), _p(rq), _p(rd),
                          ptrs(gate, 0), ptrs(gate, 1), ptrs(up, 0), ptrs(up, 1), ptrs(down, 0),
                          ptrs(down, 1), _p(out), _p(ids), _p(w))
    return out, ids, w
