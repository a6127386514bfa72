"""lq_q8_0_linear_noalloc: the Q8_0 Linear for callers that must not allocate device memory.

lq_q8_0_linear may call cudaMalloc/cudaFree to grow its scratch; some callers cannot allow
that (a decode loop with a latency budget, since both calls can synchronise the device, or a
host whose device memory all belongs to its own pool). The no-allocation variant keeps its
scratch in a fixed 4 MiB device array instead. These tests check, through the C ABI, that it
gives the same output as lq_q8_0_linear on two calls in a row (the second call reuses the
array the first one left behind), and that calls too large for the array are refused.

The file is named to be collected last, so a run that stops at the first failure has run
every other test before it.
"""
import ctypes as C

import numpy as np
import pytest

from test_gpu_q8 import H, T

pytestmark = pytest.mark.gpu


def _linear(ctx, lq8, name, w, x_t, dt, m):
    import torch
    y = torch.full((m, w.n), float("nan"), dtype=torch.float32, device="cuda")
    ctx.call(name, C.byref(w), x_t.data_ptr(), dt, m, y.data_ptr())
    ctx.synchronize()
    return H(y)


@pytest.mark.parametrize("m,n,k,src", [(1, 384, 1024, "f32"), (3, 4096, 4096, "bf16"),
                                       (16, 640, 3072, "f32"), (4, 300, 96, "bf16")])
def test_noalloc_linear_matches_linear_twice(ctx, lq8_lib, oracle, rng, m, n, k, src):
    w16 = oracle.f32_to_bf16((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    wq, wd = oracle.q8_0_quantize(w16)
    wq_t, wd_t = T(wq), T(wd)
    w = lq8_lib.Q8Tensor(n, k, wq_t.data_ptr(), wd_t.data_ptr())
    dt = lq8_lib.DTYPE_F32 if src == "f32" else lq8_lib.DTYPE_BF16
    for call in range(2):  # the second call starts from the first call's scratch contents
        x = (rng.standard_normal((m, k)) * (1 + call)).astype(np.float32)
        if src == "bf16":
            x = oracle.f32_to_bf16(x)
        x_t = T(x)
        ref = _linear(ctx, lq8_lib, "lq_q8_0_linear", w, x_t, dt, m)
        got = _linear(ctx, lq8_lib, "lq_q8_0_linear_noalloc", w, x_t, dt, m)
        # the tolerance of the Linear tests: f32 reordering bound against the oracle
        xq, xd = oracle.q8_0_quantize(x)
        orc, absum = oracle.q8_0_matmul(xq, xd, wq, wd, with_abs=True)
        bound = 2.0 * (k // 32 + 1) * 2.0 ** -24 * absum + 1e-30
        assert np.all(np.abs(got - ref) <= bound), call
        assert np.all(np.abs(got - orc) <= bound), call


def test_noalloc_rejects_calls_beyond_the_fixed_scratch(ctx, lq8_lib, oracle, rng):
    n, k = 64, 25600
    wq, wd = oracle.q8_0_quantize(oracle.f32_to_bf16((rng.standard_normal((n, k)) * 0.02).astype(np.float32)))
    wq_t, wd_t = T(wq), T(wd)
    w = lq8_lib.Q8Tensor(n, k, wq_t.data_ptr(), wd_t.data_ptr())
    m = 160  # 160 * 25600 * 34/32 bytes > 4 MiB
    x_t = T(np.zeros((m, k), np.float32))
    import torch
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    with pytest.raises(lq8_lib.LQ8Error) as e:
        ctx.call("lq_q8_0_linear_noalloc", C.byref(w), x_t.data_ptr(), lq8_lib.DTYPE_F32, m, y.data_ptr())
    assert e.value.code == -1 and "fixed scratch" in str(e.value)
