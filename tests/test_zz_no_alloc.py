"""lq_q8_0_linear_noalloc: the Q8_0 Linear for callers that must not allocate device memory.

lq_q8_0_linear may call cudaMalloc/cudaFree to grow its scratch (the quantized rows, and the
K-split partial sums of the 5..64-row GEMM); some callers cannot allow that (a decode loop
with a latency budget, since both calls can synchronise the device, or a host whose device
memory all belongs to its own pool). The no-allocation variant keeps all of it in a fixed
4 MiB device array instead. These tests check, through the C ABI:
- its output is bit-identical to lq_q8_0_linear's on two calls in a row (the second call
  starts from what the first left in the shared array), and within the oracle's reordering
  bound, for row counts that take the decode GEMV, the streamed small-M GEMM with K split,
  the mma.sync GEMM with K split, and the tcgen05 GEMM;
- it allocates nothing: on a context that has never allocated scratch, with every library
  allocation turned into an error (LQ_FAULT=ensure_scratch,ensure_split), the calls succeed
  and the device's free memory does not change;
- calls whose rows or K-split partials exceed the array are refused with a clear error.

The file is named to be collected last, so a run that stops at the first failure has run
every other test before it.
"""
import ctypes as C

import numpy as np
import pytest

from test_gpu_q8 import H, T

pytestmark = pytest.mark.gpu

# (m, n, k, source dtype): GEMV (m <= 4), streamed GEMM split over K (n % 64 == 0, few row
# tiles), mma.sync GEMM split over K (n % 64 != 0), tcgen05 GEMM (m > 64)
CASES = [(1, 384, 1024, "f32"), (3, 4096, 4096, "bf16"), (5, 640, 3072, "f32"), (16, 640, 3072, "f32"),
         (64, 640, 3072, "bf16"), (16, 300, 1024, "f32"), (40, 200, 2048, "bf16"), (80, 256, 1024, "f32")]


def _weight(lq8, oracle, rng, n, k):
    w16 = oracle.f32_to_bf16((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    wq, wd = oracle.q8_0_quantize(w16)
    wq_t, wd_t = T(wq), T(wd)
    return lq8.Q8Tensor(n, k, wq_t.data_ptr(), wd_t.data_ptr()), (wq, wd), (wq_t, wd_t)


def _inputs(oracle, rng, m, k, src, calls=2):
    xs = []
    for call in range(calls):
        x = (rng.standard_normal((m, k)) * (1 + call)).astype(np.float32)
        if src == "bf16":
            x = oracle.f32_to_bf16(x)
        xs.append(x)
    return xs


def _run(c, name, w, x_t, dt, y):
    c.call(name, C.byref(w), x_t.data_ptr(), dt, y.shape[0], y.data_ptr())


@pytest.mark.parametrize("m,n,k,src", CASES)
def test_noalloc_linear_matches_linear_twice(ctx, lq8_lib, oracle, rng, m, n, k, src):
    import torch
    w, (wq, wd), keep = _weight(lq8_lib, oracle, rng, n, k)
    dt = lq8_lib.DTYPE_F32 if src == "f32" else lq8_lib.DTYPE_BF16
    for call, x in enumerate(_inputs(oracle, rng, m, k, src)):
        x_t = T(x)
        ref = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        got = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        _run(ctx, "lq_q8_0_linear", w, x_t, dt, ref)
        _run(ctx, "lq_q8_0_linear_noalloc", w, x_t, dt, got)
        ctx.synchronize()
        ref, got = H(ref), H(got)
        # same kernels, same K slices, same reduce order: the same bits
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), call
        # and the Linear tests' tolerance against the oracle (f32 reordering bound)
        xq, xd = oracle.q8_0_quantize(x)
        orc, absum = oracle.q8_0_matmul(xq, xd, wq, wd, with_abs=True)
        bound = 2.0 * (k // 32 + 1) * 2.0 ** -24 * absum + 1e-30
        assert np.all(np.abs(got - orc) <= bound), call


def test_noalloc_allocates_nothing_on_a_fresh_context(ctx, lq8_lib, oracle, rng, monkeypatch):
    import torch
    setups = []
    for m, n, k, src in CASES:
        w, _, keep = _weight(lq8_lib, oracle, rng, n, k)
        dt = lq8_lib.DTYPE_F32 if src == "f32" else lq8_lib.DTYPE_BF16
        xs = [T(x) for x in _inputs(oracle, rng, m, k, src)]
        ref = [torch.empty((m, n), dtype=torch.float32, device="cuda") for _ in xs]
        got = [torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda") for _ in xs]
        setups.append((w, keep, dt, xs, ref, got))
    # outputs of the allocating entry point, and every kernel loaded and configured once, so
    # that nothing the driver does on first use shows up in the free-memory figure below
    for w, _, dt, xs, ref, got in setups:
        for x_t, r, g in zip(xs, ref, got):
            _run(ctx, "lq_q8_0_linear", w, x_t, dt, r)
            _run(ctx, "lq_q8_0_linear_noalloc", w, x_t, dt, g)
    ctx.synchronize()
    for _, _, _, _, _, got in setups:
        for g in got:
            g.fill_(float("nan"))
    torch.cuda.synchronize()

    fresh = lq8_lib.Context(0)  # no scratch and no split buffer yet
    try:
        fresh.synchronize()
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        # any scratch or split-buffer allocation the library tries now fails the call
        monkeypatch.setenv("LQ_FAULT", "ensure_scratch,ensure_split")
        for w, _, dt, xs, _, got in setups:
            for x_t, g in zip(xs, got):
                _run(fresh, "lq_q8_0_linear_noalloc", w, x_t, dt, g)
        fresh.synchronize()
        monkeypatch.delenv("LQ_FAULT")
        free_after = torch.cuda.mem_get_info()[0]
        assert free_after == free_before, (free_before, free_after)
        for w, _, _, _, ref, got in setups:
            for r, g in zip(ref, got):
                assert torch.equal(g.view(torch.int32), r.view(torch.int32))
    finally:
        fresh.close()


def test_noalloc_rejects_calls_beyond_the_fixed_scratch(ctx, lq8_lib, oracle, rng):
    import torch
    # quantized rows alone too large: 160 * 25600 * 34/32 bytes > 4 MiB
    # K-split partials too large: 64 rows over 32 row tiles of 2048 x 8192 split 16 ways
    # (16 * 64 * 2048 * 4 bytes = 8 MiB) while the rows take 0.5 MiB
    for m, n, k in [(160, 64, 25600), (64, 2048, 8192)]:
        w, _, keep = _weight(lq8_lib, oracle, rng, n, k)
        x_t = T(np.zeros((m, k), np.float32))
        y = torch.empty((m, n), dtype=torch.float32, device="cuda")
        with pytest.raises(lq8_lib.LQ8Error) as e:
            ctx.call("lq_q8_0_linear_noalloc", C.byref(w), x_t.data_ptr(), lq8_lib.DTYPE_F32, m, y.data_ptr())
        assert e.value.code == -1 and "fixed scratch" in str(e.value), str(e.value)
