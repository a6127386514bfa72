"""GPU parity of the Q8_0 kernels against the CPU oracle, through the C ABI.

Quantization is bit-exact (int8 values and fp16 scales). The GEMM paths (M > 4) keep the
oracle's per-output summation order and are bit-exact, except that a 5-64-token GEMM on a
short grid splits K across CTAs (LQ_GEMM_NO_SPLIT=1 turns that off); the split and the
decode GEMV (M <= 4) regroup the f32 block sum and are checked against the reordering bound
|y_gpu - y_oracle| <= 2 * (nb + 1) * 2^-24 * sum_b |term_b|.
"""
import ctypes as C
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def T(a):
    import torch
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(a).cuda()


def H(t, dtype=None):
    a = t.detach().cpu().numpy()
    if dtype is not None:
        a = a.view(dtype)
    return a


def gpu_quantize(ctx, lq8, x: np.ndarray):
    import torch
    xt = T(x)
    rows, k = x.shape
    qs = torch.empty((rows, k), dtype=torch.int8, device="cuda")
    d = torch.empty((rows, k // 32), dtype=torch.int16, device="cuda")
    dt = lq8.DTYPE_F32 if x.dtype == np.float32 else lq8.DTYPE_BF16
    ctx.call("lq_q8_0_quantize", xt.data_ptr(), dt, rows, k, qs.data_ptr(), d.data_ptr())
    ctx.synchronize()
    return qs, d


@pytest.mark.parametrize("shape", [(1, 32), (3, 96), (64, 1024), (257, 4096), (5, 25600)])
@pytest.mark.parametrize("src", ["f32", "bf16"])
def test_quantize_bit_exact(ctx, lq8_lib, oracle, rng, shape, src):
    x = (rng.standard_normal(shape) * rng.choice([1e-3, 0.02, 1.0, 50.0])).astype(np.float32)
    if src == "bf16":
        x = oracle.f32_to_bf16(x)
    qs, d = gpu_quantize(ctx, lq8_lib, x)
    oq, od = oracle.q8_0_quantize(x)
    assert np.array_equal(H(qs), oq)
    assert np.array_equal(H(d, np.uint16), od)


@pytest.mark.parametrize("name", ["w", "x", "xb", "edge"])
def test_quantize_matches_gguf_fixture(ctx, lq8_lib, oracle, name):
    fx = np.load(os.path.join(GOLDEN, "q8_0_gguf.npz"))
    x = fx[f"{name}_in"]
    qs, d = gpu_quantize(ctx, lq8_lib, x)
    assert np.array_equal(oracle.q8_0_pack(H(qs), H(d, np.uint16)), fx[f"{name}_blocks"])


def test_pack_unpack_blocks(ctx, lq8_lib, oracle, rng):
    import torch
    x = rng.standard_normal((9, 320)).astype(np.float32)
    qs, d = gpu_quantize(ctx, lq8_lib, x)
    blocks = torch.empty((9, 10 * 34), dtype=torch.uint8, device="cuda")
    ctx.call("lq_q8_0_pack_blocks", qs.data_ptr(), d.data_ptr(), 9, 320, blocks.data_ptr())
    q2 = torch.empty_like(qs)
    d2 = torch.empty_like(d)
    ctx.call("lq_q8_0_unpack_blocks", blocks.data_ptr(), 9, 320, q2.data_ptr(), d2.data_ptr())
    ctx.synchronize()
    assert np.array_equal(H(blocks), oracle.q8_0_pack(H(qs), H(d, np.uint16)))
    assert torch.equal(q2, qs) and torch.equal(d2, d)


def _weights(oracle, rng, n, k):
    w = oracle.f32_to_bf16((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    return oracle.q8_0_quantize(w)


def _matmul(ctx, lq8, wq, wd, xq, xd, resid=None, ldy=None):
    import torch
    m, n = xq.shape[0], wq.shape[0]
    ldy = ldy or n
    y = torch.full((m, ldy), float("nan"), dtype=torch.float32, device="cuda")
    r = T(resid) if resid is not None else None
    if r is not None:
        y.copy_(r)
    wq_t, wd_t, xq_t, xd_t = T(wq), T(wd), T(xq), T(xd)
    w = lq8.Q8Tensor(n, wq.shape[1], wq_t.data_ptr(), wd_t.data_ptr())
    ctx.call("lq_q8_0_matmul", C.byref(w), xq_t.data_ptr(), xd_t.data_ptr(), m, y.data_ptr(),
             y.data_ptr() if r is not None else None, ldy)
    ctx.synchronize()
    return H(y)


@pytest.mark.parametrize("m", [1, 2, 3, 4])
@pytest.mark.parametrize("n,k", [(1, 32), (17, 96), (300, 1024), (1024, 3072), (4096, 4096)])
def test_gemv_within_reorder_bound(ctx, lq8_lib, oracle, rng, m, n, k):
    wq, wd = _weights(oracle, rng, n, k)
    xq, xd = oracle.q8_0_quantize(rng.standard_normal((m, k)).astype(np.float32))
    y = _matmul(ctx, lq8_lib, wq, wd, xq, xd)
    ref, absum = oracle.q8_0_matmul(xq, xd, wq, wd, with_abs=True)
    nb = k // 32
    bound = 2.0 * (nb + 1) * 2.0 ** -24 * absum + 1e-30
    assert np.all(np.abs(y - ref) <= bound), float(np.max(np.abs(y - ref) / bound))


@pytest.mark.parametrize("m", [5, 8, 16, 17, 33, 64, 100, 257])
@pytest.mark.parametrize("n,k", [(1, 32), (17, 96), (300, 1024), (640, 3072)])
def test_gemm_bit_exact(ctx, lq8_lib, oracle, rng, monkeypatch, m, n, k):
    """Without the K split (LQ_GEMM_NO_SPLIT=1) every GEMM output is one thread's sum in the
    oracle's block order: bit-identical."""
    monkeypatch.setenv("LQ_GEMM_NO_SPLIT", "1")
    wq, wd = _weights(oracle, rng, n, k)
    xq, xd = oracle.q8_0_quantize(rng.standard_normal((m, k)).astype(np.float32))
    y = _matmul(ctx, lq8_lib, wq, wd, xq, xd)
    assert np.array_equal(y, oracle.q8_0_matmul(xq, xd, wq, wd))


@pytest.mark.parametrize("m", [5, 8, 16, 33, 64])
@pytest.mark.parametrize("n,k", [(300, 1024), (640, 3072), (4096, 4096), (1000, 12288)])
def test_gemm_small_m_split_within_reorder_bound(ctx, lq8_lib, oracle, rng, m, n, k):
    """Decode batches of 5-64 tokens on short grids split K across CTAs; the slices are added
    in a fixed order (deterministic), which regroups the f32 block sum within the bound."""
    wq, wd = _weights(oracle, rng, n, k)
    xq, xd = oracle.q8_0_quantize(rng.standard_normal((m, k)).astype(np.float32))
    y = _matmul(ctx, lq8_lib, wq, wd, xq, xd)
    ref, absum = oracle.q8_0_matmul(xq, xd, wq, wd, with_abs=True)
    bound = 2.0 * (k // 32 + 1) * 2.0 ** -24 * absum + 1e-30
    assert np.all(np.abs(y - ref) <= bound), float(np.max(np.abs(y - ref) / bound))
    assert np.array_equal(y, _matmul(ctx, lq8_lib, wq, wd, xq, xd))  # deterministic


@pytest.mark.parametrize("m,n,k", [(5, 320, 2048), (6, 1280, 5120), (7, 64, 256), (8, 320, 2048), (8, 1280, 5120),
                                   (8, 5120, 25600), (5, 10240, 5120), (8, 10240, 5120), (7, 3200, 5120),
                                   (5, 1000, 2048), (8, 18992, 5120)])
def test_gemm_skinny_stream_k_within_reorder_bound(ctx, lq8_lib, oracle, rng, m, n, k):
    """The 5-8-token GEMM deals 256-byte K units of 128-row tiles evenly over one CTA per SM,
    so tiles are cut between CTAs at arbitrary units (the decode shapes of Qwen3-32B and its
    tensor-parallel shards here, incl. the tp8 rank's 18992-row LM head, whose last tile is
    ragged); the last CTA of a cut tile adds the pieces in CTA order.
    Every output is written (NaN-filled y), within the regrouping bound, and deterministic."""
    wq, wd = _weights(oracle, rng, n, k)
    xq, xd = oracle.q8_0_quantize(rng.standard_normal((m, k)).astype(np.float32))
    y = _matmul(ctx, lq8_lib, wq, wd, xq, xd)
    assert not np.isnan(y).any()
    ref, absum = oracle.q8_0_matmul(xq, xd, wq, wd, with_abs=True)
    bound = 2.0 * (k // 32 + 1) * 2.0 ** -24 * absum + 1e-30
    assert np.all(np.abs(y - ref) <= bound), float(np.max(np.abs(y - ref) / bound))
    assert np.array_equal(y, _matmul(ctx, lq8_lib, wq, wd, xq, xd))


@pytest.mark.parametrize("m,n,k", [(8, 10240, 5120), (5, 1000, 2048), (8, 5120, 25600)])
def test_gemm_skinny_two_ctas_per_sm(ctx, lq8_lib, oracle, rng, monkeypatch, m, n, k):
    """The opt-in configuration with two CTAs per SM and 3-stage rings (LQ_SK_DUAL=1): twice the
    CTAs, so tiles are cut at other units; within the regrouping bound and deterministic."""
    monkeypatch.setenv("LQ_SK_DUAL", "1")
    wq, wd = _weights(oracle, rng, n, k)
    xq, xd = oracle.q8_0_quantize(rng.standard_normal((m, k)).astype(np.float32))
    y = _matmul(ctx, lq8_lib, wq, wd, xq, xd)
    assert not np.isnan(y).any()
    ref, absum = oracle.q8_0_matmul(xq, xd, wq, wd, with_abs=True)
    bound = 2.0 * (k // 32 + 1) * 2.0 ** -24 * absum + 1e-30
    assert np.all(np.abs(y - ref) <= bound), float(np.max(np.abs(y - ref) / bound))
    assert np.array_equal(y, _matmul(ctx, lq8_lib, wq, wd, xq, xd))


def test_gemm_skinny_counters_reset_between_launches(ctx, lq8_lib, oracle, rng):
    """The per-tile arrival counters of the stream-K combine are reset by each tile's last CTA:
    shapes with different cut points launched in turn, three rounds, give the same bits every
    round (a counter left mid-count would skip or double a combine)."""
    cases = []
    for n, k in [(1280, 5120), (5120, 25600), (640, 3072), (10240, 5120)]:
        wq, wd = _weights(oracle, rng, n, k)
        xq, xd = oracle.q8_0_quantize(rng.standard_normal((8, k)).astype(np.float32))
        cases.append((wq, wd, xq, xd))
    first = [_matmul(ctx, lq8_lib, *c) for c in cases]
    for _ in range(2):
        for c, y0 in zip(cases, first):
            assert np.array_equal(_matmul(ctx, lq8_lib, *c), y0)


def _matmul_prefill(ctx, lq8, wq, wd, xq, xd, resid=None, ldy=None):
    import torch
    m, n = xq.shape[0], wq.shape[0]
    ldy = ldy or n
    y = torch.full((m, ldy), float("nan"), dtype=torch.float32, device="cuda")
    r = T(resid) if resid is not None else None
    if r is not None:
        y.copy_(r)
    wq_t, wd_t, xq_t, xd_t = T(wq), T(wd), T(xq), T(xd)
    w = lq8.Q8Tensor(n, wq.shape[1], wq_t.data_ptr(), wd_t.data_ptr())
    ctx.call("lq_q8_0_matmul_prefill", C.byref(w), xq_t.data_ptr(), xd_t.data_ptr(), m, y.data_ptr(),
             y.data_ptr() if r is not None else None, ldy)
    ctx.synchronize()
    return H(y)


def _prefill_bound(oracle, xq, xd, absum, k):
    """fp16 operands: 2^-11 relative rounding each (2^-10 per product), the f32 regrouping bound,
    and the fp16 subnormal range of the weights (an absolute 2^-25 per weight times |x|)."""
    x = xq.astype(np.float32).reshape(xq.shape[0], -1, 32) * xd.view(np.float16).astype(np.float32)[:, :, None]
    xabs = np.abs(x).reshape(xq.shape[0], -1).sum(axis=1)[:, None]
    return (2.0 ** -10 + 2.0 * (k // 32 + 1) * 2.0 ** -24) * absum + 2.0 ** -24 * xabs + 1e-30


@pytest.mark.parametrize("m,n,k,scale", [(128, 640, 3072, 1.0), (300, 1000, 1024, 1.0), (257, 384, 2048, 3e4),
                                         (513, 256, 4096, 1.0)])
def test_gemm_prefill_f16_within_bound(ctx, lq8_lib, oracle, rng, m, n, k, scale):
    """lq_q8_0_matmul_prefill (m >= 128): the weights and activations dequantized to fp16 (a
    power-of-two row scale keeps large activations, here up to ~1e5, in range) and one fp16
    tcgen05 GEMM with f32 accumulation. Ragged token and row tiles; every output against the
    oracle within the fp16 operand bound; deterministic."""
    wq, wd = _weights(oracle, rng, n, k)
    xq, xd = oracle.q8_0_quantize((rng.standard_normal((m, k)) * scale).astype(np.float32))
    y = _matmul_prefill(ctx, lq8_lib, wq, wd, xq, xd)
    assert not np.isnan(y).any()
    ref, absum = oracle.q8_0_matmul(xq, xd, wq, wd, with_abs=True)
    bound = _prefill_bound(oracle, xq, xd, absum, k)
    assert np.all(np.abs(y - ref) <= bound), float(np.max(np.abs(y - ref) / bound))
    assert np.array_equal(y, _matmul_prefill(ctx, lq8_lib, wq, wd, xq, xd))


@pytest.mark.parametrize("m,n,k", [(512, 12288, 4096), (512, 5120, 25600), (2048, 4096, 12288)])
def test_gemm_prefill_config2_shapes(ctx, lq8_lib, oracle, rng, m, n, k):
    """The prefill GEMM shapes of Qwen3-8B and -32B (gate|up / down sizes) at 512 and 2048
    tokens, through both prefill kernels: the exact tcgen05 GEMM (lq_q8_0_matmul) against the
    oracle bit for bit, and the fp16-operand GEMM within its bound, on 48 token rows."""
    wq, wd = _weights(oracle, rng, n, k)
    xq, xd = oracle.q8_0_quantize(rng.standard_normal((m, k)).astype(np.float32))
    y_exact = _matmul(ctx, lq8_lib, wq, wd, xq, xd)
    y_fast = _matmul_prefill(ctx, lq8_lib, wq, wd, xq, xd)
    rows = np.unique(np.concatenate([np.arange(16), rng.choice(m, 16, replace=False), np.arange(m - 16, m)]))
    ref, absum = oracle.q8_0_matmul(xq[rows], xd[rows], wq, wd, with_abs=True)
    assert np.array_equal(y_exact[rows], ref)
    bound = _prefill_bound(oracle, xq[rows], xd[rows], absum, k)
    assert np.all(np.abs(y_fast[rows] - ref) <= bound), float(np.max(np.abs(y_fast[rows] - ref) / bound))
    assert not np.isnan(y_fast).any()


def test_gemm_prefill_residual_stride_and_fallback(ctx, lq8_lib, oracle, rng, monkeypatch):
    """y = residual + x.W^T into a wider row stride (columns past n untouched); fewer than 128
    rows, or LQ_PREFILL_EXACT=1, take the exact kernels (bit-identical to lq_q8_0_matmul)."""
    n, k, ldy = 320, 2048, 384
    wq, wd = _weights(oracle, rng, n, k)
    for m in (200, 100):
        xq, xd = oracle.q8_0_quantize(rng.standard_normal((m, k)).astype(np.float32))
        resid = rng.standard_normal((m, ldy)).astype(np.float32)
        y = _matmul_prefill(ctx, lq8_lib, wq, wd, xq, xd, resid=resid, ldy=ldy)
        assert np.array_equal(y[:, n:], resid[:, n:])
        ref, absum = oracle.q8_0_matmul(xq, xd, wq, wd, with_abs=True)
        bound = _prefill_bound(oracle, xq, xd, absum, k) + 2.0 ** -23 * np.abs(resid[:, :n] + ref)
        assert np.all(np.abs(y[:, :n] - (resid[:, :n] + ref)) <= bound)
        if m < 128:
            assert np.array_equal(y, _matmul(ctx, lq8_lib, wq, wd, xq, xd, resid=resid, ldy=ldy))
    monkeypatch.setenv("LQ_PREFILL_EXACT", "1")
    xq, xd = oracle.q8_0_quantize(rng.standard_normal((200, k)).astype(np.float32))
    assert np.array_equal(_matmul_prefill(ctx, lq8_lib, wq, wd, xq, xd), _matmul(ctx, lq8_lib, wq, wd, xq, xd))


@pytest.mark.parametrize("m", [65, 127, 128, 300, 513])
@pytest.mark.parametrize("n,k", [(128, 256), (129, 512), (1000, 4096), (4096, 1024)])
def test_gemm_tcgen05_bit_exact(ctx, lq8_lib, oracle, rng, m, n, k):
    """The tcgen05 prefill GEMM (m > 64, k % 256 == 0): ragged row/token tiles, one stage
    (k = 256) up to many, scales across a wide dynamic range, all-zero blocks."""
    w = rng.standard_normal((n, k)) * 0.02
    w[:, :32] *= 1e3
    w[n // 2, 64:96] = 0.0
    wq, wd = oracle.q8_0_quantize(oracle.f32_to_bf16(w.astype(np.float32)))
    x = rng.standard_normal((m, k)) * rng.choice([1e-2, 1.0, 30.0], size=(m, 1))
    x[m // 3, 32:64] = 0.0
    xq, xd = oracle.q8_0_quantize(x.astype(np.float32))
    y = _matmul(ctx, lq8_lib, wq, wd, xq, xd)
    assert np.array_equal(y, oracle.q8_0_matmul(xq, xd, wq, wd))


@pytest.mark.parametrize("m", [96, 200])
def test_gemm_tcgen05_residual_and_stride(ctx, lq8_lib, oracle, rng, m):
    n, k, ldy = 300, 768, 320
    wq, wd = _weights(oracle, rng, n, k)
    xq, xd = oracle.q8_0_quantize(rng.standard_normal((m, k)).astype(np.float32))
    resid = rng.standard_normal((m, ldy)).astype(np.float32)
    y = _matmul(ctx, lq8_lib, wq, wd, xq, xd, resid=resid, ldy=ldy)
    ref = oracle.q8_0_matmul(xq, xd, wq, wd)
    assert np.array_equal(y[:, :n], (resid[:, :n] + ref).astype(np.float32))
    assert np.array_equal(y[:, n:], resid[:, n:])


def test_gemm_tcgen05_matches_mma_sync_path(ctx, lq8_lib, oracle, rng, monkeypatch):
    """Both prefill GEMM paths keep the oracle's summation order: identical bits at a
    model-sized shape (LQ_NO_TCGEN05 routes the same call to the mma.sync kernel)."""
    m, n, k = 256, 4096, 4096
    wq, wd = _weights(oracle, rng, n, k)
    xq, xd = oracle.q8_0_quantize(rng.standard_normal((m, k)).astype(np.float32))
    y_tc = _matmul(ctx, lq8_lib, wq, wd, xq, xd)
    monkeypatch.setenv("LQ_NO_TCGEN05", "1")
    y_mma = _matmul(ctx, lq8_lib, wq, wd, xq, xd)
    monkeypatch.delenv("LQ_NO_TCGEN05")
    assert np.array_equal(y_tc, y_mma)
    rows = rng.choice(m, 8, replace=False)
    assert np.array_equal(y_tc[rows], oracle.q8_0_matmul(xq[rows], xd[rows], wq, wd))


@pytest.mark.parametrize("m", [1, 16])
def test_matmul_residual_and_stride(ctx, lq8_lib, oracle, rng, monkeypatch, m):
    monkeypatch.setenv("LQ_GEMM_NO_SPLIT", "1")
    n, k, ldy = 200, 512, 256
    wq, wd = _weights(oracle, rng, n, k)
    xq, xd = oracle.q8_0_quantize(rng.standard_normal((m, k)).astype(np.float32))
    resid = rng.standard_normal((m, ldy)).astype(np.float32)
    y = _matmul(ctx, lq8_lib, wq, wd, xq, xd, resid=resid, ldy=ldy)
    ref = oracle.q8_0_matmul(xq, xd, wq, wd)
    np.testing.assert_allclose(y[:, :n], resid[:, :n] + ref, rtol=1e-5, atol=1e-5)
    assert np.array_equal(y[:, n:], resid[:, n:])          # columns past n untouched
    if m > 4:
        assert np.array_equal(y[:, :n], (resid[:, :n] + ref).astype(np.float32))


@pytest.mark.parametrize("m", [5, 8, 16, 23, 40, 64])
@pytest.mark.parametrize("split", [False, True])
def test_gemm_stream_residual_and_stride(ctx, lq8_lib, oracle, rng, monkeypatch, m, split):
    """The streamed small-M GEMMs (5 <= m <= 64, n % 64 == 0, k % 256 == 0; 5-8 tokens take the
    skinny stream-K GEMM, whose last 128-row tile is half past n here): passes of 16 or 32
    tokens with a ragged last pass, y = residual + W.x into a wider row stride, columns past n
    untouched. Unsplit it is bit-identical to the oracle; with K slices (a 5-tile grid) within
    the regrouping bound and deterministic."""
    if not split:
        monkeypatch.setenv("LQ_GEMM_NO_SPLIT", "1")
    n, k, ldy = 320, 2048, 384
    wq, wd = _weights(oracle, rng, n, k)
    xq, xd = oracle.q8_0_quantize(rng.standard_normal((m, k)).astype(np.float32))
    resid = rng.standard_normal((m, ldy)).astype(np.float32)
    y = _matmul(ctx, lq8_lib, wq, wd, xq, xd, resid=resid, ldy=ldy)
    ref, absum = oracle.q8_0_matmul(xq, xd, wq, wd, with_abs=True)
    assert np.array_equal(y[:, n:], resid[:, n:])
    if not split:
        assert np.array_equal(y[:, :n], (resid[:, :n] + ref).astype(np.float32))
    else:
        bound = 2.0 * (k // 32 + 1) * 2.0 ** -24 * absum + 1e-30 + 2.0 ** -23 * np.abs(resid[:, :n] + ref)
        assert np.all(np.abs(y[:, :n] - (resid[:, :n] + ref)) <= bound)
        assert np.array_equal(y, _matmul(ctx, lq8_lib, wq, wd, xq, xd, resid=resid, ldy=ldy))


@pytest.mark.parametrize("m", [1, 3, 12])
@pytest.mark.parametrize("src", ["f32", "bf16"])
def test_linear_forward(ctx, lq8_lib, oracle, rng, m, src):
    import torch
    n, k = 384, 1024
    wq, wd = _weights(oracle, rng, n, k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    if src == "bf16":
        x = oracle.f32_to_bf16(x)
    lin = lq8_lib.Linear(ctx, lq8_lib.QTensor(T(wq), T(wd)))
    xt = T(x) if src == "f32" else T(x).view(torch.bfloat16)
    y = H(lin.forward(xt))
    ctx.synchronize()
    ref = oracle.q8_0_linear(x, wq, wd)
    xq, xd = oracle.q8_0_quantize(x)
    _, absum = oracle.q8_0_matmul(xq, xd, wq, wd, with_abs=True)
    assert np.all(np.abs(y - ref) <= 2.0 * (k // 32 + 1) * 2.0 ** -24 * absum + 1e-30)


def test_linear_shape_mismatch_is_an_error(ctx, lq8_lib, oracle, rng):
    wq, wd = _weights(oracle, rng, 64, 256)
    lin = lq8_lib.Linear(ctx, lq8_lib.QTensor(T(wq), T(wd)))
    with pytest.raises(ValueError):
        lin.forward(T(np.zeros((2, 128), np.float32)))
    wq_t, wd_t = T(wq), T(wd)
    bad = lq8_lib.Q8Tensor(64, 100, wq_t.data_ptr(), wd_t.data_ptr())  # k not a multiple of 32
    y = T(np.zeros((1, 64), np.float32))
    x = T(np.zeros((1, 100), np.float32))
    with pytest.raises(lq8_lib.LQ8Error) as e:
        ctx.call("lq_q8_0_linear", C.byref(bad), x.data_ptr(), lq8_lib.DTYPE_F32, 1, y.data_ptr())
    assert e.value.code == -1


def test_fill_bf16_matches_oracle_generator(ctx, lq8_lib, oracle):
    import torch
    out = torch.empty(100003, dtype=torch.int16, device="cuda")
    ctx.call("lq_fill_bf16", 1234, 0x305, 17, 100003, 0.02, out.data_ptr())
    ctx.synchronize()
    assert np.array_equal(H(out, np.uint16), oracle.gen_bf16(1234, 0x305, 100003, 0.02, offset=17))
