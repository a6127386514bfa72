"""The oracle's Q8_0 format and matmul, pinned against GGML's published algorithm through
gguf-py 0.19.0 (committed fixtures, plus a live comparison when gguf is importable), and the
oracle's other outputs against the committed regression fixtures."""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def gguf_fx():
    return np.load(os.path.join(GOLDEN, "q8_0_gguf.npz"))


@pytest.fixture(scope="module")
def small_fx():
    return np.load(os.path.join(GOLDEN, "oracle_small.npz"))


@pytest.mark.parametrize("name", ["w", "x", "xb", "edge"])
def test_q8_0_bit_exact_vs_gguf_fixture(oracle, gguf_fx, name):
    a = gguf_fx[f"{name}_in"]
    qs, d = oracle.q8_0_quantize(a)
    assert np.array_equal(oracle.q8_0_pack(qs, d), gguf_fx[f"{name}_blocks"])


def test_q8_0_bit_exact_vs_gguf_live(oracle, rng):
    gq = pytest.importorskip("gguf.quants")
    for scale in (1e-3, 0.02, 1.0, 300.0):
        a = (rng.standard_normal((33, 320)) * scale).astype(np.float32)
        ref = np.asarray(gq.quantize(a, gq.GGMLQuantizationType.Q8_0)).reshape(33, -1)
        qs, d = oracle.q8_0_quantize(a)
        assert np.array_equal(oracle.q8_0_pack(qs, d), ref)


def test_q8_0_bf16_input_equals_widened_f32(oracle, rng):
    xb = oracle.f32_to_bf16(rng.standard_normal((7, 256)).astype(np.float32))
    q1, d1 = oracle.q8_0_quantize(xb)
    q2, d2 = oracle.q8_0_quantize(oracle.bf16_to_f32(xb))
    assert np.array_equal(q1, q2) and np.array_equal(d1, d2)


def test_q8_0_pack_unpack_roundtrip(oracle, rng):
    a = rng.standard_normal((5, 128)).astype(np.float32)
    qs, d = oracle.q8_0_quantize(a)
    blocks = oracle.q8_0_pack(qs, d)
    assert blocks.shape == (5, 4 * 34)
    qs2, d2 = oracle.q8_0_unpack(blocks, 128)
    assert np.array_equal(qs, qs2) and np.array_equal(d, d2)


def test_q8_0_edge_blocks(oracle):
    e = np.zeros((3, 32), np.float32)
    e[1, :] = np.linspace(-127, 127, 32)
    e[2, :] = 63.5
    e[2, 0] = 127.0
    qs, d = oracle.q8_0_quantize(e)
    assert d[0, 0] == 0 and not qs[0].any()                     # zero block: d = 0, q = 0
    assert oracle.f16_bits_to_f32(int(d[1, 0])) == 1.0          # amax 127 -> d = 1
    assert qs[1, 0] == -127 and qs[1, -1] == 127
    assert qs[2, 1] == 64                                       # 63.5 rounds away from zero
    assert np.abs(qs.astype(np.int32)).max() <= 127


def test_q8_0_matmul_matches_float64(oracle, rng):
    """y = sum_b sumi_b * (d_w d_x): compare with the same sum in float64; the only
    difference allowed is f32 accumulation error, bounded by (nb-1) * 2^-24 * sum |term|."""
    k, n, m = 512, 40, 6
    w = oracle.f32_to_bf16((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    x = rng.standard_normal((m, k)).astype(np.float32)
    wq, wd = oracle.q8_0_quantize(w)
    xq, xd = oracle.q8_0_quantize(x)
    y, absum = oracle.q8_0_matmul(xq, xd, wq, wd, with_abs=True)
    nb = k // 32
    dw = np.array([[oracle.f16_bits_to_f32(v) for v in r] for r in wd], np.float64)
    dx = np.array([[oracle.f16_bits_to_f32(v) for v in r] for r in xd], np.float64)
    sumi = np.einsum("mbi,nbi->mnb", xq.reshape(m, nb, 32).astype(np.int64),
                     wq.reshape(n, nb, 32).astype(np.int64)).astype(np.float64)
    exact = np.einsum("mnb,nb,mb->mn", sumi, dw, dx)
    bound = (nb - 1 + 2) * 2.0 ** -24 * absum.astype(np.float64)
    assert np.all(np.abs(y - exact) <= bound)


def test_q8_0_linear_close_to_dense(oracle, rng):
    # the Q8_0 Linear approximates the dense product (MSE/cosine, tests/validation.rs:228-293)
    w = (rng.standard_normal((64, 1024)) * 0.02).astype(np.float32)
    x = rng.standard_normal((4, 1024)).astype(np.float32)
    wq, wd = oracle.q8_0_quantize(w)
    y = oracle.q8_0_linear(x, wq, wd)
    ref = x.astype(np.float64) @ w.T.astype(np.float64)
    cos = float((y.ravel() @ ref.ravel()) / (np.linalg.norm(y) * np.linalg.norm(ref)))
    assert cos > 0.9999


def _splitmix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = x + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def test_generator_numpy_restatement(oracle):
    """The integer-exact generator restated in numpy: SplitMix64 -> Irwin-Hall(4) -> one f32
    multiply -> bf16 RNE. The GPU implements the same function; identical bits on both."""
    seed, tid, n = 99, 0x305, 2000
    with np.errstate(over="ignore"):
        key = _splitmix64(np.array([seed ^ ((tid * 0xD1B54A32D192ED03) & (2**64 - 1))], np.uint64))[0]
        h = _splitmix64(key + np.arange(n, dtype=np.uint64))
    m16 = np.uint64(0xFFFF)
    s = sum(((h >> np.uint64(sh)) & m16).astype(np.int64) for sh in (0, 16, 32, 48)) - 131070
    scale = np.float32(oracle.gen_scale(0.02))
    vals = s.astype(np.float32) * scale
    assert np.array_equal(oracle.f32_to_bf16(vals), oracle.gen_bf16(seed, tid, n, 0.02))
    # the distribution approximates N(0, 0.02)
    big = oracle.bf16_to_f32(oracle.gen_bf16(seed, tid, 200000, 0.02))
    assert abs(big.mean()) < 2e-4 and abs(big.std() - 0.02) < 2e-4


def test_oracle_regression_fixture(oracle, small_fx):
    f = small_fx
    wq, wd = oracle.q8_0_quantize(f["mm_w_bf16"])
    assert np.array_equal(oracle.q8_0_linear(f["mm_x"], wq, wd), f["mm_y"])
    assert np.array_equal(oracle.rmsnorm(f["rms_x"], f["rms_w"], 1e-6), f["rms_y"])
    c, s = oracle.rope_tables(128, 32, 1e6)
    assert np.array_equal(oracle.rope_apply(f["rope_x"], 7, c, s), f["rope_y"])
    assert np.array_equal(oracle.attend_row(f["att_q"], f["att_k"], f["att_v"]), f["att_y"])
    assert np.array_equal(oracle.attend_row(f["att_q"], f["att_k"], f["att_v"], True, 17), f["att_y_masked"])
    assert np.array_equal(oracle.gen_bf16(1234, 0x12345, 4096, 0.02), f["gen_bf16"])


def test_tiny_model_fixture_and_thread_independence(oracle, small_fx):
    cfg = oracle.make_config(hidden=256, layers=2, n_heads=4, n_kv_heads=2, head_dim=128, inter=512,
                             vocab=1000, tied=1, norm_std=0.1)
    saved = oracle.get_threads()
    try:
        for threads in (1, saved):
            oracle.set_threads(threads)
            m = oracle.Qwen3Model(cfg, 1234, ctx_max=64)
            toks, logits = m.generate(small_fx["tiny_prompt"], 8)
            assert np.array_equal(toks, small_fx["tiny_tokens"])
            assert np.array_equal(logits, small_fx["tiny_logits"])
    finally:
        oracle.set_threads(saved)


def test_prefill_equals_incremental_decode(oracle):
    """The reference's prefill (masked L x L attention) equals feeding the tokens one at a
    time: masked entries contribute exp(-inf) = 0 exactly."""
    cfg = oracle.make_config(hidden=256, layers=2, n_heads=4, n_kv_heads=2, head_dim=128, inter=512,
                             vocab=500, tied=0)
    prompt = oracle.gen_tokens(7, 1, 6, cfg.vocab)
    a = oracle.Qwen3Model(cfg, 7, ctx_max=16)
    la = a.forward(prompt, 0)
    b = oracle.Qwen3Model(cfg, 7, ctx_max=16)
    for i, t in enumerate(prompt):
        lb = b.forward(np.array([t]), i)
    assert np.array_equal(la, lb)


@pytest.mark.parametrize("name", ["w", "x", "xb", "edge"])
def test_host_quantizer_of_the_c_abi_matches_gguf_fixture(lq8_lib, oracle, gguf_fx, name):
    """lq_q8_0_quantize_host (the C ABI's host mirror of the device quantizer; no GPU needed)
    against the gguf-py fixtures, from f32 and from the bf16 rounding of the same rows."""
    import ctypes as C
    lib = lq8_lib.load()
    a = np.ascontiguousarray(gguf_fx[f"{name}_in"], dtype=np.float32)
    rows, k = a.shape
    for src, dt in ((a, lq8_lib.DTYPE_F32), (oracle.f32_to_bf16(a), lq8_lib.DTYPE_BF16)):
        src = np.ascontiguousarray(src)
        qs = np.empty((rows, k), np.int8)
        d = np.empty((rows, k // 32), np.uint16)
        assert lib.lq_q8_0_quantize_host(src.ctypes.data, dt, rows, k, qs.ctypes.data, d.ctypes.data) == 0
        oq, od = oracle.q8_0_quantize(src)
        assert np.array_equal(qs, oq) and np.array_equal(d, od)
        if dt == lq8_lib.DTYPE_F32:
            assert np.array_equal(oracle.q8_0_pack(qs, d), gguf_fx[f"{name}_blocks"])


def test_host_quantizer_rejects_bad_shapes(lq8_lib):
    lib = lq8_lib.load()
    assert lib.lq_q8_0_quantize_host(None, 0, 1, 33, None, None) == -1
    assert b"multiple of 32" in lib.lq_last_error(None)
