"""The oracle against the reference's own known-answer tests (restated from the Rust test
modules; values copied from the cited assertions)."""
import math

import numpy as np
import pytest


def test_matmul_2d_basic(oracle):
    # tensor.rs:3360-3375: [[1,2],[3,4]] @ [[5,6],[7,8]] = [19,22,43,50]
    c = oracle.matmul_2d(np.array([[1, 2], [3, 4]]), np.array([[5, 6], [7, 8]]))
    assert c.ravel().tolist() == [19.0, 22.0, 43.0, 50.0]


def test_matmul_bf16_inputs(oracle):
    # tensor.rs:3504-3539: the same product from bf16 operands is exact
    a = oracle.bf16_to_f32(oracle.f32_to_bf16(np.array([[1, 2], [3, 4]], np.float32)))
    b = oracle.bf16_to_f32(oracle.f32_to_bf16(np.array([[5, 6], [7, 8]], np.float32)))
    assert oracle.matmul_2d(a, b).ravel().tolist() == [19.0, 22.0, 43.0, 50.0]


def test_matmul_2d_non_square_and_identity(oracle):
    # tensor.rs:3377-3419
    a = np.arange(1, 7, dtype=np.float32).reshape(2, 3)
    b = np.arange(7, 13, dtype=np.float32).reshape(3, 2)
    assert oracle.matmul_2d(a, b).ravel().tolist() == [58.0, 64.0, 139.0, 154.0]
    eye = np.eye(3, dtype=np.float32)
    assert np.array_equal(oracle.matmul_2d(a, eye), a)


def test_gemv_known_answer(oracle):
    # gpu/gemv.rs:561-587: 4x3 matrix times [1,2,3] = [14,32,50,68]
    m = np.arange(1, 13, dtype=np.float32).reshape(4, 3)
    v = np.array([[1], [2], [3]], np.float32)
    assert oracle.matmul_2d(m, v).ravel().tolist() == [14.0, 32.0, 50.0, 68.0]


def test_gemv_known_answer_q8_0(oracle):
    # the same GEMV through the Q8_0 path: pad K to one 32-block with zeros. The weights are
    # integers 1..12 with block amax 3|6|9|12, and the vector [1,2,3]: the products are exact
    # only up to Q8_0 rounding, so compare within the format's step (amax/127 per block).
    w = np.zeros((4, 32), np.float32)
    w[:, :3] = np.arange(1, 13, dtype=np.float32).reshape(4, 3)
    x = np.zeros((1, 32), np.float32)
    x[0, :3] = [1, 2, 3]
    qs, d = oracle.q8_0_quantize(w)
    y = oracle.q8_0_linear(x, qs, d)
    np.testing.assert_allclose(y.ravel(), [14, 32, 50, 68], rtol=2e-2)


@pytest.mark.parametrize("val,bits", [
    (0.0, 0x0000), (-0.0, 0x8000), (1.0, 0x3F80), (-1.0, 0xBF80),
    (math.inf, 0x7F80), (-math.inf, 0xFF80),
])
def test_bf16_special_values(oracle, val, bits):
    # bf16.rs:163-214 (zero, negative zero, one, infinities)
    assert int(oracle.f32_to_bf16(np.array([val], np.float32))[0]) == bits


def test_bf16_round_to_nearest_even(oracle):
    # bf16.rs:238-252: 1.0 + exact half ulp (0x3F808000) ties to even -> 0x3F80
    x = np.array([0x3F808000, 0x3F818000, 0x3F808001], np.uint32).view(np.float32)
    got = oracle.f32_to_bf16(x).tolist()
    assert got == [0x3F80, 0x3F82, 0x3F81]


def test_bf16_nan_and_subnormal(oracle):
    # bf16.rs:217-236 (test_nan, test_subnormal_flush_to_zero): NaN stays NaN; the smallest subnormal rounds to (signed) zero
    nan = oracle.f32_to_bf16(np.array([np.nan], np.float32))
    assert math.isnan(float(oracle.bf16_to_f32(nan)[0]))
    sub = np.array([0x00000001], np.uint32).view(np.float32)
    assert float(oracle.bf16_to_f32(oracle.f32_to_bf16(sub))[0]) == 0.0


def test_bf16_from_bits(oracle):
    # bf16.rs:388-400
    assert float(oracle.bf16_to_f32(np.array([0x3F80], np.uint16))[0]) == 1.0
    assert float(oracle.bf16_to_f32(np.array([0x0000], np.uint16))[0]) == 0.0


def test_silu_values(oracle):
    # tensor.rs:1946-1953 doc test: silu(0)=0, silu(1)~0.7311, silu(-1)~-0.2689
    assert abs(oracle.silu(0.0)) < 1e-5
    assert abs(oracle.silu(1.0) - 0.7311) < 1e-3
    assert abs(oracle.silu(-1.0) + 0.2689) < 1e-3


def test_softmax_ordering_and_sum(oracle):
    # tensor.rs:1901-1912 doc test: increasing inputs give increasing probabilities
    p = oracle.softmax(np.array([1.0, 2.0, 3.0], np.float32))
    assert p[2] > p[1] > p[0]
    assert abs(float(p.sum()) - 1.0) < 1e-6


def test_argmax_ties_resolve_to_last(oracle):
    # tensor.rs:2451-2482 uses Iterator::max_by, which returns the last maximum
    assert oracle.argmax(np.array([1.0, 4.0, 2.0, 3.0])) == 1
    assert oracle.argmax(np.array([5.0, 2.0, 3.0, 1.0])) == 0
    assert oracle.argmax(np.array([3.0, 1.0, 3.0, 2.0])) == 2
    assert oracle.argmax(np.array([7.0, 7.0, 7.0])) == 2


def test_rope_identity_at_position_zero(oracle, rng):
    # rope.rs:341-371: position 0 leaves q and k unchanged
    c, s = oracle.rope_tables(128, 16, 1e6)
    x = rng.standard_normal((3, 1, 128)).astype(np.float32)
    y = oracle.rope_apply(x, 0, c, s)
    assert np.array_equal(x, y)


def test_rope_preserves_norm(oracle, rng):
    # rope.rs:373-411: a rotation keeps each head vector's norm
    c, s = oracle.rope_tables(128, 64, 1e6)
    x = rng.standard_normal((2, 8, 128)).astype(np.float32)
    y = oracle.rope_apply(x, 5, c, s)
    np.testing.assert_allclose(np.linalg.norm(y, axis=-1), np.linalg.norm(x, axis=-1), rtol=1e-5)


def test_rope_table_frequency_pattern(oracle):
    # rope.rs:89-117: entries 2i and 2i+1 share angle pos * theta^(-2i/64) (not HF's -j/64)
    c, s = oracle.rope_tables(128, 8, 1e6)
    for pos in range(8):
        for i in range(32):
            ang = pos * (1.0 / (1e6 ** ((2 * i) / 64)))
            assert c[pos, 2 * i] == c[pos, 2 * i + 1] == np.float32(math.cos(ang))
            assert s[pos, 2 * i] == s[pos, 2 * i + 1] == np.float32(math.sin(ang))


def test_causal_mask_semantics(oracle, rng):
    # causal_mask.rs:104-164: row i attends to positions <= i + offset; masking by -inf equals
    # attending over the visible prefix only
    k = rng.standard_normal((6, 128)).astype(np.float32)
    v = rng.standard_normal((6, 128)).astype(np.float32)
    q = rng.standard_normal(128).astype(np.float32)
    masked = oracle.attend_row(q, k, v, masked=True, causal_limit=3)
    prefix = oracle.attend_row(q, k[:4], v[:4])
    np.testing.assert_array_equal(masked, prefix)


def test_rope_cos_sin_known_positions(oracle):
    # rope.rs:514-543: head_dim 4, theta 1e4: position 0 -> (1, 0); position 1 -> (cos 1, sin 1)
    c, s = oracle.rope_tables(4, 100, 1e4)
    assert c[0, 0] == 1.0 and s[0, 0] == 0.0
    assert c[1, 0] == c[1, 1] == np.float32(math.cos(1.0))
    assert s[1, 0] == s[1, 1] == np.float32(math.sin(1.0))
