"""The oracle's restatement of the reference's sampling (generate.rs) on the CPU, pinned to the
known answers of the reference's own unit tests (generate.rs:420-588) and to the tie and
rounding rules its code implies: greedy and temperature sampling break ties to the last index
(max_by), top-k and top-p take the first element of a stable descending sort (ties to the
first index), and the repetition penalty is applied once per generated occurrence, in order."""
import numpy as np
import pytest


def test_reference_known_answers(oracle):
    S = oracle.sample
    # test_sample_greedy, test_sample_greedy_3d (last position)
    assert S([1.0, 2.0, 5.0, 1.0, 0.5]) == 2
    assert S([2.0, 1.0, 0.5, 4.0, 1.0]) == 3
    # test_sample_temperature_zero (T = 0.01 through sample_temperature), _one
    assert S([1.0, 3.0, 2.0, 0.5], temperature=0.01) == 1
    assert S([1.0, 3.0, 2.0, 0.5], temperature=1.0) == 1
    # test_sample_top_k, test_sample_top_k_zero
    assert S([1.0, 5.0, 2.0, 4.0, 3.0], top_k=3, temperature=1.0) == 1
    assert S([1.0, 5.0, 2.0, 4.0, 3.0], top_k=0, temperature=1.0) == 1
    # test_sample_top_p, test_sample_top_p_one
    assert S([1.0, 5.0, 2.0, 4.0, 3.0], top_p=0.9, temperature=1.0) == 1
    assert S([1.0, 5.0, 2.0, 4.0, 3.0], top_p=1.0, temperature=1.0) == 1
    # test_apply_repetition_penalty: tokens 1 and 3 halved -> [1, 1, 3, 2, 5]
    assert S([1.0, 2.0, 3.0, 4.0, 5.0], generated=[1, 3], repetition_penalty=2.0) == 4
    assert S([1.0, 2.0, 3.0, 4.0, 5.0], generated=[4], repetition_penalty=2.0) == 3   # 5 -> 2.5
    # penalty 1.0 and an empty history change nothing
    assert S([1.0, 2.0, 3.0], generated=[2], repetition_penalty=1.0) == 2
    assert S([1.0, 2.0, 3.0], generated=[], repetition_penalty=2.0) == 2


def test_tie_rules(oracle):
    S = oracle.sample
    x = [1.0, 7.0, 3.0, 7.0, 2.0]
    assert S(x) == 3                                    # greedy: last
    assert S(x, temperature=0.5) == 3                   # temperature: greedy over x * 2
    assert S(x, top_k=2, temperature=0.7) == 1          # top-k: first
    assert S(x, top_p=0.5, temperature=0.7) == 1        # top-p: first
    assert S(x, top_p=0.5, temperature=1.0) == 1


def test_penalty_signs_and_repeats(oracle):
    S = oracle.sample
    # a negative logit is multiplied: -1 * 2 = -2 ties token 1 (-2) -> greedy picks the last
    assert S([-1.0, -2.0], generated=[0], repetition_penalty=2.0) == 1
    # zero stays zero
    assert S([0.0, -0.5], generated=[0, 0, 0], repetition_penalty=4.0) == 0
    # repeats compound in order: 8 / 2 / 2 / 2 = 1 < 1.5
    assert S([8.0, 1.5], generated=[0, 0, 0], repetition_penalty=2.0) == 1
    assert S([8.0, 1.5], generated=[0, 0], repetition_penalty=2.0) == 0
    # out-of-range ids are ignored (generate.rs:398)
    assert S([1.0, 2.0], generated=[5], repetition_penalty=3.0) == 1


def test_rounding_is_the_references(oracle, rng):
    """Temperature multiplies by the f32 reciprocal (mul_scalar), top-p divides by T: the
    oracle applies exactly those f32 operations, so ties created by rounding resolve as in
    the reference. Checked against a numpy float32 restatement."""
    for _ in range(50):
        V = 257
        x = (rng.standard_normal(V) * 3).astype(np.float32)
        x[rng.integers(0, V, 4)] = x[int(np.argmax(x))]  # plant ties at the maximum
        T = np.float32(rng.uniform(0.2, 3.0))
        inv = np.float32(1.0) / T
        y = x * inv
        want_t = int(np.flatnonzero(y == y.max())[-1])
        assert oracle.sample(x, temperature=float(T)) == want_t
        s = x / T
        want_p = int(np.flatnonzero(s == s.max())[0])
        assert oracle.sample(x, top_p=0.8, temperature=float(T)) == want_p
        want_k = int(np.flatnonzero(x == x.max())[0])
        assert oracle.sample(x, top_k=5, temperature=float(T)) == want_k


@pytest.mark.parametrize("cfg", [dict(temperature=0.7, repetition_penalty=1.3), dict(top_k=4, repetition_penalty=1.1),
                                 dict(top_p=0.9, temperature=0.8)])
def test_generate_with_sampling_runs(oracle, cfg):
    """The oracle model's generate with a sampling configuration: the first token ignores the
    penalty (no history yet) and equals the greedy-over-transformed-logits choice."""
    c = oracle.make_config(hidden=256, layers=1, n_heads=4, n_kv_heads=2, head_dim=128, inter=512, vocab=300,
                           tied=1, norm_std=0.1)
    m = oracle.Qwen3Model(c, 11, ctx_max=32)
    prompt = oracle.gen_tokens(11, 0, 5, c.vocab)
    toks, _ = m.generate(prompt, 6, sampling=cfg)
    lg = m.forward(prompt, 0)
    assert toks[0] == oracle.sample(lg, **cfg)
    assert np.all((toks >= 0) & (toks < c.vocab))
