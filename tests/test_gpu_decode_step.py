"""The persistent decode step -- one cooperative kernel runs every layer and the LM head of a
dense model's decode step on one GPU -- against the per-layer decode kernels and the CPU oracle.

The persistent kernel performs every arithmetic step of the per-layer kernels in the same
order (the same row functions, per-lane block order, warp sums and attention order), so the
logits of the two paths must be bit-identical at every step; the per-layer path itself is
checked against the oracle in test_gpu_model.py, and the oracle comparison here repeats that
check through the persistent path. Shapes cover the single-chunk K (hidden 256), K split into
2 KiB chunks with a ragged last chunk (hidden 2560, inter 9728), GQA groups of 2 and 8, a
ragged last LM-head unit (vocab 1003), batches 1-4 and decode positions across the
64-position attention chunk boundary.
"""
import numpy as np
import pytest

from conftest import cos_sim

pytestmark = pytest.mark.gpu

TINY = dict(hidden=256, layers=2, n_heads=4, n_kv_heads=2, head_dim=128, inter=512, vocab=1000,
            tied=1, norm_std=0.1)
CONFIGS = {
    "tiny": TINY,
    "gqa8_ragged_vocab": dict(TINY, n_heads=8, n_kv_heads=1, tied=0, vocab=1003),
    "wide": dict(TINY, hidden=2560, inter=9728, n_heads=32, n_kv_heads=8, vocab=1024, tied=0),
}


def _pair(lq8, ctx, cfgd, seed, B, ctx_max, monkeypatch):
    cfg = lq8.make_config(**cfgd)
    monkeypatch.setenv("LQ_NO_PERSIST", "1")
    ref = lq8.Qwen3ForCausalLM(ctx, cfg, seed, max_batch=B, ctx_max=ctx_max)
    monkeypatch.delenv("LQ_NO_PERSIST")
    per = lq8.Qwen3ForCausalLM(ctx, cfg, seed, max_batch=B, ctx_max=ctx_max)
    return per, ref


@pytest.mark.parametrize("cfg_name,B", [("tiny", 1), ("tiny", 2), ("tiny", 4), ("gqa8_ragged_vocab", 3),
                                        ("wide", 1), ("wide", 2)])
def test_persistent_step_bit_identical(ctx, lq8_lib, oracle, monkeypatch, cfg_name, B):
    cfgd = CONFIGS[cfg_name]
    seed, L, steps = 77, 60, 10  # decode positions 60..69 cross the first chunk boundary
    per, ref = _pair(lq8_lib, ctx, cfgd, seed, B, 256, monkeypatch)
    prompts = np.stack([oracle.gen_tokens(seed, s, L, cfgd["vocab"]) for s in range(B)])
    for m in (per, ref):
        m.clear_kv_cache()
        m.set_batch(B)
    n1, l1 = per.prefill(prompts, want_logits=True)
    n2, l2 = ref.prefill(prompts, want_logits=True)
    assert np.array_equal(l1, l2) and np.array_equal(n1, n2)
    tok = n1
    for i in range(steps):
        a, la = per.decode_step(tok, want_logits=True)
        b, lb = ref.decode_step(tok, want_logits=True)
        assert np.array_equal(la, lb), (i, float(np.max(np.abs(la - lb))))
        assert np.array_equal(a, b), i
        for r in range(B):
            assert a[r] == oracle.argmax(la[r]), (i, r)  # ties -> the highest index
        tok = a
    # embedding, the persistent step and the argmax finalisation; the per-layer path
    # launches five kernels per layer
    assert per.graph_kernels() == 3
    assert ref.graph_kernels() == 3 + 5 * cfgd["layers"]
    per.close()
    ref.close()


@pytest.mark.parametrize("cfg_name,B", [("wide", 1), ("wide", 3), ("tiny", 4), ("gqa8_ragged_vocab", 4)])
def test_persistent_step_bit_identical_long_context(ctx, lq8_lib, oracle, monkeypatch, cfg_name, B):
    """Contexts of ~1280 positions: 20-21 chunks per (row, kv head), so 80-480 attention items
    against 148 SMs (GQA groups of 2, 4 and 8). CTAs take several items in turn, with the next
    item's cache rows copied in while the current one is computed, and merge tasks wait on
    chunks of other CTAs; decode positions 1276..1281 cross the chunk boundary at 1280."""
    cfgd = CONFIGS[cfg_name]
    seed, L, steps = 91, 1276, 6
    per, ref = _pair(lq8_lib, ctx, cfgd, seed, B, 1296, monkeypatch)
    prompts = np.stack([oracle.gen_tokens(seed, s, L, cfgd["vocab"]) for s in range(B)])
    for m in (per, ref):
        m.clear_kv_cache()
        m.set_batch(B)
    tok = per.prefill(prompts)
    ref.prefill(prompts)
    for i in range(steps):
        a, la = per.decode_step(tok, want_logits=True)
        b, lb = ref.decode_step(tok, want_logits=True)
        assert np.array_equal(la, lb), (i, float(np.max(np.abs(la - lb))))
        assert np.array_equal(a, b), i
        tok = a
    per.close()
    ref.close()


def test_persistent_step_matches_oracle(ctx, lq8_lib, oracle):
    """Teacher-forced decode through the persistent step against the oracle on the tiny
    config, with the per-layer decode path's tolerance (cosine >= 0.99999, max |diff| <=
    1e-3 max |logit|) and the greedy token wherever the oracle's top-1/top-2 margin clears it.
    (Longer prompts push this 2-layer model's activations across Q8_0 rounding boundaries --
    cosine 0.99997 at a 62-token prompt on either decode path -- so the chunk-boundary
    positions are covered by the bit-identity test above.)"""
    seed, L, steps = 1234, 12, 16
    gm = lq8_lib.Qwen3ForCausalLM(ctx, lq8_lib.make_config(**TINY), seed, max_batch=1, ctx_max=64)
    ocfg = oracle.make_config(**TINY)
    om = oracle.Qwen3Model(ocfg, seed, ctx_max=64)
    prompt = oracle.gen_tokens(seed, 0, L, ocfg.vocab)
    gm.prefill(prompt)
    tok = oracle.argmax(om.forward(prompt, 0))
    for i in range(steps):
        g_next, g_lg = gm.decode_step(np.array([tok], np.int32), want_logits=True)
        olg = om.forward(np.array([tok]), L + i)
        assert cos_sim(g_lg[0], olg) >= 0.99999, i
        assert np.max(np.abs(g_lg[0] - olg)) <= 1e-3 * np.max(np.abs(olg)), i
        s = np.sort(olg)
        if s[-1] - s[-2] > 2e-3 * np.max(np.abs(olg)):
            assert g_next[0] == oracle.argmax(olg), i
        tok = oracle.argmax(olg)
    assert gm.graph_kernels() == 3
    gm.close()


@pytest.mark.parametrize("cfg_name,cfgd", [("wide", CONFIGS["wide"]), ("gqa8_ragged_vocab", CONFIGS["gqa8_ragged_vocab"]),
                                           ("qwen3_8b_2l", dict(TINY, hidden=4096, inter=12288, n_heads=32,
                                                                n_kv_heads=8, vocab=151936, tied=0))])
def test_persistent_batch_rows_are_independent(ctx, lq8_lib, oracle, monkeypatch, cfg_name, cfgd):
    """Batches of 5-8 rows run the persistent step's tensor-core consumer: each token is its own
    MMA column with its own scales, the warps' partial sums are added in warp order, and
    attention and the norms work per row, so a row's logits do not depend on the batch size.
    Decoding 8 sequences must give rows 0-4 exactly the logits of decoding only those 5 (same
    tokens fed, same prefill); the 8B shapes run a 5-stage ring at batch 8, the ragged vocabulary
    a partial last LM-head unit."""
    seed, L, steps = 5, 70, 4
    cfg = lq8_lib.make_config(**cfgd)
    prompts = np.stack([oracle.gen_tokens(seed, s, L, cfgd["vocab"]) for s in range(8)])
    monkeypatch.setenv("LQ_PERSIST_MAX_BATCH", "8")  # batches of 5-8 are opt-in
    big = lq8_lib.Qwen3ForCausalLM(ctx, cfg, seed, max_batch=8, ctx_max=96)
    small = lq8_lib.Qwen3ForCausalLM(ctx, cfg, seed, max_batch=5, ctx_max=96)
    monkeypatch.delenv("LQ_PERSIST_MAX_BATCH")
    try:
        t8 = big.prefill(prompts)
        big.set_batch(8)
        outs, tok = [], t8
        for _ in range(steps):
            nxt, lg = big.decode_step(tok, want_logits=True)
            outs.append((tok, nxt, lg))
            tok = nxt
        assert big.graph_kernels() == 3
        small.prefill(prompts[:5])
        small.set_batch(5)
        for i, (fed, nxt, lg) in enumerate(outs):
            n5, l5 = small.decode_step(fed[:5], want_logits=True)
            assert np.array_equal(l5, lg[:5]), (i, float(np.max(np.abs(l5 - lg[:5]))))
            assert np.array_equal(n5, nxt[:5]), i
            for r in range(5):
                assert n5[r] == oracle.argmax(l5[r]), (i, r)
        assert small.graph_kernels() == 3
    finally:
        big.close()
        small.close()
