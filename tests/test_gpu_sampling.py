"""The device token choice (lq_sample, lq_qwen3_set_sampling) against the oracle's restatement
of the reference's sample_with_config + apply_repetition_penalty (generate.rs:374-418,
:687-705), itself pinned to the reference's unit-test answers (test_sampling_oracle.py).

Integer results: the chosen token must be identical for identical logits. The model test runs
free-running generation on both sides; their logits agree to the model tolerance, so the
tokens must agree wherever the oracle's decision margin exceeds that tolerance."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CONFIGS = [
    dict(),
    dict(temperature=0.37),
    dict(temperature=2.5, repetition_penalty=1.7),
    dict(top_k=5, temperature=0.8),
    dict(top_k=1, repetition_penalty=3.0),
    dict(top_p=0.9, temperature=0.6),
    dict(top_p=0.5, temperature=1.0, repetition_penalty=1.2),
    dict(temperature=1.0, repetition_penalty=2.0),   # greedy dispatch, penalty still applied
]


def _device(lq8, ctx, logits, gen, cfg):
    import torch
    lg = torch.from_numpy(logits).cuda()
    g = torch.from_numpy(gen).cuda() if gen.size else None
    out = lq8.sample(ctx, lg, g, gen.shape[1] if gen.size else 0, **cfg)
    ctx.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("cfg", CONFIGS)
@pytest.mark.parametrize("V", [1000, 151936])
def test_sample_matches_oracle(ctx, lq8_lib, oracle, rng, cfg, V):
    rows, n_gen = 4, 40
    logits = (rng.standard_normal((rows, V)) * 4).astype(np.float32)
    gen = rng.integers(0, 64, (rows, n_gen)).astype(np.int32)      # repeats guaranteed
    for r in range(rows):  # ties at the maximum, some of them on penalized tokens
        m = logits[r].max()
        logits[r, rng.integers(0, V, 3)] = m
        logits[r, gen[r, :3]] = m
    got = _device(lq8_lib, ctx, logits, gen, cfg)
    for r in range(rows):
        assert got[r] == oracle.sample(logits[r], gen[r], **cfg), (cfg, r)
    got0 = _device(lq8_lib, ctx, logits, np.zeros((rows, 0), np.int32), cfg)
    for r in range(rows):
        assert got0[r] == oracle.sample(logits[r], [], **cfg), (cfg, r)


def test_top_p_near_ties(ctx, lq8_lib, oracle):
    """Scaled logits at the maximum one ulp apart and small enough that exp(s - max) lies
    within 2^-22 below 1: the probability itself decides (the kernel's exact path). The
    decision then depends on the last bit of a sum of exponentials, so both sides use the
    correctly rounded exp (the device's choice); libm's expf rounds a few inputs the other way."""
    V = 3000
    base = np.full(V, -3.0, np.float32)
    cases = []
    # 0.01: neighbours' exp(s - max) round to 1 (exact ties); 0.75 .. 1.5: one and two ulps
    # below the maximum give exp within 2^-22 below 1 (the probabilities decide)
    for mx in (np.float32(0.01), np.float32(0.75), np.float32(1.0), np.float32(1.5)):
        x = base.copy()
        x[100] = np.nextafter(mx, np.float32(-1))
        x[2000] = mx
        x[50] = np.nextafter(np.nextafter(mx, np.float32(-1)), np.float32(-1))
        cases.append(x)
    logits = np.stack(cases)
    for cfg in (dict(top_p=0.9, temperature=1.0), dict(top_p=0.3, temperature=0.5)):
        got = _device(lq8_lib, ctx, logits, np.zeros((len(cases), 0), np.int32), cfg)
        for r in range(len(cases)):
            assert got[r] == oracle.sample(logits[r], [], exact_exp=True, **cfg), (cfg, r)


@pytest.mark.parametrize("bad", [dict(temperature=-0.1), dict(top_p=1.5), dict(top_p=-0.1),
                                 dict(repetition_penalty=0.5), dict(top_k=-1)])
def test_sample_rejects_invalid_config(ctx, lq8_lib, bad):
    """GenerationConfig::new's checks (generate.rs:93-126) as LQ_ERR_INVALID_ARG."""
    import torch
    lg = torch.zeros((1, 10), dtype=torch.float32, device="cuda")
    with pytest.raises(lq8_lib.LQ8Error):
        lq8_lib.sample(ctx, lg, None, 0, **bad)


TINY = dict(hidden=256, layers=2, n_heads=4, n_kv_heads=2, head_dim=128, inter=512, vocab=1000, tied=1,
            norm_std=0.1)


def _transformed(logits, gen, cfg):
    """The values the reference's strategy compares (for the decision margin)."""
    x = logits.astype(np.float32).copy()
    pen = np.float32(cfg.get("repetition_penalty", 1.0))
    if abs(pen - 1) >= 1e-6:
        for t in gen:
            v = x[t]
            x[t] = v / pen if v > 0 else (v * pen if v < 0 else v)
    T = np.float32(cfg.get("temperature", 0.0))
    if T == 0 or cfg.get("top_k", 0) > 0:
        return x
    if abs(cfg.get("top_p", 1.0) - 1) >= 1e-6:
        return x / T if abs(T - 1) > 1e-6 else x
    return x * (np.float32(1.0) / T) if abs(T - 1) >= 1e-6 else x


@pytest.mark.parametrize("cfg", [dict(temperature=0.7, repetition_penalty=1.3), dict(top_k=3, repetition_penalty=1.5),
                                 dict(top_p=0.8, temperature=0.9, repetition_penalty=1.1)])
@pytest.mark.parametrize("persist", [True, False])
def test_generate_with_sampling_matches_oracle(ctx, lq8_lib, oracle, monkeypatch, cfg, persist):
    if not persist:
        monkeypatch.setenv("LQ_NO_PERSIST", "1")
    seed, L, steps = 1234, 12, 16
    gm = lq8_lib.Qwen3ForCausalLM(ctx, lq8_lib.make_config(**TINY), seed, max_batch=1, ctx_max=64)
    gm.set_sampling(**cfg)
    om = oracle.Qwen3Model(oracle.make_config(**TINY), seed, ctx_max=64)
    prompt = oracle.gen_tokens(seed, 0, L, TINY["vocab"])
    toks = gm.generate(prompt, steps)[0]
    gen = []
    lg = om.forward(prompt, 0)
    for i in range(steps):
        want = oracle.sample(lg, gen, **cfg)
        if toks[i] != want:
            v = np.sort(_transformed(lg, gen, cfg))
            assert v[-1] - v[-2] <= 2e-3 * np.max(np.abs(lg)), (i, toks[i], want)
            break
        gen.append(want)
        lg = om.forward(np.array([want]), L + i)
    assert gm.graph_kernels() == (4 if persist else 3 + 5 * TINY["layers"] + 1)
    gm.close()
