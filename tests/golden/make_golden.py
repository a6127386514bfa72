"""Generates the committed golden fixtures in tests/golden/.

  q8_0_gguf.npz   Q8_0 blocks produced by gguf-py 0.19.0 (gguf.quants.quantize, documented as
                  bit-exact with ggml-quants.c quantize_row_q8_0_ref) for seeded f32 inputs,
                  bf16-valued inputs and hand-made edge blocks. This pins the oracle's Q8_0
                  format against a third-party implementation of the GGML algorithm.
  oracle_small.npz  Outputs of the CPU oracle on small seeded cases (Q8_0 matmul, RMSNorm,
                  RoPE, attention row, tiny Qwen3 greedy tokens + logits). These pin the
                  oracle against regressions and give the GPU tests fixed expectations.

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import oracle as O  # noqa: E402

SEED = 1234


def q8_inputs() -> dict[str, np.ndarray]:
    rng = np.random.default_rng(SEED)
    w = (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)          # weight-like
    x = rng.standard_normal((16, 512)).astype(np.float32)                    # activation-like
    xb = O.bf16_to_f32(O.f32_to_bf16(rng.standard_normal((8, 1024)).astype(np.float32)))
    edge = np.zeros((8, 32), np.float32)
    edge[1, :] = np.linspace(-127, 127, 32)                                  # d = 1 exactly
    edge[2, :] = 63.5                                                        # ties away from zero
    edge[2, 1::2] = -63.5
    edge[2, 0] = 127.0
    edge[3, :] = 1e-30 * np.arange(32)                                       # scale underflows fp16
    edge[4, :] = 1e7 * (np.arange(32) - 16)                                  # scale overflows fp16
    edge[5, 7] = -3.0                                                        # amax at a negative
    edge[6, :] = 0.5 + np.arange(32, dtype=np.float32) / 64.0
    edge[7, :] = np.float32(1.0) / 3.0
    return {"w": w, "x": x, "xb": xb.astype(np.float32), "edge": edge}


def gguf_blocks(a: np.ndarray) -> np.ndarray:
    from gguf.quants import GGMLQuantizationType, quantize
    with np.errstate(all="ignore"):
        return np.asarray(quantize(a, GGMLQuantizationType.Q8_0)).reshape(a.shape[0], -1)


def make_q8() -> None:
    out = {}
    for name, a in q8_inputs().items():
        out[f"{name}_in"] = a
        out[f"{name}_blocks"] = gguf_blocks(a)
    np.savez_compressed(os.path.join(HERE, "q8_0_gguf.npz"), **out)


def make_oracle() -> None:
    rng = np.random.default_rng(SEED + 1)
    out = {}
    # Q8_0 matmul: f32 activations x bf16-valued weights
    w = O.f32_to_bf16((rng.standard_normal((96, 256)) * 0.02).astype(np.float32))
    x = rng.standard_normal((5, 256)).astype(np.float32)
    wq, wd = O.q8_0_quantize(w)
    out["mm_w_bf16"], out["mm_x"] = w, x
    out["mm_y"] = O.q8_0_linear(x, wq, wd)
    # RMSNorm of f32 input with random weights
    xr = (rng.standard_normal((4, 1024)) * 3).astype(np.float32)
    nw = O.f32_to_bf16((1 + 0.1 * rng.standard_normal(1024)).astype(np.float32))
    out["rms_x"], out["rms_w"] = xr, nw
    out["rms_y"] = O.rmsnorm(xr, nw, 1e-6)
    # RoPE at an offset
    c, s = O.rope_tables(128, 32, 1e6)
    xp = rng.standard_normal((3, 4, 128)).astype(np.float32)
    out["rope_x"] = xp
    out["rope_y"] = O.rope_apply(xp, 7, c, s)
    # one attention row (decode) and a masked row (prefill)
    q = rng.standard_normal(128).astype(np.float32)
    k = rng.standard_normal((40, 128)).astype(np.float32)
    v = rng.standard_normal((40, 128)).astype(np.float32)
    out["att_q"], out["att_k"], out["att_v"] = q, k, v
    out["att_y"] = O.attend_row(q, k, v)
    out["att_y_masked"] = O.attend_row(q, k, v, masked=True, causal_limit=17)
    # tiny Qwen3: greedy tokens and final logits
    cfg = O.make_config(hidden=256, layers=2, n_heads=4, n_kv_heads=2, head_dim=128, inter=512,
                        vocab=1000, tied=1, norm_std=0.1)
    m = O.Qwen3Model(cfg, SEED, ctx_max=64)
    prompt = O.gen_tokens(SEED, 0, 12, cfg.vocab)
    toks, logits = m.generate(prompt, 8)
    out["tiny_prompt"], out["tiny_tokens"], out["tiny_logits"] = prompt, toks, logits
    # generator samples
    out["gen_bf16"] = O.gen_bf16(SEED, 0x12345, 4096, 0.02)
    np.savez_compressed(os.path.join(HERE, "oracle_small.npz"), **out)


if __name__ == "__main__":
    O.build()
    make_q8()
    make_oracle()
    for f in ("q8_0_gguf.npz", "oracle_small.npz"):
        print(f, os.path.getsize(os.path.join(HERE, f)), "bytes")
