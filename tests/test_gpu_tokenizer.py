"""Text generation through the device runner: tokenizer.generate_text (generate.rs:611-661)
on a tiny Qwen3 whose vocabulary is the byte-level test tokenizer's 259 ids, against the
runner's own token loop (prefill + decode steps) on the same prompt ids, cut at the first EOS
id and decoded with special tokens skipped -- greedy and with the sampling knobs."""
import numpy as np
import pytest

pytest.importorskip("tokenizers")

import tokenizer as T  # qwen-omni-inference-rs_b200/tokenizer.py
from test_tokenizer import BOS, IM_END, _hf

pytestmark = pytest.mark.gpu

CFG = dict(hidden=256, layers=2, n_heads=4, n_kv_heads=2, head_dim=128, inter=512, vocab=259, tied=1,
           norm_std=0.1)


def _loop(model, ids, n, tok, **sampling):
    model.clear_kv_cache()
    model.set_batch(1)
    model.set_sampling(**sampling)
    out = list(ids)
    nxt = int(model.prefill(np.asarray(ids, np.int32))[0])
    out.append(nxt)
    for _ in range(1, n):
        if tok.is_eos(nxt):
            break
        nxt = int(model.decode_step(np.asarray([nxt], np.int32))[0])
        out.append(nxt)
    return out


@pytest.mark.parametrize("sampling", [{}, {"temperature": 0.8, "top_k": 20, "repetition_penalty": 1.3}])
def test_generate_text_matches_the_runner_loop(ctx, lq8_lib, tmp_path, sampling):
    p = tmp_path / "tokenizer.json"
    _hf().save(str(p))
    tok = T.Tokenizer.from_file(p, BOS, [IM_END, BOS])
    model = lq8_lib.Qwen3ForCausalLM(ctx, lq8_lib.make_config(**CFG), 4321, max_batch=1, ctx_max=64)
    prompt = "Qwen3 on B200"
    n = 12
    text = T.generate_text(model, tok, prompt, n, **sampling)
    ref_ids = _loop(model, tok.encode(prompt, True), n, tok, **sampling)
    assert text == tok.decode(ref_ids, True)
    assert text.startswith(prompt)
    model.close()
