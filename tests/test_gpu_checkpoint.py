"""Loading a packed checkpoint into the device runner. A bf16 SafeTensors checkpoint holding
exactly the weights of a seed-1234 model (the seeded generator's values; norms read back from
that model) is packed to a Q8_0 GGUF file and loaded into a model built with another seed:
every Q8_0 linear, norm and the embedding must then equal the seed-1234 model's bit for bit,
and so must its logits and greedy tokens."""
import os

import numpy as np
import pytest

from test_gpu_q8 import H

pytestmark = pytest.mark.gpu

# tensor ids of the seeded generator (shared by the runner and the oracle)
K_Q, K_K, K_V, K_O, K_GATE, K_UP, K_DOWN = range(7)
TID_EMBED, TID_LMHEAD = 0x7FFF0001, 0x7FFF0002


def _tid(layer, kind):
    return (layer << 8) | kind


def _bf16(lq8, ptr, n):
    return H(lq8.wrap_device(ptr, (n,), "<u2")).view(np.uint16).copy()


def _checkpoint(lq8, oracle, model, cfgd, seed, path):
    import torch
    from safetensors.torch import save_file
    c = oracle.make_config(**cfgd)
    H_, I, V = cfgd["hidden"], cfgd["inter"], cfgd["vocab"]
    Hq, Hkv, D = cfgd["n_heads"], cfgd["n_kv_heads"], cfgd["head_dim"]
    std = float(c.init_std)

    def gen(tid, n, k):
        return oracle.gen_bf16(seed, tid, n * k, std).reshape(n, k)

    sd = {"model.embed_tokens.weight": gen(TID_EMBED, V, H_),
          "model.norm.weight": _bf16(lq8, *model.tensor(-1, "final_norm"))}
    if not cfgd["tied"]:
        sd["lm_head.weight"] = gen(TID_LMHEAD, V, H_)
    for i in range(cfgd["layers"]):
        p = f"model.layers.{i}."
        sd.update({p + "self_attn.q_proj.weight": gen(_tid(i, K_Q), Hq * D, H_),
                   p + "self_attn.k_proj.weight": gen(_tid(i, K_K), Hkv * D, H_),
                   p + "self_attn.v_proj.weight": gen(_tid(i, K_V), Hkv * D, H_),
                   p + "self_attn.o_proj.weight": gen(_tid(i, K_O), H_, Hq * D),
                   p + "mlp.gate_proj.weight": gen(_tid(i, K_GATE), I, H_),
                   p + "mlp.up_proj.weight": gen(_tid(i, K_UP), I, H_),
                   p + "mlp.down_proj.weight": gen(_tid(i, K_DOWN), H_, I),
                   p + "input_layernorm.weight": _bf16(lq8, *model.tensor(i, "in_norm")),
                   p + "post_attention_layernorm.weight": _bf16(lq8, *model.tensor(i, "post_norm")),
                   p + "self_attn.q_norm.weight": _bf16(lq8, *model.tensor(i, "q_norm")),
                   p + "self_attn.k_norm.weight": _bf16(lq8, *model.tensor(i, "k_norm"))})
    save_file({k: torch.from_numpy(np.ascontiguousarray(v).view(np.int16)).view(torch.bfloat16)
               for k, v in sd.items()}, path)


@pytest.mark.parametrize("tied", [0, 1])
def test_loaded_checkpoint_equals_seeded_model(ctx, lq8_lib, oracle, tmp_path, tied):
    import checkpoint as ck
    cfgd = dict(hidden=256, layers=2, n_heads=4, n_kv_heads=2, head_dim=128, inter=512, vocab=1000,
                tied=tied, norm_std=0.1, max_pos=4096)
    ref = lq8_lib.Qwen3ForCausalLM(ctx, lq8_lib.make_config(**cfgd), 1234, max_batch=1, ctx_max=64)
    st = os.path.join(str(tmp_path), "model.safetensors")
    _checkpoint(lq8_lib, oracle, ref, cfgd, 1234, st)
    gg = os.path.join(str(tmp_path), "model-q8_0.gguf")
    run_cfg = {k: cfgd[k] for k in ("hidden", "layers", "n_heads", "n_kv_heads", "head_dim", "inter", "vocab", "tied",
                                    "max_pos")}
    run_cfg.update(eps=float(np.float32(1e-6)), theta=1e6)
    ck.pack_safetensors(st, gg, run_cfg)
    meta, _ = ck.read_gguf(gg)
    fcfg = ck.config_from_gguf(meta)
    model = lq8_lib.Qwen3ForCausalLM(ctx, lq8_lib.make_config(**dict(cfgd, **fcfg)), 999, max_batch=1, ctx_max=64)
    ck.load_gguf(model, gg)
    kinds = ["q", "k", "v", "o", "gate", "up", "down"]
    for i in range(cfgd["layers"]):
        for kind in kinds:
            a = lq8_lib.QTensor.from_struct(model.linear(i, kind))
            b = lq8_lib.QTensor.from_struct(ref.linear(i, kind))
            assert np.array_equal(H(a.qs), H(b.qs)) and np.array_equal(H(a.d, np.uint16), H(b.d, np.uint16)), (i, kind)
        for kind in ("in_norm", "post_norm", "q_norm", "k_norm"):
            assert np.array_equal(_bf16(lq8_lib, *model.tensor(i, kind)), _bf16(lq8_lib, *ref.tensor(i, kind)))
    a = lq8_lib.QTensor.from_struct(model.linear(-1, "lm_head"))
    b = lq8_lib.QTensor.from_struct(ref.linear(-1, "lm_head"))
    assert np.array_equal(H(a.qs), H(b.qs)) and np.array_equal(H(a.d, np.uint16), H(b.d, np.uint16))
    assert np.array_equal(_bf16(lq8_lib, *model.tensor(-1, "embed")), _bf16(lq8_lib, *ref.tensor(-1, "embed")))
    prompt = oracle.gen_tokens(5, 0, 9, cfgd["vocab"])
    n1, l1 = model.prefill(prompt, want_logits=True)
    n2, l2 = ref.prefill(prompt, want_logits=True)
    assert np.array_equal(l1, l2) and np.array_equal(n1, n2)
    assert np.array_equal(model.generate(prompt, 8), ref.generate(prompt, 8))
    model.close()
    ref.close()


def test_mismatched_checkpoint_is_rejected(ctx, lq8_lib, oracle, tmp_path):
    import checkpoint as ck
    cfgd = dict(hidden=256, layers=2, n_heads=4, n_kv_heads=2, head_dim=128, inter=512, vocab=1000, tied=0,
                norm_std=0.1, max_pos=4096)
    ref = lq8_lib.Qwen3ForCausalLM(ctx, lq8_lib.make_config(**cfgd), 1234, max_batch=1, ctx_max=64)
    st = os.path.join(str(tmp_path), "m.safetensors")
    _checkpoint(lq8_lib, oracle, ref, cfgd, 1234, st)
    gg = os.path.join(str(tmp_path), "m.gguf")
    ck.pack_safetensors(st, gg, dict(cfgd, eps=float(np.float32(1e-6)), theta=1e6))
    other = lq8_lib.Qwen3ForCausalLM(ctx, lq8_lib.make_config(**dict(cfgd, inter=768)), 1, max_batch=1, ctx_max=64)
    with pytest.raises(ValueError):
        ck.load_gguf(other, gg)
    other.close()
    ref.close()
