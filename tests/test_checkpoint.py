"""The checkpoint packer on the CPU: SafeTensors (bf16) -> Q8_0 GGUF. The host quantizer must
equal the oracle's GGML Q8_0 (and so the device quantizer) bit for bit; the GGUF file must read
back identically with this package's reader and with the independent `gguf` package reader."""
import json
import os

import numpy as np
import pytest

import checkpoint as ck

TINY_HF = {"hidden_size": 256, "num_hidden_layers": 2, "num_attention_heads": 4, "num_key_value_heads": 2,
           "head_dim": 128, "intermediate_size": 512, "vocab_size": 300, "max_position_embeddings": 4096,
           "tie_word_embeddings": False, "rms_norm_eps": 1e-6, "rope_theta": 1000000.0}


def test_quantizer_matches_oracle(oracle, rng):
    x = (rng.standard_normal((37, 256)) * 0.05).astype(np.float32)
    x[3, :32] = 0.0                                   # all-zero block: d = 0
    x[4, :32] = np.linspace(-127, 127, 32)            # amax 127 -> d = 1: halves round away
    x[4, 5], x[4, 6] = 2.5, -2.5
    x[5, 32:64] = 1e-30                               # subnormal-scale block
    for src in (x, oracle.f32_to_bf16(x)):
        qs, d = ck.quantize_q8_0(src)
        oq, od = oracle.q8_0_quantize(oracle.bf16_to_f32(src) if src.dtype == np.uint16 else src)
        assert np.array_equal(qs, oq) and np.array_equal(d, od)
    qs, d = ck.quantize_q8_0(x)
    assert qs[4, 5] == 3 and qs[4, 6] == -3
    blocks = ck.q8_0_to_blocks(qs, d)
    assert np.array_equal(blocks.reshape(37, -1), oracle.q8_0_pack(qs, d).reshape(37, -1))
    q2, d2 = ck.blocks_to_q8_0(blocks, 256)
    assert np.array_equal(q2, qs) and np.array_equal(d2, d)


def _write_hf(tmp_path, cfg_hf, rng, tied=False):
    import torch
    from safetensors.torch import save_file
    H, I, V = cfg_hf["hidden_size"], cfg_hf["intermediate_size"], cfg_hf["vocab_size"]
    Hq, Hkv, D = cfg_hf["num_attention_heads"], cfg_hf["num_key_value_heads"], cfg_hf["head_dim"]

    def t(*shape, std=0.02, base=0.0):
        return torch.from_numpy((base + rng.standard_normal(shape) * std).astype(np.float32)).to(torch.bfloat16)

    sd = {"model.embed_tokens.weight": t(V, H), "model.norm.weight": t(H, base=1.0, std=0.1)}
    if not tied:
        sd["lm_head.weight"] = t(V, H)
    for i in range(cfg_hf["num_hidden_layers"]):
        p = f"model.layers.{i}."
        sd.update({p + "input_layernorm.weight": t(H, base=1.0, std=0.1),
                   p + "post_attention_layernorm.weight": t(H, base=1.0, std=0.1),
                   p + "self_attn.q_proj.weight": t(Hq * D, H), p + "self_attn.k_proj.weight": t(Hkv * D, H),
                   p + "self_attn.v_proj.weight": t(Hkv * D, H), p + "self_attn.o_proj.weight": t(H, Hq * D),
                   p + "self_attn.q_norm.weight": t(D, base=1.0, std=0.1),
                   p + "self_attn.k_norm.weight": t(D, base=1.0, std=0.1),
                   p + "mlp.gate_proj.weight": t(I, H), p + "mlp.up_proj.weight": t(I, H),
                   p + "mlp.down_proj.weight": t(H, I)})
    # two shards, as real checkpoints come
    names = sorted(sd)
    half = len(names) // 2
    paths = []
    for j, part in enumerate((names[:half], names[half:])):
        path = os.path.join(tmp_path, f"model-0000{j + 1}.safetensors")
        save_file({n: sd[n].contiguous() for n in part}, path)
        paths.append(path)
    with open(os.path.join(tmp_path, "config.json"), "w") as f:
        json.dump(dict(cfg_hf, tie_word_embeddings=tied), f)
    return paths, {n: sd[n].view(__import__("torch").int16).numpy().view(np.uint16) for n in sd}


@pytest.mark.parametrize("tied", [False, True])
def test_pack_safetensors_round_trip(tmp_path, oracle, rng, tied):
    paths, sd = _write_hf(str(tmp_path), TINY_HF, rng, tied)
    cfg = ck.config_from_hf(json.load(open(os.path.join(str(tmp_path), "config.json"))))
    out = os.path.join(str(tmp_path), "model-q8_0.gguf")
    ck.pack_safetensors(paths, out, cfg)
    meta, tens = ck.read_gguf(out)
    assert ck.config_from_gguf(meta) == cfg
    assert ("output.weight" in tens) == (not tied)
    linears = {"attn_q": "self_attn.q_proj", "attn_k": "self_attn.k_proj", "attn_v": "self_attn.v_proj",
               "attn_output": "self_attn.o_proj", "ffn_gate": "mlp.gate_proj", "ffn_up": "mlp.up_proj",
               "ffn_down": "mlp.down_proj"}
    norms = {"attn_norm": "input_layernorm", "ffn_norm": "post_attention_layernorm",
             "attn_q_norm": "self_attn.q_norm", "attn_k_norm": "self_attn.k_norm"}
    for i in range(TINY_HF["num_hidden_layers"]):
        for gg, hf in linears.items():
            typ, ne, raw = tens[f"blk.{i}.{gg}.weight"]
            w = sd[f"model.layers.{i}.{hf}.weight"]
            assert typ == ck.GGML_Q8_0 and ne == [w.shape[1], w.shape[0]]
            qs, d = ck.blocks_to_q8_0(np.frombuffer(raw, np.uint8), w.shape[1])
            oq, od = oracle.q8_0_quantize(oracle.bf16_to_f32(w))
            assert np.array_equal(qs, oq) and np.array_equal(d, od), gg
        for gg, hf in norms.items():
            typ, ne, raw = tens[f"blk.{i}.{gg}.weight"]
            assert typ == ck.GGML_BF16 and np.array_equal(np.frombuffer(raw, np.uint16),
                                                          sd[f"model.layers.{i}.{hf}.weight"])
    typ, ne, raw = tens["token_embd.weight"]
    assert typ == ck.GGML_BF16 and ne == [TINY_HF["hidden_size"], TINY_HF["vocab_size"]]
    assert np.array_equal(np.frombuffer(raw, np.uint16).reshape(sd["model.embed_tokens.weight"].shape),
                          sd["model.embed_tokens.weight"])


def test_gguf_readable_by_the_gguf_package(tmp_path, rng):
    """The file parses with llama.cpp's gguf-py reader: same tensors, types, shapes, bytes and
    metadata values."""
    gguf = pytest.importorskip("gguf")
    paths, _ = _write_hf(str(tmp_path), TINY_HF, rng)
    cfg = ck.config_from_hf(json.load(open(os.path.join(str(tmp_path), "config.json"))))
    out = os.path.join(str(tmp_path), "m.gguf")
    ck.pack_safetensors(paths, out, cfg)
    meta, tens = ck.read_gguf(out)
    r = gguf.GGUFReader(out)
    assert {t.name for t in r.tensors} == set(tens)
    for t in r.tensors:
        typ, ne, raw = tens[t.name]
        assert int(t.tensor_type) == typ
        assert [int(v) for v in t.shape] == ne
        assert bytes(np.asarray(t.data).view(np.uint8).ravel()) == bytes(raw), t.name
    assert int(r.fields["qwen3.block_count"].parts[-1][0]) == TINY_HF["num_hidden_layers"]
    assert int(r.fields["qwen3.embedding_length"].parts[-1][0]) == TINY_HF["hidden_size"]
    assert bytes(r.fields["general.architecture"].parts[-1]).decode() == "qwen3"


def test_missing_tensor_is_an_error(tmp_path, rng):
    paths, _ = _write_hf(str(tmp_path), TINY_HF, rng)
    cfg = ck.config_from_hf(TINY_HF)
    cfg["layers"] = 3  # the checkpoint has 2
    with pytest.raises(KeyError):
        ck.pack_safetensors(paths, os.path.join(str(tmp_path), "x.gguf"), cfg)
