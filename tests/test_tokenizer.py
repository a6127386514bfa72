"""Host-side text in/out (qwen-omni-inference-rs_b200/tokenizer.py) against the reference's
tokenizer tests (tokenizer.rs:138-260) and generate loop (generate.rs:611-692).

The reference's tests load the Qwen3 tokenizer.json, which is not in this repository; these
build a byte-level BPE tokenizer of the same kind in a temporary directory (the 256 byte
symbols, no merges, Qwen's special tokens, BOS added by the post-processor), so every string
round-trips. The generate loop runs against a scripted stand-in for the device runner, which
records the calls the loop makes."""
import numpy as np
import pytest

tokenizers = pytest.importorskip("tokenizers")

import tokenizer as T  # qwen-omni-inference-rs_b200/tokenizer.py

BOS, IM_START, IM_END = 256, 257, 258


def _hf(with_bos=True):
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers, processors
    alphabet = sorted(pre_tokenizers.ByteLevel.alphabet())
    tok = Tokenizer(models.BPE(vocab={ch: i for i, ch in enumerate(alphabet)}, merges=[]))
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    tok.decoder = decoders.ByteLevel()
    tok.add_special_tokens(["<|endoftext|>", "<|im_start|>", "<|im_end|>"])
    if with_bos:
        tok.post_processor = processors.TemplateProcessing(single="<|endoftext|> $A",
                                                          special_tokens=[("<|endoftext|>", BOS)])
    return tok


@pytest.fixture
def tok_path(tmp_path):
    p = tmp_path / "tokenizer.json"
    _hf().save(str(p))
    return p


@pytest.fixture
def tok(tok_path):
    return T.Tokenizer.from_file(tok_path, BOS, [IM_END, BOS])


def test_from_file_missing_is_an_error(tmp_path):
    with pytest.raises(T.TokenizerError):
        T.Tokenizer.from_file(tmp_path / "missing.json")


def test_load_ids_and_vocab(tok):
    assert tok.vocab_size() == 259
    assert tok.bos_token_id() == BOS
    assert tok.eos_token_ids() == (IM_END, BOS)
    assert T.QWEN3_BOS == 151643 and T.QWEN3_EOS == (151645, 151643)


def test_encode_decode_roundtrip(tok):
    text = "Hello, world!"
    ids = tok.encode(text, False)
    assert ids and max(ids) < 256
    assert tok.decode(ids, False) == text


def test_encode_with_special_tokens_adds_bos(tok):
    plain = tok.encode("Test", False)
    special = tok.encode("Test", True)
    assert special == [BOS] + plain


def test_decode_skip_special_tokens(tok):
    ids = tok.encode("Hello", True)
    assert tok.decode(ids, True) == "Hello"
    assert tok.decode(ids, False) == "<|endoftext|>Hello"


@pytest.mark.parametrize("text", ["你好世界", "Hello 👋 World 🌍", "こんにちは"])
def test_unicode_roundtrip(tok, text):
    assert tok.decode(tok.encode(text, False), False) == text


def test_is_eos(tok):
    assert tok.is_eos(IM_END) and tok.is_eos(BOS)
    assert not tok.is_eos(IM_START) and not tok.is_eos(65)


class _Cfg:
    vocab = 259


class ScriptedModel:
    """Stand-in for lq8.Qwen3ForCausalLM: returns scripted next tokens and records calls."""

    cfg = _Cfg()

    def __init__(self, script):
        self.script = list(script)
        self.calls = []

    def clear_kv_cache(self):
        self.calls.append(("clear",))

    def set_batch(self, b):
        self.calls.append(("batch", b))

    def set_sampling(self, **cfg):
        self.calls.append(("sampling", cfg))

    def prefill(self, ids):
        self.calls.append(("prefill", np.asarray(ids).tolist()))
        return np.array([self.script.pop(0)], np.int32)

    def decode_step(self, ids):
        self.calls.append(("decode", np.asarray(ids).tolist()))
        return np.array([self.script.pop(0)], np.int32)


def test_generate_stops_at_eos_and_skips_special_tokens(tok):
    prompt = "Hi"
    pids = tok.encode(prompt, True)
    new = tok.encode(" there", False)
    m = ScriptedModel(new + [IM_END, 65, 66])
    out = T.generate_text(m, tok, prompt, 16, temperature=0.7, top_k=5)
    assert out == "Hi there"
    assert m.calls[0] == ("clear",) and m.calls[1] == ("batch", 1)
    assert m.calls[2] == ("sampling", {"temperature": 0.7, "top_k": 5})
    assert m.calls[3] == ("prefill", pids)
    # each decode step feeds the previous token; none after the EOS
    fed = [c[1][0] for c in m.calls if c[0] == "decode"]
    assert fed == new
    assert m.script == [65, 66]


def test_generate_respects_max_new_tokens(tok):
    m = ScriptedModel(tok.encode("ABCDE", False))
    assert T.generate_text(m, tok, "x", 3) == "xABC"
    assert sum(c[0] == "decode" for c in m.calls) == 2
    assert ("sampling", {}) in m.calls  # greedy unless asked otherwise


def test_generate_eos_at_prefill(tok):
    m = ScriptedModel([BOS])
    assert T.generate_text(m, tok, "abc", 8) == "abc"
    assert not any(c[0] == "decode" for c in m.calls)


def test_generate_rejects_empty_and_out_of_vocab(tmp_path):
    p = tmp_path / "t.json"
    _hf(with_bos=False).save(str(p))
    bare = T.Tokenizer.from_file(p, BOS, [IM_END])
    with pytest.raises(T.TokenizerError, match="Empty input"):
        T.generate_text(ScriptedModel([1]), bare, "", 4)

    class Small(ScriptedModel):
        class cfg:
            vocab = 50
    assert bare.encode("z", False)[0] >= 50
    with pytest.raises(T.TokenizerError, match="outside the model's vocabulary"):
        T.generate_text(Small([1]), bare, "z", 4)
    with pytest.raises(ValueError):
        T.generate_text(ScriptedModel([1]), bare, "a", 0)
