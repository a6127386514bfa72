"""Text in and out for the Qwen3 runner: the reference's tokenizer wrapper and its text-level
generation loop, host-side.

The reference wraps the Rust crate of HuggingFace `tokenizers` (lluda-inference/src/
tokenizer.rs:1-136); this module wraps the same library's Python binding, so a Qwen3
`tokenizer.json` encodes and decodes to the same ids and text. `generate_text` follows the
reference's `generate` (generate.rs:611-692): clear the KV cache, encode the prompt with special
tokens, prefill, then one decode step per new token until an EOS id or `max_new_tokens`, and
decode prompt + new tokens with special tokens skipped. Token choice runs on the device (the
runner's greedy argmax or its sampling knobs, `Qwen3ForCausalLM.set_sampling`).
"""
from __future__ import annotations

import os
from typing import Iterable, Sequence

import numpy as np

# Qwen3's special ids (tokenizer.rs:13-16): BOS <|endoftext|>, EOS <|im_end|> and <|endoftext|>
QWEN3_BOS = 151643
QWEN3_EOS = (151645, 151643)


class TokenizerError(RuntimeError):
    """A tokenizer file that cannot be loaded, or text/ids the tokenizer rejects
    (LludaError::Tokenizer in error.rs)."""


class Tokenizer:
    """Tokenizer with BOS/EOS ids (tokenizer.rs:17-136)."""

    def __init__(self, hf, bos_token_id: int = QWEN3_BOS, eos_token_ids: Iterable[int] = QWEN3_EOS):
        self._tok = hf
        self._bos = int(bos_token_id)
        self._eos = tuple(int(t) for t in eos_token_ids)

    @classmethod
    def from_file(cls, path: str | os.PathLike, bos_token_id: int = QWEN3_BOS,
                  eos_token_ids: Iterable[int] = QWEN3_EOS) -> "Tokenizer":
        """Load a `tokenizer.json` (tokenizer.rs:44-58); raises TokenizerError if it cannot."""
        try:
            from tokenizers import Tokenizer as HfTokenizer
        except ImportError as e:  # the library is a dependency of this path, not optional
            raise TokenizerError(f"the `tokenizers` library is not installed: {e}") from e
        try:
            hf = HfTokenizer.from_file(os.fspath(path))
        except Exception as e:
            raise TokenizerError(f"cannot load tokenizer {os.fspath(path)!r}: {e}") from e
        return cls(hf, bos_token_id, eos_token_ids)

    def encode(self, text: str, add_special_tokens: bool) -> list[int]:
        """Token ids of `text`; with add_special_tokens the tokenizer's post-processor adds its
        special tokens (tokenizer.rs:76-83)."""
        try:
            return list(self._tok.encode(text, add_special_tokens=add_special_tokens).ids)
        except Exception as e:
            raise TokenizerError(str(e)) from e

    def decode(self, ids: Sequence[int], skip_special_tokens: bool) -> str:
        """Text of `ids` (tokenizer.rs:101-108)."""
        try:
            return self._tok.decode([int(t) for t in ids], skip_special_tokens=skip_special_tokens)
        except Exception as e:
            raise TokenizerError(str(e)) from e

    def vocab_size(self) -> int:
        """Vocabulary size including added tokens (tokenizer.rs:119-121; 151936 for Qwen3)."""
        return int(self._tok.get_vocab_size(with_added_tokens=True))

    def bos_token_id(self) -> int:
        return self._bos

    def eos_token_ids(self) -> tuple[int, ...]:
        return self._eos

    def is_eos(self, token: int) -> bool:
        """generate.rs:691-693."""
        return int(token) in self._eos


def generate_text(model, tokenizer: Tokenizer, prompt: str, max_new_tokens: int, **sampling) -> str:
    """Generate text from `prompt` with `model` (a `lq8.Qwen3ForCausalLM` of batch 1), the
    reference's `generate` (generate.rs:611-661): the KV cache is cleared, the prompt is encoded
    with special tokens and prefilled, each further token is one decode step, generation stops
    at the first EOS id (kept in the ids, then skipped by the decode) or after max_new_tokens
    new tokens. `sampling` (temperature, top_k, top_p, repetition_penalty) is handed to the
    runner's device-side token choice; without it the choice is greedy."""
    if max_new_tokens < 1:
        raise ValueError("max_new_tokens must be >= 1")
    model.clear_kv_cache()
    model.set_batch(1)
    model.set_sampling(**sampling)
    ids = tokenizer.encode(prompt, True)
    if not ids:
        raise TokenizerError("Empty input after tokenization")
    vocab = int(model.cfg.vocab)
    if max(ids) >= vocab:
        raise TokenizerError(f"token id {max(ids)} is outside the model's vocabulary ({vocab})")
    nxt = int(model.prefill(np.asarray(ids, dtype=np.int32))[0])
    ids.append(nxt)
    if tokenizer.is_eos(nxt):
        return tokenizer.decode(ids, True)
    for _ in range(1, max_new_tokens):
        nxt = int(model.decode_step(np.asarray([nxt], dtype=np.int32))[0])
        ids.append(nxt)
        if tokenizer.is_eos(nxt):
            break
    return tokenizer.decode(ids, True)
