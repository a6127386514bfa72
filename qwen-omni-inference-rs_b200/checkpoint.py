"""Checkpoints for the Q8_0 runner: Hugging Face Qwen3 SafeTensors (bf16) -> a Q8_0-packed GGUF
file -> the model's device buffers.

The reference loads bf16 SafeTensors (lluda-inference/src/loader.rs:68-188, tensor names of
model.rs:273-302 and attention.rs/mlp.rs) and names GGUF Q8_0 as its packed on-disk format
(docs/architecture/arch-2026-01-31-qwen3-omni-q8-rust.md:36-38, 278-279). Here a checkpoint is
packed once on the host: every linear is quantized with GGML's Q8_0 rule (the same rule as the
device quantizer, bit for bit), norms and the embedding table stay bf16, and everything is
written as a GGUF v3 file with llama.cpp's qwen3 tensor names and metadata keys. Loading reads
the file (memory-mapped) and writes the model's device buffers: Q8_0 blocks (GGML's 34-byte
block: fp16 scale, then 32 int8) are unpacked on the device into the runner's layout (int8
rows + fp16 scale rows), bf16 tensors are copied. A tied model (no output.weight) gets its LM
head by quantizing the loaded embedding table on the device, as the runner does at creation.

Dense Qwen3 only (the MoE expert tensors are not mapped)."""
from __future__ import annotations

import ctypes as C
import json
import struct

import numpy as np

GGUF_MAGIC = 0x46554747          # "GGUF"
GGUF_VERSION = 3
GGML_F32, GGML_F16, GGML_Q8_0, GGML_BF16 = 0, 1, 8, 30
QK8_0 = 32
Q8_0_BLOCK = 34
ALIGN = 32
# GGUF metadata value types
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)

# per-layer tensors: (HF name, GGUF name, kind for the runner)
_LAYER = [
    ("input_layernorm.weight", "attn_norm.weight", "in_norm"),
    ("self_attn.q_proj.weight", "attn_q.weight", "q"),
    ("self_attn.k_proj.weight", "attn_k.weight", "k"),
    ("self_attn.v_proj.weight", "attn_v.weight", "v"),
    ("self_attn.o_proj.weight", "attn_output.weight", "o"),
    ("self_attn.q_norm.weight", "attn_q_norm.weight", "q_norm"),
    ("self_attn.k_norm.weight", "attn_k_norm.weight", "k_norm"),
    ("post_attention_layernorm.weight", "ffn_norm.weight", "post_norm"),
    ("mlp.gate_proj.weight", "ffn_gate.weight", "gate"),
    ("mlp.up_proj.weight", "ffn_up.weight", "up"),
    ("mlp.down_proj.weight", "ffn_down.weight", "down"),
]
_GLOBAL = [
    ("model.embed_tokens.weight", "token_embd.weight", "embed"),
    ("model.norm.weight", "output_norm.weight", "final_norm"),
    ("lm_head.weight", "output.weight", "lm_head"),
]
_LINEAR = {"q", "k", "v", "o", "gate", "up", "down", "lm_head"}


# ------------------------------------------------------------------------------ Q8_0
def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def quantize_q8_0(x: np.ndarray):
    """GGML Q8_0 of rows x [N][K] (f32, or bf16 bits as uint16), K % 32 == 0: per block of 32,
    d = amax / 127 (f32 division), id = d ? 1/d : 0, q = clamp(round_half_away(x * id), -127,
    127), scale stored as fp16 (round to nearest even). Returns (qs int8 [N][K], d uint16
    [N][K/32] fp16 bits)."""
    x = bf16_to_f32(x) if x.dtype == np.uint16 else np.asarray(x, dtype=np.float32)
    n, k = x.shape
    if k % QK8_0:
        raise ValueError(f"K={k} is not a multiple of {QK8_0}")
    b = x.reshape(n, k // QK8_0, QK8_0)
    amax = np.max(np.abs(b), axis=2)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    v = (b * inv[:, :, None]).astype(np.float32).astype(np.float64)   # exact product, then
    q = np.sign(v) * np.floor(np.abs(v) + 0.5)                         # half away from zero
    q = np.clip(q, -127, 127).astype(np.int8).reshape(n, k)
    return q, d.astype(np.float16).view(np.uint16)


def q8_0_to_blocks(qs: np.ndarray, d: np.ndarray) -> np.ndarray:
    """Runner layout -> GGML blocks [N][K/32][34] (little-endian fp16 scale, then 32 int8)."""
    n, k = qs.shape
    out = np.empty((n, k // QK8_0, Q8_0_BLOCK), dtype=np.uint8)
    out[:, :, :2] = np.ascontiguousarray(d, dtype=np.uint16).view(np.uint8).reshape(n, k // QK8_0, 2)
    out[:, :, 2:] = np.ascontiguousarray(qs, dtype=np.int8).view(np.uint8).reshape(n, k // QK8_0, QK8_0)
    return out


def blocks_to_q8_0(blocks: np.ndarray, k: int):
    """GGML blocks -> (qs int8 [N][K], d uint16 [N][K/32])."""
    b = np.asarray(blocks, dtype=np.uint8).reshape(-1, k // QK8_0, Q8_0_BLOCK)
    d = np.ascontiguousarray(b[:, :, :2]).view(np.uint16).reshape(b.shape[0], k // QK8_0)
    qs = np.ascontiguousarray(b[:, :, 2:]).view(np.int8).reshape(b.shape[0], k)
    return qs, d


# ------------------------------------------------------------------------------ SafeTensors
def read_safetensors(path: str) -> dict:
    """{name: (dtype string, shape, memory-mapped bytes)} of a .safetensors file (an 8-byte
    little-endian header length, a JSON header, then the raw tensor bytes)."""
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    n = int.from_bytes(bytes(mm[:8]), "little")
    header = json.loads(bytes(mm[8:8 + n]))
    base = 8 + n
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        a, b = info["data_offsets"]
        out[name] = (info["dtype"], tuple(info["shape"]), mm[base + a:base + b])
    return out


def _st_array(entry) -> np.ndarray:
    dt, shape, raw = entry
    if dt == "BF16":
        return np.frombuffer(raw, dtype=np.uint16).reshape(shape)
    if dt == "F32":
        return np.frombuffer(raw, dtype=np.float32).reshape(shape)
    if dt == "F16":
        return np.frombuffer(raw, dtype=np.float16).astype(np.float32).reshape(shape)
    raise ValueError(f"unsupported SafeTensors dtype {dt}")


def _to_bf16(a: np.ndarray) -> np.ndarray:
    if a.dtype == np.uint16:
        return a
    bits = np.asarray(a, dtype=np.float32).view(np.uint32)
    return ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)   # bf16.rs:112-131


# ------------------------------------------------------------------------------ GGUF
def _w_str(f, s: str):
    b = s.encode()
    f.write(struct.pack("<Q", len(b)))
    f.write(b)


def _w_value(f, v):
    if isinstance(v, bool):
        f.write(struct.pack("<IB", _BOOL, int(v)))
    elif isinstance(v, int):  # llama.cpp reads counts and sizes as uint32
        if 0 <= v < (1 << 32):
            f.write(struct.pack("<II", _U32, v))
        else:
            f.write(struct.pack("<Iq", _I64, v) if v < 0 else struct.pack("<IQ", _U64, v))
    elif isinstance(v, float):
        f.write(struct.pack("<If", _F32, v))
    elif isinstance(v, str):
        f.write(struct.pack("<I", _STR))
        _w_str(f, v)
    else:
        raise TypeError(f"metadata value {v!r}")


def write_gguf(path: str, metadata: dict, tensors: list):
    """GGUF v3: tensors = [(name, ggml type, ne (innermost first), raw bytes)]; data aligned
    to 32 bytes."""
    infos, off = [], 0
    for name, typ, ne, raw in tensors:
        infos.append((name, typ, ne, off))
        off += (len(raw) + ALIGN - 1) // ALIGN * ALIGN
    with open(path, "wb") as f:
        f.write(struct.pack("<IIQQ", GGUF_MAGIC, GGUF_VERSION, len(tensors), len(metadata)))
        for k, v in metadata.items():
            _w_str(f, k)
            _w_value(f, v)
        for name, typ, ne, o in infos:
            _w_str(f, name)
            f.write(struct.pack("<I", len(ne)))
            f.write(struct.pack(f"<{len(ne)}Q", *ne))
            f.write(struct.pack("<IQ", typ, o))
        pad = (-f.tell()) % ALIGN
        f.write(b"\0" * pad)
        for (_, _, _, raw), (_, _, _, o) in zip(tensors, infos):
            f.write(raw)
            f.write(b"\0" * ((-len(raw)) % ALIGN))


def read_gguf(path: str):
    """(metadata dict, {name: (ggml type, ne, memory-mapped bytes)}) of a GGUF v2/v3 file."""
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    pos = 0

    def take(fmt):
        nonlocal pos
        size = struct.calcsize(fmt)
        v = struct.unpack(fmt, bytes(mm[pos:pos + size]))
        pos += size
        return v if len(v) > 1 else v[0]

    def string():
        nonlocal pos
        n = take("<Q")
        s = bytes(mm[pos:pos + n]).decode()
        pos += n
        return s

    scalar = {_U8: "<B", _I8: "<b", _U16: "<H", _I16: "<h", _U32: "<I", _I32: "<i", _F32: "<f", _BOOL: "<B",
              _U64: "<Q", _I64: "<q", _F64: "<d"}

    def value(t):
        if t == _STR:
            return string()
        if t == _ARR:
            et, n = take("<I"), take("<Q")
            return [value(et) for _ in range(n)]
        v = take(scalar[t])
        return bool(v) if t == _BOOL else v

    magic, version = take("<I"), take("<I")
    if magic != GGUF_MAGIC or version not in (2, 3):
        raise ValueError(f"{path}: not a GGUF v2/v3 file")
    n_t, n_kv = take("<Q"), take("<Q")
    meta = {}
    for _ in range(n_kv):
        k = string()
        meta[k] = value(take("<I"))
    infos = []
    for _ in range(n_t):
        name = string()
        nd = take("<I")
        ne = [take("<Q") for _ in range(nd)]
        typ, off = take("<I"), take("<Q")
        infos.append((name, typ, ne, off))
    align = int(meta.get("general.alignment", ALIGN))
    base = (pos + align - 1) // align * align
    tensors = {}
    for name, typ, ne, off in infos:
        count = int(np.prod(ne))
        if typ == GGML_Q8_0:
            nbytes = count // QK8_0 * Q8_0_BLOCK
        elif typ in (GGML_BF16, GGML_F16):
            nbytes = count * 2
        elif typ == GGML_F32:
            nbytes = count * 4
        else:
            raise ValueError(f"{name}: unsupported ggml type {typ}")
        tensors[name] = (typ, ne, mm[base + off:base + off + nbytes])
    return meta, tensors


# ------------------------------------------------------------------------------ pack / load
def config_from_hf(config_json: dict) -> dict:
    """The runner's config (lq8.make_config keys) from a Hugging Face Qwen3 config.json."""
    c = config_json
    return dict(hidden=c["hidden_size"], layers=c["num_hidden_layers"], n_heads=c["num_attention_heads"],
                n_kv_heads=c["num_key_value_heads"], head_dim=c.get("head_dim", c["hidden_size"] // c["num_attention_heads"]),
                inter=c["intermediate_size"], vocab=c["vocab_size"], max_pos=c.get("max_position_embeddings", 40960),
                tied=1 if c.get("tie_word_embeddings", False) else 0,
                # stored as f32 in the file (llama.cpp's types), and the runner's eps is f32
                eps=float(np.float32(c.get("rms_norm_eps", 1e-6))), theta=float(np.float32(c.get("rope_theta", 1e6))))


def config_from_gguf(meta: dict) -> dict:
    a = meta.get("general.architecture", "qwen3")
    return dict(hidden=int(meta[f"{a}.embedding_length"]), layers=int(meta[f"{a}.block_count"]),
                n_heads=int(meta[f"{a}.attention.head_count"]), n_kv_heads=int(meta[f"{a}.attention.head_count_kv"]),
                head_dim=int(meta[f"{a}.attention.key_length"]), inter=int(meta[f"{a}.feed_forward_length"]),
                vocab=int(meta[f"{a}.vocab_size"]), max_pos=int(meta[f"{a}.context_length"]),
                tied=1 if meta.get("lq8.tied_embeddings", False) else 0,
                eps=float(meta[f"{a}.attention.layer_norm_rms_epsilon"]), theta=float(meta[f"{a}.rope.freq_base"]))


def pack_safetensors(paths, out_path: str, cfg: dict, name: str = "qwen3") -> None:
    """Pack HF Qwen3 SafeTensors shards (bf16/f16/f32) into a Q8_0 GGUF file: the linears as
    Q8_0 (GGML rule), norms and the embedding as bf16. cfg: the runner's config (e.g. from
    config_from_hf)."""
    if isinstance(paths, str):
        paths = [paths]
    src = {}
    for p in paths:
        src.update(read_safetensors(p))
    meta = {
        "general.architecture": "qwen3", "general.name": name, "general.file_type": 7,   # mostly Q8_0
        "general.alignment": ALIGN,
        "qwen3.context_length": int(cfg["max_pos"]), "qwen3.embedding_length": int(cfg["hidden"]),
        "qwen3.block_count": int(cfg["layers"]), "qwen3.feed_forward_length": int(cfg["inter"]),
        "qwen3.attention.head_count": int(cfg["n_heads"]), "qwen3.attention.head_count_kv": int(cfg["n_kv_heads"]),
        "qwen3.attention.key_length": int(cfg["head_dim"]), "qwen3.attention.value_length": int(cfg["head_dim"]),
        "qwen3.rope.freq_base": float(cfg["theta"]), "qwen3.attention.layer_norm_rms_epsilon": float(cfg["eps"]),
        "qwen3.vocab_size": int(cfg["vocab"]), "lq8.tied_embeddings": bool(cfg["tied"]),
    }
    names = [(hf, gg, kind) for hf, gg, kind in _GLOBAL if not (kind == "lm_head" and cfg["tied"])]
    for i in range(int(cfg["layers"])):
        names += [(f"model.layers.{i}.{hf}", f"blk.{i}.{gg}", kind) for hf, gg, kind in _LAYER]
    tensors = []
    for hf, gg, kind in names:
        if hf not in src:
            raise KeyError(f"{hf} missing from the checkpoint")
        a = _st_array(src[hf])
        if kind in _LINEAR:
            qs, d = quantize_q8_0(a)
            tensors.append((gg, GGML_Q8_0, [a.shape[1], a.shape[0]], q8_0_to_blocks(qs, d).tobytes()))
        else:
            b = _to_bf16(a)
            ne = [b.shape[-1]] + ([b.shape[0]] if b.ndim == 2 else [])
            tensors.append((gg, GGML_BF16, ne, np.ascontiguousarray(b).tobytes()))
    write_gguf(out_path, meta, tensors)


def load_gguf(model, path: str) -> None:
    """Write a packed checkpoint into a Qwen3ForCausalLM's device buffers (the model's config
    must match the file's; see config_from_gguf)."""
    import torch

    import lq8
    meta, tens = read_gguf(path)
    fc = config_from_gguf(meta)
    c = model.cfg
    for k in ("hidden", "layers", "n_heads", "n_kv_heads", "head_dim", "inter", "vocab", "tied"):
        if int(getattr(c, k)) != int(fc[k]):
            raise ValueError(f"{path}: {k}={fc[k]} but the model has {getattr(c, k)}")
    ctx = model.ctx
    dev = torch.device("cuda", torch.cuda.current_device())

    def put_bf16(layer, kind, raw):
        ptr, n = model.tensor(layer, kind)
        if len(raw) != 2 * n:
            raise ValueError(f"{kind} of layer {layer}: {len(raw) // 2} values, the model holds {n}")
        h = np.ascontiguousarray(np.frombuffer(raw, dtype=np.uint16))
        ctx.call("lq_memcpy_h2d", C.c_void_p(ptr), h.ctypes.data, h.nbytes)

    def put_q8(layer, kind, ne, raw):
        t = model.linear(layer, kind)
        if (t.k, t.n) != (ne[0], ne[1]):
            raise ValueError(f"{kind} of layer {layer}: file [{ne[1]}][{ne[0]}], model [{t.n}][{t.k}]")
        blocks = torch.from_numpy(np.array(np.frombuffer(raw, dtype=np.uint8))).to(dev)
        ctx.call("lq_q8_0_unpack_blocks", blocks.data_ptr(), t.n, t.k, t.qs, t.d)
        ctx.synchronize()

    def put(layer, gg, kind):
        typ, ne, raw = tens[gg]
        if kind in _LINEAR:
            if typ != GGML_Q8_0:
                raise ValueError(f"{gg}: expected Q8_0 (type {typ})")
            put_q8(layer, kind, ne, raw)
        else:
            if typ != GGML_BF16:
                raise ValueError(f"{gg}: expected BF16 (type {typ})")
            put_bf16(layer, kind, raw)

    put(-1, "token_embd.weight", "embed")
    put(-1, "output_norm.weight", "final_norm")
    if "output.weight" in tens:
        put(-1, "output.weight", "lm_head")
    else:  # tied: the LM head is the Q8_0 of the embedding table, as at creation
        t = model.linear(-1, "lm_head")
        ptr, _ = model.tensor(-1, "embed")
        ctx.call("lq_q8_0_quantize", C.c_void_p(ptr), lq8.DTYPE_BF16, t.n, t.k, t.qs, t.d)
    for i in range(int(c.layers)):
        for _, gg, kind in _LAYER:
            put(i, f"blk.{i}.{gg}", kind)
    ctx.synchronize()
    model.clear_kv_cache()
