"""The Rust binding crate (rust/lluda-cuda-sys, source only: no Rust toolchain here) against the C
ABI: every function include/lq8.h declares appears in src/ffi.rs with the same argument count,
order and types (C -> Rust by the table below), the same return type, and every struct the
ABI passes has the same fields in the same order with the same types. Also checks that
build.rs compiles every CUDA source of the library for sm_100a."""
import os
import re

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CRATE = os.path.join(REPO, "rust", "lluda-cuda-sys")

SCALAR = {"int": "c_int", "int64_t": "i64", "int32_t": "i32", "uint64_t": "u64", "size_t": "usize",
          "double": "f64", "float": "f32", "uint8_t": "u8", "int8_t": "i8", "uint16_t": "u16", "void": "c_void",
          "char": "c_char", "lq_dtype": "c_int", "lq_ctx": "LqCtx", "lq_model": "LqModel", "lq_comm": "LqComm",
          "lq_q8_tensor": "LqQ8Tensor", "lq_qwen3_config": "LqQwen3Config", "lq_moe_experts": "LqMoeExperts",
          "lq_sampling": "LqSampling"}
RUST_ALIAS = {"LqDtype": "c_int"}


def c_to_rust(ctype: str) -> str:
    t = " ".join(ctype.split())
    const = t.startswith("const ")
    if const:
        t = t[len("const "):]
    stars = t.count("*")
    base = SCALAR[t.replace("*", "").strip()]
    if stars == 0:
        return base
    first = "*const " if const else "*mut "
    return first + base if stars == 1 else "*mut " + first + base


def norm_rust(t: str) -> str:
    t = " ".join(t.split())
    for a, b in RUST_ALIAS.items():
        t = re.sub(rf"\b{a}\b", b, t)
    return t


def header():
    src = open(os.path.join(REPO, "include", "lq8.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    fns = {}
    for ret, name, args in re.findall(r"^\s*(int|void\s*\*|const char\s*\*)\s*(lq_\w+)\s*\(([^;]*?)\)\s*;", src,
                                      flags=re.M | re.S):
        args = " ".join(args.split())
        types = []
        if args and args != "void":
            for a in args.split(","):
                m = re.match(r"(.*?)(\w+)$", a.strip())
                types.append(c_to_rust(m.group(1)))
        fns[name] = (c_to_rust(ret), types)
    structs = {}
    for body, name in re.findall(r"typedef struct(?: \w+)? \{(.*?)\} (\w+);", src, flags=re.S):
        fields = []
        for line in body.split(";"):
            line = " ".join(line.split())
            if not line:
                continue
            m = re.match(r"(.*?)(\w+(?:\s*,\s*\w+)*)$", line)
            ty = m.group(1).strip()
            for nm in m.group(2).split(","):
                fields.append((nm.strip(), c_to_rust(ty)))
        structs[name] = fields
    return fns, structs


def rust():
    src = open(os.path.join(CRATE, "src", "ffi.rs")).read()
    block = src[src.index('extern "C" {'):]
    fns = {}
    for name, args, ret in re.findall(r"pub fn (lq_\w+)\((.*?)\)\s*->\s*([^;]+);", block, flags=re.S):
        types = [norm_rust(a.split(":", 1)[1]) for a in re.split(r",\s*(?=\w+\s*:)", args.strip()) if a.strip()]
        fns[name] = (norm_rust(ret), types)
    structs = {}
    for name, body in re.findall(r"pub struct (Lq\w+) \{(.*?)\}", src, flags=re.S):
        structs[name] = [(f.strip(), norm_rust(t)) for f, t in re.findall(r"pub (\w+):\s*([^,\n]+),", body)]
    return fns, structs


def test_every_header_function_has_a_matching_rust_declaration():
    hf, _ = header()
    rf, _ = rust()
    assert len(hf) >= 50
    assert set(hf) == set(rf), (sorted(set(hf) - set(rf)), sorted(set(rf) - set(hf)))
    for name, (ret, args) in hf.items():
        rret, rargs = rf[name]
        assert rret == ret, (name, rret, ret)
        assert rargs == args, (name, rargs, args)


def test_abi_structs_match():
    _, hs = header()
    _, rs = rust()
    pairs = {"lq_q8_tensor": "LqQ8Tensor", "lq_sampling": "LqSampling", "lq_moe_experts": "LqMoeExperts",
             "lq_qwen3_config": "LqQwen3Config"}
    for c_name, r_name in pairs.items():
        assert hs[c_name] == rs[r_name], (c_name, hs[c_name], rs[r_name])


def test_constants_match_header():
    hdr = open(os.path.join(REPO, "include", "lq8.h")).read()
    ffi = open(os.path.join(CRATE, "src", "ffi.rs")).read()
    abi = re.search(r"#define LQ8_ABI_VERSION (\d+)", hdr).group(1)
    assert re.search(rf"pub const LQ8_ABI_VERSION: c_int = {abi};", ffi)
    for name, val in re.findall(r"(LQ_(?:OK|ERR_\w+|DTYPE_\w+))\s*=\s*(-?\d+)", hdr):
        assert re.search(rf"pub const {name}: \w+ = {val};", ffi), name


def test_build_script_compiles_every_source_for_sm_100a():
    build = open(os.path.join(CRATE, "build.rs")).read()
    import build as lq8_build  # qwen-omni-inference-rs_b200/build.py
    listed = re.findall(r'"(lq8_\w+\.cu)"', build)
    assert sorted(listed) == sorted(lq8_build.SOURCES)
    assert "arch=compute_100a,code=sm_100a" in build
