"""The C-ABI library builds, loads, and exports every entry point include/lq8.h declares;
failures come back as status codes (no abort). No GPU compute is called here."""
import ctypes as C
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(REPO, "include", "lq8.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int|void\s*\*|const char\s*\*)\s*(lq_\w+)\s*\(", src, flags=re.M)))


def test_header_declares_entry_points():
    fns = header_functions()
    assert len(fns) >= 35
    for must in ("lq_init", "lq_q8_0_quantize", "lq_q8_0_matmul", "lq_q8_0_linear", "lq_attention",
                 "lq_qwen3_decode_step"):
        assert must in fns


def test_library_exports_every_declared_symbol(lq8_lib):
    lib = lq8_lib.load()
    missing = [f for f in header_functions() if not hasattr(lib, f)]
    assert not missing, missing


def test_binding_covers_header(lq8_lib):
    assert set(header_functions()) == set(lq8_lib.SIGNATURES)


def test_abi_version(lq8_lib):
    import re
    hdr = open(os.path.join(REPO, "include", "lq8.h")).read()
    want = int(re.search(r"#define LQ8_ABI_VERSION (\d+)", hdr).group(1))
    assert lq8_lib.load().lq_abi_version() == want == lq8_lib.ABI_VERSION


def test_init_failure_is_a_status_not_an_abort(lq8_lib, monkeypatch):
    lib = lq8_lib.load()
    h = C.c_void_p()
    monkeypatch.setenv("LQ_FAULT", "lq_init")
    assert lib.lq_init(0, C.byref(h)) == -5
    assert b"injected" in lib.lq_last_error(None)
    monkeypatch.delenv("LQ_FAULT")
    assert lib.lq_init(-1, C.byref(h)) != 0
    assert not h.value


def test_null_context_is_rejected(lq8_lib):
    lib = lq8_lib.load()
    assert lib.lq_synchronize(None) == -1
    assert lib.lq_q8_0_quantize(None, None, 0, 1, 32, None, None) == -1


def test_no_gpu_gives_cuda_error(lq8_lib):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = lq8_lib.load()
    h = C.c_void_p()
    rc = lib.lq_init(0, C.byref(h))
    assert rc == -2 and lib.lq_last_error(None)


def test_python_binding_raises_without_library(lq8_lib, monkeypatch, tmp_path):
    monkeypatch.setattr(lq8_lib, "LIB_PATH", str(tmp_path / "missing.so"))
    monkeypatch.setattr(lq8_lib, "_lib", None)
    with pytest.raises(OSError):
        lq8_lib.load()
