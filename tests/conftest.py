"""Shared fixtures. `-m gpu` tests need a B200 and call liblq8.so through its C ABI; the rest
run on CPU (oracle vs golden vectors, host logic, ABI surface)."""
import json
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "qwen-omni-inference-rs_b200")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a); calls liblq8.so")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.lib()
    return O


@pytest.fixture(scope="session")
def lq8_lib():
    import build  # qwen-omni-inference-rs_b200/build.py
    build.build()
    import lq8
    return lq8


@pytest.fixture(scope="session")
def ctx(lq8_lib):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    c = lq8_lib.Context(0)
    yield c
    c.synchronize()


@pytest.fixture
def rng():
    return np.random.default_rng(1234)


def cos_sim(a, b) -> float:
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))


def parity_metrics(got, ref) -> dict:
    """The reference's validation metrics for one output vector (tests/validation.rs:46-67 of
    lluda-inference reports MSE, cosine, max-abs and mean-abs per layer), plus max-abs
    relative to the largest reference magnitude."""
    g = np.asarray(got, dtype=np.float64).ravel()
    r = np.asarray(ref, dtype=np.float64).ravel()
    d = np.abs(g - r)
    return {"cos": cos_sim(g, r), "max_abs": float(d.max()), "max_rel": float(d.max() / (np.abs(r).max() + 1e-300)),
            "mse": float(np.mean(d * d)), "mean_abs": float(d.mean())}


def record(test: str, **fields) -> None:
    """Appends one JSON line of measured parity figures to $LQ_PARITY_LOG (when set), so a GPU
    run keeps the numbers the assertions were made on."""
    path = os.environ.get("LQ_PARITY_LOG")
    if not path:
        return
    with open(path, "a") as f:
        f.write(json.dumps({"test": test, **fields}) + "\n")
