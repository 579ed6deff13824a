"""Shared fixtures. GPU tests are marked `gpu`; everything else runs on a CPU-only host."""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "ane-infer_b200")
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def load_pkg():
    """Import the ane-infer_b200 directory as the package `ane_infer_b200`."""
    name = "ane_infer_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libab2.so")


@pytest.fixture(scope="session")
def pkg():
    return load_pkg()


@pytest.fixture(scope="session")
def synth(pkg):
    from ane_infer_b200 import synth as s
    return s


@pytest.fixture(scope="session")
def oracle():
    import oracle as o
    o.lib()
    return o


@pytest.fixture(scope="session")
def tiny_gguf(synth):
    return synth.build_model_gguf(synth.tiny_shape(), seed=0)


@pytest.fixture(scope="session")
def tiny_model(oracle, tiny_gguf):
    return oracle.Model(tiny_gguf, ctx_cap=4096)


@pytest.fixture(scope="session")
def cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def argmax_consistent(got_idx: int, ref_logits, got_logits) -> bool:
    """The device's greedy pick equals the reference's, or the two candidates are closer in
    the reference logits than the observed logit error (a near-tie the tolerance allows)."""
    ref = np.asarray(ref_logits, dtype=np.float64)
    want = int(np.argmax(ref))
    if got_idx == want or (ref[got_idx] == ref[want]):
        return True
    err = float(np.max(np.abs(np.asarray(got_logits, dtype=np.float64) - ref)))
    return ref[want] - ref[got_idx] <= 2.0 * err


def rel_err(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def attn_mma_plan(B, Hkv, max_len, sms):
    """The tensor-core launcher's choice between chunk splits and the balanced partition
    (attn_mma_chunk, sk_per and the cost comparison in attn_mma.cu's launch_mma_t)."""
    kT, kmax = 64, 64
    pairs = B * Hkv
    best = None
    c = (max(4 * kT, -(-max_len // kmax)) + kT - 1) // kT * kT
    while True:
        s = -(-max_len // c)
        cost = -(-(pairs * s) // sms) * (c // kT + 1)
        if best is None or cost < best[0]:
            best = (cost, c)
        if s == 1:
            break
        c += kT
    chunk = best[1]
    splits = -(-max_len // chunk)
    if splits <= 1:
        return "chunk"
    items = pairs * splits
    grid = min(items, sms)
    mt = -(-max_len // kT)
    per = max(-(-(pairs * mt) // sms), (mt + kmax - 2) // (kmax - 1), 4)
    chunk_cost = -(-items // grid) * (chunk // kT + 1)
    return "balanced" if per + -(-per // mt) + 1 < chunk_cost else "chunk"
