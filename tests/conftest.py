import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
PKG_DIR = os.path.join(ROOT, "tabicl-anywhere_b200")
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def load_package():
    """The package lives in a directory whose name is not an identifier; load it as tabicl_anywhere_b200."""
    if "tabicl_anywhere_b200" in sys.modules:
        return sys.modules["tabicl_anywhere_b200"]
    spec = importlib.util.spec_from_file_location("tabicl_anywhere_b200", os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["tabicl_anywhere_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


tcu = load_package()
from tabicl_anywhere_b200 import synth, tirs  # noqa: E402
import oracle  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libtabicl_b200.so")


def has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device here")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


def to_rows(ref, heads, n, hd):
    """Reference dump keys/values [heads][n][hd] to row-major [n][d] (tests/reference.rs:27-37 reorders to [d][n])."""
    return np.ascontiguousarray(np.asarray(ref, np.float32).reshape(heads, n, hd).transpose(1, 0, 2).reshape(n, heads * hd))


@pytest.fixture(scope="session")
def tiny():
    """The reference's tiny classifier and its golden in-context numbers (tests/golden, from tests/data)."""
    wb = tirs.Bundle(os.path.join(GOLDEN, "tiny-clf.tirs"))
    fx = tirs.Bundle(os.path.join(GOLDEN, "tiny-raw-icl.tirs"))
    m = oracle.model_from_bundle(wb)
    n = fx["train_rep"].shape[0]
    hd = m.d // m.heads
    k = [to_rows(fx[f"icl_k{l}"], m.heads, n, hd) for l in range(m.layers)]
    v = [to_rows(fx[f"icl_v{l}"], m.heads, n, hd) for l in range(m.layers)]
    scales = np.stack([m.query_scale(l, n) for l in range(m.layers)])
    return dict(wb=wb, fx=fx, m=m, n=n, k=k, v=v, scales=scales, path=os.path.join(GOLDEN, "tiny-clf.tirs"),
                test_rep=np.array(fx["test_rep"], np.float32), logits=np.array(fx["logits"], np.float32))
