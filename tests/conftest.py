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


def golden_col_kv(fx, rm, heads):
    """The reference dump's column-stage keys/values (col_k{b}, col_v{b}: [columns][heads][inducing][head width],
    class-token columns first) as a fitted bundle's col_kv stores them (fit.rs:230): [features][1][blocks][2][e][inds]
    (tests/reference.rs:56-72 reorders the same way)."""
    feats = fx["x_test"].shape[1]
    e, inds = rm.e, rm.inds
    ck = np.zeros((feats, 1, rm.ncol, 2, e, inds), np.float32)
    for b in range(rm.ncol):
        for which, kind in enumerate(("col_k", "col_v")):
            r = np.asarray(fx[f"{kind}{b}"], np.float32)
            for g in range(feats):
                ck[g, 0, b, which] = r[g + rm.cls].transpose(0, 2, 1).reshape(e, inds)
    return ck


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
    rm = oracle.rows_model_from_bundle(wb)
    cfg = __import__("json").loads(bytes(wb["config.json"]).decode())
    return dict(wb=wb, fx=fx, m=m, n=n, k=k, v=v, scales=scales, path=os.path.join(GOLDEN, "tiny-clf.tirs"),
                test_rep=np.array(fx["test_rep"], np.float32), logits=np.array(fx["logits"], np.float32),
                rm=rm, col_kv=golden_col_kv(fx, rm, cfg["col_nhead"]), x_test=np.array(fx["x_test"], np.float32),
                test_emb=np.array(fx["test_emb"], np.float32))
