"""The column and row stages on the device (the AttendCached `rows` hook, src/predict.rs:282-372, 642-652), through the
C ABI, against the oracle (pinned to the reference's golden dump) and against PyTorch's own numbers in that dump.

Bars: test embeddings and row representations within 5e-5 (tests/reference.rs:148 for the same dump), raw decoder
scores within 5e-5 per cached stage, class probabilities within 1e-5. A missing cell (-100) keeps a magnitude near
100 through the column stage's residual stream, where one f32 step is 7.6e-6: there the token bar is 5e-5 times the
token's magnitude (relative 5e-7).
"""
import numpy as np
import pytest

from conftest import synth, tcu
import oracle

pytestmark = pytest.mark.gpu

TINY = 5e-5
STAGE = 5e-5
PROBA = 1e-5


def softmax(x, t=0.9):
    z = (x - x.max(1, keepdims=True)) / t
    e = np.exp(z)
    return e / e.sum(1, keepdims=True)


@pytest.fixture(scope="module")
def gpu():
    g = tcu.Gpu(0)
    yield g
    g.close()


def assert_tokens_close(got, want):
    err = np.abs(got - want) / np.maximum(1.0, np.abs(want))
    i = np.unravel_index(np.argmax(err), err.shape)
    assert err[i] < TINY, (err[i], i, float(want[i]), float(got[i]))


def _device_stages(vm, x, e, cls):
    """embed then represent on device buffers (queued on the library's own stream: synchronised before torch reads
    the results); returns (tokens, representations)."""
    import torch
    n, feats = x.shape
    xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    tok = torch.empty((n, cls + feats, e), device="cuda")
    rep = torch.empty((n, cls * e), device="cuda")
    torch.cuda.synchronize()
    vm.embed_device(xd.data_ptr(), n, tok.data_ptr())
    vm.gpu.sync()
    tok_h = tok.cpu().numpy()
    vm.represent_device(tok.data_ptr(), n, rep.data_ptr())
    vm.gpu.sync()
    return tok_h, rep.cpu().numpy()


def test_golden_tiny_classifier(gpu, tiny):
    """The dump's normalised test rows through the device's column, row and in-context stages: PyTorch's test
    embeddings, row representations and logits (tests/reference.rs:96-116)."""
    t = tiny
    m, rm = t["m"], t["rm"]
    w = tcu.GpuWeights.from_bundle(gpu, t["path"])
    assert w.rows_shape["e"] == rm.e and w.rows_shape["cls"] == rm.cls
    layers = [oracle.pack_layer(1, m.d, t["k"][l], t["v"][l], 48) for l in range(m.layers)]
    feats = t["x_test"].shape[1]
    vm = tcu.VramModel.from_parts(w, [t["n"], feats, 3, 48, 1, 1, 1], t["n"], 3, t["scales"], layers, col_kv=t["col_kv"])
    tok, rep = _device_stages(vm, t["x_test"], rm.e, rm.cls)
    assert np.abs(tok[:, rm.cls:] - t["test_emb"][:, rm.cls:]).max() < TINY
    assert np.array_equal(tok[:, :rm.cls], oracle.embed(rm, t["x_test"], t["col_kv"])[:, :rm.cls])
    assert np.abs(rep - t["test_rep"]).max() < TINY
    got = vm.rows(t["x_test"], 3)
    want = oracle.in_context(m, 1, layers, t["scales"], t["n"], 48, oracle.represent(rm, oracle.embed(rm, t["x_test"], t["col_kv"])), 3)
    assert np.abs(got - want).max() < STAGE
    assert np.abs(got - t["logits"]).max() < 1e-4  # i16 cache against PyTorch's f32 numbers
    vm.free(), w.free()


def _full(gpu, feats, n, kv, seed, digits=1, **over):
    cfg = synth.config("full", icl_num_blocks=2, **over)
    wt = synth.weights(cfg, seed=seed, std=0.05)
    shape, rshape = synth.icl_shape(cfg), synth.rows_shape(cfg)
    w = tcu.GpuWeights.from_tensors(gpu, shape, wt, rows_shape=rshape, for_fit=True)
    m = oracle.Model({k: v for k, v in wt.items() if k.startswith("icl_predictor.")}, cfg["icl_nhead"], 2, cfg["max_classes"])
    rm = oracle.RowsModel({k: v for k, v in wt.items() if k.startswith(("col_embedder.", "row_interactor."))}, cfg)
    h = synth.row_reps(n, m.d, seed + 1)
    layers, scales = oracle.icl_fit(m, h, synth.labels(n, 10, seed + 2), 256, kv)
    ck = synth.col_kv(feats, rshape["col_blocks"], rshape["e"], rshape["inds"], seed + 3, digits)
    vm = tcu.VramModel.from_parts(w, [n, feats, 10, 256, kv, digits, 1], n, 10, scales, layers, col_kv=ck)
    return w, vm, m, rm, layers, scales, ck


@pytest.mark.parametrize("rows", [1, 9, 130])
def test_full_size_stages(gpu, rows):
    """The full-size architecture (column width 128, 128 inducing points, 3 ISABs of 4 heads; 3 row blocks of 8
    heads, 4 class tokens, rotary positions) over 100 features, 5% of the cells missing."""
    feats, n, kv = 100, 700, 1
    w, vm, m, rm, layers, scales, ck = _full(gpu, feats, n, kv, seed=200 + rows)
    x = synth.features(rows, feats, 300 + rows, missing=0.05)
    tok, rep = _device_stages(vm, x, rm.e, rm.cls)
    want_tok = oracle.embed(rm, x, ck)
    assert_tokens_close(tok, want_tok)
    want_rep = oracle.represent(rm, want_tok)
    assert np.abs(rep - want_rep).max() < TINY, np.abs(rep - want_rep).max()
    got = vm.rows(x, 10)
    want = oracle.in_context(m, kv, layers, scales, n, 256, want_rep, 10)
    assert np.abs(got - want).max() < STAGE, np.abs(got - want).max()
    assert np.abs(softmax(got) - softmax(want)).max() < PROBA
    vm.free(), w.free()


def test_label_digits_are_averaged(gpu):
    """Several label digits: the column stage runs once per digit's cache and the cells are averaged
    (src/predict.rs:326-346)."""
    feats, n = 12, 300
    w, vm, m, rm, layers, scales, ck = _full(gpu, feats, n, 2, seed=410, digits=3)
    x = synth.features(20, feats, 411, missing=0.1)
    tok, rep = _device_stages(vm, x, rm.e, rm.cls)
    want_tok = oracle.embed(rm, x, ck, digits=3)
    assert_tokens_close(tok, want_tok)
    assert np.abs(rep - oracle.represent(rm, want_tok)).max() < TINY
    vm.free(), w.free()


def test_long_rows_keep_keys_in_global_memory(gpu):
    """500 features (BASELINE config 5's width): 504 tokens per row, too many for the row attention's shared memory;
    its keys and values are read from global memory instead."""
    feats, n = 500, 300
    w, vm, m, rm, layers, scales, ck = _full(gpu, feats, n, 1, seed=420)
    x = synth.features(3, feats, 421, missing=0.05)
    tok, rep = _device_stages(vm, x, rm.e, rm.cls)
    want_tok = oracle.embed(rm, x, ck)
    assert_tokens_close(tok, want_tok)
    assert np.abs(rep - oracle.represent(rm, want_tok)).max() < TINY
    vm.free(), w.free()


def test_rows_declines_without_column_stages(gpu, tiny):
    """Weights without the column and row stages, or a cache without col_kv: the hook declines (None), the caller's
    CPU path answers (src/predict.rs:58-61)."""
    t = tiny
    m = t["m"]
    cfg_shape = dict(d=m.d, heads=m.heads, layers=m.layers, ff=m.ff, hid=m.hid, dec_ff=m.dff, outs=m.outs, max_classes=10)
    w = tcu.GpuWeights.from_tensors(gpu, cfg_shape, {n: np.asarray(t["wb"][n]) for n in t["wb"].names() if n.startswith("icl_")})
    assert w.rows_shape is None
    layers = [oracle.pack_layer(0, m.d, t["k"][l], t["v"][l], 48) for l in range(m.layers)]
    feats = t["x_test"].shape[1]
    vm = tcu.VramModel.from_parts(w, [t["n"], feats, 3, 48, 0, 1, 1], t["n"], 3, t["scales"], layers)
    assert vm.rows(t["x_test"], 3) is None
    w2 = tcu.GpuWeights.from_bundle(gpu, t["path"])
    vm2 = tcu.VramModel.from_parts(w2, [t["n"], feats, 3, 48, 0, 1, 1], t["n"], 3, t["scales"], layers)
    assert vm2.rows(t["x_test"], 3) is None  # no col_kv
    vm.free(), vm2.free(), w.free(), w2.free()

