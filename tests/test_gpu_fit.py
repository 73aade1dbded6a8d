"""Fitting on the device (src/fit.rs:285-752): the column stage (298-481), the row stage (487-540) and the
in-context stage per node of the class tree (577-747), through the C ABI, against the oracle and the reference's
golden dump; the fit::Attend hooks (src/fit.rs:25-74) one by one; the fitted member written as fit::raw_entries
names its tensors (224-241) and read back.

Bars: the reference's own test compares its CPU fit with PyTorch at TINY = 5e-5 for the column cache and the
training rows' representations, 2.5 x TINY for the in-context keys and values (tests/reference.rs:79-99, 145-148).
The same bars hold here against the golden dump; against the oracle on seeded models of the full shape the column
cache (values of order 1) is held to 1e-4 and the representations to 1e-4 (more rounding steps in longer sums).
"""
import numpy as np
import pytest

from conftest import GOLDEN, synth, tcu, tirs, to_rows
import oracle

pytestmark = pytest.mark.gpu

TINY = 5e-5


def _close(a, b, bar):
    """Within bar of b, relative to b's magnitude where that is past 1 (cells hold the -100 of missing values)."""
    return np.abs(a - b).max() < bar * max(1.0, float(np.abs(b).max()))


@pytest.fixture(scope="module")
def gpu():
    g = tcu.Gpu(0)
    yield g
    g.close()


@pytest.fixture(scope="module")
def golden(gpu):
    import os
    path = os.path.join(GOLDEN, "tiny-clf.tirs")
    w = tcu.GpuWeights.from_bundle(gpu, path, for_fit=True)
    yield w
    w.free()


def test_golden_fit_on_the_device(golden, tiny):
    """The whole fit of the reference's tiny classifier from the dump's normalised training rows: the column cache,
    every layer's in-context keys and values and the query scales, as the reference's own test checks them."""
    t, fx = tiny, tiny["fx"]
    x, y = np.array(fx["x_train"], np.float32), np.array(fx["y_train"], np.float32)
    classes = t["logits"].shape[1]
    mb, ent = tcu.fit_raw(golden, x, y, classes, chunk=48, kv=tcu.KV_F32, prefix="m0/")
    assert np.abs(ent["m0/col_kv"] - t["col_kv"]).max() < TINY
    m = t["m"]
    for l in range(m.layers):
        k, v = oracle.layer_rows(0, m.d, ent[f"m0/n0_kv{l}"], t["n"], 48)
        assert np.abs(k - t["k"][l]).max() < 2.5 * TINY, l
        assert np.abs(v - t["v"][l]).max() < 2.5 * TINY, l
    assert np.array_equal(ent["m0/n0_scale"], t["scales"])
    assert ent["m0/meta"].tolist() == [t["n"], x.shape[1], classes, 48, tcu.KV_F32, 1, 1]
    # and the member it leaves predicts the dump's logits from the normalised test rows
    got = mb.rows(t["x_test"])
    assert np.abs(got - t["logits"]).max() < TINY
    mb.free()


@pytest.fixture(scope="module")
def full(gpu):
    cfg = synth.config("full")
    wt = synth.weights(cfg, seed=5)
    w = tcu.GpuWeights.from_tensors(gpu, synth.icl_shape(cfg), wt, rows_shape=synth.rows_shape(cfg), for_fit=True)
    rm = oracle.RowsModel({k: v for k, v in wt.items() if k.startswith(("col_embedder.", "row_interactor."))}, cfg)
    m = oracle.Model({k: v for k, v in wt.items() if k.startswith("icl_predictor.")}, cfg["icl_nhead"],
                     cfg["icl_num_blocks"], cfg["max_classes"])
    yield dict(cfg=cfg, w=w, rm=rm, m=m)
    w.free()


@pytest.mark.parametrize("n,features", [(300, 12), (97, 5)])
def test_columns_and_rows_match_oracle(full, n, features):
    """The column and row stages of the full-shape model against the oracle (fewer training rows than inducing
    points in the second case)."""
    t = full
    x = synth.features(n, features, 21 + n, missing=0.05)
    y = synth.labels(n, 10, 22 + n).astype(np.float32)
    mb, ent = tcu.fit_raw(t["w"], x, y, 10, chunk=64, kv=tcu.KV_I16)
    ck, tok = oracle.fit_columns(t["rm"], x, y, 64)
    assert np.abs(ent["col_kv"] - ck).max() < 1e-4
    rep = oracle.represent(t["rm"], tok)
    # the in-context stage sees the representations: its first layer's keys (f32 widened from i16) follow them
    layers, scales = oracle.icl_fit(t["m"], rep, y, 64, tcu.KV_I16)
    assert np.allclose(ent["n0_scale"], scales, rtol=0, atol=1e-6)
    k, v = oracle.layer_rows(tcu.KV_I16, t["m"].d, ent["n0_kv0"], n, 64)
    k0, v0 = oracle.layer_rows(tcu.KV_I16, t["m"].d, layers[0], n, 64)
    assert np.abs(k - k0).max() < 1e-3 and np.abs(v - v0).max() < 1e-3
    mb.free()


def _tiny_synth(gpu, regression=False):
    cfg = synth.config("tiny", regression=regression)
    wt = synth.weights(cfg, seed=13, std=0.08)
    w = tcu.GpuWeights.from_tensors(gpu, synth.icl_shape(cfg), wt, rows_shape=synth.rows_shape(cfg), for_fit=True)
    rm = oracle.RowsModel({k: v for k, v in wt.items() if k.startswith(("col_embedder.", "row_interactor."))}, cfg)
    return cfg, w, rm


def test_many_classes_fit_label_digits(gpu):
    """A table of more classes than the model tells apart: the column stage runs once per label digit
    (fit.rs:316-324) and the class tree's nodes are fitted on their own rows."""
    cfg, w, rm = _tiny_synth(gpu)
    n, features, classes = 400, 6, 37
    x = synth.features(n, features, 31, missing=0.1)
    y = synth.labels(n, classes, 32).astype(np.float32)
    plan = tcu.Plan.new(cfg["max_classes"], y, classes)
    assert len(plan.bases) > 1 and len(plan.nodes) > 1
    mb, ent = tcu.fit_raw(w, x, y, classes, chunk=48, kv=tcu.KV_F32)
    ck, _ = oracle.fit_columns(rm, x, y, 48, bases=plan.bases)
    assert np.abs(ent["col_kv"] - ck).max() < 1e-4
    assert ent["tree"].tolist() == plan.tree(n).tolist()
    assert mb.n_nodes == len(plan.nodes) and mb.classes == classes
    mb.free(), w.free()


def test_regression_fit(gpu):
    cfg, w, rm = _tiny_synth(gpu, regression=True)
    n, features = 250, 7
    x = synth.features(n, features, 41)
    y = np.random.default_rng(42).standard_normal(n).astype(np.float32)
    mb, ent = tcu.fit_raw(w, x, y, w.shape["outs"], chunk=32, kv=tcu.KV_F32)
    ck, _ = oracle.fit_columns(rm, x, y, 32)
    assert np.abs(ent["col_kv"] - ck).max() < 1e-4
    mb.free(), w.free()


def test_fit_hooks_one_by_one(full):
    """fit::Attend's columns, rows and in_context hooks with host arrays, each against the oracle's same step."""
    t = full
    rm, m = t["rm"], t["m"]
    fit = tcu.CudaFit(t["w"])
    n, features = 200, 9
    x = synth.features(n, features, 51, missing=0.05)
    y = synth.labels(n, 10, 52).astype(np.float32)
    assert fit.column_batch(n) >= features and fit.row_batch(features) >= n
    cells = oracle.fit_cells(rm, x, y)
    rec = fit.columns(cells, oracle.ind_queries(rm, n))
    ck, tok = oracle.fit_columns(rm, x, y, 64)
    assert np.abs(rec - ck[:, 0]).max() < 1e-4
    assert _close(cells, tok[:, rm.cls:], 1e-5)
    reps = fit.rows(cells)
    want = oracle.represent(rm, tok)
    assert _close(reps, want, 1e-4)
    h = oracle.add_y(m, want, y)
    scales = np.stack([m.query_scale(l, n) for l in range(m.layers)])
    got = {}
    assert fit.in_context(h, scales, lambda l, k, v: got.__setitem__(l, (k, v)))
    layers, _ = oracle.icl_fit(m, want, y, 256, 0)
    assert sorted(got) == list(range(m.layers))
    for l in range(m.layers):
        k0, v0 = oracle.layer_rows(0, m.d, layers[l], n, 256)
        assert np.abs(got[l][0] - k0).max() < 1e-4 and np.abs(got[l][1] - v0).max() < 1e-4, l


def test_fit_hook_sink_failure_stops_the_pass(full):
    fit = tcu.CudaFit(full["w"])
    m = full["m"]
    h = synth.row_reps(40, m.d, 61)
    scales = np.stack([m.query_scale(l, 40) for l in range(m.layers)])
    seen = []

    def sink(l, k, v):
        seen.append(l)
        if l == 1:
            raise ValueError("sink full")

    with pytest.raises(ValueError, match="sink full"):
        fit.in_context(h, scales, sink)
    assert seen == [0, 1]


def test_written_fit_reads_back(golden, tiny, tmp_path):
    """The entries of a device fit, written with the weights' tensors as one bundle, load as a member that answers
    bit for bit as the one fitted, and their names and sizes are fit::raw_entries'."""
    t, fx = tiny, tiny["fx"]
    x, y = np.array(fx["x_train"], np.float32), np.array(fx["y_train"], np.float32)
    classes = t["logits"].shape[1]
    mb, ent = tcu.fit_raw(golden, x, y, classes, chunk=48, kv=tcu.KV_I8, prefix="m0/")
    plan = tcu.Plan.new(golden.shape["max_classes"], y, classes)
    names = tcu.raw_entries(golden, "m0/", len(y), x.shape[1], 48, tcu.KV_I8, plan)
    assert [nm for nm, _, _ in names] == list(ent)
    for nm, dt, dims in names:
        assert ent[nm].dtype.name == dt and list(ent[nm].shape) == dims, nm
    wb = t["wb"]
    tensors = {k: np.asarray(wb[k]) for k in wb.names()}
    tensors.update(ent)
    path = tmp_path / "fitted.tirs"
    tirs.write(str(path), tensors)
    back = tcu.VramMember.from_bundle(golden, str(path), "m0/")
    xt = t["x_test"]
    assert np.array_equal(back.rows(xt), mb.rows(xt))
    back.free(), mb.free()
