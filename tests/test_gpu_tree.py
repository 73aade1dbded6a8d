"""A member of several in-context problems on the device: the class tree of a table with more classes than the model
tells apart (src/predict.rs:638-699), fitted per node on the device from fit::Plan (src/fit.rs:159-221), through
the C ABI, against the oracle.

Bars: the tree step alone (expf/logf on both sides) within 1e-5 of the oracle's scores, relative to their magnitude
past 1. A whole pass: each problem's stage is within 5e-5 of the oracle (the stage bar); carried through the tempered
softmax (2 / 0.9) and the log (0.9) that is 1e-4 of score per level of the tree; the class probabilities
exp(score / 0.9) within 1e-5.
"""
import numpy as np
import pytest

from conftest import synth, tcu, tirs
import oracle

pytestmark = pytest.mark.gpu

COMBINE = 1e-5
PER_LEVEL = 1e-4
PROBA = 1e-5


@pytest.fixture(scope="module")
def gpu():
    g = tcu.Gpu(0)
    yield g
    g.close()


@pytest.fixture(scope="module")
def tiny(gpu):
    cfg = synth.config("tiny")
    wt = synth.weights(cfg, seed=11, std=0.08)
    w = tcu.GpuWeights.from_tensors(gpu, synth.icl_shape(cfg), wt, rows_shape=synth.rows_shape(cfg), for_fit=True)
    m = oracle.Model({k: v for k, v in wt.items() if k.startswith("icl_predictor.")}, cfg["icl_nhead"],
                     cfg["icl_num_blocks"], cfg["max_classes"])
    rm = oracle.RowsModel({k: v for k, v in wt.items() if k.startswith(("col_embedder.", "row_interactor."))}, cfg)
    yield dict(cfg=cfg, w=w, m=m, rm=rm, rs=synth.rows_shape(cfg))
    w.free()


def _levels(plan):
    depth = {0: 1}
    for i, n in enumerate(plan.nodes):
        for c in ([] if n.leaf else n.map):
            depth[c] = depth[i] + 1
    return max(depth.values())


def _fit(t, n, classes, features, kv, chunk, seed):
    y = synth.labels(n, classes, seed)
    plan = tcu.Plan.new(10, y, classes)
    rs = t["rs"]
    ck = synth.col_kv(features, rs["col_blocks"], rs["e"], rs["inds"], seed + 1, len(plan.bases))
    h = synth.row_reps(n, t["m"].d, seed + 2)
    mb, plan2 = tcu.fit_member(t["w"], h, y, classes, features, ck, chunk=chunk, kv=kv)
    assert plan2.tree(n).tolist() == plan.tree(n).tolist()
    return mb, plan, ck


def _oracle_pass(t, mb, plan, ck, x, kv, chunk, n):
    m = t["m"]
    tok = oracle.embed(t["rm"], x, ck, digits=len(plan.bases))
    rep = oracle.represent(t["rm"], tok)
    scores = []
    for i, nd in enumerate(plan.nodes):
        rows = n if nd.rows is None else len(nd.rows)
        node = mb.node(i)
        layers = [node.layer_bytes(l, oracle.layer_len(kv, m.d, rows, chunk)) for l in range(m.layers)]
        scores.append(oracle.in_context(m, kv, layers, node.scales(), rows, chunk, rep, nd.k))
    return scores, oracle.tree_scores(scores, plan.tree(n), len(plan.nodes), mb.classes)


@pytest.mark.parametrize("classes,kv", [(25, tcu.KV_F32), (150, tcu.KV_I16)])
def test_member_pass_matches_oracle(tiny, classes, kv):
    n, features, chunk = 600, 6, 64
    mb, plan, ck = _fit(tiny, n, classes, features, kv, chunk, seed=classes)
    assert mb.n_nodes == len(plan.nodes) > 1 and mb.classes == classes
    x = synth.features(40, features, 7 + classes, missing=0.1)
    got = mb.rows(x)
    _, want = _oracle_pass(tiny, mb, plan, ck, x, kv, chunk, n)
    bar = PER_LEVEL * _levels(plan)
    assert np.abs(got - want).max() < bar, (np.abs(got - want).max(), bar)
    assert np.abs(np.exp(got / 0.9) - np.exp(want / 0.9)).max() < PROBA
    mb.free()


def test_combine_alone_matches_oracle(tiny):
    n, classes = 500, 150
    mb, plan, _ = _fit(tiny, n, classes, 4, tcu.KV_F32, 64, seed=3)
    import torch
    rng = np.random.default_rng(5)
    R = 333
    per = [rng.standard_normal((R, nd.k)).astype(np.float32) * 4 for nd in plan.nodes]
    per[1][0, :] = np.float32(30.0)  # ties of large scores
    flat = np.concatenate([p.reshape(-1) for p in per])
    sd = torch.from_numpy(flat).cuda()
    out = torch.empty((R, classes), device="cuda")
    torch.cuda.synchronize()
    mb.combine_device(sd.data_ptr(), R, out.data_ptr())
    mb.gpu.sync()
    got = out.cpu().numpy()
    want = oracle.tree_scores(per, plan.tree(n), len(plan.nodes), classes)
    err = np.abs(got - want) / np.maximum(1.0, np.abs(want))
    assert err.max() < COMBINE, err.max()
    mb.free()


def test_member_from_fitted_bundle(tiny, tmp_path):
    """A many-class member written the way fit_raw stores it (src/fit.rs:224-241, 291-292) loads whole through
    tcu_member_from_bundle and answers bit for bit as the member it was written from; each problem loads alone
    for the per-problem `stage` hook too."""
    t = tiny
    n, classes, features, kv, chunk = 400, 25, 5, tcu.KV_I8, 48
    mb, plan, ck = _fit(t, n, classes, features, kv, chunk, seed=77)
    m = t["m"]
    p = "m0/"
    tensors = {p + "meta": np.array([n, features, classes, chunk, kv, len(plan.bases), len(plan.nodes)], np.int32),
               p + "tree": plan.tree(n), p + "col_kv": ck}
    for i, nd in enumerate(plan.nodes):
        rows = n if nd.rows is None else len(nd.rows)
        node = mb.node(i)
        tensors[p + f"n{i}_scale"] = node.scales()
        for l in range(m.layers):
            tensors[p + f"n{i}_kv{l}"] = node.layer_bytes(l, oracle.layer_len(kv, m.d, rows, chunk))
    path = tmp_path / "many.tirs"
    tirs.write(str(path), tensors)
    x = synth.features(17, features, 78, missing=0.05)
    back = tcu.VramMember.from_bundle(t["w"], str(path), p)
    assert back.n_nodes == len(plan.nodes) and back.classes == classes
    assert np.array_equal(back.rows(x), mb.rows(x))
    h = synth.row_reps(9, m.d, 79)
    for i, nd in enumerate(plan.nodes):
        one = tcu.VramModel.from_bundle(t["w"], str(path), p, i)
        assert np.array_equal(one.stage(h, nd.k), mb.node(i).stage(h, nd.k))
        one.free()
    back.free(), mb.free()


def test_one_problem_member_is_the_rows_hook(tiny):
    n, classes, features = 300, 7, 5
    mb, plan, ck = _fit(tiny, n, classes, features, tcu.KV_I16, 64, seed=21)
    assert mb.n_nodes == 1
    x = synth.features(12, features, 22)
    assert np.array_equal(mb.rows(x), mb.node(0).rows(x, classes))
    mb.free()


def test_predict_raw_in_passes(tiny):
    n, classes, features, kv, chunk = 500, 25, 6, tcu.KV_I16, 64
    mb, plan, ck = _fit(tiny, n, classes, features, kv, chunk, seed=31)
    x = synth.features(30, features, 32, missing=0.1)
    st = tcu.Stats()
    got = tcu.predict_raw(mb, x, rows_per_pass=8, stats=st)
    assert (st.rows, st.passes, st.card_layers) == (30, 4, 4 * tiny["m"].layers * len(plan.nodes))
    _, want = _oracle_pass(tiny, mb, plan, ck, x, kv, chunk, n)
    assert np.abs(got - want).max() < PER_LEVEL * _levels(plan)
    mb.free()


def test_bad_trees_are_refused(tiny):
    t = tiny
    w, d = t["w"], t["m"].d
    import torch

    def node(seed):
        h = torch.from_numpy(synth.row_reps(100, d, seed)).cuda()
        y = torch.from_numpy(synth.labels(100, 2, seed)).cuda()
        torch.cuda.synchronize()
        return tcu.fit_icl(w, h.data_ptr(), y.data_ptr(), 100, 32, tcu.KV_F32)

    nodes = [node(s) for s in (1, 2, 3)]
    bad = {
        "reached twice": [0, 100, 2, 1, 1, 1, 50, 2, 0, 1, 1, 50, 2, 2, 3],
        "class out of range": [0, 100, 2, 1, 2, 1, 50, 2, 0, 1, 1, 50, 2, 2, 9],
        "child out of range": [0, 100, 2, 1, 5, 1, 50, 2, 0, 1, 1, 50, 2, 2, 3],
        "damaged": [0, 100, 2, 1, 2, 1, 50, 2, 0, 1, 1, 50, 2],
    }
    for why, tree in bad.items():
        with pytest.raises(tcu.TcuError) as e:
            tcu.VramMember.from_nodes(nodes, tree, 4)
        assert e.value.code == -2, why
    mb = tcu.VramMember.from_nodes(nodes, [0, 100, 2, 1, 2, 1, 50, 2, 0, 1, 1, 50, 2, 2, 3], 4)
    assert mb.n_nodes == 3
    mb.free()


@pytest.mark.parametrize("arch,rows,kv", [("tiny", 1, 1), ("tiny", 5, 2), ("tiny", 33, 0), ("full", 3, 1),
                                          ("full", 40, 2)])
def test_fit_of_small_nodes(gpu, arch, rows, kv):
    """A node of a class tree can hold very few training rows: the device fit (whose attention over the training
    rows then takes the few-row kernels) against the oracle's fit."""
    import torch
    cfg = synth.config(arch, icl_num_blocks=2)
    wt = synth.weights(cfg, seed=41, std=0.08)
    m = oracle.Model({k: v for k, v in wt.items() if k.startswith("icl_predictor.")}, cfg["icl_nhead"], 2, 10)
    w = tcu.GpuWeights.from_tensors(gpu, synth.icl_shape(cfg), {k: v for k, v in wt.items() if k.startswith("icl_")},
                                    for_fit=True)
    chunk = 16
    h = synth.row_reps(rows, m.d, 42)
    y = synth.labels(rows, 3, 43)
    want_layers, want_scales = oracle.icl_fit(m, h, y, chunk, kv)
    hd, yd = torch.from_numpy(h.copy()).cuda(), torch.from_numpy(y).cuda()
    torch.cuda.synchronize()
    vm = tcu.fit_icl(w, hd.data_ptr(), yd.data_ptr(), rows, chunk, kv)
    assert np.array_equal(vm.scales(), want_scales)
    nbytes = oracle.layer_len(kv, m.d, rows, max(chunk, 8))
    for l in range(2):
        gk, gv = oracle.layer_rows(kv, m.d, vm.layer_bytes(l, nbytes), rows, chunk)
        wk, wv = oracle.layer_rows(kv, m.d, want_layers[l], rows, chunk)
        step = {0: 0.0, 1: 1.0 / 32767, 2: 1.0 / 127}[kv] * max(np.abs(wk).max(), np.abs(wv).max())
        assert np.abs(gk - wk).max() < 1e-4 + 1.01 * step
        assert np.abs(gv - wv).max() < 1e-4 + 1.01 * step
    vm.free(), w.free()
