"""The card tier on a device (gpu::VramTier and VramHandle, src/gpu.rs:2450-2701): problems loaded from fitted bundles
through the pinned upload pipeline answer like problems put piece by piece; budgets per tenant and in all, least
recently used first; a problem larger than its tenant's budget is never loaded; a load started by a prediction runs
on a thread of its own while that prediction declines; a device failure declines and is counted; evicted problems
still in use stay until released; tenants predicting at once while one of them is evicted over and over (the
reference's tests/card.rs:276-328)."""
import threading

import numpy as np
import pytest

from conftest import synth, tcu, tirs
import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu():
    g = tcu.Gpu(0)
    yield g
    g.close()


@pytest.fixture(scope="module")
def tiny(gpu, tmp_path_factory):
    """Tiny weights with the column and row stages, and a bundle of three members: m0/ and m1/ one problem each with
    the column cache, m2/ a class tree of three problems."""
    cfg = synth.config("tiny")
    wt = synth.weights(cfg, seed=21, std=0.08)
    w = tcu.GpuWeights.from_tensors(gpu, synth.icl_shape(cfg), wt, rows_shape=synth.rows_shape(cfg), for_fit=True)
    m = oracle.Model({k: v for k, v in wt.items() if k.startswith("icl_predictor.")}, cfg["icl_nhead"],
                     cfg["icl_num_blocks"], cfg["max_classes"])
    rs = synth.rows_shape(cfg)
    features, t = 5, {}
    for i, (n, chunk, kv) in enumerate([(300, 48, 1), (300, 48, 1)]):
        layers, scales = oracle.icl_fit(m, synth.row_reps(n, m.d, 60 + i), synth.labels(n, 10, 70 + i), chunk, kv)
        p = f"m{i}/"
        t[p + "meta"] = np.array([n, features, 10, chunk, kv, 1, 1], np.int32)
        t[p + "tree"] = np.array([1, n, 10] + list(range(10)), np.int32)
        t[p + "col_kv"] = synth.col_kv(features, rs["col_blocks"], rs["e"], rs["inds"], 80 + i)
        t[p + "n0_scale"] = scales
        for l, b in enumerate(layers):
            t[p + f"n0_kv{l}"] = np.frombuffer(bytes(b), np.uint8)
    # m2/: 14 classes, a root over two leaves of 7
    y = synth.labels(200, 14, 90)
    plan = tcu.Plan.new(10, y, 14)
    h = synth.row_reps(200, m.d, 91)
    p = "m2/"
    t[p + "meta"] = np.array([200, features, 14, 32, 0, len(plan.bases), len(plan.nodes)], np.int32)
    t[p + "tree"] = plan.tree(200)
    t[p + "col_kv"] = synth.col_kv(features, rs["col_blocks"], rs["e"], rs["inds"], 92, len(plan.bases))
    for j, nd in enumerate(plan.nodes):
        rows = np.arange(200) if nd.rows is None else np.asarray(nd.rows)
        layers, scales = oracle.icl_fit(m, h[rows], nd.y, 32, 0)
        t[p + f"n{j}_scale"] = scales
        for l, b in enumerate(layers):
            t[p + f"n{j}_kv{l}"] = np.frombuffer(bytes(b), np.uint8)
    path = tmp_path_factory.mktemp("tier") / "fitted.tirs"
    tirs.write(str(path), t)
    yield dict(w=w, m=m, path=str(path), features=features, plan=plan)
    w.free()


def _direct(t, prefix, node=0):
    return tcu.VramModel.from_bundle(t["w"], t["path"], prefix, node)


def test_hooks_answer_like_the_model(tiny):
    t, d = tiny, tiny["m"].d
    tier = tcu.VramTier(tiny["w"].gpu, 1 << 30, 1 << 30, background=False)
    h = tier.handle("t", "a", t["path"], t["w"])
    assert h.preload("m0/", 0)
    vm = _direct(t, "m0/")
    assert tier.held("t") == (vm.nbytes, vm.nbytes) == tier.on_card("t") and tier.ready("t") == vm.nbytes
    x = synth.row_reps(9, d, 1)
    assert np.array_equal(h.stage("m0/", 0, x, d, 10), vm.stage(x, 10))
    q = synth.row_reps(4, d, 2)
    assert np.array_equal(h.attend("m0/", 0, 1, q, d, t["m"].heads), vm.attend(1, q))
    feats = synth.features(6, t["features"], 3, missing=0.1)
    assert np.array_equal(h.rows("m0/", feats, 10), vm.rows(feats, 10))
    assert tier.fallbacks == 0 and tier.last_error() is None
    vm.free(), h.free(), tier.free()


def test_background_load_declines_then_answers(tiny):
    t, d = tiny, tiny["m"].d
    tier = tcu.VramTier(t["w"].gpu, 1 << 30, 1 << 30, background=True)
    h = tier.handle("t", "a", t["path"], t["w"])
    x = synth.row_reps(3, d, 4)
    assert h.stage("m1/", 0, x, d, 10) is None  # not resident: its load starts on a thread
    tier.wait()
    vm = _direct(t, "m1/")
    assert np.array_equal(h.stage("m1/", 0, x, d, 10), vm.stage(x, 10))
    assert tier.ready("t") == vm.nbytes
    vm.free(), h.free(), tier.free()


def test_tenant_shares_and_least_recently_used(tiny):
    t = tiny
    one = _direct(t, "m0/").nbytes
    tier = tcu.VramTier(t["w"].gpu, 2 * one, one, background=False)
    assert tier.preload("alice", "a", t["path"], t["w"], "m0/", 0)
    assert tier.preload("bob", "a", t["path"], t["w"], "m0/", 0)
    assert tier.on_card("alice") == (2 * one, one)
    # alice's second member goes over her share: her own first one makes room, bob's stays
    assert tier.preload("alice", "a", t["path"], t["w"], "m1/", 0)
    assert tier.held("alice") == (2 * one, one) and tier.held("bob") == (2 * one, one)
    h = tier.handle("bob", "a", t["path"], t["w"])
    assert h.stage("m0/", 0, synth.row_reps(2, t["m"].d, 5), t["m"].d, 10) is not None
    h.free(), tier.free()


def test_problem_larger_than_tenant_budget_stays_off_the_card(tiny):
    t = tiny
    tier = tcu.VramTier(t["w"].gpu, 1 << 30, 1 << 10, background=False)
    assert not tier.preload("carol", "a", t["path"], t["w"], "m0/", 0)
    h = tier.handle("carol", "a", t["path"], t["w"])
    for _ in range(3):
        assert h.stage("m0/", 0, synth.row_reps(2, t["m"].d, 6), t["m"].d, 10) is None
    assert tier.on_card("carol") == (0, 0) and tier.fallbacks == 0
    h.free(), tier.free()


def test_device_failure_declines_and_is_counted(tiny):
    t, d = tiny, tiny["m"].d
    tier = tcu.VramTier(t["w"].gpu, 1 << 30, 1 << 30, background=False)
    h = tier.handle("t", "a", t["path"], t["w"])
    assert h.stage("m0/", 0, synth.row_reps(2, d, 7), d, 99) is None  # more outputs than the decoder has
    assert tier.fallbacks == 1 and "out_n" in tier.last_error()
    assert h.stage("m0/", 0, synth.row_reps(2, d, 7), d, 10) is not None  # the next call answers
    assert tier.fallbacks == 1
    h.free(), tier.free()


def test_rows_hook_only_for_one_problem(tiny):
    """A class tree: `rows` declines (the reference calls it only for one problem and one label digit) without
    counting a failure; its problems answer `stage` one by one."""
    t, d = tiny, tiny["m"].d
    tier = tcu.VramTier(t["w"].gpu, 1 << 30, 1 << 30, background=False)
    h = tier.handle("t", "a", t["path"], t["w"])
    assert h.rows("m2/", synth.features(3, t["features"], 8), 14) is None
    x = synth.row_reps(3, d, 9)
    for j, nd in enumerate(t["plan"].nodes):
        vm = _direct(t, "m2/", j)
        assert np.array_equal(h.stage("m2/", j, x, d, nd.k), vm.stage(x, nd.k))
        vm.free()
    assert tier.fallbacks == 0
    h.free(), tier.free()


def test_bundle_read_through_a_source(tiny):
    t, d = tiny, tiny["m"].d
    data = open(t["path"], "rb").read()
    tier = tcu.VramTier(t["w"].gpu, 1 << 30, 1 << 30, background=True)
    h = tier.handle("t", "mem", data, t["w"])
    x = synth.row_reps(4, d, 10)
    assert h.stage("m0/", 0, x, d, 10) is None
    tier.wait()
    vm = _direct(t, "m0/")
    assert np.array_equal(h.stage("m0/", 0, x, d, 10), vm.stage(x, 10))
    vm.free(), h.free(), tier.free()


def test_evicted_problem_in_use_stays_until_released(tiny):
    t, d = tiny, tiny["m"].d
    one = _direct(t, "m0/").nbytes
    tier = tcu.VramTier(t["w"].gpu, one, one, background=False)
    h = tier.handle("t", "a", t["path"], t["w"])
    assert h.preload("m0/", 0)
    pin = tier.debug_pin("t", "a", "m0/", 0)
    tier.evict("t")
    assert tier.held("t") == (0, 0) and tier.on_card("t") == (one, one)
    x = synth.row_reps(2, d, 11)
    assert h.stage("m0/", 0, x, d, 10) is None  # its room is still taken
    tcu.VramTier.debug_unpin(pin)
    assert tier.on_card("t") == (0, 0)
    assert h.stage("m0/", 0, x, d, 10) is not None
    h.free(), tier.free()


def test_tenants_at_once_and_eviction_in_flight(tiny):
    t, d = tiny, tiny["m"].d
    vm = _direct(t, "m0/")
    one = vm.nbytes
    x = synth.row_reps(5, d, 12)
    want = vm.stage(x, 10)
    vm.free()
    tier = tcu.VramTier(t["w"].gpu, 2 * one, one, background=True)
    assert tier.preload("alice", "a", t["path"], t["w"], "m0/", 0)
    assert tier.preload("bob", "a", t["path"], t["w"], "m0/", 0)
    stop, errors, answered = threading.Event(), [], {"alice": 0, "bob": 0}

    def predict(who):
        h = tier.handle(who, "a", t["path"], t["w"])
        try:
            for _ in range(20):
                got = h.stage("m0/", 0, x, d, 10)
                if got is not None:
                    answered[who] += 1
                    if not np.array_equal(got, want):
                        errors.append(f"{who}: wrong answer")
                all_, mine = tier.on_card(who)
                if all_ > 2 * one or mine > one:
                    errors.append(f"{who}: over budget on the card")
        finally:
            h.free()

    def evictor():
        while not stop.is_set():
            tier.evict("alice")

    ev = threading.Thread(target=evictor)
    ev.start()
    runs = [threading.Thread(target=predict, args=(w,)) for w in ("alice", "bob")]
    for r in runs:
        r.start()
    for r in runs:
        r.join()
    stop.set()
    ev.join()
    assert not errors, errors
    assert answered["bob"] == 20
    assert tier.fallbacks == 0, tier.last_error()
    tier.wait()
    tier.evict("alice"), tier.evict("bob")
    assert tier.on_card("alice") == (0, 0)
    tier.free()


def test_layers_larger_than_the_staging_buffers(gpu, tmp_path):
    """Stored layers of 18 MB, more than two of the 8 MB pinned staging pieces: the bytes on the device are the
    bytes in the file, and the stage answers as the cache put piece by piece."""
    cfg = synth.config("tiny")
    wt = synth.weights(cfg, seed=22, std=0.08)
    w = tcu.GpuWeights.from_tensors(gpu, synth.icl_shape(cfg), {k: v for k, v in wt.items() if k.startswith("icl_")})
    d, rows, chunk = 32, 70000, 256
    rng = np.random.default_rng(23)
    layers = [oracle.pack_layer(0, d, rng.standard_normal((rows, d)).astype(np.float32),
                                rng.standard_normal((rows, d)).astype(np.float32), chunk) for _ in range(2)]
    scales = rng.standard_normal((2, d)).astype(np.float32) * 0.1
    tensors = {"m0/meta": np.array([rows, 4, 10, chunk, 0, 1, 1], np.int32),
               "m0/tree": np.array([1, rows, 10] + list(range(10)), np.int32), "m0/n0_scale": scales}
    for l, b in enumerate(layers):
        tensors[f"m0/n0_kv{l}"] = b
    path = tmp_path / "big.tirs"
    tirs.write(str(path), tensors)
    vm = tcu.VramModel.from_bundle(w, str(path), "m0/", 0)
    for l, b in enumerate(layers):
        assert np.array_equal(vm.layer_bytes(l, b.size), b)
    parts = tcu.VramModel.from_parts(w, [rows, 4, 10, chunk, 0, 1, 1], rows, 10, scales, layers)
    x = synth.row_reps(3, d, 24)
    assert np.array_equal(vm.stage(x, 10), parts.stage(x, 10))
    vm.free(), parts.free(), w.free()
