"""The boundary on a device: bundles read the way tabicl-anywhere writes them, the AttendCached hook's decline and
fallback behaviour, and the report of kernels that gave up a bounded wait.

* A fitted bundle in the layout `fit::raw_entries` writes (src/fit.rs:224-241: `m{i}/meta`, `m{i}/tree`,
  `m{i}/col_kv`, `m{i}/n{j}_scale`, `m{i}/n{j}_kv{l}`) loads through tcu_model_from_bundle and answers exactly as
  the same cache put piece by piece.
* A weight bundle stored in float16 (as the published weights are) is widened exactly on upload
  (src/store.rs:363-375): the stage equals the one on the widened float32 tensors bit for bit.
* CudaAttend declines (None) and counts a fallback when the device cannot answer, and answers again afterwards,
  as the card handle does (src/gpu.rs:2658-2671; the reference's own model of this is tests/accel.rs:91-111,
  175-179: the CPU takes over the layers the accelerator declines).
* A give-up inside the one-kernel stage (made with the test hook tcu_debug_abort_next, so that no wait has to run
  out) is reported as TCU_ERR_CUDA naming the wait, by the host form directly and by tcu_sync after a device
  form; the next call answers correctly.
"""
import json

import numpy as np
import pytest

from conftest import GOLDEN, synth, tcu, tirs
import oracle

pytestmark = pytest.mark.gpu

STAGE = 5e-5
ATTEND = 1e-5


@pytest.fixture(scope="module")
def gpu():
    g = tcu.Gpu(0)
    yield g
    g.close()


def _tiny_model(seed=3):
    cfg = synth.config("tiny")
    wt = synth.weights(cfg, seed=seed, std=0.08)
    m = oracle.Model({k: v for k, v in wt.items() if k.startswith("icl_predictor.")}, cfg["icl_nhead"],
                     cfg["icl_num_blocks"], cfg["max_classes"])
    return cfg, wt, m


def _fitted_bundle(path, members):
    """members: list of (rows, chunk, kv, classes, scales, layers, features): the tensors fit_raw fills, per member
    prefix m{i}/, one node each (fit.rs:284-291 meta; fit.rs:218-220 tree = [leaf, rows, k, map...])."""
    t = {}
    for i, (rows, chunk, kv, classes, scales, layers, features) in enumerate(members):
        p = f"m{i}/"
        t[p + "meta"] = np.array([rows, features, classes, chunk, kv, 1, 1], np.int32)
        t[p + "tree"] = np.array([1, rows, classes] + list(range(classes)), np.int32)
        t[p + "col_kv"] = np.zeros((features, 1, 1, 2, 16, 4), np.float32)  # column stage: not read by this path
        t[p + "n0_scale"] = np.ascontiguousarray(scales, np.float32)
        for l, b in enumerate(layers):
            t[p + f"n0_kv{l}"] = np.frombuffer(bytes(b), np.uint8)
    tirs.write(str(path), t)


def test_model_from_fitted_bundle(gpu, tmp_path):
    cfg, wt, m = _tiny_model()
    w = tcu.GpuWeights.from_tensors(gpu, synth.icl_shape(cfg), {k: v for k, v in wt.items() if k.startswith("icl_")})
    members = []
    for i, (n, chunk, kv) in enumerate([(300, 48, 1), (211, 37, 2)]):
        h = synth.row_reps(n, m.d, 40 + i)
        y = synth.labels(n, 10, 50 + i)
        layers, scales = oracle.icl_fit(m, h, y, chunk, kv)
        members.append((n, chunk, kv, 10, scales, layers, 7))
    path = tmp_path / "fitted.tirs"
    _fitted_bundle(path, members)
    ht = synth.row_reps(11, m.d, 60)
    for i, (n, chunk, kv, classes, scales, layers, features) in enumerate(members):
        from_file = tcu.VramModel.from_bundle(w, str(path), f"m{i}/", 0)
        by_parts = tcu.VramModel.from_parts(w, [n, features, classes, chunk, kv, 1, 1], n, classes, scales, layers)
        assert from_file.nbytes == by_parts.nbytes
        got = from_file.stage(ht, 10)
        assert np.array_equal(got, by_parts.stage(ht, 10))
        assert np.abs(got - oracle.in_context(m, kv, layers, scales, n, chunk, ht, 10)).max() < STAGE
        for l in range(m.layers):
            assert np.array_equal(from_file.layer_bytes(l, len(layers[l])), np.frombuffer(bytes(layers[l]), np.uint8))
        from_file.free(), by_parts.free()
    with pytest.raises(tcu.TcuError) as e:
        tcu.VramModel.from_bundle(w, str(path), "m0/", 1)  # one node only
    assert e.value.code == -1
    w.free()


def test_float16_weight_bundle_is_widened_exactly(gpu, tmp_path):
    cfg, wt, m = _tiny_model(seed=4)
    half = {}
    for k, v in wt.items():
        half[k] = v.astype(np.float16) if k.startswith("icl_predictor.") else v
    path = tmp_path / "weights-half.tirs"
    tirs.write(str(path), half)
    w16 = tcu.GpuWeights.from_bundle(gpu, str(path))
    widened = {k: (v.astype(np.float32) if v.dtype == np.float16 else v) for k, v in half.items()}
    w32 = tcu.GpuWeights.from_tensors(gpu, synth.icl_shape(cfg),
                                      {k: v for k, v in widened.items() if k.startswith("icl_")})
    assert w16.shape == w32.shape
    m32 = oracle.Model({k: v for k, v in widened.items() if k.startswith("icl_predictor.")}, cfg["icl_nhead"],
                       cfg["icl_num_blocks"], cfg["max_classes"])
    n, chunk, kv = 260, 64, 1
    layers, scales = oracle.icl_fit(m32, synth.row_reps(n, m.d, 70), synth.labels(n, 10, 71), chunk, kv)
    meta = [n, 7, 10, chunk, kv, 1, 1]
    a = tcu.VramModel.from_parts(w16, meta, n, 10, scales, layers)
    b = tcu.VramModel.from_parts(w32, meta, n, 10, scales, layers)
    ht = synth.row_reps(9, m.d, 72)
    got = a.stage(ht, 10)
    assert np.array_equal(got, b.stage(ht, 10))
    assert np.abs(got - oracle.in_context(m32, kv, layers, scales, n, chunk, ht, 10)).max() < STAGE
    a.free(), b.free(), w16.free(), w32.free()


def test_cuda_attend_declines_and_recovers(gpu, tmp_path):
    cfg, wt, m = _tiny_model(seed=5)
    w = tcu.GpuWeights.from_tensors(gpu, synth.icl_shape(cfg), {k: v for k, v in wt.items() if k.startswith("icl_")})
    n, chunk, kv = 180, 48, 2
    layers, scales = oracle.icl_fit(m, synth.row_reps(n, m.d, 80), synth.labels(n, 10, 81), chunk, kv)
    path = tmp_path / "fitted.tirs"
    _fitted_bundle(path, [(n, chunk, kv, 10, scales, layers, 5)])
    acc = tcu.CudaAttend(w, str(path))
    ht = synth.row_reps(6, m.d, 82)
    got = acc.stage("m0/", 0, ht, m.d, 10)
    assert got is not None and acc.fallbacks == 0
    assert np.abs(got - oracle.in_context(m, kv, layers, scales, n, chunk, ht, 10)).max() < STAGE
    q = np.random.default_rng(83).normal(0, 1, (4, m.d)).astype(np.float32)
    for l in range(m.layers):
        att = acc.attend("m0/", 0, l, q, m.d, m.heads)
        assert np.abs(att - oracle.attend(kv, m.d, m.heads, layers[l], n, chunk, q)).max() < ATTEND
    # the device cannot answer: a member the bundle does not hold, a width that is not the model's
    assert acc.stage("m7/", 0, ht, m.d, 10) is None
    assert acc.fallbacks == 1 and "m7/meta" in acc.last_error
    assert acc.attend("m0/", 0, 0, np.zeros((2, m.d + 4), np.float32), m.d + 4, m.heads) is None
    assert acc.fallbacks == 2
    # weights made without the column and row stages: the rows hook declines, the caller's CPU path answers
    assert acc.rows("m0/", np.zeros((2, 5), np.float32), 10) is None
    # and after declining it answers again, with the same numbers
    assert np.array_equal(acc.stage("m0/", 0, ht, m.d, 10), got)
    w.free()


def test_give_up_is_reported_and_the_next_call_recovers(gpu):
    import torch
    cfg = synth.config("full", icl_num_blocks=2)
    wt = synth.weights(cfg, seed=90, std=0.08)
    m = oracle.Model({k: v for k, v in wt.items() if k.startswith("icl_predictor.")}, cfg["icl_nhead"], 2, 10)
    n, chunk, kv = 1000, 256, 1
    layers, scales = oracle.icl_fit(m, synth.row_reps(n, m.d, 91), synth.labels(n, 10, 92), chunk, kv)
    w = tcu.GpuWeights.from_tensors(gpu, synth.icl_shape(cfg), {k: v for k, v in wt.items() if k.startswith("icl_")})
    vm = tcu.VramModel.from_parts(w, [n, 7, 10, chunk, kv, 1, 1], n, 10, scales, layers)
    ht = synth.row_reps(3, m.d, 93)
    want = vm.stage(ht, 10)                      # the one-kernel stage (3 rows, head width 128)
    assert np.abs(want - oracle.in_context(m, kv, layers, scales, n, chunk, ht, 10)).max() < STAGE
    before = gpu.launches
    gpu.debug_abort_next()
    with pytest.raises(tcu.TcuError) as e:
        vm.stage(ht, 10)                         # host form: reported by the call itself
    assert e.value.code == -3 and "left after another CTA gave up" in str(e.value)
    assert gpu.launches - before == 1
    assert np.array_equal(vm.stage(ht, 10), want)
    # device form: queued, then reported by tcu_sync; the context is usable afterwards
    hd = torch.from_numpy(ht).cuda()
    out = torch.empty((3, 10), device="cuda")
    gpu.debug_abort_next()
    vm.stage_device(hd.data_ptr(), 3, 10, out.data_ptr())
    with pytest.raises(tcu.TcuError) as e:
        gpu.sync()
    assert e.value.code == -3
    gpu.sync()                                   # reported once
    vm.stage_device(hd.data_ptr(), 3, 10, out.data_ptr())
    gpu.sync()
    assert np.array_equal(out.cpu().numpy(), want)
    # one row (the one-kernel stage's one-row form): the same report and recovery
    one = vm.stage(ht[:1], 10)
    assert np.abs(one - oracle.in_context(m, kv, layers, scales, n, chunk, ht[:1], 10)).max() < STAGE
    gpu.debug_abort_next()
    with pytest.raises(tcu.TcuError) as e:
        vm.stage(ht[:1], 10)
    assert e.value.code == -3 and "left after another CTA gave up" in str(e.value)
    assert np.array_equal(vm.stage(ht[:1], 10), one)
    vm.free(), w.free()


def test_weights_bundle_config_whitelist(gpu, tmp_path):
    """Model::load accepts only the TabICL v2 layout this path implements (src/model.rs:204-219)."""
    cfg, wt, m = _tiny_model(seed=6)
    bad = dict(wt)
    c = dict(cfg, norm_first=False)
    bad["config.json"] = np.frombuffer(json.dumps(c).encode(), np.uint8)
    path = tmp_path / "post-norm.tirs"
    tirs.write(str(path), bad)
    with pytest.raises(tcu.TcuError) as e:
        tcu.GpuWeights.from_bundle(gpu, str(path))
    assert e.value.code == -2 and "norm_first" in str(e.value)
    assert tcu.GpuWeights.from_bundle(gpu, GOLDEN + "/tiny-clf.tirs").shape["d"] == 16
