"""Parity of the device path (through the C ABI) with the oracle and with the reference's golden vectors.

Bars (stated per test): stage outputs (raw decoder scores) within 5e-5 of the CPU path on the same cache, class
probabilities within 1e-5, attention outputs within 1e-5, integer unpacking and chunk packing bit-exact.
"""
import numpy as np
import pytest

from conftest import GOLDEN, synth, tcu
import oracle

pytestmark = pytest.mark.gpu

STAGE = 5e-5   # raw scores, per cached stage
PROBA = 1e-5   # probabilities
ATTEND = 1e-5  # attention outputs


@pytest.fixture(scope="module")
def gpu():
    g = tcu.Gpu(0)
    yield g
    g.close()


def softmax(x, t=0.9):
    z = (x - x.max(1, keepdims=True)) / t
    e = np.exp(z)
    return e / e.sum(1, keepdims=True)


def _meta(rows, chunk, kv, classes):
    return [rows, 7, classes, chunk, kv, 1, 1]


def test_tensor_core_operand_layouts(gpu):
    """Exact small-integer products on the tcgen05 units equal CUDA-core sums for every operand layout used."""
    assert gpu.selftest_mma() == 0.0


# ---- the reference's tiny classifier and PyTorch's golden numbers -----------------------------------------------

@pytest.mark.parametrize("kv", [0, 1, 2])
@pytest.mark.parametrize("chunk", [48, 37, 256])
def test_stage_on_golden_cache(gpu, tiny, kv, chunk):
    t = tiny
    m = t["m"]
    w = tcu.GpuWeights.from_bundle(gpu, t["path"])
    layers = [oracle.pack_layer(kv, m.d, t["k"][l], t["v"][l], chunk) for l in range(m.layers)]
    vm = tcu.VramModel.from_parts(w, _meta(t["n"], chunk, kv, 3), t["n"], 3, t["scales"], layers)
    got = vm.stage(t["test_rep"], 3)
    want = oracle.in_context(m, kv, layers, t["scales"], t["n"], chunk, t["test_rep"], 3)
    assert np.abs(got - want).max() < STAGE
    assert np.abs(softmax(got) - softmax(want)).max() < PROBA
    if kv == 0:
        assert np.abs(got - t["logits"]).max() < 5e-5  # PyTorch's own logits (tests/reference.rs:107-116)


@pytest.mark.parametrize("rows", [1, 3, 8, 13, 40, 100])
def test_attend_hook_on_golden_cache(gpu, tiny, rows):
    t = tiny
    m = t["m"]
    w = tcu.GpuWeights.from_bundle(gpu, t["path"])
    rng = np.random.default_rng(rows)
    for kv in (0, 1, 2):
        layers = [oracle.pack_layer(kv, m.d, t["k"][l], t["v"][l], 48) for l in range(m.layers)]
        vm = tcu.VramModel.from_parts(w, _meta(t["n"], 48, kv, 3), t["n"], 3, t["scales"], layers)
        q = rng.normal(0, 1, (rows, m.d)).astype(np.float32)
        for l in range(m.layers):
            got = vm.attend(l, q)
            want = oracle.attend(kv, m.d, m.heads, layers[l], t["n"], 48, q)
            assert np.abs(got - want).max() < ATTEND, (kv, l)


# ---- synthetic models at several head widths, row counts and chunkings -------------------------------------

def _synthetic(arch, layers, n, chunk, kv, seed, std=0.08, **over):
    cfg = synth.config(arch, icl_num_blocks=layers, **over)
    wt = synth.weights(cfg, seed=seed, std=std)
    m = oracle.Model({k: v for k, v in wt.items() if k.startswith("icl_predictor.")}, cfg["icl_nhead"], layers,
                     cfg["max_classes"])
    h = synth.row_reps(n, m.d, seed + 1)
    y = synth.labels(n, 10, seed + 2)
    caches, scales = oracle.icl_fit(m, h, y, chunk, kv)
    return cfg, wt, m, caches, scales


def _weights(gpu, cfg, wt, for_fit=False):
    return tcu.GpuWeights.from_tensors(gpu, synth.icl_shape(cfg), {k: v for k, v in wt.items() if k.startswith("icl_")},
                                       for_fit=for_fit)


CASES = [
    # arch, layers, training rows, chunk, head count override
    ("tiny", 2, 200, 48, {}),            # config 1 shape: d 32, 2 heads of 16
    ("tiny", 2, 333, 37, {}),            # odd chunk: rows of the stored chunk not 16-byte aligned
    ("full", 2, 700, 256, {}),           # d 512, 4 heads of 128, ragged last chunk of 188
    ("full", 1, 300, 8, {"icl_nhead": 8}),  # heads of 64, smallest chunk
]


@pytest.mark.parametrize("case", range(len(CASES)))
@pytest.mark.parametrize("kv", [0, 1, 2])
def test_stage_synthetic(gpu, case, kv):
    arch, layers, n, chunk, over = CASES[case]
    cfg, wt, m, caches, scales = _synthetic(arch, layers, n, chunk, kv, seed=10 + case, **over)
    w = _weights(gpu, cfg, wt)
    vm = tcu.VramModel.from_parts(w, _meta(n, chunk, kv, 10), n, 10, scales, caches)
    for rows in (1, 5, 9, 33, 70):
        h = synth.row_reps(rows, m.d, 100 + rows)
        got = vm.stage(h, 10)
        want = oracle.in_context(m, kv, caches, scales, n, chunk, h, 10)
        assert np.abs(got - want).max() < STAGE, (rows, np.abs(got - want).max())
        assert np.abs(softmax(got) - softmax(want)).max() < PROBA


@pytest.mark.parametrize("kv", [0, 1, 2])
def test_few_rows_run_as_one_kernel(gpu, kv):
    """Up to 8 rows at head widths 64/128 take the one-kernel stage: one launch per call, every row count 1..8
    within the stage bar of the CPU path, and bit-identical when repeated."""
    n, chunk = 1000, 256   # 16-byte aligned chunks (bulk-copied tiles) and a ragged last chunk of 232 rows
    cfg, wt, m, caches, scales = _synthetic("full", 2, n, chunk, kv, seed=60 + kv)
    w = _weights(gpu, cfg, wt)
    vm = tcu.VramModel.from_parts(w, _meta(n, chunk, kv, 10), n, 10, scales, caches)
    for rows in range(1, 9):
        h = synth.row_reps(rows, m.d, 70 + rows)
        before = gpu.launches
        got = vm.stage(h, 10)
        assert gpu.launches - before == 1, gpu.launches - before
        want = oracle.in_context(m, kv, caches, scales, n, chunk, h, 10)
        assert np.abs(got - want).max() < STAGE, (rows, np.abs(got - want).max())
        assert np.abs(softmax(got) - softmax(want)).max() < PROBA
        assert np.array_equal(vm.stage(h, 10), got)


def test_rows_are_independent(gpu):
    """A row's answer does not depend on the rows predicted with it (tests/pipeline.rs:122-135)."""
    cfg, wt, m, caches, scales = _synthetic("full", 2, 500, 256, 1, seed=5)
    w = _weights(gpu, cfg, wt)
    vm = tcu.VramModel.from_parts(w, _meta(500, 256, 1, 10), 500, 10, scales, caches)
    h = synth.row_reps(150, m.d, 7)
    all_rows = vm.stage(h, 10)
    for lo, hi in [(0, 1), (10, 14), (40, 80), (149, 150)]:
        part = vm.stage(h[lo:hi], 10)
        # few rows take the keys-parallel path, many the row-blocked one: sums in another order
        assert np.abs(part - all_rows[lo:hi]).max() < STAGE
        assert np.abs(softmax(part) - softmax(all_rows[lo:hi])).max() < 1e-6


def test_graph_replays_and_regrowth(gpu):
    """The stage is captured as a CUDA graph per row count and replayed; growing the working memory for a larger
    call must not leave earlier graphs pointing at freed buffers."""
    cfg, wt, m, caches, scales = _synthetic("full", 2, 400, 256, 1, seed=41)
    w = _weights(gpu, cfg, wt)
    vm = tcu.VramModel.from_parts(w, _meta(400, 256, 1, 10), 400, 10, scales, caches)
    h5, h70 = synth.row_reps(5, m.d, 42), synth.row_reps(70, m.d, 43)
    first = vm.stage(h5, 10)
    assert np.array_equal(vm.stage(h5, 10), first)      # replay
    big = vm.stage(h70, 10)                              # buffers grow: graphs dropped
    assert np.array_equal(vm.stage(h5, 10), first)      # recaptured on the new buffers
    assert np.abs(big - oracle.in_context(m, 1, caches, scales, 400, 256, h70, 10)).max() < STAGE
    assert np.abs(vm.stage(h5, 3) - first[:, :3]).max() == 0.0  # fewer outputs: its own graph


def test_regression_outputs(gpu):
    """The regression model's quantile decoder (999 outputs) through the stage."""
    cfg = synth.config("tiny", regression=True)
    wt = synth.weights(cfg, seed=21, std=0.08)
    m = oracle.Model({k: v for k, v in wt.items() if k.startswith("icl_predictor.")}, cfg["icl_nhead"], 2, 0)
    h = synth.row_reps(150, m.d, 22)
    y = np.random.default_rng(23).normal(0, 1, 150).astype(np.float32)
    caches, scales = oracle.icl_fit(m, h, y, 64, 1)
    w = _weights(gpu, cfg, wt)
    vm = tcu.VramModel.from_parts(w, _meta(150, 64, 1, 999), 150, 999, scales, caches)
    ht = synth.row_reps(6, m.d, 24)
    got = vm.stage(ht, 999)
    want = oracle.in_context(m, 1, caches, scales, 150, 64, ht, 999)
    assert np.abs(got - want).max() < STAGE


# ---- fitting's in-context stage and the packer on the device -----------------------------------------------

@pytest.mark.parametrize("kv", [0, 1, 2])
def test_pack_is_bit_exact(gpu, kv):
    import torch
    rng = np.random.default_rng(kv)
    for d, rc in [(16, 48), (512, 256), (32, 37), (8, 1)]:
        c = rng.normal(0, 1, (2 * d, rc)).astype(np.float32)
        c[0] = 0.0                                   # all-zero coordinate: scale 1
        c[1, :] = np.arange(rc) - rc / 2             # halves: ties round away from zero
        if rc > 3:
            c[2, :3] = [np.nan, 1e-30, -1e-30]
        want = oracle.pack(kv, d, c)
        dc = torch.from_numpy(c).cuda()
        out = torch.zeros(tcu.record(kv, d, rc), dtype=torch.uint8, device="cuda")
        gpu.pack(kv, d, rc, dc.data_ptr(), out.data_ptr())
        got = out.cpu().numpy()
        assert np.array_equal(got, want), (d, rc)


@pytest.mark.parametrize("kv", [0, 1, 2])
def test_integer_unpacking_is_bit_exact(gpu, kv):
    """predict.rs:590-629 layer_rows through the device's own widening (the vector unpack the attention kernels
    read the cache with): equal bit for bit to the CPU path, with full 16-byte-aligned chunks, ragged last chunks,
    and chunks whose rows are not 16-byte aligned."""
    import torch
    rng = np.random.default_rng(30 + kv)
    for d, rows, chunk in [(512, 700, 256), (32, 333, 37), (16, 101, 48), (64, 9, 8)]:
        k = (rng.standard_normal((rows, d)) * rng.uniform(0.1, 30, (1, d))).astype(np.float32)
        v = (rng.standard_normal((rows, d)) * rng.uniform(0.1, 30, (1, d))).astype(np.float32)
        k[:, 0] = 0.0                       # an all-zero coordinate: scale 1
        v[:, 1] = np.round(v[:, 1])         # exact integers and halves
        layer = oracle.pack_layer(kv, d, k, v, chunk)
        wk, wv = oracle.layer_rows(kv, d, layer, rows, chunk)
        ld = torch.from_numpy(np.frombuffer(bytes(layer), np.uint8).copy()).cuda()
        gk = torch.full((rows, d), float("nan"), device="cuda")
        gv = torch.full((rows, d), float("nan"), device="cuda")
        gpu.layer_rows(kv, d, ld.data_ptr(), rows, chunk, gk.data_ptr(), gv.data_ptr())
        assert np.array_equal(gk.cpu().numpy().view(np.uint32), wk.view(np.uint32)), (d, rows, chunk)
        assert np.array_equal(gv.cpu().numpy().view(np.uint32), wv.view(np.uint32)), (d, rows, chunk)


@pytest.mark.parametrize("kv", [0, 1, 2])
def test_fit_on_device_matches_oracle(gpu, kv):
    import torch
    cfg = synth.config("full", icl_num_blocks=2)
    wt = synth.weights(cfg, seed=31, std=0.08)
    m = oracle.Model({k: v for k, v in wt.items() if k.startswith("icl_predictor.")}, cfg["icl_nhead"], 2, 10)
    n, chunk = 600, 256
    h = synth.row_reps(n, m.d, 32)
    y = synth.labels(n, 10, 33)
    want_layers, want_scales = oracle.icl_fit(m, h, y, chunk, kv)
    w = _weights(gpu, cfg, wt, for_fit=True)
    hd, yd = torch.from_numpy(h.copy()).cuda(), torch.from_numpy(y).cuda()
    vm = tcu.fit_icl(w, hd.data_ptr(), yd.data_ptr(), n, chunk, kv)
    assert np.array_equal(vm.scales(), want_scales)
    nbytes = oracle.layer_len(kv, m.d, n, chunk)
    for l in range(2):
        got = vm.layer_bytes(l, nbytes)
        gk, gv = oracle.layer_rows(kv, m.d, got, n, chunk)
        wk, wv = oracle.layer_rows(kv, m.d, want_layers[l], n, chunk)
        # f32 sums in another order; integers may then round to the neighbouring step
        step = {0: 0.0, 1: 1.0 / 32767, 2: 1.0 / 127}[kv] * max(np.abs(wk).max(), np.abs(wv).max())
        assert np.abs(gk - wk).max() < 1e-4 + 1.01 * step
        assert np.abs(gv - wv).max() < 1e-4 + 1.01 * step
    ht = synth.row_reps(5, m.d, 34)
    got = vm.stage(ht, 10)
    dev_layers = [vm.layer_bytes(l, nbytes) for l in range(2)]
    want = oracle.in_context(m, kv, dev_layers, want_scales, n, chunk, ht, 10)
    assert np.abs(got - want).max() < STAGE


# ---- heads -------------------------------------------------------------------------------------------------

def test_class_head(gpu):
    import torch
    rng = np.random.default_rng(1)
    rows, classes, members = 257, 10, 3
    sums_want = np.zeros((rows, classes))
    sums = torch.zeros((rows, classes), dtype=torch.float64, device="cuda")
    for i in range(members):
        logits = rng.normal(0, 2, (rows, classes)).astype(np.float32)
        mc = np.array([(c + classes - i) % classes for c in range(classes)], np.int32)
        oracle.add_member(sums_want, logits, mc)
        lt, mt = torch.from_numpy(logits).cuda(), torch.from_numpy(mc).cuda()
        gpu.class_head(lt.data_ptr(), rows, classes, classes, mt.data_ptr(), sums.data_ptr(), finish=(i == members - 1),
                       members=members, temperature=0.9)
    want = oracle.finish_proba(sums_want, members, 0.9)
    assert np.abs(sums.cpu().numpy() - want).max() < 1e-12


def test_regression_head(gpu):
    import torch
    rng = np.random.default_rng(2)
    rows, nq = 300, 999
    alphas = np.array([0.05, 0.5, 0.95, 0.0001], np.float64)
    q = (rng.normal(0, 1, (rows, nq)) * rng.uniform(0.1, 3, (rows, 1)) + rng.normal(0, 1, (rows, 1))).astype(np.float32)
    want = oracle.regression_add(q, alphas, 50.0, 7.0)
    dq, da = torch.from_numpy(q).cuda(), torch.from_numpy(alphas).cuda()
    out = {k: torch.zeros(rows, dtype=torch.float64, device="cuda") for k in ("mean", "variance", "median")}
    qs = torch.zeros((rows, alphas.size), dtype=torch.float64, device="cuda")
    gpu.regression_head(dq.data_ptr(), rows, nq, nq, da.data_ptr(), alphas.size, 50.0, 7.0, out["mean"].data_ptr(),
                        out["variance"].data_ptr(), out["median"].data_ptr(), qs.data_ptr())
    spread = 7.0
    assert np.abs(out["mean"].cpu().numpy() - want["mean"]).max() < 1e-5 * spread
    assert np.abs(out["median"].cpu().numpy() - want["median"]).max() < 1e-5 * spread
    assert np.abs(qs.cpu().numpy() - want["quantiles"]).max() < 1e-5 * spread
    assert np.abs(out["variance"].cpu().numpy() - want["variance"]).max() < 1e-4 * spread


# ---- the boundary's error behaviour ------------------------------------------------------------------------

def test_errors_are_statuses(gpu, tiny):
    t = tiny
    w = tcu.GpuWeights.from_bundle(gpu, t["path"])
    lib = tcu.lib()
    import ctypes
    h = ctypes.c_void_p()
    meta = (ctypes.c_int32 * 7)(t["n"], 7, 3, 48, 0, 1, 1)
    assert lib.tcu_model_new(w._h, meta, t["n"], 3, ctypes.byref(h)) == tcu.OK
    vm = tcu.VramModel(w, h)
    x = np.zeros((2, t["m"].d), np.float32)
    with pytest.raises(tcu.TcuError) as e:
        vm.stage(x, 3)  # nothing put yet
    assert e.value.code == -5 and "never put" in gpu.last_error
    big = np.zeros(10, np.uint8)
    assert lib.tcu_model_put_layer(h, 0, 10 ** 9, big.ctypes.data, 10) == -1
    assert lib.tcu_model_put_layer(h, 9, 0, big.ctypes.data, 10) == -1
    meta_bad = (ctypes.c_int32 * 7)(t["n"], 7, 3, 48, 3, 1, 1)  # Kv code 3 does not exist (fit.rs:120-122)
    assert lib.tcu_model_new(w._h, meta_bad, t["n"], 3, ctypes.byref(ctypes.c_void_p())) == -2
    with pytest.raises(tcu.TcuError):
        tcu.GpuWeights.from_tensors(gpu, dict(d=16, heads=2, layers=1, ff=32, hid=64, dec_ff=32, outs=10, max_classes=10), {})
    with pytest.raises(tcu.TcuError):
        tcu.GpuWeights.from_bundle(gpu, GOLDEN + "/does-not-exist.tirs")
