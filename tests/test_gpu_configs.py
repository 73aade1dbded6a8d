"""Parity at the configurations the benchmark times, through the C ABI.

Each case builds the configuration's cache the way bench.py does (the full-size architecture's random-init
weights, seeded training rows fitted on the device), copies the stored cache bytes back, and runs the oracle's
in-context stage on those same bytes and rows. Bars as everywhere else: raw decoder scores within 5e-5 per cached
stage, class probabilities within 1e-5; regression outputs through the quantile head within 1e-5 of the spread
when the head reads the same scores, and within 5e-5 of the spread end to end.

Sizes: config 2 is compared on all 2,048 rows of the timed call (the oracle takes about 3 s for them on the GPU
box's host cores), and on 1, 8, 64, 200 and 256 rows, which cover the one-kernel stage, the split-K decode and
per-row query-MLP kernels, the tensor-core query MLP (above 128 rows) and the 128-row tensor-core tiles. Config 4's
100,000-row i8 cache is compared on 64 and 256 rows, config 3's f32 cache on 300 rows, config 5's 50,000-row
regressor on 128 rows.
"""
import numpy as np
import pytest

from conftest import synth, tcu
import oracle

pytestmark = pytest.mark.gpu

STAGE = 5e-5
PROBA = 1e-5
CHUNK = 256


def softmax(x, t=0.9):
    z = (x - x.max(1, keepdims=True)) / t
    e = np.exp(z)
    return e / e.sum(1, keepdims=True)


@pytest.fixture(scope="module")
def gpu():
    g = tcu.Gpu(0)
    yield g
    g.close()


class Full:
    """The full-size architecture (configs 2-5) on the device and in the oracle."""

    def __init__(self, gpu, regression=False, seed=0):
        cfg = synth.config("full", regression=regression)
        wt = synth.weights(cfg, seed=seed)
        self.shape = synth.icl_shape(cfg)
        icl = {k: v for k, v in wt.items() if k.startswith("icl_")}
        self.w = tcu.GpuWeights.from_tensors(gpu, self.shape, icl, for_fit=True)
        self.m = oracle.Model({k: v for k, v in icl.items() if k.startswith("icl_predictor.")}, cfg["icl_nhead"],
                              cfg["icl_num_blocks"], cfg["max_classes"])
        self.d = self.shape["d"]

    def fit(self, rows, kv, seed, classes=10):
        import torch
        h = torch.from_numpy(synth.row_reps(rows, self.d, seed)).cuda()
        if classes:
            y = synth.labels(rows, classes, seed + 1)
        else:
            y = np.random.default_rng(seed + 1).standard_normal(rows).astype(np.float32)
        yd = torch.from_numpy(y).cuda()
        vm = tcu.fit_icl(self.w, h.data_ptr(), yd.data_ptr(), rows, CHUNK, kv)
        del h, yd
        nbytes = oracle.layer_len(kv, self.d, rows, CHUNK)
        layers = [vm.layer_bytes(l, nbytes) for l in range(self.m.layers)]
        return vm, layers, vm.scales()

    def free(self):
        self.w.free()


def _stage_device(vm, h, out_n):
    """The stage on device buffers (tcu_stage_device), as the benchmark's timed step calls it."""
    import torch
    hd = torch.from_numpy(np.ascontiguousarray(h)).cuda()
    out = torch.empty((h.shape[0], out_n), device="cuda")
    vm.stage_device(hd.data_ptr(), h.shape[0], out_n, out.data_ptr())
    vm.gpu.sync()
    return out.cpu().numpy()


def test_config2_full_shape(gpu):
    """Config 2: 12 layers, d 512, 10,000 training rows, i16 cache; the timed 2,048-row call and the other call
    sizes, through both the device-buffer and the host-buffer entry points."""
    f = Full(gpu)
    n = 10000
    vm, layers, scales = f.fit(n, 1, seed=1)
    h = synth.row_reps(2048, f.d, 100)
    got = _stage_device(vm, h, 10)
    want = oracle.in_context(f.m, 1, layers, scales, n, CHUNK, h, 10)
    worst = np.abs(got - want).max()
    assert worst < STAGE, worst
    assert np.abs(softmax(got) - softmax(want)).max() < PROBA
    for rows in (1, 8, 64, 200, 256):
        part = vm.stage(h[:rows], 10)
        assert np.abs(part - want[:rows]).max() < STAGE, (rows, np.abs(part - want[:rows]).max())
        assert np.abs(softmax(part) - softmax(want[:rows])).max() < PROBA
    vm.free()
    f.free()


def test_config2_query_mlp_above_128_rows(gpu):
    """Calls of 129-300 rows take the tensor-core query MLP and 128-row tensor-core linear tiles with a partial
    last tile: compared with the oracle directly (2 layers of the full-size width keep the oracle quick)."""
    cfg = synth.config("full", icl_num_blocks=2)
    wt = synth.weights(cfg, seed=7)
    icl = {k: v for k, v in wt.items() if k.startswith("icl_")}
    w = tcu.GpuWeights.from_tensors(gpu, synth.icl_shape(cfg), icl, for_fit=True)
    m = oracle.Model({k: v for k, v in icl.items() if k.startswith("icl_predictor.")}, cfg["icl_nhead"], 2, 10)
    import torch
    n = 2500
    hd = torch.from_numpy(synth.row_reps(n, m.d, 8)).cuda()
    yd = torch.from_numpy(synth.labels(n, 10, 9)).cuda()
    vm = tcu.fit_icl(w, hd.data_ptr(), yd.data_ptr(), n, CHUNK, 1)
    nbytes = oracle.layer_len(1, m.d, n, CHUNK)
    layers = [vm.layer_bytes(l, nbytes) for l in range(2)]
    scales = vm.scales()
    for rows in (129, 191, 300):
        h = synth.row_reps(rows, m.d, 200 + rows)
        got = vm.stage(h, 10)
        want = oracle.in_context(m, 1, layers, scales, n, CHUNK, h, 10)
        assert np.abs(got - want).max() < STAGE, (rows, np.abs(got - want).max())
        assert np.abs(softmax(got) - softmax(want)).max() < PROBA
    vm.free()
    w.free()


def test_config3_f32_cache(gpu):
    """Config 3's member: the f32 cache of 10,000 rows (3 f16 products per term on the tensor cores)."""
    f = Full(gpu)
    n = 10000
    vm, layers, scales = f.fit(n, 0, seed=300)
    h = synth.row_reps(300, f.d, 500)
    got = _stage_device(vm, h, 10)
    want = oracle.in_context(f.m, 0, layers, scales, n, CHUNK, h, 10)
    assert np.abs(got - want).max() < STAGE, np.abs(got - want).max()
    assert np.abs(softmax(got) - softmax(want)).max() < PROBA
    vm.free()
    f.free()


def test_config4_large_i8_cache(gpu):
    """Config 4 on one device: the 100,000-row i8 cache (1.25 GB), 64 and 256 rows."""
    f = Full(gpu)
    n = 100000
    vm, layers, scales = f.fit(n, 2, seed=600)
    for rows in (64, 256):
        h = synth.row_reps(rows, f.d, 602 + rows)
        got = _stage_device(vm, h, 10)
        want = oracle.in_context(f.m, 2, layers, scales, n, CHUNK, h, 10)
        assert np.abs(got - want).max() < STAGE, (rows, np.abs(got - want).max())
        assert np.abs(softmax(got) - softmax(want)).max() < PROBA
    vm.free()
    f.free()


def test_config5_regressor(gpu):
    """Config 5: the regressor (999 quantile outputs) over a 50,000-row i16 cache, then the quantile head
    (mean, variance, median, 5% and 95%), against the oracle's stage and head (table.rs:292-346, 457-496)."""
    import torch
    f = Full(gpu, regression=True, seed=5)
    n = 50000
    vm, layers, scales = f.fit(n, 1, seed=700, classes=0)
    rows, nq = 128, 999
    h = synth.row_reps(rows, f.d, 701)
    got = _stage_device(vm, h, nq)
    want = oracle.in_context(f.m, 1, layers, scales, n, CHUNK, h, nq)
    assert np.abs(got - want).max() < STAGE, np.abs(got - want).max()
    alphas = np.array([0.05, 0.95], np.float64)
    tmean, tscale = 3.0, 2.5
    qd = torch.from_numpy(got).cuda()
    ad = torch.from_numpy(alphas).cuda()
    out = {k: torch.zeros(rows, dtype=torch.float64, device="cuda") for k in ("mean", "variance", "median")}
    qs = torch.zeros((rows, 2), dtype=torch.float64, device="cuda")
    gpu.regression_head(qd.data_ptr(), rows, nq, nq, ad.data_ptr(), 2, tmean, tscale, out["mean"].data_ptr(),
                        out["variance"].data_ptr(), out["median"].data_ptr(), qs.data_ptr())
    same = oracle.regression_add(got, alphas, tmean, tscale)       # the head on the same scores
    e2e = oracle.regression_add(want, alphas, tmean, tscale)       # the whole path on the CPU
    dev = {k: v.cpu().numpy() for k, v in out.items()}
    dev["quantiles"] = qs.cpu().numpy()
    for k in ("mean", "median", "quantiles"):
        assert np.abs(dev[k] - same[k]).max() < 1e-5 * tscale, k
        assert np.abs(dev[k] - e2e[k]).max() < STAGE * tscale, k
    assert np.all(dev["quantiles"][:, 0] <= dev["median"]) and np.all(dev["median"] <= dev["quantiles"][:, 1])
    vm.free()
    f.free()
