"""Pin the oracle (the C restatement of tabicl-anywhere's CPU path) to the reference's own golden vectors and
known-answer tests, before it is trusted as the checker of the device path.

* tests/golden/tiny-raw-icl.tirs is PyTorch TabICL's dump for the reference's tiny classifier: row
  representations, every layer's in-context keys/values and the logits. The reference's own test compares its
  CPU path with it at TINY = 5e-5 (tests/reference.rs:107-116, 145-148).
* Known answers of kern.rs:383-392, 395-402, 521-528 and the streaming-softmax tests of nn.rs:483-540.
"""
import math

import numpy as np
import pytest

import oracle

TINY = 5e-5  # tests/reference.rs:148


def _layers(t, kv, chunk):
    return [oracle.pack_layer(kv, t["m"].d, t["k"][l], t["v"][l], chunk) for l in range(t["m"].layers)]


@pytest.mark.parametrize("chunk", [48, 7, 120, 256])
def test_in_context_matches_pytorch_logits(tiny, chunk):
    """predict.rs:381-586 on PyTorch's keys/values reproduces PyTorch's logits (tests/reference.rs:107-116)."""
    t = tiny
    classes = t["logits"].shape[1]
    got = oracle.in_context(t["m"], 0, _layers(t, 0, chunk), t["scales"], t["n"], chunk, t["test_rep"], classes)
    bad = np.abs(got - t["logits"]).max()
    assert bad < TINY, bad


def test_key_threads_merge_matches(tiny):
    """key_threads readers merged by Soft::merge: same answers within rounding (tests/pipeline.rs:103-119)."""
    t = tiny
    c = t["logits"].shape[1]
    one = oracle.in_context(t["m"], 0, _layers(t, 0, 16), t["scales"], t["n"], 16, t["test_rep"], c)
    four = oracle.in_context(t["m"], 0, _layers(t, 0, 16), t["scales"], t["n"], 16, t["test_rep"], c, parts=4)
    assert np.abs(one - four).max() < 1e-6


@pytest.mark.parametrize("kv,bound", [(1, 1e-4), (2, 1e-2)])
def test_integer_caches_stay_close(tiny, kv, bound):
    """i16 within 1e-4 and i8 within 1e-2 of the float answers (tests/pipeline.rs:138-156, README.md:103-105)."""
    t = tiny
    c = t["logits"].shape[1]
    f = oracle.in_context(t["m"], 0, _layers(t, 0, 48), t["scales"], t["n"], 48, t["test_rep"], c)
    q = oracle.in_context(t["m"], kv, _layers(t, kv, 48), t["scales"], t["n"], 48, t["test_rep"], c)
    assert np.abs(q - f).max() < bound


def test_icl_fit_matches_pytorch_keys_values(tiny):
    """fit.rs:577-747 from PyTorch's training row representations gives PyTorch's keys and values of every layer
    (tests/reference.rs:79-99 at 2.5 x TINY)."""
    t = tiny
    fx, m = t["fx"], t["m"]
    layers, scales = oracle.icl_fit(m, fx["train_rep"], fx["y_train"], 48, 0)
    for l in range(m.layers):
        k, v = oracle.layer_rows(0, m.d, layers[l], t["n"], 48)
        assert np.abs(k - t["k"][l]).max() < 2.5 * TINY, l
        assert np.abs(v - t["v"][l]).max() < 2.5 * TINY, l
    assert np.array_equal(scales, t["scales"])


def test_exp_erf_tanh_gelu_known_answers():
    lib = oracle.lib()
    xs = np.arange(-80.0, 80.0, 0.0137, dtype=np.float32)
    rel = max(abs(lib.or_exp1(float(x)) - math.exp(float(x))) / math.exp(float(x)) for x in xs[::7])
    assert rel < 2e-7  # kern.rs:383-392
    for x in np.arange(-6.0, 6.0, 0.0171, dtype=np.float32):
        assert abs(lib.or_erf1(float(x)) - math.erf(float(x))) < 3e-7  # kern.rs:395-402
        assert abs(lib.or_tanh1(float(x)) - math.tanh(float(x))) < 4e-7
    want = [-0.0, -0.15865525, 0.0, 0.0539828, 0.8413447, 10.0]  # kern.rs:521-528
    for x, w in zip([-10.0, -1.0, 0.0, 0.1, 1.0, 10.0], want):
        assert abs(lib.or_gelu1(x) - w) < 1e-6
    assert lib.or_exp1(-1000.0) == lib.or_exp1(-87.0) and math.isfinite(lib.or_exp1(1000.0))
    assert lib.or_tanh1(100.0) == lib.or_tanh1(10.0) and abs(lib.or_tanh1(-0.5) + 0.46211716) < 1e-6


def _plain_attention(q, k, v, heads):
    """Softmax attention in f64, keys/values row by row (tests/accel.rs:20-36)."""
    n, d = k.shape
    hd = d // heads
    out = np.zeros((q.shape[0], d))
    for h in range(heads):
        s = q[:, h * hd:(h + 1) * hd].astype(np.float64) @ k[:, h * hd:(h + 1) * hd].T.astype(np.float64)
        w = np.exp(s - s.max(axis=1, keepdims=True))
        out[:, h * hd:(h + 1) * hd] = (w @ v[:, h * hd:(h + 1) * hd].astype(np.float64)) / w.sum(axis=1, keepdims=True)
    return out


def _data(n, seed):
    return np.array([((i + seed) * 7919 % 2003 - 1001) * 2e-3 for i in range(n)], np.float32)


@pytest.mark.parametrize("chunk", [37, 1, 10, 36])
def test_streaming_softmax_in_any_pieces(chunk):
    """nn.rs:483-515: the running softmax over keys in pieces equals plain attention; merged halves too."""
    d, heads, r = 16, 4, 37
    q = _data(d, 1)[None, :]
    k, v = _data(d * r, 2).reshape(r, d), _data(d * r, 3).reshape(r, d)
    want = _plain_attention(q, k, v, heads)
    layer = oracle.pack_layer(0, d, k, v, chunk)
    for parts in (1, 2, 3):
        got = oracle.attend(0, d, heads, layer, r, chunk, q, parts=parts)
        assert np.abs(got - want).max() < 1e-5


def test_integer_keys_and_values():
    """nn.rs:518-540: i16 keys/values with per-coordinate scales against f64 attention of what they stand for."""
    d, heads, r = 8, 2, 13
    rng = np.random.default_rng(4)
    k, v = rng.normal(0, 0.3, (r, d)).astype(np.float32), rng.normal(0, 0.5, (r, d)).astype(np.float32)
    q = rng.normal(0, 1, (3, d)).astype(np.float32)
    for kv, bound in [(1, 1e-4), (2, 1e-2)]:
        layer = oracle.pack_layer(kv, d, k, v, r)
        kw, vw = oracle.layer_rows(kv, d, layer, r, r)
        got = oracle.attend(kv, d, heads, layer, r, r, q)
        assert np.abs(got - _plain_attention(q, kw, vw, heads)).max() < 1e-5
        assert np.abs(got - _plain_attention(q, k, v, heads)).max() < bound


def test_pack_known_answers():
    """fit.rs:549-576: per-coordinate scale max|x| / 32767 (or / 127), 1 when all zero; round half away from 0."""
    d = 2
    c = np.array([[0.0, 0.0, 0.0], [1.0, -0.5, 0.25], [3.0, -3.0, 1.5], [-2.0, 1.0, 0.0]], np.float32)
    rec = oracle.pack(1, d, c)
    sc = np.frombuffer(rec[:16].tobytes(), np.float32)
    body = np.frombuffer(rec[16:].tobytes(), np.int16).reshape(4, 3)
    assert sc[0] == 1.0 and sc[1] == np.float32(1.0) / np.float32(32767.0)
    assert body[0].tolist() == [0, 0, 0]
    assert body[1].tolist() == [32767, -16384, 8192]  # -0.5 * 32767 = -16383.5 rounds away from zero
    assert body[2].tolist() == [32767, -32767, 16384]
    rec8 = oracle.pack(2, d, c)
    b8 = np.frombuffer(rec8[16:].tobytes(), np.int8).reshape(4, 3)
    assert b8[1].tolist() == [127, -64, 32]  # -63.5 -> -64
    assert oracle.record(2, 512, 255) == 2 * 512 * 255 + 8 * 512
    assert oracle.record(0, 512, 256) == 2 * 512 * 256 * 4


def test_finish_proba_and_member_sums():
    """table.rs:70-78 and 265-269 against a direct numpy restatement."""
    rng = np.random.default_rng(0)
    sums = np.zeros((5, 3))
    for mc in ([0, 1, 2], [2, 0, 1]):
        logits = rng.normal(0, 2, (5, 10)).astype(np.float32)
        oracle.add_member(sums, logits, mc)
    want_sums = sums.copy()
    p = oracle.finish_proba(sums, 2, 0.9)
    z = (want_sums - want_sums.max(1, keepdims=True)) / (2 * 0.9)
    want = np.exp(z) / np.exp(z).sum(1, keepdims=True)
    assert np.abs(p - want).max() < 1e-15
    assert np.allclose(p.sum(1), 1.0)


def _qdist_numpy(q, alphas):
    """table.rs:292-346 written again in float32 numpy, for cross-checking the C restatement."""
    f = np.float32
    q = np.sort(np.asarray(q, f))
    n = q.size
    lv = (np.arange(1, n + 1, dtype=f) / f(n + 1)).astype(f)
    k = max(1, min(20, n // 4))

    def slope(xs, ys):
        mx, my = f(np.add.reduce(xs, dtype=f) / f(k)), f(np.add.reduce(ys, dtype=f) / f(k))
        cov = f(sum(f((x - mx) * (y - my)) for x, y in zip(xs, ys)) / f(k))
        var = f(sum(f((x - mx) * (x - mx)) for x in xs) / f(k))
        return f(min(max(abs(cov / max(var, f(1e-6))), f(0.01)), f(100.0)))

    bl = slope(np.log(np.maximum(lv[:k], f(1e-6))).astype(f), q[:k])
    br = slope(np.log(np.maximum(f(1) - lv[n - k:], f(1e-6))).astype(f), q[n - k:])
    tl = (bl, q[0] - bl * f(np.log(max(lv[0], f(1e-6)))))
    tr = (-br, q[n - 1] + br * f(np.log(f(1) - min(lv[n - 1], f(1 - 1e-6)))))

    def icdf(a):
        a = f(a)
        if a < lv[0]:
            return tl[0] * f(np.log(max(a, f(1e-6)))) + tl[1]
        if a > lv[n - 1]:
            return tr[0] * f(np.log(max(f(1) - a, f(1e-6)))) + tr[1]
        if a >= lv[n - 1]:
            return q[n - 1]
        i = max(int(np.searchsorted(lv[:n - 1], a, side="right")) - 1, 0)
        i = min(i, n - 2)
        t = min(max((a - lv[i]) / max(lv[i + 1] - lv[i], f(1e-6)), f(0)), f(1))
        return q[i] + t * (q[i + 1] - q[i])

    mean = f(0)
    for v in q:
        mean = f(mean + v)
    mean = f(mean / f(n))
    return mean, icdf(0.5), [icdf(a) for a in alphas]


def test_quantile_distribution():
    rng = np.random.default_rng(3)
    alphas = [0.0005, 0.05, 0.5, 0.95, 0.9995]
    qout = np.stack([rng.normal(0, 1, 999) * (1 + r) for r in range(4)] + [np.linspace(-3, 3, 999)]).astype(np.float32)
    acc = oracle.regression_add(qout, alphas, 50.0, 2.0)
    for r in range(qout.shape[0]):
        mean, med, qs = _qdist_numpy(qout[r], alphas)
        assert abs(acc["mean"][r] - (float(mean) * 2.0 + 50.0)) < 1e-4
        assert abs(acc["median"][r] - (float(med) * 2.0 + 50.0)) < 1e-4
        for a in range(len(alphas)):
            assert abs(acc["quantiles"][r, a] - (float(qs[a]) * 2.0 + 50.0)) < 1e-3
    # a straight line of quantiles: the median is its middle
    assert abs(acc["median"][4] - 50.0) < 1e-5


# ---- the column and row stages (predict.rs:282-372) against PyTorch's numbers ------------------------------------

TINY = 5e-5  # tests/reference.rs:148


def test_column_stage_matches_reference(tiny):
    """embed on the dump's normalised test rows and its column-stage cache gives the dump's test embeddings
    (the feature cells; tests/reference.rs:96-105 compares the same part), the class tokens first."""
    t = tiny
    rm = t["rm"]
    tok = oracle.embed(rm, t["x_test"], t["col_kv"])
    assert np.abs(tok[:, rm.cls:] - t["test_emb"][:, rm.cls:]).max() < TINY
    assert np.array_equal(tok[:, :rm.cls], np.broadcast_to(np.asarray(t["wb"]["row_interactor.cls_tokens"]).reshape(rm.cls, rm.e), tok[:, :rm.cls].shape))


def test_row_stage_matches_reference(tiny):
    t = tiny
    rm = t["rm"]
    tok = oracle.embed(rm, t["x_test"], t["col_kv"])
    rep = oracle.represent(rm, tok)
    assert np.abs(rep - t["test_rep"]).max() < TINY


def test_normalised_rows_to_logits(tiny):
    """The whole prediction of one member from normalised features: column stage, row stage, in-context stage on
    the dump's in-context cache, against the dump's logits (tests/reference.rs:107-116)."""
    t = tiny
    rm, m = t["rm"], t["m"]
    rep = oracle.represent(rm, oracle.embed(rm, t["x_test"], t["col_kv"]))
    layers = [oracle.pack_layer(0, m.d, t["k"][l], t["v"][l], 48) for l in range(m.layers)]
    logits = oracle.in_context(m, 0, layers, t["scales"], t["n"], 48, rep, t["logits"].shape[1])
    assert np.abs(logits - t["logits"]).max() < TINY


def test_digit_average_of_identical_caches_is_the_plain_stage(tiny):
    """With several label digits the column stage runs once per digit and averages (predict.rs:326-346): the same
    cache for every digit gives the one-digit answer up to the average's rounding."""
    t = tiny
    rm = t["rm"]
    one = oracle.embed(rm, t["x_test"], t["col_kv"])
    ck = t["col_kv"]
    three = np.concatenate([ck, ck, ck], axis=1)
    got = oracle.embed(rm, t["x_test"], three, digits=3)
    assert np.abs(got - one).max() < 1e-5


def test_column_fit_matches_reference(tiny):
    """fit.rs:298-420 on the dump's normalised training rows and labels (FitOpts chunk 48, tests/reference.rs:42-72)
    gives the dump's column-stage cache (tests/reference.rs:79-95), its training embeddings, and through the row
    stage its training row representations."""
    t = tiny
    rm, fx = t["rm"], t["fx"]
    x, y = np.array(fx["x_train"], np.float32), np.array(fx["y_train"], np.float32)
    col_kv, tok = oracle.fit_columns(rm, x, y, 48)
    assert np.abs(col_kv - t["col_kv"]).max() < TINY
    emb = np.array(fx["train_emb"], np.float32)
    assert np.abs(tok[:, rm.cls:] - emb[:, rm.cls:]).max() < TINY
    rep = oracle.represent(rm, tok)
    assert np.abs(rep - np.array(fx["train_rep"], np.float32)).max() < TINY
