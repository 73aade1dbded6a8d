"""TEST INFRASTRUCTURE ONLY: Python binding of the parity oracle (tabicl_oracle.c), a plain-C restatement of
tabicl-anywhere's CPU prediction path. Used by tests/ as the checker, by __graft_entry__.smoke() to check one
small device call, and by bench.py's CPU-baseline leg. The product never imports this.

Parity pin: tests/test_oracle_golden.py checks it against the reference's golden vectors (PyTorch TabICL's
numbers, tests/golden/).
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "liboracle.so")
LIB_V3 = os.path.join(HERE, "_build", "liboracle_v3.so")


def _has_v3():
    """x86-64-v3 (AVX2, FMA, BMI1/2, F16C, MOVBE, LZCNT) on this host's CPU"""
    try:
        flags = set()
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    flags = set(line.split(":", 1)[1].split())
                    break
        return {"avx2", "fma", "bmi1", "bmi2", "f16c", "movbe", "abm"} <= flags
    except OSError:
        return False
_lib = None
_P = ctypes.POINTER
_fp = _P(ctypes.c_float)


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


class OrLayer(ctypes.Structure):
    _fields_ = [(n, _fp) for n in ("n1w", "n1b", "wq", "bq", "q0w", "q0b", "q2w", "q2b", "wo", "bo", "n2w", "n2b",
                                   "w1", "b1", "w2", "b2", "wkv", "bkv", "sb0w", "sb0b", "sb2w", "sb2b")]


class OrModel(ctypes.Structure):
    _fields_ = [("d", ctypes.c_int), ("heads", ctypes.c_int), ("ff", ctypes.c_int), ("hid", ctypes.c_int),
                ("layers", ctypes.c_int), ("dff", ctypes.c_int), ("outs", ctypes.c_int), ("max_classes", ctypes.c_int),
                ("layer", _P(OrLayer)), ("lnw", _fp), ("lnb", _fp), ("dec0w", _fp), ("dec0b", _fp), ("dec2w", _fp),
                ("dec2b", _fp), ("icl_y", _fp)]


class OrCBlock(ctypes.Structure):
    _fields_ = [(n, _fp) for n in ("n1w", "n1b", "inw", "inb", "ow", "ob", "n2w", "n2b", "w1", "b1", "w2", "b2")] + \
               [("ff", ctypes.c_int)]


class OrIsab1(ctypes.Structure):
    _fields_ = [("b", OrCBlock)] + [(n, _fp) for n in ("sb0w", "sb0b", "sb2w", "sb2b", "q0w", "q0b", "q2w", "q2b")] + \
               [("hid", ctypes.c_int), ("ind", _fp)]


class OrRowsModel(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("e", "group", "inds", "cls", "col_heads", "row_heads", "ncol", "nrow")] + \
               [("in_w", _fp), ("in_b", _fp), ("col", _P(OrCBlock)), ("cls_tokens", _fp), ("row", _P(OrCBlock)),
                ("rope_freqs", _fp), ("out_lnw", _fp), ("out_lnb", _fp), ("col1", _P(OrIsab1)), ("col_y", _fp),
                ("max_classes", ctypes.c_int)]


def lib():
    global _lib
    if _lib is None:
        src = os.path.getmtime(os.path.join(HERE, "tabicl_oracle.c"))
        if any(not os.path.exists(p) or os.path.getmtime(p) < src for p in (LIB, LIB_V3)):
            build()
        L = ctypes.CDLL(LIB_V3 if _has_v3() and os.environ.get("ORACLE_BASELINE_ISA") != "1" else LIB)
        v, i, f, sz, d = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_double
        M = _P(OrModel)
        sig = {
            "or_exp1": (f, [f]), "or_erf1": (f, [f]), "or_gelu1": (f, [f]), "or_tanh1": (f, [f]),
            "or_record": (sz, [i, i, i]),
            "or_query_scale": (None, [M, i, i, _fp]),
            "or_query": (None, [M, i, _fp, _fp, _fp]),
            "or_attend": (None, [i, i, i, v, i, i, _fp, i, i, _fp]),
            "or_in_context": (None, [M, i, _P(v), _fp, i, i, _fp, i, i, i, _fp]),
            "or_pack": (None, [i, i, i, _fp, v]),
            "or_layer_rows": (None, [i, i, v, i, i, _fp, _fp]),
            "or_add_y": (None, [M, _fp, i, _fp]),
            "or_icl_fit": (None, [M, _fp, i, i, i, _P(v), _fp]),
            "or_add_member": (None, [_P(d), _fp, i, i, i, _P(ctypes.c_int32)]),
            "or_finish_proba": (None, [_P(d), i, i, i, d]),
            "or_regression_add": (None, [_fp, i, i, i, _P(d), i, d, d, _P(d), _P(d), _P(d), _P(d)]),
            "or_embed": (None, [_P(OrRowsModel), _fp, i, i, _fp, i, _fp]),
            "or_represent": (None, [_P(OrRowsModel), _fp, i, i, _fp]),
            "or_fit_columns": (None, [_P(OrRowsModel), _fp, _fp, i, i, i, i, _P(ctypes.c_int32), _fp, _fp]),
            "or_ind_queries": (None, [_P(OrRowsModel), i, _fp]),
            "or_fit_cells": (None, [_P(OrRowsModel), _fp, _fp, i, i, _fp]),
            "or_threads": (i, []),
            "or_set_threads": (None, [i]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(_fp)


class Model:
    """The in-context part of a weight bundle as the oracle sees it (src/model.rs:27-143)."""

    def __init__(self, tensors, heads, layers, max_classes):
        g = lambda n: np.ascontiguousarray(tensors[n], dtype=np.float32).reshape(-1)
        self._keep = []
        d = g("icl_predictor.ln.weight").size
        keep = self._keep

        def k(a):
            a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
            keep.append(a)
            return _p(a)

        def opt(n, size):
            return g(n) if n in tensors else np.zeros(size, np.float32)

        arr = (OrLayer * layers)()
        for l in range(layers):
            b = f"icl_predictor.tf_icl.blocks.{l}."
            inw, inb = g(b + "attn.in_proj_weight"), g(b + "attn.in_proj_bias")
            s = b + "attn.ssmax_layer."
            L = arr[l]
            L.n1w, L.n1b = k(g(b + "norm1.weight")), k(opt(b + "norm1.bias", d))
            L.wq, L.bq = k(inw[:d * d]), k(inb[:d])
            L.q0w, L.q0b, L.q2w, L.q2b = (k(g(s + "query_mlp.0.weight")), k(g(s + "query_mlp.0.bias")),
                                          k(g(s + "query_mlp.2.weight")), k(g(s + "query_mlp.2.bias")))
            L.wo, L.bo = k(g(b + "attn.out_proj.weight")), k(g(b + "attn.out_proj.bias"))
            L.n2w, L.n2b = k(g(b + "norm2.weight")), k(opt(b + "norm2.bias", d))
            L.w1, L.b1 = k(g(b + "linear1.weight")), k(g(b + "linear1.bias"))
            L.w2, L.b2 = k(g(b + "linear2.weight")), k(g(b + "linear2.bias"))
            L.wkv, L.bkv = k(inw[d * d:]), k(inb[d:])
            L.sb0w, L.sb0b = k(g(s + "base_mlp.0.weight")), k(g(s + "base_mlp.0.bias"))
            L.sb2w, L.sb2b = k(g(s + "base_mlp.2.weight")), k(g(s + "base_mlp.2.bias"))
        self._layers = arr
        m = OrModel()
        m.d, m.heads, m.layers, m.max_classes = d, heads, layers, max_classes
        m.ff = g("icl_predictor.tf_icl.blocks.0.linear1.bias").size
        m.hid = g("icl_predictor.tf_icl.blocks.0.attn.ssmax_layer.query_mlp.0.bias").size
        m.dff = g("icl_predictor.decoder.0.bias").size
        m.outs = g("icl_predictor.decoder.2.bias").size
        m.layer = ctypes.cast(arr, _P(OrLayer))
        m.lnw, m.lnb = k(g("icl_predictor.ln.weight")), k(opt("icl_predictor.ln.bias", d))
        m.dec0w, m.dec0b = k(g("icl_predictor.decoder.0.weight")), k(g("icl_predictor.decoder.0.bias"))
        m.dec2w, m.dec2b = k(g("icl_predictor.decoder.2.weight")), k(g("icl_predictor.decoder.2.bias"))
        # model.rs:163-177 class_table
        yw, yb = g("icl_predictor.y_encoder.weight"), g("icl_predictor.y_encoder.bias")
        if max_classes > 0:
            t = yw.reshape(d, max_classes).T + yb[None, :]
        else:
            t = np.concatenate([yw, yb])
        m.icl_y = k(t)
        self.m = m
        self.d, self.heads, self.layers, self.max_classes = d, heads, layers, max_classes
        self.ff, self.hid, self.dff, self.outs = m.ff, m.hid, m.dff, m.outs

    @property
    def ref(self):
        return ctypes.byref(self.m)

    def query_scale(self, l, n):
        out = np.empty(self.d, np.float32)
        lib().or_query_scale(self.ref, l, n, _p(out))
        return out


class RowsModel:
    """The column and row stages of a weight bundle as the oracle sees them (src/model.rs:199-245: the column
    blocks' second attention, the class tokens, the row blocks, the rotary frequencies, the final LayerNorm)."""

    def __init__(self, tensors, cfg):
        g = lambda n: np.ascontiguousarray(tensors[n], dtype=np.float32).reshape(-1)
        self._keep = []
        keep = self._keep

        def k(a):
            a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
            keep.append(a)
            return _p(a)

        e = g("col_embedder.in_linear.bias").size

        def block(p):
            b = OrCBlock()
            opt = lambda n: g(p + n) if p + n in tensors else np.zeros(e, np.float32)
            b.n1w, b.n1b = k(g(p + "norm1.weight")), k(opt("norm1.bias"))
            b.inw, b.inb = k(g(p + "attn.in_proj_weight")), k(g(p + "attn.in_proj_bias"))
            b.ow, b.ob = k(g(p + "attn.out_proj.weight")), k(g(p + "attn.out_proj.bias"))
            b.n2w, b.n2b = k(g(p + "norm2.weight")), k(opt("norm2.bias"))
            b.w1, b.b1 = k(g(p + "linear1.weight")), k(g(p + "linear1.bias"))
            b.w2, b.b2 = k(g(p + "linear2.weight")), k(g(p + "linear2.bias"))
            b.ff = g(p + "linear1.bias").size
            return b

        ncol, nrow = cfg["col_num_blocks"], cfg["row_num_blocks"]
        cols = (OrCBlock * ncol)(*[block(f"col_embedder.tf_col.blocks.{i}.multihead_attn2.") for i in range(ncol)])
        rows = (OrCBlock * nrow)(*[block(f"row_interactor.tf_row.blocks.{i}.") for i in range(nrow)])
        self._blocks = (cols, rows)
        m = OrRowsModel()
        m.e, m.group, m.inds, m.cls = e, cfg["col_feature_group_size"], cfg["col_num_inds"], cfg["row_num_cls"]
        m.col_heads, m.row_heads, m.ncol, m.nrow = cfg["col_nhead"], cfg["row_nhead"], ncol, nrow
        m.in_w, m.in_b = k(g("col_embedder.in_linear.weight")), k(g("col_embedder.in_linear.bias"))
        m.col, m.row = ctypes.cast(cols, _P(OrCBlock)), ctypes.cast(rows, _P(OrCBlock))
        m.cls_tokens, m.rope_freqs = k(g("row_interactor.cls_tokens")), k(g("row_interactor.tf_row.rope.freqs"))
        m.out_lnw = k(g("row_interactor.out_ln.weight"))
        m.out_lnb = k(g("row_interactor.out_ln.bias") if "row_interactor.out_ln.bias" in tensors else np.zeros(e, np.float32))
        # fitting: each column block's first attention with its scalable softmax and inducing points, and the label's
        # embedding table (model.rs:163-177: a class's row = weight column + bias; regression: [weight][bias])
        p1 = "col_embedder.tf_col.blocks.0.multihead_attn1."
        self.fit = p1 + "attn.in_proj_weight" in tensors and "col_embedder.y_encoder.weight" in tensors
        if self.fit:
            isabs = []
            for i in range(ncol):
                p = f"col_embedder.tf_col.blocks.{i}."
                a = OrIsab1()
                a.b = block(p + "multihead_attn1.")
                ss = p + "multihead_attn1.attn.ssmax_layer."
                a.sb0w, a.sb0b = k(g(ss + "base_mlp.0.weight")), k(g(ss + "base_mlp.0.bias"))
                a.sb2w, a.sb2b = k(g(ss + "base_mlp.2.weight")), k(g(ss + "base_mlp.2.bias"))
                a.q0w, a.q0b = k(g(ss + "query_mlp.0.weight")), k(g(ss + "query_mlp.0.bias"))
                a.q2w, a.q2b = k(g(ss + "query_mlp.2.weight")), k(g(ss + "query_mlp.2.bias"))
                a.hid = g(ss + "base_mlp.0.bias").size
                a.ind = k(g(p + "ind_vectors"))
                isabs.append(a)
            self._isabs = (OrIsab1 * ncol)(*isabs)
            m.col1 = ctypes.cast(self._isabs, _P(OrIsab1))
            yw, yb = g("col_embedder.y_encoder.weight"), g("col_embedder.y_encoder.bias")
            mc = cfg["max_classes"]
            if mc > 0:
                table = (yw.reshape(e, mc).T + yb[None, :]).astype(np.float32)
            else:
                table = np.concatenate([yw, yb]).astype(np.float32)
            m.col_y, m.max_classes = k(table), mc
        self.m = m
        self.e, self.cls, self.inds, self.ncol, self.nrow = e, m.cls, m.inds, ncol, nrow

    @property
    def ref(self):
        return ctypes.byref(self.m)


def rows_model_from_bundle(b):
    import json
    cfg = json.loads(bytes(b["config.json"]).decode())
    return RowsModel({n: b[n] for n in b.names() if n.startswith(("col_embedder.", "row_interactor."))}, cfg)


def embed(rm, x, col_kv, digits=1):
    """predict.rs:282-353: normalised test rows x [n][features] to tokens [n][cls + features][e]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, feats = x.shape
    ck = np.ascontiguousarray(col_kv, dtype=np.float32).reshape(-1)
    assert ck.size == feats * digits * rm.ncol * 2 * rm.e * rm.inds
    tok = np.empty((n, rm.cls + feats, rm.e), np.float32)
    lib().or_embed(rm.ref, _p(x), n, feats, _p(ck), digits, _p(tok))
    return tok


def fit_columns(rm, x, y, chunk, bases=(0,)):
    """fit.rs:298-420: training rows x [n][features] (normalised) and targets y to the member's column cache
    [features][digits][blocks][2][e][inds] and the training tokens [n][cls + features][e]; `bases` the plan's label
    digits (one entry, unused, for a single digit)."""
    assert rm.fit, "the weights have no column-stage fit tensors"
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, feats = x.shape
    y = np.ascontiguousarray(y, dtype=np.float32)
    digits = len(bases)
    b = np.ascontiguousarray(bases, dtype=np.int32)
    col_kv = np.zeros((feats, digits, rm.ncol, 2, rm.e, rm.inds), np.float32)
    tok = np.zeros((n, rm.cls + feats, rm.e), np.float32)
    lib().or_fit_columns(rm.ref, _p(x), _p(y), n, feats, chunk, digits, b.ctypes.data_as(_P(ctypes.c_int32)), _p(col_kv),
                         _p(tok))
    return col_kv, tok


def ind_queries(rm, n):
    """fit.rs:300-314: every column block's inducing-point queries (scaled) for n training rows, [blocks][inds][e]."""
    assert rm.fit, "the weights have no column-stage fit tensors"
    out = np.empty((rm.ncol, rm.inds, rm.e), np.float32)
    lib().or_ind_queries(rm.ref, n, _p(out))
    return out


def fit_cells(rm, x, y):
    """fit.rs:316-345 for one label digit: training cells [n][features][e] through the input layer, the label's
    embedding added."""
    assert rm.fit, "the weights have no column-stage fit tensors"
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.ascontiguousarray(y, dtype=np.float32)
    n, feats = x.shape
    out = np.empty((n, feats, rm.e), np.float32)
    lib().or_fit_cells(rm.ref, _p(x), _p(y), n, feats, _p(out))
    return out


def represent(rm, tok):
    """predict.rs:356-372: tokens [n][tokens][e] to row representations [n][cls e]."""
    tok = np.array(tok, dtype=np.float32)  # a copy: consumed
    n, tokens, e = tok.shape
    rep = np.empty((n, rm.cls * e), np.float32)
    lib().or_represent(rm.ref, _p(tok), n, tokens, _p(rep))
    return rep


def model_from_bundle(b):
    """Oracle model from a weight bundle (tabicl-anywhere_b200.tirs.Bundle); config keys as model.rs:220-236."""
    import json
    cfg = json.loads(bytes(b["config.json"]).decode())
    tensors = {n: b[n] for n in b.names() if n.startswith("icl_predictor.")}
    return Model(tensors, cfg["icl_nhead"], cfg["icl_num_blocks"], cfg["max_classes"])


def record(kv, d, rc):
    return int(lib().or_record(kv, d, rc))


def layer_len(kv, d, rows, chunk):
    """fit.rs:234: bytes of one layer's stored keys and values"""
    return (rows // chunk) * record(kv, d, chunk) + (record(kv, d, rows % chunk) if rows % chunk else 0)


def pack(kv, d, c):
    """fit.rs:549-576: c [2d][rc] -> the stored record bytes"""
    c = np.ascontiguousarray(c, dtype=np.float32)
    rc = c.shape[1]
    out = np.zeros(record(kv, d, rc), np.uint8)
    lib().or_pack(kv, d, rc, _p(c), out.ctypes.data)
    return out


def pack_layer(kv, d, k, v, chunk):
    """One layer's keys and values [rows][d] each to the stored n{j}_kv{l} bytes, chunk by chunk."""
    rows = k.shape[0]
    parts = []
    for r0 in range(0, rows, chunk):
        kt = k[r0:r0 + chunk].T
        vt = v[r0:r0 + chunk].T
        parts.append(pack(kv, d, np.concatenate([kt, vt], axis=0)))
    return np.concatenate(parts)


def layer_rows(kv, d, layer, rows, chunk):
    k = np.empty((rows, d), np.float32)
    v = np.empty((rows, d), np.float32)
    layer = np.ascontiguousarray(np.frombuffer(bytes(layer), np.uint8))
    lib().or_layer_rows(kv, d, layer.ctypes.data, rows, chunk, _p(k), _p(v))
    return k, v


def attend(kv, d, heads, layer, rows, chunk, q, parts=1):
    q = np.ascontiguousarray(q, dtype=np.float32).reshape(-1, d)
    out = np.empty_like(q)
    layer = np.ascontiguousarray(np.frombuffer(bytes(layer), np.uint8))
    lib().or_attend(kv, d, heads, layer.ctypes.data, rows, chunk, _p(q), q.shape[0], parts, _p(out))
    return out


def in_context(model, kv, layers, scales, rows, chunk, h, out_n, parts=1):
    """predict.rs:381-586: row representations h [n][d] to the first out_n decoder outputs."""
    h = np.array(h, dtype=np.float32).reshape(-1, model.d)  # a copy: consumed
    n = h.shape[0]
    bufs = [np.ascontiguousarray(np.frombuffer(bytes(x), np.uint8)) for x in layers]
    ptrs = (ctypes.c_void_p * len(bufs))(*[b.ctypes.data for b in bufs])
    sc = np.ascontiguousarray(scales, dtype=np.float32).reshape(-1)
    out = np.empty((n, out_n), np.float32)
    lib().or_in_context(model.ref, kv, ptrs, _p(sc), rows, chunk, _p(h), n, out_n, parts, _p(out))
    return out


def add_y(model, h, y):
    """model.rs:185-200 add_y for the in-context stage: h [rows][d] plus the targets' embedding (a copy)."""
    h = np.array(h, dtype=np.float32).reshape(-1, model.d)
    y = np.ascontiguousarray(y, dtype=np.float32)
    lib().or_add_y(model.ref, _p(y), h.shape[0], _p(h))
    return h


def icl_fit(model, h, y, chunk, kv):
    """fit.rs:577-747: training rows h [rows][d] (before the target embedding) and targets y to every layer's
    stored bytes and the query scales."""
    h = np.array(h, dtype=np.float32).reshape(-1, model.d)
    rows = h.shape[0]
    y = np.ascontiguousarray(y, dtype=np.float32)
    lib().or_add_y(model.ref, _p(y), rows, _p(h))
    n = layer_len(kv, model.d, rows, chunk)
    outs = [np.zeros(n, np.uint8) for _ in range(model.layers)]
    ptrs = (ctypes.c_void_p * model.layers)(*[o.ctypes.data for o in outs])
    scales = np.empty((model.layers, model.d), np.float32)
    lib().or_icl_fit(model.ref, _p(h), rows, chunk, kv, ptrs, _p(scales))
    return outs, scales


def parse_tree(tree, n_nodes):
    """predict.rs:141-148: per node (leaf, rows, k, map)."""
    out, at = [], 0
    for _ in range(n_nodes):
        leaf, rows, k = (int(v) for v in tree[at:at + 3])
        out.append((bool(leaf), rows, k, [int(v) for v in tree[at + 3:at + 3 + k]]))
        at += 3 + k
    return out


def tree_scores(node_scores, tree, n_nodes, classes):
    """predict.rs:664-692 in f32: every node's scores (node_scores[i], [n][k_i]) to class scores [n][classes]. Per row,
    each node's scores become probabilities (the largest, from f32::MIN and ignoring NaN, subtracted; exp((v - top) /
    0.9) summed in order; each over the sum), the recursive walk from node 0 multiplies them down the tree and adds
    each leaf's share to its classes, and the result goes back to scores as 0.9 ln(p + 1e-6)."""
    f = np.float32
    nodes = parse_tree(tree, n_nodes)
    n = np.asarray(node_scores[0]).shape[0]
    probs = []
    for i, (_, _, k, _) in enumerate(nodes):
        p = np.array(node_scores[i], dtype=np.float32).reshape(n, k)
        for r in range(n):
            top = f(-3.4028235e38)
            for v in p[r]:
                top = np.fmax(top, v)
            e = np.exp(((p[r] - top) / f(0.9)).astype(np.float32)).astype(np.float32)
            total = f(0.0)
            for v in e:
                total = f(total + v)
            p[r] = e / total
        probs.append(p)

    def walk(ni, r, weight, out):
        leaf, _, _, mp = nodes[ni]
        pr = probs[ni][r]
        for j, target in enumerate(mp):
            if leaf:
                out[target] = f(out[target] + f(weight * pr[j]))
            else:
                walk(target, r, f(weight * pr[j]), out)

    res = np.zeros((n, classes), np.float32)
    for r in range(n):
        walk(0, r, f(1.0), res[r])
    return (f(0.9) * np.log(res + f(1e-6))).astype(np.float32)


def finish_proba(sums, members, temperature):
    s = np.array(sums, dtype=np.float64)
    n, c = s.shape
    lib().or_finish_proba(s.ctypes.data_as(_P(ctypes.c_double)), n, c, members, temperature)
    return s


def add_member(sums, logits, member_classes):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    mc = np.ascontiguousarray(member_classes, dtype=np.int32)
    n, c = sums.shape
    lib().or_add_member(sums.ctypes.data_as(_P(ctypes.c_double)), _p(logits), n, c, logits.shape[1],
                        mc.ctypes.data_as(_P(ctypes.c_int32)))


def regression_add(qout, alphas, target_mean, target_scale, acc=None):
    """table.rs:476-490 for one member: adds mean, variance, median, quantiles to `acc` (created if None)."""
    q = np.ascontiguousarray(qout, dtype=np.float32)
    n, nq = q.shape
    al = np.ascontiguousarray(alphas, dtype=np.float64)
    if acc is None:
        acc = {k: np.zeros(n) for k in ("mean", "variance", "median")}
        acc["quantiles"] = np.zeros((n, al.size))
    D = _P(ctypes.c_double)
    lib().or_regression_add(_p(q), n, nq, nq, al.ctypes.data_as(D), al.size, target_mean, target_scale,
                            acc["mean"].ctypes.data_as(D), acc["variance"].ctypes.data_as(D),
                            acc["median"].ctypes.data_as(D), acc["quantiles"].ctypes.data_as(D))
    return acc


def threads():
    return int(lib().or_threads())


def set_threads(n):
    lib().or_set_threads(int(n))
