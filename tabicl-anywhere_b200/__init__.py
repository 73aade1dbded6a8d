"""B200 backend for tabicl-anywhere's prediction hot path: the Python binding of the C ABI (include/tabicl_b200.h).

The objects mirror the reference's accelerator side (src/gpu.rs, src/predict.rs:63-79):

* `Gpu` - one device (gpu::Gpu)
* `GpuWeights` - the in-context weights on it (gpu::GpuWeights)
* `VramModel` - one fitted problem's key/value cache resident on it (gpu::VramModel)
* `VramMember` - a fitted member's problems and its class tree, predicted whole (predict::predict_raw)
* `VramTier` / `VramHandle` - problems resident for many tenants within byte budgets; the handle is an AttendCached
* `CudaAttend` - the `AttendCached` implementation: `attend`, `stage`, `rows`, each returning None to decline

Everything computes on the GPU through libtabicl_b200.so; there is no CPU path here. The library is built in-tree
by build.py (sm_100a); importing this package does not build it.
"""
import ctypes
import os

import numpy as np

from . import tirs  # noqa: F401  (bundle reader/writer for callers)
from .plan import Plan  # noqa: F401

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtabicl_b200.so")

OK, DECLINED = 0, 1
KV_F32, KV_I16, KV_I8 = 0, 1, 2
_c_int, _c_size, _c_void, _c_float_p = ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p, ctypes.POINTER(ctypes.c_float)


class TcuError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"tabicl_b200 error {code}: {msg}")
        self.code = code


class IclShape(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("d", "heads", "layers", "ff", "hid", "dec_ff", "outs", "max_classes")]

    def as_dict(self):
        return {n: getattr(self, n) for n, _ in self._fields_}


class RowsShape(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("e", "group", "inds", "cls", "col_heads", "row_heads", "col_blocks",
                                              "row_blocks", "col_ff", "row_ff")]

    def as_dict(self):
        return {n: getattr(self, n) for n, _ in self._fields_}


_lib = None


_READ_AT = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_size_t)


class _Source(ctypes.Structure):
    _fields_ = [("user", ctypes.c_void_p), ("read_at", _READ_AT), ("size", ctypes.c_uint64)]


# tcu_layer_sink: (user, layer, k [rows][d], v [rows][d]) -> 0 to go on
_LayerSink = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_float),
                              ctypes.POINTER(ctypes.c_float))


def lib():
    """The loaded C library (fails loudly if it is not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is not built: run python tabicl-anywhere_b200/build.py")
    L = ctypes.CDLL(LIB_PATH)
    P = ctypes.POINTER
    sig = {
        "tcu_open": (_c_int, [_c_int, P(_c_void)]),
        "tcu_close": (None, [_c_void]),
        "tcu_last_error": (ctypes.c_char_p, [_c_void]),
        "tcu_launches": (ctypes.c_uint64, [_c_void]),
        "tcu_weights_new": (_c_int, [_c_void, P(IclShape), _c_int, P(_c_void)]),
        "tcu_weights_put": (_c_int, [_c_void, ctypes.c_char_p, _c_int, _c_void, _c_size]),
        "tcu_weights_ready": (_c_int, [_c_void]),
        "tcu_weights_from_bundle": (_c_int, [_c_void, ctypes.c_char_p, _c_int, P(_c_void)]),
        "tcu_weights_shape": (_c_int, [_c_void, P(IclShape)]),
        "tcu_weights_set_rows_shape": (_c_int, [_c_void, P(RowsShape)]),
        "tcu_weights_rows_shape": (_c_int, [_c_void, P(RowsShape)]),
        "tcu_model_put_col_kv": (_c_int, [_c_void, _c_float_p, _c_size]),
        "tcu_rows": (_c_int, [_c_void, _c_float_p, _c_int, _c_int, _c_int, _c_float_p]),
        "tcu_rows_device": (_c_int, [_c_void, _c_void, _c_int, _c_int, _c_void, _c_void]),
        "tcu_embed_device": (_c_int, [_c_void, _c_void, _c_int, _c_void, _c_void]),
        "tcu_represent_device": (_c_int, [_c_void, _c_void, _c_int, _c_void, _c_void]),
        "tcu_weights_free": (None, [_c_void]),
        "tcu_model_new": (_c_int, [_c_void, P(ctypes.c_int32), ctypes.c_int32, ctypes.c_int32, P(_c_void)]),
        "tcu_model_put_scales": (_c_int, [_c_void, _c_float_p, _c_size]),
        "tcu_model_put_layer": (_c_int, [_c_void, _c_int, _c_size, _c_void, _c_size]),
        "tcu_model_from_bundle": (_c_int, [_c_void, ctypes.c_char_p, ctypes.c_char_p, _c_int, P(_c_void)]),
        "tcu_model_bytes": (_c_size, [_c_void]),
        "tcu_model_get_layer": (_c_int, [_c_void, _c_int, _c_void, _c_size]),
        "tcu_model_get_scales": (_c_int, [_c_void, _c_float_p, _c_size]),
        "tcu_model_free": (None, [_c_void]),
        "tcu_attend": (_c_int, [_c_void, _c_int, _c_float_p, _c_int, _c_int, _c_int, _c_float_p]),
        "tcu_stage": (_c_int, [_c_void, _c_float_p, _c_int, _c_int, _c_int, _c_float_p]),
        "tcu_attend_device": (_c_int, [_c_void, _c_int, _c_void, _c_int, _c_void, _c_void]),
        "tcu_stage_device": (_c_int, [_c_void, _c_void, _c_int, _c_int, _c_void, _c_void]),
        "tcu_class_head_device": (_c_int, [_c_void, _c_void, _c_int, _c_int, _c_int, _c_void, _c_void, _c_int, _c_int,
                                           ctypes.c_double]),
        "tcu_regression_head_device": (_c_int, [_c_void, _c_void, _c_int, _c_int, _c_int, _c_void, _c_int,
                                                ctypes.c_double, ctypes.c_double, _c_void, _c_void, _c_void, _c_void]),
        "tcu_fit_icl_device": (_c_int, [_c_void, _c_void, _c_void, _c_int, _c_int, _c_int, P(_c_void)]),
        "tcu_fit_rows_device": (_c_int, [_c_void, _c_void, _c_void, _c_int, _c_int, _c_int, P(ctypes.c_int32), _c_void,
                                         _c_void, _c_void]),
        "tcu_fit_column_batch": (_c_int, [_c_void, _c_int]),
        "tcu_fit_columns": (_c_int, [_c_void, _c_float_p, _c_int, _c_int, _c_float_p, _c_float_p]),
        "tcu_fit_row_batch": (_c_int, [_c_void, _c_int]),
        "tcu_fit_rows": (_c_int, [_c_void, _c_float_p, _c_int, _c_int, _c_float_p]),
        "tcu_fit_in_context": (_c_int, [_c_void, _c_float_p, _c_int, _c_float_p, _LayerSink, _c_void]),
        "tcu_pack_device": (_c_int, [_c_void, _c_int, _c_int, _c_int, _c_void, _c_void]),
        "tcu_record": (_c_size, [_c_int, _c_int, _c_int]),
        "tcu_layer_rows_device": (_c_int, [_c_void, _c_int, _c_int, _c_void, _c_int, _c_int, _c_void, _c_void]),
        "tcu_sync": (_c_int, [_c_void, _c_void]),
        "tcu_debug_abort_next": (_c_int, [_c_void]),
        "tcu_profile": (_c_int, [_c_void, _c_int, P(ctypes.c_double), P(ctypes.c_uint64)]),
        "tcu_selftest_mma": (_c_int, [_c_void, P(ctypes.c_double)]),
        "tcu_attend_noalloc": (_c_int, [_c_int, _c_int, _c_int, _c_void, _c_int, _c_int, _c_void, _c_int, _c_void,
                                        _c_void, ctypes.c_char_p, _c_size]),
        "tcu_comm_unique_id": (_c_int, [ctypes.c_char_p]),
        "tcu_comm_init": (_c_int, [_c_void, ctypes.c_char_p, _c_int, _c_int, P(_c_void)]),
        "tcu_comm_free": (None, [_c_void]),
        "tcu_comm_allreduce_f64": (_c_int, [_c_void, _c_void, _c_size, _c_void]),
        "tcu_comm_wait": (_c_int, [_c_void, _c_void, _c_int]),
        "tcu_model_slice": (_c_int, [_c_void, _c_int, _c_int, P(_c_void)]),
        "tcu_model_set_columns": (_c_int, [_c_void, _c_int, _c_int]),
        "tcu_member_new": (_c_int, [P(_c_void), _c_int, P(ctypes.c_int32), _c_size, _c_int, P(_c_void)]),
        "tcu_member_from_bundle": (_c_int, [_c_void, ctypes.c_char_p, ctypes.c_char_p, P(_c_void)]),
        "tcu_member_nodes": (_c_int, [_c_void]),
        "tcu_member_classes": (_c_int, [_c_void]),
        "tcu_member_node": (_c_void, [_c_void, _c_int]),
        "tcu_member_bytes": (_c_size, [_c_void]),
        "tcu_member_rows": (_c_int, [_c_void, _c_float_p, _c_int, _c_int, _c_float_p]),
        "tcu_member_rows_device": (_c_int, [_c_void, _c_void, _c_int, _c_void, _c_void]),
        "tcu_member_combine_device": (_c_int, [_c_void, _c_void, _c_int, _c_void, _c_void]),
        "tcu_member_free": (None, [_c_void]),
        "tcu_tier_new": (_c_int, [_c_void, _c_size, _c_size, _c_int, P(_c_void)]),
        "tcu_tier_free": (None, [_c_void]),
        "tcu_tier_wait": (None, [_c_void]),
        "tcu_tier_held": (None, [_c_void, ctypes.c_char_p, P(_c_size), P(_c_size)]),
        "tcu_tier_ready": (_c_size, [_c_void, ctypes.c_char_p]),
        "tcu_tier_on_card": (None, [_c_void, ctypes.c_char_p, P(_c_size), P(_c_size)]),
        "tcu_tier_fallbacks": (ctypes.c_uint64, [_c_void]),
        "tcu_tier_last_error": (_c_size, [_c_void, ctypes.c_char_p, _c_size]),
        "tcu_tier_evict": (None, [_c_void, ctypes.c_char_p, ctypes.c_char_p]),
        "tcu_tier_handle": (_c_int, [_c_void, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, _c_void, P(_c_void)]),
        "tcu_tier_handle_source": (_c_int, [_c_void, ctypes.c_char_p, ctypes.c_char_p, P(_Source), _c_void,
                                            P(_c_void)]),
        "tcu_handle_free": (None, [_c_void]),
        "tcu_handle_preload": (_c_int, [_c_void, ctypes.c_char_p, _c_int]),
        "tcu_handle_attend": (_c_int, [_c_void, ctypes.c_char_p, _c_int, _c_int, _c_float_p, _c_int, _c_int, _c_int,
                                       _c_float_p]),
        "tcu_handle_stage": (_c_int, [_c_void, ctypes.c_char_p, _c_int, _c_float_p, _c_int, _c_int, _c_int, _c_float_p]),
        "tcu_handle_rows": (_c_int, [_c_void, ctypes.c_char_p, _c_float_p, _c_int, _c_int, _c_int, _c_float_p]),
        "tcu_tier_debug_admit": (_c_int, [_c_void, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, _c_int, _c_size]),
        "tcu_tier_debug_pin": (_c_int, [_c_void, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, _c_int, P(_c_void)]),
        "tcu_tier_debug_unpin": (None, [_c_void]),
        "tcu_stage_sharded_device": (_c_int, [_c_void, _c_void, _c_void, _c_int, _c_int, _c_void, _c_void]),
        "tcu_comm_breakdown": (_c_int, [_c_void, _c_int, P(ctypes.c_double)]),
        "tcu_comm_abort": (_c_int, [_c_void]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype, f.argtypes = res, args
    _lib = L
    return L


def exported_symbols():
    """Names of the entry points this binding declares (every one is in include/tabicl_b200.h)."""
    lib()
    return [n for n in dir(_lib) if n.startswith("tcu_")]


def record(kv, d, rc):
    """Bytes of one stored chunk of rc rows (src/fit.rs:124-126)."""
    return int(lib().tcu_record(kv, d, rc))


def _f32p(a):
    return a.ctypes.data_as(_c_float_p)


class Gpu:
    """One device (gpu::Gpu, src/gpu.rs:725-747)."""

    def __init__(self, device=0):
        self._h = _c_void()
        r = lib().tcu_open(device, ctypes.byref(self._h))
        if r != OK:
            raise TcuError(r, f"cannot open CUDA device {device}")
        self.device = device

    def check(self, r):
        if r < 0:
            raise TcuError(r, self.last_error)
        return r

    @property
    def last_error(self):
        return lib().tcu_last_error(self._h).decode()

    @property
    def launches(self):
        return int(lib().tcu_launches(self._h))

    def profile(self, enable):
        """Start (or stop) event timing of the attention passes; returns (total ms, passes) since the last call."""
        ms, n = ctypes.c_double(), ctypes.c_uint64()
        self.check(lib().tcu_profile(self._h, int(enable), ctypes.byref(ms), ctypes.byref(n)))
        return ms.value, n.value

    def close(self):
        if self._h:
            lib().tcu_close(self._h)
            self._h = _c_void()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # heads (src/table.rs) on device buffers given as raw pointers (e.g. torch tensors' data_ptr())
    def class_head(self, logits_ptr, rows, classes, stride, member_classes_ptr, sums_ptr, finish=False, members=1,
                   temperature=0.9):
        return self.check(lib().tcu_class_head_device(self._h, logits_ptr, rows, classes, stride, member_classes_ptr,
                                                      sums_ptr, int(finish), members, temperature))

    def regression_head(self, qout_ptr, rows, nq, stride, alphas_ptr, na, target_mean, target_scale, mean_ptr,
                        var_ptr, median_ptr, quant_ptr):
        return self.check(lib().tcu_regression_head_device(self._h, qout_ptr, rows, nq, stride, alphas_ptr, na,
                                                           target_mean, target_scale, mean_ptr, var_ptr, median_ptr,
                                                           quant_ptr))

    def selftest_mma(self):
        """Largest error of exact small products on the tensor cores (0.0 when the operand layouts are right)."""
        e = ctypes.c_double()
        self.check(lib().tcu_selftest_mma(self._h, ctypes.byref(e)))
        return e.value

    def pack(self, kv, d, rc, c_ptr, rec_ptr):
        return self.check(lib().tcu_pack_device(self._h, kv, d, rc, c_ptr, rec_ptr))

    def layer_rows(self, kv, d, layer_ptr, rows, chunk, k_ptr, v_ptr):
        """predict.rs:590-629 on device buffers: stored chunks to keys and values [rows][d] floats."""
        return self.check(lib().tcu_layer_rows_device(self._h, kv, d, layer_ptr, rows, chunk, k_ptr, v_ptr))

    def sync(self, stream=None):
        """Wait for `stream` (None: the context's) and raise if kernels gave up a bounded wait since the last
        report."""
        return self.check(lib().tcu_sync(self._h, stream))

    def debug_abort_next(self):
        """Test hook: the next one-kernel stage launch starts as if a wait had given up."""
        return self.check(lib().tcu_debug_abort_next(self._h))


class GpuWeights:
    """The in-context weights on the device (gpu::GpuWeights, src/gpu.rs:1838-2028)."""

    def __init__(self, gpu, handle):
        self.gpu, self._h = gpu, handle

    @staticmethod
    def from_bundle(gpu, path, for_fit=False):
        h = _c_void()
        gpu.check(lib().tcu_weights_from_bundle(gpu._h, os.fsencode(path), int(for_fit), ctypes.byref(h)))
        return GpuWeights(gpu, h)

    @staticmethod
    def from_tensors(gpu, shape, tensors, for_fit=False, rows_shape=None):
        """`shape`: dict of IclShape fields; `tensors`: bundle name -> float32/float16 array; `rows_shape` (dict of
        RowsShape fields): also keep the column and row stages (their tensors among `tensors`)."""
        h = _c_void()
        s = IclShape(**shape)
        gpu.check(lib().tcu_weights_new(gpu._h, ctypes.byref(s), int(for_fit), ctypes.byref(h)))
        w = GpuWeights(gpu, h)
        if rows_shape is not None:
            rs = RowsShape(**rows_shape)
            gpu.check(lib().tcu_weights_set_rows_shape(h, ctypes.byref(rs)))
        for name, a in tensors.items():
            a = np.ascontiguousarray(a)
            dt = 1 if a.dtype == np.float16 else 0
            if dt == 0:
                a = np.ascontiguousarray(a, dtype=np.float32)
            gpu.check(lib().tcu_weights_put(h, name.encode(), dt, a.ctypes.data, a.size))
        gpu.check(lib().tcu_weights_ready(h))
        return w

    @property
    def shape(self):
        s = IclShape()
        self.gpu.check(lib().tcu_weights_shape(self._h, ctypes.byref(s)))
        return s.as_dict()

    @property
    def rows_shape(self):
        """The column and row stages' sizes, or None when the weights have none."""
        s = RowsShape()
        r = self.gpu.check(lib().tcu_weights_rows_shape(self._h, ctypes.byref(s)))
        return s.as_dict() if r == OK else None

    def free(self):
        if self._h:
            lib().tcu_weights_free(self._h)
            self._h = _c_void()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class VramModel:
    """One fitted problem's cache resident on the device (gpu::VramModel, src/gpu.rs:2033-2116)."""

    def __init__(self, weights, handle, owner=None):
        self.weights, self.gpu, self._h = weights, weights.gpu, handle
        self.d = weights.shape["d"]
        self._owner = owner  # a VramMember holding this problem (it frees the handle), or None

    @staticmethod
    def from_bundle(weights, path, prefix="", node=0):
        h = _c_void()
        weights.gpu.check(lib().tcu_model_from_bundle(weights._h, os.fsencode(path), prefix.encode(), node,
                                                      ctypes.byref(h)))
        return VramModel(weights, h)

    @staticmethod
    def from_parts(weights, meta, node_rows, node_k, scales, layers, col_kv=None):
        """`meta`: the member's 7 meta ints; `scales` [layers][d] floats; `layers`: each layer's stored bytes; `col_kv`:
        the column stage's cache (fit.rs:230), for the `rows` hook."""
        h = _c_void()
        meta = np.ascontiguousarray(meta, dtype=np.int32)
        g = weights.gpu
        g.check(lib().tcu_model_new(weights._h, meta.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), node_rows, node_k,
                                    ctypes.byref(h)))
        m = VramModel(weights, h)
        sc = np.ascontiguousarray(scales, dtype=np.float32).reshape(-1)
        g.check(lib().tcu_model_put_scales(h, _f32p(sc), sc.size))
        for l, b in enumerate(layers):
            b = np.frombuffer(bytes(b), dtype=np.uint8)
            g.check(lib().tcu_model_put_layer(h, l, 0, b.ctypes.data, b.size))
        if col_kv is not None:
            ck = np.ascontiguousarray(col_kv, dtype=np.float32).reshape(-1)
            g.check(lib().tcu_model_put_col_kv(h, _f32p(ck), ck.size))
        m.features = int(meta[1])
        return m

    @property
    def nbytes(self):
        return int(lib().tcu_model_bytes(self._h))

    def attend(self, layer, q, d=None, heads=None):
        """AttendCached::attend on host buffers: scaled queries [rows][d] to attention outputs [rows][d]. `d` and
        `heads` are the caller's (the library refuses ones that are not the weights')."""
        d = self.d if d is None else d
        heads = self.weights.shape["heads"] if heads is None else heads
        q = np.ascontiguousarray(q, dtype=np.float32).reshape(-1)
        if q.size % d:
            raise TcuError(-1, f"attend: {q.size} query values are not rows of width {d}")
        out = np.empty_like(q)
        self.gpu.check(lib().tcu_attend(self._h, layer, _f32p(q), q.size // d, d, heads, _f32p(out)))
        return out.reshape(-1, d)

    def stage(self, h, out_n, out=None, d=None):
        """AttendCached::stage on host buffers: [rows][d] representations to [rows][out_n] decoder outputs
        (`out`, if given, is filled: pinned host buffers make the copies faster)."""
        d = self.d if d is None else d
        h = np.ascontiguousarray(h, dtype=np.float32).reshape(-1)
        if h.size % d:
            raise TcuError(-1, f"stage: {h.size} values are not rows of width {d}")
        rows = h.size // d
        if out is None:
            out = np.empty((rows, out_n), dtype=np.float32)
        assert out.dtype == np.float32 and out.flags.c_contiguous and out.size == rows * out_n
        self.gpu.check(lib().tcu_stage(self._h, _f32p(h), rows, d, out_n, _f32p(out)))
        return out

    def put_col_kv(self, col_kv):
        """The column stage's cache (fit.rs:230: [features][digits][blocks][2][e][inds] floats) for the rows hook."""
        ck = np.ascontiguousarray(col_kv, dtype=np.float32).reshape(-1)
        self.gpu.check(lib().tcu_model_put_col_kv(self._h, _f32p(ck), ck.size))

    def rows(self, x, out_n, out=None):
        """AttendCached::rows on host buffers: normalised rows [rows][features] through the column, row and in-context
        stages to [rows][out_n] decoder outputs. Returns None when the library declines (no column and row stages)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        n, feats = x.shape
        if out is None:
            out = np.empty((n, out_n), dtype=np.float32)
        r = self.gpu.check(lib().tcu_rows(self._h, _f32p(x), n, feats, out_n, _f32p(out)))
        return None if r == DECLINED else out

    def rows_device(self, x_ptr, rows, out_n, out_ptr, stream=None):
        return self.gpu.check(lib().tcu_rows_device(self._h, x_ptr, rows, out_n, out_ptr, stream))

    def embed_device(self, x_ptr, rows, tok_ptr, stream=None):
        """predict::embed on device buffers: tokens [rows][cls + features][e]."""
        return self.gpu.check(lib().tcu_embed_device(self._h, x_ptr, rows, tok_ptr, stream))

    def represent_device(self, tok_ptr, rows, rep_ptr, stream=None):
        """predict::represent on device buffers (the tokens are used as scratch): [rows][cls e]."""
        return self.gpu.check(lib().tcu_represent_device(self._h, tok_ptr, rows, rep_ptr, stream))

    def attend_device(self, layer, q_ptr, rows, out_ptr, stream=None):
        return self.gpu.check(lib().tcu_attend_device(self._h, layer, q_ptr, rows, out_ptr, stream))

    def stage_device(self, h_ptr, rows, out_n, out_ptr, stream=None):
        return self.gpu.check(lib().tcu_stage_device(self._h, h_ptr, rows, out_n, out_ptr, stream))

    def slice(self, first_chunk, nchunks):
        """A new resident cache of chunks [first_chunk, first_chunk + nchunks) (a shard of the training rows)."""
        h = _c_void()
        self.gpu.check(lib().tcu_model_slice(self._h, first_chunk, nchunks, ctypes.byref(h)))
        return VramModel(self.weights, h)

    def stage_sharded_device(self, comm, h_ptr, rows, out_n, out_ptr, stream=None):
        """The stage with this cache one shard of the training rows: every layer's attention merged over `comm`."""
        return self.gpu.check(lib().tcu_stage_sharded_device(self._h, comm._h, h_ptr, rows, out_n, out_ptr, stream))

    def layer_bytes(self, layer, nbytes):
        out = np.empty(nbytes, dtype=np.uint8)
        self.gpu.check(lib().tcu_model_get_layer(self._h, layer, out.ctypes.data, nbytes))
        return out

    def scales(self):
        s = self.weights.shape
        out = np.empty(s["layers"] * s["d"], dtype=np.float32)
        self.gpu.check(lib().tcu_model_get_scales(self._h, _f32p(out), out.size))
        return out.reshape(s["layers"], s["d"])

    def free(self):
        if self._h and self._owner is None:
            lib().tcu_model_free(self._h)
        self._h = _c_void()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Stats:
    """The counters of predict::Stats (src/predict.rs) that a pass on the device moves: rows, passes and in-context
    layers run on the card."""

    def __init__(self):
        self.rows = self.passes = self.card_layers = 0


class VramMember:
    """A fitted member resident on the device: its problems (one VramModel each, node 0 with the column stage's
    cache) and its class tree (predict::Cache, src/predict.rs:115-161), predicted whole (src/predict.rs:638-699)."""

    def __init__(self, weights, handle):
        self.weights, self.gpu, self._h = weights, weights.gpu, handle
        self.classes = int(lib().tcu_member_classes(handle))
        self.n_nodes = int(lib().tcu_member_nodes(handle))

    @staticmethod
    def from_bundle(weights, path, prefix=""):
        h = _c_void()
        weights.gpu.check(lib().tcu_member_from_bundle(weights._h, os.fsencode(path), prefix.encode(), ctypes.byref(h)))
        return VramMember(weights, h)

    @staticmethod
    def from_nodes(nodes, tree, classes):
        """The member of problems `nodes` (VramModel, node 0 first; the member takes them over: their handles then
        belong to it) with tree ints `tree` (Plan.tree) over `classes` classes."""
        w = nodes[0].weights
        arr = (_c_void * len(nodes))(*[n._h.value for n in nodes])
        t = np.ascontiguousarray(tree, dtype=np.int32)
        h = _c_void()
        w.gpu.check(lib().tcu_member_new(arr, len(nodes), t.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), t.size,
                                         int(classes), ctypes.byref(h)))
        mb = VramMember(w, h)
        for n in nodes:
            n._owner = mb
        return mb

    def node(self, i):
        """Problem i as a VramModel (valid while the member is)."""
        p = lib().tcu_member_node(self._h, i)
        if not p:
            raise IndexError(i)
        return VramModel(self.weights, _c_void(p), owner=self)

    @property
    def nbytes(self):
        return int(lib().tcu_member_bytes(self._h))

    def rows(self, x, out=None):
        """Class scores [rows][classes] of normalised rows x [rows][features] (host buffers)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        n, f = x.shape
        out = np.empty((n, self.classes), dtype=np.float32) if out is None else out
        self.gpu.check(lib().tcu_member_rows(self._h, _f32p(x), n, f, _f32p(out)))
        return out

    def rows_device(self, x_ptr, rows, out_ptr, stream=None):
        return self.gpu.check(lib().tcu_member_rows_device(self._h, x_ptr, rows, out_ptr, stream))

    def combine_device(self, scores_ptr, rows, out_ptr, stream=None):
        return self.gpu.check(lib().tcu_member_combine_device(self._h, scores_ptr, rows, out_ptr, stream))

    def free(self):
        if self._h:
            lib().tcu_member_free(self._h)
            self._h = _c_void()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def predict_raw(member, x, rows_per_pass=256, stats=None):
    """predict::predict_raw (src/predict.rs:631-699) on the device: class scores [n][classes] of n normalised rows x
    [n][features], in passes of rows_per_pass rows (PredictOpts::rows_per_pass, default 256); each pass runs the
    column and row stages, every problem's in-context stage and the class tree."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[0]
    out = np.empty((n, member.classes), dtype=np.float32)
    step = max(1, int(rows_per_pass))
    layers = member.weights.shape["layers"] * member.n_nodes
    for r0 in range(0, n, step):
        member.rows(x[r0:r0 + step], out=out[r0:r0 + step])
        if stats is not None:
            stats.rows += min(step, n - r0)
            stats.passes += 1
            stats.card_layers += layers
    return out


def fit_member(weights, h, y, classes, features, col_kv, chunk=256, kv=KV_F32):
    """The in-context part of fitting one member on the device, for any number of classes: the plan's tree
    (fit::Plan, src/fit.rs:159-221) and each node fitted on its own rows and targets (src/fit.rs:577-747). h: the
    training rows' representations [rows][d] (host), y: their classes; col_kv: the member's column-stage cache over
    `features` features (one copy per label digit of the plan).
    Returns (VramMember, Plan)."""
    import torch  # device buffers for the fit

    h = np.ascontiguousarray(h, dtype=np.float32)
    plan = Plan.new(weights.shape["max_classes"], y, classes)
    nodes = []
    try:
        for nd in plan.nodes:
            rows = np.arange(len(h)) if nd.rows is None else np.asarray(nd.rows)
            hd = torch.from_numpy(np.ascontiguousarray(h[rows])).cuda()
            yd = torch.from_numpy(np.ascontiguousarray(nd.y, dtype=np.float32)).cuda()
            torch.cuda.synchronize()
            nodes.append(fit_icl(weights, hd.data_ptr(), yd.data_ptr(), len(rows), chunk, kv))
            torch.cuda.synchronize()
        ck = np.ascontiguousarray(col_kv, dtype=np.float32)
        weights.gpu.check(lib().tcu_model_set_columns(nodes[0]._h, features, len(plan.bases)))
        nodes[0].put_col_kv(ck)
        return VramMember.from_nodes(nodes, plan.tree(len(h)), classes), plan
    except Exception:
        for m in nodes:
            m.free()
        raise


def layer_len(kv, d, rows, chunk):
    """Bytes of one layer's stored keys and values (fit.rs:234 raw_entries): the full chunks, then the rest."""
    chunk = max(int(chunk), 8)
    return (rows // chunk) * record(kv, d, chunk) + (record(kv, d, rows % chunk) if rows % chunk else 0)


def raw_entries(weights, prefix, rows, features, chunk, kv, plan):
    """fit::raw_entries (src/fit.rs:224-241): the tensors a member's fit fills, as (name, dtype, dims)."""
    s, rs = weights.shape, weights.rows_shape
    chunk = max(int(chunk), 8)
    v = [(prefix + "meta", "int32", [7]), (prefix + "tree", "int32", [len(plan.tree(rows))]),
         (prefix + "col_kv", "float32", [features, len(plan.bases), rs["col_blocks"], 2, rs["e"], rs["inds"]])]
    for i, nd in enumerate(plan.nodes):
        nr = rows if nd.rows is None else len(nd.rows)
        v.append((prefix + f"n{i}_scale", "float32", [s["layers"], s["d"]]))
        for l in range(s["layers"]):
            v.append((prefix + f"n{i}_kv{l}", "uint8", [layer_len(kv, s["d"], nr, chunk)]))
    return v


def fit_raw(weights, x, y, classes, chunk=256, kv=KV_F32, prefix=""):
    """fit_raw_async (src/fit.rs:285-752) for one member, every stage on the device: normalised training rows x
    [rows][features] and labels y (class indices as floats, or standardised targets; host) through the column stage
    (fit.rs:298-481), the row stage (487-540) and, per node of fit::Plan's class tree (159-221), the in-context stage
    (577-747). `classes` is what prediction returns (classes, or the model's quantile outputs).

    Returns (member, entries): the fitted member resident on the device (VramMember), and the tensors raw_entries
    names with their contents, in that order, ready for tirs.write (with the weights, or on their own)."""
    import torch  # device buffers for the fit

    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.ascontiguousarray(y, dtype=np.float32)
    rows, features = x.shape
    s, rs = weights.shape, weights.rows_shape
    chunk = max(int(chunk), 8)
    plan = Plan.new(s["max_classes"], y, classes)
    D = len(plan.bases)
    bases = np.ascontiguousarray(plan.bases, dtype=np.int32)
    xd, yd = torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()
    ck = torch.empty((features, D, rs["col_blocks"], 2, rs["e"], rs["inds"]), dtype=torch.float32, device="cuda")
    rep = torch.empty((rows, s["d"]), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    weights.gpu.check(lib().tcu_fit_rows_device(weights._h, xd.data_ptr(), yd.data_ptr(), rows, features, D,
                                                bases.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), ck.data_ptr(),
                                                rep.data_ptr(), None))
    nodes = []
    try:
        for nd in plan.nodes:
            if nd.rows is None:
                hd = rep if len(plan.nodes) == 1 else rep.clone()
            else:
                hd = rep[torch.as_tensor(np.asarray(nd.rows, dtype=np.int64), device="cuda")].contiguous()
            yn = torch.from_numpy(np.ascontiguousarray(nd.y, dtype=np.float32)).cuda()
            torch.cuda.synchronize()
            nodes.append(fit_icl(weights, hd.data_ptr(), yn.data_ptr(), hd.shape[0], chunk, kv))
            torch.cuda.synchronize()
        col_kv = ck.cpu().numpy()
        weights.gpu.check(lib().tcu_model_set_columns(nodes[0]._h, features, D))
        nodes[0].put_col_kv(col_kv)
        tree = plan.tree(rows)
        member = VramMember.from_nodes(nodes, tree, classes)
    except Exception:
        for m in nodes:
            m.free()
        raise
    out = {prefix + "meta": np.array([rows, features, classes, chunk, kv, D, len(plan.nodes)], np.int32),
           prefix + "tree": tree, prefix + "col_kv": col_kv}
    for i, nd in enumerate(plan.nodes):
        nr = rows if nd.rows is None else len(nd.rows)
        out[prefix + f"n{i}_scale"] = nodes[i].scales()
        for l in range(s["layers"]):
            out[prefix + f"n{i}_kv{l}"] = nodes[i].layer_bytes(l, layer_len(kv, s["d"], nr, chunk))
    return member, out


class CudaFit:
    """fit::Attend on the device (src/fit.rs:25-74; the reference's card implements it at src/gpu.rs:1471-1716): the
    column stage, the row stage and the in-context stage of fitting, offered to a CPU fitting pass, host arrays in and
    out. Weights made with for_fit."""

    def __init__(self, weights):
        self.weights = weights

    def column_batch(self, rows):
        """Feature groups `columns` takes at once (0: not offered)."""
        return int(lib().tcu_fit_column_batch(self.weights._h, rows))

    def columns(self, cells, ind_q):
        """cells [rows][groups][e] (replaced in place by the cells after the stage; through the input layer, the
        target's embedding added), ind_q [blocks][inds][e]: returns rec [groups][blocks][2][e][inds]."""
        assert cells.dtype == np.float32 and cells.flags.c_contiguous
        rows, groups, e = cells.shape
        rs = self.weights.rows_shape
        q = np.ascontiguousarray(ind_q, dtype=np.float32)
        rec = np.empty((groups, rs["col_blocks"], 2, e, rs["inds"]), np.float32)
        self.weights.gpu.check(lib().tcu_fit_columns(self.weights._h, _f32p(cells), rows, groups, _f32p(q), _f32p(rec)))
        return rec

    def row_batch(self, features):
        return int(lib().tcu_fit_row_batch(self.weights._h, features))

    def rows(self, cells):
        """cells [n][features][e] to the rows' representations [n][d]."""
        c = np.ascontiguousarray(cells, dtype=np.float32)
        n, features, _ = c.shape
        reps = np.empty((n, self.weights.shape["d"]), np.float32)
        self.weights.gpu.check(lib().tcu_fit_rows(self.weights._h, _f32p(c), n, features, _f32p(reps)))
        return reps

    def in_context(self, h, scales, sink):
        """h [rows][d] (target's embedding added), scales [layers][d]; sink(layer, k, v) gets each layer's keys and
        values ([rows][d] arrays, copies) in order. Returns True (the stage was done)."""
        h = np.ascontiguousarray(h, dtype=np.float32)
        sc = np.ascontiguousarray(scales, dtype=np.float32)
        rows, d = h.shape
        failed = []

        def cb(_user, layer, k, v):
            try:
                sink(layer, np.ctypeslib.as_array(k, (rows, d)).copy(), np.ctypeslib.as_array(v, (rows, d)).copy())
                return 0
            except Exception as e:  # carried back to the caller after the pass stops
                failed.append(e)
                return 1

        fn = _LayerSink(cb)
        r = lib().tcu_fit_in_context(self.weights._h, _f32p(h), rows, _f32p(sc), fn, None)
        if failed:
            raise failed[0]
        self.weights.gpu.check(r)
        return True


def _b(text):
    return text.encode() if isinstance(text, str) else text


class VramTier:
    """gpu::VramTier (src/gpu.rs:2486-2626): fitted problems resident on one device for many tenants, within `budget`
    bytes in all and `tenant_budget` per tenant (the ledger of src/warm.rs:28-115: the least recently used problem
    makes room, one in use by a prediction is released when it finishes). With background=True a first prediction
    starts its problem's load on a thread and declines meanwhile; otherwise it loads in the call. gpu=None: a tier
    that only keeps its books (the debug_* methods), without a device."""

    def __init__(self, gpu, budget, tenant_budget, background=True):
        self.gpu, self._h = gpu, _c_void()
        r = lib().tcu_tier_new(gpu._h if gpu is not None else None, int(budget), int(tenant_budget), int(background),
                               ctypes.byref(self._h))
        if r != OK:
            raise TcuError(r, "cannot make a tier")

    def _pair(self, f, tenant):
        a, b = _c_size(), _c_size()
        f(self._h, _b(tenant), ctypes.byref(a), ctypes.byref(b))
        return a.value, b.value

    def held(self, tenant):
        """Bytes the tier holds, in all and by `tenant` (loads in progress included)."""
        return self._pair(lib().tcu_tier_held, tenant)

    def ready(self, tenant):
        return int(lib().tcu_tier_ready(self._h, _b(tenant)))

    def on_card(self, tenant):
        """Bytes really on the device, in all and of `tenant` (evicted problems still in use included)."""
        return self._pair(lib().tcu_tier_on_card, tenant)

    @property
    def fallbacks(self):
        return int(lib().tcu_tier_fallbacks(self._h))

    def last_error(self):
        n = lib().tcu_tier_last_error(self._h, None, 0)
        if not n:
            return None
        buf = ctypes.create_string_buffer(n + 1)
        lib().tcu_tier_last_error(self._h, buf, n + 1)
        return buf.value.decode(errors="replace")

    def evict(self, tenant, model=None):
        lib().tcu_tier_evict(self._h, _b(tenant), None if model is None else _b(model))

    def wait(self):
        """Wait for loads started by predictions."""
        lib().tcu_tier_wait(self._h)

    def handle(self, tenant, model, bundle, weights):
        """VramTier::handle: tenant's use of fitted bundle `model` (a name of the caller's), read from `bundle` (a
        path, or the bundle's bytes, read through a positional-read source), an AttendCached."""
        return VramHandle(self, tenant, model, bundle, weights)

    def preload(self, tenant, model, bundle, weights, prefix, node):
        """VramTier::preload: True when problem `node` of member `prefix` is resident afterwards, False when the
        budgets do not allow it (now, or ever)."""
        h = self.handle(tenant, model, bundle, weights)
        try:
            return h.preload(prefix, node)
        finally:
            h.free()

    def debug_admit(self, tenant, model, prefix, node, nbytes):
        """Test hook: a ready entry of `nbytes` through the same claim as a load; True when admitted."""
        r = lib().tcu_tier_debug_admit(self._h, _b(tenant), _b(model), _b(prefix), node, int(nbytes))
        if r < 0:
            raise TcuError(r, "debug_admit")
        return r == 1

    def debug_pin(self, tenant, model, prefix, node):
        """Test hook: hold a ready entry as a prediction holds its problem; returns the pin (or None), released by
        debug_unpin."""
        p = _c_void()
        r = lib().tcu_tier_debug_pin(self._h, _b(tenant), _b(model), _b(prefix), node, ctypes.byref(p))
        return p if r == 1 else None

    @staticmethod
    def debug_unpin(pin):
        lib().tcu_tier_debug_unpin(pin)

    def free(self):
        if self._h:
            lib().tcu_tier_free(self._h)
            self._h = _c_void()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class VramHandle:
    """VramHandle (src/gpu.rs:2628-2701), the AttendCached implementation over a tier: `attend`, `stage` and `rows`
    return None to decline (not resident yet, too large for the tenant, or the device failed: counted in the tier's
    fallbacks)."""

    def __init__(self, tier, tenant, model, bundle, weights):
        self.tier, self.weights, self._h = tier, weights, _c_void()
        if isinstance(bundle, (bytes, bytearray, memoryview)):
            data = np.frombuffer(bundle, dtype=np.uint8)

            def read_at(_user, offset, buf, n):
                if offset + n > data.size:
                    return 1
                ctypes.memmove(buf, data.ctypes.data + offset, n)
                return 0

            self._keep = (data, _READ_AT(read_at))
            src = _Source(None, self._keep[1], data.size)
            r = lib().tcu_tier_handle_source(tier._h, _b(tenant), _b(model), ctypes.byref(src), weights._h,
                                             ctypes.byref(self._h))
        else:
            r = lib().tcu_tier_handle(tier._h, _b(tenant), _b(model), os.fsencode(bundle), weights._h,
                                      ctypes.byref(self._h))
        if r != OK:
            raise TcuError(r, "cannot make a tier handle")

    def preload(self, prefix, node):
        r = lib().tcu_handle_preload(self._h, _b(prefix), node)
        if r < 0:
            raise TcuError(r, self.tier.last_error())
        return r == 1

    def _answer(self, r, out):
        if r < 0:
            raise TcuError(r, self.tier.last_error())
        return out if r == OK else None

    def attend(self, prefix, node, layer, q, d, heads):
        q = np.ascontiguousarray(q, dtype=np.float32).reshape(-1, d)
        out = np.empty_like(q)
        return self._answer(lib().tcu_handle_attend(self._h, _b(prefix), node, layer, _f32p(q), q.shape[0], d, heads,
                                                    _f32p(out)), out)

    def stage(self, prefix, node, h, d, out_n):
        h = np.ascontiguousarray(h, dtype=np.float32).reshape(-1, d)
        out = np.empty((h.shape[0], out_n), dtype=np.float32)
        return self._answer(lib().tcu_handle_stage(self._h, _b(prefix), node, _f32p(h), h.shape[0], d, out_n,
                                                   _f32p(out)), out)

    def rows(self, prefix, x, out_n):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty((x.shape[0], out_n), dtype=np.float32)
        return self._answer(lib().tcu_handle_rows(self._h, _b(prefix), _f32p(x), x.shape[0], x.shape[1], out_n,
                                                  _f32p(out)), out)

    def free(self):
        if self._h:
            lib().tcu_handle_free(self._h)
            self._h = _c_void()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


COMM_ID_BYTES = 128


def comm_unique_id():
    """A fresh id for a communicator over several devices (make it on rank 0, hand it to the others)."""
    buf = ctypes.create_string_buffer(COMM_ID_BYTES)
    r = lib().tcu_comm_unique_id(buf)
    if r != OK:
        raise TcuError(r, "cannot make a communicator id (is libnccl.so.2 installed?)")
    return buf.raw


class Comm:
    """A communicator over the devices of several processes, one rank per device (no reference counterpart)."""

    def __init__(self, gpu, uid, nranks, rank):
        assert len(uid) == COMM_ID_BYTES
        self.gpu, self._h = gpu, _c_void()
        gpu.check(lib().tcu_comm_init(gpu._h, uid, nranks, rank, ctypes.byref(self._h)))
        self.nranks, self.rank = nranks, rank

    def allreduce_f64(self, ptr, count, stream=None):
        return self.gpu.check(lib().tcu_comm_allreduce_f64(self._h, ptr, count, stream))

    def wait(self, timeout_ms, stream=None):
        return self.gpu.check(lib().tcu_comm_wait(self._h, stream, int(timeout_ms)))

    def abort(self):
        """Abort the communicator (a peer has left): nothing waits on it; later collectives fail."""
        return self.gpu.check(lib().tcu_comm_abort(self._h))

    SHARD_PHASES = ("attention", "local_merge", "exchange_states", "merge_states", "dense", "exchange_queries",
                    "decoder_outputs")

    def breakdown(self, enable):
        """Device ms per phase of the last sharded stage run while timing was on (waits for it), then timing on or
        off for the calls that follow."""
        ms = (ctypes.c_double * len(self.SHARD_PHASES))()
        self.gpu.check(lib().tcu_comm_breakdown(self._h, int(enable), ms))
        return dict(zip(self.SHARD_PHASES, [float(v) for v in ms]))

    def free(self):
        if self._h:
            lib().tcu_comm_free(self._h)
            self._h = _c_void()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def shard_chunks(nchunks, world, rank):
    """Rank `rank`'s contiguous share (first chunk, chunks) of `nchunks` stored chunks over `world` devices: the
    first nchunks % world ranks take one more."""
    base, extra = divmod(nchunks, world)
    first = rank * base + min(rank, extra)
    return first, base + (1 if rank < extra else 0)


def attend_noalloc(kv, d, heads, layer_ptr, rows, chunk, q_ptr, nq, out_ptr, stream=None):
    """Few-row attention against one layer's stored keys/values on device buffers, allocating nothing: for
    callers that cannot allocate device memory at call time (during CUDA graph capture, under an external
    arena or allocator, on real-time paths). Its scratch is one static 16 MiB device array shared by every call:
    calls must not overlap on the GPU. Raises TcuError with the library's message when refused."""
    buf = ctypes.create_string_buffer(512)
    r = lib().tcu_attend_noalloc(kv, d, heads, layer_ptr, rows, chunk, q_ptr, nq, out_ptr, stream, buf, 512)
    if r != OK:
        raise TcuError(r, buf.value.decode())
    return r


def fit_icl(weights, h_ptr, y_ptr, rows, chunk=256, kv=KV_F32):
    """Fitting's in-context stage on the device (src/fit.rs:577-747): training rows h (device [rows][d], consumed)
    and targets y (device [rows] float) to a resident cache."""
    h = _c_void()
    weights.gpu.check(lib().tcu_fit_icl_device(weights._h, h_ptr, y_ptr, rows, chunk, kv, ctypes.byref(h)))
    return VramModel(weights, h)


class CudaAttend:
    """The `AttendCached` implementation (src/predict.rs:63-79) over the members of one fitted bundle.

    Each member's problem is loaded on first use (VramHandle::resident, src/gpu.rs:2674-2700 loads it on a thread
    and declines meanwhile; here the load happens in the call). Device failures decline (None) and are counted,
    as VramHandle::or_cpu does (src/gpu.rs:2658-2671).
    """

    def __init__(self, weights, bundle_path):
        self.weights, self.path = weights, bundle_path
        self.models = {}
        self.fallbacks = 0
        self.last_error = None

    def _model(self, prefix, node):
        key = (prefix, node)
        if key not in self.models:
            self.models[key] = VramModel.from_bundle(self.weights, self.path, prefix, node)
        return self.models[key]

    def _or_cpu(self, f):
        try:
            return f()
        except TcuError as e:
            self.fallbacks += 1
            self.last_error = str(e)
            return None

    def attend(self, prefix, node, layer, q, d, heads):
        return self._or_cpu(lambda: self._model(prefix, node).attend(layer, q, d, heads))

    def stage(self, prefix, node, h, d, out_n):
        return self._or_cpu(lambda: self._model(prefix, node).stage(h, out_n, d=d))

    def rows(self, prefix, x, out_n):
        """All three stages for a member of one node (predict.rs:642-652): None when the device declines (no column
        and row stages in the weights or the cache) or fails, as for the other hooks."""
        return self._or_cpu(lambda: self._model(prefix, 0).rows(x, out_n))
