"""ctypes binding of oracle/liboracle.so — the CPU restatement used as checker."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

import thiran_b200 as thb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
_lib = C.CDLL(os.path.join(ROOT, "oracle", "liboracle.so"))

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_lib.orc_region_eval.restype = C.c_int
_lib.orc_region_eval.argtypes = [C.POINTER(thb.RegionDesc), C.POINTER(thb.AbiArg), C.c_uint64, C.c_void_p, C.c_uint64,
                                 C.c_char_p, C.c_uint64]
for name in ("orc_softmax_rows", "orc_max_rows", "orc_sum_rows", "orc_sum_cols"):
    fn = getattr(_lib, name)
    fn.restype = None
    fn.argtypes = [_f32p, _f32p, C.c_uint64, C.c_uint64]
_lib.orc_sum_all_f64.restype = C.c_double
_lib.orc_sum_all_f64.argtypes = [_f32p, C.c_uint64]
_lib.orc_sum_all_sequential_f32.restype = C.c_float
_lib.orc_sum_all_sequential_f32.argtypes = [_f32p, C.c_uint64]
for name in ("orc_matmul_f32", "orc_matmul_f64acc"):
    fn = getattr(_lib, name)
    fn.restype = None
    fn.argtypes = [_f32p, _f32p, _f32p, C.c_uint64, C.c_uint64, C.c_uint64]
_lib.orc_round_bf16.restype = None
_lib.orc_round_bf16.argtypes = [_f32p, _f32p, C.c_uint64]
_lib.orc_mlp_step.restype = C.c_double
_lib.orc_mlp_step.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, C.c_float,
                              _f32p, _f32p, _f32p, _f32p]
_lib.orc_fnv1a64_f32.restype = C.c_uint64
_lib.orc_fnv1a64_f32.argtypes = [_f32p, C.c_uint64, C.c_uint64]
_lib.orc_sgd_update.restype = None
_lib.orc_sgd_update.argtypes = [_f32p, _f32p, C.c_void_p, C.c_float, C.c_float, C.c_uint64]


class MlpExtras(C.Structure):
    _fields_ = [("b1", C.c_void_p), ("b2", C.c_void_p), ("momentum", C.c_float), ("v_w1", C.c_void_p),
                ("v_b1", C.c_void_p), ("v_w2", C.c_void_p), ("v_b2", C.c_void_p), ("db1", C.c_void_p),
                ("db2", C.c_void_p)]


_m16 = np.ctypeslib.ndpointer(np.float32, shape=(16,), flags="C_CONTIGUOUS")
for _name in ("orc_gfx_identity",):
    getattr(_lib, _name).argtypes = [_m16]
for _name in ("orc_gfx_rotation_x", "orc_gfx_rotation_y", "orc_gfx_rotation_z"):
    getattr(_lib, _name).argtypes = [C.c_float, _m16]
for _name in ("orc_gfx_translation", "orc_gfx_scale"):
    getattr(_lib, _name).argtypes = [C.c_float, C.c_float, C.c_float, _m16]
_lib.orc_gfx_multiply.argtypes = [_m16, _m16, _m16]
_lib.orc_gfx_look_at.restype = C.c_char_p
_lib.orc_gfx_look_at.argtypes = [_f32p, _f32p, _f32p, _m16]
_lib.orc_gfx_perspective.restype = C.c_char_p
_lib.orc_gfx_perspective.argtypes = [C.c_float, C.c_float, C.c_float, C.c_float, _m16]
_lib.orc_gfx_orthographic.restype = C.c_char_p
_lib.orc_gfx_orthographic.argtypes = [C.c_float] * 6 + [_m16]
_lib.orc_render.restype = C.c_char_p
_lib.orc_render.argtypes = [_f32p, C.c_uint64, np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS"), C.c_uint64,
                            _f32p, _m16, _m16, _m16, C.c_uint64, C.c_uint64, _f32p, _f32p, _f32p,
                            np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")]
_lib.orc_mlp_step_ex.restype = C.c_double
_lib.orc_mlp_step_ex.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64,
                                 C.c_float, _f32p, _f32p, _f32p, _f32p, C.POINTER(MlpExtras)]


class OracleFailure(RuntimeError):
    def __init__(self, status, code):
        super().__init__(code)
        self.status, self.code = status, code


def region_eval(spec: "thb.RegionSpec", inputs, output_shape=None):
    """Evaluates a region on the CPU restatement; raises OracleFailure."""
    args, keep = thb._host_args(inputs)
    shape = spec.infer_output_shape(inputs) if output_shape is None else list(output_shape)
    out = np.empty(shape, dtype=thb._NP[spec.output_dtype])
    fail = C.create_string_buffer(256)
    status = _lib.orc_region_eval(C.byref(spec.desc), args, len(inputs), out.ctypes.data if out.size else None,
                                  out.size, fail, 256)
    if status:
        raise OracleFailure(status, fail.value.decode())
    return out if shape else out.reshape(()).item()


def softmax_rows(x):
    y = np.empty_like(x)
    _lib.orc_softmax_rows(x, y, x.shape[0], x.shape[1])
    return y


def max_rows(x):
    y = np.empty(x.shape[0], np.float32)
    _lib.orc_max_rows(x, y, x.shape[0], x.shape[1])
    return y


def sum_rows(x):
    y = np.empty(x.shape[0], np.float32)
    _lib.orc_sum_rows(x, y, x.shape[0], x.shape[1])
    return y


def sum_cols(x):
    y = np.empty(x.shape[1], np.float32)
    _lib.orc_sum_cols(x, y, x.shape[0], x.shape[1])
    return y


def sum_all_f64(x):
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    return _lib.orc_sum_all_f64(x, x.size)


def sum_all_sequential_f32(x):
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    return _lib.orc_sum_all_sequential_f32(x, x.size)


def matmul_f32(a, b):
    c = np.empty((a.shape[0], b.shape[1]), np.float32)
    _lib.orc_matmul_f32(np.ascontiguousarray(a), np.ascontiguousarray(b), c, a.shape[0], a.shape[1], b.shape[1])
    return c


def matmul_f64acc(a, b):
    c = np.empty((a.shape[0], b.shape[1]), np.float32)
    _lib.orc_matmul_f64acc(np.ascontiguousarray(a), np.ascontiguousarray(b), c, a.shape[0], a.shape[1], b.shape[1])
    return c


def round_bf16(x):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    _lib.orc_round_bf16(x.reshape(-1), y.reshape(-1), x.size)
    return y


def mlp_step(x, t, w1, w2, lr):
    """Returns (loss, dW1, dW2, hidden, y); updates w1/w2 in place."""
    b, i = x.shape
    h = w1.shape[1]
    o = w2.shape[1]
    dw1 = np.empty((i, h), np.float32)
    dw2 = np.empty((h, o), np.float32)
    hidden = np.empty((b, h), np.float32)
    y = np.empty((b, o), np.float32)
    loss = _lib.orc_mlp_step(x, t, w1, w2, b, i, h, o, lr, dw1, dw2, hidden, y)
    return loss, dw1, dw2, hidden, y


class gfx:
    """Matrix helpers of the oracle's renderer (16 f32, row-major)."""

    @staticmethod
    def _m(fn, *args):
        m = np.empty(16, np.float32)
        err = fn(*args, m)
        if err:
            raise OracleFailure(2, err.decode())
        return m

    identity = staticmethod(lambda: gfx._m(_lib.orc_gfx_identity))
    rotation_x = staticmethod(lambda r: gfx._m(_lib.orc_gfx_rotation_x, r))
    rotation_y = staticmethod(lambda r: gfx._m(_lib.orc_gfx_rotation_y, r))
    rotation_z = staticmethod(lambda r: gfx._m(_lib.orc_gfx_rotation_z, r))
    translation = staticmethod(lambda x, y, z: gfx._m(_lib.orc_gfx_translation, x, y, z))
    scale = staticmethod(lambda x, y, z: gfx._m(_lib.orc_gfx_scale, x, y, z))
    multiply = staticmethod(lambda a, b: gfx._m(_lib.orc_gfx_multiply, a, b))
    perspective = staticmethod(lambda fovy, aspect, n, f: gfx._m(_lib.orc_gfx_perspective, fovy, aspect, n, f))
    orthographic = staticmethod(lambda *a: gfx._m(_lib.orc_gfx_orthographic, *a))

    @staticmethod
    def look_at(eye, target, up):
        return gfx._m(_lib.orc_gfx_look_at, np.asarray(eye, np.float32), np.asarray(target, np.float32),
                      np.asarray(up, np.float32))


def render(positions, indices, colors, model, view, projection, width, height, clear=(0, 0, 0, 0)):
    """orc_render: returns (color [w*h,4], depth [w*h], stats [4])."""
    positions = np.ascontiguousarray(positions, np.float32).reshape(-1, 3)
    colors = np.ascontiguousarray(colors, np.float32).reshape(-1, 4)
    indices = np.ascontiguousarray(indices, np.int64).reshape(-1, 3)
    color = np.empty((width * height, 4), np.float32)
    depth = np.empty(width * height, np.float32)
    stats = np.zeros(4, np.uint64)
    err = _lib.orc_render(positions.reshape(-1), positions.shape[0], indices.reshape(-1), indices.shape[0],
                          colors.reshape(-1), model, view, projection, width, height,
                          np.asarray(clear, np.float32), color.reshape(-1), depth, stats)
    if err:
        raise OracleFailure(2, err.decode())
    return color, depth, stats


def fnv_floats(values, basis=14695981039346656037):
    """The reference's f32 digests: the framebuffer digest (Graphics.cpp:
    188-200) with the default basis; the qualification output digest
    (benchmarks/th023/Qualification.cpp:176-187) with 1469598103934665603."""
    flat = np.ascontiguousarray(values, np.float32).reshape(-1)
    return f"fnv1a64:{_lib.orc_fnv1a64_f32(flat, flat.size, basis):016x}"


def sgd_update(p, g, lr, v=None, momentum=0.0):
    """orc_sgd_update in place on f32 arrays (v: velocity or None)."""
    _lib.orc_sgd_update(p.reshape(-1), g.reshape(-1), None if v is None else v.ctypes.data, momentum, lr, p.size)


def mlp_step_ex(x, t, w1, w2, lr, b1=None, b2=None, momentum=0.0, velocities=None):
    """orc_mlp_step_ex: biases (updated in place) and SGD with momentum
    (`velocities` = [vW1, vb1, vW2, vb2], updated in place). Returns
    (loss, dW1, dW2, db1, db2, hidden, y)."""
    b, i = x.shape
    h = w1.shape[1]
    o = w2.shape[1]
    dw1 = np.empty((i, h), np.float32)
    dw2 = np.empty((h, o), np.float32)
    db1 = np.zeros(h, np.float32)
    db2 = np.zeros(o, np.float32)
    hidden = np.empty((b, h), np.float32)
    y = np.empty((b, o), np.float32)
    ptr = lambda a: None if a is None else a.ctypes.data
    v = velocities or [None] * 4
    ex = MlpExtras(ptr(b1), ptr(b2), momentum, ptr(v[0]), ptr(v[1]), ptr(v[2]), ptr(v[3]), db1.ctypes.data,
                   db2.ctypes.data)
    loss = _lib.orc_mlp_step_ex(x, t, w1, w2, b, i, h, o, lr, dw1, dw2, hidden, y, C.byref(ex))
    return loss, dw1, dw2, db1, db2, hidden, y
