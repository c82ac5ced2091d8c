"""ctypes front end of the CPU checkers: TEST INFRASTRUCTURE ONLY.

Loaded by the test suite, the smoke check and the CPU-baseline leg of the
benchmark, never by the shipped library.  Two checkers live here:

* ``Oracle``   -- the C restatement in conv_oracle.c (fp32 and int8), built
  into oracle/liboracle_conv.so.
* ``RefConv``  -- the reference engine's own Conv2DOp compiled from its sources
  into oracle/_ref/libref_conv.so (absent where the reference tree was not
  available at build time; callers skip in that case).

Arrays are numpy, NCHW, C-contiguous, host memory.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle_conv.so"
REF_SO = HERE / "_ref" / "libref_conv.so"

# auto_pad codes (reference src/ops/traditional/attrs_util.h:18)
AUTO_PAD = {"NOTSET": 0, "": 0, "VALID": 1, "SAME_UPPER": 2, "SAME_LOWER": 3}
# status codes: 0 ok, 1 + ie::Error::Code (reference src/core/base/error.h:10-17)
OK, INVALID_ARGUMENT, UNSUPPORTED = 0, 1, 2

_i64 = C.c_int64
_p = C.c_void_p


class Geom(C.Structure):
    _fields_ = [(name, _i64) for name in (
        "n", "c", "h", "w", "m", "cg", "kh", "kw", "stride_h", "stride_w",
        "dil_h", "dil_w", "pad_t", "pad_l", "pad_b", "pad_r", "group",
        "out_h", "out_w")]


def _ptr(a):
    return None if a is None else a.ctypes.data_as(_p)


def build_oracle() -> None:
    """Compiles the C restatement if its library is missing."""
    if not ORACLE_SO.exists():
        subprocess.run(["make", "-C", str(HERE), "liboracle_conv.so"], check=True,
                       stdout=subprocess.DEVNULL)


class OracleError(RuntimeError):
    def __init__(self, code: int):
        super().__init__(f"oracle status {code}")
        self.code = code


class Oracle:
    def __init__(self):
        build_oracle()
        lib = C.CDLL(str(ORACLE_SO))
        lib.orc_conv_resolve.restype = C.c_int
        lib.orc_conv_resolve.argtypes = [_i64] * 12 + [C.POINTER(_i64), _i64, C.c_int,
                                                        C.c_int, _i64, C.POINTER(Geom)]
        lib.orc_conv2d_f32.restype = C.c_int
        lib.orc_conv2d_f32.argtypes = [C.POINTER(Geom), _p, _p, _p, C.c_int, _p, C.c_int]
        lib.orc_conv2d_q8.restype = C.c_int
        lib.orc_conv2d_q8.argtypes = [C.POINTER(Geom), _p, C.c_int, C.c_int32, _p, _p, _p,
                                      C.c_int32, C.c_int32, C.c_int32, C.c_int, _p, _p,
                                      C.c_int]
        lib.orc_requantize.restype = C.c_int32
        lib.orc_requantize.argtypes = [C.c_int32, C.c_int32, C.c_float, C.c_int32,
                                       C.c_int32, C.c_int32]
        lib.orc_same_padding.restype = None
        lib.orc_same_padding.argtypes = [_i64, _i64, _i64, _i64, C.c_int,
                                         C.POINTER(_i64), C.POINTER(_i64)]
        self.lib = lib

    # -- geometry ---------------------------------------------------------
    def resolve(self, x_shape, w_shape, strides=(1, 1), dilations=(1, 1),
                pads=(0, 0, 0, 0), group=1, auto_pad="NOTSET", depthwise=False,
                bias_len=-1) -> Geom:
        g = Geom()
        pads4 = (_i64 * 4)(*pads)
        rc = self.lib.orc_conv_resolve(*x_shape, *w_shape, strides[0], strides[1],
                                       dilations[0], dilations[1], pads4, group,
                                       AUTO_PAD[auto_pad], int(depthwise), bias_len,
                                       C.byref(g))
        if rc != OK:
            raise OracleError(rc)
        return g

    def same_padding(self, size, kernel, dilation, stride, lower):
        b, a = _i64(), _i64()
        self.lib.orc_same_padding(size, kernel, dilation, stride, int(lower),
                                  C.byref(b), C.byref(a))
        return b.value, a.value

    # -- fp32 -------------------------------------------------------------
    def conv2d_f32(self, x, w, b=None, act=0, nthreads=1, **geom_kw):
        x = np.ascontiguousarray(x, dtype=np.float32)
        w = np.ascontiguousarray(w, dtype=np.float32)
        if b is not None:
            b = np.ascontiguousarray(b, dtype=np.float32)
        g = self.resolve(x.shape, w.shape, bias_len=-1 if b is None else b.shape[0],
                         **geom_kw)
        y = np.empty((g.n, g.m, g.out_h, g.out_w), np.float32)
        rc = self.lib.orc_conv2d_f32(C.byref(g), _ptr(x), _ptr(w), _ptr(b), act,
                                     _ptr(y), nthreads)
        if rc != OK:
            raise OracleError(rc)
        return y

    # -- int8 -------------------------------------------------------------
    def conv2d_q8(self, x, w, bias, mult, zp_x, zp_y, qmin, qmax, y_signed=False,
                  want_acc=False, nthreads=1, **geom_kw):
        assert x.dtype in (np.uint8, np.int8)
        x = np.ascontiguousarray(x)
        w = np.ascontiguousarray(w, dtype=np.int8)
        mult = np.ascontiguousarray(mult, dtype=np.float32)
        if bias is not None:
            bias = np.ascontiguousarray(bias, dtype=np.int32)
        g = self.resolve(x.shape, w.shape, bias_len=-1 if bias is None else bias.shape[0],
                         **geom_kw)
        y = np.empty((g.n, g.m, g.out_h, g.out_w), np.int8 if y_signed else np.uint8)
        acc = np.empty(y.shape, np.int32) if want_acc else None
        rc = self.lib.orc_conv2d_q8(C.byref(g), _ptr(x), int(x.dtype == np.int8), zp_x,
                                    _ptr(w), _ptr(bias), _ptr(mult), zp_y, qmin, qmax,
                                    int(y_signed), _ptr(y), _ptr(acc), nthreads)
        if rc != OK:
            raise OracleError(rc)
        return (y, acc) if want_acc else y

    def requantize(self, acc, bias, mult, zp_y, qmin, qmax):
        return self.lib.orc_requantize(acc, bias, mult, zp_y, qmin, qmax)

    def qadd(self, a, zp_a, mult_a, b, zp_b, mult_b, zp_y, qmin, qmax, y_signed=False):
        """int8 Add of two quantized tensors of one shape (orc_qadd)."""
        assert a.shape == b.shape and a.dtype in (np.uint8, np.int8) and b.dtype in (np.uint8, np.int8)
        a = np.ascontiguousarray(a)
        b = np.ascontiguousarray(b)
        y = np.empty(a.shape, np.int8 if y_signed else np.uint8)
        f = self.lib.orc_qadd
        f.restype = C.c_int
        f.argtypes = [_p, C.c_int, C.c_int32, C.c_float, _p, C.c_int, C.c_int32, C.c_float,
                      C.c_int32, C.c_int32, C.c_int32, C.c_int, _p, _i64]
        rc = f(_ptr(a), int(a.dtype == np.int8), zp_a, mult_a, _ptr(b), int(b.dtype == np.int8),
               zp_b, mult_b, zp_y, qmin, qmax, int(y_signed), _ptr(y), a.size)
        if rc != OK:
            raise OracleError(rc)
        return y


class RefConv:
    """The reference Conv2DOp / DepthwiseConv2DOp, compiled from its sources."""

    def __init__(self):
        if not REF_SO.exists():
            raise FileNotFoundError(str(REF_SO))
        lib = C.CDLL(str(REF_SO))
        lib.ref_row_kernel.restype = C.c_int
        lib.ref_conv2d_f32.restype = C.c_int
        lib.ref_conv2d_f32.argtypes = [_p, _i64, _i64, _i64, _i64, _p, _i64, _i64, _i64,
                                       _i64, _p, _p, _p, _p, _i64, C.c_int, C.c_int,
                                       C.c_int, C.c_int, _p, _p]
        self.lib = lib

    @staticmethod
    def available() -> bool:
        return REF_SO.exists()

    def row_kernel(self) -> str:
        return ["scalar", "sse2", "avx2", "avx512"][self.lib.ref_row_kernel()]

    @staticmethod
    def _explicit_dims(xs, ws, strides, dilations, pads, auto_pad):
        """Output dims for explicit padding, by the reference's own rule
        (conv2d_op.cpp:151-162): (H + pt + pb - (d*(k-1)+1)) / s + 1.  None
        when the library has to answer (auto_pad, an empty batch, a shape the
        op rejects), so its error codes stay the reference's."""
        if auto_pad != "NOTSET" or len(xs) != 4 or len(ws) != 4 or xs[0] <= 0:
            return None
        if min(strides) <= 0 or min(dilations) <= 0 or min(pads) < 0:
            return None
        eh = dilations[0] * (ws[2] - 1) + 1
        ew = dilations[1] * (ws[3] - 1) + 1
        hp = xs[2] + pads[0] + pads[2]
        wp = xs[3] + pads[1] + pads[3]
        if hp < eh or wp < ew:
            return None
        return (xs[0], ws[0], (hp - eh) // strides[0] + 1, (wp - ew) // strides[1] + 1)

    def conv2d(self, x, w, b=None, strides=(1, 1), dilations=(1, 1), pads=(0, 0, 0, 0),
               group=1, auto_pad="NOTSET", depthwise=False, kernel_choice=-1,
               nthreads=1):
        """Returns (status, y); y is None when status != 0."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        w = np.ascontiguousarray(w, dtype=np.float32)
        if b is not None:
            b = np.ascontiguousarray(b, dtype=np.float32)
        s = np.array(strides, np.int64)
        d = np.array(dilations, np.int64)
        p = np.array(pads, np.int64)
        dims = np.zeros(4, np.int64)
        known = self._explicit_dims(x.shape, w.shape, strides, dilations, pads, auto_pad)
        if known is not None:
            dims[:] = known
        else:
            rc = self.lib.ref_conv2d_f32(_ptr(x), *x.shape, _ptr(w), *w.shape, _ptr(b), _ptr(s),
                                         _ptr(d), _ptr(p), group, AUTO_PAD[auto_pad],
                                         int(depthwise), kernel_choice, 1, None, _ptr(dims))
            if rc != OK:
                return rc, None
        y = np.empty(tuple(int(v) for v in dims), np.float32)
        rc = self.lib.ref_conv2d_f32(_ptr(x), *x.shape, _ptr(w), *w.shape, _ptr(b), _ptr(s),
                                     _ptr(d), _ptr(p), group, AUTO_PAD[auto_pad],
                                     int(depthwise), kernel_choice, nthreads, _ptr(y),
                                     _ptr(dims))
        return rc, (y if rc == OK else None)


    def pool2d(self, x, kernel=(1, 1), strides=(1, 1), pads=(0, 0, 0, 0), auto_pad="NOTSET",
               ceil_mode=0, count_include_pad=0, kind="max"):
        """The reference MaxPool2DOp / AvgPool2DOp / GlobalAvgPoolOp (kind "max",
        "avg", "global").  Returns (status, y)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        k = np.array(kernel, np.int64)
        s = np.array(strides, np.int64)
        p = np.array(pads, np.int64)
        dims = np.zeros(4, np.int64)
        mode = {"max": 1, "avg": 0, "global": 2}[kind]
        f = self.lib.ref_pool2d_f32
        f.restype = C.c_int
        args = [_ptr(x), *[C.c_int64(v) for v in x.shape], C.c_int(mode), _ptr(k), _ptr(s),
                _ptr(p), C.c_int(AUTO_PAD[auto_pad]), C.c_int(ceil_mode),
                C.c_int(count_include_pad)]
        rc = f(*args, None, C.c_int64(0), _ptr(dims))
        if rc != OK:
            return rc, None
        y = np.empty(tuple(int(v) for v in dims), np.float32)
        rc = f(*args, _ptr(y), C.c_int64(y.size), _ptr(dims))
        return rc, (y if rc == OK else None)

    def gemm(self, a, b, c=None, alpha=1.0, beta=1.0, trans_a=0, trans_b=0):
        """The reference GemmOp.  Returns (status, y)."""
        a = np.ascontiguousarray(a, dtype=np.float32)
        b = np.ascontiguousarray(b, dtype=np.float32)
        m = a.shape[1] if trans_a else a.shape[0]
        n = b.shape[0] if trans_b else b.shape[1]
        cd = np.zeros(2, np.int64)
        cp, nd = None, 0
        if c is not None:
            c = np.ascontiguousarray(c, dtype=np.float32)
            nd = c.ndim
            cd[:nd] = c.shape
            cp = _ptr(c)
        y = np.empty((max(m, 1), max(n, 1)), np.float32)
        dims = np.zeros(2, np.int64)
        f = self.lib.ref_gemm_f32
        f.restype = C.c_int
        rc = f(_ptr(a), C.c_int64(a.shape[0]), C.c_int64(a.shape[1]), _ptr(b),
               C.c_int64(b.shape[0]), C.c_int64(b.shape[1]), cp, C.c_int(nd), _ptr(cd),
               C.c_double(alpha), C.c_double(beta), C.c_int(trans_a), C.c_int(trans_b), _ptr(y),
               C.c_int64(y.size), _ptr(dims))
        return rc, (y if rc == OK else None)


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def maxpool2d_nchw(x: np.ndarray, k: int, stride: int, pad: int) -> np.ndarray:
    """Max pooling restated from the reference's pool_ops.cpp (:141-166 of its
    MaxPool2D path): windows start at oy*stride - pad, only in-bounds pixels
    compete (the accumulator starts at -inf, so padding never wins), floor
    output size (no ceil_mode)."""
    n, c, h, w = x.shape
    oh = (h + 2 * pad - k) // stride + 1
    ow = (w + 2 * pad - k) // stride + 1
    work = np.float32 if np.issubdtype(x.dtype, np.floating) else np.int32
    big = -np.inf if work is np.float32 else np.iinfo(np.int32).min
    xp = np.full((n, c, h + 2 * pad, w + 2 * pad), big, work)
    xp[:, :, pad:pad + h, pad:pad + w] = x
    out = np.full((n, c, oh, ow), big, work)
    for ky in range(k):
        for kx in range(k):
            win = xp[:, :, ky:ky + stride * (oh - 1) + 1:stride, kx:kx + stride * (ow - 1) + 1:stride]
            np.maximum(out, win, out=out)
    return out.astype(x.dtype)


def resnet_q8_chain(orc: "Oracle", layers, params, x_u8: np.ndarray, nthreads: int = 1,
                    inputs=None):
    """Runs the int8 ResNet-50 conv stack on the CPU oracle.  With ``inputs``
    (a dict name -> NCHW array of the tensor each layer reads) every layer is
    checked on its own, else the chain starts from ``x_u8``.  Returns a dict of
    NCHW uint8 outputs (plus 'pool')."""
    outs = {}
    for l in layers:
        p = params[l.name]
        if inputs is not None and l.src != "input":
            src = inputs[l.src]
        else:
            src = x_u8 if l.src == "input" else outs[l.src]
        outs[l.name] = orc.conv2d_q8(src, p.w, p.bias, p.mult, p.zp_x, 0, 0, 255,
                                     strides=(l.stride, l.stride), pads=(l.pad,) * 4,
                                     nthreads=nthreads)
        if l.name == "stem":
            outs["pool"] = maxpool2d_nchw(outs["stem"], 3, 2, 1)
    return outs
