"""ctypes binding of the C ABI in include/ie_cuda_conv.h.

The library is required: importing this module without the built
libie_cuda_conv.so raises, so no caller can silently fall back to a CPU path.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libie_cuda_conv.so"

# ie_status (mirrors ie::Error::Code + 1, reference src/core/base/error.h:10-17)
IE_OK = 0
IE_INVALID_ARGUMENT = 1
IE_UNSUPPORTED = 2
IE_NOT_FOUND = 3
IE_ALREADY_EXISTS = 4
IE_OUT_OF_MEMORY = 5
IE_RUNTIME = 6
STATUS_NAMES = {0: "Ok", 1: "InvalidArgument", 2: "Unsupported", 3: "NotFound",
                4: "AlreadyExists", 5: "OutOfMemory", 6: "Runtime"}

IE_PAD = {"NOTSET": 0, "": 0, "VALID": 1, "SAME_UPPER": 2, "SAME_LOWER": 3}
IE_ACT_NONE, IE_ACT_RELU, IE_ACT_RELU6 = 0, 1, 2
IE_Y_F32_NHWC, IE_Y_F32_NCHW, IE_Y_BF16X2_NHWC = 0, 1, 2
IE_TILE_FILL, IE_TILE_DEFAULT = 0, 1

_i64 = C.c_int64
_i32 = C.c_int32
_p = C.c_void_p


class ConvDesc(C.Structure):
    _fields_ = [(n, _i64) for n in ("n", "c", "h", "w", "m", "kh", "kw", "stride_h",
                                    "stride_w", "dil_h", "dil_w", "pad_top", "pad_left",
                                    "pad_bottom", "pad_right", "group")] + \
               [("auto_pad", _i32), ("depthwise", _i32)]


class ConvShape(C.Structure):
    _fields_ = [(n, _i64) for n in ("pad_top", "pad_left", "pad_bottom", "pad_right",
                                    "out_h", "out_w")]


class PoolDesc(C.Structure):
    _fields_ = [(n, _i64) for n in ("n", "c", "h", "w", "kh", "kw", "stride_h", "stride_w",
                                    "pad_top", "pad_left", "pad_bottom", "pad_right")] + \
               [("auto_pad", _i32), ("ceil_mode", _i32), ("count_include_pad", _i32)]


class Q8Params(C.Structure):
    _fields_ = [(n, _i32) for n in ("x_signed", "zp_x", "y_signed", "zp_y", "qmin", "qmax")]


class QAddParams(C.Structure):
    _fields_ = [("a_signed", _i32), ("zp_a", _i32), ("mult_a", C.c_float),
                ("b_signed", _i32), ("zp_b", _i32), ("mult_b", C.c_float),
                ("y_signed", _i32), ("zp_y", _i32), ("qmin", _i32), ("qmax", _i32)]


class ConvPlan(C.Structure):
    _fields_ = [(n, _i32) for n in ("bn", "bk_bytes", "m_sub", "stages", "resident_weights",
                                    "out_bufs", "row_band", "grid", "a_tiled")]


class CudaConvError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {message}")
        self.code = code


def _load() -> C.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH.name} is not built; run `python -m computeengine_b200.build` "
            "(there is no CPU fallback)")
    lib = C.CDLL(str(LIB_PATH))
    P = C.POINTER
    sig = {
        "ie_conv2d_resolve": (C.c_int, [P(ConvDesc), _i64, P(ConvShape)]),
        "ie_cuda_q8_packed_weight_bytes": (C.c_size_t, [P(ConvDesc)]),
        "ie_cuda_q8_pack_weights": (C.c_int, [P(ConvDesc), _p, _p, _p]),
        "ie_cuda_q8_pack_input": (C.c_int, [_p, _p, _i64, _i64, _i64, _i64, _i64, _i32, _p]),
        "ie_cuda_q8_unpack_output": (C.c_int, [_p, _p, _i64, _i64, _i64, _i64, _i64, _p]),
        "ie_cuda_q8_halo_input_bytes": (C.c_size_t, [P(ConvDesc)]),
        "ie_cuda_q8_pack_input_halo": (C.c_int, [P(ConvDesc), _p, _p, _i32, _p]),
        "ie_cuda_q8_halo_nhwc": (C.c_int, [P(ConvDesc), _p, _p, _i32, _p]),
        "ie_cuda_conv2d_q8": (C.c_int, [P(ConvDesc), P(Q8Params), _p, _p, _p, _p, _p, _p]),
        "ie_cuda_conv2d_q8_acc": (C.c_int, [P(ConvDesc), P(Q8Params), _p, _p, _p, _p, _p]),
        "ie_cuda_dw_q8_packed_weight_bytes": (C.c_size_t, [P(ConvDesc)]),
        "ie_cuda_dw_q8_pack_weights": (C.c_int, [P(ConvDesc), _p, _p, _p]),
        "ie_cuda_dwconv2d_q8": (C.c_int, [P(ConvDesc), P(Q8Params), _p, _p, _p, _p, _p, _p]),
        "ie_cuda_q8_stem_desc": (C.c_int, [_i64, _i64, _i64, _i64, _i64, P(ConvDesc)]),
        "ie_cuda_q8_stem_pack_input": (C.c_int, [_p, _p, _i64, _i64, _i64, _i64, _i32, _p]),
        "ie_cuda_q8_stem_pack_weights": (C.c_int, [_p, _p, _i64, _i64, _p]),
        "ie_cuda_q8_maxpool2d": (C.c_int, [_p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                           _i32, _p]),
        "ie_cuda_f32_packed_weight_bytes": (C.c_size_t, [P(ConvDesc)]),
        "ie_cuda_f32_pack_weights": (C.c_int, [P(ConvDesc), _p, _p, _p]),
        "ie_cuda_f32_pack_input": (C.c_int, [_p, _p, _i64, _i64, _i64, _i64, _i64, _p]),
        "ie_cuda_conv2d_bf16x3": (C.c_int, [P(ConvDesc), _i32, _p, _p, _p, _p, _i32, _p]),
        "ie_cuda_conv2d_f32_workspace_bytes": (C.c_size_t, [P(ConvDesc)]),
        "ie_cuda_conv2d_f32": (C.c_int, [P(ConvDesc), _i32, _p, _p, _p, _p, _p, C.c_size_t, _p]),
        "ie_cuda_noalloc_scratch_bytes": (C.c_size_t, []),
        "ie_cuda_conv2d_f32_noalloc": (C.c_int, [P(ConvDesc), _i32, _p, _p, _p, _p, _p]),
        "ie_cuda_last_error": (C.c_char_p, []),
        "ie_cuda_take_device_error": (C.c_int, [P(C.c_uint32)]),
        "ie_cuda_bounded_wait_probe": (C.c_int, [C.c_uint64, P(C.c_uint64), _p]),
        "ie_cuda_qadd": (C.c_int, [P(QAddParams), _p, _p, _p, _i64, _p]),
        "ie_cuda_launch_count": (C.c_uint64, [C.c_int]),
        "ie_cuda_last_plan": (C.c_int, [P(ConvPlan)]),
        "ie_cuda_conv2d_f32_residual": (C.c_int, [P(ConvDesc), _i32, _p, _p, _p, _p, _p, _p,
                                                  C.c_size_t, _p]),
        "ie_cuda_conv2d_bf16x3_residual": (C.c_int, [P(ConvDesc), _i32, _p, _p, _p, _p, _p, _i32,
                                                     _p]),
        "ie_pool2d_resolve": (C.c_int, [P(PoolDesc), P(ConvShape)]),
        "ie_cuda_pool2d_f32": (C.c_int, [P(PoolDesc), _i32, _p, _p, _p]),
        "ie_cuda_q8_maxpool2d_nhwc": (C.c_int, [P(PoolDesc), _i32, _p, _p, _p]),
        "ie_cuda_set_tile_policy": (C.c_int, [_i32, P(_i32)]),
        "ie_cuda_mma_i8_peak": (C.c_int, [_i32, P(C.c_double), _p]),
        "ie_cuda_q8_global_avg_pool_nhwc": (C.c_int, [_p, _p, _i64, _i64, _i64, _i64, _i32, _i32,
                                                      C.c_double, _p]),
        "ie_cuda_global_avg_pool_f32": (C.c_int, [_p, _p, _i64, _i64, _i64, _i64, _p]),
        "ie_cuda_gemm_f32_workspace_bytes": (C.c_size_t, [_i64, _i64, _i64, _i32, _i32]),
        "ie_cuda_gemm_f32": (C.c_int, [_i64, _i64, _i64, _i32, _i32, C.c_float, C.c_float, _p,
                                       _p, _p, _i32, _p, _p, C.c_size_t, _p]),
        "ie_cuda_f32x2_maxpool2d": (C.c_int, [_p, _p] + [_i64] * 7 + [_p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def check(code: int) -> None:
    """Raises CudaConvError for a non-zero status, with the library's detail."""
    if code != IE_OK:
        raise CudaConvError(code, lib.ie_cuda_last_error().decode(errors="replace"))


def take_device_error() -> int:
    v = C.c_uint32(0)
    check(lib.ie_cuda_take_device_error(C.byref(v)))
    return int(v.value)


def launch_count(reset: bool = False) -> int:
    return int(lib.ie_cuda_launch_count(1 if reset else 0))


def set_tile_policy(policy: int) -> int:
    """Sets the int8 tile policy (IE_TILE_FILL / IE_TILE_DEFAULT); returns the
    previous one."""
    prev = _i32()
    check(lib.ie_cuda_set_tile_policy(policy, C.byref(prev)))
    return prev.value


def last_plan() -> ConvPlan:
    """Tile plan of this thread's last implicit-GEMM launch."""
    p = ConvPlan()
    check(lib.ie_cuda_last_plan(p))
    return p
