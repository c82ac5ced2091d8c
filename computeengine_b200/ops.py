"""Host-side mirror of the reference engine's Conv2D operator interface.

The reference drives convolution through ``Op::configure(attrs)`` and
``Op::forward(inputs, outputs, ctx)`` (src/core/ops/op.h:27-54), looked up in
an ``OpRegistry`` (src/core/ops/op_registry.h:15-30).  This module keeps those
names, argument meanings and error codes for the CUDA backend:

* ``Conv2DOp`` / ``DepthwiseConv2DOp``  -- fp32, same semantics as
  conv2d_op.h:36-67, run on the B200 kernels (bf16x3 tensor cores for dense
  convolutions, CUDA cores for grouped / depthwise ones).
* ``QLinearConv2DOp`` -- the int8-quantized form the reference only plans
  (quant_plugins.h:7-22 is a stub): uint8/int8 activations, per-channel int8
  weights, int32 bias, fused requantize + ReLU/ReLU6.
* ``OpRegistry`` + ``register_cuda_ops`` -- registration with the reference's
  AlreadyExists behaviour (op_registry.cpp:23-32).

Tensors are torch tensors on a CUDA device (NCHW).  There is no CPU fallback:
a CPU tensor is an InvalidArgument, and the module fails to import when the
CUDA library is not built.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional

import torch

from . import _lib
from ._lib import ConvDesc, ConvShape, Q8Params, lib


class Code(enum.IntEnum):
    """ie::Error::Code (reference src/core/base/error.h:10-17)."""
    InvalidArgument = 0
    Unsupported = 1
    NotFound = 2
    AlreadyExists = 3
    OutOfMemory = 4
    Runtime = 5


@dataclass
class Status:
    """ie::Status: empty on success, else an error code and message."""
    code: Optional[Code] = None
    message: str = ""

    def has_value(self) -> bool:
        return self.code is None

    __bool__ = has_value

    @staticmethod
    def error(code: Code, message: str) -> "Status":
        return Status(code, message)


OK = Status()


def _from_abi(rc: int) -> Status:
    if rc == _lib.IE_OK:
        return OK
    return Status(Code(rc - 1), lib.ie_cuda_last_error().decode(errors="replace"))


AUTO_PAD = {"NOTSET": 0, "": 0, "VALID": 1, "SAME_UPPER": 2, "SAME_LOWER": 3}


@dataclass
class ConvConfig:
    """ConvConfig (reference conv2d_op.h:13-21)."""
    strides: tuple = (1, 1)
    dilations: tuple = (1, 1)
    pads: tuple = (0, 0, 0, 0)  # top, left, bottom, right
    group: int = 1
    auto_pad: str = "NOTSET"
    kernel_shape: Optional[tuple] = None


def _int_list(attrs, key):
    if key not in attrs:
        return None, OK
    v = attrs[key]
    if not isinstance(v, (list, tuple)) or not all(isinstance(i, int) and not isinstance(i, bool)
                                                   for i in v):
        return None, Status.error(Code.InvalidArgument, f"attribute '{key}' must be an int list")
    return list(v), OK


def parse_conv_config(attrs: dict) -> tuple[ConvConfig, Status]:
    """parse_conv_config (reference conv2d_op.cpp:26-71, attrs_util.h:109-180)."""
    cfg = ConvConfig()
    for key in ("strides", "dilations"):
        v, st = _int_list(attrs, key)
        if not st:
            return cfg, st
        if v is not None:
            if len(v) != 2:
                return cfg, Status.error(Code.InvalidArgument, f"{key} must contain 2 values")
            if v[0] <= 0 or v[1] <= 0:
                return cfg, Status.error(Code.InvalidArgument, f"{key} values must be positive")
            setattr(cfg, key, tuple(v))
    v, st = _int_list(attrs, "pads")
    if not st:
        return cfg, st
    if v:
        if len(v) == 2:
            pads = (v[0], v[1], v[0], v[1])
        elif len(v) == 4:
            pads = tuple(v)
        else:
            return cfg, Status.error(Code.InvalidArgument, "pads must contain 2 or 4 values")
        if any(p < 0 for p in pads):
            return cfg, Status.error(Code.InvalidArgument, "pads must be non-negative")
        cfg.pads = pads
    if "group" in attrs:
        g = attrs["group"]
        if isinstance(g, bool):
            g = int(g)
        if not isinstance(g, int):
            return cfg, Status.error(Code.InvalidArgument, "attribute 'group' must be an int")
        if g <= 0:
            return cfg, Status.error(Code.InvalidArgument, "group must be positive")
        cfg.group = g
    if "auto_pad" in attrs:
        a = attrs["auto_pad"]
        if not isinstance(a, str):
            return cfg, Status.error(Code.InvalidArgument, "attribute 'auto_pad' must be a string")
        if a not in AUTO_PAD:
            return cfg, Status.error(Code.InvalidArgument, "unsupported auto_pad: " + a)
        cfg.auto_pad = a or "NOTSET"
    v, st = _int_list(attrs, "kernel_shape")
    if not st:
        return cfg, st
    if v is not None:
        if len(v) != 2:
            return cfg, Status.error(Code.InvalidArgument, "kernel_shape must contain 2 values")
        if v[0] <= 0 or v[1] <= 0:
            return cfg, Status.error(Code.InvalidArgument, "kernel_shape values must be positive")
        cfg.kernel_shape = tuple(v)
    return cfg, OK


def make_desc(cfg: ConvConfig, x_shape, w_shape, depthwise: bool) -> ConvDesc:
    d = ConvDesc()
    d.n, d.c, d.h, d.w = (int(v) for v in x_shape)
    d.m, _, d.kh, d.kw = (int(v) for v in w_shape)
    d.stride_h, d.stride_w = cfg.strides
    d.dil_h, d.dil_w = cfg.dilations
    d.pad_top, d.pad_left, d.pad_bottom, d.pad_right = cfg.pads
    d.group = cfg.group
    d.auto_pad = AUTO_PAD[cfg.auto_pad]
    d.depthwise = int(depthwise)
    return d


def _stream_handle() -> int:
    return torch.cuda.current_stream().cuda_stream


def _validate_common(inputs, outputs, want_dtypes, op_name) -> Status:
    """conv2d_op.cpp:77-102 guards (count, null, dtype, rank), plus device."""
    if len(inputs) < 2 or len(inputs) > 3 or len(outputs) != 1:
        return Status.error(Code.InvalidArgument, f"{op_name} expects two or three inputs and one output")
    for i, t in enumerate(inputs):
        if t is None:
            return Status.error(Code.InvalidArgument, "null tensor or buffer")
        if t.dtype not in want_dtypes[min(i, len(want_dtypes) - 1)]:
            return Status.error(Code.Unsupported, f"{op_name}: unsupported dtype {t.dtype}")
        if not t.is_cuda:
            return Status.error(Code.InvalidArgument, f"{op_name}: tensors must be on a CUDA device")
    if inputs[0].dim() != 4 or inputs[1].dim() != 4:
        return Status.error(Code.InvalidArgument, f"{op_name} expects 4D NCHW tensors")
    return OK


def _check_shapes(cfg, x, w, bias, depthwise) -> tuple[Optional[ConvDesc], Optional[ConvShape], Status]:
    d = make_desc(cfg, x.shape, w.shape, depthwise)
    if d.group > 0 and d.c % d.group == 0 and int(w.shape[1]) != d.c // d.group:
        return None, None, Status.error(Code.InvalidArgument, "Conv2D weight channels do not match C/group")
    if cfg.kernel_shape is not None and tuple(cfg.kernel_shape) != (d.kh, d.kw):
        return None, None, Status.error(Code.InvalidArgument, "kernel_shape does not match the weight tensor")
    bias_len = -1
    if bias is not None:
        if bias.dim() != 1:
            return None, None, Status.error(Code.InvalidArgument, "Conv2D bias must have shape [M]")
        bias_len = int(bias.shape[0])
    s = ConvShape()
    st = _from_abi(lib.ie_conv2d_resolve(d, bias_len, s))
    if not st:
        return None, None, st
    return d, s, OK


class Op:
    """Op (reference src/core/ops/op.h:27-54)."""

    def configure(self, attrs: dict) -> Status:  # noqa: D401
        return OK

    def forward(self, inputs: List[torch.Tensor], outputs: list, context=None) -> Status:
        raise NotImplementedError

    def backward(self, *args, **kwargs) -> Status:
        return Status.error(Code.Unsupported, "backward not implemented")

    def supports_training(self) -> bool:
        return False


def _act_from_attrs(attrs) -> tuple[int, Status]:
    act = attrs.get("activation", "NONE")
    table = {"NONE": _lib.IE_ACT_NONE, "RELU": _lib.IE_ACT_RELU, "RELU6": _lib.IE_ACT_RELU6}
    if act not in table:
        return 0, Status.error(Code.InvalidArgument, f"unsupported activation: {act}")
    return table[act], OK


class Conv2DOp(Op):
    """fp32 Conv2D on the B200 (reference Conv2DOp, conv2d_op.h:36-50).

    Inputs [x, w] or [x, w, b] NCHW fp32 CUDA tensors; outputs[0] receives the
    new [N, M, Ho, Wo] tensor, like ``*outputs[0] = std::move(*result)``
    (conv2d_op.cpp:243).  The optional attribute ``activation`` ("RELU",
    "RELU6") folds the graph's following Relu / Clip node into the epilogue.
    """

    depthwise = False

    def __init__(self):
        self.config = ConvConfig()
        self.act = _lib.IE_ACT_NONE

    def configure(self, attrs: dict) -> Status:
        self.config, st = parse_conv_config(attrs)
        if not st:
            return st
        self.act, st = _act_from_attrs(attrs)
        return st

    def forward(self, inputs, outputs, context=None) -> Status:
        st = _validate_common(inputs, outputs, [(torch.float32,)], "Conv2D")
        if not st:
            return st
        x, w = inputs[0], inputs[1]
        b = inputs[2] if len(inputs) == 3 else None
        d, s, st = _check_shapes(self.config, x, w, b, self.depthwise)
        if not st:
            return st
        x = x.contiguous()
        w = w.contiguous()
        b = b.contiguous() if b is not None else None
        y = torch.empty((d.n, d.m, s.out_h, s.out_w), dtype=torch.float32, device=x.device)
        ws_bytes = int(lib.ie_cuda_conv2d_f32_workspace_bytes(d))
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
        rc = lib.ie_cuda_conv2d_f32(d, self.act, x.data_ptr(), w.data_ptr(),
                                    b.data_ptr() if b is not None else None, y.data_ptr(),
                                    ws.data_ptr(), ws_bytes, _stream_handle())
        st = _from_abi(rc)
        if st:
            outputs[0] = y
        return st


class DepthwiseConv2DOp(Conv2DOp):
    """Depthwise fp32 convolution: Conv2D with group == C (conv2d_op.h:53-67)."""
    depthwise = True


@dataclass
class QuantParams:
    """Per-tensor activation / per-channel weight quantization of one conv."""
    x_zero_point: int = 0
    y_zero_point: int = 0
    y_signed: bool = False
    qmin: Optional[int] = None
    qmax: Optional[int] = None


class QLinearConv2DOp(Op):
    """int8-quantized Conv2D (dense or depthwise) on the B200.

    Inputs: x uint8/int8 NCHW, w int8 [M, C/g, kH, kW], optional bias int32
    [M].  Attributes: the Conv2D attributes plus ``multiplier`` (per-channel
    list, s_x * s_w[m] / s_y, computed on the host in double and rounded to
    fp32), ``x_zero_point``, ``y_zero_point``, ``y_signed``, and the output
    clamp ``qmin`` / ``qmax`` (ReLU / ReLU6 folded in).  Output uint8/int8
    NCHW, bit-exact with the int8 oracle's requantize rule.
    """

    def __init__(self):
        self.config = ConvConfig()
        self.q = QuantParams()
        self.mult: Optional[list] = None

    def configure(self, attrs: dict) -> Status:
        self.config, st = parse_conv_config(attrs)
        if not st:
            return st
        mult = attrs.get("multiplier")
        if mult is None or not isinstance(mult, (list, tuple)) or not mult:
            return Status.error(Code.InvalidArgument, "attribute 'multiplier' must be a float list")
        self.mult = [float(v) for v in mult]
        self.q = QuantParams(int(attrs.get("x_zero_point", 0)), int(attrs.get("y_zero_point", 0)),
                             bool(attrs.get("y_signed", False)), attrs.get("qmin"), attrs.get("qmax"))
        return OK

    def forward(self, inputs, outputs, context=None) -> Status:
        st = _validate_common(inputs, outputs, [(torch.uint8, torch.int8), (torch.int8,),
                                                (torch.int32,)], "QLinearConv2D")
        if not st:
            return st
        x, w = inputs[0], inputs[1]
        b = inputs[2] if len(inputs) == 3 else None
        depthwise = self.config.group > 1
        d, s, st = _check_shapes(self.config, x, w, b, False)
        if not st:
            return st
        if len(self.mult) != d.m:
            return Status.error(Code.InvalidArgument, "multiplier must have M values")
        x_signed = x.dtype == torch.int8
        lo, hi = (-128, 127) if self.q.y_signed else (0, 255)
        qp = Q8Params()
        qp.x_signed = int(x_signed)
        qp.zp_x = self.q.x_zero_point
        qp.y_signed = int(self.q.y_signed)
        qp.zp_y = self.q.y_zero_point
        qp.qmin = lo if self.q.qmin is None else int(self.q.qmin)
        qp.qmax = hi if self.q.qmax is None else int(self.q.qmax)
        dev = x.device
        mult = torch.tensor(self.mult, dtype=torch.float32, device=dev)
        stream = _stream_handle()
        c_store = (d.c + 15) // 16 * 16
        m_store = (d.m + 15) // 16 * 16
        xor, halo = 0, False
        if not depthwise:
            if d.group != 1:
                return Status.error(Code.Unsupported, "grouped int8 convolution (1 < group < C)")
            if qp.zp_x != 0:
                # uint8 with zero point 128 is int8 with zero point 0 after
                # flipping the top bit; any other zero point reads a haloed
                # input whose padding holds the zero point
                if not x_signed and qp.zp_x == 128:
                    xor, qp.zp_x, qp.x_signed = 0x80, 0, 1
                else:
                    halo = True
        elif not (d.group == d.c == d.m and int(w.shape[1]) == 1):
            return Status.error(Code.Unsupported, "grouped int8 convolution (1 < group < C)")
        if halo:
            x_nhwc = torch.empty(int(lib.ie_cuda_q8_halo_input_bytes(d)), dtype=torch.uint8,
                                 device=dev)
            rc = lib.ie_cuda_q8_pack_input_halo(d, x.contiguous().data_ptr(), x_nhwc.data_ptr(),
                                                qp.zp_x, stream)
        else:
            x_nhwc = torch.empty((d.n, d.h, d.w, c_store), dtype=torch.uint8, device=dev)
            rc = lib.ie_cuda_q8_pack_input(x.contiguous().data_ptr(), x_nhwc.data_ptr(), d.n,
                                           d.c, d.h, d.w, c_store, xor, stream)
        if rc:
            return _from_abi(rc)
        y_nhwc = torch.empty((d.n, s.out_h, s.out_w, m_store), dtype=torch.uint8, device=dev)
        bias_ptr = b.contiguous().data_ptr() if b is not None else None
        if depthwise:
            packed = torch.empty(int(lib.ie_cuda_dw_q8_packed_weight_bytes(d)), dtype=torch.uint8,
                                 device=dev)
            rc = lib.ie_cuda_dw_q8_pack_weights(d, w.contiguous().data_ptr(), packed.data_ptr(),
                                                stream)
            if not rc:
                rc = lib.ie_cuda_dwconv2d_q8(d, qp, x_nhwc.data_ptr(), packed.data_ptr(), bias_ptr,
                                             mult.data_ptr(), y_nhwc.data_ptr(), stream)
        else:
            packed = torch.empty(int(lib.ie_cuda_q8_packed_weight_bytes(d)), dtype=torch.uint8,
                                 device=dev)
            rc = lib.ie_cuda_q8_pack_weights(d, w.contiguous().data_ptr(), packed.data_ptr(), stream)
            if not rc:
                rc = lib.ie_cuda_conv2d_q8(d, qp, x_nhwc.data_ptr(), packed.data_ptr(), bias_ptr,
                                           mult.data_ptr(), y_nhwc.data_ptr(), stream)
        if rc:
            return _from_abi(rc)
        y = torch.empty((d.n, d.m, s.out_h, s.out_w),
                        dtype=torch.int8 if self.q.y_signed else torch.uint8, device=dev)
        rc = lib.ie_cuda_q8_unpack_output(y_nhwc.data_ptr(), y.data_ptr(), d.n, d.m, s.out_h,
                                          s.out_w, m_store, stream)
        st = _from_abi(rc)
        if st:
            outputs[0] = y
        return st


class OpRegistry:
    """OpRegistry (reference src/core/ops/op_registry.h:15-30)."""

    def __init__(self):
        self._creators: Dict[str, Callable[[], Op]] = {}

    def register_op(self, op_type: str, creator: Callable[[], Op]) -> Status:
        if creator is None:
            return Status.error(Code.InvalidArgument, "empty op creator")
        if op_type in self._creators:
            return Status.error(Code.AlreadyExists, "op already registered")
        self._creators[op_type] = creator
        return OK

    def create(self, op_type: str):
        creator = self._creators.get(op_type)
        if creator is None:
            return None, Status.error(Code.NotFound, "no kernel for op")
        op = creator()
        if op is None:
            return None, Status.error(Code.Runtime, "op factory returned null")
        return op, OK

    def list_ops(self) -> List[str]:
        return sorted(self._creators)


def register_cuda_ops(registry: OpRegistry) -> Status:
    """Registers the CUDA convolution ops (the reference registers Conv2D and
    DepthwiseConv2D at op_registry.cpp:76-80).  Fails with AlreadyExists if an
    op type is taken, so call it before any builtin registration."""
    for name, cls in (("Conv2D", Conv2DOp), ("DepthwiseConv2D", DepthwiseConv2DOp),
                      ("QLinearConv2D", QLinearConv2DOp)):
        st = registry.register_op(name, cls)
        if not st:
            return st
    return OK
