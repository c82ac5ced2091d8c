// CUDA convolution ops behind the reference engine's Op / OpRegistry
// interface (src/core/ops/op.h:27-54, op_registry.h:15-30).
//
//   CudaConv2DOp(false)  replaces Conv2DOp            (conv2d_op.h:36-51); also
//                        reads "activation" ("Relu" / "Relu6") and
//                        "fused_add" (a residual as fourth input), the
//                        attributes ConvBnReluFusionPass sets when it fuses a
//                        following Add / Relu / Clip node into the epilogue
//   CudaConv2DOp(true)   replaces DepthwiseConv2DOp   (conv2d_op.h:53-67)
//   CudaQLinearConv2DOp  int8 convolution the reference plans but does not
//                        implement (src/converter/quantization/quant_plugins.h:7-22)
//
// configure() parses the same attributes with the same error codes as the
// reference's parse_conv_config (conv2d_op.cpp:26-71).  forward() takes the
// reference's host NCHW tensors, runs the convolution on the current CUDA
// device through the C ABI (include/ie_cuda_conv.h), allocates outputs[0]
// with Tensor::allocate on context.allocator (conv2d_op.cpp:167) and returns
// only after the result is in host memory.  There is no CPU fallback: without
// a CUDA device forward() returns Error::Code::Runtime.
#pragma once

#include <array>
#include <cstdint>
#include <functional>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "ie_cuda_conv.h"
#include "ie_op_iface.h"

namespace ie_b200 {

enum class AutoPad { NotSet, Valid, SameUpper, SameLower };

// Fields and defaults of the reference ConvConfig (conv2d_op.h:13-21).
struct ConvConfig {
  std::array<int64_t, 2> strides{1, 1};
  std::array<int64_t, 2> dilations{1, 1};
  std::array<int64_t, 4> pads{0, 0, 0, 0};  // top, left, bottom, right
  int64_t group{1};
  AutoPad auto_pad{AutoPad::NotSet};
  bool has_kernel_shape{false};
  std::array<int64_t, 2> kernel_shape{0, 0};
};

// The reference's parse_conv_config with the attrs_util.h readers
// (read_pair :165-184, read_pads :134-158, read_int, read_auto_pad :109-132,
// read_int_list): "strides", "dilations", "pads" (2 or 4 values), "group",
// "auto_pad", "kernel_shape".
ie::Status parse_conv_config(const ie::Attrs& attrs, ConvConfig& config);

// C ABI status (1 + ie::Error::Code, 0 = OK) -> ie::Status with the library's
// last error message.
ie::Status to_status(int rc);

// Device allocation every DeviceBuffers goes through: a cudaMalloc-shaped
// function returning a cudaError_t value (cudaMalloc by default).  Tests swap
// in a failing one to check that forward() reports OutOfMemory (the reference
// convention for a failed allocation, error.h:14) and leaves the op usable;
// pass nullptr to restore cudaMalloc.  Not thread-safe against concurrent
// forward() calls: set it while no op runs.
using DeviceAllocFn = int (*)(void** ptr, size_t bytes);
void set_device_alloc(DeviceAllocFn fn);

// Device memory owned by one op: weights uploaded (and packed) once per host
// buffer, scratch buffers that only grow.  Host weight inputs are keyed by
// their buffer and size: they must be constants that outlive the op and keep
// their contents (graph weights are).  The convolutions read device-resident
// weights afresh on every call (packing them into scratch), since a device
// value's address is reused with new contents by the executor's pool.
class DeviceBuffers {
 public:
  DeviceBuffers() = default;
  DeviceBuffers(const DeviceBuffers&) = delete;
  DeviceBuffers& operator=(const DeviceBuffers&) = delete;
  ~DeviceBuffers();
  // Scratch slot `slot` with at least `bytes` bytes (256-byte aligned).
  ie::Result<void*> scratch(int slot, size_t bytes);
  // Cached device copy for a host buffer; `fresh` tells whether it was just
  // allocated (and must be filled by the caller).
  ie::Result<void*> cached(const void* host_key, size_t bytes, int kind, bool* fresh);

 private:
  struct Block {
    void* ptr = nullptr;
    size_t bytes = 0;
  };
  std::unordered_map<int, Block> scratch_;
  struct Key {
    const void* host;
    size_t bytes;
    int kind;
    bool operator==(const Key& o) const {
      return host == o.host && bytes == o.bytes && kind == o.kind;
    }
  };
  struct KeyHash {
    size_t operator()(const Key& k) const {
      return std::hash<const void*>()(k.host) ^ (k.bytes * 1315423911u) ^ static_cast<size_t>(k.kind);
    }
  };
  std::unordered_map<Key, Block, KeyHash> cache_;
};

class CudaConv2DOp final : public ie::Op {
 public:
  explicit CudaConv2DOp(bool depthwise = false) : depthwise_(depthwise) {}
  ie::Status configure(const ie::Attrs& attrs) override;
  ie::Status forward(const std::vector<ie::Tensor*>& inputs, std::vector<ie::Tensor*>& outputs,
                     ie::ExecutionContext& context) override;
  const ConvConfig& config() const { return config_; }

 private:
  ConvConfig config_{};
  bool depthwise_;
  int32_t act_ = IE_ACT_NONE;  // fused activation ("activation" attribute)
  bool fused_add_ = false;     // fourth input added in the epilogue ("fused_add")
  DeviceBuffers dev_;
};

// int8 Conv2D (dense or depthwise).  Inputs [x, w]: x U8 or I8 NCHW, w I8
// [M, C/group, kH, kW].  Attributes: the Conv2D ones plus "multiplier"
// (per-channel s_x * s_w[m] / s_y, rounded to fp32), "bias" (int32 values as
// an int list; the reference has no I32 dtype), "x_zero_point",
// "y_zero_point", "y_signed" and the output clamp "qmin" / "qmax" (ReLU /
// ReLU6 folded in).  Output U8 or I8 NCHW, bit-exact with the int8 oracle:
// y = clamp(round_half_away((acc + bias) * multiplier) + y_zero_point).
//
// Device mode (ExecutionContext::device == CUDA, as CudaExecutor runs it):
// x is a device tensor, NCHW or this backend's int8 activation layout, and
// the output is returned in that layout without synchronizing.  The layout:
// Tensor::layout == Layout::NHWC, shape the logical [N, C, H, W], buffer
// [N, H, W, round_up(C, 16)] bytes (the padding channels hold no data) --
// what the implicit-GEMM kernel reads and writes, so a chain of int8 nodes
// runs without a layout pass between them.
class CudaQLinearConv2DOp final : public ie::Op {
 public:
  ie::Status configure(const ie::Attrs& attrs) override;
  ie::Status forward(const std::vector<ie::Tensor*>& inputs, std::vector<ie::Tensor*>& outputs,
                     ie::ExecutionContext& context) override;

 private:
  ConvConfig config_{};
  std::vector<float> mult_;
  std::vector<int32_t> bias_;
  int64_t zp_x_ = 0, zp_y_ = 0;
  bool y_signed_ = false;
  bool has_qmin_ = false, has_qmax_ = false;
  int64_t qmin_ = 0, qmax_ = 0;
  DeviceBuffers dev_;
};

// int8 Add of two quantized tensors (the shortcut Add of a quantized ResNet
// block), on OpType::Add nodes that carry the int8 attributes:
// "a_zero_point", "b_zero_point", "a_multiplier" (s_a / s_y), "b_multiplier"
// (s_b / s_y), "y_zero_point", "y_signed", "qmin" / "qmax" (a following ReLU
// folds into qmin).  y = clamp(round_half_away((a - zp_a) * m_a +
// (b - zp_b) * m_b) + zp_y), exact (ie_cuda_qadd).  Inputs of one logical
// shape, NCHW or the int8 activation layout (device mode); the output takes
// the activation layout when either input has it.  An Add node without the
// int8 attributes is an fp32 Add, which this backend runs only fused into a
// convolution (ConvBnReluFusionPass): configure() returns Unsupported.
class CudaQLinearAddOp final : public ie::Op {
 public:
  ie::Status configure(const ie::Attrs& attrs) override;
  ie::Status forward(const std::vector<ie::Tensor*>& inputs, std::vector<ie::Tensor*>& outputs,
                     ie::ExecutionContext& context) override;

 private:
  ie_qadd_params q_{};
  bool has_qmin_ = false, has_qmax_ = false;
  int64_t qmin_ = 0, qmax_ = 0;
  DeviceBuffers dev_;
};

// Conv2D / DepthwiseConv2D node of the CUDA backend: a quantized node (one
// with a "multiplier" attribute, as the int8 converter emits) runs as
// CudaQLinearConv2DOp, any other as CudaConv2DOp.  The reference IR has one
// Conv2D op type for both.
class CudaConvNodeOp final : public ie::Op {
 public:
  explicit CudaConvNodeOp(bool depthwise) : depthwise_(depthwise) {}
  ie::Status configure(const ie::Attrs& attrs) override;
  ie::Status forward(const std::vector<ie::Tensor*>& inputs, std::vector<ie::Tensor*>& outputs,
                     ie::ExecutionContext& context) override;

 private:
  bool depthwise_;
  std::unique_ptr<ie::Op> impl_;
};

// Fields and defaults of the reference PoolConfig (pool_ops.h:13-21).
struct PoolConfig {
  bool has_kernel_shape{false};
  std::array<int64_t, 2> kernel_shape{0, 0};
  std::array<int64_t, 2> strides{1, 1};
  std::array<int64_t, 4> pads{0, 0, 0, 0};
  AutoPad auto_pad{AutoPad::NotSet};
  bool ceil_mode{false};
  bool count_include_pad{false};
};

// The reference's parse_pool_config (pool_ops.cpp:66-109): "kernel_shape"
// (required, two positive values), "strides", "pads", "auto_pad",
// "ceil_mode", "count_include_pad".
ie::Status parse_pool_config(const ie::Attrs& attrs, PoolConfig& config);

// CudaPool2DOp(true)  replaces MaxPool2DOp (pool_ops.h:37-51)
// CudaPool2DOp(false) replaces AvgPool2DOp (pool_ops.h:54-68)
// NCHW F32 host (or device) tensor in, host NCHW F32 out; bit-exact with the
// reference (same window order and arithmetic).  MaxPool2D also takes a U8 /
// I8 activation of a quantized graph (NCHW, or the int8 activation layout in
// device mode; ie_cuda_q8_maxpool2d_nhwc): the output keeps the input's
// dtype, scale and zero point and equals the reference pool run on the same
// integers as floats.  Average pooling of int8 is Unsupported.
class CudaPool2DOp final : public ie::Op {
 public:
  explicit CudaPool2DOp(bool max_pool) : max_pool_(max_pool) {}
  ie::Status configure(const ie::Attrs& attrs) override;
  ie::Status forward(const std::vector<ie::Tensor*>& inputs, std::vector<ie::Tensor*>& outputs,
                     ie::ExecutionContext& context) override;

 private:
  ie_pool2d_desc pool_desc(const ie::Tensor& x) const;
  ie::Status forward_q8(const ie::Tensor& x, std::vector<ie::Tensor*>& outputs,
                        ie::ExecutionContext& context);

  PoolConfig config_{};
  bool max_pool_;
  DeviceBuffers dev_;
};

// Replaces GlobalAvgPoolOp (pool_ops.h:71-79): [N, C, H, W] -> [N, C, 1, 1].
// An int8 input (U8 / I8: NCHW, or the int8 activation layout in device mode)
// is the head of a quantized graph: the node carries "x_scale" and
// "x_zero_point" (0 when absent) and the output is the fp32 mean of the
// dequantized values, fp32((sum q - zp * h * w) * x_scale / (h * w))
// (ie_cuda_q8_global_avg_pool_nhwc), ready for the fp32 Gemm after it.
class CudaGlobalAvgPoolOp final : public ie::Op {
 public:
  ie::Status configure(const ie::Attrs& attrs) override;
  ie::Status forward(const std::vector<ie::Tensor*>& inputs, std::vector<ie::Tensor*>& outputs,
                     ie::ExecutionContext& context) override;

 private:
  ie::Status forward_q8(const ie::Tensor& x, std::vector<ie::Tensor*>& outputs,
                        ie::ExecutionContext& context);

  bool has_scale_ = false;
  double x_scale_ = 0.0;
  int64_t x_zero_point_ = 0;
  DeviceBuffers dev_;
};

// Replaces GemmOp (gemm_op.h:14-31): Y = alpha * A' * B' + beta * C with the
// reference's attributes ("alpha", "beta", "transA", "transB") and C
// broadcasts (scalar, [N], [M], [M,1], [1,N], [M,N]).  B and C stay on the
// device keyed by their host buffers (the model's weights); the product runs
// as bf16x3 on the tensor cores.
class CudaGemmOp final : public ie::Op {
 public:
  ie::Status configure(const ie::Attrs& attrs) override;
  ie::Status forward(const std::vector<ie::Tensor*>& inputs, std::vector<ie::Tensor*>& outputs,
                     ie::ExecutionContext& context) override;

 private:
  double alpha_{1.0}, beta_{1.0};
  int64_t trans_a_{0}, trans_b_{0};
  DeviceBuffers dev_;
};

// Registers CudaConv2DOp for OpType::Conv2D and OpType::DepthwiseConv2D, and
// the pooling and Gemm ops for MaxPool2D, AvgPool2D, GlobalAvgPool and Gemm.  Like
// the reference registry it fails with AlreadyExists when a type is taken, so
// call it on a fresh (backend-private) registry or before
// register_builtin_ops, which skips types already present
// (op_registry.cpp:62-66).
ie::Status register_cuda_ops(ie::OpRegistry& registry);

// The CUDA backend's own op table, with the reference OpRegistry's
// register_op / create semantics (op_registry.cpp:23-50: AlreadyExists for a
// taken type, NotFound for an unknown one).  Inside the reference engine the
// OpRegistry is a process singleton whose constructor is private and which
// the CPU executor also reads (executor.h:21-24); the CUDA backend keeps its
// ops in a table of its own so that registering them leaves what the CPU
// backend runs unchanged.
class CudaOpTable {
 public:
  using Creator = std::function<std::unique_ptr<ie::Op>()>;
  ie::Status register_op(ie::OpType op, Creator creator);
  ie::Result<std::unique_ptr<ie::Op>> create(ie::OpType op);
  std::vector<ie::OpType> list() const;

 private:
  mutable std::mutex mutex_;
  std::unordered_map<ie::OpType, Creator> creators_;
};

ie::Status register_cuda_ops(CudaOpTable& table);

}  // namespace ie_b200
