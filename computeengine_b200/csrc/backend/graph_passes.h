// Graph passes for the CUDA backend behind the reference engine's compiler
// pass interface (src/core/ir/pass.h:14-25).
//
//   ConvBnReluFusionPass  folds a BatchNorm that follows a Conv2D /
//                         DepthwiseConv2D into the convolution's constant
//                         weights and bias, and (optionally) a following Relu
//                         or Clip(0, 6) into the convolution's "activation"
//                         attribute, which CudaConv2DOp runs in its epilogue.
//                         ResNet graphs from ONNX carry these as separate
//                         nodes; the reference runs each one as a full pass
//                         over the activation (batch_norm_op.cpp:78-95,
//                         relu_op.h).
//
// Folding uses the reference's own per-channel BatchNorm arithmetic
// (batch_norm_op.cpp:79-86): inv = fp32(1 / sqrt(double(var) + eps)),
// gain = scale * inv, shift = bias - mean * gain (fp32), then
// w'[m, ...] = w[m, ...] * gain[m] and b'[m] = b[m] * gain[m] + shift[m]
// (b = 0 without a conv bias), each operation rounded once.  The folded
// convolution differs from conv-then-BN only by that rounding.
//
//   With fuse_activation it also moves an Add that takes a dense Conv2D's
//   output and a residual (graph input, constant or earlier node's output)
//   into the convolution: the residual becomes its fourth input and
//   "fused_add" = 1, and CudaConv2DOp computes act((conv + b) + r) in its
//   epilogue (the ResNet bottleneck's shortcut add, fused before its Relu).
//
// The "activation" and "fused_add" attributes are this backend's extension:
// only CudaConv2DOp reads them, so run the pass with fuse_activation = true
// only on graphs executed with the CUDA registry (register_cuda_ops).
#pragma once

#include <string>

#include "ie_op_iface.h"

namespace ie_b200 {

class ConvBnReluFusionPass final : public ie::Pass {
 public:
  explicit ConvBnReluFusionPass(bool fuse_activation = true) : fuse_activation_(fuse_activation) {}
  std::string name() const override { return "conv_bn_relu_fusion"; }
  // Rewrites every Conv2D / DepthwiseConv2D -> BatchNorm [-> Add] [-> Relu | Clip(0,6)]
  // chain whose intermediate values have no other consumer and are not graph
  // outputs, and whose weights, bias and BatchNorm parameters are F32
  // constants in graph.weights.  Folded weights are added as new constants
  // ("<weight>.bn_folded"); the originals stay untouched.  Errors:
  // InvalidArgument for a BatchNorm with a non-positive var + epsilon, a
  // negative epsilon or parameters of the wrong length.
  ie::Status run(ie::Graph& graph, ie::PassContext& context) override;
  int folded_batch_norms() const { return folded_; }
  int fused_activations() const { return fused_; }
  int fused_adds() const { return fused_adds_; }

 private:
  bool fuse_activation_;
  int folded_ = 0;
  int fused_ = 0;
  int fused_adds_ = 0;
};

}  // namespace ie_b200
