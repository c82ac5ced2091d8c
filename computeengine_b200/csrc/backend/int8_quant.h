// int8 post-training quantization for the CUDA convolution ops, behind the
// reference engine's quantization plugin contract
// (src/core/plugin/quant_plugin.h:11-28).
//
//   Int8QuantPlugin      replaces the reference's Int8QuantPlugin stub
//                        (src/converter/quantization/quant_plugins.h:7-22),
//                        which returns Unsupported for both calls
//   ActivationCalibrator min/max (or percentile) range of an activation over
//                        calibration batches, the strategy the reference plans
//                        for its INT8 PTQ (docs/superpowers/specs/m4-hybrid/
//                        p9-p14-hybrid-orchestration.md:133,148)
//   make_qlinear_conv_attrs
//                        the attributes CudaQLinearConv2DOp consumes
//                        (multiplier, int32 bias, zero points, clamp) from the
//                        input, weight and output quantization of one layer
//
// Quantization rules (one place, used by every function here):
//   weights      symmetric int8, one scale per output channel (axis 0):
//                scale = max|w| / 127, q = clamp(rne(w / scale), -127, 127)
//   activations  asymmetric uint8, one scale per tensor over [min(lo, 0),
//                max(hi, 0)] so that 0.0 is exact: scale = (hi - lo) / 255,
//                zp = clamp(rne(-lo / scale), 0, 255),
//                q = clamp(rne(x / scale) + zp, 0, 255)
//   dequantize   x = (q - zp) * scale
//   requantize   multiplier[m] = fp32(s_x * s_w[m] / s_y)  (computed in double)
//                bias_q[m] = rne(b[m] / (s_x * s_w[m])), saturated to int32
// rne = round half to even; divisions in double.  A channel (or tensor) that
// is all zero gets scale 1.
#pragma once

#include <cstdint>
#include <memory>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "ie_op_iface.h"

namespace ie_b200 {

struct QuantParams {
  ie::DType dtype{ie::DType::I8};  // I8 (symmetric) or U8 (asymmetric)
  bool per_channel{false};         // scales along axis 0
  std::vector<float> scales;       // one per channel, or one
  int32_t zero_point{0};           // U8 only
};

// Parameters of an fp32 tensor under the rules above.
//   symmetric + per_channel: int8 weights, one scale per dims[0] slice
//   symmetric, per tensor:   int8, one scale
//   asymmetric:              uint8 over the tensor's own [min, max]
ie::Result<QuantParams> choose_params(const ie::Tensor& tensor, bool symmetric, bool per_channel);

// Asymmetric uint8 parameters for an observed range [lo, hi].
QuantParams u8_params_for_range(float lo, float hi);

class Int8QuantPlugin final : public ie::QuantPlugin {
 public:
  explicit Int8QuantPlugin(std::shared_ptr<ie::Allocator> allocator = nullptr);

  ie::PluginMeta meta() const override;

  // fp32 host tensor -> I8 (config.symmetric) or U8 tensor of the same shape.
  // config.bits must be 8; config.format "" or "int8" (per-channel weights
  // when symmetric, per-tensor activations otherwise) or "int8_per_tensor".
  // Errors: Unsupported for other bits / formats, non-F32 or device tensors;
  // InvalidArgument for an empty tensor, a null buffer or a non-finite value.
  // The parameters used are kept with the result (params()).
  ie::Result<ie::Tensor> quantize(const ie::Tensor& tensor, const ie::QuantConfig& config) override;

  // I8 / U8 tensor this plugin produced -> fp32 with its parameters;
  // NotFound for a tensor it did not produce.
  ie::Result<ie::Tensor> dequantize(const ie::Tensor& tensor, const ie::QuantConfig& config) override;

  // With explicit parameters (a calibrated activation range, parameters
  // stored beside a model).
  ie::Result<ie::Tensor> quantize_with(const ie::Tensor& tensor, const QuantParams& params);
  ie::Result<ie::Tensor> dequantize_with(const ie::Tensor& tensor, const QuantParams& params);

  // Parameters of a tensor returned by quantize / quantize_with (keyed by its
  // buffer), or nullptr.
  const QuantParams* params(const ie::Tensor& quantized) const;

 private:
  std::shared_ptr<ie::Allocator> allocator_;
  mutable std::mutex mutex_;
  std::unordered_map<const void*, QuantParams> params_;
};

// Range of one activation over calibration batches.  percentile = 100 keeps
// the running min / max; below 100 the observed values are kept (every
// value of each observed tensor up to 1 << 22 per call, evenly strided
// beyond that) and the range is their (100 - p)-th / p-th percentile.
class ActivationCalibrator {
 public:
  explicit ActivationCalibrator(double percentile = 100.0) : percentile_(percentile) {}
  ie::Status observe(const ie::Tensor& tensor);
  ie::Status observe(const float* values, size_t count);
  bool empty() const { return count_ == 0; }
  // asymmetric uint8 parameters of the observed range (InvalidArgument if
  // nothing was observed)
  ie::Result<QuantParams> params() const;
  float lo() const { return lo_; }
  float hi() const { return hi_; }

 private:
  double percentile_;
  size_t count_ = 0;
  float lo_ = 0.0f, hi_ = 0.0f;
  std::vector<float> samples_;
};

enum class FusedActivation { None, Relu, Relu6 };

// The attributes of CudaQLinearConv2DOp for one layer: conv_attrs (strides,
// pads, group, ...) plus "multiplier", "bias", "x_zero_point",
// "y_zero_point", "qmin" and "qmax" (ReLU / ReLU6 folded into the clamp).
// x and y: asymmetric uint8 per tensor; w: symmetric int8, per channel with
// M scales or per tensor; bias_f32 may be null (M values otherwise).
ie::Result<ie::Attrs> make_qlinear_conv_attrs(const ie::Attrs& conv_attrs, const QuantParams& x,
                                              const QuantParams& w, const QuantParams& y,
                                              int64_t m, const float* bias_f32,
                                              FusedActivation act);

}  // namespace ie_b200
