// int8 post-training quantization (see int8_quant.h for the rules).
#include "int8_quant.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <string>

#ifdef IE_B200_REFERENCE_HEADERS
#include "core/memory/malloc_allocator.h"
#endif

namespace ie_b200 {
namespace {

// round half to even of a double (the default floating-point rounding mode)
inline double rne(double v) { return std::nearbyint(v); }

template <class T>
inline T clamp_to(double v, double lo, double hi) {
  return static_cast<T>(v < lo ? lo : (v > hi ? hi : v));
}

ie::Status check_f32_host(const ie::Tensor& t) {
  if (t.dtype != ie::DType::F32) return ie::Error::unsupported("quantize expects an F32 tensor");
  if (t.device != ie::Device::CPU) return ie::Error::unsupported("quantize runs on host tensors");
  if (t.numel() <= 0 || !t.shape.is_concrete()) {
    return ie::Error::invalid_argument("quantize needs a non-empty tensor");
  }
  if (t.buffer == nullptr) return ie::Error::invalid_argument("tensor has no buffer");
  return {};
}

// elements per axis-0 slice and the slice count of a per-channel layout
void channel_geometry(const ie::Tensor& t, bool per_channel, int64_t* channels, int64_t* inner) {
  const int64_t n = t.numel();
  if (per_channel && !t.shape.dims.empty() && t.shape.dims[0] > 0) {
    *channels = t.shape.dims[0];
    *inner = n / *channels;
  } else {
    *channels = 1;
    *inner = n;
  }
}

ie::Status check_params(const QuantParams& p, const ie::Tensor& t) {
  if (p.dtype != ie::DType::I8 && p.dtype != ie::DType::U8) {
    return ie::Error::invalid_argument("quantization parameters must be I8 or U8");
  }
  int64_t channels = 0, inner = 0;
  channel_geometry(t, p.per_channel, &channels, &inner);
  if (static_cast<int64_t>(p.scales.size()) != channels) {
    return ie::Error::invalid_argument("quantization parameters: wrong number of scales");
  }
  for (float s : p.scales) {
    if (!(s > 0.0f) || !std::isfinite(s)) {
      return ie::Error::invalid_argument("quantization scales must be positive and finite");
    }
  }
  if (p.dtype == ie::DType::I8 && p.zero_point != 0) {
    return ie::Error::invalid_argument("int8 quantization is symmetric (zero point 0)");
  }
  if (p.dtype == ie::DType::U8 && (p.zero_point < 0 || p.zero_point > 255)) {
    return ie::Error::invalid_argument("uint8 zero point must lie in [0, 255]");
  }
  return {};
}

}  // namespace

QuantParams u8_params_for_range(float lo, float hi) {
  QuantParams p;
  p.dtype = ie::DType::U8;
  p.per_channel = false;
  const double l = std::min<double>(lo, 0.0), h = std::max<double>(hi, 0.0);
  float scale = static_cast<float>((h - l) / 255.0);
  if (!(scale > 0.0f) || !std::isfinite(scale)) scale = 1.0f;
  p.scales = {scale};
  p.zero_point = clamp_to<int32_t>(rne(-l / static_cast<double>(scale)), 0.0, 255.0);
  return p;
}

ie::Result<QuantParams> choose_params(const ie::Tensor& tensor, bool symmetric, bool per_channel) {
  if (auto st = check_f32_host(tensor); !st.has_value()) return st.error();
  const float* x = tensor.data<float>();
  const int64_t n = tensor.numel();
  for (int64_t i = 0; i < n; ++i) {
    if (!std::isfinite(x[i])) return ie::Error::invalid_argument("tensor holds a non-finite value");
  }
  if (!symmetric) {
    float lo = x[0], hi = x[0];
    for (int64_t i = 1; i < n; ++i) {
      lo = std::min(lo, x[i]);
      hi = std::max(hi, x[i]);
    }
    return u8_params_for_range(lo, hi);
  }
  QuantParams p;
  p.dtype = ie::DType::I8;
  p.per_channel = per_channel;
  int64_t channels = 0, inner = 0;
  channel_geometry(tensor, per_channel, &channels, &inner);
  p.scales.resize(static_cast<size_t>(channels));
  for (int64_t c = 0; c < channels; ++c) {
    float amax = 0.0f;
    for (int64_t i = 0; i < inner; ++i) amax = std::max(amax, std::fabs(x[c * inner + i]));
    float scale = static_cast<float>(static_cast<double>(amax) / 127.0);
    if (!(scale > 0.0f)) scale = 1.0f;
    p.scales[static_cast<size_t>(c)] = scale;
  }
  return p;
}

Int8QuantPlugin::Int8QuantPlugin(std::shared_ptr<ie::Allocator> allocator)
    : allocator_(allocator ? std::move(allocator) : std::make_shared<ie::MallocAllocator>()) {}

ie::PluginMeta Int8QuantPlugin::meta() const {
  return {"int8_quant", "1.0.0", "0.1", {"quantization"},
          "int8 PTQ: per-channel symmetric weights, min/max calibrated uint8 activations"};
}

ie::Result<ie::Tensor> Int8QuantPlugin::quantize(const ie::Tensor& tensor,
                                                 const ie::QuantConfig& config) {
  if (config.bits != 8) return ie::Error::unsupported("int8_quant supports 8 bits only");
  bool per_channel = config.symmetric;
  if (config.format == "int8_per_tensor") {
    per_channel = false;
  } else if (!config.format.empty() && config.format != "int8") {
    return ie::Error::unsupported("int8_quant: unknown format '" + config.format + "'");
  }
  auto p = choose_params(tensor, config.symmetric, per_channel);
  if (!p.has_value()) return p.error();
  return quantize_with(tensor, *p);
}

ie::Result<ie::Tensor> Int8QuantPlugin::quantize_with(const ie::Tensor& tensor,
                                                      const QuantParams& params) {
  if (auto st = check_f32_host(tensor); !st.has_value()) return st.error();
  if (auto st = check_params(params, tensor); !st.has_value()) return st.error();
  auto out = ie::Tensor::allocate(tensor.shape, params.dtype, allocator_);
  if (!out.has_value()) return out.error();
  const float* x = tensor.data<float>();
  int64_t channels = 0, inner = 0;
  channel_geometry(tensor, params.per_channel, &channels, &inner);
  for (int64_t c = 0; c < channels; ++c) {
    const double scale = params.scales[static_cast<size_t>(c)];
    const float* xc = x + c * inner;
    if (params.dtype == ie::DType::I8) {
      int8_t* q = out->data<int8_t>() + c * inner;
      for (int64_t i = 0; i < inner; ++i) {
        if (!std::isfinite(xc[i])) return ie::Error::invalid_argument("tensor holds a non-finite value");
        q[i] = clamp_to<int8_t>(rne(xc[i] / scale), -127.0, 127.0);
      }
    } else {
      uint8_t* q = out->data<uint8_t>() + c * inner;
      const double zp = params.zero_point;
      for (int64_t i = 0; i < inner; ++i) {
        if (!std::isfinite(xc[i])) return ie::Error::invalid_argument("tensor holds a non-finite value");
        q[i] = clamp_to<uint8_t>(rne(xc[i] / scale) + zp, 0.0, 255.0);
      }
    }
  }
  {
    std::lock_guard<std::mutex> lock(mutex_);
    params_[out->buffer] = params;
  }
  return out;
}

ie::Result<ie::Tensor> Int8QuantPlugin::dequantize(const ie::Tensor& tensor,
                                                   const ie::QuantConfig& config) {
  if (config.bits != 8) return ie::Error::unsupported("int8_quant supports 8 bits only");
  QuantParams p;
  {
    std::lock_guard<std::mutex> lock(mutex_);
    auto it = params_.find(tensor.buffer);
    if (it == params_.end()) {
      return ie::Error::not_found("tensor was not quantized by this plugin");
    }
    p = it->second;
  }
  return dequantize_with(tensor, p);
}

ie::Result<ie::Tensor> Int8QuantPlugin::dequantize_with(const ie::Tensor& tensor,
                                                        const QuantParams& params) {
  if (tensor.dtype != params.dtype) {
    return ie::Error::unsupported("dequantize: tensor dtype differs from its parameters");
  }
  if (tensor.device != ie::Device::CPU) return ie::Error::unsupported("dequantize runs on host tensors");
  if (tensor.numel() <= 0 || tensor.buffer == nullptr) {
    return ie::Error::invalid_argument("dequantize needs a non-empty tensor");
  }
  if (auto st = check_params(params, tensor); !st.has_value()) return st.error();
  auto out = ie::Tensor::allocate(tensor.shape, ie::DType::F32, allocator_);
  if (!out.has_value()) return out.error();
  int64_t channels = 0, inner = 0;
  channel_geometry(tensor, params.per_channel, &channels, &inner);
  float* y = out->data<float>();
  for (int64_t c = 0; c < channels; ++c) {
    const float scale = params.scales[static_cast<size_t>(c)];
    for (int64_t i = 0; i < inner; ++i) {
      const int32_t q = params.dtype == ie::DType::I8
                            ? tensor.data<int8_t>()[c * inner + i]
                            : static_cast<int32_t>(tensor.data<uint8_t>()[c * inner + i]);
      y[c * inner + i] = static_cast<float>(q - params.zero_point) * scale;
    }
  }
  return out;
}

const QuantParams* Int8QuantPlugin::params(const ie::Tensor& quantized) const {
  std::lock_guard<std::mutex> lock(mutex_);
  auto it = params_.find(quantized.buffer);
  return it == params_.end() ? nullptr : &it->second;
}

// ------------------------------------------------------------ calibration

ie::Status ActivationCalibrator::observe(const ie::Tensor& tensor) {
  if (auto st = check_f32_host(tensor); !st.has_value()) return st;
  return observe(tensor.data<float>(), static_cast<size_t>(tensor.numel()));
}

ie::Status ActivationCalibrator::observe(const float* values, size_t count) {
  if (!(percentile_ > 50.0 && percentile_ <= 100.0)) {
    return ie::Error::invalid_argument("calibration percentile must lie in (50, 100]");
  }
  if (values == nullptr || count == 0) return ie::Error::invalid_argument("nothing to observe");
  for (size_t i = 0; i < count; ++i) {
    if (!std::isfinite(values[i])) return ie::Error::invalid_argument("non-finite activation");
  }
  float lo = values[0], hi = values[0];
  for (size_t i = 1; i < count; ++i) {
    lo = std::min(lo, values[i]);
    hi = std::max(hi, values[i]);
  }
  if (count_ == 0) {
    lo_ = lo;
    hi_ = hi;
  } else {
    lo_ = std::min(lo_, lo);
    hi_ = std::max(hi_, hi);
  }
  count_ += count;
  if (percentile_ < 100.0) {
    constexpr size_t kMaxPerCall = size_t{1} << 22;
    const size_t stride = count > kMaxPerCall ? (count + kMaxPerCall - 1) / kMaxPerCall : 1;
    for (size_t i = 0; i < count; i += stride) samples_.push_back(values[i]);
  }
  return {};
}

ie::Result<QuantParams> ActivationCalibrator::params() const {
  if (count_ == 0) return ie::Error::invalid_argument("calibrator has observed nothing");
  if (percentile_ >= 100.0 || samples_.empty()) return u8_params_for_range(lo_, hi_);
  std::vector<float> v(samples_);
  const auto at = [&](double pct) {
    const size_t k = static_cast<size_t>(
        std::llround(pct / 100.0 * static_cast<double>(v.size() - 1)));
    std::nth_element(v.begin(), v.begin() + static_cast<std::ptrdiff_t>(k), v.end());
    return v[k];
  };
  const float hi = at(percentile_);
  const float lo = at(100.0 - percentile_);
  return u8_params_for_range(lo, hi);
}

// ------------------------------------------------------ requantize attrs

ie::Result<ie::Attrs> make_qlinear_conv_attrs(const ie::Attrs& conv_attrs, const QuantParams& x,
                                              const QuantParams& w, const QuantParams& y,
                                              int64_t m, const float* bias_f32,
                                              FusedActivation act) {
  if (m <= 0) return ie::Error::invalid_argument("output channel count must be positive");
  for (const QuantParams* p : {&x, &y}) {
    if (p->dtype != ie::DType::U8 || p->per_channel || p->scales.size() != 1 ||
        !(p->scales[0] > 0.0f) || p->zero_point < 0 || p->zero_point > 255) {
      return ie::Error::invalid_argument("activations must be per-tensor uint8");
    }
  }
  if (w.dtype != ie::DType::I8 || w.zero_point != 0 ||
      (w.per_channel ? static_cast<int64_t>(w.scales.size()) != m : w.scales.size() != 1)) {
    return ie::Error::invalid_argument("weights must be symmetric int8 with M or 1 scales");
  }
  const double s_x = x.scales[0], s_y = y.scales[0];
  std::vector<double> mult(static_cast<size_t>(m));
  std::vector<int64_t> bias(static_cast<size_t>(m), 0);
  for (int64_t c = 0; c < m; ++c) {
    const double s_w = w.scales[w.per_channel ? static_cast<size_t>(c) : 0];
    if (!(s_w > 0.0)) return ie::Error::invalid_argument("weight scales must be positive");
    mult[static_cast<size_t>(c)] = static_cast<double>(static_cast<float>(s_x * s_w / s_y));
    if (bias_f32 != nullptr) {
      if (!std::isfinite(bias_f32[c])) return ie::Error::invalid_argument("non-finite bias");
      bias[static_cast<size_t>(c)] = clamp_to<int64_t>(
          rne(static_cast<double>(bias_f32[c]) / (s_x * s_w)),
          static_cast<double>(std::numeric_limits<int32_t>::min()),
          static_cast<double>(std::numeric_limits<int32_t>::max()));
    }
  }
  int64_t qmin = 0, qmax = 255;
  if (act == FusedActivation::Relu || act == FusedActivation::Relu6) qmin = y.zero_point;
  if (act == FusedActivation::Relu6) {
    qmax = std::min<int64_t>(255, y.zero_point + static_cast<int64_t>(rne(6.0 / s_y)));
  }
  ie::Attrs out = conv_attrs;
  out["multiplier"] = mult;
  out["bias"] = bias;
  out["x_zero_point"] = static_cast<int64_t>(x.zero_point);
  out["y_zero_point"] = static_cast<int64_t>(y.zero_point);
  out["qmin"] = qmin;
  out["qmax"] = qmax;
  return out;
}

}  // namespace ie_b200
