// CUDA-core convolution kernels for the cases that are not dense contractions:
// depthwise (group == c) int8 in NHWC, and grouped / depthwise fp32 in NCHW.
// Depthwise work is ~9 MACs per output element, far below the tensor-core
// ridge point, so these kernels are written for HBM bandwidth: 128-bit
// channel-vector loads and stores, taps reused through L1/L2.
#pragma once

#include <cstdint>

#include "conv_igemm.cuh"

namespace ie_cuda {

struct DwArgs {
  int32_t n, h, w, c_store;  // input NHWC
  int32_t out_h, out_w;
  int32_t kh, kw, stride_h, stride_w, dil_h, dil_w, pad_t, pad_l;
  int32_t c;  // real channels (== m)
  int32_t x_signed, zp_x, zp_y;
  int32_t qmin, qmax;
};

// One thread = one output pixel x 16 channels.  Weights packed [kh*kw][c_store].
__global__ void __launch_bounds__(256) dwconv_q8_nhwc(const uint8_t* __restrict__ x,
                                                      const int8_t* __restrict__ wp,
                                                      const int32_t* __restrict__ bias,
                                                      const float* __restrict__ mult,
                                                      uint8_t* __restrict__ y, DwArgs a) {
  const int32_t groups = a.c_store >> 4;
  const int64_t total = static_cast<int64_t>(a.n) * a.out_h * a.out_w * groups;
  const int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (idx >= total) return;
  const int32_t g = static_cast<int32_t>(idx % groups);
  const int64_t pix = idx / groups;
  const int32_t ox = static_cast<int32_t>(pix % a.out_w);
  const int64_t t1 = pix / a.out_w;
  const int32_t oy = static_cast<int32_t>(t1 % a.out_h);
  const int32_t img = static_cast<int32_t>(t1 / a.out_h);
  const int32_t c0 = g * 16;
  int32_t acc[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) acc[j] = 0;
  const uint8_t* xi = x + static_cast<int64_t>(img) * a.h * a.w * a.c_store + c0;
  for (int ky = 0; ky < a.kh; ++ky) {
    const int32_t iy = oy * a.stride_h - a.pad_t + ky * a.dil_h;
    if (iy < 0 || iy >= a.h) continue;
    for (int kx = 0; kx < a.kw; ++kx) {
      const int32_t ix = ox * a.stride_w - a.pad_l + kx * a.dil_w;
      if (ix < 0 || ix >= a.w) continue;
      const uint4 xv = __ldg(reinterpret_cast<const uint4*>(
          xi + (static_cast<int64_t>(iy) * a.w + ix) * a.c_store));
      const uint4 wv = __ldg(reinterpret_cast<const uint4*>(
          wp + static_cast<int64_t>(ky * a.kw + kx) * a.c_store + c0));
      const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
      const uint32_t ws[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const uint32_t xb = (xs[q] >> (8 * b)) & 0xFFu;
          const int32_t xq = a.x_signed ? static_cast<int32_t>(static_cast<int8_t>(xb))
                                        : static_cast<int32_t>(xb);
          const int32_t wq = static_cast<int32_t>(static_cast<int8_t>((ws[q] >> (8 * b)) & 0xFFu));
          acc[4 * q + b] += (xq - a.zp_x) * wq;
        }
      }
    }
  }
  uint32_t out[4] = {0, 0, 0, 0};
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int32_t ch = c0 + j;
    int32_t q = 0;
    if (ch < a.c) {
      // same exact rule as the implicit-GEMM epilogue (conv_igemm.cuh)
      const int32_t t = static_cast<int32_t>(static_cast<uint32_t>(acc[j]) +
                                             static_cast<uint32_t>(bias != nullptr ? __ldg(bias + ch) : 0));
      q = requant_exact(t, split_multiplier(__ldg(mult + ch)), a.zp_y, a.qmin, a.qmax);
    }
    out[j >> 2] |= (static_cast<uint32_t>(q) & 0xFFu) << (8 * (j & 3));
  }
  *reinterpret_cast<uint4*>(y + pix * a.c_store + c0) = make_uint4(out[0], out[1], out[2], out[3]);
}

// depthwise int8 weights [c, 1, kh, kw] -> [kh*kw][c_store], zero filled.
__global__ void pack_dw_weights_q8(const int8_t* __restrict__ w, int8_t* __restrict__ out,
                                   int32_t c, int32_t taps, int32_t c_store) {
  const int64_t total = static_cast<int64_t>(taps) * c_store;
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= total) return;
  const int32_t ch = static_cast<int32_t>(i % c_store);
  const int32_t tap = static_cast<int32_t>(i / c_store);
  out[i] = ch < c ? w[static_cast<int64_t>(ch) * taps + tap] : static_cast<int8_t>(0);
}

struct DirectF32Args {
  int32_t n, c, h, w, m, cg, kh, kw;
  int32_t stride_h, stride_w, dil_h, dil_w, pad_t, pad_l;
  int32_t out_h, out_w, group;
  int32_t act;  // 0: none (NaN propagates), else clamp to [act_lo, act_hi]
  float act_lo, act_hi;
};

// Grouped / depthwise fp32 NCHW convolution, one thread per output element,
// accumulating in the reference's order: ascending (c_local, ky, kx)
// (conv2d_op.cpp:191-231), then the bias.
__global__ void __launch_bounds__(256) conv_direct_f32_nchw(const float* __restrict__ x,
                                                            const float* __restrict__ w,
                                                            const float* __restrict__ bias,
                                                            float* __restrict__ y,
                                                            DirectF32Args a) {
  const int64_t hw_out = static_cast<int64_t>(a.out_h) * a.out_w;
  const int64_t total = static_cast<int64_t>(a.n) * a.m * hw_out;
  const int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (idx >= total) return;
  const int32_t ox = static_cast<int32_t>(idx % a.out_w);
  const int32_t oy = static_cast<int32_t>((idx / a.out_w) % a.out_h);
  const int32_t mo = static_cast<int32_t>((idx / hw_out) % a.m);
  const int32_t img = static_cast<int32_t>(idx / (hw_out * a.m));
  const int32_t m_per_group = a.m / a.group;
  const int32_t grp = mo / m_per_group;
  const float* wrow = w + static_cast<int64_t>(mo) * a.cg * a.kh * a.kw;
  float acc = 0.0f;
  for (int cl = 0; cl < a.cg; ++cl) {
    const float* xc = x + (static_cast<int64_t>(img) * a.c + grp * a.cg + cl) * a.h * a.w;
    for (int ky = 0; ky < a.kh; ++ky) {
      const int32_t iy = oy * a.stride_h - a.pad_t + ky * a.dil_h;
      for (int kx = 0; kx < a.kw; ++kx) {
        const int32_t ix = ox * a.stride_w - a.pad_l + kx * a.dil_w;
        float v = 0.0f;
        if (iy >= 0 && iy < a.h && ix >= 0 && ix < a.w) v = __ldg(xc + iy * a.w + ix);
        acc = __fmaf_rn(__ldg(wrow + (cl * a.kh + ky) * a.kw + kx), v, acc);
      }
    }
  }
  if (bias != nullptr && __ldg(bias + mo) != 0.0f) acc += __ldg(bias + mo);
  if (a.act) acc = fminf(fmaxf(acc, a.act_lo), a.act_hi);
  y[idx] = acc;
}

}  // namespace ie_cuda
