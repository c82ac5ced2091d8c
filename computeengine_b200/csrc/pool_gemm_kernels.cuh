// Head-of-network fp32 ops on CUDA cores: 2D max / average pooling and
// global average pooling over NCHW, and the Gemm epilogue (alpha, beta, C
// broadcast) around a bf16x3 tensor-core product.  All HBM- or
// latency-bound; the pooling kernels follow the reference's arithmetic order
// so their results equal it bit for bit.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace ie_cuda {

struct Pool2dArgs {
  int64_t planes;  // n * c
  int32_t h, w, out_h, out_w;
  int32_t kh, kw, stride_h, stride_w;
  int32_t pad_t, pad_l, pad_b, pad_r;
  int32_t max_pool;           // 1 max, 0 average
  int32_t count_include_pad;  // average: divide by the window's padded extent
};

// One thread per output element.  The window is walked ky-major, kx
// ascending, like the reference (pool_ops.cpp:170-207): max keeps the first
// of equal values and ignores padding (the accumulator starts at -inf);
// average sums the in-image values in that order and divides by the count of
// in-image positions, or with count_include_pad of positions inside the
// padded extent, 0 for an empty window.
__global__ void pool2d_f32_nchw(const float* __restrict__ x, float* __restrict__ y,
                                const Pool2dArgs a) {
  const int64_t per_plane = static_cast<int64_t>(a.out_h) * a.out_w;
  const int64_t total = a.planes * per_plane;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t plane = idx / per_plane;
    const int32_t rem = static_cast<int32_t>(idx - plane * per_plane);
    const int32_t oy = rem / a.out_w, ox = rem - (rem / a.out_w) * a.out_w;
    const float* in = x + plane * a.h * static_cast<int64_t>(a.w);
    float acc = a.max_pool ? -INFINITY : 0.0f;
    int32_t count = 0;
    for (int32_t ky = 0; ky < a.kh; ++ky) {
      const int32_t iy = oy * a.stride_h - a.pad_t + ky;
      for (int32_t kx = 0; kx < a.kw; ++kx) {
        const int32_t ix = ox * a.stride_w - a.pad_l + kx;
        if (iy >= 0 && iy < a.h && ix >= 0 && ix < a.w) {
          const float v = in[static_cast<int64_t>(iy) * a.w + ix];
          if (a.max_pool) {
            acc = v > acc ? v : acc;
          } else {
            acc = __fadd_rn(acc, v);
            if (!a.count_include_pad) ++count;
          }
        }
        if (!a.max_pool && a.count_include_pad && iy >= -a.pad_t && iy < a.h + a.pad_b &&
            ix >= -a.pad_l && ix < a.w + a.pad_r) {
          ++count;
        }
      }
    }
    if (!a.max_pool) acc = count > 0 ? __fdiv_rn(acc, static_cast<float>(count)) : 0.0f;
    y[idx] = acc;
  }
}

// Global average pooling [planes, spatial] -> [planes]: one thread per plane
// sums in index order and divides once (pool_ops.cpp:255-263), so the result
// equals the reference's sequential float sum exactly.
__global__ void global_avg_pool_f32(const float* __restrict__ x, float* __restrict__ y,
                                    int64_t planes, int64_t spatial) {
  for (int64_t p = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; p < planes;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float* in = x + p * spatial;
    float sum = 0.0f;
    for (int64_t i = 0; i < spatial; ++i) sum = __fadd_rn(sum, in[i]);
    y[p] = __fdiv_rn(sum, static_cast<float>(spatial));
  }
}

// Global average pooling of 8-bit NHWC activations (c_store channels per
// pixel) into dequantized fp32: y[img, ch] = fp32((sum_p q - zp * hw) * scale
// / hw), the sum exact in int32 and the rest in double, rounded once.  One
// warp per (image, 16-channel group): lanes stride over the pixels with
// 16-byte loads, then the 16 per-channel sums are reduced across the warp.
// hw * 255 must fit int32 (the host checks).
template <bool kSigned>
__global__ void q8_global_avg_pool_nhwc(const uint8_t* __restrict__ x, float* __restrict__ y,
                                        int32_t n, int32_t c, int32_t c_store, int64_t hw,
                                        int32_t zp, double scale) {
  const int32_t groups = c_store >> 4;
  const int64_t warp_id = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp_id >= static_cast<int64_t>(n) * groups) return;
  const int32_t img = static_cast<int32_t>(warp_id / groups);
  const int32_t g = static_cast<int32_t>(warp_id - static_cast<int64_t>(img) * groups);
  const uint8_t* base = x + static_cast<int64_t>(img) * hw * c_store + g * 16;
  int32_t s[16] = {};
  for (int64_t p = lane; p < hw; p += 32) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(base + p * c_store));
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t byte = (w4[i] >> (8 * b)) & 0xFFu;
        s[4 * i + b] += kSigned ? static_cast<int32_t>(static_cast<int8_t>(byte))
                                : static_cast<int32_t>(byte);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 16; ++k) s[k] = __reduce_add_sync(0xFFFFFFFFu, s[k]);
  if (lane < 16) {
    const int32_t ch = g * 16 + lane;
    int32_t mine = s[0];
#pragma unroll
    for (int k = 1; k < 16; ++k) mine = lane == k ? s[k] : mine;
    if (ch < c) {
      const double centered = static_cast<double>(mine) - static_cast<double>(zp) * static_cast<double>(hw);
      y[static_cast<int64_t>(img) * c + ch] = __double2float_rn(centered * scale / static_cast<double>(hw));
    }
  }
}

// C broadcast modes of the Gemm bias (gemm_op.cpp:103-139).
enum : int32_t { kGemmCNone = 0, kGemmCScalar = 1, kGemmCRow = 2, kGemmCColumn = 3, kGemmCFull = 4 };

// y[i, j] = alpha * p[i, j] + beta * C(i, j), rounded per operation like the
// reference's separate multiply and add (no fused multiply-add).
__global__ void gemm_epilogue_f32(const float* __restrict__ p, float* __restrict__ y, int64_t m,
                                  int64_t n, float alpha, float beta, const float* __restrict__ c,
                                  int32_t c_mode) {
  const int64_t total = m * n;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = idx / n, j = idx - (idx / n) * n;
    float v = __fmul_rn(alpha, p[idx]);
    if (c_mode != kGemmCNone) {
      const float cv = c_mode == kGemmCScalar ? c[0]
                       : c_mode == kGemmCRow  ? c[i]
                       : c_mode == kGemmCColumn ? c[j]
                                                : c[idx];
      v = __fadd_rn(v, __fmul_rn(beta, cv));
    }
    y[idx] = v;
  }
}

// [rows, cols] -> [cols, rows] through 32 x 33 shared-memory tiles.
__global__ void transpose_f32(const float* __restrict__ in, float* __restrict__ out, int64_t rows,
                              int64_t cols) {
  __shared__ float tile[32][33];
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * 32, r0 = static_cast<int64_t>(blockIdx.y) * 32;
  for (int dy = threadIdx.y; dy < 32; dy += blockDim.y) {
    const int64_t r = r0 + dy, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[dy][threadIdx.x] = in[r * cols + c];
  }
  __syncthreads();
  for (int dy = threadIdx.y; dy < 32; dy += blockDim.y) {
    const int64_t c = c0 + dy, r = r0 + threadIdx.x;
    if (r < rows && c < cols) out[c * rows + r] = tile[threadIdx.x][dy];
  }
}

}  // namespace ie_cuda
