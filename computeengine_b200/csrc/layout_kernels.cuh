// Bandwidth-bound layout kernels: activation NCHW <-> NHWC (8-bit and fp32
// -> bf16 hi/lo planes) and weight repacking into the K-major order the
// implicit-GEMM kernels read.  The reference works in NCHW only
// (conv2d_op.cpp:91-93); the backend converts at graph entry / exit and keeps
// NHWC in between.
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

namespace ie_cuda {

// NCHW 8-bit -> NHWC with c_store channels per pixel (zero filled), XOR mask
// applied to real channels.  Tiles of 32 pixels x 32 channels through shared
// memory so both the read and the write are coalesced.
__global__ void pack_nchw_to_nhwc_u8(const uint8_t* __restrict__ x, uint8_t* __restrict__ y,
                                     int32_t c, int64_t hw, int32_t c_store, uint8_t xor_mask) {
  __shared__ uint8_t tile[32][33];
  const int64_t img = blockIdx.z;
  const int64_t p0 = static_cast<int64_t>(blockIdx.x) * 32;
  const int32_t c0 = blockIdx.y * 32;
  const uint8_t* xi = x + img * c * hw;
  uint8_t* yi = y + img * hw * c_store;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int32_t ch = c0 + r;
    const int64_t p = p0 + threadIdx.x;
    uint8_t v = 0;
    if (ch < c && p < hw) v = xi[static_cast<int64_t>(ch) * hw + p] ^ xor_mask;
    tile[r][threadIdx.x] = v;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int64_t p = p0 + r;
    const int32_t ch = c0 + threadIdx.x;
    if (p < hw && ch < c_store) yi[p * c_store + ch] = tile[threadIdx.x][r];
  }
}

// NHWC (c_store per pixel) -> NCHW, 8-bit.
__global__ void unpack_nhwc_to_nchw_u8(const uint8_t* __restrict__ x, uint8_t* __restrict__ y,
                                       int32_t c, int64_t hw, int32_t c_store) {
  __shared__ uint8_t tile[32][33];
  const int64_t img = blockIdx.z;
  const int64_t p0 = static_cast<int64_t>(blockIdx.x) * 32;
  const int32_t c0 = blockIdx.y * 32;
  const uint8_t* xi = x + img * hw * c_store;
  uint8_t* yi = y + img * c * hw;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int64_t p = p0 + r;
    const int32_t ch = c0 + threadIdx.x;
    uint8_t v = 0;
    if (p < hw && ch < c) v = xi[p * c_store + ch];
    tile[r][threadIdx.x] = v;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int32_t ch = c0 + r;
    const int64_t p = p0 + threadIdx.x;
    if (ch < c && p < hw) yi[static_cast<int64_t>(ch) * hw + p] = tile[threadIdx.x][r];
  }
}

// NCHW fp32 -> NHWC bf16 [hi plane (c_store) | lo plane (c_store)] per pixel,
// x = hi + lo + O(2^-17 |x|).
__global__ void pack_nchw_f32_to_bf16x2(const float* __restrict__ x,
                                        __nv_bfloat16* __restrict__ y, int32_t c, int64_t hw,
                                        int32_t c_store) {
  __shared__ float tile[32][33];
  const int64_t img = blockIdx.z;
  const int64_t p0 = static_cast<int64_t>(blockIdx.x) * 32;
  const int32_t c0 = blockIdx.y * 32;
  const float* xi = x + img * c * hw;
  __nv_bfloat16* yi = y + img * hw * 2 * c_store;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int32_t ch = c0 + r;
    const int64_t p = p0 + threadIdx.x;
    float v = 0.0f;
    if (ch < c && p < hw) v = xi[static_cast<int64_t>(ch) * hw + p];
    tile[r][threadIdx.x] = v;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int64_t p = p0 + r;
    const int32_t ch = c0 + threadIdx.x;
    if (p < hw && ch < c_store) {
      const float v = tile[threadIdx.x][r];
      const __nv_bfloat16 hi = __float2bfloat16_rn(v);
      const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
      yi[p * 2 * c_store + ch] = hi;
      yi[p * 2 * c_store + c_store + ch] = lo;
    }
  }
}

// int8 weights [m, c, kh, kw] -> [m][kh*kw][ck] (ck >= c, zero filled).
__global__ void pack_weights_q8(const int8_t* __restrict__ w, int8_t* __restrict__ out,
                                int32_t m, int32_t c, int32_t taps, int32_t ck) {
  const int64_t total = static_cast<int64_t>(m) * taps * ck;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t ch = static_cast<int32_t>(i % ck);
    const int64_t rest = i / ck;
    const int32_t tap = static_cast<int32_t>(rest % taps);
    const int32_t mo = static_cast<int32_t>(rest / taps);
    int8_t v = 0;
    if (ch < c) v = w[(static_cast<int64_t>(mo) * c + ch) * taps + tap];
    out[i] = v;
  }
}

// fp32 weights [m, c, kh, kw] -> bf16 [m][kh*kw][hi (ck) | lo (ck)].
__global__ void pack_weights_bf16x2(const float* __restrict__ w, __nv_bfloat16* __restrict__ out,
                                    int32_t m, int32_t c, int32_t taps, int32_t ck) {
  const int64_t total = static_cast<int64_t>(m) * taps * ck;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t ch = static_cast<int32_t>(i % ck);
    const int64_t rest = i / ck;
    const int32_t tap = static_cast<int32_t>(rest % taps);
    const int32_t mo = static_cast<int32_t>(rest / taps);
    float v = 0.0f;
    if (ch < c) v = w[(static_cast<int64_t>(mo) * c + ch) * taps + tap];
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
    __nv_bfloat16* row = out + (static_cast<int64_t>(mo) * taps + tap) * 2 * ck;
    row[ch] = hi;
    row[ck + ch] = lo;
  }
}

}  // namespace ie_cuda
