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

// Per-output-channel sums of packed int8 weights: wsum[mo] = sum of the
// k_row bytes of row mo (rows past m, up to m_store, get 0).  The epilogue
// folds -zp_x * wsum[mo] into the int32 bias, which turns the accumulator of
// raw stored activations into sum (x - zp_x) * w.  One warp per row; k_row is
// a multiple of 16 and rows start 16-byte aligned.
__global__ void q8_weight_sums(const int8_t* __restrict__ packed, int32_t* __restrict__ wsum,
                               int32_t m, int32_t m_store, int64_t k_row) {
  const int32_t row = static_cast<int32_t>((blockIdx.x * static_cast<int64_t>(blockDim.x) +
                                            threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= m_store) return;
  int32_t acc = 0;
  if (row < m) {
    const int4* r = reinterpret_cast<const int4*>(packed + static_cast<int64_t>(row) * k_row);
    for (int64_t i = lane; i < k_row / 16; i += 32) {
      const int4 v = __ldg(r + i);
      // __dp4a with all-ones multipliers sums four signed bytes
      acc = __dp4a(v.x, 0x01010101, acc);
      acc = __dp4a(v.y, 0x01010101, acc);
      acc = __dp4a(v.z, 0x01010101, acc);
      acc = __dp4a(v.w, 0x01010101, acc);
    }
  }
  acc = __reduce_add_sync(0xFFFFFFFFu, acc);
  if (lane == 0) wsum[row] = acc;
}

// NCHW 8-bit -> NHWC with a halo: y is [n, hp, wp, c_store] and pixel (iy, ix)
// of y holds x[., iy - pt, ix - pl] when that lies inside the image, else the
// fill byte; channels past c hold the fill byte too.  With fill = zp_x the
// padding of a convolution run over y with zero pads contributes
// (zp_x - zp_x) * w = 0, the reference's "padding is real 0.0".
__global__ void pack_nchw_to_nhwc_halo_u8(const uint8_t* __restrict__ x, uint8_t* __restrict__ y,
                                          int32_t c, int32_t h, int32_t w, int32_t c_store,
                                          int32_t pt, int32_t pl, int32_t hp, int32_t wp,
                                          uint8_t fill) {
  __shared__ uint8_t tile[32][33];
  const int64_t img = blockIdx.z;
  const int64_t hw = static_cast<int64_t>(h) * w, hwp = static_cast<int64_t>(hp) * wp;
  const int64_t p0 = static_cast<int64_t>(blockIdx.x) * 32;  // halo pixel index
  const int32_t c0 = blockIdx.y * 32;
  const uint8_t* xi = x + img * c * hw;
  uint8_t* yi = y + img * hwp * c_store;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int32_t ch = c0 + r;
    const int64_t p = p0 + threadIdx.x;
    uint8_t v = fill;
    if (ch < c && p < hwp) {
      const int32_t iy = static_cast<int32_t>(p / wp) - pt;
      const int32_t ix = static_cast<int32_t>(p % wp) - pl;
      if (iy >= 0 && iy < h && ix >= 0 && ix < w) {
        v = xi[static_cast<int64_t>(ch) * hw + static_cast<int64_t>(iy) * w + ix];
      }
    }
    tile[r][threadIdx.x] = v;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int64_t p = p0 + r;
    const int32_t ch = c0 + threadIdx.x;
    if (p < hwp && ch < c_store) yi[p * c_store + ch] = tile[threadIdx.x][r];
  }
}

// NHWC 8-bit [n, h, w, c_store] -> the same with a halo, [n, hp, wp, c_store]
// (pixel (iy, ix) from (iy - pt, ix - pl), the fill byte outside the image).
// One thread per output pixel x 16 channels, 16-byte loads and stores.
__global__ void halo_nhwc_u8(const uint8_t* __restrict__ x, uint8_t* __restrict__ y, int32_t n,
                             int32_t h, int32_t w, int32_t c_store, int32_t pt, int32_t pl,
                             int32_t hp, int32_t wp, uint8_t fill) {
  const int32_t groups = c_store >> 4;
  const int64_t total = static_cast<int64_t>(n) * hp * wp * groups;
  const uint32_t f4 = 0x01010101u * fill;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t g = static_cast<int32_t>(i % groups);
    const int64_t pix = i / groups;
    const int32_t ix = static_cast<int32_t>(pix % wp) - pl;
    const int64_t t = pix / wp;
    const int32_t iy = static_cast<int32_t>(t % hp) - pt;
    const int64_t img = t / hp;
    uint4 v = make_uint4(f4, f4, f4, f4);
    if (iy >= 0 && iy < h && ix >= 0 && ix < w) {
      v = __ldg(reinterpret_cast<const uint4*>(
          x + ((img * h + iy) * w + ix) * c_store + g * 16));
    }
    *reinterpret_cast<uint4*>(y + pix * c_store + g * 16) = v;
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

namespace ie_cuda {

// Stem re-layout for a 7x7 / stride 2 / pad 3 convolution on c <= 4 channels.
// Space-to-depth by 2 plus a 4-column unroll turns the stem into a 4x1,
// stride-1 convolution over 16*c channels (stored as 64), so it runs on the
// same implicit-GEMM kernel as every other layer:
//   out[i][j][(ch*2+dy)*8 + 2b+dx] = x[ch][2i+dy][2(j+b-2)+dx]   (0 if j+b-2
//   is outside [0, w/2)), i in [0, h/2), j in [0, w/2); channels 16c..63 are 0
// For a fixed (ch, dy) the eight bytes 2b+dx = 0..7 are the input columns
// 2j-4 .. 2j+3 of one row, in order, so every output word is one
// funnel-shifted word of that row, and 16-byte chunk ch of a pixel is
// channel ch's two rows.  One block per (image, output row i): input rows 2i
// and 2i+1 of every channel are staged in shared memory between 16-byte zero
// margins (so columns outside the image read as 0), then each thread builds
// one 16-byte chunk of one output pixel from two funnel-shifted word pairs
// and stores it directly (consecutive threads, consecutive chunks: coalesced
// 16-byte stores).  The channel order is this layout's own; the weights are
// packed to match (stem_pack_weights_q8).
constexpr int kStemMargin = 16;

// Staged row stride: margins, the row, rounded to 16 bytes, plus 16 bytes so
// that the 2C staged rows start in different shared-memory banks.
__host__ __device__ constexpr int stem_row_stride(int w) {
  return ((w + 2 * kStemMargin + 15) / 16) * 16 + 16;
}

template <int C>
__global__ void __launch_bounds__(128) stem_pack_s2d_u8(const uint8_t* __restrict__ x,
                                                        uint8_t* __restrict__ y, int32_t h,
                                                        int32_t w, uint8_t xor_mask) {
  extern __shared__ __align__(16) uint8_t stem_smem[];
  const int32_t ho = h / 2, wo = w / 2;
  const int32_t rs = stem_row_stride(w);
  uint8_t* rows = stem_smem;  // [C][2][rs]: margin | w columns | margin
  const int32_t i = blockIdx.x % ho;
  const int64_t img = blockIdx.x / ho;
  const uint8_t* xi = x + img * C * h * static_cast<int64_t>(w);
  const uint32_t mask4 = 0x01010101u * xor_mask;

  // zero margins
  const int32_t right = rs - kStemMargin - w;
  for (int t = threadIdx.x; t < C * 2 * (kStemMargin + right); t += blockDim.x) {
    const int32_t r = t / (kStemMargin + right), k = t % (kStemMargin + right);
    rows[r * rs + (k < kStemMargin ? k : kStemMargin + w + k - kStemMargin)] = 0;
  }
  // rows 2i, 2i+1 of every channel (contiguous 2w bytes per channel in NCHW)
  if ((w & 15) == 0 && ((reinterpret_cast<uintptr_t>(xi) + 2 * i * static_cast<int64_t>(w)) & 15) == 0) {
    // all channels' 16-byte pieces in one pass
    const int32_t per = (2 * w) >> 4;
    for (int t = threadIdx.x; t < C * per; t += blockDim.x) {
      const int32_t cc = t / per, q = t - cc * per;
      uint4 v = __ldg(reinterpret_cast<const uint4*>(xi + (static_cast<int64_t>(cc) * h + 2 * i) * w) + q);
      v.x ^= mask4;
      v.y ^= mask4;
      v.z ^= mask4;
      v.w ^= mask4;
      const int32_t off = q << 4, dy = off >= w;
      *reinterpret_cast<uint4*>(rows + cc * 2 * rs + kStemMargin + dy * rs + off - dy * w) = v;
    }
  } else {
#pragma unroll
    for (int cc = 0; cc < C; ++cc) {
      const uint8_t* src = xi + (static_cast<int64_t>(cc) * h + 2 * i) * w;
      uint8_t* dst = rows + cc * 2 * rs + kStemMargin;
      for (int t = threadIdx.x; t < 2 * w; t += blockDim.x) {
        const int32_t dy = t >= w;
        dst[dy * rs + t - dy * w] = src[t] ^ xor_mask;
      }
    }
  }
  __syncthreads();

  // 16-byte chunk k of pixel j = words 4k .. 4k+3 = channel k: input
  // columns 2j-4 .. 2j+3 of rows 2i and 2i+1 (zero for k >= C).  Consecutive
  // threads write consecutive chunks: coalesced 16-byte stores.
  uint4* out = reinterpret_cast<uint4*>(y + ((img * ho + i) * static_cast<int64_t>(wo)) * 64);
  for (int t = threadIdx.x; t < wo * 4; t += blockDim.x) {
    const int32_t j = t >> 2, k = t & 3;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (k < C) {
      // columns 2j-4 .. 2j+3 start at byte kStemMargin - 4 + 2j (even)
      const int32_t base = kStemMargin - 4 + 2 * j;
      const uint32_t sh = (base & 3) * 8;
      const uint32_t* r0 = reinterpret_cast<const uint32_t*>(rows + (k * 2) * rs + (base & ~3));
      const uint32_t* r1 = reinterpret_cast<const uint32_t*>(rows + (k * 2 + 1) * rs + (base & ~3));
      v.x = __funnelshift_r(r0[0], r0[1], sh);
      v.y = __funnelshift_r(r0[1], r0[2], sh);
      v.z = __funnelshift_r(r1[0], r1[1], sh);
      v.w = __funnelshift_r(r1[1], r1[2], sh);
    }
    out[t] = v;
  }
}

// Weights of the same stem, [m, c, 7, 7] int8 -> the 4x1 layer's weights in
// packed form [m][4 taps][64 channels].
__global__ void stem_pack_weights_q8(const int8_t* __restrict__ w, int8_t* __restrict__ out,
                                     int32_t m, int32_t c) {
  const int64_t total = static_cast<int64_t>(m) * 4 * 64;
  const int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (idx >= total) return;
  const int32_t chan = static_cast<int32_t>(idx % 64);
  const int32_t a = static_cast<int32_t>((idx / 64) % 4);
  const int32_t mo = static_cast<int32_t>(idx / 256);
  int8_t v = 0;
  if (chan < 16 * c) {
    const int32_t cc = chan >> 4, dy = (chan >> 3) & 1, k = chan & 7;
    const int32_t b = k >> 1, dx = k & 1;
    const int32_t ky = 2 * a + dy - 1, kx = 2 * b + dx - 1;
    if (ky >= 0 && ky < 7 && kx >= 0 && kx < 7) {
      v = w[((static_cast<int64_t>(mo) * c + cc) * 7 + ky) * 7 + kx];
    }
  }
  out[idx] = v;
}

// Max pooling over split fp32 activations: bf16 NHWC with [hi plane (c_store)
// | lo plane (c_store)] per pixel.  The pair with the largest hi + lo (exact
// in fp32) is copied, so the pool keeps the stored values bit for bit.  One
// thread per output pixel x 8 channels; padding never wins.
__global__ void maxpool_f32x2_nhwc(const __nv_bfloat16* __restrict__ x,
                                   __nv_bfloat16* __restrict__ y, int32_t n, int32_t h, int32_t w,
                                   int32_t c_store, int32_t oh, int32_t ow, int32_t k,
                                   int32_t stride, int32_t pad) {
  const int32_t groups = c_store >> 3;
  const int64_t total = static_cast<int64_t>(n) * oh * ow * groups;
  const int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (idx >= total) return;
  const int32_t g = static_cast<int32_t>(idx % groups);
  const int64_t pix = idx / groups;
  const int32_t ox = static_cast<int32_t>(pix % ow);
  const int32_t oy = static_cast<int32_t>((pix / ow) % oh);
  const int32_t img = static_cast<int32_t>(pix / (static_cast<int64_t>(ow) * oh));
  float best[8];
  uint4 bh = make_uint4(0, 0, 0, 0), bl = make_uint4(0, 0, 0, 0);
#pragma unroll
  for (int j = 0; j < 8; ++j) best[j] = -INFINITY;
  for (int ky = 0; ky < k; ++ky) {
    const int32_t iy = oy * stride - pad + ky;
    if (iy < 0 || iy >= h) continue;
    for (int kx = 0; kx < k; ++kx) {
      const int32_t ix = ox * stride - pad + kx;
      if (ix < 0 || ix >= w) continue;
      const __nv_bfloat16* px = x + ((static_cast<int64_t>(img) * h + iy) * w + ix) * 2 * c_store;
      const uint4 vh = __ldg(reinterpret_cast<const uint4*>(px + g * 8));
      const uint4 vl = __ldg(reinterpret_cast<const uint4*>(px + c_store + g * 8));
      const __nv_bfloat16* hh = reinterpret_cast<const __nv_bfloat16*>(&vh);
      const __nv_bfloat16* ll = reinterpret_cast<const __nv_bfloat16*>(&vl);
      __nv_bfloat16* bhh = reinterpret_cast<__nv_bfloat16*>(&bh);
      __nv_bfloat16* bll = reinterpret_cast<__nv_bfloat16*>(&bl);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float v = __bfloat162float(hh[j]) + __bfloat162float(ll[j]);
        if (v > best[j]) {
          best[j] = v;
          bhh[j] = hh[j];
          bll[j] = ll[j];
        }
      }
    }
  }
  __nv_bfloat16* out = y + pix * 2 * c_store;
  *reinterpret_cast<uint4*>(out + g * 8) = bh;
  *reinterpret_cast<uint4*>(out + c_store + g * 8) = bl;
}

// Byte-wise maximum of 16-byte channel vectors on 16-bit lanes: a vector is
// spread over 8 words of two lanes (even and odd bytes, zero- or
// sign-extended by one byte permute each), the maximum is the sm_90+ SIMD
// max.u16x2 / max.s16x2, and the low bytes of the lanes are packed back.
struct Lanes16 {
  uint32_t v[8];
};

// prmt.b32 with the full 4-bit selectors: a selector's top bit replicates the
// sign of the selected byte (the __byte_perm intrinsic reads 3 bits only).
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

template <bool kSigned>
__device__ __forceinline__ Lanes16 lanes_of(uint4 q) {
  // selectors: bytes 0 and 2 (1 and 3) of the word, each followed by a zero
  // byte (unsigned) or by its own sign replicated (signed)
  constexpr uint32_t kEven = kSigned ? 0xA280u : 0x4240u;
  constexpr uint32_t kOdd = kSigned ? 0xB391u : 0x4341u;
  Lanes16 l;
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    l.v[2 * i] = prmt(w[i], 0u, kEven);
    l.v[2 * i + 1] = prmt(w[i], 0u, kOdd);
  }
  return l;
}

template <bool kSigned>
__device__ __forceinline__ uint32_t max16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  if constexpr (kSigned) {
    asm("max.s16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  } else {
    asm("max.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  }
  return d;
}

template <bool kSigned>
__device__ __forceinline__ void lanes_max(Lanes16& acc, const Lanes16& l) {
#pragma unroll
  for (int i = 0; i < 8; ++i) acc.v[i] = max16x2<kSigned>(acc.v[i], l.v[i]);
}

// The identity of the maximum: every lane at the storage type's minimum.
template <bool kSigned>
__device__ __forceinline__ Lanes16 lanes_min() {
  Lanes16 l;
#pragma unroll
  for (int i = 0; i < 8; ++i) l.v[i] = kSigned ? 0xFF80FF80u : 0u;
  return l;
}

__device__ __forceinline__ uint4 lanes_pack(const Lanes16& l) {
  // byte 0 of each lane: even lane words give bytes 0 / 2, odd ones 1 / 3
  return make_uint4(__byte_perm(l.v[0], l.v[1], 0x6240u), __byte_perm(l.v[2], l.v[3], 0x6240u),
                    __byte_perm(l.v[4], l.v[5], 0x6240u), __byte_perm(l.v[6], l.v[7], 0x6240u));
}

// Max pooling over 8-bit NHWC activations (k x k, stride, symmetric pad),
// 16 channels per thread, one output pixel per thread; windows only cover
// real pixels (padding never wins).
template <bool kSigned>
__global__ void maxpool_q8_nhwc(const uint8_t* __restrict__ x, uint8_t* __restrict__ y,
                                int32_t n, int32_t h, int32_t w, int32_t c_store, int32_t oh,
                                int32_t ow, int32_t k, int32_t stride, int32_t pad) {
  const int32_t groups = c_store >> 4;
  const int64_t total = static_cast<int64_t>(n) * oh * ow * groups;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t g = static_cast<int32_t>(idx % groups);
    const int64_t pix = idx / groups;
    const int32_t ox = static_cast<int32_t>(pix % ow);
    const int32_t oy = static_cast<int32_t>((pix / ow) % oh);
    const int64_t img = pix / (static_cast<int64_t>(ow) * oh);
    Lanes16 best = lanes_min<kSigned>();
    for (int ky = 0; ky < k; ++ky) {
      const int32_t iy = oy * stride - pad + ky;
      if (iy < 0 || iy >= h) continue;
      for (int kx = 0; kx < k; ++kx) {
        const int32_t ix = ox * stride - pad + kx;
        if (ix < 0 || ix >= w) continue;
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(
            x + ((img * h + iy) * w + ix) * c_store + g * 16));
        lanes_max<kSigned>(best, lanes_of<kSigned>(v));
      }
    }
    reinterpret_cast<uint4*>(y)[idx] = lanes_pack(best);
  }
}

// The 3x3 / stride-2 pool of the ResNet stem (pad < 3).  Each thread walks
// `rows` output rows of one 16-channel group at one output column: the
// maximum of each input row over the window's three columns is taken once,
// and the last row of one window is the first row of the next, so an output
// row costs two new input rows (six 16-byte loads) instead of nine taps.
// Columns outside the image are replaced by the window's first in-image
// column (always present: pad < 3), which leaves the maximum unchanged.
template <bool kSigned>
__global__ void __launch_bounds__(256) maxpool3x3s2_q8_nhwc(
    const uint8_t* __restrict__ x, uint8_t* __restrict__ y, int32_t n, int32_t h, int32_t w,
    int32_t c_store, int32_t oh, int32_t ow, int32_t pad, int32_t rows, int32_t chunks) {
  const int32_t groups = c_store >> 4;
  const int64_t total = static_cast<int64_t>(n) * chunks * ow * groups;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t g = static_cast<int32_t>(idx % groups);
    int64_t t = idx / groups;
    const int32_t ox = static_cast<int32_t>(t % ow);
    t /= ow;
    const int32_t chunk = static_cast<int32_t>(t % chunks);
    const int64_t img = t / chunks;
    const int32_t x0 = 2 * ox - pad;
    const int32_t fx = min(max(x0, 0), w - 1);
    const int32_t c0 = fx, c1 = (x0 + 1 >= 0 && x0 + 1 < w) ? x0 + 1 : fx;
    const int32_t c2 = x0 + 2 < w ? x0 + 2 : fx;
    const uint8_t* base = x + img * h * static_cast<int64_t>(w) * c_store + g * 16;
    auto row_max = [&](int32_t iy) {
      const uint8_t* r = base + static_cast<int64_t>(iy) * w * c_store;
      const uint4 a = __ldg(reinterpret_cast<const uint4*>(r + static_cast<int64_t>(c0) * c_store));
      const uint4 b = __ldg(reinterpret_cast<const uint4*>(r + static_cast<int64_t>(c1) * c_store));
      const uint4 c = __ldg(reinterpret_cast<const uint4*>(r + static_cast<int64_t>(c2) * c_store));
      Lanes16 m = lanes_of<kSigned>(a);
      lanes_max<kSigned>(m, lanes_of<kSigned>(b));
      lanes_max<kSigned>(m, lanes_of<kSigned>(c));
      return m;
    };
    const int32_t oy0 = chunk * rows;
    const int32_t oy1 = min(oh, oy0 + rows);
    Lanes16 carry = lanes_min<kSigned>();  // row max of the window's first row
    bool have_carry = false;
    for (int32_t oy = oy0; oy < oy1; ++oy) {
      const int32_t y0 = 2 * oy - pad;
      Lanes16 acc = lanes_min<kSigned>();
      if (have_carry) {
        acc = carry;
      } else if (y0 >= 0 && y0 < h) {
        acc = row_max(y0);
      }
      if (y0 + 1 >= 0 && y0 + 1 < h) lanes_max<kSigned>(acc, row_max(y0 + 1));
      carry = lanes_min<kSigned>();
      if (y0 + 2 >= 0 && y0 + 2 < h) {
        carry = row_max(y0 + 2);
        lanes_max<kSigned>(acc, carry);
      }
      have_carry = true;
      reinterpret_cast<uint4*>(y)[((img * oh + oy) * ow + ox) * groups + g] = lanes_pack(acc);
    }
  }
}

// Max pooling of 8-bit NHWC activations under any resolved pooling
// configuration (rectangular kernel, per-axis strides, asymmetric padding,
// ceil_mode output size): the window of output (oy, ox) starts at
// (oy * stride_h - pad_t, ox * stride_w - pad_l), out-of-image positions are
// skipped, and a window with no in-image position gives the storage type's
// minimum (the 8-bit counterpart of the fp32 pool's -inf start).
struct Q8PoolArgs {
  int32_t n, h, w, c_store, out_h, out_w;
  int32_t kh, kw, stride_h, stride_w, pad_t, pad_l;
};

template <bool kSigned>
__global__ void maxpool_q8_nhwc_any(const uint8_t* __restrict__ x, uint8_t* __restrict__ y,
                                    const Q8PoolArgs a) {
  const int32_t groups = a.c_store >> 4;
  const int64_t total = static_cast<int64_t>(a.n) * a.out_h * a.out_w * groups;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t g = static_cast<int32_t>(idx % groups);
    const int64_t pix = idx / groups;
    const int32_t ox = static_cast<int32_t>(pix % a.out_w);
    const int32_t oy = static_cast<int32_t>((pix / a.out_w) % a.out_h);
    const int64_t img = pix / (static_cast<int64_t>(a.out_w) * a.out_h);
    const int32_t y0 = oy * a.stride_h - a.pad_t, x0 = ox * a.stride_w - a.pad_l;
    const int32_t ky0 = max(0, -y0), ky1 = min(a.kh, a.h - y0);
    const int32_t kx0 = max(0, -x0), kx1 = min(a.kw, a.w - x0);
    const uint8_t* base = x + img * a.h * static_cast<int64_t>(a.w) * a.c_store + g * 16;
    Lanes16 best = lanes_min<kSigned>();
    for (int32_t ky = ky0; ky < ky1; ++ky) {
      const uint8_t* row = base + static_cast<int64_t>(y0 + ky) * a.w * a.c_store;
      for (int32_t kx = kx0; kx < kx1; ++kx) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(row + static_cast<int64_t>(x0 + kx) * a.c_store));
        lanes_max<kSigned>(best, lanes_of<kSigned>(v));
      }
    }
    reinterpret_cast<uint4*>(y)[idx] = lanes_pack(best);
  }
}

}  // namespace ie_cuda
