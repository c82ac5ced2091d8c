// CUDA-core convolution kernels for the cases that are not dense contractions:
// depthwise (group == c) int8 in NHWC, and grouped / depthwise fp32 in NCHW.
// Depthwise work is ~9 MACs per output element, far below the tensor-core
// ridge point, so these kernels are written for HBM bandwidth: 128-bit
// channel-vector loads and stores, taps reused through L1/L2.
#pragma once

#include <cstdint>
#include <type_traits>

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

// ------------------------------------------------ 3x3 depthwise, dp4a rows
//
// The MobileNetV2 depthwise layers (3x3, stride 1 or 2, dilation 1) on
// packed-byte arithmetic.  A thread owns 4 channels (one 32-bit word of each
// NHWC pixel) x 4 output columns and walks down a chunk of output rows.  Each
// input row it needs is loaded once (6 or 9 pixel words, requested one output
// row ahead), byte-transposed in registers so that a word holds 4 consecutive
// pixels of one channel, and shifted by funnel shifts into the 4 windows
// [x(ox-1), x(ox), x(ox+1), .] of its output columns; the windows of the
// three input rows under an output row slide down as the thread moves on, and
// one dp4a per (window, filter row) adds three taps.  Filter words and
// requantize constants are set up once per thread.  The
// activation zero point is handled like the dense kernel's: pixels outside
// the image read as the zero point's byte and -zp_x * sum(w[c]) is folded
// into the bias, so every tap contributes (x - zp_x) * w.  The requantize
// constants of the thread's 4 channels stay in registers.
struct Dw3Args {
  int32_t n, h, w, c_store;  // input NHWC
  int32_t out_h, out_w, pad_t, pad_l;
  int32_t c;                 // real channels (== m)
  int32_t zp_x;
  uint32_t zp4;              // zp_x's byte, replicated
  int32_t zp_y, qmin, qmax;
  int32_t words, col_groups;  // c_store / 4, ceil(out_w / 4)
  int32_t chunk, chunks;       // output rows per thread, ceil(out_h / chunk)
};

// Blocks of 128 threads the 3x3 row kernel is compiled to fit per SM.
constexpr int kDwMinBlocks = 3;

template <bool kXSigned>
__device__ __forceinline__ int32_t dp4a_xw(uint32_t x, uint32_t w, int32_t c) {
  int32_t d;
  if constexpr (kXSigned) {
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(x), "r"(w), "r"(c));
  } else {
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(x), "r"(w), "r"(c));
  }
  return d;
}

// 4x4 byte transpose: out[j] = [p0.j, p1.j, p2.j, p3.j].
__device__ __forceinline__ void transpose4x4(uint32_t p0, uint32_t p1, uint32_t p2, uint32_t p3,
                                             uint32_t (&out)[4]) {
  const uint32_t t0 = __byte_perm(p0, p1, 0x5140), t1 = __byte_perm(p2, p3, 0x5140);
  const uint32_t t2 = __byte_perm(p0, p1, 0x7362), t3 = __byte_perm(p2, p3, 0x7362);
  out[0] = __byte_perm(t0, t1, 0x5410);
  out[1] = __byte_perm(t0, t1, 0x7632);
  out[2] = __byte_perm(t2, t3, 0x5410);
  out[3] = __byte_perm(t2, t3, 0x7632);
}

// Windows of one input row for the thread's 4 output columns and 4 channels:
// win[k][j] = [x(c0 + j) at the 4 pixels starting under output column k]
// (stride 1: pixels k .. k+3 of the row segment; stride 2: 2k .. 2k+3).
template <int kStride>
__device__ __forceinline__ void dw_row_windows(const uint32_t (&p)[3 * kStride + 3],
                                               uint32_t (&win)[4][4]) {
  uint32_t A[4], B[4];
  transpose4x4(p[0], p[1], p[2], p[3], A);
  if constexpr (kStride == 1) {
    const uint32_t u0 = __byte_perm(p[4], p[5], 0x5140), u1 = __byte_perm(p[4], p[5], 0x7362);
    B[0] = u0;
    B[1] = u0 >> 16;
    B[2] = u1;
    B[3] = u1 >> 16;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      win[0][j] = A[j];
      win[1][j] = __funnelshift_r(A[j], B[j], 8);
      win[2][j] = __funnelshift_r(A[j], B[j], 16);
      win[3][j] = __funnelshift_r(A[j], B[j], 24);
    }
  } else {
    transpose4x4(p[4], p[5], p[6], p[7], B);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      win[0][j] = A[j];
      win[1][j] = __funnelshift_r(A[j], B[j], 16);
      win[2][j] = B[j];
      win[3][j] = __funnelshift_r(B[j], p[8] >> (8 * j), 16);
    }
  }
}

template <int kStride, bool kXSigned, bool kYSigned>
__global__ void __launch_bounds__(128, kDwMinBlocks) dwconv3x3_q8_nhwc(const uint8_t* __restrict__ x,
                                                         const int8_t* __restrict__ wp,
                                                         const int32_t* __restrict__ bias,
                                                         const float* __restrict__ mult,
                                                         uint8_t* __restrict__ y, Dw3Args a) {
  constexpr int kPix = 3 * kStride + 3;  // input pixels under 4 output columns
  constexpr int kNew = kStride;          // input rows each further output row adds
  // grid: x = (column group, channel word) with the word fastest, y = chunk
  // of a.chunk output rows, z = image; one 32-bit division splits x.
  const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= static_cast<uint32_t>(a.col_groups * a.words)) return;
  const int32_t grp = static_cast<int32_t>(idx / static_cast<uint32_t>(a.words));
  const int32_t wd = static_cast<int32_t>(idx) - grp * a.words;
  const int32_t img = blockIdx.z;
  const int32_t c0 = wd * 4;
  const int32_t ox0 = grp * 4, oy_begin = blockIdx.y * a.chunk;
  const int32_t oy_end = min(oy_begin + a.chunk, a.out_h);

  // filter rows of the 4 channels: wk[ky][j] = [w(ky,0), w(ky,1), w(ky,2), 0]
  uint32_t wk[3][4];
#pragma unroll
  for (int ky = 0; ky < 3; ++ky) {
    const uint32_t w0 = __ldg(reinterpret_cast<const uint32_t*>(wp + (ky * 3 + 0) * a.c_store + c0));
    const uint32_t w1 = __ldg(reinterpret_cast<const uint32_t*>(wp + (ky * 3 + 1) * a.c_store + c0));
    const uint32_t w2 = __ldg(reinterpret_cast<const uint32_t*>(wp + (ky * 3 + 2) * a.c_store + c0));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t t01 = __byte_perm(w0, w1, j | ((4 + j) << 4));
      const uint32_t t2 = __byte_perm(w2, 0u, j | 0x4440);
      wk[ky][j] = __byte_perm(t01, t2, 0x5410);
    }
  }

  // Input row loader: pixel words of row iy under the thread's columns; rows
  // and columns outside the image read as the zero point.
  const uint8_t* const xb = x + static_cast<int64_t>(img) * a.h * a.w * a.c_store + c0;
  const int32_t ix0 = ox0 * kStride - a.pad_l;
  // byte offsets of the thread's input columns within a row (the same for
  // every row), and which of them lie inside the image
  int32_t col_off[kPix];
  uint32_t col_in = 0;
#pragma unroll
  for (int q = 0; q < kPix; ++q) {
    const int32_t ix = ix0 + q;
    const bool in = ix >= 0 && ix < a.w;
    col_off[q] = (in ? ix : 0) * a.c_store;
    col_in |= in ? (1u << q) : 0u;
  }
  const int64_t row_bytes = static_cast<int64_t>(a.w) * a.c_store;
  auto load_row = [&](int32_t iy, uint32_t (&p)[kPix]) {
    const bool row_in = iy >= 0 && iy < a.h;
    const uint8_t* const row = xb + (row_in ? iy : 0) * row_bytes;
#pragma unroll
    for (int q = 0; q < kPix; ++q) {
      p[q] = (row_in && ((col_in >> q) & 1u))
                 ? __ldg(reinterpret_cast<const uint32_t*>(row + col_off[q]))
                 : a.zp4;
    }
  };

  // requantize constants (the implicit-GEMM epilogue's rules, per thread)
  int32_t beff[4], mnt[4];
  long long add[4];
  RequantConst rq[4];
  int32_t smin = 1 << 20;
  bool fast = true, fits = true;
  const long long acc_bound = 9ll * 255 * 128;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int32_t ch = c0 + j;
    const bool in = ch < a.c;
    const int32_t wsum = dp4a_xw<true>(wk[0][j], 0x01010101u,
                                       dp4a_xw<true>(wk[1][j], 0x01010101u,
                                                     dp4a_xw<true>(wk[2][j], 0x01010101u, 0)));
    const int32_t b = (in && bias != nullptr) ? __ldg(bias + ch) : 0;
    beff[j] = static_cast<int32_t>(static_cast<uint32_t>(b) -
                                   static_cast<uint32_t>(a.zp_x) * static_cast<uint32_t>(wsum));
    rq[j] = split_multiplier(in ? __ldg(mult + ch) : 0.0f);
    if (rq[j].mant != 0) smin = min(smin, rq[j].shift);
    fast = fast && rq[j].mant >= 0;
    const long long bb = beff[j];
    fits = fits && (bb < 0 ? -bb : bb) + acc_bound < (1ll << 31);
  }
  if (smin == (1 << 20)) smin = 33;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (rq[j].mant != 0 && rq[j].shift - smin > 7) fast = false;
  }
  fast = fast && smin >= 32 && smin <= 53;
  const int mode = (fast && a.zp_y <= a.qmin && fits) ? kReqFold
                   : (fast && smin >= 33)             ? kReqSigned
                                                      : kReqExact;
  const long long c_add = (1ll << (smin - 1)) + static_cast<long long>(a.zp_y) * (1ll << smin);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    mnt[j] = (mode != kReqExact && rq[j].mant != 0) ? (rq[j].mant >> (rq[j].shift - smin)) : 0;
    add[j] = static_cast<long long>(beff[j]) * mnt[j] + c_add;
  }
  const int32_t hi_c = static_cast<int32_t>(c_add >> 32), shm = smin - 32;

  // Windows of the input rows under the current output row, kept in three
  // slots: relative input row r lives in slot r % 3, so walking down by
  // kStride rows only overwrites the slots of the rows that drop out.  The
  // row loop is unrolled by three so every slot index is a constant (no
  // register moves).  The kNew new rows of each output row are requested one
  // output row ahead.
  uint32_t win[3][4][4];
  uint32_t pf[kNew][kPix];
  const int32_t iy_base = oy_begin * kStride - a.pad_t;  // relative input row 0
  {
    uint32_t p[kPix];
#pragma unroll
    for (int r = 0; r < 3 - kNew; ++r) {
      load_row(iy_base + r, p);
      dw_row_windows<kStride>(p, win[r]);
    }
#pragma unroll
    for (int r = 0; r < kNew; ++r) load_row(iy_base + 3 - kNew + r, pf[r]);
  }
  const int64_t y_row_step = static_cast<int64_t>(a.out_w) * a.c_store;
  const bool col_ok[4] = {ox0 < a.out_w, ox0 + 1 < a.out_w, ox0 + 2 < a.out_w, ox0 + 3 < a.out_w};

  // One output row t of the chunk (T = t % 3 as a constant).
  auto row = [&](auto phase, int32_t t) {
    constexpr int T = decltype(phase)::value;
    constexpr int s0 = (kStride * T) % 3, s1 = (kStride * T + 1) % 3, s2 = (kStride * T + 2) % 3;
    const int32_t oy = oy_begin + t;
#pragma unroll
    for (int r = 0; r < kNew; ++r) {
      constexpr int dummy = 0;
      (void)dummy;
      dw_row_windows<kStride>(pf[r], win[(kStride * T + 3 - kNew + r) % 3]);
    }
    if (oy + 1 < oy_end) {
      const int32_t iy_next = iy_base + (t + 1) * kStride + 3 - kNew;
#pragma unroll
      for (int r = 0; r < kNew; ++r) load_row(iy_next + r, pf[r]);
    }
    uint8_t* const yrow = y + ((static_cast<int64_t>(img) * a.out_h + oy) * a.out_w + ox0) * a.c_store + c0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      int32_t acc[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        int32_t v = dp4a_xw<kXSigned>(win[s0][k][j], wk[0][j], 0);
        v = dp4a_xw<kXSigned>(win[s1][k][j], wk[1][j], v);
        acc[j] = dp4a_xw<kXSigned>(win[s2][k][j], wk[2][j], v);
      }
      int32_t q[4];
      if (mode == kReqFold) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const long long pr = static_cast<long long>(acc[j]) * mnt[j] + add[j];
          q[j] = min(max(static_cast<int32_t>(pr >> 32) >> shm, a.qmin), a.qmax);
        }
      } else if (mode == kReqSigned) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int32_t tt = static_cast<int32_t>(static_cast<uint32_t>(acc[j]) +
                                                  static_cast<uint32_t>(beff[j]));
          const int32_t sg = tt >> 31;
          const long long cs = static_cast<long long>(
              (static_cast<unsigned long long>(static_cast<uint32_t>(hi_c + sg)) << 32) |
              static_cast<uint32_t>(sg));
          const long long pr = static_cast<long long>(tt) * mnt[j] + cs;
          q[j] = min(max(static_cast<int32_t>(pr >> 32) >> shm, a.qmin), a.qmax);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int32_t tt = static_cast<int32_t>(static_cast<uint32_t>(acc[j]) +
                                                  static_cast<uint32_t>(beff[j]));
          q[j] = requant_exact(tt, rq[j], a.zp_y, a.qmin, a.qmax);
        }
      }
      if (col_ok[k]) {
        // every q is already clamped to [qmin, qmax] inside the storage type:
        // its low byte is the stored value (two's complement for int8)
        const uint32_t w = __byte_perm(__byte_perm(static_cast<uint32_t>(q[0]), static_cast<uint32_t>(q[1]), 0x0040),
                                       __byte_perm(static_cast<uint32_t>(q[2]), static_cast<uint32_t>(q[3]), 0x0040),
                                       0x5410);
        *reinterpret_cast<uint32_t*>(yrow + k * a.c_store) = w;
      }
    }
  };
  (void)y_row_step;
  const int32_t rows = oy_end - oy_begin;
#pragma unroll 1
  for (int32_t t = 0; t < rows; t += 3) {
    row(std::integral_constant<int, 0>{}, t);
    if (t + 1 >= rows) break;
    row(std::integral_constant<int, 1>{}, t + 1);
    if (t + 2 >= rows) break;
    row(std::integral_constant<int, 2>{}, t + 2);
  }
}

// ------------------------------------------------------------ int8 Add
//
// y = clamp(round_half_away((a - zp_a) * mult_a + (b - zp_b) * mult_b) + zp_y)
// over two quantized tensors of one layout, exactly: each fp32 multiplier is
// mant * 2^-shift, the two products are brought to the common shift s and
// summed in 128-bit integers (the host rejects shifts more than 60 apart).
struct QAddArgs {
  int64_t count;
  long long ma, mb;  // significands (0 for a vanishing term)
  int32_t da, db;    // s - shift_a, s - shift_b (0..60)
  int32_t s;         // common shift
  int32_t zp_a, zp_b, zp_y, qmin, qmax;
  int32_t a_signed, b_signed, y_signed;
};

// One term of the narrow (64-bit) form, and its rounding half away from zero,
// zero point and clamp.
__device__ __forceinline__ long long qadd_term64(int32_t x, int32_t zp, long long m, int32_t d) {
  return (static_cast<long long>(x - zp) * m) << d;
}
__device__ __forceinline__ uint32_t qadd_round64(long long v, const QAddArgs& k) {
  const long long r = (v + (1ll << (k.s - 1)) - (v < 0 ? 1 : 0)) >> k.s;
  long long q = r + k.zp_y;
  q = q < k.qmin ? k.qmin : (q > k.qmax ? k.qmax : q);
  return static_cast<uint32_t>(q) & 0xFFu;
}

// kWide = false when both terms and their sum fit in 64 bits and the shift is
// in [1, 62] (|x - zp| <= 255 < 2^8, significand < 2^31, da, db <= 22: each
// term < 2^61); the host checks that before choosing it.
template <bool kWide>
__device__ __forceinline__ uint32_t qadd_one(uint32_t av, uint32_t bv, const QAddArgs& k) {
  const int32_t a = k.a_signed ? static_cast<int32_t>(static_cast<int8_t>(av)) : static_cast<int32_t>(av);
  const int32_t b = k.b_signed ? static_cast<int32_t>(static_cast<int8_t>(bv)) : static_cast<int32_t>(bv);
  long long r;
  if constexpr (!kWide) {
    return qadd_round64(qadd_term64(a, k.zp_a, k.ma, k.da) + qadd_term64(b, k.zp_b, k.mb, k.db), k);
  }
  const __int128 v = (static_cast<__int128>(static_cast<long long>(a - k.zp_a) * k.ma) << k.da) +
                     (static_cast<__int128>(static_cast<long long>(b - k.zp_b) * k.mb) << k.db);
  if (k.s >= 127) {
    r = 0;
  } else if (k.s <= 0) {
    r = v == 0 ? 0 : (v > 0 ? (1ll << 40) : -(1ll << 40));
  } else {
    const __int128 half = static_cast<__int128>(1) << (k.s - 1);
    r = static_cast<long long>((v + half - (v < 0 ? 1 : 0)) >> k.s);
  }
  long long q = r + k.zp_y;
  q = q < k.qmin ? k.qmin : (q > k.qmax ? k.qmax : q);
  return static_cast<uint32_t>(q) & 0xFFu;
}

// 16 elements per thread when vec16 (pointers 16-byte aligned, count a
// multiple of 16), else one.
template <bool kWide>
__global__ void __launch_bounds__(256) qadd_u8(const uint8_t* __restrict__ a,
                                               const uint8_t* __restrict__ b,
                                               uint8_t* __restrict__ y, QAddArgs k, int vec16) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t t0 = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (vec16) {
    for (int64_t t = t0; t < k.count / 16; t += stride) {
      const uint4 va = __ldg(reinterpret_cast<const uint4*>(a) + t);
      const uint4 vb = __ldg(reinterpret_cast<const uint4*>(b) + t);
      const uint32_t wa[4] = {va.x, va.y, va.z, va.w}, wb[4] = {vb.x, vb.y, vb.z, vb.w};
      uint32_t wy[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t o = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          o |= qadd_one<kWide>((wa[q] >> (8 * i)) & 0xFFu, (wb[q] >> (8 * i)) & 0xFFu, k) << (8 * i);
        }
        wy[q] = o;
      }
      reinterpret_cast<uint4*>(y)[t] = make_uint4(wy[0], wy[1], wy[2], wy[3]);
    }
  } else {
    for (int64_t t = t0; t < k.count; t += stride) {
      y[t] = static_cast<uint8_t>(qadd_one<kWide>(__ldg(a + t), __ldg(b + t), k));
    }
  }
}

// The same Add over large tensors through a table: the result depends only on
// the two input bytes, so each block first fills a 64 KB shared-memory table
// with the exact rule above (from the two 256-entry term tables in the 64-bit
// form) and then maps 16 byte pairs per 16-byte load through it, two loads per
// thread in flight.  One 1024-thread block per SM; the table costs a few
// microseconds per launch.  The pair (a, b) sits at a * 256 + (b ^ ((a & 31)
// << 2)): with the plain a * 256 + b every row starts in bank 0, so lanes that
// share b (a ReLU output full of zeros) but differ in a would all hit one
// bank; the XOR spreads them over the 32 banks.  Requires 16-byte aligned
// pointers.
__device__ __forceinline__ uint32_t qadd_lut_slot(uint32_t i) {
  return i ^ ((i >> 6) & 0x007C007Cu);  // both 16-bit halves: b ^= (a & 31) << 2
}

__device__ __forceinline__ uint32_t qadd_lut4(uint32_t wa, uint32_t wb, const uint8_t* lut) {
  // [b0 a0 b1 a1]: a0 * 256 + b0 | a1 * 256 + b1, then the bank swizzle
  const uint32_t i01 = qadd_lut_slot(__byte_perm(wb, wa, 0x5140));
  const uint32_t i23 = qadd_lut_slot(__byte_perm(wb, wa, 0x7362));
  return static_cast<uint32_t>(lut[i01 & 0xFFFFu]) | (static_cast<uint32_t>(lut[i01 >> 16]) << 8) |
         (static_cast<uint32_t>(lut[i23 & 0xFFFFu]) << 16) | (static_cast<uint32_t>(lut[i23 >> 16]) << 24);
}

__device__ __forceinline__ uint4 qadd_lut16(const uint4 va, const uint4 vb, const uint8_t* lut) {
  return make_uint4(qadd_lut4(va.x, vb.x, lut), qadd_lut4(va.y, vb.y, lut), qadd_lut4(va.z, vb.z, lut),
                    qadd_lut4(va.w, vb.w, lut));
}

constexpr int kQAddLutThreads = 1024;
constexpr int kQAddLutBytes = 65536;

template <bool kWide>
__global__ void __launch_bounds__(kQAddLutThreads) qadd_lut_u8(const uint4* __restrict__ a,
                                                               const uint4* __restrict__ b,
                                                               uint4* __restrict__ y, QAddArgs k,
                                                               int64_t chunks) {
  extern __shared__ __align__(16) uint8_t lut[];
  __shared__ long long ta[256], tb[256];
  const int tid = threadIdx.x;
  if constexpr (!kWide) {
    if (tid < 256) {
      const int32_t x = k.a_signed ? static_cast<int32_t>(static_cast<int8_t>(tid)) : tid;
      ta[tid] = qadd_term64(x, k.zp_a, k.ma, k.da);
    } else if (tid < 512) {
      const int32_t x = k.b_signed ? static_cast<int32_t>(static_cast<int8_t>(tid - 256)) : tid - 256;
      tb[tid - 256] = qadd_term64(x, k.zp_b, k.mb, k.db);
    }
    __syncthreads();
    for (int i = tid; i < kQAddLutBytes; i += kQAddLutThreads) {
      const int av = i >> 8, bv = (i & 255) ^ ((av & 31) << 2);  // the pair stored at slot i
      lut[i] = static_cast<uint8_t>(qadd_round64(ta[av] + tb[bv], k));
    }
  } else {
    for (int i = tid; i < kQAddLutBytes; i += kQAddLutThreads) {
      const uint32_t av = static_cast<uint32_t>(i) >> 8, bv = (static_cast<uint32_t>(i) & 255u) ^ ((av & 31u) << 2);
      lut[i] = static_cast<uint8_t>(qadd_one<true>(av, bv, k));
    }
  }
  __syncthreads();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kQAddLutThreads;
  int64_t t = static_cast<int64_t>(blockIdx.x) * kQAddLutThreads + tid;
  for (; t + stride < chunks; t += 2 * stride) {
    const uint4 a0 = __ldg(a + t), b0 = __ldg(b + t);
    const uint4 a1 = __ldg(a + t + stride), b1 = __ldg(b + t + stride);
    y[t] = qadd_lut16(a0, b0, lut);
    y[t + stride] = qadd_lut16(a1, b1, lut);
  }
  if (t < chunks) y[t] = qadd_lut16(__ldg(a + t), __ldg(b + t), lut);
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
