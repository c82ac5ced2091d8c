// Implicit-GEMM convolution on tcgen05 tensor cores (sm_100a).
//
// GEMM view of an NHWC convolution (the reference computes the same sums as
// im2col + one row GEMM per output channel, conv2d_op.cpp:189-241):
//   rows    = output pixels p = (n, oy, ox), flattened; a tile holds
//             128 * M_SUB of them (M_SUB sub-tiles of 128, one MMA each)
//   columns = output channels, BN per tile
//   K       = (tap = ky*kW + kx, channel block of BK bytes)
// A tiles come straight from the NHWC activation tensor through TMA im2col
// loads (one load per k-step covers all 128 * M_SUB pixels; padding and image
// edges read as zero).  B tiles (K-major packed weights) are either streamed
// per k-step or, when the CTA's whole weight slice fits, loaded once and kept
// resident in shared memory (each CTA then keeps one output-channel tile).
// TMA instructions cost a few hundred cycles each on this part whatever
// their size, so the design moves as many bytes per instruction as it can.
// Accumulators live in tensor memory, double buffered so the epilogue of one
// tile overlaps the main loop of the next (persistent CTAs, one per SM).
//
// Warp roles: warp 0 lane 0 issues TMA, warp 1 owns TMEM and lane 0 issues
// tcgen05.mma, warps 2.. run the epilogue (TMEM -> registers -> fused
// bias + requantize -> swizzled smem -> TMA bulk store, or fp32 output with
// direct stores).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "ptx.cuh"

namespace ie_cuda {

enum : int32_t {
  kOutU8 = 0,       // requantized uint8
  kOutS8 = 1,       // requantized int8
  kOutS32 = 2,      // raw int32 accumulator + bias (diagnostics)
  kOutF32 = 3,      // fp32 (+bias, activation), NHWC
  kOutBF16x2 = 4,   // fp32 result split into bf16 hi / lo planes for the next layer
  kOutF32Nchw = 5,  // fp32 (+bias, activation) written straight to NCHW
};

// Error sites recorded in g_device_error when a bounded wait runs out.
enum : unsigned int {
  kErrWaitEmpty = 0x101,
  kErrWaitFull = 0x102,
  kErrWaitAccEmpty = 0x103,
  kErrWaitAccFull = 0x104,
  kErrWaitWeights = 0x105,
  kErrWaitOutFull = 0x106,
  kErrWaitOutFree = 0x107,
  kErrWaitPeak = 0x108,   // mma_i8_peak's final wait
  kErrWaitProbe = 0x1FF,  // the bounded-wait self-test (bounded_wait_probe)
};

constexpr int kMaxStages = 12;

struct IgemmArgs {
  // input NHWC, c = stored channels per pixel
  int32_t n, h, w, c;
  // output NHWC
  int32_t out_h, out_w, m;
  int32_t kh, kw, stride_h, stride_w, dil_h, dil_w, pad_t, pad_l;
  int32_t cblocks;    // channel blocks of BK per tap
  int32_t num_k;      // kh * kw * cblocks
  int32_t k_per_tap;  // packed weight K elements per tap (cblocks * BK elems)
  int32_t stages;     // pipeline depth (<= kMaxStages)
  int32_t out_bufs;   // requantized output: staged tiles in flight (1 or 2)
  int64_t m_total;    // n * out_h * out_w
  int32_t m_tiles, n_tiles;
  // epilogue
  const int32_t* bias_i32;   // int8 path, may be null
  // int8 path, activation zero point zp_x != 0: the A operand holds the raw
  // stored activations (padding materialised as zp_x), and the epilogue adds
  // -zp_x * wsum[ch] (wrapping int32, like the bias) so that the accumulator
  // becomes sum (x - zp_x) * w
  const int32_t* wsum;
  int32_t zp_x;
  const float* bias_f32;     // fp32 path, may be null
  const float* mult;         // int8 path: per-channel requantize multiplier
  int32_t zp_y, qmin, qmax;  // int8 path: output zero point and clamp range
  float act_lo, act_hi;      // fp32 path: clamp range after bias
  const float* residual;     // fp32 path, may be null: added after the bias, before the
                             // clamp (same layout as y: NCHW, or NHWC with y_ld)
  int32_t act;               // fp32 path: 0 = no clamp (NaN propagates)
  int32_t out_mode;
  void* y;
  int64_t y_ld;       // elements between consecutive output pixels
  int64_t acc_bound;  // int8 path: bound on |accumulator| (K * 255 * 128)
  // Row-band mode (int8, stride 1, resident weights): a tile is rows_t whole
  // output rows of a position space whose rows are wp = w + pad_l + pad_r wide,
  // so every filter tap reads the same input band shifted by
  // ky * dil_h * wp + kx * dil_w positions; one tiled TMA load per channel
  // block brings the band (rows_box input rows, padding read as zero) and the
  // taps become shifted MMA operand descriptors.  Positions with
  // ox >= out_w are computed and never stored.
  int32_t halo;
  int32_t wp, rows_t, rows_box, tiles_img;
  int32_t stage_bytes;  // shared memory per stage (band + slack for the shifted reads)
  int32_t band_bytes;   // bytes one band load delivers
  // 1x1, stride 1, no padding: the A operand is the activation tensor itself
  // viewed as a [pixels, channels] matrix, loaded with 2D tiled TMA (rows past
  // the last pixel read as zero) instead of im2col.
  int32_t a_tiled;
  // every bounded wait gives up after this many nanoseconds (kWaitLimitNs)
  uint64_t wait_limit_ns;
};

__host__ __device__ constexpr uint32_t swizzle_layout_code(int row_bytes) {
  return row_bytes == 128 ? 2u : row_bytes == 64 ? 4u : row_bytes == 32 ? 6u : 0u;
}

// ------------------------------------------------------- requantize (int8)
//
// r = round_half_away_from_zero(t * mult) exactly: the fp32 multiplier is the
// dyadic rational mant * 2^-shift with mant its 24-bit significand scaled to
// 31 bits, so the product is one 64-bit integer multiply.  No float
// conversions: those run at a fraction of the integer rate and bounded the
// epilogue.
struct RequantConst {
  int32_t mant;   // signed significand, |mant| in [2^30, 2^31)
  int32_t shift;  // mult = mant * 2^-shift
};

__device__ __forceinline__ RequantConst split_multiplier(float mult) {
  RequantConst k;
  const uint32_t bits = __float_as_uint(mult);
  const int32_t exp_field = static_cast<int32_t>((bits >> 23) & 0xFFu);
  if (exp_field == 0 || exp_field == 0xFF) {
    // zero / denormal (|t * mult| < 2^-94: rounds to 0) / inf / nan
    k.mant = 0;
    k.shift = 32;
    return k;
  }
  const int32_t sig = static_cast<int32_t>(((bits & 0x7FFFFFu) | 0x800000u) << 7);
  k.mant = (bits >> 31) ? -sig : sig;
  // mult = sig24 * 2^(exp_field - 150) = mant * 2^(exp_field - 157)
  k.shift = 157 - exp_field;
  return k;
}

// Exact general path (any shift): floor((p + 2^(s-1) - [p < 0]) / 2^s), then
// zero point and clamp, all in 64-bit.
__device__ __forceinline__ int32_t requant_exact(int32_t t, RequantConst k, int32_t zp,
                                                 int32_t qmin, int32_t qmax) {
  const long long p = static_cast<long long>(t) * k.mant;
  long long r;
  if (k.shift >= 63) {
    r = 0;
  } else if (k.shift <= 0) {
    r = p == 0 ? 0 : (p > 0 ? (1ll << 40) : -(1ll << 40));
  } else {
    r = (p + (1ll << (k.shift - 1)) - (p < 0 ? 1 : 0)) >> k.shift;
  }
  r += zp;
  r = r < qmin ? qmin : r;
  r = r > qmax ? qmax : r;
  return static_cast<int32_t>(r);
}

__device__ __forceinline__ uint32_t pack4_bytes(uint32_t q0, uint32_t q1, uint32_t q2,
                                                uint32_t q3) {
  return __byte_perm(__byte_perm(q0, q1, 0x0040), __byte_perm(q2, q3, 0x0040), 0x5410);
}

// Saturating pack of two int32 values into the low 16 bits (lo_byte first):
// cvt.pack.sat clamps each value to the storage type.
template <bool kS8>
__device__ __forceinline__ uint32_t pack2_sat(int32_t lo_byte, int32_t hi_byte) {
  uint32_t d;
  if constexpr (kS8) {
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(hi_byte), "r"(lo_byte), "r"(0u));
  } else {
    asm("cvt.pack.sat.u8.s32.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(hi_byte), "r"(lo_byte), "r"(0u));
  }
  return d;
}

// Requantize modes of the int8 epilogue, chosen per warp and output-channel
// tile.  The fast modes share one shift S for the warp's columns: each
// channel's significand is aligned to it exactly (mant' = mult * 2^S, an
// integer because mant carries 7 spare low bits and the channel's own shift is
// within 7 of S), and the rounding half and zero point form one warp-uniform
// C = 2^(S-1) + zp * 2^S.  S <= 53 and |zp| <= 255 keep every sum below 2^63.
enum : int {
  // p = acc * mant' + (bias * mant' + C): one 64-bit multiply-add per value
  // with a per-column 64-bit addend.  Valid when zp_y <= qmin (a negative
  // product lands at or below zp, so the sign correction of half-away
  // rounding cannot change the clamped result) and |bias| + |acc| < 2^31
  // (acc + bias does not wrap, so folding it into the addend is exact).
  kReqFold = 0,
  // t = acc + bias (wrapping in int32 like the oracle), p = t * mant' + C -
  // [t < 0]: exact half-away rounding for either sign.  Needs S >= 33 so that
  // C's low word is zero and C - [t < 0] is {lo: t >> 31, hi: (C >> 32) +
  // (t >> 31)}.
  kReqSigned = 1,
  // per-column shift and 64-bit rounding (requant_exact)
  kReqExact = 2,
};

struct EpiQ8 {
  const long long* s_add;  // kReqFold: bias * mant' + C per column
  const int32_t* s_bias;   // kReqSigned / kReqExact (overlays s_add)
  const int32_t* s_shift;  // kReqExact (overlays s_add)
  const int32_t* s_mant;
  int32_t hi_c, shm;       // C >> 32, S - 32
  int32_t zp, lo, hi;
  int lane;
};

// One warp's 32 rows x kCols columns of a requantized tile, TMEM -> the
// CTA's staged output tile (panels of kPanelW bytes x kRows rows, swizzled
// like the TMA store that reads them; row0 / col0 place the warp in the tile).
// The 16x256b TMEM reads give this thread rows r and r + 8 of each 16-row half
// (r = lane / 4) and the column pairs 8j + 2q, 8j + 2q + 1 (q = lane % 4):
// 8 columns per 32-column chunk, whose constants are read from shared memory
// once per chunk and serve all 4 of its rows.  The two 16-row halves of a
// chunk are read one at a time so that one half's TMEM read is in flight
// while the other half is requantized.
template <int kMode, bool kS8, bool kClamp, int kCols, int kRows, int kPanelW>
__device__ __forceinline__ void epi_q8_tile(uint32_t t_q, uint8_t* s_tile, int row0, int col0,
                                            const EpiQ8& e, uint64_t* acce) {
  static_assert(kPanelW == 128 || kPanelW == 64 || kPanelW == 32, "staging panel width");
  const int q4 = e.lane & 3, r8 = e.lane >> 2;
  // TMA's 128 B (64 B, 32 B) swizzle XORs the 16-byte chunk index with
  // row % 8 ((row / 2) % 4, (row / 4) % 2); the rows row0 + 8i + r8 this
  // thread writes all share it.
  const uint32_t xr = kPanelW == 128  ? (r8 << 4)
                      : kPanelW == 64 ? (((r8 >> 1) & 3) << 4)
                                      : (((r8 >> 2) & 1) << 4);
  uint32_t lo_part[4];  // column-within-32 part of the swizzled offset
#pragma unroll
  for (int j = 0; j < 4; ++j) lo_part[j] = (8 * j + 2 * q4) ^ (xr & 0x10u);
  uint8_t* const tb = s_tile + (row0 + r8) * kPanelW;
  uint32_t acc[2][16];  // [16-row half]
  tmem_ld_16x256b_x4(t_q, acc[0]);
  tmem_ld_wait(acc[0]);
#pragma unroll 1
  for (int cc = 0; cc < kCols; cc += 32) {
    const int col = col0 + cc;
    uint8_t* const cb = tb + (col / kPanelW) * (kRows * kPanelW) + ((col % kPanelW) ^ (xr & 0x60u));
    tmem_ld_16x256b_x4(t_q + (16u << 16) + cc, acc[1]);
    // constants of this thread's column pairs 8j + 2q, 8j + 2q + 1
    long long ka[4][2] = {};
    int32_t kb[4][2] = {}, km[4][2] = {};
    if constexpr (kMode != kReqExact) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = cc + 8 * j + 2 * q4;
        const int2 m2 = *reinterpret_cast<const int2*>(e.s_mant + c);
        km[j][0] = m2.x;
        km[j][1] = m2.y;
        if constexpr (kMode == kReqFold) {
          const longlong2 a2 = *reinterpret_cast<const longlong2*>(e.s_add + c);
          ka[j][0] = a2.x;
          ka[j][1] = a2.y;
        } else {
          const int2 b2 = *reinterpret_cast<const int2*>(e.s_bias + c);
          kb[j][0] = b2.x;
          kb[j][1] = b2.y;
        }
      }
    }
    auto half = [&](const uint32_t(&a16)[16], int h) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = cc + 8 * j + 2 * q4;
#pragma unroll
        for (int rs = 0; rs < 2; ++rs) {
          int32_t r[2];
#pragma unroll
          for (int x = 0; x < 2; ++x) {
            const uint32_t a = a16[4 * j + 2 * rs + x];
            if constexpr (kMode == kReqExact) {
              RequantConst k;
              k.mant = e.s_mant[c + x];
              k.shift = e.s_shift[c + x];
              r[x] = requant_exact(static_cast<int32_t>(a + static_cast<uint32_t>(e.s_bias[c + x])),
                                   k, e.zp, e.lo, e.hi);
            } else {
              long long p;
              if constexpr (kMode == kReqFold) {
                p = static_cast<long long>(static_cast<int32_t>(a)) * km[j][x] + ka[j][x];
              } else {
                const int32_t t = static_cast<int32_t>(a + static_cast<uint32_t>(kb[j][x]));
                const int32_t sg = t >> 31;
                const long long cs = static_cast<long long>(
                    (static_cast<unsigned long long>(static_cast<uint32_t>(e.hi_c + sg)) << 32) |
                    static_cast<uint32_t>(sg));
                p = static_cast<long long>(t) * km[j][x] + cs;
              }
              r[x] = static_cast<int32_t>(p >> 32) >> e.shm;
              if constexpr (kClamp) r[x] = min(max(r[x], e.lo), e.hi);
            }
          }
          *reinterpret_cast<uint16_t*>(cb + lo_part[j] + (h * 16 + rs * 8) * kPanelW) =
              static_cast<uint16_t>(pack2_sat<kS8>(r[0], r[1]));
        }
      }
    };
    half(acc[0], 0);
    tmem_ld_wait(acc[1]);
    const bool more = cc + 32 < kCols;
    if (more) {
      tmem_ld_16x256b_x4(t_q + cc + 32, acc[0]);
    } else {
      // Last read of this accumulator buffer by this warp: hand it back so
      // the MMA warp can start the next tile while we finish the epilogue.
      tc_fence_before();
      __syncwarp();
      if (e.lane == 0) mbar_arrive(acce);
    }
    half(acc[1], 1);
    if (more) tmem_ld_wait(acc[0]);
  }
}

// ------------------------------------------------------ fp32 / raw stores

// Processes 32 accumulator columns of one output pixel held by this thread
// with direct global stores (raw int32, and the fp32 output formats).
__device__ __forceinline__ void store_chunk_direct(const IgemmArgs& a, const uint32_t (&acc)[32],
                                                   int64_t pixel, int32_t col0, const int32_t* sb,
                                                   const float* sbf) {
  if (pixel >= a.m_total) return;
  const int32_t valid = a.m - col0;  // channels left in this row
  if (valid <= 0) return;
  if (a.out_mode == kOutS32) {
    int32_t* dst = static_cast<int32_t*>(a.y) + pixel * a.y_ld + col0;
    const int n16 = valid >= 32 ? 8 : (valid + 3) / 4;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      if (q < n16) {
        uint4 v;
        v.x = acc[4 * q + 0] + static_cast<uint32_t>(sb[4 * q + 0]);
        v.y = acc[4 * q + 1] + static_cast<uint32_t>(sb[4 * q + 1]);
        v.z = acc[4 * q + 2] + static_cast<uint32_t>(sb[4 * q + 2]);
        v.w = acc[4 * q + 3] + static_cast<uint32_t>(sb[4 * q + 3]);
        reinterpret_cast<uint4*>(dst)[q] = v;
      }
    }
    return;
  }
  // (acc + bias) [+ residual], then the clamp: one rounding per operation,
  // the order of the reference's Conv2D, Add and Relu nodes
  auto finish = [&](int j, const float* r) {
    float f = __fadd_rn(__uint_as_float(acc[j]), sbf[j]);
    if (r != nullptr) f = __fadd_rn(f, __ldg(r));
    if (a.act) f = fminf(fmaxf(f, a.act_lo), a.act_hi);
    return f;
  };
  auto finish0 = [&](int j) { return finish(j, nullptr); };
  if (a.out_mode == kOutF32) {
    const int64_t off = pixel * a.y_ld + col0;
    float* dst = static_cast<float*>(a.y) + off;
    const int n16 = valid >= 32 ? 8 : (valid + 3) / 4;
    if (a.residual != nullptr) {
      const float* res = a.residual + off;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (q < n16) {
          reinterpret_cast<float4*>(dst)[q] =
              make_float4(finish(4 * q, res + 4 * q), finish(4 * q + 1, res + 4 * q + 1),
                          finish(4 * q + 2, res + 4 * q + 2), finish(4 * q + 3, res + 4 * q + 3));
        }
      }
      return;
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      if (q < n16) {
        reinterpret_cast<float4*>(dst)[q] =
            make_float4(finish0(4 * q), finish0(4 * q + 1), finish0(4 * q + 2), finish0(4 * q + 3));
      }
    }
  } else if (a.out_mode == kOutF32Nchw) {
    // Lanes hold consecutive pixels, so each channel's store is coalesced.
    const int64_t hw = static_cast<int64_t>(a.out_h) * a.out_w;
    const int64_t img = pixel / hw;
    const int64_t off = (img * a.m + col0) * hw + (pixel - img * hw);
    float* dst = static_cast<float*>(a.y) + off;
    const int n = valid >= 32 ? 32 : valid;
    const float* res = a.residual != nullptr ? a.residual + off : nullptr;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j < n) dst[j * hw] = finish(j, res != nullptr ? res + j * hw : nullptr);
    }
  } else {  // kOutBF16x2: [hi plane (y_ld/2) | lo plane (y_ld/2)]
    __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(a.y) + pixel * a.y_ld + col0;
    const int n8 = valid >= 32 ? 4 : (valid + 7) / 8;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (q < n8) {
        uint4 vh, vl;
        uint32_t* ph = reinterpret_cast<uint32_t*>(&vh);
        uint32_t* pl = reinterpret_cast<uint32_t*>(&vl);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float f0 = finish0(8 * q + 2 * j), f1 = finish0(8 * q + 2 * j + 1);
          const __nv_bfloat16 h0 = __float2bfloat16_rn(f0), h1 = __float2bfloat16_rn(f1);
          const __nv_bfloat16 l0 = __float2bfloat16_rn(f0 - __bfloat162float(h0));
          const __nv_bfloat16 l1 = __float2bfloat16_rn(f1 - __bfloat162float(h1));
          ph[j] = static_cast<uint32_t>(__bfloat16_as_ushort(h0)) |
                  (static_cast<uint32_t>(__bfloat16_as_ushort(h1)) << 16);
          pl[j] = static_cast<uint32_t>(__bfloat16_as_ushort(l0)) |
                  (static_cast<uint32_t>(__bfloat16_as_ushort(l1)) << 16);
        }
        reinterpret_cast<uint4*>(dst)[q] = vh;
        reinterpret_cast<uint4*>(dst + a.y_ld / 2)[q] = vl;
      }
    }
  }
}

// ---------------------------------------------------------- smem layout

// Shared memory plan of one kernel variant; the host uses the same numbers to
// size the launch.
template <int BN, int BK_BYTES, int EPI_WARPS, int M_SUB, bool B_RES, bool KIND_I8>
struct IgemmPlan {
  static constexpr int kParts = KIND_I8 ? 1 : 2;  // bf16x3: hi and lo planes
  static constexpr int kRows = 128 * M_SUB;
  static constexpr int kA = kRows * BK_BYTES;
  static constexpr int kB = BN * BK_BYTES;  // one k-step of weights, one plane
  static constexpr int kStage = kParts * (kA + (B_RES ? 0 : kB));
  // Epilogue warps: 4 TMEM lane quarters x M_SUB sub-tiles x kColGroups
  // column groups; each warp covers 32 rows x kWarpCols columns.
  static constexpr int kColGroups = EPI_WARPS / (4 * M_SUB);
  static constexpr int kWarpCols = BN / kColGroups;
  // Requantized int8 output: the epilogue warps stage the whole tile (kRows x
  // BN bytes) as panels kPanelW bytes wide (the widest TMA swizzle is 128 B);
  // the store warp writes it with one TMA store per panel.
  static constexpr int kPanelW = BN < 128 ? BN : 128;
  static constexpr int kPanels = BN / kPanelW;
  static constexpr int kOutTile = KIND_I8 ? kRows * BN : 0;
  // per epilogue warp: per-column bias, significand and shift
  static constexpr int kConstBytes = EPI_WARPS * kWarpCols * 12;
  static constexpr int kBarBytes = 8 * (2 * kMaxStages + 10) + 32;
  static constexpr int kAccCols = M_SUB * BN;
  static constexpr uint32_t kTmemCols = 2 * kAccCols <= 64    ? 64
                                        : 2 * kAccCols <= 128 ? 128
                                        : 2 * kAccCols <= 256 ? 256
                                                              : 512;
  static_assert(2 * kAccCols <= 512, "double-buffered accumulator exceeds TMEM");
  static_assert(kColGroups >= 1 && EPI_WARPS == 4 * M_SUB * kColGroups, "epilogue warps");
  static_assert(kWarpCols >= 32 && kWarpCols % 32 == 0, "epilogue columns per warp");
  // dynamic smem for `stages` pipeline stages and `num_k` resident weight steps
  // stage_bytes: kStage, or the row-band mode's per-stage size
  static constexpr int bytes(int stages, int num_k, int out_bufs, int stage_bytes) {
    return 1024 + stages * stage_bytes + (B_RES ? kParts * num_k * kB : 0) + out_bufs * kOutTile +
           kConstBytes + kBarBytes;
  }
};

// --------------------------------------------------------------- kernel
//
// KIND_I8: int8 x int8 -> s32 (A signedness by template).
// !KIND_I8: bf16x3 for fp32 data.  The activation tensor stores each pixel as
//          [hi plane (C) | lo plane (C)] bf16 and the packed weights store per
//          tap [hi (Ck) | lo (Ck)]; every K block issues A_hi*B_hi, A_hi*B_lo
//          and A_lo*B_hi into the same f32 accumulator.
template <int BN, int BK_BYTES, int EPI_WARPS, int M_SUB, bool B_RES, bool KIND_I8, bool A_SIGNED>
__global__ void __launch_bounds__(96 + EPI_WARPS * 32, 1)
    conv_igemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                      const __grid_constant__ CUtensorMap tmap_b,
                      const __grid_constant__ CUtensorMap tmap_y, const IgemmArgs args) {
  using P = IgemmPlan<BN, BK_BYTES, EPI_WARPS, M_SUB, B_RES, KIND_I8>;
  constexpr int kParts = P::kParts;
  constexpr int kA = P::kA;
  constexpr int kB = P::kB;
  constexpr int kStage = P::kStage;
  constexpr int kWarpCols = P::kWarpCols;
  constexpr uint32_t kLayout = swizzle_layout_code(BK_BYTES);
  constexpr uint32_t kSbo = 8 * BK_BYTES;  // 8 rows of BK bytes per swizzle atom
  constexpr int kKStep = 32;               // bytes of K per MMA instruction
  constexpr int kElemBytes = KIND_I8 ? 1 : 2;
  constexpr int kBkElems = BK_BYTES / kElemBytes;
  constexpr uint32_t kIdesc =
      KIND_I8 ? make_idesc_i8(128, BN, A_SIGNED, true) : make_idesc_bf16(128, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int stages = args.stages;
  const bool halo = KIND_I8 && B_RES && args.halo != 0;
  const int stage_bytes = halo ? args.stage_bytes : kStage;
  uint8_t* stage_base = smem;
  uint8_t* b_res = stage_base + stages * stage_bytes;  // resident weights (B_RES)
  uint8_t* out_stage = b_res + (B_RES ? kParts * args.num_k * kB : 0);  // [out_bufs]
  uint8_t* const_base = out_stage + args.out_bufs * P::kOutTile;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(const_base + P::kConstBytes);
  uint64_t* empty_bar = full_bar + kMaxStages;
  uint64_t* accf_bar = empty_bar + kMaxStages;  // [2]
  uint64_t* acce_bar = accf_bar + 2;            // [2]
  uint64_t* drain_bar = acce_bar + 2;           // [1]
  uint64_t* bres_bar = drain_bar + 1;           // [1]
  uint64_t* ofull_bar = bres_bar + 1;           // [2] staged output tile written
  uint64_t* ofree_bar = ofull_bar + 2;          // [2] staged output tile read by its store
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ofree_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint32_t* kiter_issued = tmem_slot + 2;
  uint32_t* kiter_consumed = tmem_slot + 3;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Tile j of this CTA -> (m_tile, n_tile).  With resident weights each CTA
  // keeps one n_tile (the grid is a multiple of n_tiles); otherwise tiles are
  // dealt round-robin with n fastest, so CTAs running together share A in L2.
  const int cta_n = B_RES ? static_cast<int>(blockIdx.x) % args.n_tiles : 0;
  const int cta_m0 = B_RES ? static_cast<int>(blockIdx.x) / args.n_tiles : 0;
  const int m_step = B_RES ? static_cast<int>(gridDim.x) / args.n_tiles : 0;
  const int num_tiles = args.m_tiles * args.n_tiles;
  auto tile_of = [&](int j, int* m_tile, int* n_tile) -> bool {
    if constexpr (B_RES) {
      *n_tile = cta_n;
      *m_tile = cta_m0 + j * m_step;
      return *m_tile < args.m_tiles;
    } else {
      const int t = static_cast<int>(blockIdx.x) + j * static_cast<int>(gridDim.x);
      *n_tile = t % args.n_tiles;
      *m_tile = t / args.n_tiles;
      return t < num_tiles;
    }
  };

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    tma_prefetch_desc(&tmap_y);
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf_bar[b], 1);
      mbar_init(&acce_bar[b], EPI_WARPS);
    }
    mbar_init(drain_bar, 1);
    mbar_init(bres_bar, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ofull_bar[b], EPI_WARPS);
      mbar_init(&ofree_bar[b], 1);
    }
    *abort_flag = 0;
    *kiter_issued = 0;
    *kiter_consumed = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, P::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // The next layer's kernel may be scheduled now; it waits for this one to
  // complete before it reads anything this one writes.
  grid_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      if constexpr (B_RES) {
        // The CTA's whole weight slice, once.
        mbar_arrive_expect_tx(bres_bar, kParts * args.num_k * kB);
        for (int k = 0; k < args.num_k; ++k) {
          const int tap = k / args.cblocks;
          const int cb = k - tap * args.cblocks;
          const int32_t kcoord = tap * args.k_per_tap * kParts + cb * kBkElems;
          tma_load_2d(b_res + k * kParts * kB, &tmap_b, bres_bar, kcoord, cta_n * BN);
          if constexpr (!KIND_I8) {
            tma_load_2d(b_res + k * kParts * kB + kB, &tmap_b, bres_bar, kcoord + args.k_per_tap,
                        cta_n * BN);
          }
        }
      }
      // The weights above are constants; the activations may come from the
      // kernel launched just before this one.
      grid_dependency_wait();
      const int32_t hw_out = args.out_h * args.out_w;
      uint32_t kiter = 0;
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      int m_tile, n_tile;
      for (int j = 0; ok && tile_of(j, &m_tile, &n_tile); ++j) {
        if constexpr (KIND_I8 && B_RES) {
          if (halo) {
            const int32_t img = m_tile / args.tiles_img;
            const int32_t oy0 = (m_tile - img * args.tiles_img) * args.rows_t;
            for (int cb = 0; cb < args.cblocks; ++cb, ++kiter) {
              if (!mbar_wait(&empty_bar[s], ph ^ 1u, abort_flag, kErrWaitEmpty, args.wait_limit_ns)) {
                ok = false;
                break;
              }
              uint8_t* st = stage_base + s * stage_bytes;
              mbar_arrive_expect_tx(&full_bar[s], args.band_bytes);
              tma_load_4d(st, &tmap_a, &full_bar[s], cb * kBkElems, -args.pad_l,
                          oy0 - args.pad_t, img);
              if (++s == stages) {
                s = 0;
                ph ^= 1u;
              }
            }
            continue;
          }
        }
        const int64_t p0 = static_cast<int64_t>(m_tile) * P::kRows;
        const int32_t img = static_cast<int32_t>(p0 / hw_out);
        const int32_t rem = static_cast<int32_t>(p0 - static_cast<int64_t>(img) * hw_out);
        const int32_t oy = rem / args.out_w, ox = rem - (rem / args.out_w) * args.out_w;
        const int32_t wc = ox * args.stride_w - args.pad_l;
        const int32_t hc = oy * args.stride_h - args.pad_t;
        const int32_t co0 = n_tile * BN;
        int tap = 0, cb = 0, ky = 0, kx = 0;
        for (int k = 0; k < args.num_k; ++k, ++kiter) {
          if (!mbar_wait(&empty_bar[s], ph ^ 1u, abort_flag, kErrWaitEmpty, args.wait_limit_ns)) {
            ok = false;
            break;
          }
          uint8_t* st = stage_base + s * stage_bytes;
          mbar_arrive_expect_tx(&full_bar[s], kStage);
          if (args.a_tiled) {
            tma_load_2d(st, &tmap_a, &full_bar[s], cb * kBkElems, static_cast<int32_t>(p0));
            if constexpr (!KIND_I8) {
              tma_load_2d(st + kA, &tmap_a, &full_bar[s], args.c + cb * kBkElems,
                          static_cast<int32_t>(p0));
            }
          } else {
            const uint16_t offw = static_cast<uint16_t>(kx * args.dil_w);
            const uint16_t offh = static_cast<uint16_t>(ky * args.dil_h);
            tma_load_im2col_4d(st, &tmap_a, &full_bar[s], cb * kBkElems, wc, hc, img, offw, offh);
            if constexpr (!KIND_I8) {
              // lo plane: activation channels [c, 2c)
              tma_load_im2col_4d(st + kA, &tmap_a, &full_bar[s], args.c + cb * kBkElems, wc, hc,
                                 img, offw, offh);
            }
          }
          if constexpr (!B_RES) {
            const int32_t kcoord = tap * args.k_per_tap * kParts + cb * kBkElems;
            tma_load_2d(st + kParts * kA, &tmap_b, &full_bar[s], kcoord, co0);
            if constexpr (!KIND_I8) {
              tma_load_2d(st + kParts * kA + kB, &tmap_b, &full_bar[s], kcoord + args.k_per_tap,
                          co0);
            }
          }
          if (++s == stages) {
            s = 0;
            ph ^= 1u;
          }
          if (++cb == args.cblocks) {
            cb = 0;
            ++tap;
            if (++kx == args.kw) {
              kx = 0;
              ++ky;
            }
          }
        }
      }
      *kiter_issued = kiter;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      // Operand descriptors are built once per buffer and advanced by adding
      // (byte offset >> 4) to their address field (shared-memory addresses
      // stay below 2^18, so the 14-bit field never carries).
      uint32_t kiter = 0;
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      if constexpr (B_RES) {
        ok = mbar_wait(bres_bar, 0, abort_flag, kErrWaitWeights, args.wait_limit_ns);
      }
      const uint64_t stage_desc0 = make_smem_desc(smem_u32(stage_base), 16, kSbo, kLayout);
      const uint64_t bres_desc0 = make_smem_desc(smem_u32(b_res), 16, kSbo, kLayout);
      int m_tile, n_tile;
      for (int j = 0; ok && tile_of(j, &m_tile, &n_tile); ++j) {
        const int buf = j & 1;
        const uint32_t aph = (j >> 1) & 1;
        if (!mbar_wait(&acce_bar[buf], aph ^ 1u, abort_flag, kErrWaitAccEmpty, args.wait_limit_ns)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * P::kAccCols;
        if constexpr (KIND_I8 && B_RES) {
          if (halo) {
            // Tap (ky, kx) reads the band shifted by ky * dil_h * wp + kx *
            // dil_w rows.  Such a start is in general not a multiple of 8
            // rows: the tensor core applies the swizzle XOR from the absolute
            // shared-memory address bits, as the TMA unit wrote them, so the
            // plain start address places the operand (matrix base offset 0;
            // measured on B200 for the 32-, 64- and 128-byte swizzles, at
            // full MMA rate).
            const int taps = args.kh * args.kw;
            const int row_jump = args.dil_h * args.wp - args.kw * args.dil_w;
            const uint64_t tap_b_step = static_cast<uint64_t>(args.cblocks * kB) >> 4;
            for (int cb = 0; cb < args.cblocks; ++cb, ++kiter) {
              if (!mbar_wait(&full_bar[s], ph, abort_flag, kErrWaitFull, args.wait_limit_ns)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint64_t a_st = stage_desc0 + (static_cast<uint64_t>(s * stage_bytes) >> 4);
              uint64_t b_tap = bres_desc0 + (static_cast<uint64_t>(cb * kB) >> 4);
              int shift = 0, kx = 0;
              for (int tap = 0; tap < taps; ++tap) {
                const uint64_t a_tap = a_st + static_cast<uint64_t>(shift * (BK_BYTES / 16));
#pragma unroll
                for (int kk = 0; kk < BK_BYTES / kKStep; ++kk) {
#pragma unroll
                  for (int sub = 0; sub < M_SUB; ++sub) {
                    mma_i8(d_tmem + sub * BN, a_tap + ((sub * 128 * BK_BYTES + kk * kKStep) >> 4),
                           b_tap + ((kk * kKStep) >> 4), kIdesc, kk != 0 || ((cb | tap) != 0));
                  }
                }
                b_tap += tap_b_step;
                shift += args.dil_w;
                if (++kx == args.kw) {
                  kx = 0;
                  shift += row_jump;
                }
              }
              tc_commit(&empty_bar[s]);
              if (++s == stages) {
                s = 0;
                ph ^= 1u;
              }
            }
            if (ok) tc_commit(&accf_bar[buf]);
            continue;
          }
        }
        for (int k = 0; k < args.num_k; ++k, ++kiter) {
          if (!mbar_wait(&full_bar[s], ph, abort_flag, kErrWaitFull, args.wait_limit_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t a_st = stage_desc0 + (static_cast<uint64_t>(s * stage_bytes) >> 4);
          const uint64_t b_k = B_RES ? bres_desc0 + (static_cast<uint64_t>(k * kParts * kB) >> 4)
                                     : a_st + ((kParts * kA) >> 4);
#pragma unroll
          for (int kk = 0; kk < BK_BYTES / kKStep; ++kk) {
            const uint64_t bd = b_k + ((kk * kKStep) >> 4);
#pragma unroll
            for (int sub = 0; sub < M_SUB; ++sub) {
              const uint64_t ad = a_st + ((sub * 128 * BK_BYTES + kk * kKStep) >> 4);
              const uint32_t d = d_tmem + sub * BN;
              if constexpr (KIND_I8) {
                mma_i8(d, ad, bd, kIdesc, (k | kk) != 0);
              } else {
                const uint64_t adl = ad + (kA >> 4);
                const uint64_t bdl = bd + (kB >> 4);
                mma_f16(d, ad, bd, kIdesc, (k | kk) != 0);
                mma_f16(d, ad, bdl, kIdesc, 1);
                mma_f16(d, adl, bd, kIdesc, 1);
              }
            }
          }
          tc_commit(&empty_bar[s]);  // frees the stage once these MMAs finish
          if (++s == stages) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (ok) tc_commit(&accf_bar[buf]);
      }
      *kiter_consumed = kiter;
      // Drain: every MMA issued above has finished once this barrier flips, so
      // tensor memory can be released safely even on the abort path.
      tc_commit(drain_bar);
      int dummy_abort = 0;
      mbar_wait(drain_bar, 0, &dummy_abort, kErrWaitFull, args.wait_limit_ns);
    }
  } else if (warp == 2 + EPI_WARPS) {
    // ------------------------------------------------ output store warp
    // One TMA store per panel of each staged tile, so the TMA unit sees
    // kPanels stores per tile rather than one per epilogue warp.
    const bool tma_out = KIND_I8 && (args.out_mode == kOutU8 || args.out_mode == kOutS8);
    if (tma_out && lane == 0) {
      int m_tile, n_tile;
      for (int j = 0; tile_of(j, &m_tile, &n_tile); ++j) {
        const int ob = args.out_bufs == 2 ? (j & 1) : 0;
        const uint32_t oph = args.out_bufs == 2 ? ((j >> 1) & 1) : (j & 1);
        if (!mbar_wait(&ofull_bar[ob], oph, abort_flag, kErrWaitOutFull, args.wait_limit_ns)) break;
        const uint8_t* s_tile = out_stage + ob * P::kOutTile;
        const int32_t row0 = m_tile * P::kRows;
        const int32_t img = halo ? m_tile / args.tiles_img : 0;
        const int32_t oy0 = halo ? (m_tile - img * args.tiles_img) * args.rows_t : 0;
#pragma unroll
        for (int p = 0; p < P::kPanels; ++p) {
          const int32_t col = n_tile * BN + p * P::kPanelW;
          if (col >= args.y_ld) continue;
          const uint8_t* panel = s_tile + p * P::kRows * P::kPanelW;
          if (halo) {
            // rows_t x wp positions; columns ox >= out_w fall outside the
            // tensor and are not written
            tma_store_4d(&tmap_y, panel, col, 0, oy0, img);
          } else {
            tma_store_2d(&tmap_y, panel, col, row0);
          }
        }
        bulk_commit_group();
        bulk_wait_group_read0();  // the staged tile may be overwritten
        mbar_arrive(&ofree_bar[ob]);
      }
      bulk_wait_group0();
    }
  } else {
    // ------------------------------------------------ epilogue warps
    grid_dependency_wait();  // a residual input may come from the previous kernel
    const int ew = warp - 2;       // 0 .. EPI_WARPS-1
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int idx = ew / 4;
    const int sub = idx / P::kColGroups;
    const int col_lo = (idx % P::kColGroups) * kWarpCols;
    // 12 bytes of constants per column: kReqFold's 64-bit addends overlay
    // bias + shift (fp32 bias in the bf16 path), then the significands
    uint8_t* s_const = const_base + ew * kWarpCols * 12;
    long long* s_add = reinterpret_cast<long long*>(s_const);
    int32_t* s_bias = reinterpret_cast<int32_t*>(s_const);
    int32_t* s_shift = s_bias + kWarpCols;
    int32_t* s_mant = reinterpret_cast<int32_t*>(s_const + 8 * kWarpCols);
    const bool tma_out = KIND_I8 && (args.out_mode == kOutU8 || args.out_mode == kOutS8);
    const bool y_s8 = args.out_mode == kOutS8;
    const bool sign_free = args.zp_y <= args.qmin;  // negative products clamp to qmin
    // clamp range equal to the storage type: the saturating pack is the clamp
    const bool clamp_free = args.qmin == (y_s8 ? -128 : 0) && args.qmax == (y_s8 ? 127 : 255);
    int loaded_n_tile = -1;
    int req_mode = kReqExact;
    EpiQ8 eq;
    eq.s_add = s_add;
    eq.s_bias = s_bias;
    eq.s_mant = s_mant;
    eq.s_shift = s_shift;
    eq.hi_c = eq.shm = 0;
    eq.zp = args.zp_y;
    eq.lo = args.qmin;
    eq.hi = args.qmax;
    eq.lane = lane;
    int m_tile, n_tile;
    for (int j = 0; tile_of(j, &m_tile, &n_tile); ++j) {
      const int buf = j & 1;
      const uint32_t aph = (j >> 1) & 1;
      const int32_t wcol0 = n_tile * BN + col_lo;  // first output channel of this warp
      if (n_tile != loaded_n_tile) {
        __syncwarp();
        if constexpr (KIND_I8) {
          // per-column constants; the warp's common shift S is the smallest
          // one (largest multiplier), every other significand shifts right by
          // shift_c - S <= 7 bits, exactly (its 7 low bits are zero)
          RequantConst rc[kWarpCols / 32];
          int32_t bias[kWarpCols / 32];
          int32_t smin = 1 << 20;
          bool fast = true, bias_fits = true;
#pragma unroll
          for (int r = 0; r < kWarpCols / 32; ++r) {
            const int32_t ch = wcol0 + lane + 32 * r;
            const bool in = ch < args.m;
            bias[r] = (in && args.bias_i32 != nullptr) ? __ldg(args.bias_i32 + ch) : 0;
            if (in && args.zp_x != 0) {
              bias[r] = static_cast<int32_t>(static_cast<uint32_t>(bias[r]) -
                                             static_cast<uint32_t>(args.zp_x) *
                                                 static_cast<uint32_t>(__ldg(args.wsum + ch)));
            }
            rc[r] = split_multiplier((in && args.mult != nullptr) ? __ldg(args.mult + ch) : 0.0f);
            if (rc[r].mant != 0) smin = min(smin, rc[r].shift);
            fast = fast && rc[r].mant >= 0;
            const long long b = bias[r];
            bias_fits = bias_fits && (b < 0 ? -b : b) + args.acc_bound < (1ll << 31);
          }
          // the common shift S is the smallest one (largest multiplier); every
          // other significand shifts right by shift_c - S <= 7 bits, exactly
          smin = __reduce_min_sync(0xFFFFFFFFu, smin);
          if (smin == (1 << 20)) smin = 33;  // all multipliers zero: any S works
#pragma unroll
          for (int r = 0; r < kWarpCols / 32; ++r) {
            if (rc[r].mant != 0 && rc[r].shift - smin > 7) fast = false;
          }
          fast = __all_sync(0xFFFFFFFFu, fast) && smin >= 32 && smin <= 53;
          bias_fits = __all_sync(0xFFFFFFFFu, bias_fits);
          // raw int32 output reads the plain bias: exact mode's layout
          req_mode = !tma_out ? kReqExact
                              : (fast && sign_free && bias_fits)
                                    ? kReqFold
                                    : ((fast && smin >= 33) ? kReqSigned : kReqExact);
          const long long c_add =
              (1ll << (smin - 1)) + static_cast<long long>(args.zp_y) * (1ll << smin);
#pragma unroll
          for (int r = 0; r < kWarpCols / 32; ++r) {
            const int c = lane + 32 * r;
            const int32_t m_al = (req_mode != kReqExact && rc[r].mant != 0)
                                     ? (rc[r].mant >> (rc[r].shift - smin)) : 0;
            if (req_mode == kReqFold) {
              s_add[c] = static_cast<long long>(bias[r]) * m_al + c_add;
              s_mant[c] = m_al;
            } else {
              s_bias[c] = bias[r];
              if (req_mode == kReqSigned) {
                s_mant[c] = m_al;
              } else {
                s_mant[c] = rc[r].mant;
                s_shift[c] = rc[r].shift;
              }
            }
          }
          eq.hi_c = static_cast<int32_t>(c_add >> 32);
          eq.shm = smin - 32;
        } else {
          for (int c = lane; c < kWarpCols; c += 32) {
            const int32_t ch = wcol0 + c;
            const bool in = ch < args.m;
            s_bias[c] = __float_as_int((in && args.bias_f32 != nullptr)
                                           ? __ldg(args.bias_f32 + ch) : 0.0f);
          }
        }
        loaded_n_tile = n_tile;
        __syncwarp();
      }
      if (!mbar_wait_warp(&accf_bar[buf], aph, abort_flag, kErrWaitAccFull, args.wait_limit_ns)) break;
      tc_fence_after();
      const int64_t row0 = static_cast<int64_t>(m_tile) * P::kRows + sub * 128 + quarter * 32;
      const int64_t pixel = row0 + lane;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             buf * P::kAccCols + sub * BN + col_lo;
      if (tma_out) {
        // the staged tile buffer is free once its previous store has read it
        const int ob = args.out_bufs == 2 ? (j & 1) : 0;
        const uint32_t oph = args.out_bufs == 2 ? ((j >> 1) & 1) : (j & 1);
        if (!mbar_wait_warp(&ofree_bar[ob], oph ^ 1u, abort_flag, kErrWaitOutFree, args.wait_limit_ns)) break;
        uint8_t* s_tile = out_stage + ob * P::kOutTile;
        const int r0 = sub * 128 + quarter * 32;
        const uint32_t t_q = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             buf * P::kAccCols + sub * BN + col_lo;
        uint64_t* ae = &acce_bar[buf];
        constexpr int W = kWarpCols, R = P::kRows, Z = P::kPanelW;
        switch (req_mode * 4 + (y_s8 ? 2 : 0) + (clamp_free ? 0 : 1)) {
          case 0: epi_q8_tile<kReqFold, false, false, W, R, Z>(t_q, s_tile, r0, col_lo, eq, ae); break;
          case 1: epi_q8_tile<kReqFold, false, true, W, R, Z>(t_q, s_tile, r0, col_lo, eq, ae); break;
          case 2: epi_q8_tile<kReqFold, true, false, W, R, Z>(t_q, s_tile, r0, col_lo, eq, ae); break;
          case 3: epi_q8_tile<kReqFold, true, true, W, R, Z>(t_q, s_tile, r0, col_lo, eq, ae); break;
          case 4: epi_q8_tile<kReqSigned, false, false, W, R, Z>(t_q, s_tile, r0, col_lo, eq, ae); break;
          case 5: epi_q8_tile<kReqSigned, false, true, W, R, Z>(t_q, s_tile, r0, col_lo, eq, ae); break;
          case 6: epi_q8_tile<kReqSigned, true, false, W, R, Z>(t_q, s_tile, r0, col_lo, eq, ae); break;
          case 7: epi_q8_tile<kReqSigned, true, true, W, R, Z>(t_q, s_tile, r0, col_lo, eq, ae); break;
          case 8:
          case 9: epi_q8_tile<kReqExact, false, false, W, R, Z>(t_q, s_tile, r0, col_lo, eq, ae); break;
          default: epi_q8_tile<kReqExact, true, false, W, R, Z>(t_q, s_tile, r0, col_lo, eq, ae); break;
        }
        fence_proxy_async_smem();  // generic-proxy smem writes -> visible to the TMA unit
        __syncwarp();
        if (lane == 0) mbar_arrive(&ofull_bar[ob]);
        continue;
      }
#pragma unroll 1
      for (int cc = 0; cc < kWarpCols; cc += 32) {
        uint32_t acc[32];
        tmem_ld_32x32b_x32(t_row + cc, acc);
        tmem_ld_wait();
        if (cc + 32 >= kWarpCols) {
          // Last read of this accumulator buffer by this warp: hand it back so
          // the MMA warp can start the next tile while we finish the epilogue.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acce_bar[buf]);
        }
        {
          int32_t sb[32];
          float sbf[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            sb[e] = KIND_I8 ? s_bias[cc + e] : 0;
            sbf[e] = KIND_I8 ? 0.0f : __int_as_float(s_bias[cc + e]);
          }
          store_chunk_direct(args, acc, pixel, wcol0 + cc, sb, sbf);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag && threadIdx.x == 0) {
    // Loads issued but never consumed are still landing in shared memory:
    // wait for them (bounded) before the CTA exits.
    int dummy_abort = 0;
    for (uint32_t k = *kiter_consumed; k < *kiter_issued; ++k) {
      mbar_wait(&full_bar[k % stages], (k / stages) & 1u, &dummy_abort, kErrWaitFull, args.wait_limit_ns);
    }
    if (B_RES) mbar_wait(bres_bar, 0, &dummy_abort, kErrWaitWeights, args.wait_limit_ns);
  }
  if (warp == 1) {
    tc_fence_after();
    __syncwarp();
    tmem_dealloc(tmem_base, P::kTmemCols);
  }
}

// Self-test of the bounded-wait path: one CTA allocates tensor memory, then
// thread 0 waits on an mbarrier that nothing ever arrives on.  The wait gives
// up after limit_ns, records kErrWaitProbe in the device error word and
// raises the CTA's abort flag; the CTA then frees its tensor memory and
// returns, exactly as the convolution kernel winds down when one of its waits
// runs out.  out[0] = 1 if the wait (wrongly) completed, 2 if it gave up,
// out[1] = nanoseconds waited.
__global__ void __launch_bounds__(64, 1) bounded_wait_probe(uint64_t limit_ns, uint64_t* out) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0) {
    const uint64_t t0 = globaltimer_ns();
    const bool ok = mbar_wait(&bar, 0, &abort_flag, kErrWaitProbe, limit_ns);
    out[0] = ok ? 1 : 2;
    out[1] = globaltimer_ns() - t0;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    __syncwarp();
    tmem_dealloc(tmem_slot, 32);
  }
}

// Rate of the int8 tensor cores on this GPU: every CTA (one per SM) issues
// `iters` back-to-back tcgen05.mma kind::i8 of M=128, N=256, K=32 from one
// thread into one tensor-memory accumulator, its operands a zeroed 128 x 32 B
// A and 256 x 32 B B tile in shared memory (32-byte rows, 32-byte swizzle: the
// operand form the implicit GEMM uses for 32-byte channel blocks).  One
// commit, a bounded wait for it, then the accumulator is freed.  The host
// times the launch: 2 * 128 * 256 * 32 * iters ops per CTA.
__global__ void __launch_bounds__(128, 1) mma_i8_peak(uint32_t iters, uint64_t wait_limit_ns) {
  __shared__ __align__(1024) uint8_t ops[128 * 32 + 256 * 32];
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < static_cast<int>(sizeof(ops) / 16); i += blockDim.x) {
    reinterpret_cast<uint4*>(ops)[i] = make_uint4(0u, 0u, 0u, 0u);
  }
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  fence_proxy_async_smem();  // the zeroed operands -> visible to the tensor core
  if (warp == 1) {
    tmem_alloc(&tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  if (threadIdx.x == 0) {
    const uint64_t a = make_smem_desc(smem_u32(ops), 16, 8 * 32, swizzle_layout_code(32));
    const uint64_t b = make_smem_desc(smem_u32(ops + 128 * 32), 16, 8 * 32, swizzle_layout_code(32));
    constexpr uint32_t kIdesc = make_idesc_i8(128, 256, false, true);
    for (uint32_t i = 0; i < iters; ++i) mma_i8(tmem, a, b, kIdesc, i != 0 ? 1u : 0u);
    tc_commit(&bar);
    mbar_wait(&bar, 0, &abort_flag, kErrWaitPeak, wait_limit_ns);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    __syncwarp();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace ie_cuda
