// Implicit-GEMM convolution on tcgen05 tensor cores (sm_100a).
//
// GEMM view of an NHWC convolution (the reference computes the same sums as
// im2col + one row GEMM per output channel, conv2d_op.cpp:189-241):
//   rows    = output pixels p = (n, oy, ox), flattened, 128 per tile
//   columns = output channels, BN per tile
//   K       = (tap = ky*kW + kx, channel block of BK bytes)
// A tiles come straight from the NHWC activation tensor through TMA im2col
// loads (one load per tap and channel block; padding and image edges read as
// zero), B tiles from the K-major packed weights through 2D tiled TMA loads.
// Accumulators live in tensor memory, double buffered so the epilogue of one
// tile overlaps the main loop of the next (persistent CTAs, one per SM).
//
// Warp roles: warp 0 lane 0 issues TMA, warp 1 owns TMEM and lane 0 issues
// tcgen05.mma, warps 2.. run the epilogue (TMEM -> registers -> fused
// bias / requantize or fp32 output -> 128-bit global stores).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "ptx.cuh"

namespace ie_cuda {

enum : int32_t {
  kOutU8 = 0,      // requantized uint8
  kOutS8 = 1,      // requantized int8
  kOutS32 = 2,     // raw int32 accumulator + bias (diagnostics)
  kOutF32 = 3,     // fp32 (+bias, activation)
  kOutBF16x2 = 4,  // fp32 result split into bf16 hi / lo planes for the next layer
  kOutF32Nchw = 5, // fp32 (+bias, activation) written straight to NCHW
};

// Error sites recorded in g_device_error when a bounded wait runs out.
enum : unsigned int {
  kErrWaitEmpty = 0x101,
  kErrWaitFull = 0x102,
  kErrWaitAccEmpty = 0x103,
  kErrWaitAccFull = 0x104,
};

struct IgemmArgs {
  // input NHWC, c = stored channels per pixel
  int32_t n, h, w, c;
  // output NHWC
  int32_t out_h, out_w, m;
  int32_t kh, kw, stride_h, stride_w, dil_h, dil_w, pad_t, pad_l;
  int32_t cblocks;    // channel blocks of BK per tap
  int32_t num_k;      // kh * kw * cblocks (x3 for the bf16x3 path: see kSplit)
  int32_t k_per_tap;  // packed weight K elements per tap (cblocks * BK elems)
  int64_t m_total;    // n * out_h * out_w
  int32_t m_tiles, n_tiles;
  // epilogue
  const int32_t* bias_i32;  // int8 path, may be null
  const float* bias_f32;    // fp32 path, may be null
  const float* mult;        // int8 path: per-channel requantize multiplier
  int32_t zp_y, lo, hi;     // int8 path: clamp range minus zp_y
  float act_lo, act_hi;     // fp32 path: clamp range after bias
  int32_t out_mode;
  void* y;
  int64_t y_ld;  // elements between consecutive output pixels
};

// Number of bytes one pipeline stage holds.
template <int BN, int BK_BYTES>
struct IgemmSmem {
  static constexpr int kA = 128 * BK_BYTES;
  static constexpr int kB = BN * BK_BYTES;
  static constexpr int kStage = kA + kB;
};

__host__ __device__ constexpr uint32_t swizzle_layout_code(int row_bytes) {
  return row_bytes == 128 ? 2u : row_bytes == 64 ? 4u : row_bytes == 32 ? 6u : 0u;
}

// ------------------------------------------------------------- epilogue

// round-half-away-from-zero of v, as a float whose truncation is the result:
// adding copysign(0.5, v) with round-toward-zero and truncating gives
// floor(|v| + 0.5) * sign(v) exactly for every finite fp32 v (the directed
// rounding keeps |v| = 0.5 - 2^-25 from rounding the sum up to 1.0).
__device__ __forceinline__ float round_away_pre_trunc(float v) {
  const float half = __int_as_float((__float_as_int(v) & 0x80000000) | 0x3f000000);
  return __fadd_rz(v, half);
}

__device__ __forceinline__ uint32_t cvt_trunc_sat_u8(float x) {
  uint32_t r;
  asm("cvt.rzi.sat.u8.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ uint32_t cvt_trunc_sat_s8(float x) {
  uint32_t r;
  asm("cvt.rzi.sat.s8.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r & 0xFFu;
}

// Requantizes 4 accumulators into 4 packed output bytes.
//   kFast: zp_y == 0 and the clamp range is the whole storage type, so the
//          saturating conversion is the clamp.
template <bool kFast, bool kSigned>
__device__ __forceinline__ uint32_t requant_pack4(const uint32_t* acc, int4 b4, float4 m4,
                                                  int32_t zp, int32_t qmin, int32_t qmax) {
  const int32_t bb[4] = {b4.x, b4.y, b4.z, b4.w};
  const float mm[4] = {m4.x, m4.y, m4.z, m4.w};
  uint32_t q[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int32_t t = static_cast<int32_t>(acc[j] + static_cast<uint32_t>(bb[j]));
    const float x = round_away_pre_trunc(__fmul_rn(__int2float_rn(t), mm[j]));
    if constexpr (kFast) {
      q[j] = kSigned ? cvt_trunc_sat_s8(x) : cvt_trunc_sat_u8(x);
    } else {
      int32_t v = __float2int_rz(x) + zp;
      v = min(max(v, qmin), qmax);
      q[j] = static_cast<uint32_t>(v) & 0xFFu;
    }
  }
  return __byte_perm(__byte_perm(q[0], q[1], 0x0040), __byte_perm(q[2], q[3], 0x0040), 0x5410);
}


__device__ __forceinline__ uint32_t requant4(const uint32_t* acc, const int32_t* sb,
                                             const float* sm, int32_t zp, float lo, float hi,
                                             bool out_signed) {
  uint32_t packed = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int32_t t = static_cast<int32_t>(acc[j] + static_cast<uint32_t>(sb[j]));
    float r = roundf(__fmul_rn(__int2float_rn(t), sm[j]));
    r = fminf(fmaxf(r, lo), hi);
    const int32_t q = __float2int_rz(r) + zp;
    packed |= (static_cast<uint32_t>(q) & 0xFFu) << (8 * j);
  }
  (void)out_signed;
  return packed;
}

// Processes 32 accumulator columns of one output pixel held by this thread.
template <bool kIsF32Acc>
__device__ __forceinline__ void epilogue_chunk(const IgemmArgs& a, const uint32_t (&acc)[32],
                                               int64_t pixel, int32_t col0, const int32_t* sb,
                                               const float* sm, const float* sbf) {
  if (pixel >= a.m_total) return;
  const int32_t valid = a.m - col0;  // channels left in this row (multiple of 16)
  if (valid <= 0) return;
  if (a.out_mode == kOutU8 || a.out_mode == kOutS8) {
    uint8_t* dst = static_cast<uint8_t*>(a.y) + pixel * a.y_ld + col0;
    const float lo = static_cast<float>(a.lo), hi = static_cast<float>(a.hi);
    uint4 v0, v1;
    v0.x = requant4(acc + 0, sb + 0, sm + 0, a.zp_y, lo, hi, false);
    v0.y = requant4(acc + 4, sb + 4, sm + 4, a.zp_y, lo, hi, false);
    v0.z = requant4(acc + 8, sb + 8, sm + 8, a.zp_y, lo, hi, false);
    v0.w = requant4(acc + 12, sb + 12, sm + 12, a.zp_y, lo, hi, false);
    reinterpret_cast<uint4*>(dst)[0] = v0;
    if (valid >= 32) {
      v1.x = requant4(acc + 16, sb + 16, sm + 16, a.zp_y, lo, hi, false);
      v1.y = requant4(acc + 20, sb + 20, sm + 20, a.zp_y, lo, hi, false);
      v1.z = requant4(acc + 24, sb + 24, sm + 24, a.zp_y, lo, hi, false);
      v1.w = requant4(acc + 28, sb + 28, sm + 28, a.zp_y, lo, hi, false);
      reinterpret_cast<uint4*>(dst)[1] = v1;
    }
  } else if (a.out_mode == kOutS32) {
    int32_t* dst = static_cast<int32_t*>(a.y) + pixel * a.y_ld + col0;
    const int n16 = valid >= 32 ? 8 : 4;
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
  } else if (a.out_mode == kOutF32) {
    float* dst = static_cast<float*>(a.y) + pixel * a.y_ld + col0;
    const int n16 = valid >= 32 ? 8 : 4;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      if (q < n16) {
        float4 v;
        float* pv = reinterpret_cast<float*>(&v);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float f = __uint_as_float(acc[4 * q + j]) + sbf[4 * q + j];
          f = fminf(fmaxf(f, a.act_lo), a.act_hi);
          pv[j] = f;
        }
        reinterpret_cast<float4*>(dst)[q] = v;
      }
    }
  } else if (a.out_mode == kOutF32Nchw) {
    // Lanes hold consecutive pixels, so each channel's store is coalesced.
    const int64_t hw = static_cast<int64_t>(a.out_h) * a.out_w;
    const int64_t img = pixel / hw;
    float* dst = static_cast<float*>(a.y) + (img * a.m + col0) * hw + (pixel - img * hw);
    const int n = valid >= 32 ? 32 : valid;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j < n) {
        float f = __uint_as_float(acc[j]) + sbf[j];
        f = fminf(fmaxf(f, a.act_lo), a.act_hi);
        dst[j * hw] = f;
      }
    }
  } else {  // kOutBF16x2: [hi plane of m channels | lo plane of m channels]
    __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(a.y) + pixel * a.y_ld + col0;
    const int n8 = valid >= 32 ? 4 : 2;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (q < n8) {
        uint4 vh, vl;
        uint32_t* ph = reinterpret_cast<uint32_t*>(&vh);
        uint32_t* pl = reinterpret_cast<uint32_t*>(&vl);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float f0 = __uint_as_float(acc[8 * q + 2 * j]) + sbf[8 * q + 2 * j];
          float f1 = __uint_as_float(acc[8 * q + 2 * j + 1]) + sbf[8 * q + 2 * j + 1];
          f0 = fminf(fmaxf(f0, a.act_lo), a.act_hi);
          f1 = fminf(fmaxf(f1, a.act_lo), a.act_hi);
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

// --------------------------------------------------------------- kernel
//
// KIND_I8: int8 x int8 -> s32 (A signedness by template), one MMA pass per
//          K block.
// !KIND_I8: bf16x3 for fp32 data.  The activation tensor stores each pixel as
//          [hi plane (C) | lo plane (C)] bf16 and the packed weights store per
//          tap [hi (Ck) | lo (Ck)]; every K block issues A_hi*B_hi, A_hi*B_lo
//          and A_lo*B_hi into the same f32 accumulator.
template <int BN, int BK_BYTES, int STAGES, int EPI_WARPS, bool KIND_I8, bool A_SIGNED>
__global__ void __launch_bounds__(64 + EPI_WARPS * 32, 1)
    conv_igemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                      const __grid_constant__ CUtensorMap tmap_b,
                      const __grid_constant__ CUtensorMap tmap_y, const IgemmArgs args) {
  constexpr int kA = IgemmSmem<BN, BK_BYTES>::kA;
  constexpr int kB = IgemmSmem<BN, BK_BYTES>::kB;
  // bf16x3 stages hold A_hi, A_lo, B_hi, B_lo.
  constexpr int kParts = KIND_I8 ? 1 : 2;
  constexpr int kStageBytes = kParts * (kA + kB);
  constexpr uint32_t kLayout = swizzle_layout_code(BK_BYTES);
  constexpr uint32_t kSbo = 8 * BK_BYTES;  // 8 rows of BK bytes per swizzle atom
  constexpr int kKStep = 32;               // bytes of K per MMA instruction
  constexpr int kElemBytes = KIND_I8 ? 1 : 2;
  constexpr int kBkElems = BK_BYTES / kElemBytes;
  constexpr uint32_t kIdesc =
      KIND_I8 ? make_idesc_i8(128, BN, A_SIGNED, true) : make_idesc_bf16(128, BN);
  constexpr int kAccCols = 2 * BN;  // double-buffered accumulator
  constexpr uint32_t kTmemCols = kAccCols <= 32    ? 32
                                 : kAccCols <= 64  ? 64
                                 : kAccCols <= 128 ? 128
                                 : kAccCols <= 256 ? 256
                                                   : 512;
  static_assert(kTmemCols >= kAccCols, "TMEM columns");
  static_assert(EPI_WARPS == 4 || EPI_WARPS == 8, "epilogue warps");
  constexpr int kColsPerWarp = EPI_WARPS == 8 ? BN / 2 : BN;
  constexpr int kOutWarpBytes = 32 * kColsPerWarp;
  constexpr uint32_t kOutSwizzleMask = kColsPerWarp >= 128 ? 7u : kColsPerWarp == 64 ? 3u : 1u;
  constexpr int kEpiSmemBytes = EPI_WARPS * (kOutWarpBytes + kColsPerWarp * 8);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* stages = smem;
  // Epilogue staging (int8 outputs): per warp 32 rows x kColsPerWarp bytes,
  // swizzled like the TMA store map, then per-warp bias / multiplier copies.
  uint8_t* stage_out = stages + STAGES * kStageBytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(stage_out + kEpiSmemBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* accf_bar = empty_bar + STAGES;  // [2]
  uint64_t* acce_bar = accf_bar + 2;        // [2]
  uint64_t* drain_bar = acce_bar + 2;       // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint32_t* kiter_issued = tmem_slot + 2;
  uint32_t* kiter_consumed = tmem_slot + 3;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = args.m_tiles * args.n_tiles;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    tma_prefetch_desc(&tmap_y);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf_bar[b], 1);
      mbar_init(&acce_bar[b], EPI_WARPS);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    *kiter_issued = 0;
    *kiter_consumed = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      const int32_t hw_out = args.out_h * args.out_w;
      uint32_t kiter = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int n_tile = tile % args.n_tiles;
        const int m_tile = tile / args.n_tiles;
        const int64_t p0 = static_cast<int64_t>(m_tile) * 128;
        const int32_t img = static_cast<int32_t>(p0 / hw_out);
        const int32_t rem = static_cast<int32_t>(p0 - static_cast<int64_t>(img) * hw_out);
        const int32_t oy = rem / args.out_w, ox = rem - (rem / args.out_w) * args.out_w;
        const int32_t wc = ox * args.stride_w - args.pad_l;
        const int32_t hc = oy * args.stride_h - args.pad_t;
        const int32_t co0 = n_tile * BN;
        for (int k = 0; k < args.num_k; ++k, ++kiter) {
          const int s = kiter % STAGES;
          const uint32_t ph = (kiter / STAGES) & 1u;
          if (!mbar_wait(&empty_bar[s], ph ^ 1u, abort_flag, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          const int tap = k / args.cblocks;
          const int cb = k - tap * args.cblocks;
          const int ky = tap / args.kw, kx = tap - (tap / args.kw) * args.kw;
          uint8_t* st = stages + s * kStageBytes;
          mbar_arrive_expect_tx(&full_bar[s], kStageBytes);
          const uint16_t offw = static_cast<uint16_t>(kx * args.dil_w);
          const uint16_t offh = static_cast<uint16_t>(ky * args.dil_h);
          tma_load_im2col_4d(st, &tmap_a, &full_bar[s], cb * kBkElems, wc, hc, img, offw, offh);
          const int32_t kcoord = tap * args.k_per_tap * kParts + cb * kBkElems;
          tma_load_2d(st + kParts * kA, &tmap_b, &full_bar[s], kcoord, co0);
          if constexpr (!KIND_I8) {
            // lo planes: activation channels [c, 2c), weight K [Ck, 2Ck) of the tap
            tma_load_im2col_4d(st + kA, &tmap_a, &full_bar[s], args.c + cb * kBkElems, wc, hc,
                               img, offw, offh);
            tma_load_2d(st + 2 * kA + kB, &tmap_b, &full_bar[s], kcoord + args.k_per_tap, co0);
          }
        }
      }
      *kiter_issued = kiter;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      uint32_t kiter = 0;
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++it) {
        const int buf = it & 1;
        const uint32_t aph = (it >> 1) & 1;
        if (!mbar_wait(&acce_bar[buf], aph ^ 1u, abort_flag, kErrWaitAccEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int k = 0; k < args.num_k; ++k, ++kiter) {
          const int s = kiter % STAGES;
          const uint32_t ph = (kiter / STAGES) & 1u;
          if (!mbar_wait(&full_bar[s], ph, abort_flag, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(stages + s * kStageBytes);
          const uint32_t sb = sa + kParts * kA;
#pragma unroll
          for (int kk = 0; kk < BK_BYTES / kKStep; ++kk) {
            const uint64_t ad = make_smem_desc(sa + kk * kKStep, 16, kSbo, kLayout);
            const uint64_t bd = make_smem_desc(sb + kk * kKStep, 16, kSbo, kLayout);
            if constexpr (KIND_I8) {
              mma_i8(d_tmem, ad, bd, kIdesc, (k | kk) != 0);
            } else {
              const uint64_t adl = make_smem_desc(sa + kA + kk * kKStep, 16, kSbo, kLayout);
              const uint64_t bdl = make_smem_desc(sb + kB + kk * kKStep, 16, kSbo, kLayout);
              mma_f16(d_tmem, ad, bd, kIdesc, (k | kk) != 0);
              mma_f16(d_tmem, ad, bdl, kIdesc, 1);
              mma_f16(d_tmem, adl, bd, kIdesc, 1);
            }
          }
          tc_commit(&empty_bar[s]);  // frees the stage once these MMAs finish
        }
        if (ok) tc_commit(&accf_bar[buf]);
      }
      *kiter_consumed = kiter;
      // Drain: every MMA issued above has finished once this barrier flips, so
      // tensor memory can be released safely even on the abort path.
      tc_commit(drain_bar);
      int dummy_abort = 0;
      mbar_wait(drain_bar, 0, &dummy_abort, kErrWaitFull);
    }
  } else {
    // ------------------------------------------------ epilogue warps
    const int ew = warp - 2;             // 0 .. EPI_WARPS-1
    const int quarter = warp & 3;        // TMEM lane quarter this warp may access
    const int half = ew / 4;             // column half (EPI_WARPS == 8)
    // Per-warp bias / multiplier copy for its kColsPerWarp columns.
    int32_t* s_bias = reinterpret_cast<int32_t*>(stage_out + EPI_WARPS * kOutWarpBytes) +
                      ew * kColsPerWarp * 2;
    float* s_mult = reinterpret_cast<float*>(s_bias + kColsPerWarp);
    uint8_t* s_out = stage_out + ew * kOutWarpBytes;  // 32 rows x kColsPerWarp bytes, swizzled
    const bool tma_out = KIND_I8 && (args.out_mode == kOutU8 || args.out_mode == kOutS8);
    const bool out_signed = args.out_mode == kOutS8;
    const int32_t qmin = args.lo + args.zp_y, qmax = args.hi + args.zp_y;
    const bool fast_requant = args.zp_y == 0 && qmin == (out_signed ? -128 : 0) &&
                              qmax == (out_signed ? 127 : 255);
    int loaded_n_tile = -1;
    int it = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
      const int buf = it & 1;
      const uint32_t aph = (it >> 1) & 1;
      const int n_tile = tile % args.n_tiles;
      const int m_tile = tile / args.n_tiles;
      if (n_tile != loaded_n_tile) {
        // (re)load this warp's per-channel epilogue constants
        __syncwarp();
        for (int j = lane; j < kColsPerWarp; j += 32) {
          const int32_t ch = n_tile * BN + half * kColsPerWarp + j;
          const bool in = ch < args.m;
          if constexpr (KIND_I8) {
            s_bias[j] = (in && args.bias_i32 != nullptr) ? __ldg(args.bias_i32 + ch) : 0;
            s_mult[j] = (in && args.mult != nullptr) ? __ldg(args.mult + ch) : 0.0f;
          } else {
            s_bias[j] = __float_as_int((in && args.bias_f32 != nullptr) ? __ldg(args.bias_f32 + ch)
                                                                        : 0.0f);
            s_mult[j] = 0.0f;
          }
        }
        loaded_n_tile = n_tile;
        __syncwarp();
      }
      if (!mbar_wait(&accf_bar[buf], aph, abort_flag, kErrWaitAccFull)) break;
      tc_fence_after();
      const int64_t row0 = static_cast<int64_t>(m_tile) * 128 + quarter * 32;
      const int64_t pixel = row0 + lane;
      const int32_t wcol0 = n_tile * BN + half * kColsPerWarp;  // first output channel of this warp
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN +
                             half * kColsPerWarp;
      if (tma_out) {
        // The staging buffer is free once the previous tile's store has read it.
        if (lane == 0) bulk_wait_group_read0();
        __syncwarp();
      }
#pragma unroll 1
      for (int cc = 0; cc < kColsPerWarp; cc += 32) {
        uint32_t acc[32];
        tmem_ld_32x32b_x32(t_row + cc, acc);
        tmem_ld_wait();
        if (cc + 32 >= kColsPerWarp) {
          // Last read of this accumulator buffer by this warp: hand it back so
          // the MMA warp can start the next tile while we finish the epilogue.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acce_bar[buf]);
        }
        if (tma_out) {
          uint32_t packed[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int4 b4 = *reinterpret_cast<const int4*>(s_bias + cc + 4 * q);
            const float4 m4 = *reinterpret_cast<const float4*>(s_mult + cc + 4 * q);
            if (fast_requant) {
              packed[q] = out_signed ? requant_pack4<true, true>(acc + 4 * q, b4, m4, 0, 0, 0)
                                     : requant_pack4<true, false>(acc + 4 * q, b4, m4, 0, 0, 0);
            } else {
              packed[q] = requant_pack4<false, false>(acc + 4 * q, b4, m4, args.zp_y, qmin, qmax);
            }
          }
          // two 16-byte chunks of this lane's row, at swizzled positions
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t off = lane * kColsPerWarp + cc + 16 * h;
            const uint32_t phys = off ^ (((off >> 7) & kOutSwizzleMask) << 4);
            *reinterpret_cast<uint4*>(s_out + phys) =
                make_uint4(packed[4 * h], packed[4 * h + 1], packed[4 * h + 2], packed[4 * h + 3]);
          }
        } else {
          int32_t sb[32];
          float sm[32];
          float sbf[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if constexpr (KIND_I8) {
              sb[j] = s_bias[cc + j];
              sm[j] = s_mult[cc + j];
              sbf[j] = 0.0f;
            } else {
              sb[j] = 0;
              sm[j] = 0.0f;
              sbf[j] = __int_as_float(s_bias[cc + j]);
            }
          }
          epilogue_chunk<!KIND_I8>(args, acc, pixel, wcol0 + cc, sb, sm, sbf);
        }
      }
      if (tma_out) {
        fence_proxy_async_smem();  // generic-proxy smem writes -> visible to the TMA unit
        __syncwarp();
        if (lane == 0 && row0 < args.m_total && wcol0 < args.y_ld) {
          tma_store_2d(&tmap_y, s_out, wcol0, static_cast<int32_t>(row0));
          bulk_commit_group();
        }
      }
    }
    if (lane == 0) bulk_wait_group0();
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag && threadIdx.x == 0) {
    // Loads issued but never consumed are still landing in shared memory:
    // wait for them (bounded) before the CTA exits.
    int dummy_abort = 0;
    for (uint32_t k = *kiter_consumed; k < *kiter_issued; ++k) {
      mbar_wait(&full_bar[k % STAGES], (k / STAGES) & 1u, &dummy_abort, kErrWaitFull);
    }
  }
  if (warp == 1) {
    tc_fence_after();
    __syncwarp();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace ie_cuda
