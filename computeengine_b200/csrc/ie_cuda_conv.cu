// C ABI of the sm_100a Conv2D forward backend (declared in
// include/ie_cuda_conv.h).  One translation unit: the kernels are included
// here so the device-side error word is a single object.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <atomic>
#include <mutex>

#include "conv_igemm.cuh"
#include "direct_kernels.cuh"
#include "host_util.h"
#include "layout_kernels.cuh"
#include "pool_gemm_kernels.cuh"
#include "ptx.cuh"

using namespace ie_cuda;

namespace {

constexpr int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }
constexpr int64_t ceil_div(int64_t v, int64_t m) { return (v + m - 1) / m; }

// ------------------------------------------------------------- geometry

// conv2d_op.cpp:77-165 and attrs_util.h:185-197.
int resolve(const ie_conv2d_desc* d, int64_t bias_len, ie_conv2d_shape* out) {
  if (d == nullptr || out == nullptr) return fail(IE_INVALID_ARGUMENT, "null descriptor");
  if (d->n <= 0 || d->c <= 0 || d->h <= 0 || d->w <= 0 || d->m <= 0 || d->kh <= 0 ||
      d->kw <= 0) {
    return fail(IE_INVALID_ARGUMENT, "Conv2D expects positive dimensions");
  }
  if (d->stride_h <= 0 || d->stride_w <= 0 || d->dil_h <= 0 || d->dil_w <= 0) {
    return fail(IE_INVALID_ARGUMENT, "strides and dilations must be positive");
  }
  if (d->group <= 0 || d->c % d->group != 0 || d->m % d->group != 0) {
    return fail(IE_INVALID_ARGUMENT, "Conv2D group must divide input and output channels");
  }
  if (d->depthwise && d->group != d->c) {
    return fail(IE_INVALID_ARGUMENT, "DepthwiseConv2D requires group == input channels");
  }
  if (bias_len >= 0 && bias_len != d->m) {
    return fail(IE_INVALID_ARGUMENT, "Conv2D bias must have shape [M]");
  }
  int64_t pt = d->pad_top, pl = d->pad_left, pb = d->pad_bottom, pr = d->pad_right;
  if (pt < 0 || pl < 0 || pb < 0 || pr < 0) {
    return fail(IE_INVALID_ARGUMENT, "pads must be non-negative");
  }
  auto same = [](int64_t in, int64_t k, int64_t dil, int64_t s, bool lower, int64_t* b,
                 int64_t* a) {
    const int64_t o = (in + s - 1) / s;
    const int64_t total = std::max<int64_t>(0, (o - 1) * s + dil * (k - 1) + 1 - in);
    int64_t before = total / 2, after = total - before;
    if (lower) std::swap(before, after);
    *b = before;
    *a = after;
  };
  if (d->auto_pad == IE_PAD_VALID) {
    pt = pl = pb = pr = 0;
  } else if (d->auto_pad == IE_PAD_SAME_UPPER || d->auto_pad == IE_PAD_SAME_LOWER) {
    const bool lower = d->auto_pad == IE_PAD_SAME_LOWER;
    same(d->h, d->kh, d->dil_h, d->stride_h, lower, &pt, &pb);
    same(d->w, d->kw, d->dil_w, d->stride_w, lower, &pl, &pr);
  } else if (d->auto_pad != IE_PAD_NOTSET) {
    return fail(IE_INVALID_ARGUMENT, "unsupported auto_pad");
  }
  const int64_t eh = d->dil_h * (d->kh - 1) + 1, ew = d->dil_w * (d->kw - 1) + 1;
  if (d->h + pt + pb < eh || d->w + pl + pr < ew) {
    return fail(IE_INVALID_ARGUMENT, "Conv2D kernel exceeds padded input");
  }
  const int64_t oh = (d->h + pt + pb - eh) / d->stride_h + 1;
  const int64_t ow = (d->w + pl + pr - ew) / d->stride_w + 1;
  if (oh <= 0 || ow <= 0) return fail(IE_INVALID_ARGUMENT, "Conv2D produces an empty output");
  out->pad_top = pt;
  out->pad_left = pl;
  out->pad_bottom = pb;
  out->pad_right = pr;
  out->out_h = oh;
  out->out_w = ow;
  return IE_OK;
}

// --------------------------------------------------------- tile choices

// Channel block (bytes of K per tap per stage) that pads the channel count
// least; ties go to the wider block.
int choose_bk_bytes(int64_t c_store, int elem_bytes, bool must_divide, int max_bk = 128) {
  int best = 0;
  int64_t best_cost = INT64_MAX;
  for (int bk : {128, 64, 32}) {
    if (bk > max_bk) continue;
    const int64_t elems = bk / elem_bytes;
    if (must_divide && c_store % elems != 0) continue;
    const int64_t cost = round_up(c_store, elems);
    if (cost < best_cost) {
      best_cost = cost;
      best = bk;
    }
  }
  return best;
}

int choose_bn(int64_t m) {
  int best = 256;
  int64_t best_cost = INT64_MAX;
  for (int bn : {256, 128, 64}) {
    const int64_t cost = round_up(m, bn);
    if (cost < best_cost) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

// Widest channel block allowed for a tile width: the bf16x3 path keeps its
// stages (A hi/lo + B hi/lo) small enough for a 3-deep pipeline.
int igemm_max_bk(int bn, bool i8) {
  if (i8) return 128;
  return bn >= 256 ? 64 : 128;
}

constexpr int kSmemLimit = 227 * 1024;
constexpr int kMaxDevices = 64;

// One compiled variant of the implicit-GEMM kernel.
struct Variant {
  int bn, bkb, m_sub, epi;
  int out_bufs;    // staged requantized output tiles (int8 path), 0 otherwise
  int halo_stage;  // row-band mode: bytes per stage; 0 = im2col mode
  bool b_res, i8, a_signed;
};

template <int BN, int BKB, int EPI, int MSUB, bool BRES, bool I8, bool AS>
int launch_variant(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ty,
                   const IgemmArgs& args, int grid, cudaStream_t st) {
  using P = IgemmPlan<BN, BKB, EPI, MSUB, BRES, I8>;
  auto kern = conv_igemm_kernel<BN, BKB, EPI, MSUB, BRES, I8, AS>;
  if (args.halo && !(I8 && BRES)) return fail(IE_RUNTIME, "row-band mode needs resident int8 weights");
  const int smem = P::bytes(args.stages, args.num_k, args.out_bufs,
                            args.halo ? args.stage_bytes : P::kStage);
  if (smem > kSmemLimit) return fail(IE_UNSUPPORTED, "shared memory plan too large (%d)", smem);
  if (args.wait_limit_ns == 0) return fail(IE_RUNTIME, "no wait limit set");
  // The shared-memory opt-in is a property of the function in each device's
  // context: set it once per device this variant runs on.
  static std::mutex mu;
  static bool attr_set[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(IE_RUNTIME, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(IE_UNSUPPORTED, "device ordinal %d out of range", dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!attr_set[dev]) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
      if (e != cudaSuccess) {
        return fail(IE_RUNTIME, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      }
      attr_set[dev] = true;
    }
  }
  // producer, MMA issuer, EPI epilogue warps, output store warp.  Launched
  // with programmatic stream serialization: the prologue (barriers, tensor
  // memory, tensor-map prefetch, resident weights) overlaps the tail of the
  // kernel before it, which the producer waits for (griddepcontrol.wait)
  // before its first activation load.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(96 + EPI * 32);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  // right after this stream's weights were packed: plain stream order, so the
  // resident-weight loads issued before griddepcontrol.wait see them
  cfg.numAttrs = g_packed_weights_stream.load(std::memory_order_relaxed) == stream_key(st) ? 0 : 1;
  const cudaError_t le = cudaLaunchKernelEx(&cfg, kern, ta, tb, ty, args);
  if (le != cudaSuccess) {
    ++g_launches;
    return fail(IE_RUNTIME, "conv_igemm_kernel launch: %s", cudaGetErrorString(le));
  }
  return check_launch("conv_igemm_kernel");
}

using LaunchFn = int (*)(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                         const IgemmArgs&, int, cudaStream_t);

template <int BN, int BKB, bool I8, bool AS>
LaunchFn pick_bn_bk(int m_sub, bool b_res) {
  if constexpr (I8) {
    // The requantize epilogue is the limiter of the small-K layers.  It runs
    // on 8 warps (4 lane quarters x 2 sub-tiles or x 2 column groups) rather
    // than 16: ~125-135 registers per thread instead of 96 let each warp
    // interleave more requantize chains, which measured 3-12% faster per
    // layer than twice the warps.
    if constexpr (BN <= 128) {
      // 256 positions per tile by default; 128 where the default tiles cannot
      // fill the GPU (not for 32 channels: 8 epilogue warps need 32 columns
      // each, so that tile always has two sub-tiles)
      if (m_sub == 2) {
        return b_res ? launch_variant<BN, BKB, 8, 2, true, I8, AS>
                     : launch_variant<BN, BKB, 8, 2, false, I8, AS>;
      }
      if constexpr (BN >= 64) {
        return b_res ? launch_variant<BN, BKB, 8, 1, true, I8, AS>
                     : launch_variant<BN, BKB, 8, 1, false, I8, AS>;
      } else {
        return nullptr;
      }
    } else {
      return b_res ? launch_variant<BN, BKB, 8, 1, true, I8, AS>
                   : launch_variant<BN, BKB, 8, 1, false, I8, AS>;
    }
  } else {
    if (m_sub != 1 || b_res) return nullptr;
    if constexpr (BN < 64 || (BN >= 256 && BKB > 64)) {
      return nullptr;
    } else {
      return launch_variant<BN, BKB, (BN >= 256 ? 8 : 4), 1, false, I8, AS>;
    }
  }
}

template <bool I8, bool AS>
LaunchFn pick_launch(const Variant& v) {
#define IE_CASE(BN_, BK_) \
  if (v.bn == BN_ && v.bkb == BK_) return pick_bn_bk<BN_, BK_, I8, AS>(v.m_sub, v.b_res);
  IE_CASE(32, 32) IE_CASE(32, 64) IE_CASE(32, 128)
  IE_CASE(64, 32) IE_CASE(64, 64) IE_CASE(64, 128)
  IE_CASE(128, 32) IE_CASE(128, 64) IE_CASE(128, 128)
  IE_CASE(256, 32) IE_CASE(256, 64) IE_CASE(256, 128)
#undef IE_CASE
  return nullptr;
}

// Shared-memory bytes of a variant (mirrors IgemmPlan::bytes).
int plan_bytes(const Variant& v, int stages, int num_k) {
  const int parts = v.i8 ? 1 : 2;
  const int rows = 128 * v.m_sub;
  const int ka = rows * v.bkb, kb = v.bn * v.bkb;
  const int stage = v.halo_stage > 0 ? v.halo_stage : parts * (ka + (v.b_res ? 0 : kb));
  const int warp_cols = v.bn / (v.epi / (4 * v.m_sub));
  const int out_tile = v.i8 ? rows * v.bn : 0;
  const int consts = v.epi * warp_cols * 12;
  const int bars = 8 * (2 * kMaxStages + 10) + 32;
  return 1024 + stages * stage + (v.b_res ? parts * num_k * kb : 0) + v.out_bufs * out_tile +
         consts + bars;
}

struct IgemmSetup {
  IgemmArgs args;
  CUtensorMap ta, tb, ty;
  Variant v;
  int grid;
};

// Shared set-up of the implicit GEMM for both element kinds.
//   elem_bytes: 1 (int8) or 2 (bf16; activation and weights hold hi|lo planes)
//   allow_halo: the caller's output goes through the staged TMA store (int8
//   requantized), so the row-band mode may be used
std::atomic<int32_t> g_tile_policy{IE_TILE_FILL};

// One tile plan of the implicit GEMM: the kernel variant, its pipeline depth,
// the row-band geometry when that mode is used, the tile counts and grid, and
// a cycle estimate used to choose between plans.
struct TilePlan {
  Variant v;
  int stages = 0;
  int64_t h_wp = 0, h_rows_t = 0, h_rows_box = 0, h_tiles_img = 0, h_band = 0;
  int64_t m_tiles = 0, n_tiles = 0;
  int grid = 0;
  double est = 0.0;
  double mma_cycles = 0.0;  // estimated MMA time of one tile
  int64_t ck = 0;           // channels per tap in the packed weights
};

// Builds the plan for tiles of bn output channels x 128 * m_sub positions.
// Returns false when no pipeline of that shape fits in shared memory.
//
// The estimate: the CTAs of a persistent grid each run ceil(tiles / CTAs)
// tiles; a tile costs its 32-byte K steps times the cycles of one 128-row MMA
// step at that width -- int8: the shared-memory operand rate bounds N=64 and
// N=128, the tensor pipe N=256 (~68, ~91 and ~137 cycles, measured); bf16x3
// (three products per step): the tensor pipe N=128 and N=256 (~203, ~406),
// the operand rate N=64 (~133) -- its outputs at the epilogue's ~11.7 per
// cycle per SM, and ~1000 cycles of hand-offs; a CTA with resident weights
// first loads its bn x K slice at ~64 B/cycle.
bool plan_tiles(const ie_conv2d_desc* d, const ie_conv2d_shape& s, bool i8, int elem_bytes,
                int64_t x_c_store, bool allow_halo, int bn, int m_sub, int sms, TilePlan* p) {
  *p = TilePlan{};
  Variant& v = p->v;
  v.i8 = i8;
  v.bn = bn;
  v.bkb = choose_bk_bytes(x_c_store, elem_bytes, !i8, igemm_max_bk(bn, i8));
  if (v.bkb == 0) return false;
  v.m_sub = m_sub;
  v.epi = i8 ? 8 : (v.bn >= 256 ? 8 : 4);
  const int64_t bk_elems = v.bkb / elem_bytes;
  const int64_t cblocks = ceil_div(x_c_store, bk_elems);
  const int64_t taps = d->kh * d->kw;
  const int64_t num_k = taps * cblocks;
  const int64_t m_total = d->n * s.out_h * s.out_w;
  // Weights resident in shared memory when the CTA's slice fits beside a
  // pipeline of at least 4 activation stages; two staged output tiles (the
  // epilogue never waits for a store) unless that costs pipeline depth below 4.
  v.out_bufs = i8 ? 2 : 0;
  v.b_res = false;
  if (i8) {
    v.b_res = true;
    if (plan_bytes(v, 4, static_cast<int>(num_k)) > kSmemLimit) {
      v.out_bufs = 1;
      if (plan_bytes(v, 4, static_cast<int>(num_k)) > kSmemLimit) {
        v.out_bufs = 2;
        v.b_res = false;
      }
    }
  }
  auto max_stages = [&] {
    int st = kMaxStages;
    while (st > 2 && plan_bytes(v, st, static_cast<int>(num_k)) > kSmemLimit) --st;
    return st;
  };
  int stages = max_stages();
  if (i8 && v.out_bufs == 2 && stages < 4) {
    v.out_bufs = 1;
    stages = max_stages();
  }
  if (plan_bytes(v, stages, static_cast<int>(num_k)) > kSmemLimit) return false;
  // Row-band mode for stride-1 multi-tap int8 convolutions: tiles of whole
  // output rows in a (w + pad_l + pad_r)-wide position space, one band load
  // per channel block.  Used when the rows fill the tiles well and the
  // natural tile width keeps the weights resident with at least 3 stages
  // (measured: narrowing the tiles to make the weights fit costs more than
  // the band saves).
  if (allow_halo && i8 && d->stride_h == 1 && d->stride_w == 1 && taps > 1) {
    const int64_t wp = d->w + s.pad_left + s.pad_right;
    do {
      Variant hv = v;
      hv.b_res = true;
      hv.out_bufs = 2;
      const int64_t rows = 128 * hv.m_sub;
      const int64_t rows_t = rows / wp;
      if (rows_t < 1 || wp > 256) break;
      const int64_t tiles_img = ceil_div(s.out_h, rows_t);
      const double fill = static_cast<double>(s.out_h * s.out_w) / static_cast<double>(tiles_img * rows);
      const int64_t rows_box = rows_t + (d->kh - 1) * d->dil_h;
      const int64_t slack = (d->kh - 1) * d->dil_h * wp + (d->kw - 1) * d->dil_w;
      hv.halo_stage = static_cast<int>(round_up(round_up(rows + slack, 8) * v.bkb, 1024));
      if (fill < 0.7 || rows_box > 256) break;
      int st = kMaxStages;
      while (st > 3 && plan_bytes(hv, st, static_cast<int>(num_k)) > kSmemLimit) --st;
      if (plan_bytes(hv, st, static_cast<int>(num_k)) > kSmemLimit) {
        hv.out_bufs = 1;
        st = kMaxStages;
        while (st > 3 && plan_bytes(hv, st, static_cast<int>(num_k)) > kSmemLimit) --st;
        if (plan_bytes(hv, st, static_cast<int>(num_k)) > kSmemLimit) break;
      }
      v = hv;
      stages = st;
      p->h_wp = wp;
      p->h_rows_t = rows_t;
      p->h_rows_box = rows_box;
      p->h_tiles_img = tiles_img;
      p->h_band = rows_box * wp * v.bkb;
    } while (false);
  }
  p->stages = stages;
  p->m_tiles = p->h_wp > 0 ? d->n * p->h_tiles_img : ceil_div(m_total, 128 * v.m_sub);
  p->n_tiles = ceil_div(d->m, v.bn);
  int64_t waves;
  if (v.b_res) {
    // each CTA keeps one n_tile: the grid is a multiple of n_tiles
    const int64_t per_n = std::max<int64_t>(
        1, std::min<int64_t>(p->m_tiles, std::max<int64_t>(1, sms / p->n_tiles)));
    p->grid = static_cast<int>(per_n * p->n_tiles);
    waves = ceil_div(p->m_tiles, per_n);
  } else {
    p->grid = static_cast<int>(std::min<int64_t>(p->m_tiles * p->n_tiles, sms));
    waves = ceil_div(p->m_tiles * p->n_tiles, static_cast<int64_t>(p->grid));
  }
  const double k_steps = static_cast<double>(num_k) * (v.bkb / 32.0);
  const double mma = i8 ? (v.bn <= 32 ? 52.0 : v.bn <= 64 ? 68.0 : (v.bn <= 128 ? 91.0 : 137.0))
                       : (v.bn <= 64 ? 133.0 : (v.bn <= 128 ? 203.0 : 406.0));
  p->ck = cblocks * bk_elems;
  const double rows = 128.0 * v.m_sub;
  p->mma_cycles = k_steps * mma * v.m_sub;
  const double t_tile = p->mma_cycles + rows * v.bn / 11.7 + 1000.0;
  p->est = static_cast<double>(waves) * t_tile +
           (v.b_res ? static_cast<double>(v.bn) * num_k * v.bkb / 64.0 : 0.0);
  return true;
}

// Shared set-up of the implicit GEMM for both element kinds.
//   elem_bytes: 1 (int8) or 2 (bf16; activation and weights hold hi|lo planes)
//   allow_halo: the caller's output goes through the staged TMA store (int8
//   requantized), so the row-band mode may be used
//
// Narrower or shorter tiles are considered beside the default (the widest
// channel tile that wastes least; int8: 256 positions below 256 channels):
// a launch whose default tiles cannot fill the GPU and carry at least ~2000
// cycles of MMA work each takes the plan with the smallest estimate when that
// is at least 10% below the default's.  Shallower launches keep the default:
// they are bound by launch and pipeline latency, and a narrow grid leaves
// SMs to the next launch's prologue (measured: MobileNetV2's K = 160-192 1x1
// layers at batch 64 ran 13-16% slower on twice the CTAs).  The packed int8
// weights do not depend on the tile shape; the packed bf16x3 weights do only
// through the channel-block rounding, so an fp32 candidate must keep the
// default's channels per tap.
int setup_igemm(const ie_conv2d_desc* d, const ie_conv2d_shape& s, int elem_bytes,
                int64_t x_c_store, const void* x, const void* packed, IgemmSetup* out,
                bool allow_halo = false) {
  const bool i8 = elem_bytes == 1;
  const int64_t m_total = d->n * s.out_h * s.out_w;
  {
    const int bkb = choose_bk_bytes(x_c_store, elem_bytes, !i8, igemm_max_bk(choose_bn(d->m), i8));
    if (bkb == 0) return fail(IE_UNSUPPORTED, "no channel block divides c_store=%lld",
                              static_cast<long long>(x_c_store));
    const int64_t num_k = d->kh * d->kw * ceil_div(x_c_store, static_cast<int64_t>(bkb / elem_bytes));
    if (m_total > (int64_t{1} << 40) || d->n > INT32_MAX || d->h > INT32_MAX || d->w > INT32_MAX ||
        num_k > (1 << 20)) {
      return fail(IE_UNSUPPORTED, "tensor too large");
    }
  }
  const int sms = num_sms();
  // int8 layers of at most 32 channels (MobileNet's narrow projections) run
  // 32-channel tiles instead of 64-channel ones that are half padding
  const int bn0 = (i8 && d->m <= 32) ? 32 : choose_bn(d->m);
  const int ms0 = (i8 && bn0 <= 128) ? 2 : 1;
  TilePlan plan;
  if (!plan_tiles(d, s, i8, elem_bytes, x_c_store, allow_halo, bn0, ms0, sms, &plan)) {
    return fail(IE_UNSUPPORTED, "no pipeline fits in shared memory");
  }
  if (plan.grid < sms && plan.mma_cycles >= 2000.0 &&
      g_tile_policy.load(std::memory_order_relaxed) == IE_TILE_FILL) {
    const double limit = 0.9 * plan.est;
    const int cand[][2] = {{bn0, 1}, {128, 1}, {64, 2}, {64, 1}};
    TilePlan best = plan;
    for (const auto& c : cand) {
      if (c[0] > bn0 || (c[0] == bn0 && c[1] == ms0)) continue;
      if (!i8 && c[1] != 1) continue;  // the bf16x3 kernel runs 128-position tiles
      if (c[0] == 32 && c[1] == 1) continue;  // 32-channel tiles need two sub-tiles
      TilePlan t;
      if (plan_tiles(d, s, i8, elem_bytes, x_c_store, allow_halo, c[0], c[1], sms, &t) &&
          (i8 || t.ck == plan.ck) && t.est < limit && t.est < best.est) {
        best = t;
      }
    }
    plan = best;
  }
  Variant& v = out->v;
  v = plan.v;
  const int stages = plan.stages;
  const int64_t h_wp = plan.h_wp, h_rows_t = plan.h_rows_t, h_rows_box = plan.h_rows_box;
  const int64_t h_tiles_img = plan.h_tiles_img, h_band = plan.h_band;
  const int64_t bk_elems = v.bkb / elem_bytes;
  const int64_t cblocks = ceil_div(x_c_store, bk_elems);
  const int64_t taps = d->kh * d->kw;
  const int64_t ck = cblocks * bk_elems;
  const int64_t num_k = taps * cblocks;
  const CUtensorMapDataType dt = i8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int64_t a_chan = i8 ? x_c_store : 2 * x_c_store;
  int rc;
  const bool a_tiled = h_wp == 0 && d->kh == 1 && d->kw == 1 && d->stride_h == 1 &&
                       d->stride_w == 1 && s.pad_top == 0 && s.pad_left == 0 &&
                       s.pad_bottom == 0 && s.pad_right == 0 && m_total < (int64_t{1} << 31);
  if (a_tiled) {
    // [n*h*w pixels, a_chan] matrix, box = bk elements x one tile of rows
    rc = encode_2d(&out->ta, x, dt, elem_bytes, m_total, a_chan, static_cast<int>(bk_elems),
                   128 * v.m_sub);
  } else if (h_wp > 0) {
    // band box: bk channels x wp columns (from -pad_left) x rows_box rows
    rc = encode_nhwc_4d(&out->ta, x, dt, elem_bytes, d->n, d->h, d->w, a_chan,
                        static_cast<int>(bk_elems), static_cast<int>(h_wp),
                        static_cast<int>(h_rows_box));
  } else {
    // TMA im2col corner limits for 4D tensors: [-128, 127]; offsets < 256.
    const int64_t lower_w = -s.pad_left, lower_h = -s.pad_top;
    const int64_t upper_w = s.pad_right - (d->kw - 1) * d->dil_w;
    const int64_t upper_h = s.pad_bottom - (d->kh - 1) * d->dil_h;
    for (int64_t val : {lower_w, lower_h, upper_w, upper_h}) {
      if (val < -128 || val > 127) {
        return fail(IE_UNSUPPORTED, "padding / kernel extent too large for TMA im2col");
      }
    }
    if ((d->kw - 1) * d->dil_w > 255 || (d->kh - 1) * d->dil_h > 255 || d->stride_h > 8 ||
        d->stride_w > 8) {
      return fail(IE_UNSUPPORTED, "kernel extent or stride too large for TMA im2col");
    }
    rc = encode_im2col(&out->ta, x, dt, elem_bytes, d->n, d->h, d->w, a_chan,
                       static_cast<int>(bk_elems), 128 * v.m_sub, static_cast<int>(lower_w),
                       static_cast<int>(lower_h), static_cast<int>(upper_w),
                       static_cast<int>(upper_h), static_cast<int>(d->stride_w),
                       static_cast<int>(d->stride_h));
  }
  if (rc != IE_OK) return rc;
  const int64_t b_cols = taps * ck * (i8 ? 1 : 2);
  rc = encode_2d(&out->tb, packed, dt, elem_bytes, d->m, b_cols, static_cast<int>(bk_elems), v.bn);
  if (rc != IE_OK) return rc;

  IgemmArgs& a = out->args;
  std::memset(&a, 0, sizeof(a));
  a.wait_limit_ns = kWaitLimitNs;
  a.n = static_cast<int32_t>(d->n);
  a.h = static_cast<int32_t>(d->h);
  a.w = static_cast<int32_t>(d->w);
  a.c = static_cast<int32_t>(x_c_store);
  a.out_h = static_cast<int32_t>(s.out_h);
  a.out_w = static_cast<int32_t>(s.out_w);
  a.m = static_cast<int32_t>(d->m);
  a.kh = static_cast<int32_t>(d->kh);
  a.kw = static_cast<int32_t>(d->kw);
  a.stride_h = static_cast<int32_t>(d->stride_h);
  a.stride_w = static_cast<int32_t>(d->stride_w);
  a.dil_h = static_cast<int32_t>(d->dil_h);
  a.dil_w = static_cast<int32_t>(d->dil_w);
  a.pad_t = static_cast<int32_t>(s.pad_top);
  a.pad_l = static_cast<int32_t>(s.pad_left);
  a.cblocks = static_cast<int32_t>(cblocks);
  a.num_k = static_cast<int32_t>(num_k);
  a.k_per_tap = static_cast<int32_t>(ck);
  a.stages = stages;
  a.out_bufs = v.out_bufs;
  a.m_total = m_total;
  // |x| <= 255 (uint8) or 128 (int8), |w| <= 128: |acc| <= K * 255 * 128
  a.acc_bound = d->kh * d->kw * d->c * 255 * 128;
  a.m_tiles = static_cast<int32_t>(plan.m_tiles);
  a.n_tiles = static_cast<int32_t>(plan.n_tiles);
  a.a_tiled = a_tiled ? 1 : 0;
  if (h_wp > 0) {
    a.halo = 1;
    a.wp = static_cast<int32_t>(h_wp);
    a.rows_t = static_cast<int32_t>(h_rows_t);
    a.rows_box = static_cast<int32_t>(h_rows_box);
    a.tiles_img = static_cast<int32_t>(h_tiles_img);
    a.stage_bytes = v.halo_stage;
    a.band_bytes = static_cast<int32_t>(h_band);
  }
  out->grid = plan.grid;
  return IE_OK;
}

// Packed-weight geometry for a dense convolution on x_c_store input channels.
void packed_geom(const ie_conv2d_desc* d, int elem_bytes, int64_t* taps, int64_t* ck) {
  const int64_t c_store = round_up(d->c, 16);
  const int bkb = choose_bk_bytes(c_store, elem_bytes, elem_bytes != 1,
                                  igemm_max_bk(choose_bn(d->m), elem_bytes == 1));
  const int64_t bk_elems = bkb / elem_bytes;
  *taps = d->kh * d->kw;
  *ck = ceil_div(c_store, bk_elems) * bk_elems;
}

// Bytes of the packed int8 weights proper; the per-channel weight sums
// (int32 [round_up(m, 16)]) follow them in the same buffer.
int64_t q8_packed_body_bytes(const ie_conv2d_desc* d) {
  int64_t taps, ck;
  packed_geom(d, 1, &taps, &ck);
  return d->m * taps * ck;
}

// Fills the weight-sum trailer of a packed int8 weight buffer.
int q8_write_weight_sums(const ie_conv2d_desc* d, void* packed, cudaStream_t st) {
  const int64_t body = q8_packed_body_bytes(d);
  const int64_t m_store = round_up(d->m, 16);
  q8_weight_sums<<<static_cast<unsigned>(ceil_div(m_store * 32, 256)), 256, 0, st>>>(
      static_cast<const int8_t*>(packed), reinterpret_cast<int32_t*>(static_cast<uint8_t*>(packed) + body),
      static_cast<int32_t>(d->m), static_cast<int32_t>(m_store), body / d->m);
  return check_launch("q8_weight_sums");
}

int check_dense(const ie_conv2d_desc* d) {
  if (d->group != 1) return fail(IE_UNSUPPORTED, "the tensor-core path runs group == 1 only");
  return IE_OK;
}

int check_ptr(const void* p, const char* what, size_t align) {
  if (p == nullptr) return fail(IE_INVALID_ARGUMENT, "%s is null", what);
  if (reinterpret_cast<uintptr_t>(p) % align != 0) {
    return fail(IE_INVALID_ARGUMENT, "%s must be %zu-byte aligned", what, align);
  }
  return IE_OK;
}

thread_local ie_conv_plan g_last_plan{};

int launch_setup(IgemmSetup& su, bool a_signed, cudaStream_t st) {
  g_last_plan.bn = su.v.bn;
  g_last_plan.bk_bytes = su.v.bkb;
  g_last_plan.m_sub = su.v.m_sub;
  g_last_plan.stages = su.args.stages;
  g_last_plan.resident_weights = su.v.b_res ? 1 : 0;
  g_last_plan.out_bufs = su.v.out_bufs;
  g_last_plan.row_band = su.args.halo;
  g_last_plan.grid = su.grid;
  g_last_plan.a_tiled = su.args.a_tiled;
  LaunchFn fn = su.v.i8 ? (a_signed ? pick_launch<true, true>(su.v) : pick_launch<true, false>(su.v))
                        : pick_launch<false, false>(su.v);
  if (fn == nullptr) {
    return fail(IE_UNSUPPORTED, "no kernel variant for BN=%d BK=%d m_sub=%d resident=%d", su.v.bn,
                su.v.bkb, su.v.m_sub, static_cast<int>(su.v.b_res));
  }
  return fn(su.ta, su.tb, su.ty, su.args, su.grid, st);
}

int run_q8(const ie_conv2d_desc* d, const ie_q8_params* q, const void* x, const void* packed,
           const int32_t* bias, const float* mult, void* y, int out_mode, void* stream) {
  ie_conv2d_shape s;
  int rc = resolve(d, -1, &s);
  if (rc != IE_OK) return rc;
  if ((rc = check_dense(d)) != IE_OK) return rc;
  if (q == nullptr) return fail(IE_INVALID_ARGUMENT, "null quantization parameters");
  if (q->x_signed ? (q->zp_x < -128 || q->zp_x > 127) : (q->zp_x < 0 || q->zp_x > 255)) {
    return fail(IE_INVALID_ARGUMENT, "activation zero point outside the storage type");
  }
  const int32_t lo_lim = q->y_signed ? -128 : 0, hi_lim = q->y_signed ? 127 : 255;
  if (q->qmin < lo_lim || q->qmax > hi_lim || q->qmin > q->qmax || q->zp_y < lo_lim ||
      q->zp_y > hi_lim) {
    return fail(IE_INVALID_ARGUMENT, "output clamp range outside the storage type");
  }
  if ((rc = check_ptr(x, "x", 16)) != IE_OK) return rc;
  if ((rc = check_ptr(packed, "packed weights", 16)) != IE_OK) return rc;
  if ((rc = check_ptr(y, "y", 16)) != IE_OK) return rc;
  if (out_mode != kOutS32 && mult == nullptr) return fail(IE_INVALID_ARGUMENT, "mult is null");
  const int64_t c_store = round_up(d->c, 16);
  // A nonzero activation zero point runs on the haloed input (padding stored
  // as zp_x, see ie_cuda_q8_pack_input_halo): the same convolution with zero
  // pads over an input grown by the pads, same output extent.
  ie_conv2d_desc dh = *d;
  ie_conv2d_shape sh = s;
  if (q->zp_x != 0 && (s.pad_top | s.pad_left | s.pad_bottom | s.pad_right) != 0) {
    dh.h = d->h + s.pad_top + s.pad_bottom;
    dh.w = d->w + s.pad_left + s.pad_right;
    dh.pad_top = dh.pad_left = dh.pad_bottom = dh.pad_right = 0;
    dh.auto_pad = IE_PAD_NOTSET;
    if ((rc = resolve(&dh, -1, &sh)) != IE_OK) return rc;
    if (sh.out_h != s.out_h || sh.out_w != s.out_w) {
      return fail(IE_RUNTIME, "haloed geometry changed the output extent");
    }
  }
  IgemmSetup su;
  if ((rc = setup_igemm(&dh, sh, 1, c_store, x, packed, &su, out_mode != kOutS32)) != IE_OK) {
    return rc;
  }
  IgemmArgs& a = su.args;
  a.bias_i32 = bias;
  a.zp_x = q->zp_x;
  a.wsum = q->zp_x != 0 ? reinterpret_cast<const int32_t*>(static_cast<const uint8_t*>(packed) +
                                                           q8_packed_body_bytes(d))
                        : nullptr;
  a.mult = mult;
  a.zp_y = q->zp_y;
  a.qmin = q->qmin;
  a.qmax = q->qmax;
  a.out_mode = out_mode == kOutS32 ? kOutS32 : (q->y_signed ? kOutS8 : kOutU8);
  a.y = y;
  a.y_ld = round_up(d->m, 16);
  if (a.out_mode == kOutU8 || a.out_mode == kOutS8) {
    // the store warp writes each staged tile as panels of up to 128 channels
    // x 128 * m_sub rows
    const int panel = std::min(su.v.bn, 128);
    if (a.halo) {
      // rows_t output rows x wp positions per tile; positions past out_w are
      // outside the tensor and the TMA store skips them
      rc = encode_nhwc_4d(&su.ty, y, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, d->n, s.out_h, s.out_w,
                          a.y_ld, panel, a.wp, a.rows_t);
    } else {
      rc = encode_2d(&su.ty, y, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.m_total, a.y_ld, panel,
                     128 * su.v.m_sub);
    }
    if (rc != IE_OK) {
      return rc;
    }
  } else {
    su.ty = su.tb;  // not read by the kernel in this output mode
  }
  return launch_setup(su, q->x_signed != 0, as_stream(stream));
}

int grid_1d(int64_t total, int block) {
  return static_cast<int>(std::min<int64_t>(ceil_div(total, block), int64_t{1} << 30));
}

}  // namespace

// ======================================================= no-allocation path
//
// Scratch for ie_cuda_conv2d_f32_noalloc: a fixed array in the library's own
// device image, so that entry point never allocates.  Every GPU that loads
// the library holds it until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t{16} << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// Result words of the bounded-wait self-test (state, nanoseconds waited).
static __device__ uint64_t g_probe_out[2];

namespace {

// Device address of g_noalloc_scratch on each device.  In host code the
// array's name is only a host-side stand-in, so the address must come from
// cudaGetSymbolAddress with that device current; it is looked up on the first
// call made on each device and cached.
std::mutex g_noalloc_mutex;
void* g_noalloc_addr[kMaxDevices] = {};

int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(IE_RUNTIME, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(IE_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      return fail(IE_RUNTIME, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    }
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return IE_OK;
}

}  // namespace

// ===================================================================== ABI

extern "C" {

int ie_conv2d_resolve(const ie_conv2d_desc* desc, int64_t bias_len, ie_conv2d_shape* out) {
  return resolve(desc, bias_len, out);
}

const char* ie_cuda_last_error(void) { return g_last_error.c_str(); }

int ie_cuda_set_tile_policy(int32_t policy, int32_t* previous) {
  if (policy != IE_TILE_FILL && policy != IE_TILE_DEFAULT) {
    return fail(IE_INVALID_ARGUMENT, "unknown tile policy %d", policy);
  }
  const int32_t old = g_tile_policy.exchange(policy);
  if (previous != nullptr) *previous = old;
  return IE_OK;
}

int ie_cuda_last_plan(ie_conv_plan* out) {
  if (out == nullptr) return fail(IE_INVALID_ARGUMENT, "null plan");
  *out = g_last_plan;
  return IE_OK;
}

uint64_t ie_cuda_launch_count(int reset) {
  const uint64_t v = g_launches;
  if (reset) g_launches = 0;
  return v;
}

int ie_cuda_take_device_error(uint32_t* code) {
  unsigned int v = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail(IE_RUNTIME, "cudaDeviceSynchronize: %s", cudaGetErrorString(e));
  e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v));
  if (e != cudaSuccess) return fail(IE_RUNTIME, "read error word: %s", cudaGetErrorString(e));
  const unsigned int zero = 0;
  e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
  if (e != cudaSuccess) return fail(IE_RUNTIME, "clear error word: %s", cudaGetErrorString(e));
  if (code != nullptr) *code = v;
  return IE_OK;
}

// -------------------------------------------------------------- int8

size_t ie_cuda_q8_packed_weight_bytes(const ie_conv2d_desc* desc) {
  if (desc == nullptr || desc->m <= 0) return 0;
  return static_cast<size_t>(q8_packed_body_bytes(desc) + 4 * round_up(desc->m, 16));
}

int ie_cuda_q8_pack_weights(const ie_conv2d_desc* desc, const int8_t* w, void* packed,
                            void* stream) {
  ie_conv2d_shape s;
  int rc = resolve(desc, -1, &s);
  if (rc != IE_OK) return rc;
  if ((rc = check_dense(desc)) != IE_OK) return rc;
  if (w == nullptr || packed == nullptr) return fail(IE_INVALID_ARGUMENT, "null pointer");
  int64_t taps, ck;
  packed_geom(desc, 1, &taps, &ck);
  const int64_t total = desc->m * taps * ck;
  pack_weights_q8<<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(
      w, static_cast<int8_t*>(packed), static_cast<int32_t>(desc->m),
      static_cast<int32_t>(desc->c), static_cast<int32_t>(taps), static_cast<int32_t>(ck));
  if ((rc = check_launch("pack_weights_q8")) != IE_OK) return rc;
  if ((rc = q8_write_weight_sums(desc, packed, as_stream(stream))) != IE_OK) return rc;
  mark_weights_packed(as_stream(stream));
  return IE_OK;
}

int ie_cuda_q8_pack_input(const void* x_nchw, void* x_nhwc, int64_t n, int64_t c, int64_t h,
                          int64_t w, int64_t c_store, int32_t xor_mask, void* stream) {
  if (x_nchw == nullptr || x_nhwc == nullptr) return fail(IE_INVALID_ARGUMENT, "null pointer");
  if (n <= 0 || c <= 0 || h <= 0 || w <= 0 || c_store < c) {
    return fail(IE_INVALID_ARGUMENT, "bad activation shape");
  }
  const int64_t hw = h * w;
  dim3 grid(static_cast<unsigned>(ceil_div(hw, 32)), static_cast<unsigned>(ceil_div(c_store, 32)),
            static_cast<unsigned>(n));
  if (grid.z > 65535 || grid.y > 65535) return fail(IE_UNSUPPORTED, "batch or channels too large");
  pack_nchw_to_nhwc_u8<<<grid, dim3(32, 8), 0, as_stream(stream)>>>(
      static_cast<const uint8_t*>(x_nchw), static_cast<uint8_t*>(x_nhwc),
      static_cast<int32_t>(c), hw, static_cast<int32_t>(c_store),
      static_cast<uint8_t>(xor_mask & 0xFF));
  return check_launch("pack_nchw_to_nhwc_u8");
}

int ie_cuda_q8_unpack_output(const void* y_nhwc, void* y_nchw, int64_t n, int64_t c,
                             int64_t h, int64_t w, int64_t c_store, void* stream) {
  if (y_nhwc == nullptr || y_nchw == nullptr) return fail(IE_INVALID_ARGUMENT, "null pointer");
  if (n <= 0 || c <= 0 || h <= 0 || w <= 0 || c_store < c) {
    return fail(IE_INVALID_ARGUMENT, "bad activation shape");
  }
  const int64_t hw = h * w;
  dim3 grid(static_cast<unsigned>(ceil_div(hw, 32)), static_cast<unsigned>(ceil_div(c, 32)),
            static_cast<unsigned>(n));
  if (grid.z > 65535 || grid.y > 65535) return fail(IE_UNSUPPORTED, "batch or channels too large");
  unpack_nhwc_to_nchw_u8<<<grid, dim3(32, 8), 0, as_stream(stream)>>>(
      static_cast<const uint8_t*>(y_nhwc), static_cast<uint8_t*>(y_nchw),
      static_cast<int32_t>(c), hw, static_cast<int32_t>(c_store));
  return check_launch("unpack_nhwc_to_nchw_u8");
}

size_t ie_cuda_q8_halo_input_bytes(const ie_conv2d_desc* desc) {
  ie_conv2d_shape s;
  if (desc == nullptr || resolve(desc, -1, &s) != IE_OK) return 0;
  return static_cast<size_t>(desc->n * (desc->h + s.pad_top + s.pad_bottom) *
                             (desc->w + s.pad_left + s.pad_right) * round_up(desc->c, 16));
}

int ie_cuda_q8_pack_input_halo(const ie_conv2d_desc* desc, const void* x_nchw, void* x_halo,
                               int32_t zp_x, void* stream) {
  ie_conv2d_shape s;
  int rc = resolve(desc, -1, &s);
  if (rc != IE_OK) return rc;
  if (x_nchw == nullptr || x_halo == nullptr) return fail(IE_INVALID_ARGUMENT, "null pointer");
  if (zp_x < -128 || zp_x > 255) return fail(IE_INVALID_ARGUMENT, "zero point outside 8 bits");
  const int64_t hp = desc->h + s.pad_top + s.pad_bottom, wp = desc->w + s.pad_left + s.pad_right;
  const int64_t c_store = round_up(desc->c, 16);
  if (hp > INT32_MAX || wp > INT32_MAX || hp * wp > (int64_t{1} << 40)) {
    return fail(IE_UNSUPPORTED, "activation too large");
  }
  dim3 grid(static_cast<unsigned>(ceil_div(hp * wp, 32)), static_cast<unsigned>(ceil_div(c_store, 32)),
            static_cast<unsigned>(desc->n));
  if (grid.z > 65535 || grid.y > 65535) return fail(IE_UNSUPPORTED, "batch or channels too large");
  pack_nchw_to_nhwc_halo_u8<<<grid, dim3(32, 8), 0, as_stream(stream)>>>(
      static_cast<const uint8_t*>(x_nchw), static_cast<uint8_t*>(x_halo),
      static_cast<int32_t>(desc->c), static_cast<int32_t>(desc->h), static_cast<int32_t>(desc->w),
      static_cast<int32_t>(c_store), static_cast<int32_t>(s.pad_top),
      static_cast<int32_t>(s.pad_left), static_cast<int32_t>(hp), static_cast<int32_t>(wp),
      static_cast<uint8_t>(zp_x & 0xFF));
  return check_launch("pack_nchw_to_nhwc_halo_u8");
}

int ie_cuda_q8_halo_nhwc(const ie_conv2d_desc* desc, const void* x_nhwc, void* x_halo,
                         int32_t zp_x, void* stream) {
  ie_conv2d_shape s;
  int rc = resolve(desc, -1, &s);
  if (rc != IE_OK) return rc;
  if ((rc = check_ptr(x_nhwc, "x", 16)) != IE_OK) return rc;
  if ((rc = check_ptr(x_halo, "x_halo", 16)) != IE_OK) return rc;
  if (zp_x < -128 || zp_x > 255) return fail(IE_INVALID_ARGUMENT, "zero point outside 8 bits");
  const int64_t hp = desc->h + s.pad_top + s.pad_bottom, wp = desc->w + s.pad_left + s.pad_right;
  if (hp > INT32_MAX || wp > INT32_MAX || desc->n > INT32_MAX) {
    return fail(IE_UNSUPPORTED, "activation too large");
  }
  const int64_t c_store = round_up(desc->c, 16);
  const int64_t total = desc->n * hp * wp * (c_store / 16);
  halo_nhwc_u8<<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(
      static_cast<const uint8_t*>(x_nhwc), static_cast<uint8_t*>(x_halo),
      static_cast<int32_t>(desc->n), static_cast<int32_t>(desc->h), static_cast<int32_t>(desc->w),
      static_cast<int32_t>(c_store), static_cast<int32_t>(s.pad_top),
      static_cast<int32_t>(s.pad_left), static_cast<int32_t>(hp), static_cast<int32_t>(wp),
      static_cast<uint8_t>(zp_x & 0xFF));
  return check_launch("halo_nhwc_u8");
}

int ie_cuda_conv2d_q8(const ie_conv2d_desc* desc, const ie_q8_params* q, const void* x,
                      const void* packed, const int32_t* bias, const float* mult, void* y,
                      void* stream) {
  return run_q8(desc, q, x, packed, bias, mult, y, kOutU8, stream);
}

int ie_cuda_conv2d_q8_acc(const ie_conv2d_desc* desc, const ie_q8_params* q, const void* x,
                          const void* packed, const int32_t* bias, int32_t* y, void* stream) {
  return run_q8(desc, q, x, packed, bias, nullptr, y, kOutS32, stream);
}

size_t ie_cuda_dw_q8_packed_weight_bytes(const ie_conv2d_desc* desc) {
  if (desc == nullptr) return 0;
  return static_cast<size_t>(desc->kh * desc->kw * round_up(desc->c, 16));
}

int ie_cuda_dw_q8_pack_weights(const ie_conv2d_desc* desc, const int8_t* w, void* packed,
                               void* stream) {
  ie_conv2d_shape s;
  int rc = resolve(desc, -1, &s);
  if (rc != IE_OK) return rc;
  if (desc->group != desc->c || desc->m != desc->c) {
    return fail(IE_UNSUPPORTED, "depthwise path needs group == c == m");
  }
  if (w == nullptr || packed == nullptr) return fail(IE_INVALID_ARGUMENT, "null pointer");
  const int64_t taps = desc->kh * desc->kw, cs = round_up(desc->c, 16);
  pack_dw_weights_q8<<<grid_1d(taps * cs, 256), 256, 0, as_stream(stream)>>>(
      w, static_cast<int8_t*>(packed), static_cast<int32_t>(desc->c),
      static_cast<int32_t>(taps), static_cast<int32_t>(cs));
  return check_launch("pack_dw_weights_q8");
}

int ie_cuda_dwconv2d_q8(const ie_conv2d_desc* desc, const ie_q8_params* q, const void* x,
                        const void* packed, const int32_t* bias, const float* mult, void* y,
                        void* stream) {
  ie_conv2d_shape s;
  int rc = resolve(desc, -1, &s);
  if (rc != IE_OK) return rc;
  if (desc->group != desc->c || desc->m != desc->c) {
    return fail(IE_UNSUPPORTED, "depthwise path needs group == c == m");
  }
  if (q == nullptr || mult == nullptr) return fail(IE_INVALID_ARGUMENT, "null parameters");
  if ((rc = check_ptr(x, "x", 16)) != IE_OK) return rc;
  if ((rc = check_ptr(packed, "packed weights", 16)) != IE_OK) return rc;
  if ((rc = check_ptr(y, "y", 16)) != IE_OK) return rc;
  const int32_t lo_lim = q->y_signed ? -128 : 0, hi_lim = q->y_signed ? 127 : 255;
  if (q->qmin < lo_lim || q->qmax > hi_lim || q->qmin > q->qmax) {
    return fail(IE_INVALID_ARGUMENT, "output clamp range outside the storage type");
  }
  const bool zp_fits = q->x_signed ? (q->zp_x >= -128 && q->zp_x <= 127)
                                   : (q->zp_x >= 0 && q->zp_x <= 255);
  if (desc->kh == 3 && desc->kw == 3 && desc->dil_h == 1 && desc->dil_w == 1 &&
      desc->stride_h == desc->stride_w && (desc->stride_h == 1 || desc->stride_h == 2) &&
      zp_fits && desc->n <= 65535 && s.out_h <= 65535 && desc->h <= INT32_MAX &&
      desc->w * round_up(desc->c, 16) <= INT32_MAX &&
      ceil_div(s.out_w, 4) * round_up(desc->c, 16) / 4 <= INT32_MAX) {
    // 3x3, stride 1 or 2: the packed-byte (dp4a) row kernel
    Dw3Args a;
    a.n = static_cast<int32_t>(desc->n);
    a.h = static_cast<int32_t>(desc->h);
    a.w = static_cast<int32_t>(desc->w);
    a.c_store = static_cast<int32_t>(round_up(desc->c, 16));
    a.out_h = static_cast<int32_t>(s.out_h);
    a.out_w = static_cast<int32_t>(s.out_w);
    a.pad_t = static_cast<int32_t>(s.pad_top);
    a.pad_l = static_cast<int32_t>(s.pad_left);
    a.c = static_cast<int32_t>(desc->c);
    a.zp_x = q->zp_x;
    a.zp4 = 0x01010101u * static_cast<uint32_t>(q->zp_x & 0xFF);
    a.zp_y = q->zp_y;
    a.qmin = q->qmin;
    a.qmax = q->qmax;
    a.words = a.c_store / 4;
    a.col_groups = static_cast<int32_t>(ceil_div(s.out_w, 4));
    // Output rows per thread: long chunks amortise each thread's set-up and
    // re-read fewer input rows (measured: chunks of 2 rows made the 28x28 and
    // 14x14 MobileNetV2 layers 15-20% slower than chunks of 8); layers with
    // many rows per image get up to 16 while there are about
    // kDwTargetThreads threads.
    constexpr int64_t kDwTargetThreads = int64_t{148} * 128 * kDwMinBlocks * 4;
    const int64_t per_row = desc->n * a.col_groups * a.words;
    a.chunk = static_cast<int32_t>(std::min<int64_t>(
        s.out_h, std::clamp<int64_t>(s.out_h * per_row / kDwTargetThreads, 8, 16)));
    a.chunks = static_cast<int32_t>(ceil_div(s.out_h, a.chunk));
    const auto xp = static_cast<const uint8_t*>(x);
    const auto wpk = static_cast<const int8_t*>(packed);
    const auto yp = static_cast<uint8_t*>(y);
    const dim3 grid(static_cast<unsigned>(ceil_div(int64_t{a.col_groups} * a.words, 128)),
                    static_cast<unsigned>(a.chunks), static_cast<unsigned>(desc->n));
    const cudaStream_t st = as_stream(stream);
    const int sel = (desc->stride_h == 2 ? 4 : 0) + (q->x_signed ? 2 : 0) + (q->y_signed ? 1 : 0);
    switch (sel) {
      case 0: dwconv3x3_q8_nhwc<1, false, false><<<grid, 128, 0, st>>>(xp, wpk, bias, mult, yp, a); break;
      case 1: dwconv3x3_q8_nhwc<1, false, true><<<grid, 128, 0, st>>>(xp, wpk, bias, mult, yp, a); break;
      case 2: dwconv3x3_q8_nhwc<1, true, false><<<grid, 128, 0, st>>>(xp, wpk, bias, mult, yp, a); break;
      case 3: dwconv3x3_q8_nhwc<1, true, true><<<grid, 128, 0, st>>>(xp, wpk, bias, mult, yp, a); break;
      case 4: dwconv3x3_q8_nhwc<2, false, false><<<grid, 128, 0, st>>>(xp, wpk, bias, mult, yp, a); break;
      case 5: dwconv3x3_q8_nhwc<2, false, true><<<grid, 128, 0, st>>>(xp, wpk, bias, mult, yp, a); break;
      case 6: dwconv3x3_q8_nhwc<2, true, false><<<grid, 128, 0, st>>>(xp, wpk, bias, mult, yp, a); break;
      default: dwconv3x3_q8_nhwc<2, true, true><<<grid, 128, 0, st>>>(xp, wpk, bias, mult, yp, a); break;
    }
    return check_launch("dwconv3x3_q8_nhwc");
  }
  DwArgs a;
  a.n = static_cast<int32_t>(desc->n);
  a.h = static_cast<int32_t>(desc->h);
  a.w = static_cast<int32_t>(desc->w);
  a.c_store = static_cast<int32_t>(round_up(desc->c, 16));
  a.out_h = static_cast<int32_t>(s.out_h);
  a.out_w = static_cast<int32_t>(s.out_w);
  a.kh = static_cast<int32_t>(desc->kh);
  a.kw = static_cast<int32_t>(desc->kw);
  a.stride_h = static_cast<int32_t>(desc->stride_h);
  a.stride_w = static_cast<int32_t>(desc->stride_w);
  a.dil_h = static_cast<int32_t>(desc->dil_h);
  a.dil_w = static_cast<int32_t>(desc->dil_w);
  a.pad_t = static_cast<int32_t>(s.pad_top);
  a.pad_l = static_cast<int32_t>(s.pad_left);
  a.c = static_cast<int32_t>(desc->c);
  a.x_signed = q->x_signed;
  a.zp_x = q->zp_x;
  a.zp_y = q->zp_y;
  a.qmin = q->qmin;
  a.qmax = q->qmax;
  const int64_t total = desc->n * s.out_h * s.out_w * (a.c_store / 16);
  dwconv_q8_nhwc<<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(
      static_cast<const uint8_t*>(x), static_cast<const int8_t*>(packed), bias, mult,
      static_cast<uint8_t*>(y), a);
  return check_launch("dwconv_q8_nhwc");
}

// -------------------------------------------------------------- stem

int ie_cuda_q8_stem_desc(int64_t n, int64_t c, int64_t h, int64_t w, int64_t m,
                         ie_conv2d_desc* out) {
  if (out == nullptr) return fail(IE_INVALID_ARGUMENT, "null descriptor");
  if (n <= 0 || c <= 0 || c > 4 || h <= 0 || w <= 0 || h % 2 || w % 2 || m <= 0) {
    return fail(IE_UNSUPPORTED, "stem re-layout needs 1 <= c <= 4 and even h, w");
  }
  std::memset(out, 0, sizeof(*out));
  out->n = n;
  out->c = 64;
  out->h = h / 2;
  out->w = w / 2;
  out->m = m;
  out->kh = 4;
  out->kw = 1;
  out->stride_h = out->stride_w = 1;
  out->dil_h = out->dil_w = 1;
  out->pad_top = 2;
  out->pad_bottom = 1;
  out->group = 1;
  return IE_OK;
}

int ie_cuda_q8_stem_pack_input(const void* x_nchw, void* x_packed, int64_t n, int64_t c,
                               int64_t h, int64_t w, int32_t xor_mask, void* stream) {
  ie_conv2d_desc d;
  int rc = ie_cuda_q8_stem_desc(n, c, h, w, 1, &d);
  if (rc != IE_OK) return rc;
  if (x_nchw == nullptr) return fail(IE_INVALID_ARGUMENT, "null pointer");
  if ((rc = check_ptr(x_packed, "x_packed", 16)) != IE_OK) return rc;
  const int64_t blocks = n * (h / 2);
  const size_t smem = static_cast<size_t>(c * 2 * stem_row_stride(static_cast<int>(w)));
  if (blocks > INT32_MAX || w > 2048 || smem > 48 * 1024) {
    return fail(IE_UNSUPPORTED, "stem input too large");
  }
  // threads walk the 16-byte chunks of an output row (4 per pixel); blocks of
  // at most 128 threads keep ~12 blocks per SM in flight, which hides the
  // latency of each block's input-row loads (448-thread blocks, one per
  // chunk of a 224-wide image, ran 3x slower)
  const int threads = static_cast<int>(std::min<int64_t>(128, ((w / 2 * 4 + 31) / 32) * 32));
  const auto xp = static_cast<const uint8_t*>(x_nchw);
  const auto yp = static_cast<uint8_t*>(x_packed);
  const auto hh = static_cast<int32_t>(h), ww = static_cast<int32_t>(w);
  const auto m8 = static_cast<uint8_t>(xor_mask & 0xFF);
  const dim3 grid(static_cast<unsigned>(blocks));
  switch (c) {
    case 1: stem_pack_s2d_u8<1><<<grid, threads, smem, as_stream(stream)>>>(xp, yp, hh, ww, m8); break;
    case 2: stem_pack_s2d_u8<2><<<grid, threads, smem, as_stream(stream)>>>(xp, yp, hh, ww, m8); break;
    case 3: stem_pack_s2d_u8<3><<<grid, threads, smem, as_stream(stream)>>>(xp, yp, hh, ww, m8); break;
    default: stem_pack_s2d_u8<4><<<grid, threads, smem, as_stream(stream)>>>(xp, yp, hh, ww, m8); break;
  }
  return check_launch("stem_pack_s2d_u8");
}

int ie_cuda_q8_stem_pack_weights(const int8_t* w, void* packed, int64_t m, int64_t c,
                                 void* stream) {
  if (w == nullptr || packed == nullptr) return fail(IE_INVALID_ARGUMENT, "null pointer");
  if (m <= 0 || c <= 0 || c > 4) return fail(IE_UNSUPPORTED, "stem re-layout needs 1 <= c <= 4");
  const int64_t total = m * 4 * 64;
  stem_pack_weights_q8<<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(
      w, static_cast<int8_t*>(packed), static_cast<int32_t>(m), static_cast<int32_t>(c));
  int rc = check_launch("stem_pack_weights_q8");
  if (rc != IE_OK) return rc;
  ie_conv2d_desc d;
  if ((rc = ie_cuda_q8_stem_desc(1, c, 2, 2, m, &d)) != IE_OK) return rc;
  if ((rc = q8_write_weight_sums(&d, packed, as_stream(stream))) != IE_OK) return rc;
  mark_weights_packed(as_stream(stream));
  return IE_OK;
}

namespace {

// The row-walking 3x3 / stride-2 pool: 4 output rows per thread (oh, ow and
// the arguments already checked to fit int32; pad < 3 keeps every window's
// first row and column inside the image).
int launch_maxpool3x3s2(const void* x, void* y, int64_t n, int64_t h, int64_t w,
                        int64_t c_store, int64_t oh, int64_t ow, int64_t pad, int32_t is_signed,
                        void* stream) {
  constexpr int64_t kRows = 4;
  const int64_t chunks = ceil_div(oh, kRows);
  const int64_t total = n * chunks * ow * (c_store / 16);
  const auto xp = static_cast<const uint8_t*>(x);
  const auto yp = static_cast<uint8_t*>(y);
  const auto nn = static_cast<int32_t>(n), hh = static_cast<int32_t>(h), ww = static_cast<int32_t>(w),
             cs = static_cast<int32_t>(c_store), ohh = static_cast<int32_t>(oh),
             oww = static_cast<int32_t>(ow), pp = static_cast<int32_t>(pad),
             rr = static_cast<int32_t>(kRows), ch = static_cast<int32_t>(chunks);
  if (is_signed) {
    maxpool3x3s2_q8_nhwc<true><<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(
        xp, yp, nn, hh, ww, cs, ohh, oww, pp, rr, ch);
  } else {
    maxpool3x3s2_q8_nhwc<false><<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(
        xp, yp, nn, hh, ww, cs, ohh, oww, pp, rr, ch);
  }
  return check_launch("maxpool3x3s2_q8_nhwc");
}

}  // namespace

int ie_cuda_q8_maxpool2d(const void* x, void* y, int64_t n, int64_t h, int64_t w,
                         int64_t c_store, int64_t k, int64_t stride, int64_t pad,
                         int32_t is_signed, void* stream) {
  int rc;
  if ((rc = check_ptr(x, "x", 16)) != IE_OK) return rc;
  if ((rc = check_ptr(y, "y", 16)) != IE_OK) return rc;
  if (n <= 0 || h <= 0 || w <= 0 || c_store <= 0 || c_store % 16 || k <= 0 || stride <= 0 ||
      pad < 0 || pad >= k) {
    return fail(IE_INVALID_ARGUMENT, "bad pooling shape");
  }
  const int64_t oh = (h + 2 * pad - k) / stride + 1, ow = (w + 2 * pad - k) / stride + 1;
  if (oh <= 0 || ow <= 0) return fail(IE_INVALID_ARGUMENT, "pooling produces an empty output");
  if (n > INT32_MAX || h > INT32_MAX || w > INT32_MAX || c_store > INT32_MAX || k > INT32_MAX ||
      stride > INT32_MAX || (oh - 1) * stride > INT32_MAX || (ow - 1) * stride > INT32_MAX) {
    return fail(IE_UNSUPPORTED, "pooling extent too large");
  }
  if (k == 3 && stride == 2) {
    return launch_maxpool3x3s2(x, y, n, h, w, c_store, oh, ow, pad, is_signed, stream);
  }
  const int64_t total = n * oh * ow * (c_store / 16);
  const auto xp = static_cast<const uint8_t*>(x);
  const auto yp = static_cast<uint8_t*>(y);
  const auto nn = static_cast<int32_t>(n), hh = static_cast<int32_t>(h), ww = static_cast<int32_t>(w),
             cs = static_cast<int32_t>(c_store), ohh = static_cast<int32_t>(oh),
             oww = static_cast<int32_t>(ow), kk = static_cast<int32_t>(k),
             ss = static_cast<int32_t>(stride), pp = static_cast<int32_t>(pad);
  if (is_signed) {
    maxpool_q8_nhwc<true><<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(
        xp, yp, nn, hh, ww, cs, ohh, oww, kk, ss, pp);
  } else {
    maxpool_q8_nhwc<false><<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(
        xp, yp, nn, hh, ww, cs, ohh, oww, kk, ss, pp);
  }
  return check_launch("maxpool_q8_nhwc");
}

int ie_cuda_f32x2_maxpool2d(const void* x, void* y, int64_t n, int64_t h, int64_t w,
                            int64_t c_store, int64_t k, int64_t stride, int64_t pad,
                            void* stream) {
  int rc;
  if ((rc = check_ptr(x, "x", 16)) != IE_OK) return rc;
  if ((rc = check_ptr(y, "y", 16)) != IE_OK) return rc;
  if (n <= 0 || h <= 0 || w <= 0 || c_store <= 0 || c_store % 16 || k <= 0 || stride <= 0 ||
      pad < 0 || pad >= k) {
    return fail(IE_INVALID_ARGUMENT, "bad pooling shape");
  }
  const int64_t oh = (h + 2 * pad - k) / stride + 1, ow = (w + 2 * pad - k) / stride + 1;
  if (oh <= 0 || ow <= 0) return fail(IE_INVALID_ARGUMENT, "pooling produces an empty output");
  const int64_t total = n * oh * ow * (c_store / 8);
  maxpool_f32x2_nhwc<<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(y),
      static_cast<int32_t>(n), static_cast<int32_t>(h), static_cast<int32_t>(w),
      static_cast<int32_t>(c_store), static_cast<int32_t>(oh), static_cast<int32_t>(ow),
      static_cast<int32_t>(k), static_cast<int32_t>(stride), static_cast<int32_t>(pad));
  return check_launch("maxpool_f32x2_nhwc");
}

// -------------------------------------------------------------- fp32

size_t ie_cuda_f32_packed_weight_bytes(const ie_conv2d_desc* desc) {
  if (desc == nullptr) return 0;
  int64_t taps, ck;
  packed_geom(desc, 2, &taps, &ck);
  return static_cast<size_t>(desc->m * taps * 2 * ck * 2);
}

int ie_cuda_f32_pack_weights(const ie_conv2d_desc* desc, const float* w, void* packed,
                             void* stream) {
  ie_conv2d_shape s;
  int rc = resolve(desc, -1, &s);
  if (rc != IE_OK) return rc;
  if ((rc = check_dense(desc)) != IE_OK) return rc;
  if (w == nullptr || packed == nullptr) return fail(IE_INVALID_ARGUMENT, "null pointer");
  int64_t taps, ck;
  packed_geom(desc, 2, &taps, &ck);
  const int64_t total = desc->m * taps * ck;
  pack_weights_bf16x2<<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(
      w, static_cast<__nv_bfloat16*>(packed), static_cast<int32_t>(desc->m),
      static_cast<int32_t>(desc->c), static_cast<int32_t>(taps), static_cast<int32_t>(ck));
  return check_launch("pack_weights_bf16x2");
}

int ie_cuda_f32_pack_input(const float* x_nchw, void* x_split, int64_t n, int64_t c, int64_t h,
                           int64_t w, int64_t c_store, void* stream) {
  if (x_nchw == nullptr || x_split == nullptr) return fail(IE_INVALID_ARGUMENT, "null pointer");
  if (n <= 0 || c <= 0 || h <= 0 || w <= 0 || c_store < c || c_store % 16 != 0) {
    return fail(IE_INVALID_ARGUMENT, "bad activation shape");
  }
  const int64_t hw = h * w;
  dim3 grid(static_cast<unsigned>(ceil_div(hw, 32)), static_cast<unsigned>(ceil_div(c_store, 32)),
            static_cast<unsigned>(n));
  if (grid.z > 65535 || grid.y > 65535) return fail(IE_UNSUPPORTED, "batch or channels too large");
  pack_nchw_f32_to_bf16x2<<<grid, dim3(32, 8), 0, as_stream(stream)>>>(
      x_nchw, static_cast<__nv_bfloat16*>(x_split), static_cast<int32_t>(c), hw,
      static_cast<int32_t>(c_store));
  return check_launch("pack_nchw_f32_to_bf16x2");
}

int ie_cuda_conv2d_bf16x3(const ie_conv2d_desc* desc, int32_t act, const void* x_split,
                          const void* packed, const float* bias, void* y, int32_t y_format,
                          void* stream) {
  return ie_cuda_conv2d_bf16x3_residual(desc, act, x_split, packed, bias, nullptr, y, y_format,
                                        stream);
}

int ie_cuda_conv2d_bf16x3_residual(const ie_conv2d_desc* desc, int32_t act, const void* x_split,
                                   const void* packed, const float* bias, const float* residual,
                                   void* y, int32_t y_format, void* stream) {
  ie_conv2d_shape s;
  int rc = resolve(desc, -1, &s);
  if (rc != IE_OK) return rc;
  if ((rc = check_dense(desc)) != IE_OK) return rc;
  if ((rc = check_ptr(x_split, "x", 16)) != IE_OK) return rc;
  if ((rc = check_ptr(packed, "packed weights", 16)) != IE_OK) return rc;
  if ((rc = check_ptr(y, "y", 16)) != IE_OK) return rc;
  if (act < IE_ACT_NONE || act > IE_ACT_RELU6) return fail(IE_INVALID_ARGUMENT, "bad activation");
  const int64_t c_store = round_up(desc->c, 16);
  IgemmSetup su;
  if ((rc = setup_igemm(desc, s, 2, c_store, x_split, packed, &su)) != IE_OK) return rc;
  if (residual != nullptr && y_format == IE_Y_BF16X2_NHWC) {
    return fail(IE_UNSUPPORTED, "a residual needs an fp32 output format");
  }
  IgemmArgs& a = su.args;
  a.bias_f32 = bias;
  a.residual = residual;
  a.act = act != IE_ACT_NONE;
  a.act_lo = 0.0f;
  a.act_hi = act == IE_ACT_RELU6 ? 6.0f : INFINITY;
  a.y = y;
  switch (y_format) {
    case IE_Y_F32_NHWC:
      a.out_mode = kOutF32;
      a.y_ld = round_up(desc->m, 16);
      break;
    case IE_Y_BF16X2_NHWC:
      a.out_mode = kOutBF16x2;
      a.y_ld = 2 * round_up(desc->m, 16);
      break;
    case IE_Y_F32_NCHW:
      a.out_mode = kOutF32Nchw;
      a.y_ld = 0;
      break;
    default:
      return fail(IE_INVALID_ARGUMENT, "bad output format");
  }
  su.ty = su.tb;  // fp32 outputs use direct stores; the map is not read
  return launch_setup(su, false, as_stream(stream));
}

size_t ie_cuda_conv2d_f32_workspace_bytes(const ie_conv2d_desc* desc) {
  if (desc == nullptr || desc->group != 1) return 0;
  const int64_t c_store = round_up(desc->c, 16);
  const size_t x_bytes =
      static_cast<size_t>(round_up(desc->n * desc->h * desc->w * c_store * 2 * 2, 256));
  return x_bytes + round_up(static_cast<int64_t>(ie_cuda_f32_packed_weight_bytes(desc)), 256);
}

int ie_cuda_conv2d_f32(const ie_conv2d_desc* desc, int32_t act, const float* x, const float* w,
                       const float* bias, float* y, void* workspace, size_t workspace_bytes,
                       void* stream) {
  ie_conv2d_shape s;
  int rc = resolve(desc, -1, &s);
  if (rc != IE_OK) return rc;
  if (x == nullptr || w == nullptr || y == nullptr) return fail(IE_INVALID_ARGUMENT, "null tensor");
  if (act < IE_ACT_NONE || act > IE_ACT_RELU6) return fail(IE_INVALID_ARGUMENT, "bad activation");
  if (desc->group != 1) {
    DirectF32Args a;
    a.n = static_cast<int32_t>(desc->n);
    a.c = static_cast<int32_t>(desc->c);
    a.h = static_cast<int32_t>(desc->h);
    a.w = static_cast<int32_t>(desc->w);
    a.m = static_cast<int32_t>(desc->m);
    a.cg = static_cast<int32_t>(desc->c / desc->group);
    a.kh = static_cast<int32_t>(desc->kh);
    a.kw = static_cast<int32_t>(desc->kw);
    a.stride_h = static_cast<int32_t>(desc->stride_h);
    a.stride_w = static_cast<int32_t>(desc->stride_w);
    a.dil_h = static_cast<int32_t>(desc->dil_h);
    a.dil_w = static_cast<int32_t>(desc->dil_w);
    a.pad_t = static_cast<int32_t>(s.pad_top);
    a.pad_l = static_cast<int32_t>(s.pad_left);
    a.out_h = static_cast<int32_t>(s.out_h);
    a.out_w = static_cast<int32_t>(s.out_w);
    a.group = static_cast<int32_t>(desc->group);
    a.act = act;
    a.act_lo = 0.0f;
    a.act_hi = act == IE_ACT_RELU6 ? 6.0f : INFINITY;
    const int64_t total = desc->n * desc->m * s.out_h * s.out_w;
    conv_direct_f32_nchw<<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(x, w, bias, y, a);
    return check_launch("conv_direct_f32_nchw");
  }
  const size_t need = ie_cuda_conv2d_f32_workspace_bytes(desc);
  if (workspace == nullptr || workspace_bytes < need) {
    return fail(IE_INVALID_ARGUMENT, "workspace too small: need %zu bytes", need);
  }
  if ((rc = check_ptr(workspace, "workspace", 256)) != IE_OK) return rc;
  const int64_t c_store = round_up(desc->c, 16);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* x_split = ws;
  void* packed = ws + round_up(desc->n * desc->h * desc->w * c_store * 4, 256);
  if ((rc = ie_cuda_f32_pack_input(x, x_split, desc->n, desc->c, desc->h, desc->w, c_store,
                                   stream)) != IE_OK) {
    return rc;
  }
  if ((rc = ie_cuda_f32_pack_weights(desc, w, packed, stream)) != IE_OK) return rc;
  return ie_cuda_conv2d_bf16x3(desc, act, x_split, packed, bias, y, IE_Y_F32_NCHW, stream);
}

// ------------------------------------------------------------ head ops

int ie_pool2d_resolve(const ie_pool2d_desc* d, ie_conv2d_shape* out) {
  if (d == nullptr || out == nullptr) return fail(IE_INVALID_ARGUMENT, "null descriptor");
  if (d->n <= 0 || d->c <= 0 || d->h <= 0 || d->w <= 0) {
    return fail(IE_INVALID_ARGUMENT, "Pooling expects positive dimensions");
  }
  if (d->kh <= 0 || d->kw <= 0) return fail(IE_INVALID_ARGUMENT, "kernel_shape values must be positive");
  if (d->stride_h <= 0 || d->stride_w <= 0) return fail(IE_INVALID_ARGUMENT, "strides must be positive");
  int64_t pt = d->pad_top, pl = d->pad_left, pb = d->pad_bottom, pr = d->pad_right;
  if (pt < 0 || pl < 0 || pb < 0 || pr < 0) return fail(IE_INVALID_ARGUMENT, "pads must be non-negative");
  auto same = [](int64_t in, int64_t k, int64_t s, bool lower, int64_t* b, int64_t* a) {
    const int64_t o = (in + s - 1) / s;
    const int64_t total = std::max<int64_t>(0, (o - 1) * s + k - in);
    int64_t before = total / 2, after = total - before;
    if (lower) std::swap(before, after);
    *b = before;
    *a = after;
  };
  if (d->auto_pad == IE_PAD_VALID) {
    pt = pl = pb = pr = 0;
  } else if (d->auto_pad == IE_PAD_SAME_UPPER || d->auto_pad == IE_PAD_SAME_LOWER) {
    const bool lower = d->auto_pad == IE_PAD_SAME_LOWER;
    same(d->h, d->kh, d->stride_h, lower, &pt, &pb);
    same(d->w, d->kw, d->stride_w, lower, &pl, &pr);
  } else if (d->auto_pad != IE_PAD_NOTSET) {
    return fail(IE_INVALID_ARGUMENT, "unsupported auto_pad");
  }
  const int64_t span_h = d->h + pt + pb, span_w = d->w + pl + pr;
  if (span_h < d->kh || span_w < d->kw) return fail(IE_INVALID_ARGUMENT, "Pool kernel exceeds padded input");
  int64_t oh, ow;
  if (d->ceil_mode) {
    oh = ceil_div(span_h - d->kh, d->stride_h) + 1;
    ow = ceil_div(span_w - d->kw, d->stride_w) + 1;
    if ((oh - 1) * d->stride_h >= d->h + pt) --oh;  // a last window starting in the padding
    if ((ow - 1) * d->stride_w >= d->w + pl) --ow;
  } else {
    oh = (span_h - d->kh) / d->stride_h + 1;
    ow = (span_w - d->kw) / d->stride_w + 1;
  }
  if (oh <= 0 || ow <= 0) return fail(IE_INVALID_ARGUMENT, "Pool produces an empty output");
  out->pad_top = pt;
  out->pad_left = pl;
  out->pad_bottom = pb;
  out->pad_right = pr;
  out->out_h = oh;
  out->out_w = ow;
  return IE_OK;
}

int ie_cuda_pool2d_f32(const ie_pool2d_desc* d, int32_t max_pool, const float* x, float* y,
                       void* stream) {
  ie_conv2d_shape s;
  int rc = ie_pool2d_resolve(d, &s);
  if (rc != IE_OK) return rc;
  if (x == nullptr || y == nullptr) return fail(IE_INVALID_ARGUMENT, "null tensor");
  if (d->h > INT32_MAX || d->w > INT32_MAX || d->kh > INT32_MAX || d->kw > INT32_MAX ||
      d->stride_h > INT32_MAX || d->stride_w > INT32_MAX || s.out_h * s.out_w > INT32_MAX ||
      s.pad_top + s.pad_bottom + d->h > INT32_MAX || s.pad_left + s.pad_right + d->w > INT32_MAX) {
    return fail(IE_UNSUPPORTED, "pooling extent too large");
  }
  Pool2dArgs a;
  a.planes = d->n * d->c;
  a.h = static_cast<int32_t>(d->h);
  a.w = static_cast<int32_t>(d->w);
  a.out_h = static_cast<int32_t>(s.out_h);
  a.out_w = static_cast<int32_t>(s.out_w);
  a.kh = static_cast<int32_t>(d->kh);
  a.kw = static_cast<int32_t>(d->kw);
  a.stride_h = static_cast<int32_t>(d->stride_h);
  a.stride_w = static_cast<int32_t>(d->stride_w);
  a.pad_t = static_cast<int32_t>(s.pad_top);
  a.pad_l = static_cast<int32_t>(s.pad_left);
  a.pad_b = static_cast<int32_t>(s.pad_bottom);
  a.pad_r = static_cast<int32_t>(s.pad_right);
  a.max_pool = max_pool ? 1 : 0;
  a.count_include_pad = d->count_include_pad ? 1 : 0;
  const int64_t total = a.planes * s.out_h * s.out_w;
  pool2d_f32_nchw<<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(x, y, a);
  return check_launch("pool2d_f32_nchw");
}

int ie_cuda_q8_maxpool2d_nhwc(const ie_pool2d_desc* d, int32_t is_signed, const void* x,
                              void* y, void* stream) {
  ie_conv2d_shape s;
  int rc = ie_pool2d_resolve(d, &s);
  if (rc != IE_OK) return rc;
  if ((rc = check_ptr(x, "x", 16)) != IE_OK) return rc;
  if ((rc = check_ptr(y, "y", 16)) != IE_OK) return rc;
  const int64_t c_store = round_up(d->c, 16);
  if (d->n > INT32_MAX || d->h > INT32_MAX || d->w > INT32_MAX || c_store > INT32_MAX ||
      d->kh > INT32_MAX || d->kw > INT32_MAX || d->stride_h > INT32_MAX ||
      d->stride_w > INT32_MAX || s.out_h > INT32_MAX || s.out_w > INT32_MAX ||
      s.pad_top + s.pad_bottom + d->h > INT32_MAX || s.pad_left + s.pad_right + d->w > INT32_MAX ||
      (s.out_h - 1) * d->stride_h > INT32_MAX || (s.out_w - 1) * d->stride_w > INT32_MAX) {
    return fail(IE_UNSUPPORTED, "pooling extent too large");
  }
  Q8PoolArgs a;
  a.n = static_cast<int32_t>(d->n);
  a.h = static_cast<int32_t>(d->h);
  a.w = static_cast<int32_t>(d->w);
  a.c_store = static_cast<int32_t>(c_store);
  a.out_h = static_cast<int32_t>(s.out_h);
  a.out_w = static_cast<int32_t>(s.out_w);
  a.kh = static_cast<int32_t>(d->kh);
  a.kw = static_cast<int32_t>(d->kw);
  a.stride_h = static_cast<int32_t>(d->stride_h);
  a.stride_w = static_cast<int32_t>(d->stride_w);
  a.pad_t = static_cast<int32_t>(s.pad_top);
  a.pad_l = static_cast<int32_t>(s.pad_left);
  if (a.kh == 3 && a.kw == 3 && a.stride_h == 2 && a.stride_w == 2 && a.pad_t == a.pad_l &&
      s.pad_top < 3 && s.pad_bottom < 3 && s.pad_left < 3 && s.pad_right < 3) {
    // every pad below the kernel size: each window holds an in-image pixel,
    // and its bottom / right edge clips at the image
    return launch_maxpool3x3s2(x, y, d->n, d->h, d->w, c_store, s.out_h, s.out_w, a.pad_t,
                               is_signed, stream);
  }
  const int64_t total = d->n * s.out_h * s.out_w * (c_store / 16);
  if (is_signed) {
    maxpool_q8_nhwc_any<true><<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(
        static_cast<const uint8_t*>(x), static_cast<uint8_t*>(y), a);
  } else {
    maxpool_q8_nhwc_any<false><<<grid_1d(total, 256), 256, 0, as_stream(stream)>>>(
        static_cast<const uint8_t*>(x), static_cast<uint8_t*>(y), a);
  }
  return check_launch("maxpool_q8_nhwc_any");
}

int ie_cuda_global_avg_pool_f32(const float* x, float* y, int64_t n, int64_t c, int64_t h,
                                int64_t w, void* stream) {
  if (n <= 0 || c <= 0 || h <= 0 || w <= 0) {
    return fail(IE_INVALID_ARGUMENT, "GlobalAvgPool expects positive dimensions");
  }
  if (x == nullptr || y == nullptr) return fail(IE_INVALID_ARGUMENT, "null tensor");
  const int64_t planes = n * c;
  global_avg_pool_f32<<<grid_1d(planes, 128), 128, 0, as_stream(stream)>>>(x, y, planes, h * w);
  return check_launch("global_avg_pool_f32");
}

int ie_cuda_q8_global_avg_pool_nhwc(const void* x, float* y, int64_t n, int64_t c, int64_t h,
                                    int64_t w, int32_t is_signed, int32_t zp, double scale,
                                    void* stream) {
  if (n <= 0 || c <= 0 || h <= 0 || w <= 0) {
    return fail(IE_INVALID_ARGUMENT, "GlobalAvgPool expects positive dimensions");
  }
  int rc;
  if ((rc = check_ptr(x, "x", 16)) != IE_OK) return rc;
  if (y == nullptr) return fail(IE_INVALID_ARGUMENT, "null tensor");
  const int64_t c_store = round_up(c, 16);
  if (h * w > INT32_MAX / 255 || n > INT32_MAX || c_store > INT32_MAX) {
    return fail(IE_UNSUPPORTED, "GlobalAvgPool plane too large for the int32 sums");
  }
  const int64_t warps = n * (c_store / 16);
  const auto xp = static_cast<const uint8_t*>(x);
  if (is_signed) {
    q8_global_avg_pool_nhwc<true><<<grid_1d(warps * 32, 256), 256, 0, as_stream(stream)>>>(
        xp, y, static_cast<int32_t>(n), static_cast<int32_t>(c), static_cast<int32_t>(c_store),
        h * w, zp, scale);
  } else {
    q8_global_avg_pool_nhwc<false><<<grid_1d(warps * 32, 256), 256, 0, as_stream(stream)>>>(
        xp, y, static_cast<int32_t>(n), static_cast<int32_t>(c), static_cast<int32_t>(c_store),
        h * w, zp, scale);
  }
  return check_launch("q8_global_avg_pool_nhwc");
}

namespace {

// 1x1 convolution view of a Gemm: M "pixels" of K channels against N filters.
ie_conv2d_desc gemm_as_conv(int64_t m, int64_t n, int64_t k) {
  ie_conv2d_desc d;
  std::memset(&d, 0, sizeof(d));
  d.n = m;
  d.c = k;
  d.h = d.w = 1;
  d.m = n;
  d.kh = d.kw = 1;
  d.stride_h = d.stride_w = d.dil_h = d.dil_w = 1;
  d.group = 1;
  return d;
}

int transpose(const float* in, float* out, int64_t rows, int64_t cols, cudaStream_t st) {
  if (ceil_div(rows, 32) > 65535) return fail(IE_UNSUPPORTED, "transpose: too many rows");
  const dim3 grid(static_cast<unsigned>(ceil_div(cols, 32)), static_cast<unsigned>(ceil_div(rows, 32)));
  transpose_f32<<<grid, dim3(32, 8), 0, st>>>(in, out, rows, cols);
  return check_launch("transpose_f32");
}

}  // namespace

size_t ie_cuda_gemm_f32_workspace_bytes(int64_t m, int64_t n, int64_t k, int32_t trans_a,
                                        int32_t trans_b) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  const ie_conv2d_desc d = gemm_as_conv(m, n, k);
  size_t bytes = ie_cuda_conv2d_f32_workspace_bytes(&d);
  if (trans_a) bytes += static_cast<size_t>(round_up(m * k * 4, 256));
  if (!trans_b) bytes += static_cast<size_t>(round_up(n * k * 4, 256));
  bytes += static_cast<size_t>(round_up(m * n * 4, 256));  // product before the epilogue
  return bytes;
}

int ie_cuda_gemm_f32(int64_t m, int64_t n, int64_t k, int32_t trans_a, int32_t trans_b,
                     float alpha, float beta, const float* a, const float* b, const float* c,
                     int32_t c_mode, float* y, void* workspace, size_t workspace_bytes,
                     void* stream) {
  if (m <= 0 || n <= 0 || k <= 0) return fail(IE_INVALID_ARGUMENT, "Gemm expects positive dimensions");
  if (a == nullptr || b == nullptr || y == nullptr) return fail(IE_INVALID_ARGUMENT, "null tensor");
  if (c_mode < IE_GEMM_C_NONE || c_mode > IE_GEMM_C_FULL) return fail(IE_INVALID_ARGUMENT, "bad C mode");
  if (c_mode != IE_GEMM_C_NONE && c == nullptr) return fail(IE_INVALID_ARGUMENT, "C is null");
  const size_t need = ie_cuda_gemm_f32_workspace_bytes(m, n, k, trans_a, trans_b);
  if (workspace == nullptr || workspace_bytes < need) {
    return fail(IE_INVALID_ARGUMENT, "Gemm workspace too small (%zu < %zu)", workspace_bytes, need);
  }
  const cudaStream_t st = as_stream(stream);
  const ie_conv2d_desc d = gemm_as_conv(m, n, k);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* conv_ws = ws;
  ws += round_up(static_cast<int64_t>(ie_cuda_conv2d_f32_workspace_bytes(&d)), 256);
  int rc;
  const float* a_rows = a;  // [M, K]
  if (trans_a) {
    float* t = reinterpret_cast<float*>(ws);
    ws += round_up(m * k * 4, 256);
    if ((rc = transpose(a, t, k, m, st)) != IE_OK) return rc;
    a_rows = t;
  }
  const float* b_rows = b;  // [N, K]
  if (!trans_b) {
    float* t = reinterpret_cast<float*>(ws);
    ws += round_up(n * k * 4, 256);
    if ((rc = transpose(b, t, k, n, st)) != IE_OK) return rc;
    b_rows = t;
  }
  const bool fused = c_mode == IE_GEMM_C_COLUMN && alpha == 1.0f && beta == 1.0f;
  if (fused || (c_mode == IE_GEMM_C_NONE && alpha == 1.0f)) {
    return ie_cuda_conv2d_f32(&d, IE_ACT_NONE, a_rows, b_rows, fused ? c : nullptr, y, conv_ws,
                              ie_cuda_conv2d_f32_workspace_bytes(&d), stream);
  }
  float* p = reinterpret_cast<float*>(ws);
  if ((rc = ie_cuda_conv2d_f32(&d, IE_ACT_NONE, a_rows, b_rows, nullptr, p, conv_ws,
                               ie_cuda_conv2d_f32_workspace_bytes(&d), stream)) != IE_OK) {
    return rc;
  }
  gemm_epilogue_f32<<<grid_1d(m * n, 256), 256, 0, st>>>(p, y, m, n, alpha, beta, c, c_mode);
  return check_launch("gemm_epilogue_f32");
}

int ie_cuda_conv2d_f32_residual(const ie_conv2d_desc* desc, int32_t act, const float* x,
                                const float* w, const float* bias, const float* residual,
                                float* y, void* workspace, size_t workspace_bytes, void* stream) {
  ie_conv2d_shape s;
  int rc = resolve(desc, -1, &s);
  if (rc != IE_OK) return rc;
  if (x == nullptr || w == nullptr || y == nullptr || residual == nullptr) {
    return fail(IE_INVALID_ARGUMENT, "null tensor");
  }
  if (desc->group != 1) return fail(IE_UNSUPPORTED, "residual fusion runs dense convolutions only");
  if (act < IE_ACT_NONE || act > IE_ACT_RELU6) return fail(IE_INVALID_ARGUMENT, "bad activation");
  const size_t need = ie_cuda_conv2d_f32_workspace_bytes(desc);
  if (workspace == nullptr || workspace_bytes < need) {
    return fail(IE_INVALID_ARGUMENT, "workspace too small (%zu < %zu)", workspace_bytes, need);
  }
  const int64_t c_store = round_up(desc->c, 16);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* x_split = ws;
  void* packed = ws + round_up(desc->n * desc->h * desc->w * c_store * 4, 256);
  if ((rc = ie_cuda_f32_pack_input(x, x_split, desc->n, desc->c, desc->h, desc->w, c_store,
                                   stream)) != IE_OK) {
    return rc;
  }
  if ((rc = ie_cuda_f32_pack_weights(desc, w, packed, stream)) != IE_OK) return rc;
  return ie_cuda_conv2d_bf16x3_residual(desc, act, x_split, packed, bias, residual, y,
                                        IE_Y_F32_NCHW, stream);
}

int ie_cuda_qadd(const ie_qadd_params* p, const void* a, const void* b, void* y, int64_t count,
                 void* stream) {
  if (p == nullptr) return fail(IE_INVALID_ARGUMENT, "null parameters");
  if (count < 0) return fail(IE_INVALID_ARGUMENT, "negative element count");
  if (count == 0) return IE_OK;
  if (a == nullptr || b == nullptr || y == nullptr) return fail(IE_INVALID_ARGUMENT, "null tensor");
  auto in_type = [](int32_t sgn, int32_t v) { return sgn ? (v >= -128 && v <= 127) : (v >= 0 && v <= 255); };
  if (!in_type(p->a_signed, p->zp_a) || !in_type(p->b_signed, p->zp_b)) {
    return fail(IE_INVALID_ARGUMENT, "input zero point outside its storage type");
  }
  const int32_t lo = p->y_signed ? -128 : 0, hi = p->y_signed ? 127 : 255;
  if (p->qmin < lo || p->qmax > hi || p->qmin > p->qmax || !in_type(p->y_signed, p->zp_y)) {
    return fail(IE_INVALID_ARGUMENT, "output clamp range outside the storage type");
  }
  if (!std::isfinite(p->mult_a) || !std::isfinite(p->mult_b)) {
    return fail(IE_INVALID_ARGUMENT, "multipliers must be finite");
  }
  // host split of the fp32 multipliers (the same rule as split_multiplier)
  auto split = [](float m, long long* mant, int* shift) {
    if (m == 0.0f) {
      *mant = 0;
      *shift = 32;
      return;
    }
    int e = 0;
    const double f = std::frexp(static_cast<double>(m), &e);
    *mant = static_cast<long long>(std::ldexp(f, 31));
    *shift = 31 - e;
  };
  long long ma, mb;
  int sa, sb;
  split(p->mult_a, &ma, &sa);
  split(p->mult_b, &mb, &sb);
  if (ma == 0) sa = sb;
  if (mb == 0) sb = sa;
  const int sh = std::max(sa, sb);
  if (sh - std::min(sa, sb) > 60) {
    return fail(IE_UNSUPPORTED, "multipliers more than 2^60 apart");
  }
  QAddArgs k;
  k.count = count;
  k.ma = ma;
  k.mb = mb;
  k.da = sh - sa;
  k.db = sh - sb;
  k.s = sh;
  k.zp_a = p->zp_a;
  k.zp_b = p->zp_b;
  k.zp_y = p->zp_y;
  k.qmin = p->qmin;
  k.qmax = p->qmax;
  k.a_signed = p->a_signed;
  k.b_signed = p->b_signed;
  k.y_signed = p->y_signed;
  const bool vec = count % 16 == 0 && reinterpret_cast<uintptr_t>(a) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(b) % 16 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0;
  const int64_t work = vec ? count / 16 : count;
  const int blocks = static_cast<int>(std::min<int64_t>(ceil_div(work, 256), int64_t{num_sms()} * 16));
  // 64-bit arithmetic is exact when each term stays below 2^61 and the
  // rounding shift is in [1, 62]
  const bool narrow = k.da <= 22 && k.db <= 22 && k.s >= 1 && k.s <= 62;
  if (vec && count >= (int64_t{1} << 22)) {
    // large tensors: the 64 KB table per block pays for itself
    auto lut_kern = narrow ? qadd_lut_u8<false> : qadd_lut_u8<true>;
    cudaFuncSetAttribute(lut_kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kQAddLutBytes);
    const int64_t chunks = count / 16;
    const int lut_blocks = static_cast<int>(std::min<int64_t>(ceil_div(chunks, kQAddLutThreads), num_sms()));
    lut_kern<<<lut_blocks, kQAddLutThreads, kQAddLutBytes, as_stream(stream)>>>(
        static_cast<const uint4*>(a), static_cast<const uint4*>(b), static_cast<uint4*>(y), k, chunks);
    return check_launch("qadd_lut_u8");
  }
  auto kern = narrow ? qadd_u8<false> : qadd_u8<true>;
  kern<<<blocks, 256, 0, as_stream(stream)>>>(static_cast<const uint8_t*>(a),
                                             static_cast<const uint8_t*>(b),
                                             static_cast<uint8_t*>(y), k, vec ? 1 : 0);
  return check_launch("qadd_u8");
}

int ie_cuda_bounded_wait_probe(uint64_t wait_limit_ns, uint64_t* waited_ns, void* stream) {
  if (wait_limit_ns < 1000 || wait_limit_ns > 2000000000ull) {
    return fail(IE_INVALID_ARGUMENT, "wait limit must lie in [1 us, 2 s]");
  }
  void* out = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&out, g_probe_out);
  if (e != cudaSuccess) return fail(IE_RUNTIME, "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
  const cudaStream_t st = as_stream(stream);
  bounded_wait_probe<<<1, 64, 0, st>>>(wait_limit_ns, static_cast<uint64_t*>(out));
  int rc = check_launch("bounded_wait_probe");
  if (rc != IE_OK) return rc;
  uint64_t host[2] = {0, 0};
  e = cudaMemcpyAsync(host, out, sizeof(host), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return fail(IE_RUNTIME, "bounded_wait_probe: %s", cudaGetErrorString(e));
  if (waited_ns != nullptr) *waited_ns = host[1];
  if (host[0] != 2) return fail(IE_RUNTIME, "the probe's wait did not give up (state %llu)",
                                static_cast<unsigned long long>(host[0]));
  return IE_OK;
}

int ie_cuda_mma_i8_peak(int32_t iters, double* tops, void* stream) {
  if (tops == nullptr) return fail(IE_INVALID_ARGUMENT, "null output");
  if (iters < 1000 || iters > 10000000) return fail(IE_INVALID_ARGUMENT, "iters must lie in [1000, 1e7]");
  const cudaStream_t st = as_stream(stream);
  const int sms = num_sms();
  cudaEvent_t ev[2] = {nullptr, nullptr};
  cudaError_t e = cudaEventCreate(&ev[0]);
  if (e == cudaSuccess) e = cudaEventCreate(&ev[1]);
  if (e != cudaSuccess) {
    if (ev[0] != nullptr) cudaEventDestroy(ev[0]);
    return fail(IE_RUNTIME, "cudaEventCreate: %s", cudaGetErrorString(e));
  }
  int rc = IE_OK;
  // one untimed launch (clocks up, code loaded), then the timed one
  mma_i8_peak<<<sms, 128, 0, st>>>(1000u, kWaitLimitNs);
  rc = check_launch("mma_i8_peak");
  if (rc == IE_OK) {
    e = cudaEventRecord(ev[0], st);
    mma_i8_peak<<<sms, 128, 0, st>>>(static_cast<uint32_t>(iters), kWaitLimitNs);
    rc = check_launch("mma_i8_peak");
    if (rc == IE_OK && e == cudaSuccess) e = cudaEventRecord(ev[1], st);
    if (rc == IE_OK && e == cudaSuccess) e = cudaEventSynchronize(ev[1]);
    float ms = 0.0f;
    if (rc == IE_OK && e == cudaSuccess) e = cudaEventElapsedTime(&ms, ev[0], ev[1]);
    if (rc == IE_OK && e != cudaSuccess) rc = fail(IE_RUNTIME, "mma_i8_peak timing: %s", cudaGetErrorString(e));
    if (rc == IE_OK) {
      uint32_t code = 0;
      if (ie_cuda_take_device_error(&code) != IE_OK || code != 0) {
        rc = fail(IE_RUNTIME, "mma_i8_peak: device-side wait gave up (site 0x%x)", code);
      } else {
        *tops = 2.0 * 128 * 256 * 32 * static_cast<double>(iters) * sms / (ms * 1e-3) / 1e12;
      }
    }
  }
  cudaEventDestroy(ev[0]);
  cudaEventDestroy(ev[1]);
  return rc;
}

size_t ie_cuda_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

int ie_cuda_conv2d_f32_noalloc(const ie_conv2d_desc* desc, int32_t act, const float* x,
                               const float* w, const float* bias, float* y, void* stream) {
  ie_conv2d_shape s;
  int rc = resolve(desc, -1, &s);
  if (rc != IE_OK) return rc;
  // the size check comes first and touches no device state
  const size_t need = ie_cuda_conv2d_f32_workspace_bytes(desc);
  if (need > kNoAllocScratchBytes) {
    return fail(IE_INVALID_ARGUMENT,
                "convolution needs %zu bytes of scratch; the no-allocation entry point has %zu "
                "(use ie_cuda_conv2d_f32 with a caller-provided workspace)",
                need, kNoAllocScratchBytes);
  }
  void* scratch = nullptr;
  if (need > 0 && (rc = noalloc_scratch(&scratch)) != IE_OK) return rc;
  return ie_cuda_conv2d_f32(desc, act, x, w, bias, y, scratch, need, stream);
}

}  // extern "C"
