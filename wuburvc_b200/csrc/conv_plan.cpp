// conv_plan.cpp — TMA descriptors and launch parameters for the tcgen05 convolution kernels.
#include "conv_plan.h"

#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

namespace wb {

namespace {
std::atomic<unsigned long long> g_wait_limit_ns{kWaitLimitNs};
}  // namespace

unsigned long long wait_limit_ns() { return g_wait_limit_ns.load(); }
void set_wait_limit_ns(unsigned long long ns) { g_wait_limit_ns.store(ns ? ns : kWaitLimitNs); }

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int pow2_cols(int n) {
  int c = 32;
  while (c < n) c <<= 1;
  return c;
}

constexpr size_t kSmemBudget = 220 * 1024;
// the persistent conv keeps ~24 KB of static shared memory (epilogue vectors, column sums, the
// epilogue warps' store staging).  Its dynamic budget leaves ~7 KB of the SM's 228 KB free: one
// block of the side stream's reductions (4 KB + the 1 KB per-block reserve) then runs beside it
// instead of waiting for an SM between launches (measured 1.6 % faster on the step than 202 KB).
constexpr size_t kSmemBudget2 = 196 * 1024;
constexpr int kMaxHaloStages = 6;  // halo ring depth of the persistent conv (barriers: 512 B reserved)

}  // namespace

bool make_map_bf16_3d(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                      uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1, uint32_t b2) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t es[3] = {1, 1, 1};
  CUtensorMapSwizzle sw = (b0 * 2 == 128) ? CU_TENSOR_MAP_SWIZZLE_128B
                          : (b0 * 2 == 64) ? CU_TENSOR_MAP_SWIZZLE_64B
                                           : CU_TENSOR_MAP_SWIZZLE_32B;
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    fprintf(stderr, "wuburvc_b200: cuTensorMapEncodeTiled failed (%d) dims %llu %llu %llu box %u %u %u\n", (int)r,
            (unsigned long long)d0, (unsigned long long)d1, (unsigned long long)d2, b0, b1, b2);
    return false;
  }
  return true;
}

// choose K chunk / stages for the forward-type kernel: about three stages, each holding as many
// (tap, chunk) steps as fit (every stage costs the MMA warp one barrier round trip)
static void pick_fwd_tiling(int c_in, int n_tile, int split, int& kc, int& stages, int& kgroup, size_t& smem) {
  kc = (c_in % 64 == 0) ? 64 : 32;
  for (;;) {
    const int nA = split ? 2 : 1;
    const size_t step = (size_t)nA * (128 * kc * 2 + (size_t)n_tile * kc * 2);
    const size_t room = kSmemBudget - 1024 - 256;
    kgroup = (int)std::max<size_t>(1, std::min<size_t>(4, room / (3 * step)));
    stages = (int)std::min<size_t>(8, room / (kgroup * step));
    if (stages >= 3 || kc == 32) {
      smem = stages * kgroup * step + 1024 /*align*/ + 256 /*barriers*/;
      return;
    }
    kc = 32;
  }
}

// GEMM N per CTA of the general conv kernel: up to 256 columns, 128 under the bf16x3 split (its
// first MMA is 2N wide)
static int fwd_n_tile(int n_total, int split) {
  int n_tile = std::min(n_total, split ? 128 : 256);
  while (n_tile > 16 && n_total % n_tile) n_tile -= 16;
  return n_tile;
}

static bool finish_fwd(ConvLaunch& L, int B, int c_in, int n_total, int split, int nphase, int* err) {
  TcConvParams& p = L.p;
  const int n_tile = fwd_n_tile(n_total, split);
  if (n_tile < 16 || n_tile % 16 || n_total % 32) return false;
  if (c_in % 32) return false;
  pick_fwd_tiling(c_in, n_tile, split, L.kc, p.stages, p.kgroup, L.smem);
  p.n_tile = n_tile;
  p.n_total = n_total;
  p.n_chunks = c_in / L.kc;
  p.split = split;
  p.tmem_cols = pow2_cols(n_tile * (split ? 2 : 1));  // 2n columns under the two-MMA bf16x3 split
  p.tiles_per_item = (p.m_rows + 127) / 128;
  p.err = err;
  p.wait_ns = wait_limit_ns();
  L.grid = dim3(B * p.tiles_per_item, n_total / n_tile, nphase);
  return true;
}

bool plan_conv(ConvLaunch& L, const ConvGeom& g, const void* x_hi, const void* x_lo, const void* w_hi,
               const void* w_lo, int split, const Epi& epi, int* err) {
  memset(&L.p, 0, sizeof(L.p));
  memset(&L.maps, 0, sizeof(L.maps));
  TcConvParams& p = L.p;
  if (g.k > kMaxTapList) return false;
  p.m_rows = g.T_out;
  p.t_out = g.T_out;
  p.out_stride = 1;
  p.out_off[0] = 0;
  p.tap_start[0] = 0;
  p.tap_start[1] = g.k;
  for (int t = 0; t < g.k; ++t) {
    p.tap_map[t] = 0;
    p.tap_shift[t] = (short)(-g.pad + g.dil * t);
    p.tap_w[t] = (short)t;
  }
  p.lo_base = 1;
  p.epi = epi;
  const int n_tile = fwd_n_tile(g.C_out, split);
  int kc, stages, kgroup;
  size_t smem;
  pick_fwd_tiling(g.C_in, n_tile, split, kc, stages, kgroup, smem);
  const uint64_t rs = (uint64_t)g.C_in * 2, is = rs * g.T_in;
  if (!make_map_bf16_3d(&L.maps.a[0], x_hi, g.C_in, g.T_in, g.B, rs, is, kc, 128, 1)) return false;
  if (split && !make_map_bf16_3d(&L.maps.a[1], x_lo, g.C_in, g.T_in, g.B, rs, is, kc, 128, 1)) return false;
  const uint64_t wr = (uint64_t)g.C_in * 2, wt = wr * g.C_out;
  if (!make_map_bf16_3d(&L.maps.w_hi, w_hi, g.C_in, g.C_out, g.k, wr, wt, kc, n_tile, 1)) return false;
  if (split && !make_map_bf16_3d(&L.maps.w_lo, w_lo, g.C_in, g.C_out, g.k, wr, wt, kc, n_tile, 1)) return false;
  return finish_fwd(L, g.B, g.C_in, g.C_out, split, 1, err);
}

static int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  }
  return n;
}

bool plan_conv2(Conv2Launch& L, const ConvGeom& g, const void* x_hi, const void* x_lo, const void* w_hi,
                const void* w_lo, int split, const Epi& epi, int* err) {
  memset(&L.p, 0, sizeof(L.p));
  memset(&L.maps, 0, sizeof(L.maps));
  TcConv2Params& p = L.p;
  if (g.T_in != g.T_out || g.C_out > 256 || g.C_out % 32 || g.C_in % 32 || g.k > kMaxTaps2) return false;
  const int span = g.dil * (g.k - 1);
  // rows of the halo tile, a multiple of 16 so each tile is a whole number of 1 KB swizzle atoms
  const int R = (128 + span + 15) / 16 * 16;
  if (R > 256) return false;
  p.ntaps = g.k;
  p.dil = g.dil;
  p.halo_start = -g.pad;
  p.halo_rows = R;
  p.tiles_per_item = (g.T_out + 127) / 128;
  const int mtiles = g.B * p.tiles_per_item;
  // split N in two when the row tiles alone cannot fill the SMs
  p.n_tiles = (mtiles < sm_count() && g.C_out >= 128) ? 2 : 1;
  p.n = g.C_out / p.n_tiles;
  p.n_total = g.C_out;
  p.ntiles = mtiles * p.n_tiles;
  p.t_rows = g.T_out;
  p.split = split;
  p.epi = epi;
  p.err = err;
  p.wait_ns = wait_limit_ns();
  const int nA = split ? 2 : 1;
  // weights: resident (every chunk and tap of the CTA's N tile loaded once) when they fit beside two
  // A stages, else a ring of stages holding w_group taps each.  The wider channel chunk is preferred:
  // a tap then carries twice the MMAs for the same loop overhead of the MMA warp.
  struct Opt {
    int kc = 0, resident = 0, G = 0, WS = 0;
    size_t a_sub = 0, smem = 0;
    long long score = -1;
  } best;
  for (int kc_try : {64, 32}) {
    if (g.C_in % kc_try) continue;
    Opt o;
    o.kc = kc_try;
    o.a_sub = ((size_t)R * kc_try * 2 + 1023) / 1024 * 1024;
    const size_t a_stage = nA * o.a_sub, w_tap = (size_t)nA * p.n * kc_try * 2;
    const long long nch = g.C_in / kc_try;
    const long long room = (long long)kSmemBudget2 - 2048 - 2 * (long long)a_stage;
    const long long total_w = nch * g.k * (long long)w_tap;
    if (room > 0 && total_w <= room) {
      o.resident = 1;
      o.G = g.k;
      o.WS = 1;
      o.smem = 2 * a_stage + (size_t)total_w + 1024 + 512;
      o.score = 1LL << 40;  // no weight waits at all
    } else {
      const long long G = room > 0 ? std::min<long long>(g.k, room / (2 * (long long)w_tap)) : 0;
      if (G < 1) continue;
      o.G = (int)G;
      o.WS = (int)std::min<long long>(4, room / (G * (long long)w_tap));
      o.smem = 2 * a_stage + (size_t)o.WS * G * w_tap + 1024 + 512;
      o.score = (long long)kc_try * 1000 + G;
    }
    if (o.score > best.score) best = o;
  }
  if (best.score < 0) return false;
  const int kc = best.kc;
  // 32 input channels: every tile is one halo load and little MMA work, so resident weights leave
  // the rest of the budget to a deeper halo ring that keeps the MMAs from waiting on TMA latency
  // (measured faster at 32 channels; at 64 the deeper ring costs the input gradients more than it
  // gives, as it leaves the side stream's reductions no room on the SM)
  int a_stages = 2;
  if (best.resident && g.C_in <= 32) {
    const size_t a_stage = (size_t)nA * best.a_sub;
    while (a_stages < kMaxHaloStages && best.smem + a_stage <= kSmemBudget2 - 512) {
      best.smem += a_stage;
      ++a_stages;
    }
  }
  p.a_stages = a_stages;
  p.w_resident = best.resident;
  p.w_group = best.G;
  p.w_stages = best.WS;
  p.a_sub_bytes = (uint32_t)best.a_sub;
  L.smem = best.smem;
  L.kc = kc;
  p.n_chunks = g.C_in / kc;
  // two accumulators (double buffering) of n columns, 2n under the two-MMA bf16x3 split
  p.tmem_cols = pow2_cols(2 * p.n * (split ? 2 : 1));
  if (p.tmem_cols > 512) return false;
  const uint64_t xs = (uint64_t)g.C_in * 2, xt = xs * g.T_in;
  if (!make_map_bf16_3d(&L.maps.a_hi, x_hi, g.C_in, g.T_in, g.B, xs, xt, kc, R, 1)) return false;
  if (split && !make_map_bf16_3d(&L.maps.a_lo, x_lo, g.C_in, g.T_in, g.B, xs, xt, kc, R, 1)) return false;
  const uint64_t wr = (uint64_t)g.C_in * 2, wt = wr * g.C_out;
  if (!make_map_bf16_3d(&L.maps.w_hi, w_hi, g.C_in, g.C_out, g.k, wr, wt, kc, p.n, 1)) return false;
  if (split && !make_map_bf16_3d(&L.maps.w_lo, w_lo, g.C_in, g.C_out, g.k, wr, wt, kc, p.n, 1)) return false;
  // one CTA per SM (320 threads x ~128 registers), persistent over its tiles
  L.grid = std::min(p.ntiles, sm_count()) / p.n_tiles * p.n_tiles;
  return true;
}

bool plan_conv_any(ConvOp& op, const ConvGeom& g, const void* x_hi, const void* x_lo, const void* w_hi,
                   const void* w_lo, int split, const Epi& epi, int* err) {
  static const bool force_v1 = getenv("WUBU_B200_CONV_V1") != nullptr;
  op.v2 = !force_v1 && plan_conv2(op.c2, g, x_hi, x_lo, w_hi, w_lo, split, epi, err);
  if (op.v2) return true;
  return plan_conv(op.v1, g, x_hi, x_lo, w_hi, w_lo, split, epi, err);
}

bool plan_convT(ConvLaunch& L, int B, int T_in, int C_in, int C_out, int k, int s, int pad, const void* x_hi,
                const void* x_lo, const void* wp_hi, const void* wp_lo, int split, const Epi& epi, int* err) {
  memset(&L.p, 0, sizeof(L.p));
  memset(&L.maps, 0, sizeof(L.maps));
  TcConvParams& p = L.p;
  if (s > kMaxPhases || k > kMaxTapList || pad >= s) return false;
  p.m_rows = T_in + 1;
  p.t_out = T_in * s;
  p.out_stride = s;
  int n = 0;
  for (int r = 0; r < s; ++r) {
    p.out_off[r] = r - pad;
    p.tap_start[r] = n;
    for (int m = 0; r + s * m < k; ++m) {
      p.tap_map[n] = 0;
      p.tap_shift[n] = (short)(-m);
      p.tap_w[n] = (short)n;  // packed phase-tap order
      ++n;
    }
  }
  p.tap_start[s] = n;
  p.lo_base = 1;
  p.epi = epi;
  const int n_tile = fwd_n_tile(C_out, split);
  int kc, stages, kgroup;
  size_t smem;
  pick_fwd_tiling(C_in, n_tile, split, kc, stages, kgroup, smem);
  const uint64_t rs = (uint64_t)C_in * 2, is = rs * T_in;
  if (!make_map_bf16_3d(&L.maps.a[0], x_hi, C_in, T_in, B, rs, is, kc, 128, 1)) return false;
  if (split && !make_map_bf16_3d(&L.maps.a[1], x_lo, C_in, T_in, B, rs, is, kc, 128, 1)) return false;
  const uint64_t wr = (uint64_t)C_in * 2, wt = wr * C_out;
  if (!make_map_bf16_3d(&L.maps.w_hi, wp_hi, C_in, C_out, k, wr, wt, kc, n_tile, 1)) return false;
  if (split && !make_map_bf16_3d(&L.maps.w_lo, wp_lo, C_in, C_out, k, wr, wt, kc, n_tile, 1)) return false;
  return finish_fwd(L, B, C_in, C_out, split, s, err);
}

static int floordiv(int a, int b) { return (a >= 0) ? a / b : -((-a + b - 1) / b); }

bool plan_convT_dgrad(ConvLaunch& L, int B, int T_in, int C_in, int C_out, int k, int s, int pad, const void* dy,
                      const void* wd, const void* dy_lo, const void* wd_lo, const Epi& epi, int* err) {
  memset(&L.p, 0, sizeof(L.p));
  memset(&L.maps, 0, sizeof(L.maps));
  TcConvParams& p = L.p;
  const int split = (dy_lo && wd_lo) ? 1 : 0;
  if ((split ? 2 * s : s) > kMaxMapsA || k > kMaxTapList) return false;
  const int T_out = T_in * s;
  p.m_rows = T_in;
  p.t_out = T_in;
  p.out_stride = 1;
  p.out_off[0] = 0;
  p.tap_start[0] = 0;
  p.tap_start[1] = k;
  for (int t = 0; t < k; ++t) {
    const int d = t - pad;
    const int r = ((d % s) + s) % s;
    p.tap_map[t] = (signed char)r;
    p.tap_shift[t] = (short)floordiv(d, s);
    p.tap_w[t] = (short)t;
  }
  p.lo_base = s;  // lo views (split) after the s hi views
  p.epi = epi;
  const int n_tile = fwd_n_tile(C_in, split);
  int kc, stages, kgroup;
  size_t smem;
  pick_fwd_tiling(C_out, n_tile, split, kc, stages, kgroup, smem);
  for (int h = 0; h <= split; ++h)
    for (int r = 0; r < s; ++r) {
      const uint64_t rows = (uint64_t)(T_out - r + s - 1) / s;
      const char* base = static_cast<const char*>(h ? dy_lo : dy) + (size_t)r * C_out * 2;
      if (!make_map_bf16_3d(&L.maps.a[h * s + r], base, C_out, rows, B, (uint64_t)s * C_out * 2,
                            (uint64_t)T_out * C_out * 2, kc, 128, 1))
        return false;
    }
  const uint64_t wr = (uint64_t)C_out * 2, wt = wr * C_in;
  if (!make_map_bf16_3d(&L.maps.w_hi, wd, C_out, C_in, k, wr, wt, kc, n_tile, 1)) return false;
  if (split && !make_map_bf16_3d(&L.maps.w_lo, wd_lo, C_out, C_in, k, wr, wt, kc, n_tile, 1)) return false;
  if (!finish_fwd(L, B, C_out, C_in, split, 1, err)) return false;
  p.split_bf16 = 1;  // gradient pairs are bf16 hi + bf16 lo
  return true;
}

// ------------------------------------------------------------------------------------------------
// weight gradients
// ------------------------------------------------------------------------------------------------
// Time rows per weight-gradient K block: the largest of 256 / 128 / 64 for which two pipeline stages
// (128 dOut rows + n_tile activation channels, bf16) fit in shared memory.
static int wgrad_kb_rows(int n_tile) {
  const size_t room = kSmemBudget - 1024 - 256;
  for (int kr = 256; kr > 64; kr >>= 1)
    if ((size_t)(128 + n_tile) * kr * 2 * 2 <= room) return kr;
  return 64;
}

static bool finish_wgrad(WgradLaunch& L, int B, int T_rows, int C_in, int C_out, int n_atoms_total,
                         const int* a_map, const int* a_shift, const int* a_oc0, const int* a_tap, float* part,
                         size_t cap, int target_ctas, int* err) {
  TcWgParams& p = L.p;
  p.atom_m = std::min(C_out, 64);
  if (C_out % p.atom_m || (p.atom_m != 32 && p.atom_m != 64)) return false;
  p.m_atoms = 128 / p.atom_m;
  p.n_mtiles = (n_atoms_total + p.m_atoms - 1) / p.m_atoms;
  if (p.n_mtiles > 64) return false;
  for (int mt = 0; mt < p.n_mtiles; ++mt)
    for (int j = 0; j < 4; ++j) {
      const int a = mt * p.m_atoms + j;
      const bool use = j < p.m_atoms && a < n_atoms_total;
      p.atom_map[mt][j] = use ? (signed char)a_map[a] : 0;
      p.atom_shift[mt][j] = use ? (short)a_shift[a] : 0;
      p.atom_oc0[mt][j] = use ? (short)a_oc0[a] : 0;
      p.atom_tap[mt][j] = use ? (short)a_tap[a] : -1;
    }
  int n_tile = std::min(C_in, 256);
  while (C_in % n_tile) n_tile -= 16;
  if (n_tile % 32 && n_tile != 16) return false;
  p.n_in = n_tile;
  p.n_total = C_in;
  const int atom_n = std::min(n_tile, 64);
  if (n_tile % atom_n || (atom_n != 32 && atom_n != 64)) return false;
  p.n_atoms = n_tile / atom_n;
  p.c_out = C_out;
  p.t_rows = T_rows;
  p.kb_rows = wgrad_kb_rows(n_tile);
  p.kblocks_per_item = (T_rows + p.kb_rows - 1) / p.kb_rows;
  p.total_kblocks = B * p.kblocks_per_item;
  const int n_ntiles = C_in / n_tile;
  const int base = p.n_mtiles * n_ntiles;
  // at most target_ctas CTAs (whole waves; rounding up would start a nearly empty extra wave)
  int splits = std::max(1, std::min(p.total_kblocks, target_ctas / base));
  p.kb_per_split = (p.total_kblocks + splits - 1) / splits;
  splits = (p.total_kblocks + p.kb_per_split - 1) / p.kb_per_split;
  // stages of kb_group 64-row blocks: about three stages, each as many blocks as fit
  const size_t kb = (size_t)(128 + n_tile) * p.kb_rows * 2;
  const size_t room = kSmemBudget - 1024 - 256;
  p.kb_group = (int)std::max<size_t>(1, std::min<size_t>(8, room / (3 * kb)));
  p.stages = (int)std::min<size_t>(4, room / (p.kb_group * kb));
  if (p.stages < 2) return false;
  L.smem = p.stages * p.kb_group * kb + 1024 + 256;
  p.tmem_cols = pow2_cols(n_tile);
  p.err = err;
  p.wait_ns = wait_limit_ns();
  p.part = part;
  L.splits = splits;
  L.grid = dim3(p.n_mtiles, splits, n_ntiles);
  if ((size_t)splits * p.n_mtiles * 128 * C_in > cap) return false;
  L.row_tap.assign((size_t)p.n_mtiles * 128, -1);
  L.row_oc.assign((size_t)p.n_mtiles * 128, 0);
  for (int mt = 0; mt < p.n_mtiles; ++mt)
    for (int m = 0; m < 128; ++m) {
      const int j = m / p.atom_m;
      L.row_tap[mt * 128 + m] = p.atom_tap[mt][j];
      L.row_oc[mt * 128 + m] = p.atom_oc0[mt][j] + m % p.atom_m;
    }
  return true;
}

size_t wgrad_part_floats(const WgradLaunch& L) {
  return (size_t)L.splits * L.p.n_mtiles * 128 * L.p.n_total;
}

// Halo-mode weight gradient (stride 1): see TcWgParams.  K blocks of 128 time rows.
//   C_out % 128 == 0: tg = 2 taps per CTA (at most 512 / n_in accumulator columns); the halo tile of
//     128 channels x R rows arrives as two SW128 boxes of 64 channels.
//   C_out 32 / 64: pack = 128 / C_out taps per accumulator, at most 4 accumulators (and 512 / n_in
//     columns) per CTA, the taps spread evenly over tap groups; one halo box of C_out channels
//     (SW64 / SW128).
static bool plan_wgrad_halo(WgradLaunch& L, const ConvGeom& g, const void* dy, const void* x, float* part, size_t cap,
                            int target_ctas, int* err) {
  TcWgParams& p = L.p;
  int n_tile = std::min(g.C_in, 256);
  while (g.C_in % n_tile) n_tile -= 16;
  const int x_atom = n_tile % 64 == 0 ? 64 : 32;
  if (n_tile % x_atom) return false;
  const int pack = g.C_out % 128 == 0 ? 1 : (g.C_out == 32 || g.C_out == 64) ? 128 / g.C_out : 0;
  if (!pack) return false;
  int nacc;
  if (pack == 1) {
    nacc = std::min(2, 512 / n_tile);  // 2 taps per CTA: more CTAs per split, smaller partials
  } else {
    // at most 4 accumulators per CTA (more tap groups instead: smaller split-K partials), balanced
    const int need = (g.k + pack - 1) / pack;
    const int groups = (need + 3) / 4;
    nacc = std::min((need + groups - 1) / groups, 512 / n_tile);
  }
  const int tg = nacc * pack;
  const int kr = 128;  // K block rows; the halo kernel is compiled for 128 (kHaloKR)
  // halo rows: whole 1 KB swizzle periods (8 rows of 128 B, 16 rows of 64 B)
  const int rq = (pack == 1 || g.C_out == 64) ? 8 : 16;
  const int R = (kr + (tg - 1) * g.dil + rq - 1) / rq * rq;
  if (R > 256) return false;
  p.halo = 1;
  p.pack = pack;
  p.nacc = nacc;
  p.tg = tg;
  p.x_atom = x_atom;
  p.ntaps = g.k;
  p.dil = g.dil;
  p.pad = g.pad;
  p.oc_chunks = pack == 1 ? g.C_out / 128 : 1;
  p.halo_rows = R;
  p.n_in = n_tile;
  p.n_total = g.C_in;
  p.n_atoms = n_tile / x_atom;
  p.c_out = g.C_out;
  p.t_rows = g.T_in;
  p.kb_rows = kr;
  p.kb_group = 1;
  p.kblocks_per_item = (g.T_in + kr - 1) / kr;
  p.total_kblocks = g.B * p.kblocks_per_item;
  p.n_mtiles = (g.k * g.C_out + 127) / 128;  // partial rows: tap * C_out + oc
  const int tap_groups = (g.k + tg - 1) / tg;
  const int n_ntiles = g.C_in / n_tile;
  const int base = tap_groups * p.oc_chunks * n_ntiles;
  // at most target_ctas CTAs: the kernel holds one CTA per SM at 128+ channels, so a grid just above
  // the SM count (6 x 25 = 150) would run a second wave of two CTAs
  int splits = std::max(1, std::min(p.total_kblocks, target_ctas / base));
  p.kb_per_split = (p.total_kblocks + splits - 1) / splits;
  splits = (p.total_kblocks + p.kb_per_split - 1) / p.kb_per_split;
  const size_t a_bytes = (size_t)(pack == 1 ? 128 : g.C_out) * R * 2;
  const size_t stage = a_bytes + (size_t)n_tile * kr * 2;
  const size_t room = kSmemBudget - 1024 - 256;
  p.stages = (int)std::min<size_t>(pack == 1 ? 3 : 4, room / stage);
  if (p.stages < 2) return false;
  L.smem = p.stages * stage + 1024 + 256;
  p.tmem_cols = pow2_cols(nacc * n_tile);
  if (p.tmem_cols > 512) return false;
  p.err = err;
  p.wait_ns = wait_limit_ns();
  p.part = part;
  L.splits = splits;
  L.grid = dim3(tap_groups * p.oc_chunks, splits, n_ntiles);
  if ((size_t)splits * p.n_mtiles * 128 * g.C_in > cap) return false;
  L.row_tap.assign((size_t)p.n_mtiles * 128, -1);
  L.row_oc.assign((size_t)p.n_mtiles * 128, 0);
  for (int r = 0; r < g.k * g.C_out; ++r) {
    L.row_tap[r] = r / g.C_out;
    L.row_oc[r] = r % g.C_out;
  }
  // dOut halo: (C_out, T, B) with a 64-channel (or, packed, C_out-channel) x R-row box
  if (!make_map_bf16_3d(&L.maps.d[0], dy, g.C_out, g.T_out, g.B, (uint64_t)g.C_out * 2,
                        (uint64_t)g.C_out * 2 * g.T_out, pack == 1 ? 64 : g.C_out, R, 1))
    return false;
  return make_map_bf16_3d(&L.maps.x, x, g.C_in, g.T_in, g.B, (uint64_t)g.C_in * 2, (uint64_t)g.C_in * 2 * g.T_in,
                          x_atom, kr, 1);
}

bool plan_wgrad(WgradLaunch& L, const ConvGeom& g, const void* dy, const void* x, float* part, size_t cap,
                int target_ctas, int* err) {
  memset(&L.p, 0, sizeof(L.p));
  memset(&L.maps, 0, sizeof(L.maps));
  if ((g.C_out % 128 == 0 || g.C_out == 32 || g.C_out == 64) && g.T_in == g.T_out &&
      !getenv("WUBU_B200_WGRAD_ATOMS")) {
    // a halo CTA carries tg taps' MMAs per K block: half the CTAs keep the split-K partials small
    if (plan_wgrad_halo(L, g, dy, x, part, cap, std::max(1, target_ctas / 2), err)) return true;
    memset(&L.p, 0, sizeof(L.p));
    memset(&L.maps, 0, sizeof(L.maps));
  }
  const int atom_m = std::min(g.C_out, 64);
  const int oc_chunks = g.C_out / atom_m;
  std::vector<int> am, ash, aoc, atap;
  for (int t = 0; t < g.k; ++t)
    for (int c = 0; c < oc_chunks; ++c) {
      am.push_back(0);
      ash.push_back(g.pad - g.dil * t);
      aoc.push_back(c * atom_m);
      atap.push_back(t);
    }
  const int n_tile = std::min(g.C_in, 256);
  const int atom_n = std::min(n_tile, 64);
  const int kr = wgrad_kb_rows(n_tile);
  if (!make_map_bf16_3d(&L.maps.d[0], dy, g.C_out, g.T_out, g.B, (uint64_t)g.C_out * 2,
                        (uint64_t)g.C_out * 2 * g.T_out, atom_m, kr, 1))
    return false;
  if (!make_map_bf16_3d(&L.maps.x, x, g.C_in, g.T_in, g.B, (uint64_t)g.C_in * 2, (uint64_t)g.C_in * 2 * g.T_in,
                        atom_n, kr, 1))
    return false;
  return finish_wgrad(L, g.B, g.T_in, g.C_in, g.C_out, (int)am.size(), am.data(), ash.data(), aoc.data(),
                      atap.data(), part, cap, target_ctas, err);
}

bool plan_convT_wgrad(WgradLaunch& L, int B, int T_in, int C_in, int C_out, int k, int s, int pad, const void* x,
                      const void* dy, float* part, size_t cap, int target_ctas, int* err) {
  memset(&L.p, 0, sizeof(L.p));
  memset(&L.maps, 0, sizeof(L.maps));
  if (s > kMaxMaps) return false;
  const int T_out = T_in * s;
  const int atom_m = std::min(C_out, 64);
  const int oc_chunks = C_out / atom_m;
  const int kr = wgrad_kb_rows(std::min(C_in, 256));
  for (int r = 0; r < s; ++r) {
    const uint64_t rows = (uint64_t)(T_out - r + s - 1) / s;
    const char* base = static_cast<const char*>(dy) + (size_t)r * C_out * 2;
    if (!make_map_bf16_3d(&L.maps.d[r], base, C_out, rows, B, (uint64_t)s * C_out * 2, (uint64_t)T_out * C_out * 2,
                          atom_m, kr, 1))
      return false;
  }
  std::vector<int> am, ash, aoc, atap;
  for (int t = 0; t < k; ++t)
    for (int c = 0; c < oc_chunks; ++c) {
      const int d = t - pad;
      const int r = ((d % s) + s) % s;
      am.push_back(r);
      ash.push_back(floordiv(d, s));
      aoc.push_back(c * atom_m);
      atap.push_back(t);
    }
  const int n_tile = std::min(C_in, 256);
  const int atom_n = std::min(n_tile, 64);
  if (!make_map_bf16_3d(&L.maps.x, x, C_in, T_in, B, (uint64_t)C_in * 2, (uint64_t)C_in * 2 * T_in, atom_n, kr, 1))
    return false;
  return finish_wgrad(L, B, T_in, C_in, C_out, (int)am.size(), am.data(), ash.data(), aoc.data(), atap.data(), part,
                      cap, target_ctas, err);
}

}  // namespace wb
