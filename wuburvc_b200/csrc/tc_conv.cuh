// tc_conv.cuh — tcgen05/TMEM implicit-GEMM kernels for the generator's convolutions.
//
// Two kernels cover every dense contraction of the training step:
//
//  * tc_conv  : out[b, q*stride+off, n] = epilogue( sum_taps sum_c A_tap[b, q+shift, c] * W[tap, n, c] )
//               A is a channels-last activation tensor [B][T][C] read through TMA with a per-tap row
//               shift (padding and dilation come from TMA out-of-bounds zero fill).  It serves the
//               Conv1d forward, the Conv1d input-gradient (flipped taps, transposed weights), the
//               polyphase ConvTranspose1d forward (one phase per blockIdx.z) and the ConvTranspose1d
//               input-gradient (one strided A view per tap residue).  In split mode the A and W
//               operands are hi/lo pairs (fp16 hi + fp16 lo*2^11 for the forward, or bf16 hi + bf16
//               lo) and three products (hi*hi + lo*hi + hi*lo) give an fp32-accurate result.
//  * tc_wgrad : dW[tap, o, i] = sum_{b,t} dOut[b, t - shift_tap, o] * A[b, t, i], split over time
//               (K) across CTAs with deterministic fp32 partials.  Both operands are MN-major in
//               shared memory; several taps are packed into one 128-row M tile when C_out < 128.
#pragma once
#include "common.cuh"

namespace wb {

constexpr int kMaxMaps = 14;   // dOut views of the weight-gradient kernel (one per ConvTranspose residue)
constexpr int kMaxMapsA = 24;  // A views of the conv kernel: hi and lo per ConvTranspose residue (stride <= 12)
constexpr int kMaxTapList = 48;
constexpr int kMaxPhases = 12;

// ---------------------------------------------------------------------------------------------
// forward-type kernel (conv fwd / dgrad / convT polyphase)
// ---------------------------------------------------------------------------------------------
struct Epi {
  const float* bias;        // [n_total]
  const float* rowadd;      // [B][n_total], broadcast over time (cond(g))
  const bf16* mask_src;     // [B][T][n_total]: activated value (lrelu) or pre-activation (snake)
  const float* mask_alpha;  // [n_total] snake alpha for the mask
  float* alpha_part;        // [tiles][n_total] snake d(alpha) partial sums
  const float* res;         // [B][T][n_total] fp32 residual added after the mask
  float* out_f32;           // [B][T][n_total]
  bf16* out_bf16;           // [B][T][n_total]
  f16* act_hi;              // [B][T][n_total] activation of the result, fp16 hi part (forward operand)
  f16* act_lo;              //                   ... its fp16 lo part scaled by 2^11 (with act_hi)
  bf16* act_bf;             //                   ... bf16 copy (weight-gradient operand, LeakyReLU masks)
  int* range_err;           // error word: set to ERR_RANGE if |activation| >= 65504
  int act_bf16pair;         // write act_hi / act_lo as a bf16 hi + bf16 lo pair instead (the
                            // range-safe operand format a context falls back to after ERR_RANGE)
  const float* act_alpha;   // [n_total] snake alpha of the activation
  bf16* pre_hi;             // [B][T][n_total] bf16 copy of the result (snake pre-activation)
  float* colsum;            // [tiles][n_total] column-sum partials (bias gradients)
  float scale;
  float slope;              // lrelu slope (activation and mask)
  int accumulate;           // out_f32 += result
  int act_kind;             // 0 lrelu, 1 snake
  // fp32 precision: bf16 lo companions (value = hi + lo, ~2^-17 relative) of the bf16 tensors above
  bf16* out_bf16_lo;        // of out_bf16 (the next input-gradient GEMM's A operand pair)
  bf16* act_bflo;           // of act_bf (the weight gradient's activation operand pair)
  bf16* pre_lo;             // of pre_hi (Snake pre-activation)
  const bf16* mask_lo;      // of mask_src (the Snake derivative from the pair; LeakyReLU needs the sign only)
};

struct TcMaps {
  CUtensorMap a[kMaxMapsA];  // A operand maps; lo maps at a[lo_base + i]
  CUtensorMap w_hi;
  CUtensorMap w_lo;
};

struct TcConvParams {
  int m_rows;          // q rows per item
  int tiles_per_item;  // ceil(m_rows / 128)
  int n_tile;          // GEMM N per CTA (multiple of 16, <= 256)
  int n_total;         // channel pitch of every [B][T][C] output
  int n_chunks;        // C_in / KC
  int split;           // operands as hi/lo pairs, three products (fp32-accurate)
  int split_bf16;      // split pair format: 0 = fp16 hi + fp16 lo*2^11 (forward), 1 = bf16 hi + bf16 lo
  int single_f16;      // without the split: the single operands are fp16 (fast inference), else bf16
  int lo_base;
  int stages;
  int kgroup;          // (tap, chunk) steps per pipeline stage
  int tmem_cols;
  int t_out;           // output rows per item
  int out_stride;      // output row = q * out_stride + out_off[phase]
  int out_off[kMaxPhases];
  int tap_start[kMaxPhases + 1];
  signed char tap_map[kMaxTapList];
  short tap_shift[kMaxTapList];
  short tap_w[kMaxTapList];
  int pdl;             // launched with programmatic stream serialization
  unsigned long long wait_ns;  // bounded-wait limit
  Epi epi;
  int* err;
};

// ---------------------------------------------------------------------------------------------
// persistent stride-1 conv kernel with halo reuse (tc_conv2)
//   Each CTA loops over 128-row output tiles.  Per input-channel chunk it loads ONE halo tile
//   (rows q0+sh_min .. q0+127+sh_max) with one swizzled TMA box; the swizzle is a function of the
//   absolute shared-memory address, so every tap's A operand is the same tile started tap*dil rows
//   further on.  Weights are resident or stream in multi-tap stages.  Two TMEM accumulators let the
//   epilogue of one tile overlap the MMAs of the next.
// ---------------------------------------------------------------------------------------------
constexpr int kMaxTaps2 = 16;

struct TcConv2Maps {
  CUtensorMap a_hi, a_lo;   // (C_in, T, B) views with a KC-channel x R-row box, 128B/64B swizzle
  CUtensorMap w_hi, w_lo;   // 3-D (C_in, C_out, taps), 128B/64B swizzle
};

struct TcConv2Params {
  int ntiles, tiles_per_item, t_rows;  // ntiles counts (row tile, N tile) pairs
  int n;                    // GEMM N per tile (<= 256)
  int n_tiles;              // C_out / n; N tile = tile % n_tiles (grid is a multiple of n_tiles)
  int n_total;              // C_out: output channel pitch
  int n_chunks;             // C_in / KC
  int split;
  int split_bf16;           // split pair format (as TcConvParams::split_bf16)
  int single_f16;           // as TcConvParams::single_f16
  int ntaps;
  int dil;                  // tap t reads halo rows t*dil .. t*dil+127
  int halo_start;           // row offset of the halo tile relative to the tile's first output row
  int halo_rows;            // 128 + taps span
  int a_stages, w_stages;
  int w_group;              // taps per weight stage
  int w_resident;           // every weight tap of the CTA's N tile is loaded once and kept
  uint32_t a_sub_bytes;     // one A (hi or lo) halo tile, 1024-aligned
  int tmem_cols;            // 2 accumulators
  // launched with programmatic stream serialization: the prologue (barriers, TMEM, epilogue vectors,
  // the first weight stages) overlaps the previous kernel.  Only for callers whose weights and
  // epilogue vectors are not written by the immediately preceding kernel.
  int pdl;
  unsigned long long wait_ns;  // bounded-wait limit
  Epi epi;
  int* err;
};

// ---------------------------------------------------------------------------------------------
// weight-gradient kernel
// ---------------------------------------------------------------------------------------------
struct TcWgMaps {
  CUtensorMap d[kMaxMaps];  // dOut views (one per tap residue for ConvTranspose)
  CUtensorMap x;            // activation operand [B][T][C_in]
};

struct TcWgParams {
  int t_rows;          // time rows of the activation operand per item
  int kblocks_per_item;
  int total_kblocks;   // items * kblocks_per_item
  int kb_per_split;
  int n_in;            // GEMM N per CTA (input channels of one N tile), multiple of 16, <= 256
  int n_total;         // total input channels (partial row pitch); N tile = blockIdx.z
  int n_atoms;         // N atoms of the activation tile (n_in / atom_n)
  int c_out;           // channels of dOut
  int m_atoms;         // 128 / atom_m
  int atom_m;          // 32 or 64 (dOut channels per atom)
  int stages;
  int kb_group;        // K blocks per pipeline stage
  int kb_rows;         // time rows per K block (64, 128 or 256)
  int tmem_cols;
  // per M tile: atoms (tap, oc0) packed along M
  int n_mtiles;
  signed char atom_map[64][4];   // [mtile][atom] -> dOut map index
  short atom_shift[64][4];       // row shift of the dOut view
  short atom_oc0[64][4];         // first output channel of the atom
  short atom_tap[64][4];         // tap index (for the partial layout); -1 = unused atom
  float* part;                   // [split][n_mtiles*128][n_total] fp32 partials
  int* err;
  // halo mode (stride-1 conv): the dOut halo of a K block (kb_rows + (tg-1)*dil rows of the CTA's
  // channels) is loaded once and every tap reads it at its own row offset.
  //   pack == 1 (C_out a multiple of 128): a CTA owns 128 output channels x `tg` taps, one TMEM
  //     accumulator per tap; the 128 channels are two SW128 MN-major atoms of 64 (LBO = halo bytes).
  //   pack == 128 / C_out (C_out 32 or 64): the M = 128 rows of one accumulator are `pack` taps x all
  //     C_out channels: the M atoms are the same halo started dil rows apart (LBO = dil rows), so one
  //     MMA covers `pack` taps; `nacc` accumulators, tg = nacc * pack taps per CTA.
  // blockIdx.x = tap_group * oc_chunks + oc chunk.  Partial rows stay tap * c_out + oc.
  int halo, tg, ntaps, dil, pad, oc_chunks, halo_rows;
  int pack, nacc;
  int x_atom;          // channels per activation (B) atom: 64 (SW128) or 32 (SW64)
  int pdl;             // launched with programmatic stream serialization
  unsigned long long wait_ns;  // bounded-wait limit
};

}  // namespace wb
