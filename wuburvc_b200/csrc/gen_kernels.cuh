// gen_kernels.cuh — bandwidth-bound kernels of the generator training step (declarations).
#pragma once
#include "common.cuh"

namespace wb {

// ---- weights -------------------------------------------------------------------------------
// Effective weight W (= g*v/||v|| under weight norm, else the raw parameter) -> GEMM layouts: the
// forward's operand pair (fp16 hi + scaled lo, or bf16 hi + lo) and the input gradient's bf16.
// Storage of a weight is tap-major [k][P][Q] f32 (Q fastest): conv P = C_out, Q = C_in (weight-norm
// rows are p); ConvTranspose P = C_out, Q = C_in (weight-norm rows are q, the reference's dim 0).
//   conv : fwd [k][C_out][C_in] hi/lo (the storage layout),   dgrad [k][C_in][C_out], taps flipped
//   convT: fwd [k][C_out][C_in] hi/lo in polyphase tap order, dgrad [k][C_in][C_out]
// `norm` receives ||v|| per weight-norm row.  Two launches for all weights of a step:
//   prep_norm : norms (conv: warp per row; ConvTranspose: partial sums of squares over chunks of
//               kPrepPairs (tap, p) pairs x 32 columns, summed in fixed order by the tile kernel)
//   prep_tile : one tap x 32 p x 32*qs q tile per block: the scaled operand pair in the storage
//               layout and the transposed bf16 through shared memory, both written coalesced.
// P and Q must be multiples of 32.
constexpr int kPrepPairs = 256;
struct PrepDesc {
  const float* v;   // [k][P][Q]
  const float* g;   // weight-norm gains, or null (plain weight)
  float* norm;      // [rows] ||v|| per weight-norm row (when g)
  float* npart;     // ConvTranspose under weight norm: [nchunks][Q] partial sums of squares
  f16 *fwd_hi, *fwd_lo;  // forward operand pair (fp16 hi + fp16 lo * 2^11, or the bf16 pair)
  bf16* dg;               // input-gradient operand (bf16)
  bf16* dg_lo;            // its lo companion (fp32 precision), or null
  int* range_err;         // set to ERR_RANGE if |W| >= 65504
  int fmt_bf16;           // forward pair as bf16 hi + bf16 lo (the range-safe fallback format)
  int P, Q, k, is_convT, stride;
  int qs;           // q columns per lane in the tile kernel (1, 2 or 4)
  int nchunks;      // ConvTranspose norm chunks
  int norm_first, tile_first;
};
int prep_norm_blocks(const PrepDesc& d);
int prep_tile_blocks(const PrepDesc& d);
void prep_weights(const PrepDesc* descs, int ndesc, int norm_blocks, int tile_blocks, cudaStream_t st);

// Weight-norm backward of many tensors in one launch (block = one dim-0 row of one tensor).
struct WnDesc {
  const float *dW, *v, *g, *norm;
  float *dv, *dg;
  int rows, cols, k, is_convT, first;
};
void wn_backward_batched(const WnDesc* descs, int ndesc, int total_rows, cudaStream_t st);

// weight-norm backward: dg[r] = <dW[r], v[r]>/n[r];  dv[r] = g[r]/n[r] * (dW[r] - dg[r]/n[r] * v[r])
// over dim-0 rows of a tap-major [k][C_out][C_in] tensor (rows x cols = C_out x C_in for a conv,
// C_in x C_out for a ConvTranspose).
void wn_backward(const float* dW, const float* v, const float* g, const float* norm, int rows, int cols, int k,
                 int is_convT, float* dv, float* dg, cudaStream_t st);

// Per-context step state kept on the device (a captured step graph advances it itself).
struct StepState {
  unsigned long long noise_stream;  // source-noise stream of the current step
  int adam_t;                       // AdamW step count
  int pad;
};
// Both skip a step whose forward reported a range error (err == ERR_RANGE), or, under data
// parallelism, on which any rank did (skip_flag > 0: the ranks' flags summed by the all-reduce); the
// step then leaves the parameters, moments and counters as they were, to be recomputed.  adamw also
// raises ERR_RANGE on this rank when only another rank overflowed, so every rank's host sees it.
void step_bump(StepState* s, int bump_noise, const int* err, const float* skip_flag, cudaStream_t st);

// AdamW over a flat buffer, restating the reference update (bias correction applied twice).
// Gradients are multiplied by grad_scale first (1/world under data parallelism).
void adamw(float* p, const float* g, float* m, float* v, long long n, float lr, float b1, float b2, float eps,
           float wd, const StepState* state, float grad_scale, int* err, const float* skip_flag, cudaStream_t st);
// flag = (err == ERR_RANGE) as a float, for the data-parallel all-reduce
void range_flag(const int* err, float* flag, cudaStream_t st);

// ---- inputs --------------------------------------------------------------------------------
// z [B][C][F] f32 -> [B][F][C] operand pair (fp16 hi / scaled lo, or the bf16 pair) and a bf16 copy
// (the conv_pre weight gradient's operand) with, when zb_lo is given, its lo companion (fp32 precision)
void pack_z(const float* z, int B, int C, int F, f16* hi, f16* lo, bf16* zb, bf16* zb_lo, int* range_err,
            int fmt_bf16, cudaStream_t st);

// cond(g): rowadd[b][c] = bias[c] + sum_i W[c][i] g[b][i]
void cond_forward(const float* W, const float* bias, const float* g, int B, int C, int gin, float* rowadd,
                  cudaStream_t st);
// per-item column sums of d_pre (from colsum tile partials) -> dW_cond, db_cond
void cond_backward(const float* tile_part, int tiles_per_item, int B, int C, const float* g, int gin, float* dW,
                   float* db, cudaStream_t st);

// ---- harmonic source ------------------------------------------------------------------------
struct NsfArgs {
  const float* f0;       // [B][F] Hz
  const float* noise;    // [B][T][dim] standard normals, or null -> counter generator
  const float* lin_w;    // [dim]
  const float* lin_b;    // [1]
  float* har;            // [B][T] tanh(l_linear(source))
  float* sw;             // [B][T][dim] source before l_linear (kept for the backward)
  double* acc;           // [B][F] scratch: phase carried into each frame
  int B, F, upp, dim;
  float sr, sine_amp, noise_std;
  unsigned long long seed;
  const unsigned long long* stream;  // device word: noise stream of this step
};
void nsf_forward(const NsfArgs& a, cudaStream_t st);
// l_linear gradients from d_har [B][T] (deterministic block partials + reduce)
void nsf_backward(const float* d_har, const float* har, const float* sw, int n, int dim, float* part, int nparts,
                  float* dlin_w, float* dlin_b, cudaStream_t st);

// ---- noise convs + activation of the stage input --------------------------------------------
// w [C][k] -> wt [k][C] (noise-conv weights, read coalesced by the kernels below)
void transpose_ck(const float* w, int C, int k, float* wt, cudaStream_t st);

struct NoiseActArgs {
  float* x;               // [B][T][C] ups output -> stage input (in place)
  const float* har;       // [B][T_full] or null (no source)
  const float* w;         // [k][C] (transposed)
  const float* bias;      // [C]
  int B, T, C, k, stride, pad, T_full;
  int act_kind;           // 0 lrelu 1 snake
  float slope;
  int n_act;              // snake: one activation per stack (alpha differs); lrelu: 1
  const float* alpha[3];
  f16* act_hi[3];         // activation: forward operand pair (fp16 hi + fp16 lo * 2^11) ...
  f16* act_lo[3];
  bf16* act_bf[3];        // ... and its bf16 copy (weight-gradient operand, LeakyReLU masks)
  bf16* act_bflo[3];      // lo companions of act_bf (fp32 precision), or null
  bf16* pre;              // bf16 copy of x (snake masks)
  bf16* pre_lo;           // its lo companion (fp32 precision), or null
  int* range_err;         // set to ERR_RANGE if |activation| >= 65504
  int fmt_bf16;           // operand pair as bf16 hi + lo (fallback format)
};
void noise_add_act(const NoiseActArgs& a, cudaStream_t st);

// backward of the noise conv: d_har[b][t] (+)= ..., weight-gradient partials
//   wt [k][C] transposed weights; wpart [noise_backward_parts][C][k]; g scratch [B*T][k]
void noise_backward(const float* dx, const float* har, const float* wt, int B, int T, int C, int k, int stride, int pad,
                    int T_full, float* d_har, int accumulate_dhar, float* wpart, float* g, cudaStream_t st);
int noise_backward_parts(int B, int T, int C, int k);
// dynamic shared memory of noise_add_act for a noise conv of k taps and the given stride
size_t noise_act_smem(int k, int stride);
void noise_wgrad_reduce(const float* wpart, int nparts, int C, int k, float* dW, float* scratch, size_t scratch_floats,
                        cudaStream_t st);

// ---- conv_post ------------------------------------------------------------------------------
// audio[b][t] = tanh(sum_{c,tap} a[b][t-3+tap][c] * W[c][tap]), a = the operand pair (hi, lo)
void post_forward(const f16* a_hi, const f16* a_lo, int fmt_bf16, const float* W, int B, int T, int C, int k,
                  float* audio, cudaStream_t st);
// d_pre = dy*(1-y^2); d_a = conv_post^T(d_pre); d_stage = d_a * act'(stage) * scale -> f32 + bf16
// partials: colsum of d_stage (64-row blocks), dW_post, snake d(alpha)
struct PostBwdArgs {
  const float* dy;        // [B][T]
  const float* audio;     // [B][T]
  const float* W;         // [C][k]
  const f16* a_hi;        // [B][T][C] activation (wgrad operand): the operand pair
  const f16* a_lo;
  int fmt_bf16;           // pair format of a_hi / a_lo
  const bf16* mask_src;   // activated (lrelu sign) or pre-activation (snake)
  const bf16* mask_lo;    // lo companion of a Snake mask source (fp32 precision), or null
  const float* alpha;     // snake alpha [C]
  int act_kind;
  float slope, scale;
  int B, T, C, k;
  float* d_stage;         // [B][T][C] f32
  bf16* d_stage_bf;       // [B][T][C]
  bf16* d_stage_bf_lo;    // its lo companion (fp32 precision), or null
  float* colsum_part;     // [nblk][C]
  float* w_part;          // [nblk][C*k]
  float* alpha_part;      // [nblk][C]
};
int post_backward_blocks(int B, int T);
void post_backward(const PostBwdArgs& a, cudaStream_t st);

// generic [nparts][n] -> out[n] fixed-order reduction (optionally accumulating)
void rows_reduce(const float* part, int nparts, int n, float* out, int accumulate, cudaStream_t st);

}  // namespace wb
