// gen_model.h — internal state of one generator training context (one GPU).
#pragma once
#include <memory>
#include <string>
#include <vector>

#include "conv_plan.h"
#include "gen_kernels.cuh"
#include "param_table.h"
#include "small_kernels.cuh"

namespace wb {

struct Comm;  // NCCL communicator + bucket plan (comm.cpp)

// Derived GEMM weights of one convolution and where its gradient goes.
struct ConvWeights {
  int pv = -1, pg = -1, pb = -1;  // param indices (v or W, g, bias)
  int rows = 0, cols = 0, k = 0;  // param dims: conv [C_out][C_in][k], convT [C_in][C_out][k]
  int convT = 0, stride = 1;
  f16 *fwd_hi = nullptr, *fwd_lo = nullptr;  // forward operand pair (see Gen::op_bf16)
  bf16* dg = nullptr;                         // input-gradient operand
  bf16* dg_lo = nullptr;                      // its lo companion (fp32 precision)
  float* norm = nullptr;  // ||v|| rows (weight norm)
  float* dW = nullptr;    // gradient in param layout (grad buffer directly, or a temp under weight norm)
};

struct WgradJob {
  WgradLaunch L;
  // fp32 precision: the products dy_hi x x_lo and dy_lo x x_hi, same plan, their partials after L's
  WgradLaunch lo[2];
  int nl = 1;  // launches (1, or 3 under fp32 precision)
  float* part = nullptr;  // this job's split-K partials (reduced later in a batched launch)
  int flush = -1;         // WgradBatch of the stage to launch after this job's kernel (-1: none)
  const ConvWeights* w = nullptr;
  int layout = 0;      // 0 conv, 1 convT
  int c_out = 0, k = 0;
  float* dW = nullptr;
};

// Split-K reductions of several weight gradients (one launch) and their weight-norm backward (one).
struct WgradBatch {
  ReduceDesc* wg_d = nullptr;
  int wg_n = 0, wg_blocks = 0;
  WnDesc* wn_d = nullptr;
  int wn_n = 0, wn_rows = 0;
};

struct StackBufs {
  // forward (index = pair)
  // activations: forward operand pair (see Gen::op_bf16), bf16 copy (weight-gradient operand and
  // LeakyReLU mask), bf16 pre-activation (Snake masks)
  f16 *a1_hi[3] = {}, *a1_lo[3] = {};                    // activation of the pair input
  bf16 *a1_bf[3] = {}, *a1_pre[3] = {};
  float* p[3] = {};                                      // pair input (p[0] aliases the stage input)
  f16 *a2_hi[3] = {}, *a2_lo[3] = {};                    // activation of conv1's output
  bf16 *a2_bf[3] = {}, *a2_pre[3] = {};
  // fp32 precision: bf16 lo companions of the bf16 tensors (null otherwise)
  bf16 *a1_bflo[3] = {}, *a1_prelo[3] = {}, *a2_bflo[3] = {}, *a2_prelo[3] = {};
  // backward
  bf16* d_c1 = nullptr;
  bf16* d_c1_lo = nullptr;
  float* pp[2] = {};
  bf16* pp_bf[2] = {};
  bf16* pp_bflo[2] = {};
  float *cs_dc1[3] = {}, *cs_dp[3] = {}, *ap1[3] = {}, *ap2[3] = {};
  int tiles = 0;
  ConvWeights w1[3], w2[3];
  ConvOp f1[3], f2[3], d2[3], d1[3];
  ConvOp f1f[3], f2f[3];  // fast inference: single fp16 operands (planned on first use)
  WgradJob g1[3], g2[3];
};

struct StageBufs {
  int T = 0, C = 0, Cin = 0, rows = 0, ku = 0, su = 0, pu = 0;
  int kn = 0, sn = 0, pn = 0;
  float* x_in = nullptr;
  f16 *xa_hi[3] = {}, *xa_lo[3] = {};
  bf16 *xa_bf[3] = {}, *x_pre = nullptr;
  float* sout = nullptr;
  f16 *sa_hi = nullptr, *sa_lo = nullptr;
  bf16 *sa_bf = nullptr, *s_pre = nullptr;
  float* d_s = nullptr;
  bf16* d_s_bf = nullptr;
  float* d_x = nullptr;
  bf16* d_x_bf = nullptr;
  // fp32 precision: bf16 lo companions (null otherwise)
  bf16 *xa_bflo[3] = {}, *x_prelo = nullptr, *sa_bflo = nullptr, *s_prelo = nullptr;
  bf16 *d_s_bflo = nullptr, *d_x_bflo = nullptr;
  float* cs_ds = nullptr;  // colsum partials of d_s (from its producer)
  int cs_ds_tiles = 0;
  float* ap_up = nullptr;  // snake alpha partials of the activation feeding ups L (from up_dg)
  int ap_up_tiles = 0;
  float* noise_wpart = nullptr;
  float* noise_g = nullptr;  // noise-conv input-gradient rows [B*T][k]
  float* noise_wt = nullptr;  // noise-conv weights transposed to [k][C]
  int noise_parts = 0;
  ConvWeights wu;
  ConvLaunch up_fwd, up_dg;
  ConvLaunch up_fast;  // fast inference
  WgradJob up_wg;
  StackBufs st[3];
  float* cs_dx = nullptr;  // the stacks' cs_dp[0] partial slots, contiguous (ups / noise-conv bias)
  // batched reductions (device descriptor tables): the weight gradients in groups whose split-K
  // partials stay L2-sized, and all of the stage's bias / Snake-alpha column sums at its end
  std::vector<WgradBatch> wg_batches;
  ReduceDesc* cs_d = nullptr;
  int cs_n = 0, cs_blocks = 0;
};

struct Gen {
  WubuB200GenConfig cfg{};
  WubuB200TrainOptions opt{};
  ParamTable table;
  int B = 0, F = 0, T = 0, dim = 0, upp = 0;
  int nk = 3, nd = 3;
  cudaStream_t stream = nullptr;
  // the backward's reductions (split-K sums, weight-norm backward, bias / alpha column sums) run on
  // a second stream, overlapping the next convolutions; `evs` is a pool for the fork / join edges
  cudaStream_t side = nullptr;
  std::vector<cudaEvent_t> evs;
  int ev_next = 0;
  std::vector<void*> allocs;
  int* err = nullptr;

  float *params = nullptr, *grads = nullptr, *adam_m = nullptr, *adam_v = nullptr;
  StepState* state = nullptr;  // device: noise stream + AdamW step

  // inputs
  float *z = nullptr, *f0 = nullptr, *g = nullptr, *noise = nullptr, *dldy = nullptr;
  bool has_noise_input = false;
  f16 *z_hi = nullptr, *z_lo = nullptr;
  bf16* z_bf = nullptr;
  bf16* z_bflo = nullptr;  // fp32 precision
  // source
  float *har = nullptr, *sw = nullptr, *d_har = nullptr, *nsf_part = nullptr;
  double* nsf_acc = nullptr;
  int nsf_parts = 0;
  // conv_pre / cond
  ConvWeights wpre;
  float* rowadd = nullptr;
  f16 *pre_hi = nullptr, *pre_lo = nullptr;
  bf16 *pre_bf = nullptr, *pre_pre = nullptr;
  bf16* d_pre_bf = nullptr;
  bf16 *pre_bflo = nullptr, *pre_prelo = nullptr, *d_pre_bflo = nullptr;  // fp32 precision
  float* cs_pre = nullptr;
  int cs_pre_tiles = 0, pre_tiles_per_item = 0;
  ConvLaunch pre_fwd;
  ConvLaunch pre_fast;  // fast inference
  WgradJob pre_wg;
  // conv_post
  float* audio = nullptr;
  float *post_cs = nullptr, *post_wpart = nullptr, *post_ap = nullptr;
  int post_blocks = 0;

  StageBufs sg[4];
  PrepDesc* prep_descs = nullptr;  // device table: every GEMM weight's preparation
  std::vector<PrepDesc> prep_host; // host copy (re-uploaded when the operand format changes)
  std::vector<const ConvWeights*> all_weights;  // the weights of prep_host, in its order
  // forward operand format: 0 = fp16 hi + fp16 lo*2^11 (fp32-accurate, |x| < 65504); 1 = bf16 hi +
  // bf16 lo (range-safe, ~2^-17), the format a context switches to for good after a range error
  int op_bf16 = 0;
  // backward GEMM operands as bf16 hi + lo pairs (opt.precision == WUBU_B200_PRECISION_FP32)
  int fp32 = 0;
  // forward-only (inference): the forward skips what only the backward reads (bf16 activation copies,
  // Snake pre-activations, z's bf16 copy, the input-gradient weight layout); no backward runs
  int forward_only = 0;
  // fast inference (forward-only): single fp16 operands, one product per K step (forward rel-L2 ~4e-4
  // against fp64); left for the exact pairs after a range error
  int fast = 0;
  bool fast_planned = false;
  int n_prep = 0, prep_norm_blocks = 0, prep_tile_blocks = 0;
  float* red_scratch = nullptr;  // two-pass deterministic reductions
  size_t red_scratch_n = 0;
  float* noise_scratch = nullptr;  // the same for the noise-conv weight gradients (side stream)
  size_t noise_scratch_n = 0;

  // CUDA graph of the resident-input step
  cudaGraphExec_t graph = nullptr;
  int graph_kernels = 0;  // kernel nodes in the captured step



  Comm* comm = nullptr;  // owned; released by comm_destroy

  int pidx(const std::string& n) const { return table.find(n); }
  float* P(int i) { return params + table.e[i].off; }
  float* G(int i) { return grads + table.e[i].off; }
};

}  // namespace wb
