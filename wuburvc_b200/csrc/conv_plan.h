// conv_plan.h — host-side planning of the tcgen05 convolution launches.
//
// A plan holds the encoded TMA descriptors and the kernel parameters of one launch; plans
// are built once per model (buffers are persistent) and replayed every step.
#pragma once
#include <vector>

#include "tc_conv.cuh"

namespace wb {

void tc_kernels_init();  // raises the kernels' shared-memory limit (call before graph capture)
// Bounded-wait limit (ns) written into every plan built afterwards (default kWaitLimitNs; 0 restores it).
unsigned long long wait_limit_ns();
void set_wait_limit_ns(unsigned long long ns);
cudaError_t launch_tc_conv(const TcMaps& maps, const TcConvParams& p, int kc, dim3 grid, size_t smem,
                           cudaStream_t st);
cudaError_t launch_tc_wgrad(const TcWgMaps& maps, const TcWgParams& p, dim3 grid, size_t smem,
                            cudaStream_t st);

// Encodes a 3-D bf16 tensor map: dims (d0 inner, d1, d2), byte strides of d1 and d2.
bool make_map_bf16_3d(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                      uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1, uint32_t b2);

struct ConvLaunch {
  TcMaps maps;
  TcConvParams p;
  dim3 grid;
  size_t smem = 0;
  int kc = 64;
  cudaError_t run(cudaStream_t st) const { return launch_tc_conv(maps, p, kc, grid, smem, st); }
};

cudaError_t launch_tc_conv2(const TcConv2Maps& maps, const TcConv2Params& p, int kc, int grid, size_t smem,
                            cudaStream_t st);

struct Conv2Launch {
  TcConv2Maps maps;
  TcConv2Params p;
  int grid = 0;
  size_t smem = 0;
  int kc = 64;
  cudaError_t run(cudaStream_t st) const { return launch_tc_conv2(maps, p, kc, grid, smem, st); }
};

// A stride-1 convolution planned on the persistent halo kernel when its shape allows, else on
// the general kernel.
struct ConvOp {
  bool v2 = false;
  ConvLaunch v1;
  Conv2Launch c2;
  cudaError_t run(cudaStream_t st) const { return v2 ? c2.run(st) : v1.run(st); }
  // rows of the [partials][C] column-sum buffers this launch writes (one per CTA or per tile)
  int partials() const { return v2 ? 2 * c2.grid : (int)(v1.grid.x * v1.grid.z); }
  // programmatic dependent launch for the persistent kernel (see TcConv2Params::pdl)
  void set_pdl(bool on) {
    c2.p.pdl = on ? 1 : 0;
    v1.p.pdl = on ? 1 : 0;
  }
  // re-points the epilogue's column-sum partial buffer
  void set_colsum(float* p) {
    v1.p.epi.colsum = p;
    c2.p.epi.colsum = p;
  }
};

struct WgradLaunch {
  TcWgMaps maps;
  TcWgParams p;
  dim3 grid;
  size_t smem = 0;
  int splits = 1;
  // reduce: rows (mtile*128 + m) -> (tap, oc); layout of the final dW
  std::vector<int> row_tap, row_oc;
  cudaError_t run(cudaStream_t st) const { return launch_tc_wgrad(maps, p, grid, smem, st); }
};

// Geometry of a stride-1 Conv1d on channels-last [B][T][C] tensors.
struct ConvGeom {
  int B, T_in, T_out, C_in, C_out, k, dil, pad;
};

// Forward conv (also dgrad with flipped taps when `flip` is set: weights are then laid out
// [tap][C_out_of_dgrad][C_in_of_dgrad] already flipped by the weight-prep kernel).
//   x_hi/x_lo : [B][T_in][C_in] bf16 (x_lo may be null when split == 0)
//   w_hi/w_lo : [k][C_out][C_in] bf16
bool plan_conv(ConvLaunch& L, const ConvGeom& g, const void* x_hi, const void* x_lo, const void* w_hi,
               const void* w_lo, int split, const Epi& epi, int* err);

// Persistent halo-reuse plan (stride-1, T_in == T_out, C_out <= 256); false if the shape does not fit.
bool plan_conv2(Conv2Launch& L, const ConvGeom& g, const void* x_hi, const void* x_lo, const void* w_hi,
                const void* w_lo, int split, const Epi& epi, int* err);
// plan_conv2 when possible (unless WUBU_B200_CONV_V1 is set), else plan_conv.
bool plan_conv_any(ConvOp& op, const ConvGeom& g, const void* x_hi, const void* x_lo, const void* w_hi,
                   const void* w_lo, int split, const Epi& epi, int* err);

// ConvTranspose1d forward as polyphase conv: x [B][T_in][C_in], w (per-phase packed)
// [n_phase_taps][C_out][C_in]; output [B][T_in*s][C_out].
bool plan_convT(ConvLaunch& L, int B, int T_in, int C_in, int C_out, int k, int s, int pad,
                const void* x_hi, const void* x_lo, const void* wp_hi, const void* wp_lo, int split,
                const Epi& epi, int* err);

// ConvTranspose1d input-gradient: dx[b,i,ci] = sum_tap sum_co dy[b, i*s - pad + tap, co] * W[ci][co][tap]
//   dy [B][T_out][C_out] bf16; wd [k][C_in][C_out] bf16 (tap-major, K-major in C_out).  With dy_lo and
//   wd_lo (their bf16 lo companions) the operands are bf16 pairs and three products are taken.
bool plan_convT_dgrad(ConvLaunch& L, int B, int T_in, int C_in, int C_out, int k, int s, int pad,
                      const void* dy, const void* wd, const void* dy_lo, const void* wd_lo, const Epi& epi,
                      int* err);

// Conv1d weight gradient: dW[co][ci][tap] = sum_{b,t} dy[b,t,co] * x[b, t - pad + dil*tap, ci]
bool plan_wgrad(WgradLaunch& L, const ConvGeom& g, const void* dy, const void* x, float* part,
                size_t part_capacity_floats, int target_ctas, int* err);

// ConvTranspose1d weight gradient: dW[ci][co][tap] = sum_{b,i} x[b,i,ci] * dy[b, i*s - pad + tap, co]
bool plan_convT_wgrad(WgradLaunch& L, int B, int T_in, int C_in, int C_out, int k, int s, int pad,
                      const void* x, const void* dy, float* part, size_t part_capacity_floats,
                      int target_ctas, int* err);

size_t wgrad_part_floats(const WgradLaunch& L);

}  // namespace wb
