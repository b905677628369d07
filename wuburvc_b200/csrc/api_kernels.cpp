// api_kernels.cpp — C-ABI entry points for single convolution primitives on device buffers.
// Each call plans, launches and synchronises one operation (used by the kernel-level tests and
// by callers that want one layer at a time); the training step uses persistent plans instead.
#include <cstdio>
#include <vector>

#include "../../include/wuburvc_b200.h"
#include "conv_plan.h"
#include "small_kernels.cuh"

namespace wb {
// stft_loss.cu
size_t stft_scratch_floats(int B, int n, int n_scales);
cudaError_t stft_loss_grad(const float* a, const float* b, int B, int n, int n_scales, float* grad, float* loss,
                           float* scratch, cudaStream_t st);
}  // namespace wb

using namespace wb;

namespace {

// One warp waits, with the kernels' bounded wait, on a barrier that nothing arrives on: the wait runs
// out after limit_ns by design and records ERR_WAIT_FULL.  Nothing is in flight, so the kernel simply
// returns.
__global__ void wait_probe_kernel(int* err, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  mbar_wait_warp(&bar, 0, err, ERR_WAIT_FULL, limit_ns);
}

struct Scratch {
  int* err = nullptr;
  float* part = nullptr;
  int* tabs = nullptr;
  ~Scratch() {
    if (err) cudaFree(err);
    if (part) cudaFree(part);
    if (tabs) cudaFree(tabs);
  }
};

int finish(cudaStream_t st, int* derr) {
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    fprintf(stderr, "wuburvc_b200: CUDA error %s\n", cudaGetErrorString(e));
    return WUBU_B200_ERR_CUDA;
  }
  int h = 0;
  cudaMemcpy(&h, derr, sizeof(int), cudaMemcpyDeviceToHost);
  if (h) {
    fprintf(stderr, "wuburvc_b200: kernel reported error %d\n", h);
    return h == ERR_RANGE ? WUBU_B200_ERR_RANGE : WUBU_B200_ERR_TIMEOUT;
  }
  return WUBU_B200_OK;
}

bool launched(cudaError_t e) {
  if (e != cudaSuccess) fprintf(stderr, "wuburvc_b200: launch failed: %s\n", cudaGetErrorString(e));
  return e == cudaSuccess;
}

// Positive sizes and the pointers a launch dereferences (a null operand would become a tensor map at
// address 0, which the kernel would then read).
bool dims_ok(int B, int a, int b, int c, int k) { return B > 0 && a > 0 && b > 0 && c > 0 && k > 0; }

Epi plain_epi(const float* bias, float* out) {
  Epi e{};
  e.bias = bias;
  e.out_f32 = out;
  e.scale = 1.f;
  e.slope = 0.1f;
  return e;
}

int run_wgrad(WgradLaunch& L, Scratch& s, int layout, int c_out, int k, float* dw, cudaStream_t st) {
  std::vector<int> tab(L.row_tap);
  tab.insert(tab.end(), L.row_oc.begin(), L.row_oc.end());
  if (cudaMalloc(&s.tabs, tab.size() * sizeof(int)) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  cudaMemcpy(s.tabs, tab.data(), tab.size() * sizeof(int), cudaMemcpyHostToDevice);
  if (!launched(L.run(st))) return WUBU_B200_ERR_CUDA;
  const int rows = L.p.n_mtiles * 128;
  wgrad_reduce(s.part, L.splits, rows, L.p.n_total, s.tabs, s.tabs + rows, layout, c_out, k, dw, 0, nullptr, 0, st);
  return finish(st, s.err);
}

}  // namespace

extern "C" {

int wubu_b200_conv1d(const void* x_hi, const void* x_lo, const void* w_hi, const void* w_lo, const float* bias,
                     float* out, int B, int C_in, int T, int C_out, int k, int dil, int pad, int split,
                     void* stream) {
  if (!x_hi || !w_hi || !out || (split && (!x_lo || !w_lo)) || !dims_ok(B, C_in, T, C_out, k) || dil < 1 ||
      pad < 0 || T + 2 * pad - dil * (k - 1) < 1)
    return WUBU_B200_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  Scratch s;
  if (cudaMalloc(&s.err, sizeof(int)) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  cudaMemsetAsync(s.err, 0, sizeof(int), st);
  ConvGeom g{B, T, T + 2 * pad - dil * (k - 1), C_in, C_out, k, dil, pad};
  ConvOp L;
  if (!plan_conv_any(L, g, x_hi, x_lo, w_hi, w_lo, split, plain_epi(bias, out), s.err)) return WUBU_B200_ERR_SHAPE;
  if (!launched(L.run(st))) return WUBU_B200_ERR_CUDA;
  return finish(st, s.err);
}

int wubu_b200_conv1d_wgrad(const void* dy, const void* x, float* dw, int B, int C_in, int T, int C_out, int k,
                           int dil, int pad, void* stream) {
  if (!dy || !x || !dw || !dims_ok(B, C_in, T, C_out, k) || dil < 1 || pad < 0 || T + 2 * pad - dil * (k - 1) < 1)
    return WUBU_B200_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  Scratch s;
  if (cudaMalloc(&s.err, sizeof(int)) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  cudaMemsetAsync(s.err, 0, sizeof(int), st);
  ConvGeom g{B, T, T + 2 * pad - dil * (k - 1), C_in, C_out, k, dil, pad};
  WgradLaunch L;
  if (!plan_wgrad(L, g, dy, x, nullptr, ~size_t(0), 296, s.err)) return WUBU_B200_ERR_SHAPE;
  if (cudaMalloc(&s.part, wgrad_part_floats(L) * sizeof(float)) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  L.p.part = s.part;
  return run_wgrad(L, s, 0, C_out, k, dw, st);
}

int wubu_b200_convT(const void* x_hi, const void* x_lo, const void* wp_hi, const void* wp_lo, const float* bias,
                    float* out, int B, int C_in, int T_in, int C_out, int k, int stride, int pad, int split,
                    void* stream) {
  if (!x_hi || !wp_hi || !out || (split && (!x_lo || !wp_lo)) || !dims_ok(B, C_in, T_in, C_out, k) || stride < 1 ||
      pad < 0)
    return WUBU_B200_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  Scratch s;
  if (cudaMalloc(&s.err, sizeof(int)) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  cudaMemsetAsync(s.err, 0, sizeof(int), st);
  ConvLaunch L;
  if (!plan_convT(L, B, T_in, C_in, C_out, k, stride, pad, x_hi, x_lo, wp_hi, wp_lo, split, plain_epi(bias, out),
                  s.err))
    return WUBU_B200_ERR_SHAPE;
  if (!launched(L.run(st))) return WUBU_B200_ERR_CUDA;
  return finish(st, s.err);
}

int wubu_b200_convT_dgrad(const void* dy, const void* wd, float* dx, int B, int C_in, int T_in, int C_out, int k,
                          int stride, int pad, void* stream) {
  if (!dy || !wd || !dx || !dims_ok(B, C_in, T_in, C_out, k) || stride < 1 || pad < 0) return WUBU_B200_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  Scratch s;
  if (cudaMalloc(&s.err, sizeof(int)) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  cudaMemsetAsync(s.err, 0, sizeof(int), st);
  ConvLaunch L;
  if (!plan_convT_dgrad(L, B, T_in, C_in, C_out, k, stride, pad, dy, wd, nullptr, nullptr, plain_epi(nullptr, dx), s.err))
    return WUBU_B200_ERR_SHAPE;
  if (!launched(L.run(st))) return WUBU_B200_ERR_CUDA;
  return finish(st, s.err);
}

int wubu_b200_convT_wgrad(const void* x, const void* dy, float* dw, int B, int C_in, int T_in, int C_out, int k,
                          int stride, int pad, void* stream) {
  if (!x || !dy || !dw || !dims_ok(B, C_in, T_in, C_out, k) || stride < 1 || pad < 0) return WUBU_B200_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  Scratch s;
  if (cudaMalloc(&s.err, sizeof(int)) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  cudaMemsetAsync(s.err, 0, sizeof(int), st);
  WgradLaunch L;
  if (!plan_convT_wgrad(L, B, T_in, C_in, C_out, k, stride, pad, x, dy, nullptr, ~size_t(0), 296, s.err))
    return WUBU_B200_ERR_SHAPE;
  if (cudaMalloc(&s.part, wgrad_part_floats(L) * sizeof(float)) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  L.p.part = s.part;
  return run_wgrad(L, s, 1, C_out, k, dw, st);
}

int wubu_b200_stft_loss_grad(const float* a, const float* b, int B, int n, int n_scales, float* grad, float* loss,
                             void* stream) {
  if (!a || !b || !grad || !loss || B < 1 || n < 1 || B > 65535) return WUBU_B200_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  float* scratch = nullptr;
  if (cudaMallocAsync(&scratch, stft_scratch_floats(B, n, n_scales) * sizeof(float), st) != cudaSuccess)
    return WUBU_B200_ERR_CUDA;
  const cudaError_t e = stft_loss_grad(a, b, B, n, n_scales, grad, loss, scratch, st);
  cudaFreeAsync(scratch, st);
  if (e != cudaSuccess) return WUBU_B200_ERR_CUDA;
  const cudaError_t s2 = cudaStreamSynchronize(st);
  if (s2 != cudaSuccess) {
    fprintf(stderr, "wuburvc_b200: CUDA error %s\n", cudaGetErrorString(s2));
    return WUBU_B200_ERR_CUDA;
  }
  return WUBU_B200_OK;
}

int wubu_b200_stft_loss_grad_host(const float* a, const float* b, int B, int n, int n_scales, float* grad,
                                  float* loss) {
  if (!a || !b || !grad || !loss || B < 1 || n < 1 || B > 65535) return WUBU_B200_ERR_ARG;
  const size_t bytes = sizeof(float) * (size_t)B * n;
  float *da = nullptr, *db = nullptr, *dg = nullptr, *dl = nullptr;
  int rc = WUBU_B200_ERR_CUDA;
  if (cudaMalloc(&da, bytes) == cudaSuccess && cudaMalloc(&db, bytes) == cudaSuccess &&
      cudaMalloc(&dg, bytes) == cudaSuccess && cudaMalloc(&dl, sizeof(float) * B) == cudaSuccess &&
      cudaMemcpy(da, a, bytes, cudaMemcpyHostToDevice) == cudaSuccess &&
      cudaMemcpy(db, b, bytes, cudaMemcpyHostToDevice) == cudaSuccess) {
    rc = wubu_b200_stft_loss_grad(da, db, B, n, n_scales, dg, dl, nullptr);
    if (rc == WUBU_B200_OK && (cudaMemcpy(grad, dg, bytes, cudaMemcpyDeviceToHost) != cudaSuccess ||
                               cudaMemcpy(loss, dl, sizeof(float) * B, cudaMemcpyDeviceToHost) != cudaSuccess))
      rc = WUBU_B200_ERR_CUDA;
  }
  cudaFree(da);
  cudaFree(db);
  cudaFree(dg);
  cudaFree(dl);
  return rc;
}

int wubu_b200_set_wait_limit_ns(unsigned long long ns) {
  set_wait_limit_ns(ns);
  return WUBU_B200_OK;
}

int wubu_b200_wait_selftest(unsigned long long limit_ns, void* stream) {
  if (limit_ns == 0 || limit_ns > 10000000000ull) return WUBU_B200_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  Scratch s;
  if (cudaMalloc(&s.err, sizeof(int)) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  if (cudaMemsetAsync(s.err, 0, sizeof(int), st) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  wait_probe_kernel<<<1, 32, 0, st>>>(s.err, limit_ns);
  if (!launched(cudaGetLastError())) return WUBU_B200_ERR_CUDA;
  return finish(st, s.err);
}

}  // extern "C"
