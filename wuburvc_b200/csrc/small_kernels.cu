// small_kernels.cu — bandwidth-bound helper kernels shared by the step.
#include "small_kernels.cuh"

namespace wb {

// dW from split-K partial tiles, fixed summation order (deterministic).
__global__ void wgrad_reduce_kernel(const float* __restrict__ part, int splits, int rows, int n_total,
                                    const int* __restrict__ row_tap, const int* __restrict__ row_oc, int layout,
                                    int c_out, int k, float* __restrict__ dw, int accumulate) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)rows * n_total) return;
  const int row = (int)(idx / n_total), ic = (int)(idx % n_total);
  const int tap = row_tap[row];
  if (tap < 0) return;
  const int oc = row_oc[row];
  float s = 0.f;
  for (int sp = 0; sp < splits; ++sp) s += part[((size_t)sp * rows + row) * n_total + ic];
  size_t o = (layout == 0) ? ((size_t)oc * n_total + ic) * k + tap : ((size_t)ic * c_out + oc) * k + tap;
  dw[o] = accumulate ? dw[o] + s : s;
}

void wgrad_reduce(const float* part, int splits, int rows, int n_total, const int* row_tap, const int* row_oc,
                  int layout, int c_out, int k, float* dw, int accumulate, cudaStream_t st) {
  const long long n = (long long)rows * n_total;
  wgrad_reduce_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(part, splits, rows, n_total, row_tap, row_oc,
                                                                   layout, c_out, k, dw, accumulate);
}

// column partial sums [tiles][C] -> out[C] (fixed order)
__global__ void colsum_reduce_kernel(const float* __restrict__ part, int tiles, int C, float* __restrict__ out,
                                     int accumulate) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  float s = 0.f;
  for (int t = 0; t < tiles; ++t) s += part[(size_t)t * C + c];
  out[c] = accumulate ? out[c] + s : s;
}

void colsum_reduce(const float* part, int tiles, int C, float* out, int accumulate, cudaStream_t st) {
  colsum_reduce_kernel<<<(C + 127) / 128, 128, 0, st>>>(part, tiles, C, out, accumulate);
}

}  // namespace wb
