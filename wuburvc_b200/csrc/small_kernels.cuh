// small_kernels.cuh — declarations of the bandwidth-bound helper kernels.
#pragma once
#include "common.cuh"

namespace wb {

// layout 0: dW[oc][ic][tap] (Conv1d), layout 1: dW[ic][oc][tap] (ConvTranspose1d)
void wgrad_reduce(const float* part, int splits, int rows, int n_total, const int* row_tap, const int* row_oc,
                  int layout, int c_out, int k, float* dw, int accumulate, cudaStream_t st);

void colsum_reduce(const float* part, int tiles, int C, float* out, int accumulate, cudaStream_t st);

}  // namespace wb
