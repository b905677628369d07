// small_kernels.cuh — deterministic reductions (fixed summation order, no atomics).
#pragma once
#include "common.cuh"

namespace wb {

// out[j] (+)= sum_p part[p][j] for j < n.  With scratch (>= ceil(nparts/64) * n floats) large part
// counts are reduced in two passes.
void col_reduce(const float* part, int nparts, long long n, float* out, int accumulate, float* scratch,
                size_t scratch_floats, cudaStream_t st);

// dW from split-K partial tiles part[split][rows][n_total]; rows map to (tap, oc) through row_tap /
// row_oc.  layout 0: dW[oc][ic][tap] (Conv1d), layout 1: dW[ic][oc][tap] (ConvTranspose1d).
void wgrad_reduce(const float* part, int splits, int rows, int n_total, const int* row_tap, const int* row_oc,
                  int layout, int c_out, int k, float* dw, int accumulate, float* scratch, size_t scratch_floats,
                  cudaStream_t st);

// Split-K reduction of weight-gradient partials into the parameter layout (one block per dim-0
// row), fused with the weight-norm backward when g != null:
//   conv  (layout 0): row r = oc, dW[oc][ic][tap];  convT (layout 1): row r = ic, dW[ic][oc][tap]
//   inv[oc * k + tap] = partial row of (tap, oc).  Without weight norm dv receives dW.
void wgrad_finish(const float* part, int splits, int rows, int n_total, const int* inv, int layout, int c_out, int k,
                  int dim0_rows, const float* v, const float* g, const float* norm, float* dv, float* dg,
                  cudaStream_t st);

// Many column reductions in one launch: out_i[j] = sum_{p < nparts_i} part_i[p * ld_i + j], j < n_i.
// A descriptor is served by colblocks x nchunks blocks (128 columns x up to kReduceChunk parts each);
// with several chunks, each block stores its chunk sum in `scratch` [nchunks][n] and the last block of
// a column group (counted in `counter`, which it resets) adds the chunk sums in chunk order, so the
// result does not depend on block scheduling.
constexpr int kReduceChunk = 64;
struct ReduceDesc {
  const float* part;
  float* out;
  long long ld, n;
  int nparts, first_block, colblocks, nchunks;
  float* scratch;          // nchunks * n floats when nchunks > 1
  unsigned int* counter;   // colblocks zeroed words when nchunks > 1
};
// Fills the launch shape of d (first_block = blocks already in the table); returns its block count and
// the scratch floats / counters it needs, or -1 when n or ld is not a multiple of 4 or part is not
// 16-byte aligned (the kernel reads float4 partials).
int reduce_desc_shape(ReduceDesc& d, int first_block, size_t* scratch_floats, size_t* counters);
void reduce_batched(const ReduceDesc* descs, int ndesc, int total_blocks, cudaStream_t st);

// column sums of per-tile partials part[tiles][C]
void colsum_reduce(const float* part, int tiles, int C, float* out, int accumulate, float* scratch,
                   size_t scratch_floats, cudaStream_t st);

// Scratch used by the overloads below (set by the training context before it enqueues work).
void set_reduce_scratch(float* scratch, size_t floats);
void col_reduce(const float* part, int nparts, long long n, float* out, int accumulate, cudaStream_t st);
// parts of length n placed ld floats apart
void col_reduce_ld(const float* part, int nparts, long long n, long long ld, float* out, int accumulate,
                   cudaStream_t st);
void colsum_reduce(const float* part, int tiles, int C, float* out, int accumulate, cudaStream_t st);
void wgrad_reduce(const float* part, int splits, int rows, int n_total, const int* row_tap, const int* row_oc,
                  int layout, int c_out, int k, float* dw, int accumulate, cudaStream_t st);

}  // namespace wb
