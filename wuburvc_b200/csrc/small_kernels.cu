// small_kernels.cu — deterministic reductions shared by the step.
#include "small_kernels.cuh"

namespace wb {

namespace {

constexpr int kRowsPerThread = 8;   // parts summed by one thread in a pass
constexpr int kYLanes = 8;          // part-lanes per block (block = 32 columns x 8 lanes)
constexpr int kPartsPerBlock = kRowsPerThread * kYLanes;

struct Scatter {
  int mode;  // 0 identity, 1 conv dW[oc][ic][tap], 2 convT dW[ic][oc][tap]
  int n_total, c_out, k;
  const int* row_tap;
  const int* row_oc;
};

__device__ __forceinline__ long long scatter_index(const Scatter& s, long long j) {
  if (s.mode == 0) return j;
  const int row = (int)(j / s.n_total), ic = (int)(j % s.n_total);
  const int tap = s.row_tap[row];
  if (tap < 0) return -1;
  const int oc = s.row_oc[row];
  return s.mode == 1 ? ((long long)oc * s.n_total + ic) * s.k + tap : ((long long)ic * s.c_out + oc) * s.k + tap;
}

// out[g][j] = sum of parts [g*kPartsPerBlock, (g+1)*kPartsPerBlock) of column j  (pass 1), or the
// final sum with scatter/accumulate when gridDim.y == 1 (single pass / pass 2).
__global__ void col_reduce_kernel(const float* __restrict__ part, int nparts, long long n, long long ld,
                                  float* __restrict__ out, int accumulate, Scatter sc, int final_pass) {
  __shared__ float sh[kYLanes][33];
  const long long j = (long long)blockIdx.x * 32 + threadIdx.x;
  const int p0 = final_pass ? 0 : blockIdx.y * kPartsPerBlock;
  const int p1 = final_pass ? nparts : min(nparts, p0 + kPartsPerBlock);
  float s = 0.f;
  if (j < n) {
#pragma unroll 4
    for (int p = p0 + threadIdx.y; p < p1; p += kYLanes) s += part[(long long)p * ld + j];
  }
  sh[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && j < n) {
    float t = 0.f;
#pragma unroll
    for (int y = 0; y < kYLanes; ++y) t += sh[y][threadIdx.x];
    if (!final_pass) {
      out[(long long)blockIdx.y * n + j] = t;
    } else {
      const long long o = scatter_index(sc, j);
      if (o >= 0) out[o] = accumulate ? out[o] + t : t;
    }
  }
}

void col_reduce_impl(const float* part, int nparts, long long n, long long ld, float* out, int accumulate,
                     const Scatter& sc, float* scratch, size_t scratch_floats, cudaStream_t st) {
  const unsigned gx = (unsigned)((n + 31) / 32);
  const dim3 blk(32, kYLanes);
  if (nparts <= 4 * kPartsPerBlock || !scratch) {
    col_reduce_kernel<<<dim3(gx, 1), blk, 0, st>>>(part, nparts, n, ld, out, accumulate, sc, 1);
    return;
  }
  const int G = (nparts + kPartsPerBlock - 1) / kPartsPerBlock;
  if ((size_t)G * n > scratch_floats) {  // not enough scratch: single pass
    col_reduce_kernel<<<dim3(gx, 1), blk, 0, st>>>(part, nparts, n, ld, out, accumulate, sc, 1);
    return;
  }
  col_reduce_kernel<<<dim3(gx, G), blk, 0, st>>>(part, nparts, n, ld, scratch, 0, Scatter{0, 0, 0, 0, 0, 0}, 0);
  col_reduce_kernel<<<dim3(gx, 1), blk, 0, st>>>(scratch, G, n, n, out, accumulate, sc, 1);
}

}  // namespace

void col_reduce(const float* part, int nparts, long long n, float* out, int accumulate, float* scratch,
                size_t scratch_floats, cudaStream_t st) {
  col_reduce_impl(part, nparts, n, n, out, accumulate, Scatter{0, 0, 0, 0, nullptr, nullptr}, scratch,
                  scratch_floats, st);
}

void wgrad_reduce(const float* part, int splits, int rows, int n_total, const int* row_tap, const int* row_oc,
                  int layout, int c_out, int k, float* dw, int accumulate, float* scratch, size_t scratch_floats,
                  cudaStream_t st) {
  const long long n = (long long)rows * n_total;
  col_reduce_impl(part, splits, n, n, dw, accumulate, Scatter{layout == 0 ? 1 : 2, n_total, c_out, k, row_tap, row_oc},
                  scratch, scratch_floats, st);
}

void colsum_reduce(const float* part, int tiles, int C, float* out, int accumulate, float* scratch,
                   size_t scratch_floats, cudaStream_t st) {
  col_reduce(part, tiles, C, out, accumulate, scratch, scratch_floats, st);
}

// ------------------------------------------------------------------------------------------------
// Weight-gradient finish: split-K reduction of part[split][rows][n_total] straight into the
// parameter layout, with the weight-norm backward fused when g != null.  One block per dim-0 row r
// of the parameter (conv: r = oc, elements (ic, tap); convT: r = ic, elements (oc, tap)).
// inv[oc * k + tap] = partial row holding (tap, oc).  Block = 32 columns x 8 split-lanes.
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) wgrad_finish_kernel(const float* __restrict__ part, int splits, int rows,
                                                           int n_total, const int* __restrict__ inv, int layout,
                                                           int c_out, int k, const float* __restrict__ v,
                                                           const float* __restrict__ g,
                                                           const float* __restrict__ norm, float* __restrict__ dv,
                                                           float* __restrict__ dg) {
  extern __shared__ float buf[];  // [per] + 8*33 reduction scratch
  const int r = blockIdx.x;
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int cols = layout == 0 ? n_total : c_out;  // elements per tap in this row
  const int per = cols * k;
  float* red = buf + per;
  for (int tap = 0; tap < k; ++tap) {
    for (int x0 = 0; x0 < cols; x0 += 32) {
      const int x = x0 + tx;
      float s = 0.f;
      if (x < cols) {
        const int row = layout == 0 ? inv[r * k + tap] : inv[x * k + tap];
        const int col = layout == 0 ? x : r;
        for (int sp = ty; sp < splits; sp += 8) s += part[((size_t)sp * rows + row) * n_total + col];
      }
      red[ty * 33 + tx] = s;
      __syncthreads();
      if (ty == 0 && x < cols) {
        float t = 0.f;
#pragma unroll
        for (int y = 0; y < 8; ++y) t += red[y * 33 + tx];
        buf[x * k + tap] = t;
      }
      __syncthreads();
    }
  }
  const int tid = ty * 32 + tx;
  float* out = dv + (size_t)r * per;
  if (!g) {
    for (int e = tid; e < per; e += 256) out[e] = buf[e];
    return;
  }
  // weight norm: dg = <dW, v>/n;  dv = g/n * (dW - dg/n * v)
  const float* vr = v + (size_t)r * per;
  float d = 0.f;
  for (int e = tid; e < per; e += 256) d += buf[e] * vr[e];
  for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
  __syncthreads();
  if (tx == 0) red[ty] = d;
  __syncthreads();
  float dot = 0.f;
#pragma unroll
  for (int y = 0; y < 8; ++y) dot += red[y];
  const float n = norm[r];
  const float dgr = dot / n;
  if (tid == 0) dg[r] = dgr;
  const float a = g[r] / n, b = dgr / n;
  for (int e = tid; e < per; e += 256) out[e] = a * (buf[e] - b * vr[e]);
}

void wgrad_finish(const float* part, int splits, int rows, int n_total, const int* inv, int layout, int c_out, int k,
                  int dim0_rows, const float* v, const float* g, const float* norm, float* dv, float* dg,
                  cudaStream_t st) {
  const int per = (layout == 0 ? n_total : c_out) * k;
  const size_t smem = (size_t)(per + 8 * 33) * sizeof(float);
  wgrad_finish_kernel<<<dim0_rows, dim3(32, 8), smem, st>>>(part, splits, rows, n_total, inv, layout, c_out, k, v, g,
                                                           norm, dv, dg);
}

// Block = 32 lanes x 8 part-lanes; a lane owns 4 consecutive columns (float4 loads of the partials),
// so a block covers 128 columns.  n and ld are multiples of 4 and the partial / scratch buffers
// 16-byte aligned; outputs are written per element (they may sit anywhere in the gradient buffer).
__global__ void __launch_bounds__(256) reduce_batched_kernel(const ReduceDesc* __restrict__ descs, int ndesc) {
  __shared__ float4 sh[kYLanes][32];
  __shared__ int di, last;
  const int tx = threadIdx.x, ty = threadIdx.y;
  if (tx == 0 && ty == 0) {
    int lo = 0, hi = ndesc - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (descs[mid].first_block <= (int)blockIdx.x) lo = mid;
      else hi = mid - 1;
    }
    di = lo;
  }
  __syncthreads();
  const ReduceDesc d = descs[di];
  const int b = blockIdx.x - d.first_block;
  const int cb = b % d.colblocks, ch = b / d.colblocks;
  const long long j = ((long long)cb * 32 + tx) * 4;
  const bool in = j < d.n;
  const int p0 = d.nchunks == 1 ? 0 : ch * kReduceChunk;
  const int p1 = d.nchunks == 1 ? d.nparts : min(d.nparts, p0 + kReduceChunk);
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  if (in) {
#pragma unroll 4
    for (int p = p0 + ty; p < p1; p += kYLanes) {
      const float4 x = __ldcs(reinterpret_cast<const float4*>(d.part + (long long)p * d.ld + j));
      s.x += x.x; s.y += x.y; s.z += x.z; s.w += x.w;
    }
  }
  sh[ty][tx] = s;
  __syncthreads();
  float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
  if (ty == 0) {
#pragma unroll
    for (int y = 0; y < kYLanes; ++y) {
      const float4 x = sh[y][tx];
      t.x += x.x; t.y += x.y; t.z += x.z; t.w += x.w;
    }
  }
  if (d.nchunks == 1) {
    if (ty == 0 && in) {
      d.out[j] = t.x; d.out[j + 1] = t.y; d.out[j + 2] = t.z; d.out[j + 3] = t.w;
    }
    return;
  }
  if (ty == 0 && in) *reinterpret_cast<float4*>(d.scratch + (long long)ch * d.n + j) = t;
  __threadfence();
  __syncthreads();
  if (tx == 0 && ty == 0) last = atomicAdd(&d.counter[cb], 1u) == (unsigned)(d.nchunks - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  // last block of this column group: chunk sums in chunk order
  s = make_float4(0.f, 0.f, 0.f, 0.f);
  if (in)
    for (int c = ty; c < d.nchunks; c += kYLanes) {
      const float4 x = __ldcg(reinterpret_cast<const float4*>(d.scratch + (long long)c * d.n + j));
      s.x += x.x; s.y += x.y; s.z += x.z; s.w += x.w;
    }
  sh[ty][tx] = s;
  __syncthreads();
  if (ty == 0 && in) {
    t = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int y = 0; y < kYLanes; ++y) {
      const float4 x = sh[y][tx];
      t.x += x.x; t.y += x.y; t.z += x.z; t.w += x.w;
    }
    d.out[j] = t.x; d.out[j + 1] = t.y; d.out[j + 2] = t.z; d.out[j + 3] = t.w;
  }
  if (tx == 0 && ty == 0) d.counter[cb] = 0u;
}

int reduce_desc_shape(ReduceDesc& d, int first_block, size_t* scratch_floats, size_t* counters) {
  // the kernel reads the partials as float4: columns and pitch in multiples of 4, 16-byte base
  if (d.n % 4 || d.ld % 4 || reinterpret_cast<uintptr_t>(d.part) % 16) return -1;
  d.first_block = first_block;
  d.colblocks = (int)((d.n + 127) / 128);
  d.nchunks = d.nparts > 2 * kReduceChunk ? (d.nparts + kReduceChunk - 1) / kReduceChunk : 1;
  *scratch_floats = d.nchunks > 1 ? (size_t)d.nchunks * d.n : 0;
  *counters = d.nchunks > 1 ? (size_t)d.colblocks : 0;
  return d.colblocks * d.nchunks;
}

void reduce_batched(const ReduceDesc* descs, int ndesc, int total_blocks, cudaStream_t st) {
  if (ndesc > 0 && total_blocks > 0) reduce_batched_kernel<<<total_blocks, dim3(32, kYLanes), 0, st>>>(descs, ndesc);
}

static float* g_scratch = nullptr;
static size_t g_scratch_n = 0;

void set_reduce_scratch(float* scratch, size_t floats) {
  g_scratch = scratch;
  g_scratch_n = floats;
}

void col_reduce(const float* part, int nparts, long long n, float* out, int accumulate, cudaStream_t st) {
  col_reduce(part, nparts, n, out, accumulate, g_scratch, g_scratch_n, st);
}

void col_reduce_ld(const float* part, int nparts, long long n, long long ld, float* out, int accumulate,
                   cudaStream_t st) {
  col_reduce_impl(part, nparts, n, ld, out, accumulate, Scatter{0, 0, 0, 0, nullptr, nullptr}, g_scratch, g_scratch_n,
                  st);
}

void colsum_reduce(const float* part, int tiles, int C, float* out, int accumulate, cudaStream_t st) {
  col_reduce(part, tiles, C, out, accumulate, g_scratch, g_scratch_n, st);
}

void wgrad_reduce(const float* part, int splits, int rows, int n_total, const int* row_tap, const int* row_oc,
                  int layout, int c_out, int k, float* dw, int accumulate, cudaStream_t st) {
  wgrad_reduce(part, splits, rows, n_total, row_tap, row_oc, layout, c_out, k, dw, accumulate, g_scratch, g_scratch_n,
               st);
}

}  // namespace wb
