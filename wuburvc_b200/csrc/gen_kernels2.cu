// gen_kernels2.cu — noise convs and conv_post of the generator step (bandwidth-bound kernels).
#include "gen_kernels.cuh"
#include "small_kernels.cuh"

namespace wb {

namespace {
__device__ __forceinline__ float act_fwd2(float x, int kind, float slope, float alpha) {
  return kind == 1 ? snake(x, alpha) : lrelu(x, slope);
}
__device__ __forceinline__ float warp_sum(float v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// Warp transpose-reduction: on return lane l holds the sum over lanes of input v[l].
__device__ __forceinline__ float warp_transpose_sum32(float* v, int lane) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      const float send = upper ? v[i] : v[i + off];
      const float keep = upper ? v[i + off] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  return v[0];
}
}  // namespace

// w [C][k] -> wt [k][C]
__global__ void transpose_ck_kernel(const float* __restrict__ w, int C, int k, float* __restrict__ wt) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= C * k) return;
  const int tap = i / C, c = i % C;
  wt[i] = w[(size_t)c * k + tap];
}

void transpose_ck(const float* w, int C, int k, float* wt, cudaStream_t st) {
  transpose_ck_kernel<<<(C * k + 255) / 256, 256, 0, st>>>(w, C, k, wt);
}

// =============================================================================================
// noise conv (+ activation of the stage input); weights transposed wt[tap][C]
//   x[b][j][c] += bias[c] + sum_tap wt[tap][c] * har[b][j*stride - pad + tap]
// Block = 32 channels (lanes) x 64 rows of one item (8 warps x 8 rows); the weights of the 32
// channels and the har window of the 64 rows sit in shared memory.
// =============================================================================================
constexpr int kNaRowsPerWarp = 8;
constexpr int kNaRows = 8 * kNaRowsPerWarp;

__global__ void __launch_bounds__(256) noise_add_act_kernel(NoiseActArgs a) {
  extern __shared__ float sh[];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int c = blockIdx.y * 32 + lane;
  const int b = blockIdx.z;
  const int j0 = blockIdx.x * kNaRows;
  float* ws = sh;                 // [k][32]
  float* hs = sh + a.k * 32;      // har window, (kNaRows - 1) * stride + k samples from j0 * stride - pad
  if (a.har) {
    const int hw = (kNaRows - 1) * a.stride + a.k, h0 = j0 * a.stride - a.pad;
    for (int i = threadIdx.x; i < a.k * 32; i += blockDim.x)
      ws[i] = a.w[(size_t)(i >> 5) * a.C + blockIdx.y * 32 + (i & 31)];
    for (int i = threadIdx.x; i < hw; i += blockDim.x) {
      const int t = h0 + i;
      hs[i] = (t >= 0 && t < a.T_full) ? a.har[(size_t)b * a.T_full + t] : 0.f;
    }
  }
  __syncthreads();
  const int jw = j0 + w * kNaRowsPerWarp;  // this warp's first row
  const int nr = max(0, min(kNaRowsPerWarp, a.T - jw));
  float x[kNaRowsPerWarp];
#pragma unroll
  for (int r = 0; r < kNaRowsPerWarp; ++r) x[r] = r < nr ? a.x[((size_t)b * a.T + jw + r) * a.C + c] : 0.f;
  if (a.har) {
    float acc[kNaRowsPerWarp];
    const float bc = a.bias[c];
#pragma unroll
    for (int r = 0; r < kNaRowsPerWarp; ++r) acc[r] = bc;
    const float* hw0 = hs + (w * kNaRowsPerWarp) * a.stride;
    for (int tap = 0; tap < a.k; ++tap) {
      const float wv = ws[tap * 32 + lane];
#pragma unroll
      for (int r = 0; r < kNaRowsPerWarp; ++r) acc[r] += wv * hw0[r * a.stride + tap];
    }
#pragma unroll
    for (int r = 0; r < kNaRowsPerWarp; ++r) {
      x[r] += acc[r];
      if (r < nr) a.x[((size_t)b * a.T + jw + r) * a.C + c] = x[r];
    }
  }
  float al[3];
#pragma unroll
  for (int q = 0; q < 3; ++q) al[q] = (q < a.n_act && a.alpha[q]) ? a.alpha[q][c] : 1.f;
#pragma unroll
  for (int r = 0; r < kNaRowsPerWarp; ++r) {
    if (r >= nr) break;
    const size_t i = ((size_t)b * a.T + jw + r) * a.C + c;
    if (a.pre) {
      const bf16 h = __float2bfloat16_rn(x[r]);
      a.pre[i] = h;
      if (a.pre_lo) a.pre_lo[i] = __float2bfloat16_rn(x[r] - __bfloat162float(h));
    }
    for (int q = 0; q < a.n_act; ++q) {
      const float y = act_fwd2(x[r], a.act_kind, a.slope, al[q]);
      f16 hi, lo;
      split_op(y, a.fmt_bf16, hi, lo);
      a.act_hi[q][i] = hi;
      a.act_lo[q][i] = lo;
      const bf16 yb = __float2bfloat16_rn(y);
      if (a.act_bf[q]) a.act_bf[q][i] = yb;
      if (a.act_bflo[q]) a.act_bflo[q][i] = __float2bfloat16_rn(y - __bfloat162float(yb));
      if (!a.fmt_bf16 && !(fabsf(y) < kF16Max) && a.range_err) atomicCAS(a.range_err, 0, ERR_RANGE);
    }
  }
}

void noise_add_act(const NoiseActArgs& a, cudaStream_t st) {
  const dim3 grid((unsigned)((a.T + kNaRows - 1) / kNaRows), (unsigned)(a.C / 32), (unsigned)a.B);
  const size_t smem = a.har ? sizeof(float) * ((size_t)a.k * 32 + (size_t)(kNaRows - 1) * a.stride + a.k) : 0;
  noise_add_act_kernel<<<grid, 256, smem, st>>>(a);
}

size_t noise_act_smem(int k, int stride) {
  return sizeof(float) * ((size_t)k * 32 + (size_t)(kNaRows - 1) * stride + k);
}

// ---- noise-conv backward ------------------------------------------------------------------------
// Phase 1: g[row][tap] = sum_c dx[row][c] * wt[tap][c] (warp per (row, group of 16 taps), lanes over
// channels, transpose-reduction across lanes).  Phase 2: d_har[b][t] (+)= overlap-add of g over the
// rows j whose window covers t (tap = t + pad - j*stride).
__device__ __forceinline__ float warp_colsum16(float* v, int lane) {
  // v[0..15] per lane; on return lane q < 16 holds sum over lanes of v[q]
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const bool upper = (lane & off) != 0;
    const int n = off < 16 ? off : 16;
#pragma unroll
    for (int i = 0; i < n; ++i) {
      if (off == 16) {
        v[i] += __shfl_xor_sync(0xffffffffu, v[i], 16);
      } else {
        const float send = upper ? v[i] : v[i + off];
        const float keep = upper ? v[i + off] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
      }
    }
  }
  return v[0];
}

__global__ void __launch_bounds__(256) noise_g_kernel(const float* __restrict__ dx, const float* __restrict__ wt,
                                                      long long rows, int C, int k, float* __restrict__ g) {
  const int lane = threadIdx.x & 31;
  const int ngroups = (k + 15) / 16;
  const long long wid = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const long long row = wid / ngroups;
  const int grp = (int)(wid - row * ngroups);
  if (row >= rows) return;
  float v[16];
#pragma unroll
  for (int q = 0; q < 16; ++q) v[q] = 0.f;
  const float* xr = dx + (size_t)row * C;
  for (int c = lane; c < C; c += 32) {
    const float x = xr[c];
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      const int tap = grp * 16 + q;
      if (tap < k) v[q] += x * wt[(size_t)tap * C + c];
    }
  }
  const float sum = warp_colsum16(v, lane);
  const int tap = grp * 16 + lane;
  if (lane < 16 && tap < k) g[(size_t)row * k + tap] = sum;
}

__global__ void noise_dhar_kernel(const float* __restrict__ g, int B, int T, int k, int stride, int pad, int T_full,
                                  float* __restrict__ d_har, int accumulate) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)B * T_full) return;
  const int b = (int)(i / T_full), t = (int)(i % T_full);
  // rows j with 0 <= t + pad - j*stride < k
  int jhi = (t + pad) / stride;
  int jlo = t + pad - k + 1;
  jlo = jlo <= 0 ? 0 : (jlo + stride - 1) / stride;
  if (jhi > T - 1) jhi = T - 1;
  float s = 0.f;
  for (int j = jlo; j <= jhi; ++j) s += g[((size_t)b * T + j) * k + (t + pad - j * stride)];
  d_har[i] = accumulate ? d_har[i] + s : s;
}

// dW partials part[b * row_blocks + rb][c][tap] = sum over the block's rows of dx[row][c] * har[...]
// Block = 32 channels (lanes) x kNwRows rows of one item; har window in shared memory.
//   k <= 16: the warps split the rows, every thread keeps all k taps, shared-memory reduce at the end.
//   k > 16 : the warps split the taps (tap = warp + 8q), every thread walks all rows of the block.
constexpr int kNoiseTaps = 16;
constexpr int kNwRows = 128;

int noise_backward_parts_rows(int B, int T) { return B * ((T + kNwRows - 1) / kNwRows); }

__global__ void __launch_bounds__(256) noise_wgrad_kernel(const float* __restrict__ dx, const float* __restrict__ har,
                                                          int B, int T, int C, int k, int stride, int pad, int T_full,
                                                          float* __restrict__ part) {
  extern __shared__ float hs[];  // har window: (kNwRows - 1) * stride + k samples from j0 * stride - pad
  __shared__ float red[8][kNoiseTaps][33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  const int nrb = (T + kNwRows - 1) / kNwRows;
  const int b = blockIdx.y / nrb, rb = blockIdx.y % nrb;
  const int j0 = rb * kNwRows, nrows = min(kNwRows, T - j0);
  const int hw = (kNwRows - 1) * stride + k, h0 = j0 * stride - pad;
  for (int i = threadIdx.x; i < hw; i += blockDim.x) {
    const int t = h0 + i;
    hs[i] = (t >= 0 && t < T_full) ? har[(size_t)b * T_full + t] : 0.f;
  }
  __syncthreads();
  float acc[kNoiseTaps];
#pragma unroll
  for (int q = 0; q < kNoiseTaps; ++q) acc[q] = 0.f;
  const float* xb = dx + ((size_t)b * T + j0) * C + c;
  float* o = part + (size_t)blockIdx.y * C * k + (size_t)c * k;
  if (k <= kNoiseTaps) {
#pragma unroll 4
    for (int jl = w; jl < nrows; jl += 8) {
      const float x = xb[(size_t)jl * C];
      const float* h = hs + jl * stride;
#pragma unroll
      for (int q = 0; q < kNoiseTaps; ++q)
        if (q < k) acc[q] += x * h[q];
    }
#pragma unroll
    for (int q = 0; q < kNoiseTaps; ++q) red[w][q][lane] = acc[q];
    __syncthreads();
    for (int q = w; q < k; q += 8) {
      float sum = 0.f;
#pragma unroll
      for (int y = 0; y < 8; ++y) sum += red[y][q][lane];
      o[q] = sum;
    }
  } else {
#pragma unroll 4
    for (int jl = 0; jl < nrows; ++jl) {
      const float x = xb[(size_t)jl * C];
      const float* h = hs + jl * stride + w;
#pragma unroll
      for (int q = 0; q < kNoiseTaps; ++q)
        if (w + 8 * q < k) acc[q] += x * h[8 * q];
    }
#pragma unroll
    for (int q = 0; q < kNoiseTaps; ++q) {
      const int tap = w + 8 * q;
      if (tap < k) o[tap] = acc[q];
    }
  }
}

// Phase 1 for few taps (k <= 8): thread per row, float4 walk over the row's channels.
__global__ void __launch_bounds__(256) noise_g_small_kernel(const float* __restrict__ dx, const float* __restrict__ wt,
                                                            long long rows, int C, int k, float* __restrict__ g) {
  const long long row = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  float acc[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) acc[q] = 0.f;
  const float4* x4 = reinterpret_cast<const float4*>(dx + (size_t)row * C);
  const float4* w4 = reinterpret_cast<const float4*>(wt);
  const int c4n = C / 4;
  for (int c4 = 0; c4 < c4n; ++c4) {
    const float4 x = x4[c4];
#pragma unroll
    for (int q = 0; q < 8; ++q)
      if (q < k) {
        const float4 w = w4[(size_t)q * c4n + c4];
        acc[q] += x.x * w.x + x.y * w.y + x.z * w.z + x.w * w.w;
      }
  }
#pragma unroll
  for (int q = 0; q < 8; ++q)
    if (q < k) g[(size_t)row * k + q] = acc[q];
}

// ---- fused noise-conv backward: one pass over dx gives both g and the weight-gradient partials ----
// Block = 8 warps x `rpw` consecutive rows (rows = B*T, items back to back) x one group of TP taps
// (blockIdx.y).  Lane l holds channels [l*CPL, l*CPL + CPL) of every row it reads (C = 32*CPL).
// A pass covers RP = 32/TP rows: v[r*TP + t] = sum over the lane's channels of dx[r][c] * wt[t][c],
// and one transpose-reduction leaves lane l with g of (row l/TP, tap l%TP).  The same dx registers
// feed the weight gradient acc[c][t] += dx[r][c] * har[b][j*stride - pad + tap] (lane l loads the
// har sample of (l/TP, l%TP), shuffles broadcast it).  The warps' accumulators are summed in shared
// memory in a fixed order into part[blockIdx.x][c][tap].
template <int CPL, int TP>
__global__ void __launch_bounds__(256) noise_bwd_fused_kernel(const float* __restrict__ dx,
                                                              const float* __restrict__ wt,
                                                              const float* __restrict__ har, int rows, int T, int k,
                                                              int stride, int pad, int T_full, int rpw,
                                                              float* __restrict__ g, float* __restrict__ part) {
  constexpr int C = 32 * CPL, RP = 32 / TP;
  __shared__ __align__(16) float ws[TP][C];
  __shared__ float red[8][32][TP + 1];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tap0 = blockIdx.y * TP;
  for (int i = threadIdx.x; i < TP * C; i += blockDim.x) {
    const int t = i / C, c = i % C;
    ws[t][c] = (tap0 + t < k) ? wt[(size_t)(tap0 + t) * C + c] : 0.f;
  }
  __syncthreads();
  float acc[CPL][TP];
#pragma unroll
  for (int c = 0; c < CPL; ++c)
#pragma unroll
    for (int t = 0; t < TP; ++t) acc[c][t] = 0.f;
  const int my_r = lane / TP, my_t = lane % TP;
  const int row_w = (blockIdx.x * 8 + warp) * rpw;
  for (int r0 = row_w; r0 < row_w + rpw && r0 < rows; r0 += RP) {
    float x[RP][CPL];
#pragma unroll
    for (int r = 0; r < RP; ++r) {
      const int row = r0 + r;
      if (row < rows) {
        const float* src = dx + (size_t)row * C + lane * CPL;
        if constexpr (CPL % 4 == 0) {
#pragma unroll
          for (int q = 0; q < CPL / 4; ++q) {
            const float4 f = __ldcs(reinterpret_cast<const float4*>(src) + q);
            x[r][4 * q] = f.x; x[r][4 * q + 1] = f.y; x[r][4 * q + 2] = f.z; x[r][4 * q + 3] = f.w;
          }
        } else if constexpr (CPL == 2) {
          const float2 f = __ldcs(reinterpret_cast<const float2*>(src));
          x[r][0] = f.x; x[r][1] = f.y;
        } else {
          x[r][0] = __ldcs(src);
        }
      } else {
#pragma unroll
        for (int c = 0; c < CPL; ++c) x[r][c] = 0.f;
      }
    }
    // this lane's har sample: row r0 + my_r, tap tap0 + my_t
    float h = 0.f;
    {
      const int row = r0 + my_r, tap = tap0 + my_t;
      if (row < rows && tap < k) {
        const int b = row / T, j = row - b * T;
        const int idx = j * stride - pad + tap;
        if (idx >= 0 && idx < T_full) h = __ldg(har + (size_t)b * T_full + idx);
      }
    }
    float v[32];
#pragma unroll
    for (int r = 0; r < RP; ++r)
#pragma unroll
      for (int t = 0; t < TP; ++t) {
        float sum = 0.f;
#pragma unroll
        for (int c = 0; c < CPL; ++c) sum += x[r][c] * ws[t][lane * CPL + c];
        v[r * TP + t] = sum;
        const float hv = __shfl_sync(0xffffffffu, h, r * TP + t);
#pragma unroll
        for (int c = 0; c < CPL; ++c) acc[c][t] += x[r][c] * hv;
      }
    const float gs = warp_transpose_sum32(v, lane);
    {
      const int row = r0 + my_r, tap = tap0 + my_t;
      if (row < rows && tap < k) g[(size_t)row * k + tap] = gs;
    }
  }
  // fixed-order block reduction of the weight gradient, one channel of every lane at a time
#pragma unroll
  for (int c = 0; c < CPL; ++c) {
#pragma unroll
    for (int t = 0; t < TP; ++t) red[warp][lane][t] = acc[c][t];
    __syncthreads();
    if (threadIdx.x < 32 * TP) {
      const int l = threadIdx.x / TP, t = threadIdx.x % TP;
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) sum += red[w][l][t];
      if (tap0 + t < k) part[((size_t)blockIdx.x * C + l * CPL + c) * k + tap0 + t] = sum;
    }
    __syncthreads();
  }
}

namespace {
// taps per pass of the fused kernel (a power of two <= 8, <= k), channels per lane (0 = not covered)
int noise_tp(int k) { return k >= 8 ? 8 : k >= 4 ? 4 : k >= 2 ? 2 : 1; }
int noise_cpl(int C) { return (C == 32 || C == 64 || C == 128 || C == 256) ? C / 32 : 0; }
// rows per warp: about 512 blocks over (row blocks x tap groups), a multiple of the pass height
int noise_rpw(long long rows, int k) {
  const int tp = noise_tp(k), rp = 32 / tp, ntg = (k + tp - 1) / tp;
  const long long per = (rows * ntg + 8LL * 512 * rp - 1) / (8LL * 512 * rp);
  return rp * (int)std::max(1LL, per);
}
}  // namespace

int noise_backward_parts(int B, int T, int C, int k) {
  if (noise_cpl(C)) {
    const long long rows = (long long)B * T;
    return (int)((rows + 8LL * noise_rpw(rows, k) - 1) / (8LL * noise_rpw(rows, k)));
  }
  return noise_backward_parts_rows(B, T);
}

void noise_backward(const float* dx, const float* har, const float* wt, int B, int T, int C, int k, int stride, int pad,
                    int T_full, float* d_har, int accumulate_dhar, float* wpart, float* g, cudaStream_t st) {
  const long long rows = (long long)B * T;
  const int cpl = noise_cpl(C);
  if (cpl) {
    const int tp = noise_tp(k), rpw = noise_rpw(rows, k);
    const dim3 grid((unsigned)noise_backward_parts(B, T, C, k), (unsigned)((k + tp - 1) / tp));
#define WB_NB(cpl_, tp_)                                                                             \
  if (cpl == cpl_ && tp == tp_)                                                                      \
    noise_bwd_fused_kernel<cpl_, tp_><<<grid, 256, 0, st>>>(dx, wt, har, (int)rows, T, k, stride, pad, T_full, rpw, g, \
                                                            wpart);
    WB_NB(1, 1) WB_NB(1, 2) WB_NB(1, 4) WB_NB(1, 8) WB_NB(2, 1) WB_NB(2, 2) WB_NB(2, 4) WB_NB(2, 8)
    WB_NB(4, 1) WB_NB(4, 2) WB_NB(4, 4) WB_NB(4, 8) WB_NB(8, 1) WB_NB(8, 2) WB_NB(8, 4) WB_NB(8, 8)
#undef WB_NB
  } else {
    if (k <= 8) {
      noise_g_small_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, st>>>(dx, wt, rows, C, k, g);
    } else {
      const long long warps = rows * ((k + 15) / 16);
      noise_g_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(dx, wt, rows, C, k, g);
    }
    const size_t smem = sizeof(float) * ((size_t)(kNwRows - 1) * stride + k);
    noise_wgrad_kernel<<<dim3(C / 32, noise_backward_parts_rows(B, T)), 256, smem, st>>>(dx, har, B, T, C, k, stride,
                                                                                         pad, T_full, wpart);
  }
  const long long n = (long long)B * T_full;
  noise_dhar_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(g, B, T, k, stride, pad, T_full, d_har,
                                                                  accumulate_dhar);
}

void noise_wgrad_reduce(const float* wpart, int nparts, int C, int k, float* dW, float* scratch, size_t scratch_floats,
                        cudaStream_t st) {
  col_reduce(wpart, nparts, (long long)C * k, dW, 0, scratch, scratch_floats, st);
}

// =============================================================================================
// conv_post (32 -> 1, 7 taps, pad 3) + tanh.  Warp per output row, lane per channel.
// =============================================================================================
constexpr int kPostK = 7;
constexpr int kPostC = 32;

// Warp = 32 consecutive output rows of one item, lane = channel: the 38-row input window is read
// once (coalesced), each lane forms its channel's 32 partial sums, and one transpose-reduction
// gives lane r the output of row r.
constexpr int kPostWarpRows = 32;


__global__ void __launch_bounds__(256) post_forward_kernel(const f16* __restrict__ hi, const f16* __restrict__ lo,
                                                           int fmt_bf16, const float* __restrict__ W, int B, int T,
                                                           float* __restrict__ audio) {
  const int lane = threadIdx.x & 31;
  constexpr int pad = kPostK / 2, win = kPostWarpRows + kPostK - 1;
  float w[kPostK];
#pragma unroll
  for (int q = 0; q < kPostK; ++q) w[q] = W[lane * kPostK + q];
  const int wpi = (T + kPostWarpRows - 1) / kPostWarpRows;  // warps per item
  const long long nw = (long long)B * wpi;
  for (long long gw = (long long)blockIdx.x * 8 + (threadIdx.x >> 5); gw < nw; gw += (long long)gridDim.x * 8) {
    const int b = (int)(gw / wpi), t0 = (int)(gw % wpi) * kPostWarpRows;
    const size_t base = (size_t)b * T;
    float x[win];
#pragma unroll
    for (int i = 0; i < win; ++i) {
      const int r = t0 - pad + i;
      x[i] = 0.f;
      if (r >= 0 && r < T) {
        const size_t off = (base + r) * kPostC + lane;
        x[i] = lo ? join_op(hi[off], lo[off], fmt_bf16) : __half2float(hi[off]);  // no lo: fast inference
      }
    }
    float v[32];
#pragma unroll
    for (int r = 0; r < 32; ++r) {
      float acc = 0.f;
      if (r < kPostWarpRows) {
#pragma unroll
        for (int q = 0; q < kPostK; ++q) acc += x[r + q] * w[q];
      }
      v[r] = acc;
    }
    const float s = warp_transpose_sum32(v, lane);  // lane r: row t0 + r
    if (lane < kPostWarpRows && t0 + lane < T) audio[base + t0 + lane] = tanhf(s);
  }
}

void post_forward(const f16* a_hi, const f16* a_lo, int fmt_bf16, const float* W, int B, int T, int C, int k,
                  float* audio, cudaStream_t st) {
  (void)C;
  (void)k;  // 32 x 7 (checked at setup)
  post_forward_kernel<<<148 * 8, 256, 0, st>>>(a_hi, a_lo, fmt_bf16, W, B, T, audio);
}

constexpr int kPostRows = 64;

int post_backward_blocks(int B, int T) { return (int)(((long long)B * T + kPostRows - 1) / kPostRows); }

__global__ void __launch_bounds__(256) post_backward_kernel(PostBwdArgs a) {
  // lane = channel (C == 32), 8 warps x 8 rows each
  __shared__ float red[8][kPostC * (kPostK + 2)];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = lane;
  constexpr int pad = kPostK / 2;
  const long long nrows = (long long)a.B * a.T;
  float w[kPostK];
#pragma unroll
  for (int q = 0; q < kPostK; ++q) w[q] = a.W[c * kPostK + q];
  float cs = 0.f, as = 0.f, dw[kPostK];
#pragma unroll
  for (int q = 0; q < kPostK; ++q) dw[q] = 0.f;
  // warp = 8 consecutive rows; the 14 values dy * (1 - y^2) they need are formed once (one per lane)
  // and broadcast by shuffles when the rows share an item
  const long long wrow0 = (long long)blockIdx.x * kPostRows + warp * 8;
  const int t0w = (int)(wrow0 % a.T);
  const bool same_item = t0w + 7 < a.T && wrow0 + 7 < nrows;
  float dval = 0.f;
  if (same_item && lane < 8 + kPostK - 1) {
    const int tt = t0w - pad + lane;
    if (tt >= 0 && tt < a.T) {
      const long long rb = wrow0 - t0w;
      const float y = a.audio[rb + tt];
      dval = a.dy[rb + tt] * (1.f - y * y);
    }
  }
  float xin8[8], xm8[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const long long row = wrow0 + r;
    xin8[r] = xm8[r] = 0.f;
    if (row < nrows) {
      const size_t off = (size_t)row * kPostC + c;
      xin8[r] = join_op(a.a_hi[off], a.a_lo[off], a.fmt_bf16);
      xm8[r] = __bfloat162float(a.mask_src[off]);
      if (a.mask_lo) xm8[r] += __bfloat162float(a.mask_lo[off]);
    }
  }
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const long long row = wrow0 + r;
    if (row >= nrows) break;
    float dpre[kPostK];
    if (same_item) {
#pragma unroll
      for (int q = 0; q < kPostK; ++q) dpre[q] = __shfl_sync(0xffffffffu, dval, r + 2 * pad - q);
    } else {
      const int t = (int)(row % a.T);
      const long long rb = row - t;
#pragma unroll
      for (int q = 0; q < kPostK; ++q) {
        const int tt = t + pad - q;  // output sample fed by input row t through tap q
        float d = 0.f;
        if (tt >= 0 && tt < a.T) {
          const float y = a.audio[rb + tt];
          d = a.dy[rb + tt] * (1.f - y * y);
        }
        dpre[q] = d;
      }
    }
    float da = 0.f;
#pragma unroll
    for (int q = 0; q < kPostK; ++q) da += dpre[q] * w[q];
    const size_t off = (size_t)row * kPostC + c;
    const float xin = xin8[r];
#pragma unroll
    for (int q = 0; q < kPostK; ++q) dw[q] += xin * dpre[q];
    const float x = xm8[r];
    float deriv;
    if (a.act_kind == 1) {
      float dal;
      snake_grads(x, a.alpha[c], deriv, dal);
      as += da * dal;
    } else {
      deriv = x > 0.f ? 1.f : a.slope;
    }
    const float ds = da * deriv * a.scale;
    a.d_stage[off] = ds;
    const bf16 dsb = __float2bfloat16_rn(ds);
    a.d_stage_bf[off] = dsb;
    if (a.d_stage_bf_lo) a.d_stage_bf_lo[off] = __float2bfloat16_rn(ds - __bfloat162float(dsb));
    cs += ds;
  }
  red[warp][c] = cs;
  red[warp][32 + c] = as;
#pragma unroll
  for (int q = 0; q < kPostK; ++q) red[warp][64 + q * 32 + c] = dw[q];
  __syncthreads();
  constexpr int nval = 64 + kPostK * 32;
  for (int o = threadIdx.x; o < nval; o += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int y = 0; y < 8; ++y) s += red[y][o];
    if (o < 32) a.colsum_part[(size_t)blockIdx.x * kPostC + o] = s;
    else if (o < 64) {
      if (a.alpha_part) a.alpha_part[(size_t)blockIdx.x * kPostC + (o - 32)] = s;
    } else {
      const int q = (o - 64) / 32, cc = (o - 64) % 32;
      a.w_part[(size_t)blockIdx.x * (kPostC * kPostK) + (size_t)cc * kPostK + q] = s;
    }
  }
}

void post_backward(const PostBwdArgs& a, cudaStream_t st) {
  post_backward_kernel<<<post_backward_blocks(a.B, a.T), 256, 0, st>>>(a);
}

}  // namespace wb
