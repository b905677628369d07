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
// =============================================================================================
__global__ void noise_add_act_kernel(NoiseActArgs a) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long n = (long long)a.B * a.T * a.C;
  if (i >= n) return;
  const int c = (int)(i % a.C);
  const long long row = i / a.C;
  const int b = (int)(row / a.T), j = (int)(row % a.T);
  float x = a.x[i];
  if (a.har) {
    float s = a.bias[c];
    const float* h = a.har + (size_t)b * a.T_full;
    const int t0 = j * a.stride - a.pad;
    for (int tap = 0; tap < a.k; ++tap) {
      const int t = t0 + tap;
      if (t >= 0 && t < a.T_full) s += a.w[(size_t)tap * a.C + c] * h[t];
    }
    x += s;
    a.x[i] = x;
  }
  if (a.pre) a.pre[i] = __float2bfloat16_rn(x);
  for (int q = 0; q < a.n_act; ++q) {
    const float al = a.alpha[q] ? a.alpha[q][c] : 1.f;
    const float y = act_fwd2(x, a.act_kind, a.slope, al);
    bf16 hi, lo;
    split_bf16(y, hi, lo);
    a.act_hi[q][i] = hi;
    a.act_lo[q][i] = lo;
  }
}

void noise_add_act(const NoiseActArgs& a, cudaStream_t st) {
  const long long n = (long long)a.B * a.T * a.C;
  noise_add_act_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(a);
}

__global__ void noise_dhar_kernel(const float* __restrict__ dx, const float* __restrict__ wt, int B, int T, int C, int k,
                                  int stride, int pad, int T_full, float* __restrict__ d_har, int accumulate) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)B * T_full) return;
  const int b = (int)(i / T_full), t = (int)(i % T_full);
  // rows j with 0 <= t + pad - j*stride < k
  int jhi = (t + pad) / stride;
  int jlo = t + pad - k + 1;
  jlo = jlo <= 0 ? 0 : (jlo + stride - 1) / stride;
  if (jhi > T - 1) jhi = T - 1;
  float s = 0.f;
  for (int j = jlo; j <= jhi; ++j) {
    const int tap = t + pad - j * stride;
    const float4* r = reinterpret_cast<const float4*>(dx + ((size_t)b * T + j) * C);
    const float4* w = reinterpret_cast<const float4*>(wt + (size_t)tap * C);
    for (int c4 = 0; c4 < C / 4; ++c4) {
      const float4 x = r[c4], y = w[c4];
      s += x.x * y.x + x.y * y.y + x.z * y.z + x.w * y.w;
    }
  }
  d_har[i] = accumulate ? d_har[i] + s : s;
}

constexpr int kNoiseTaps = 16;

int noise_rows_per_part(int k) { return k <= kNoiseTaps ? 512 : 64; }

int noise_backward_parts(int B, int T, int k) {
  const int r = noise_rows_per_part(k);
  return (int)(((long long)B * T + r - 1) / r);
}

// dW partials part[chunk][c][tap].  Block = 32 channels (lanes) x 8 warps.
//   k <= 16: the warps split the chunk's rows, every thread keeps all k taps, smem reduce at the end.
//   k > 16 : the warps split the taps (tap = warp + 8q), every thread walks all rows of the chunk.
__global__ void __launch_bounds__(256) noise_wgrad_kernel(const float* __restrict__ dx, const float* __restrict__ har,
                                                          int B, int T, int C, int k, int stride, int pad, int T_full,
                                                          int rows_per_part, float* __restrict__ part) {
  __shared__ float red[8][kNoiseTaps][33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  const long long r0 = (long long)blockIdx.y * rows_per_part;
  const long long r1 = min((long long)B * T, r0 + rows_per_part);
  float acc[kNoiseTaps];
#pragma unroll
  for (int q = 0; q < kNoiseTaps; ++q) acc[q] = 0.f;
  float* o = part + (size_t)blockIdx.y * C * k + (size_t)c * k;
  if (k <= kNoiseTaps) {
    for (long long r = r0 + w; r < r1; r += 8) {
      const int b = (int)(r / T), j = (int)(r % T);
      const float x = dx[r * C + c];
      const int t0 = j * stride - pad;
      const float* h = har + (size_t)b * T_full;
#pragma unroll
      for (int q = 0; q < kNoiseTaps; ++q)
        if (q < k && t0 + q >= 0 && t0 + q < T_full) acc[q] += x * h[t0 + q];
    }
#pragma unroll
    for (int q = 0; q < kNoiseTaps; ++q) red[w][q][lane] = acc[q];
    __syncthreads();
    for (int q = w; q < k; q += 8) {
      float s = 0.f;
#pragma unroll
      for (int y = 0; y < 8; ++y) s += red[y][q][lane];
      o[q] = s;
    }
  } else {
    for (long long r = r0; r < r1; ++r) {
      const int b = (int)(r / T), j = (int)(r % T);
      const float x = dx[r * C + c];
      const int t0 = j * stride - pad;
      const float* h = har + (size_t)b * T_full;
#pragma unroll
      for (int q = 0; q < kNoiseTaps; ++q) {
        const int tap = w + 8 * q;
        if (tap < k && t0 + tap >= 0 && t0 + tap < T_full) acc[q] += x * h[t0 + tap];
      }
    }
#pragma unroll
    for (int q = 0; q < kNoiseTaps; ++q) {
      const int tap = w + 8 * q;
      if (tap < k) o[tap] = acc[q];
    }
  }
}

void noise_backward(const float* dx, const float* har, const float* wt, int B, int T, int C, int k, int stride, int pad,
                    int T_full, float* d_har, int accumulate_dhar, float* wpart, cudaStream_t st) {
  const long long n = (long long)B * T_full;
  noise_dhar_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(dx, wt, B, T, C, k, stride, pad, T_full, d_har,
                                                                  accumulate_dhar);
  const int parts = noise_backward_parts(B, T, k);
  noise_wgrad_kernel<<<dim3(C / 32, parts), 256, 0, st>>>(dx, har, B, T, C, k, stride, pad, T_full,
                                                          noise_rows_per_part(k), wpart);
}

void noise_wgrad_reduce(const float* wpart, int nparts, int C, int k, float* dW, cudaStream_t st) {
  col_reduce(wpart, nparts, (long long)C * k, dW, 0, st);
}

// =============================================================================================
// conv_post (32 -> 1, 7 taps, pad 3) + tanh.  Warp per output row, lane per channel.
// =============================================================================================
constexpr int kPostK = 7;
constexpr int kPostC = 32;

__global__ void __launch_bounds__(256) post_forward_kernel(const bf16* __restrict__ hi, const bf16* __restrict__ lo,
                                                           const float* __restrict__ W, int B, int T,
                                                           float* __restrict__ audio) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * 8;
  float w[kPostK];
#pragma unroll
  for (int q = 0; q < kPostK; ++q) w[q] = W[lane * kPostK + q];
  for (long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5); row < (long long)B * T; row += warps) {
    const int t = (int)(row % T);
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < kPostK; ++q) {
      const int r = t - kPostK / 2 + q;
      if (r >= 0 && r < T) {
        const size_t off = (size_t)(row - t + r) * kPostC + lane;
        s += (__bfloat162float(hi[off]) + __bfloat162float(lo[off])) * w[q];
      }
    }
    s = warp_sum(s);
    if (lane == 0) audio[row] = tanhf(s);
  }
}

void post_forward(const bf16* a_hi, const bf16* a_lo, const float* W, int B, int T, int C, int k, float* audio,
                  cudaStream_t st) {
  (void)C;
  (void)k;  // 32 x 7 (checked at setup)
  post_forward_kernel<<<148 * 8, 256, 0, st>>>(a_hi, a_lo, W, B, T, audio);
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
  for (int rr = warp; rr < kPostRows; rr += 8) {
    const long long row = (long long)blockIdx.x * kPostRows + rr;
    if (row >= nrows) break;
    const int t = (int)(row % a.T);
    const long long rb = row - t;  // first row of this item
    float dpre[kPostK];
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
    float da = 0.f;
#pragma unroll
    for (int q = 0; q < kPostK; ++q) da += dpre[q] * w[q];
    const size_t off = (size_t)row * kPostC + c;
    const float xin = __bfloat162float(a.a_hi[off]) + __bfloat162float(a.a_lo[off]);
#pragma unroll
    for (int q = 0; q < kPostK; ++q) dw[q] += xin * dpre[q];
    const float x = __bfloat162float(a.mask_src[off]);
    float deriv;
    if (a.act_kind == 1) {
      const float al = a.alpha[c];
      float sn, csn;
      sincosf(al * x, &sn, &csn);
      const float s2 = 2.f * sn * csn;
      as += da * (x * s2 / al - sn * sn / (al * al));
      deriv = 1.f + s2;
    } else {
      deriv = x > 0.f ? 1.f : a.slope;
    }
    const float ds = da * deriv * a.scale;
    a.d_stage[off] = ds;
    a.d_stage_bf[off] = __float2bfloat16_rn(ds);
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
