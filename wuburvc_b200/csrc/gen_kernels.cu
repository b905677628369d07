// gen_kernels.cu — bandwidth-bound kernels of the generator training step.
#include "gen_kernels.cuh"
#include "small_kernels.cuh"

namespace wb {

namespace {

__device__ __forceinline__ float block_sum(float v, float* sh) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x < 32) {
    t = (l < (int)(blockDim.x >> 5)) ? sh[l] : 0.f;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (l == 0) sh[0] = t;
  }
  __syncthreads();
  return sh[0];
}

// ---- counter-based normal generator (splitmix64 finaliser) ----
__device__ __forceinline__ unsigned long long mix64(unsigned long long x) {
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}
__device__ __forceinline__ void counter_u2(unsigned long long seed, unsigned long long stream, unsigned long long idx,
                                           float& u1, float& u2) {
  const unsigned long long key = mix64(seed * 0x9E3779B97F4A7C15ull + stream * 0xD1B54A32D192ED03ull);
  const unsigned long long h = mix64(key ^ (idx * 0x9E3779B97F4A7C15ull));
  u1 = (float)((h >> 40) + 1ull) * (1.0f / 16777216.0f);
  u2 = (float)(((h >> 8) & 0xFFFFFFull) + 1ull) * (1.0f / 16777216.0f);
}
__device__ __forceinline__ float counter_normal(unsigned long long seed, unsigned long long stream,
                                                unsigned long long idx) {
  float u1, u2;
  counter_u2(seed, stream, idx, u1, u2);
  return sqrtf(-2.f * logf(u1)) * cospif(2.f * u2);
}

__device__ __forceinline__ float act_fwd(float x, int kind, float slope, float alpha) {
  return kind == 1 ? snake(x, alpha) : lrelu(x, slope);
}

}  // namespace

// =============================================================================================
// weights
// =============================================================================================
// Device storage of GEMM-fed weights is tap-major [k][C_out][C_in].  A weight-norm "row" is one dim-0
// index of the reference tensor: conv r = out channel (elements (tap, in)), convT r = in channel
// (elements (tap, out)).  Element i of row r: tap = i / cols, c = i % cols.
__device__ __forceinline__ size_t wrow_addr(int i, int r, int rows, int cols, int is_convT) {
  const int t = i / cols, c = i - t * cols;
  return is_convT ? ((size_t)t * cols + c) * rows + r : ((size_t)t * rows + r) * cols + c;
}

__global__ void prep_weights_batched_kernel(const PrepDesc* __restrict__ descs, int ndesc) {
  __shared__ float sh[32];
  __shared__ int di;
  if (threadIdx.x == 0) {
    int lo = 0, hi = ndesc - 1;  // last descriptor with first <= blockIdx.x
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (descs[mid].first <= (int)blockIdx.x) lo = mid;
      else hi = mid - 1;
    }
    di = lo;
  }
  __syncthreads();
  const PrepDesc d = descs[di];
  const int r = blockIdx.x - d.first;
  const int rows = d.rows, cols = d.cols, k = d.k, is_convT = d.is_convT;
  const int per = cols * k;
  float scale = 1.f;
  if (d.g) {
    float s = 0.f;
    for (int i = threadIdx.x; i < per; i += blockDim.x) {
      const float x = d.v[wrow_addr(i, r, rows, cols, is_convT)];
      s += x * x;
    }
    s = block_sum(s, sh);
    const float n = sqrtf(s);
    scale = d.g[r] / n;
    if (threadIdx.x == 0 && d.norm) d.norm[r] = n;
  }
  // only row-contiguous layouts here (coalesced); the transposed ones come from prep_transpose
  for (int i = threadIdx.x; i < per; i += blockDim.x) {
    const int t = i / cols, c = i - t * cols;
    const float w = d.v[wrow_addr(i, r, rows, cols, is_convT)] * scale;
    bf16 hi, lo;
    split_bf16(w, hi, lo);
    const size_t f = ((size_t)t * rows + r) * cols + c;  // [t][r][c]
    if (!is_convT) {
      d.fwd_hi[f] = hi;  // conv: r = out channel, c = in channel
      d.fwd_lo[f] = lo;
    } else {
      d.dg[f] = hi;      // convT: r = in channel, c = out channel
      d.lo_tmp[f] = lo;
    }
  }
}

// Batched bf16 [R][C] -> [C][R] transposes through 32 x 32 shared-memory tiles.
__global__ void __launch_bounds__(256) prep_transpose_kernel(const TransDesc* __restrict__ descs, int ndesc) {
  __shared__ unsigned short tile[32][33];
  __shared__ int di;
  if (threadIdx.x == 0 && threadIdx.y == 0) {
    int lo = 0, hi = ndesc - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (descs[mid].first <= (int)blockIdx.x) lo = mid;
      else hi = mid - 1;
    }
    di = lo;
  }
  __syncthreads();
  const TransDesc d = descs[di];
  const int b = blockIdx.x - d.first;
  const int tc = (d.C + 31) / 32;
  const int r0 = (b / tc) * 32, c0 = (b % tc) * 32;
  const unsigned short* src = reinterpret_cast<const unsigned short*>(d.src);
  unsigned short* dst = reinterpret_cast<unsigned short*>(d.dst);
  for (int y = threadIdx.y; y < 32; y += 8) {
    const int r = r0 + y, c = c0 + threadIdx.x;
    if (r < d.R && c < d.C) tile[y][threadIdx.x] = src[(size_t)r * d.C + c];
  }
  __syncthreads();
  for (int y = threadIdx.y; y < 32; y += 8) {
    const int c = c0 + y, r = r0 + threadIdx.x;
    if (r < d.R && c < d.C) dst[(size_t)c * d.R + r] = tile[threadIdx.x][y];
  }
}

int prep_transpose_blocks(int R, int C) { return ((R + 31) / 32) * ((C + 31) / 32); }

void prep_transpose_batched(const TransDesc* descs, int ndesc, int total_blocks, cudaStream_t st) {
  if (ndesc > 0 && total_blocks > 0) prep_transpose_kernel<<<total_blocks, dim3(32, 8), 0, st>>>(descs, ndesc);
}

void prep_weights_batched(const PrepDesc* descs, int ndesc, int total_rows, cudaStream_t st) {
  prep_weights_batched_kernel<<<total_rows, 256, 0, st>>>(descs, ndesc);
}

__global__ void wn_backward_kernel(const float* __restrict__ dW, const float* __restrict__ v,
                                   const float* __restrict__ g, const float* __restrict__ norm, int rows, int cols,
                                   int k, int is_convT, float* __restrict__ dv, float* __restrict__ dgo) {
  __shared__ float sh[32];
  const int r = blockIdx.x;
  const int per = cols * k;
  float s = 0.f;
  for (int i = threadIdx.x; i < per; i += blockDim.x) {
    const size_t a = wrow_addr(i, r, rows, cols, is_convT);
    s += dW[a] * v[a];
  }
  s = block_sum(s, sh);
  const float n = norm[r];
  const float dgr = s / n;
  if (threadIdx.x == 0) dgo[r] = dgr;
  const float a = g[r] / n, b = dgr / n;
  for (int i = threadIdx.x; i < per; i += blockDim.x) {
    const size_t q = wrow_addr(i, r, rows, cols, is_convT);
    dv[q] = a * (dW[q] - b * v[q]);
  }
}

void wn_backward(const float* dW, const float* v, const float* g, const float* norm, int rows, int cols, int k,
                 int is_convT, float* dv, float* dg, cudaStream_t st) {
  wn_backward_kernel<<<rows, 256, 0, st>>>(dW, v, g, norm, rows, cols, k, is_convT, dv, dg);
}

__global__ void wn_backward_batched_kernel(const WnDesc* __restrict__ descs, int ndesc) {
  __shared__ float sh[32];
  __shared__ int di;
  if (threadIdx.x == 0) {
    int lo = 0, hi = ndesc - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (descs[mid].first <= (int)blockIdx.x) lo = mid;
      else hi = mid - 1;
    }
    di = lo;
  }
  __syncthreads();
  const WnDesc d = descs[di];
  const int r = blockIdx.x - d.first;
  const int per = d.cols * d.k;
  float s = 0.f;
  for (int i = threadIdx.x; i < per; i += blockDim.x) {
    const size_t a = wrow_addr(i, r, d.rows, d.cols, d.is_convT);
    s += d.dW[a] * d.v[a];
  }
  s = block_sum(s, sh);
  const float n = d.norm[r];
  const float dgr = s / n;
  if (threadIdx.x == 0) d.dg[r] = dgr;
  const float a = d.g[r] / n, b = dgr / n;
  for (int i = threadIdx.x; i < per; i += blockDim.x) {
    const size_t q = wrow_addr(i, r, d.rows, d.cols, d.is_convT);
    d.dv[q] = a * (d.dW[q] - b * d.v[q]);
  }
}

void wn_backward_batched(const WnDesc* descs, int ndesc, int total_rows, cudaStream_t st) {
  if (ndesc > 0 && total_rows > 0) wn_backward_batched_kernel<<<total_rows, 256, 0, st>>>(descs, ndesc);
}

// Step state lives on the device so a captured step graph advances it by itself.
__global__ void step_bump_kernel(StepState* s, int bump_noise) {
  s->adam_t += 1;
  if (bump_noise) s->noise_stream += 1;
}

void step_bump(StepState* s, int bump_noise, cudaStream_t st) { step_bump_kernel<<<1, 1, 0, st>>>(s, bump_noise); }

__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, long long n, float lr, float b1, float b2, float eps, float wd,
                             const StepState* __restrict__ state, float grad_scale) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long n4 = n >> 2;
  // bias corrections of src/wubu_train.c:97-103 (clamped, and applied twice like the reference)
  const float t = (float)state->adam_t;
  float bias1 = 1.0f - powf(b1, t);
  float bias2 = 1.0f - powf(b2, t);
  bias1 = fmaxf(bias1, 1e-12f);
  bias2 = fmaxf(bias2, 1e-12f);
  const float lr_eff = lr * sqrtf(bias2) / bias1;
  if (i < n4) {
    float4 pp = reinterpret_cast<float4*>(p)[i];
    const float4 gg = reinterpret_cast<const float4*>(g)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float* P4 = &pp.x; const float* G4 = &gg.x; float* M4 = &mm.x; float* V4 = &vv.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float gr = G4[j] * grad_scale;
      const float mn = b1 * M4[j] + (1.f - b1) * gr;
      const float vn = b2 * V4[j] + (1.f - b2) * gr * gr;
      M4[j] = mn;
      V4[j] = vn;
      const float den = sqrtf(vn / bias2) + eps;
      P4[j] -= lr_eff * (mn / bias1) / den + lr * wd * P4[j];
    }
    reinterpret_cast<float4*>(p)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
  }
}

void adamw(float* p, const float* g, float* m, float* v, long long n, float lr, float b1, float b2, float eps, float wd,
           const StepState* state, float grad_scale, cudaStream_t st) {
  // n is a multiple of 4 (flat buffer segments are 64-float aligned)
  const long long n4 = n >> 2;
  adamw_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, st>>>(p, g, m, v, n, lr, b1, b2, eps, wd, state, grad_scale);
}

// =============================================================================================
// inputs / cond
// =============================================================================================
__global__ void pack_z_kernel(const float* __restrict__ z, int B, int C, int F, bf16* __restrict__ hi,
                              bf16* __restrict__ lo) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)B * C * F) return;
  const int c = (int)(i % C);
  const long long bf = i / C;
  const int f = (int)(bf % F), b = (int)(bf / F);
  const float x = z[((size_t)b * C + c) * F + f];
  split_bf16(x, hi[i], lo[i]);
}

void pack_z(const float* z, int B, int C, int F, bf16* hi, bf16* lo, cudaStream_t st) {
  const long long n = (long long)B * C * F;
  pack_z_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(z, B, C, F, hi, lo);
}

__global__ void cond_forward_kernel(const float* __restrict__ W, const float* __restrict__ bias,
                                    const float* __restrict__ g, int B, int C, int gin, float* __restrict__ rowadd) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B * C) return;
  const int b = i / C, c = i % C;
  float s = bias ? bias[c] : 0.f;
  for (int j = 0; j < gin; ++j) s += W[(size_t)c * gin + j] * g[(size_t)b * gin + j];
  rowadd[i] = s;
}

void cond_forward(const float* W, const float* bias, const float* g, int B, int C, int gin, float* rowadd,
                  cudaStream_t st) {
  cond_forward_kernel<<<(B * C + 255) / 256, 256, 0, st>>>(W, bias, g, B, C, gin, rowadd);
}

__global__ void cond_backward_kernel(const float* __restrict__ part, int tpi, int B, int C, const float* __restrict__ g,
                                     int gin, float* __restrict__ dW, float* __restrict__ db) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= C * (gin + 1)) return;
  const int c = idx / (gin + 1), j = idx % (gin + 1);
  float acc = 0.f;
  for (int b = 0; b < B; ++b) {
    float s = 0.f;
    for (int t = 0; t < tpi; ++t) s += part[((size_t)b * tpi + t) * C + c];
    acc += (j < gin) ? s * g[(size_t)b * gin + j] : s;
  }
  if (j < gin) dW[(size_t)c * gin + j] = acc;
  else db[c] = acc;
}

void cond_backward(const float* tile_part, int tiles_per_item, int B, int C, const float* g, int gin, float* dW,
                   float* db, cudaStream_t st) {
  const int n = C * (gin + 1);
  cond_backward_kernel<<<(n + 255) / 256, 256, 0, st>>>(tile_part, tiles_per_item, B, C, g, gin, dW, db);
}

// =============================================================================================
// harmonic source (SineGen + l_linear + tanh)
// =============================================================================================
__global__ void nsf_phase_kernel(const float* __restrict__ f0, int B, int F, int upp, float sr, double* acc) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  double a = 0.0;
  for (int f = 0; f < F; ++f) {
    acc[(size_t)b * F + f] = a;  // carry into frame f = fmod(sum of rad2 over frames < f, 1)
    const double rad = (double)f0[(size_t)b * F + f] / (double)sr * (double)upp;
    const double r2 = fmod(rad + 0.5, 1.0) - 0.5;
    a = fmod(a + r2, 1.0);
  }
}

__global__ void nsf_sample_kernel(NsfArgs a) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long T = (long long)a.F * a.upp;
  if (i >= (long long)a.B * T) return;
  const int b = (int)(i / T);
  const int t = (int)(i - (long long)b * T);
  const int f = t / a.upp, u = t - f * a.upp;
  const float f0 = a.f0[(size_t)b * a.F + f];
  const double ph0 = (double)f0 / (double)a.sr * (double)(u + 1) + a.acc[(size_t)b * a.F + f];
  const float uv = f0 > 0.f ? 1.f : 0.f;
  const float namp = uv * a.noise_std + (1.f - uv) * a.sine_amp / 3.f;
  const unsigned long long nstream = *a.stream;
  float lin = a.lin_b[0];
  for (int h = 0; h < a.dim; ++h) {
    float ri = 0.f;
    if (h > 0) {
      float u1, u2;
      counter_u2(a.seed, nstream ^ 0x5A5Aull, (unsigned long long)h, u1, u2);
      ri = u1 - 1.0f / 16777216.0f;
    }
    double x = ph0 * (double)(h + 1) + (double)ri;
    x -= floor(x);
    const float s = sinpif(2.f * (float)x) * a.sine_amp;
    const unsigned long long idx = (unsigned long long)i * a.dim + h;
    const float n = a.noise ? a.noise[idx] : counter_normal(a.seed, nstream, idx);
    const float sw = s * uv + namp * n;
    a.sw[idx] = sw;
    lin += a.lin_w[h] * sw;
  }
  a.har[i] = tanhf(lin);
}

void nsf_forward(const NsfArgs& a, cudaStream_t st) {
  nsf_phase_kernel<<<(a.B + 63) / 64, 64, 0, st>>>(a.f0, a.B, a.F, a.upp, a.sr, a.acc);
  const long long n = (long long)a.B * a.F * a.upp;
  nsf_sample_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(a);
}

__global__ void nsf_backward_kernel(const float* __restrict__ d_har, const float* __restrict__ har,
                                    const float* __restrict__ sw, long long n, int dim, int nparts,
                                    float* __restrict__ part) {
  __shared__ float sh[32];
  const long long per = (n + nparts - 1) / nparts;
  const long long i0 = (long long)blockIdx.x * per, i1 = min(n, i0 + per);
  float acc[10];
  for (int h = 0; h <= dim && h < 10; ++h) acc[h] = 0.f;
  for (long long i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    const float y = har[i];
    const float d = d_har[i] * (1.f - y * y);
    for (int h = 0; h < dim && h < 9; ++h) acc[h] += d * sw[i * dim + h];
    acc[9] += d;
  }
  for (int h = 0; h < dim && h < 9; ++h) {
    const float s = block_sum(acc[h], sh);
    if (threadIdx.x == 0) part[(size_t)blockIdx.x * (dim + 1) + h] = s;
  }
  const float s = block_sum(acc[9], sh);
  if (threadIdx.x == 0) part[(size_t)blockIdx.x * (dim + 1) + dim] = s;
}

void rows_reduce(const float* part, int nparts, int n, float* out, int accumulate, cudaStream_t st) {
  col_reduce(part, nparts, n, out, accumulate, st);
}

__global__ void split_lin_kernel(const float* __restrict__ red, int dim, float* __restrict__ dw, float* __restrict__ db) {
  const int h = threadIdx.x;
  if (h < dim) dw[h] = red[h];
  if (h == 0) db[0] = red[dim];
}

void nsf_backward(const float* d_har, const float* har, const float* sw, int n, int dim, float* part, int nparts,
                  float* dlin_w, float* dlin_b, cudaStream_t st) {
  nsf_backward_kernel<<<nparts, 256, 0, st>>>(d_har, har, sw, n, dim, nparts, part);
  // reduce in place into the tail of `part`
  float* red = part + (size_t)nparts * (dim + 1);
  rows_reduce(part, nparts, dim + 1, red, 0, st);
  split_lin_kernel<<<1, 32, 0, st>>>(red, dim, dlin_w, dlin_b);
}

}  // namespace wb
