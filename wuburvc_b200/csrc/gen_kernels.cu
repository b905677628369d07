// gen_kernels.cu — bandwidth-bound kernels of the generator training step.
#include "gen_kernels.cuh"
#include "small_kernels.cuh"

namespace wb {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

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

namespace {
// descriptor i with first_i <= block < first_{i+1} (firsts ascending); `which` 0 = norm, 1 = tile
__device__ int prep_find(const PrepDesc* descs, int ndesc, int which) {
  int lo = 0, hi = ndesc - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    const int f = which ? descs[mid].tile_first : descs[mid].norm_first;
    if (f <= (int)blockIdx.x) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}
}  // namespace

int prep_norm_blocks(const PrepDesc& d) {
  if (!d.g) return 0;
  return d.is_convT ? (d.Q / 32) * d.nchunks : (d.P + 7) / 8;
}

int prep_tile_blocks(const PrepDesc& d) { return d.k * (d.P / 32) * (d.Q / (32 * d.qs)); }

__global__ void __launch_bounds__(256) prep_norm_kernel(const PrepDesc* __restrict__ descs, int ndesc) {
  __shared__ float red[8][33];
  __shared__ int di;
  if (threadIdx.x == 0) di = prep_find(descs, ndesc, 0);
  __syncthreads();
  const PrepDesc d = descs[di];
  const int b = blockIdx.x - d.norm_first;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (!d.is_convT) {  // row p: every tap's contiguous Q floats
    const int p = b * 8 + warp;
    if (p >= d.P) return;
    float s = 0.f;
    for (int t = 0; t < d.k; ++t) {
      const float* row = d.v + ((size_t)t * d.P + p) * d.Q;
#pragma unroll 4
      for (int q = lane; q < d.Q; q += 32) {
        const float x = row[q];
        s += x * x;
      }
    }
    s = warp_sum(s);
    if (lane == 0) d.norm[p] = sqrtf(s);
  } else {  // columns q0..q0+31 over one chunk of (tap, p) pairs
    const int ncb = d.Q / 32;
    const int cb = b % ncb, ch = b / ncb;
    const int q = cb * 32 + lane;
    const int i0 = ch * kPrepPairs, i1 = min(d.k * d.P, i0 + kPrepPairs);
    float s = 0.f;
#pragma unroll 4
    for (int i = i0 + warp; i < i1; i += 8) {
      const float x = d.v[(size_t)i * d.Q + q];
      s += x * x;
    }
    red[warp][lane] = s;
    __syncthreads();
    if (warp == 0) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) t += red[w][lane];
      d.npart[(size_t)ch * d.Q + q] = t;
    }
  }
}

__global__ void __launch_bounds__(256) prep_tile_kernel(const PrepDesc* __restrict__ descs, int ndesc) {
  __shared__ float s_scale[128];
  __shared__ unsigned short ht[128][34];  // transposed bf16 weight: [q - q0][p - p0]
  __shared__ unsigned short lt[128][34];  // its lo companion (fp32 precision)
  __shared__ int di;
  if (threadIdx.x == 0) di = prep_find(descs, ndesc, 1);
  __syncthreads();
  const PrepDesc d = descs[di];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int QS = d.qs, QW = 32 * QS;
  const int nqb = d.Q / QW, npb = d.P / 32;
  int b = blockIdx.x - d.tile_first;
  const int qb = b % nqb;
  b /= nqb;
  const int pb = b % npb, t = b / npb;
  const int p0 = pb * 32, q0 = qb * QW;
  if (!d.is_convT) {
    if (tid < 32) s_scale[tid] = d.g ? d.g[p0 + tid] / d.norm[p0 + tid] : 1.f;
  } else if (tid < QW) {
    float sc = 1.f;
    if (d.g) {
      float s = 0.f;
      for (int ch = 0; ch < d.nchunks; ++ch) s += d.npart[(size_t)ch * d.Q + q0 + tid];
      const float n = sqrtf(s);
      sc = d.g[q0 + tid] / n;
      if (t == 0 && pb == 0) d.norm[q0 + tid] = n;
    }
    s_scale[tid] = sc;
  }
  __syncthreads();
  // tap of the storage-layout output: t (conv) or the tap's place in the polyphase order (convT)
  int ts = t;
  if (d.is_convT) {
    const int ph = t % d.stride;
    ts = t / d.stride;
    for (int q = 0; q < ph; ++q) ts += (d.k - q + d.stride - 1) / d.stride;
  }
  const int td = d.is_convT ? t : d.k - 1 - t;  // tap of the transposed output
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int pl = warp + 8 * j, p = p0 + pl;
    const size_t src = ((size_t)t * d.P + p) * d.Q + q0 + lane * QS;
    const size_t dst = ((size_t)ts * d.P + p) * d.Q + q0 + lane * QS;
    float x[4];
    if (QS == 4) {
      const float4 f = *reinterpret_cast<const float4*>(d.v + src);
      x[0] = f.x; x[1] = f.y; x[2] = f.z; x[3] = f.w;
    } else if (QS == 2) {
      const float2 f = *reinterpret_cast<const float2*>(d.v + src);
      x[0] = f.x; x[1] = f.y;
    } else {
      x[0] = d.v[src];
    }
    f16 hi[4], lo[4];
    bool big = false;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (e < QS) {
        const float sc = d.is_convT ? s_scale[lane * QS + e] : s_scale[pl];
        const float w = x[e] * sc;
        split_op(w, d.fmt_bf16, hi[e], lo[e]);
        big |= !d.fmt_bf16 && !(fabsf(w) < kF16Max);
        const bf16 wb16 = __float2bfloat16_rn(w);
        ht[lane * QS + e][pl] = __bfloat16_as_ushort(wb16);
        if (d.dg_lo) lt[lane * QS + e][pl] = __bfloat16_as_ushort(__float2bfloat16_rn(w - __bfloat162float(wb16)));
      }
    }
    if (big && d.range_err) atomicCAS(d.range_err, 0, ERR_RANGE);
    if (QS == 4) {
      *reinterpret_cast<uint2*>(d.fwd_hi + dst) =
          make_uint2(__half_as_ushort(hi[0]) | ((uint32_t)__half_as_ushort(hi[1]) << 16),
                     __half_as_ushort(hi[2]) | ((uint32_t)__half_as_ushort(hi[3]) << 16));
      *reinterpret_cast<uint2*>(d.fwd_lo + dst) =
          make_uint2(__half_as_ushort(lo[0]) | ((uint32_t)__half_as_ushort(lo[1]) << 16),
                     __half_as_ushort(lo[2]) | ((uint32_t)__half_as_ushort(lo[3]) << 16));
    } else if (QS == 2) {
      *reinterpret_cast<uint32_t*>(d.fwd_hi + dst) =
          __half_as_ushort(hi[0]) | ((uint32_t)__half_as_ushort(hi[1]) << 16);
      *reinterpret_cast<uint32_t*>(d.fwd_lo + dst) =
          __half_as_ushort(lo[0]) | ((uint32_t)__half_as_ushort(lo[1]) << 16);
    } else {
      d.fwd_hi[dst] = hi[0];
      d.fwd_lo[dst] = lo[0];
    }
  }
  __syncthreads();
  // transposed bf16: rows q0..q0+QW-1 of dg[td] ([Q][P]), 32 p each, 16 threads x 2 values per row
  // (none in a forward-only context)
  if (!d.dg) return;
  for (int r = tid >> 4; r < QW; r += 16) {
    const int pp = (tid & 15) * 2;
    const uint32_t w = (uint32_t)ht[r][pp] | ((uint32_t)ht[r][pp + 1] << 16);
    *reinterpret_cast<uint32_t*>(d.dg + ((size_t)td * d.Q + q0 + r) * d.P + p0 + pp) = w;
    if (d.dg_lo)
      *reinterpret_cast<uint32_t*>(d.dg_lo + ((size_t)td * d.Q + q0 + r) * d.P + p0 + pp) =
          (uint32_t)lt[r][pp] | ((uint32_t)lt[r][pp + 1] << 16);
  }
}

void prep_weights(const PrepDesc* descs, int ndesc, int norm_blocks, int tile_blocks, cudaStream_t st) {
  if (ndesc <= 0) return;
  if (norm_blocks > 0) prep_norm_kernel<<<norm_blocks, 256, 0, st>>>(descs, ndesc);
  if (tile_blocks > 0) prep_tile_kernel<<<tile_blocks, 256, 0, st>>>(descs, ndesc);
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
WB_DEV bool skip_step(const int* err, const float* skip_flag) {
  return (err && *err == ERR_RANGE) || (skip_flag && *skip_flag > 0.f);
}

__global__ void step_bump_kernel(StepState* s, int bump_noise, const int* err, const float* skip_flag) {
  if (skip_step(err, skip_flag)) return;
  s->adam_t += 1;
  if (bump_noise) s->noise_stream += 1;
}

void step_bump(StepState* s, int bump_noise, const int* err, const float* skip_flag, cudaStream_t st) {
  step_bump_kernel<<<1, 1, 0, st>>>(s, bump_noise, err, skip_flag);
}

__global__ void range_flag_kernel(const int* err, float* flag) { *flag = (*err == ERR_RANGE) ? 1.f : 0.f; }

void range_flag(const int* err, float* flag, cudaStream_t st) { range_flag_kernel<<<1, 1, 0, st>>>(err, flag); }

__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, long long n, float lr, float b1, float b2, float eps, float wd,
                             const StepState* __restrict__ state, float grad_scale, int* err,
                             const float* skip_flag) {
  // a step whose forward overflowed the operand format (here or, under data parallelism, on another
  // rank) is skipped whole; the host recomputes it
  if (skip_step(err, skip_flag)) {
    if (blockIdx.x == 0 && threadIdx.x == 0 && err) atomicCAS(err, 0, ERR_RANGE);
    return;
  }
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
           const StepState* state, float grad_scale, int* err, const float* skip_flag, cudaStream_t st) {
  // n is a multiple of 4 (flat buffer segments are 64-float aligned)
  const long long n4 = n >> 2;
  adamw_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, st>>>(p, g, m, v, n, lr, b1, b2, eps, wd, state, grad_scale,
                                                             err, skip_flag);
}

// =============================================================================================
// inputs / cond
// =============================================================================================
__global__ void pack_z_kernel(const float* __restrict__ z, int B, int C, int F, f16* __restrict__ hi,
                              f16* __restrict__ lo, bf16* __restrict__ zb, bf16* __restrict__ zb_lo, int* range_err,
                              int fmt_bf16) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)B * C * F) return;
  const int c = (int)(i % C);
  const long long bf = i / C;
  const int f = (int)(bf % F), b = (int)(bf / F);
  const float x = z[((size_t)b * C + c) * F + f];
  split_op(x, fmt_bf16, hi[i], lo[i]);
  const bf16 xb = __float2bfloat16_rn(x);
  if (zb) zb[i] = xb;
  if (zb_lo) zb_lo[i] = __float2bfloat16_rn(x - __bfloat162float(xb));
  if (!fmt_bf16 && !(fabsf(x) < kF16Max) && range_err) atomicCAS(range_err, 0, ERR_RANGE);
}

void pack_z(const float* z, int B, int C, int F, f16* hi, f16* lo, bf16* zb, bf16* zb_lo, int* range_err,
            int fmt_bf16, cudaStream_t st) {
  const long long n = (long long)B * C * F;
  pack_z_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(z, B, C, F, hi, lo, zb, zb_lo, range_err, fmt_bf16);
}

// rowadd[b][c] = bias[c] + sum_j W[c][j] * g[b][j]: warp per output channel c (its weight row read
// once, coalesced), every item's dot product reduced across the lanes.
__global__ void __launch_bounds__(256) cond_forward_kernel(const float* __restrict__ W, const float* __restrict__ bias,
                                                           const float* __restrict__ g, int B, int C, int gin,
                                                           float* __restrict__ rowadd) {
  const int lane = threadIdx.x & 31;
  const int c = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (c >= C) return;
  const float* wr = W + (size_t)c * gin;
  const float b0 = bias ? bias[c] : 0.f;
  for (int b = 0; b < B; ++b) {
    const float* gb = g + (size_t)b * gin;
    float s = 0.f;
    for (int j = lane; j < gin; j += 32) s += wr[j] * gb[j];
    s = warp_sum(s);
    if (lane == 0) rowadd[(size_t)b * C + c] = b0 + s;
  }
}

void cond_forward(const float* W, const float* bias, const float* g, int B, int C, int gin, float* rowadd,
                  cudaStream_t st) {
  cond_forward_kernel<<<(C + 7) / 8, 256, 0, st>>>(W, bias, g, B, C, gin, rowadd);
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
// Phase carried into each frame: acc[b][f] = sum over frames g < f of r2(g) (mod 1), r2(g) =
// fmod(f0[g]/sr*upp + 0.5, 1) - 0.5, the cumulative carry of SineGen (models.py:313-316; the
// reference's serial loop at src/wubu_rvc_real.c:1471-1489).  Only the value mod 1 matters (the source
// takes sin(2*pi*phase)), so the carry is a parallel prefix sum in fp64 wrapped to (-1, 1): one block
// per item, each thread sums a contiguous run of frames, a block-wide exclusive scan gives every run
// its starting carry, and each thread re-walks its run from there.  Over 6000 frames |sum| <= 3000,
// so the unwrapped fp64 partial sums keep ~1e-12 absolute accuracy; the order is fixed
// (deterministic).
WB_DEV double nsf_r2(float f0, float sr, int upp) {
  // fmod(x, 1) == x - trunc(x) exactly for finite x (the difference is representable)
  const double x = (double)f0 / (double)sr * (double)upp + 0.5;
  return (x - trunc(x)) - 0.5;
}

constexpr int kPhaseThreads = 256;

__global__ void __launch_bounds__(kPhaseThreads) nsf_phase_kernel(const float* __restrict__ f0, int F, int upp,
                                                                  float sr, double* __restrict__ acc) {
  __shared__ double warp_tot[kPhaseThreads / 32];
  const int b = blockIdx.x, j = threadIdx.x, lane = j & 31, warp = j >> 5;
  const int per = (F + kPhaseThreads - 1) / kPhaseThreads;
  const int f_begin = min(F, j * per), f_end = min(F, f_begin + per);
  const float* fb = f0 + (size_t)b * F;
  double loc = 0.0;
  for (int f = f_begin; f < f_end; ++f) loc += nsf_r2(fb[f], sr, upp);
  // inclusive scan within the warp, then over the warps' totals
  double inc = loc;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double v = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += v;
  }
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    double t = lane < kPhaseThreads / 32 ? warp_tot[lane] : 0.0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double v = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += v;
    }
    if (lane < kPhaseThreads / 32) warp_tot[lane] = t;  // inclusive over warps
  }
  __syncthreads();
  const double base = (inc - loc) + (warp > 0 ? warp_tot[warp - 1] : 0.0);  // exclusive prefix
  double a = base - trunc(base);
  for (int f = f_begin; f < f_end; ++f) {
    acc[(size_t)b * F + f] = a;
    const double y = a + nsf_r2(fb[f], sr, upp);
    a = y - trunc(y);
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
  nsf_phase_kernel<<<a.B, kPhaseThreads, 0, st>>>(a.f0, a.F, a.upp, a.sr, a.acc);
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
