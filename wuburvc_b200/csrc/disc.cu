// disc.cu — the RVC GAN discriminators (MultiPeriodDiscriminator: DiscriminatorS + one
// DiscriminatorP per period) with their losses, forward and backward, and their AdamW step.
//
// Upstream (knowledge/rvc_original/): infer/module/models.py:928-1094 (the discriminators),
// train/losses.py:4-40 (discriminator_loss, generator_loss, feature_loss), train/train.py:500-525
// (the step order: the discriminator's step on (real, generated detached), then the generator's
// adversarial + feature-matching loss through the updated discriminator).
//
// Layout.  Every activation is fp32 channels-first [N][C][L].  A (k, 1) Conv2d of DiscriminatorP
// is a Conv1d along time on each of the p columns of the reflect-padded [T/p][p] view, so the p
// columns of every item become p sequences: N = 2 B p (B = 1 per item for DiscriminatorS), the real
// items' sequences first, then the generated ones.  One forward over the 2B items serves both
// halves; the real half's feature maps are the detached targets of the feature-matching loss.
//
// Kernels (fp32 FMA on the CUDA cores; the strided and grouped convolutions of the discriminators
// have no stride-1 channels-last form for the tensor-core kernels of the generator):
//   forward         out[n][co][t] = act(b[co] + sum_{ci in group, k} w[co][ci][k] x[n][ci][t s + k - pad])
//   input gradient  dx[n][ci][u]  = sum_{co in group, k : u + pad - k = t s} w[co][ci][k] dz[n][co][t]
//   weight gradient dW[co][ci, k | bias] = sum_{n, t} dz[n][co][t] x[n][ci][t s + k - pad]  (split over
//                   position ranges; partials reduced in a fixed order, so every result is deterministic)
// The dense layers (64 | channels per group), which carry nearly all the FLOPs, run these as
// register-tiled implicit GEMMs (disc_gemm_{fwd,dgrad,wgrad}_kernel); the grouped layers, the
// one-channel first layers and conv_post run them as one output row per thread
// (disc_conv_{fwd,dgrad,wgrad}_kernel, disc_post_fwd_kernel).  Plus the weight norm
// w = g v / ||v|| (per output row) and its backward, the loss terms, the LeakyReLU /
// feature-matching gradient, the reflect-pad adjoint, torch's AdamW, and the data-parallel gradient
// all-reduce.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include <sched.h>
#include <unistd.h>

#include <chrono>

#include "../../include/wuburvc_b200.h"
#include "nccl_plain.h"

namespace wb {
namespace disc {

constexpr float kSlope = 0.1f;  // modules.LRELU_SLOPE
constexpr int kPos = 128;       // positions per block of the forward / input-gradient kernels
constexpr int kCIC = 32;        // input channels per weight stage of the forward
constexpr int kOC = 32;         // output channels per weight stage of the input gradient
constexpr int kLossBlocks = 64; // partial sums per loss term

struct DLayer {
  int C_in, C_out, k, s, groups, pad, L_in, L_out, act;
};

// ------------------------------------------------------------------------------------------------
// convolutions
// ------------------------------------------------------------------------------------------------
template <int TCO>
__global__ void __launch_bounds__(kPos) disc_conv_fwd_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                            const float* __restrict__ bias, float* __restrict__ y,
                                                            DLayer L, int N) {
  extern __shared__ float4 smem_f4[];
  float* ws = reinterpret_cast<float*>(smem_f4);  // [r * k + kk][TCO]
  const int cig = L.C_in / L.groups, cog = L.C_out / L.groups;
  const int co0 = blockIdx.y * TCO, g = co0 / cog;
  const int pos = blockIdx.x * kPos + threadIdx.x;
  const bool live = pos < N * L.L_out;
  const int n = live ? pos / L.L_out : 0, t = live ? pos - n * L.L_out : 0;
  const float* xn = x + ((size_t)n * L.C_in + (size_t)g * cig) * L.L_in;
  const int in0 = t * L.s - L.pad;
  float acc[TCO];
#pragma unroll
  for (int o = 0; o < TCO; ++o) acc[o] = 0.f;
  for (int c0 = 0; c0 < cig; c0 += kCIC) {
    const int cc = min(kCIC, cig - c0), rk = cc * L.k;
    __syncthreads();
    for (int i = threadIdx.x; i < TCO * rk; i += kPos) {
      const int o = i / rk, rem = i - o * rk;
      ws[rem * TCO + o] = w[((size_t)(co0 + o) * cig + c0) * L.k + rem];
    }
    __syncthreads();
    for (int r = 0; r < cc; ++r) {
      const float* xr = xn + (size_t)(c0 + r) * L.L_in;
      for (int kk = 0; kk < L.k; ++kk) {
        const int q = in0 + kk;
        const float xv = (live && q >= 0 && q < L.L_in) ? __ldg(xr + q) : 0.f;
        const float* wp = ws + (r * L.k + kk) * TCO;
#pragma unroll
        for (int o = 0; o < TCO; ++o) acc[o] = fmaf(wp[o], xv, acc[o]);
      }
    }
  }
  if (!live) return;
#pragma unroll
  for (int o = 0; o < TCO; ++o) {
    float v = acc[o] + bias[co0 + o];
    if (L.act) v = v > 0.f ? v : v * kSlope;
    y[((size_t)n * L.C_out + co0 + o) * L.L_out + t] = v;
  }
}

template <int TCI>
__global__ void __launch_bounds__(kPos) disc_conv_dgrad_kernel(const float* __restrict__ dz, const float* __restrict__ w,
                                                              float* __restrict__ dx, DLayer L, int N) {
  extern __shared__ float4 smem_f4[];
  float* ws = reinterpret_cast<float*>(smem_f4);  // [o * k + kk][TCI]
  const int cig = L.C_in / L.groups, cog = L.C_out / L.groups;
  const int ci0 = blockIdx.y * TCI, g = ci0 / cig, cl0 = ci0 - g * cig;
  const int pos = blockIdx.x * kPos + threadIdx.x;
  const bool live = pos < N * L.L_in;
  const int n = live ? pos / L.L_in : 0, u = live ? pos - n * L.L_in : 0;
  const float* dzn = dz + ((size_t)n * L.C_out + (size_t)g * cog) * L.L_out;
  const int num0 = u + L.pad;     // t * s = num0 - kk
  const int kk0 = num0 % L.s;     // the first tap whose output position is whole
  float acc[TCI];
#pragma unroll
  for (int i = 0; i < TCI; ++i) acc[i] = 0.f;
  for (int o0 = 0; o0 < cog; o0 += kOC) {
    const int oc = min(kOC, cog - o0);
    __syncthreads();
    for (int e = threadIdx.x; e < oc * L.k * TCI; e += kPos) {
      const int i = e % TCI, okk = e / TCI, o = okk / L.k, kk = okk - o * L.k;
      ws[e] = w[((size_t)(g * cog + o0 + o) * cig + cl0 + i) * L.k + kk];
    }
    __syncthreads();
    for (int kk = kk0; kk < L.k; kk += L.s) {
      const int num = num0 - kk;
      const int t = num / L.s;
      const bool ok = live && num >= 0 && t < L.L_out;
      for (int o = 0; o < oc; ++o) {
        const float dv = ok ? __ldg(dzn + (size_t)(o0 + o) * L.L_out + t) : 0.f;
        const float* wp = ws + (o * L.k + kk) * TCI;
#pragma unroll
        for (int i = 0; i < TCI; ++i) acc[i] = fmaf(wp[i], dv, acc[i]);
      }
    }
  }
  if (!live) return;
#pragma unroll
  for (int i = 0; i < TCI; ++i) dx[((size_t)n * L.C_in + ci0 + i) * L.L_in + u] = acc[i];
}

// Register-tiled implicit GEMMs for the dense layers, which carry nearly all the FLOPs: a 256-thread
// block computes 64 rows x 128 columns, 4 x 8 per thread, over K chunks of 16 rows double-buffered in
// shared memory; the next chunk's global loads are issued into registers before the current chunk's
// FMAs.  The forward and input-gradient kernels read a tap-major copy of the weights ([co][kk][ci],
// written by the weight-norm kernel) and order K tap-major too, so one chunk lies inside one tap: the
// tap, the channel base and each position's range check are uniform over the chunk.
constexpr int kGM = 64, kGN = 128, kGK = 16;
constexpr int kGT = 128;  // threads of a GEMM block: 8 x 8 outputs each

struct GemmSmem {
  float A[2][kGK][kGM + 4];
  float B[2][kGK][kGN + 4];
};

// one K chunk: thread (ty, tx) owns rows ty*8..ty*8+7 and columns tx*4..+3, 64+tx*4..+3; the
// fragments of step kq + 1 are read while step kq's FMAs run
__device__ __forceinline__ void gemm_chunk(const float (*A)[kGM + 4], const float (*B)[kGN + 4], int ty, int tx,
                                           float (&acc)[8][8]) {
  float4 a0 = *reinterpret_cast<const float4*>(&A[0][ty * 8]);
  float4 a1 = *reinterpret_cast<const float4*>(&A[0][ty * 8 + 4]);
  float4 b0 = *reinterpret_cast<const float4*>(&B[0][tx * 4]);
  float4 b1 = *reinterpret_cast<const float4*>(&B[0][64 + tx * 4]);
#pragma unroll
  for (int kq = 0; kq < kGK; ++kq) {
    float4 a0n = a0, a1n = a1, b0n = b0, b1n = b1;
    if (kq + 1 < kGK) {
      a0n = *reinterpret_cast<const float4*>(&A[kq + 1][ty * 8]);
      a1n = *reinterpret_cast<const float4*>(&A[kq + 1][ty * 8 + 4]);
      b0n = *reinterpret_cast<const float4*>(&B[kq + 1][tx * 4]);
      b1n = *reinterpret_cast<const float4*>(&B[kq + 1][64 + tx * 4]);
    }
    const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
    for (int r = 0; r < 8; ++r)
#pragma unroll
      for (int c = 0; c < 8; ++c) acc[r][c] = fmaf(av[r], bv[c], acc[r][c]);
    a0 = a0n;
    a1 = a1n;
    b0 = b0n;
    b1 = b1n;
  }
}

// column c (0..7) of a thread's tile -> column inside the block's 128
__device__ __forceinline__ int gemm_col(int tx, int c) { return c < 4 ? tx * 4 + c : 64 + tx * 4 + c - 4; }

__device__ __forceinline__ void gemm_zero(float (&acc)[8][8]) {
#pragma unroll
  for (int r = 0; r < 8; ++r)
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[r][c] = 0.f;
}

// forward: out[co][p] = sum_{kk, ci} wt[co][kk][ci] x[n][g cig + ci][t s + kk - pad]  (cig % 16 == 0)
__global__ void __launch_bounds__(kGT, 3) disc_gemm_fwd_kernel(const float* __restrict__ x, const float* __restrict__ wt,
                                                              const float* __restrict__ bias, float* __restrict__ y,
                                                              DLayer L, int N) {
  __shared__ __align__(16) GemmSmem sm;
  const int cig = L.C_in / L.groups, cog = L.C_out / L.groups, K = cig * L.k;
  const int co0 = blockIdx.y * kGM, g = co0 / cog;
  const int p0 = blockIdx.x * kGN, P = N * L.L_out;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  // loader roles: A row akq, columns am + 8 i; B: this thread's position, all 16 rows
  const int akq = tid & 15, am = tid >> 4;
  const int p = p0 + tid;
  const bool live = p < P;
  const int n = live ? p / L.L_out : 0, t = live ? p - n * L.L_out : 0;
  const float* xb = x + ((size_t)n * L.C_in + (size_t)g * cig) * L.L_in;
  const int q0 = t * L.s - L.pad;
  const float* wrow = wt + (size_t)(co0 + am) * K;
  float ra[8], rb[kGK];
  auto load = [&](int k0) {
    const int kk = k0 / cig, ci0 = k0 - kk * cig;
#pragma unroll
    for (int i = 0; i < 8; ++i) ra[i] = __ldg(wrow + (size_t)8 * i * K + k0 + akq);
    const int q = q0 + kk;
    const bool ok = live && q >= 0 && q < L.L_in;
    const float* xq = xb + (size_t)ci0 * L.L_in + q;
#pragma unroll
    for (int i = 0; i < kGK; ++i) rb[i] = ok ? __ldg(xq + (size_t)i * L.L_in) : 0.f;
  };
  auto store = [&](int b) {
#pragma unroll
    for (int i = 0; i < 8; ++i) sm.A[b][akq][am + 8 * i] = ra[i];
#pragma unroll
    for (int i = 0; i < kGK; ++i) sm.B[b][i][tid] = rb[i];
  };
  float acc[8][8];
  gemm_zero(acc);
  load(0);
  store(0);
  __syncthreads();
  int b = 0;
  for (int k0 = 0; k0 < K; k0 += kGK) {
    const bool more = k0 + kGK < K;
    if (more) load(k0 + kGK);
    gemm_chunk(sm.A[b], sm.B[b], ty, tx, acc);
    if (more) store(b ^ 1);
    __syncthreads();
    b ^= 1;
  }
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int pc = p0 + gemm_col(tx, c);
    if (pc >= P) continue;
    const int nc = pc / L.L_out, tc = pc - nc * L.L_out;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int co = co0 + ty * 8 + r;
      float v = acc[r][c] + bias[co];
      if (L.act) v = v > 0.f ? v : v * kSlope;
      y[((size_t)nc * L.C_out + co) * L.L_out + tc] = v;
    }
  }
}

// input gradient, one stride phase r per blockIdx.z: u = r + s v.  Only the taps kk = kk0 + i s
// (kk0 = (r + pad) mod s) reach a whole output position t = v + c_r - i (c_r = (r + pad - kk0) / s), so
// dx[ci][(n, v)] = sum_{i, o} wt[o][kk0 + i s][ci] dz[n][o][v + c_r - i];  K ordered (i, o), cog % 16 == 0.
__global__ void __launch_bounds__(kGT, 3) disc_gemm_dgrad_kernel(const float* __restrict__ dz,
                                                                const float* __restrict__ wt, float* __restrict__ dx,
                                                                DLayer L, int N) {
  __shared__ __align__(16) GemmSmem sm;
  const int cig = L.C_in / L.groups, cog = L.C_out / L.groups;
  const int r = blockIdx.z;
  const int kk0 = (r + L.pad) % L.s, KT = (L.k - kk0 + L.s - 1) / L.s, c_r = (r + L.pad - kk0) / L.s;
  const int V = r < L.L_in ? (L.L_in - r + L.s - 1) / L.s : 0, P = N * V, K = cog * KT;
  const int p0 = blockIdx.x * kGN;
  if (p0 >= P || KT <= 0) return;  // uniform over the block
  const int ci0 = blockIdx.y * kGM, g = ci0 / cig, cl0 = ci0 - g * cig;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  // loader roles: A column am (ci), rows akq + 2 j (o); B: this thread's position, all 16 rows
  const int am = tid & 63, akq = tid >> 6;
  const int p = p0 + tid;
  const bool live = p < P;
  const int n = live ? p / V : 0, v = live ? p - n * V : 0;
  const float* dzb = dz + ((size_t)n * L.C_out + (size_t)g * cog) * L.L_out;
  const int v0 = v + c_r;
  const float* wcol = wt + (size_t)g * cog * L.k * cig + cl0 + am;
  float ra[8], rb[kGK];
  auto load = [&](int k0) {
    const int i = k0 / cog, o0 = k0 - i * cog, kk = kk0 + i * L.s;
#pragma unroll
    for (int j = 0; j < 8; ++j) ra[j] = __ldg(wcol + ((size_t)(o0 + akq + 2 * j) * L.k + kk) * cig);
    const int tt = v0 - i;
    const bool ok = live && tt >= 0 && tt < L.L_out;
    const float* dq = dzb + (size_t)o0 * L.L_out + tt;
#pragma unroll
    for (int j = 0; j < kGK; ++j) rb[j] = ok ? __ldg(dq + (size_t)j * L.L_out) : 0.f;
  };
  auto store = [&](int b) {
#pragma unroll
    for (int j = 0; j < 8; ++j) sm.A[b][akq + 2 * j][am] = ra[j];
#pragma unroll
    for (int j = 0; j < kGK; ++j) sm.B[b][j][tid] = rb[j];
  };
  float acc[8][8];
  gemm_zero(acc);
  load(0);
  store(0);
  __syncthreads();
  int b = 0;
  for (int k0 = 0; k0 < K; k0 += kGK) {
    const bool more = k0 + kGK < K;
    if (more) load(k0 + kGK);
    gemm_chunk(sm.A[b], sm.B[b], ty, tx, acc);
    if (more) store(b ^ 1);
    __syncthreads();
    b ^= 1;
  }
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int pc = p0 + gemm_col(tx, c);
    if (pc >= P) continue;
    const int nc = pc / V, u = r + L.s * (pc - nc * V);
#pragma unroll
    for (int a = 0; a < 8; ++a) dx[((size_t)nc * L.C_in + ci0 + ty * 8 + a) * L.L_in + u] = acc[a][c];
  }
}

// weight gradient of a dense layer: part[z][co][j] = sum_{p in split z} dz[n][co][t] X[p][j],
// j = (ci, kk) or the bias column (X = 1); K = positions, each thread decodes one per chunk
__global__ void __launch_bounds__(kGT, 3) disc_gemm_wgrad_kernel(const float* __restrict__ dz,
                                                                const float* __restrict__ x, float* __restrict__ part,
                                                                DLayer L, int N, int chunk) {
  __shared__ __align__(16) GemmSmem sm;
  __shared__ int coff[kGN], ckk[kGN];
  const int cig = L.C_in / L.groups, cog = L.C_out / L.groups, cols = cig * L.k + 1;
  const int o0 = blockIdx.y * kGM, g = o0 / cog;
  const int c_base = blockIdx.x * kGN;
  const int P = N * L.L_out, p_beg = blockIdx.z * chunk, p_end = min(P, p_beg + chunk);
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  {
    const int col = c_base + tid;
    if (col < cols - 1) {
      const int ci = col / L.k;
      coff[tid] = (g * cig + ci) * L.L_in;
      ckk[tid] = col - ci * L.k;
    } else {
      coff[tid] = 0;
      ckk[tid] = col == cols - 1 ? -1 : -2;  // -1: the bias column (ones), -2: past the end (zeros)
    }
  }
  __syncthreads();
  // loader roles: position kq (both operands); A rows m0 + 8 i (i < 8), B columns m0 + 8 i (i < 16)
  const int kq = tid & 15, m0 = tid >> 4;
  float ra[8], rb[16];
  auto load = [&](int pq0) {
    const int pp = pq0 + kq;
    const bool live = pp < p_end;
    const int n = live ? pp / L.L_out : 0, t = live ? pp - n * L.L_out : 0;
    const float* dzp = dz + (size_t)n * L.C_out * L.L_out + t + (size_t)(o0 + m0) * L.L_out;
#pragma unroll
    for (int i = 0; i < 8; ++i) ra[i] = live ? __ldg(dzp + (size_t)8 * i * L.L_out) : 0.f;
    const float* xp = x + (size_t)n * L.C_in * L.L_in;
    const int q0 = t * L.s - L.pad;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int kk = ckk[m0 + 8 * i];
      float v = 0.f;
      if (live) {
        if (kk == -1) {
          v = 1.f;
        } else if (kk >= 0) {
          const int q = q0 + kk;
          if (q >= 0 && q < L.L_in) v = __ldg(xp + coff[m0 + 8 * i] + q);
        }
      }
      rb[i] = v;
    }
  };
  auto store = [&](int b) {
#pragma unroll
    for (int i = 0; i < 8; ++i) sm.A[b][kq][m0 + 8 * i] = ra[i];
#pragma unroll
    for (int i = 0; i < 16; ++i) sm.B[b][kq][m0 + 8 * i] = rb[i];
  };
  float acc[8][8];
  gemm_zero(acc);
  load(p_beg);
  store(0);
  __syncthreads();
  int b = 0;
  for (int pq0 = p_beg; pq0 < p_end; pq0 += kGK) {
    const bool more = pq0 + kGK < p_end;
    if (more) load(pq0 + kGK);
    gemm_chunk(sm.A[b], sm.B[b], ty, tx, acc);
    if (more) store(b ^ 1);
    __syncthreads();
    b ^= 1;
  }
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int col = c_base + gemm_col(tx, c);
    if (col >= cols) continue;
#pragma unroll
    for (int r = 0; r < 8; ++r) part[((size_t)blockIdx.z * L.C_out + o0 + ty * 8 + r) * cols + col] = acc[r][c];
  }
}

// conv_post (one output channel, no groups): 32 positions per block, the 8 warps take every 8th
// input channel, lanes the positions (coalesced reads along t); partial sums added in warp order
__global__ void __launch_bounds__(256) disc_post_fwd_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                           const float* __restrict__ bias, float* __restrict__ y,
                                                           DLayer L, int N) {
  extern __shared__ float4 smem_f4[];
  float* ws = reinterpret_cast<float*>(smem_f4);  // [C_in * k]
  __shared__ float red[8][32];
  const int K = L.C_in * L.k;
  for (int i = threadIdx.x; i < K; i += 256) ws[i] = w[i];
  __syncthreads();
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  const int p = blockIdx.x * 32 + lane;
  const bool live = p < N * L.L_out;
  const int n = live ? p / L.L_out : 0, t = live ? p - n * L.L_out : 0;
  const float* xn = x + (size_t)n * L.C_in * L.L_in;
  const int q0 = t * L.s - L.pad;
  float acc = 0.f;
  if (live)
    for (int ci = wp; ci < L.C_in; ci += 8)
      for (int kk = 0; kk < L.k; ++kk) {
        const int q = q0 + kk;
        if (q >= 0 && q < L.L_in) acc = fmaf(ws[ci * L.k + kk], __ldg(xn + (size_t)ci * L.L_in + q), acc);
      }
  red[wp][lane] = acc;
  __syncthreads();
  if (wp == 0 && live) {
    float v = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) v += red[i][lane];
    v += bias[0];
    if (L.act) v = v > 0.f ? v : v * kSlope;
    y[(size_t)n * L.L_out + t] = v;
  }
}

// Weight gradient as a GEMM: rows co (a tile of TM inside one group), columns (ci, kk) of the
// group's inputs plus one column of ones (the bias gradient), K = the (n, t) positions of this
// split.  Thread tile RM x RN of a 256-thread block; rows / columns interleaved by TY / TX.
template <int TM, int TN>
__global__ void __launch_bounds__(256) disc_conv_wgrad_kernel(const float* __restrict__ dz, const float* __restrict__ x,
                                                             float* __restrict__ part, DLayer L, int N, int chunk) {
  constexpr int TY = TM < 16 ? TM : 16, TX = 256 / TY, RM = TM / TY, RN = TN / TX, KC = 32;
  static_assert(RM * TY == TM && RN * TX == TN, "tile");
  __shared__ float Ds[KC][TM + 1];
  __shared__ float Xs[KC][TN + 1];
  const int cig = L.C_in / L.groups, cog = L.C_out / L.groups;
  const int cols = cig * L.k + 1;
  const int o0 = blockIdx.y * TM, g = o0 / cog;
  const int c_base = blockIdx.x * TN;
  const int P = N * L.L_out;
  const int p_beg = blockIdx.z * chunk, p_end = min(P, p_beg + chunk);
  const int ty = threadIdx.x / TX, tx = threadIdx.x - ty * TX;
  const float* xg = x + (size_t)g * cig * L.L_in;
  float acc[RM][RN];
#pragma unroll
  for (int r = 0; r < RM; ++r)
#pragma unroll
    for (int c = 0; c < RN; ++c) acc[r][c] = 0.f;
  for (int p0 = p_beg; p0 < p_end; p0 += KC) {
    __syncthreads();
    for (int e = threadIdx.x; e < TM * KC; e += 256) {
      const int m = e / KC, j = e - m * KC, p = p0 + j;
      float v = 0.f;
      if (p < p_end) {
        const int n = p / L.L_out, t = p - n * L.L_out;
        v = dz[((size_t)n * L.C_out + o0 + m) * L.L_out + t];
      }
      Ds[j][m] = v;
    }
    for (int e = threadIdx.x; e < TN * KC; e += 256) {
      const int c = e / KC, j = e - c * KC, p = p0 + j, col = c_base + c;
      float v = 0.f;
      if (p < p_end && col < cols) {
        if (col == cols - 1) {
          v = 1.f;
        } else {
          const int ci = col / L.k, kk = col - ci * L.k;
          const int n = p / L.L_out, t = p - n * L.L_out, q = t * L.s + kk - L.pad;
          if (q >= 0 && q < L.L_in) v = xg[((size_t)n * L.C_in + ci) * L.L_in + q];
        }
      }
      Xs[j][c] = v;
    }
    __syncthreads();
#pragma unroll 4
    for (int j = 0; j < KC; ++j) {
      float a[RM], b[RN];
#pragma unroll
      for (int r = 0; r < RM; ++r) a[r] = Ds[j][ty + r * TY];
#pragma unroll
      for (int c = 0; c < RN; ++c) b[c] = Xs[j][tx + c * TX];
#pragma unroll
      for (int r = 0; r < RM; ++r)
#pragma unroll
        for (int c = 0; c < RN; ++c) acc[r][c] = fmaf(a[r], b[c], acc[r][c]);
    }
  }
#pragma unroll
  for (int r = 0; r < RM; ++r)
#pragma unroll
    for (int c = 0; c < RN; ++c) {
      const int col = c_base + tx + c * TX;
      if (col < cols) part[((size_t)blockIdx.z * L.C_out + o0 + ty + r * TY) * cols + col] = acc[r][c];
    }
}

// Sums the splits in order: dW [C_out][cols - 1] and the bias gradient (last column).
__global__ void disc_wgrad_reduce_kernel(const float* __restrict__ part, int splits, int C_out, int cols,
                                         float* __restrict__ dw, float* __restrict__ db) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= C_out * cols) return;
  const size_t plane = (size_t)C_out * cols;
  float s = 0.f;
  for (int z = 0; z < splits; ++z) s += part[z * plane + i];
  const int o = i / cols, col = i - o * cols;
  if (col == cols - 1) db[o] = s;
  else dw[(size_t)o * (cols - 1) + col] = s;
}

// ------------------------------------------------------------------------------------------------
// weight norm (torch.nn.utils.weight_norm, dim 0): w = g v / ||v||, one block per output row
// ------------------------------------------------------------------------------------------------
template <int NT>
__device__ __forceinline__ float2 block_sum2(float2 v) {
  __shared__ float2 red[NT / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    v.x += __shfl_xor_sync(0xffffffffu, v.x, o);
    v.y += __shfl_xor_sync(0xffffffffu, v.y, o);
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float2 s = red[0];
#pragma unroll
  for (int i = 1; i < NT / 32; ++i) {
    s.x += red[i].x;
    s.y += red[i].y;
  }
  return s;
}

// also writes the tap-major copy wt[o][kk][ci] of the dense layers' GEMM kernels when wt is given
__global__ void __launch_bounds__(128) disc_wn_fwd_kernel(const float* __restrict__ v, const float* __restrict__ g,
                                                          float* __restrict__ w, float* __restrict__ wt, int len,
                                                          int k, int cig) {
  const int o = blockIdx.x;
  const float* vr = v + (size_t)o * len;
  float ss = 0.f;
  for (int i = threadIdx.x; i < len; i += 128) ss = fmaf(vr[i], vr[i], ss);
  ss = block_sum2<128>(make_float2(ss, 0.f)).x;
  const float scale = g[o] / sqrtf(ss);
  for (int i = threadIdx.x; i < len; i += 128) {
    const float val = vr[i] * scale;
    w[(size_t)o * len + i] = val;
    if (wt) {
      const int ci = i / k, kk = i - ci * k;
      wt[(size_t)o * len + kk * cig + ci] = val;
    }
  }
}

// dg = <dW, v> / ||v||;  dv = (g / ||v||) (dW - v <dW, v> / ||v||^2)
__global__ void __launch_bounds__(128) disc_wn_bwd_kernel(const float* __restrict__ v, const float* __restrict__ g,
                                                          const float* __restrict__ dw, float* __restrict__ dg,
                                                          float* __restrict__ dv, int len) {
  const int o = blockIdx.x;
  const float* vr = v + (size_t)o * len;
  const float* dr = dw + (size_t)o * len;
  float ss = 0.f, dot = 0.f;
  for (int i = threadIdx.x; i < len; i += 128) {
    ss = fmaf(vr[i], vr[i], ss);
    dot = fmaf(dr[i], vr[i], dot);
  }
  const float2 s = block_sum2<128>(make_float2(ss, dot));
  const float nrm = sqrtf(s.x);
  const float a = g[o] / nrm, b = a * s.y / s.x;
  if (threadIdx.x == 0) dg[o] = s.y / nrm;
  for (int i = threadIdx.x; i < len; i += 128) dv[(size_t)o * len + i] = a * dr[i] - b * vr[i];
}

// ------------------------------------------------------------------------------------------------
// losses (train/losses.py): per term a partial sum per block, then one ordered final sum
// ------------------------------------------------------------------------------------------------
struct LossTerm {
  const float* a;  // generated (or real for kind 0 of the discriminator loss)
  const float* b;  // real feature map (kind 2)
  int count;
  int kind;        // 0: (1 - a)^2   1: a^2   2: |a - b|
  int out;         // losses[out] += coef * sum
  float coef;      // 1 / count (x 2 for the feature-matching loss)
};

__global__ void __launch_bounds__(256) disc_loss_partial_kernel(const LossTerm* __restrict__ terms,
                                                                double* __restrict__ partial) {
  const LossTerm T = terms[blockIdx.y];
  double s = 0.0;
  for (int i = blockIdx.x * 256 + threadIdx.x; i < T.count; i += kLossBlocks * 256) {
    const float a = T.a[i];
    float v;
    if (T.kind == 0) v = (1.f - a) * (1.f - a);
    else if (T.kind == 1) v = a * a;
    else v = fabsf(a - T.b[i]);
    s += (double)v;
  }
  __shared__ double red[8];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int i = 0; i < 8; ++i) t += red[i];
    partial[blockIdx.y * kLossBlocks + blockIdx.x] = t;
  }
}

__global__ void disc_loss_final_kernel(const LossTerm* __restrict__ terms, int n_terms,
                                       const double* __restrict__ partial, float* __restrict__ losses) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  double acc[4] = {0.0, 0.0, 0.0, 0.0};
  for (int t = 0; t < n_terms; ++t) {
    double s = 0.0;
    for (int b = 0; b < kLossBlocks; ++b) s += partial[t * kLossBlocks + b];
    acc[terms[t].out] += (double)terms[t].coef * s;
  }
  for (int i = 0; i < 4; ++i) losses[i] = (float)acc[i];
}

__device__ __forceinline__ float sgnf(float d) { return (float)((d > 0.f) - (d < 0.f)); }

// gradient at conv_post's output for the discriminator loss: real half -2 (1 - x) / n, generated 2 x / n
__global__ void disc_dpost_d_kernel(const float* __restrict__ x, float* __restrict__ dz, int half, float coef) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 2 * half) return;
  const float v = x[i];
  dz[i] = i < half ? -coef * (1.f - v) : coef * v;
}

// generated half only: generator_loss -2 (1 - x) / n plus the feature-matching term 2 sign(x - x_real) / n
__global__ void disc_dpost_g_kernel(const float* __restrict__ x, float* __restrict__ dz, int half, float coef) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= half) return;
  const float v = x[half + i];
  dz[half + i] = -coef * (1.f - v) + coef * sgnf(v - x[i]);
}

// da (in place) -> dz: adds the feature-matching gradient when a_real is given, then LeakyReLU's
// derivative (1 where the output is positive, the slope elsewhere, as torch takes it at 0)
__global__ void disc_act_grad_kernel(float* __restrict__ d, const float* __restrict__ a,
                                     const float* __restrict__ a_real, int n, float fm_coef) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float v = d[i];
  const float ai = a[i];
  if (a_real) v += fm_coef * sgnf(ai - a_real[i]);
  d[i] = ai > 0.f ? v : v * kSlope;
}

// ------------------------------------------------------------------------------------------------
// inputs: [B][T] real and generated -> 2 B p sequences of H = ceil(T / p) samples; right reflect
// padding (torch 'reflect': x[T + i] = x[T - 2 - i])
// ------------------------------------------------------------------------------------------------
__global__ void disc_input_kernel(const float* __restrict__ y, const float* __restrict__ yh, int B, int T, int p,
                                  int H, float* __restrict__ x0) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 2 * B * p * H) return;
  const int n = i / H, h = i - n * H, b = n / p, w = n - b * p;
  const float* src = b < B ? y + (size_t)b * T : yh + (size_t)(b - B) * T;
  const int idx = h * p + w;
  x0[i] = src[idx < T ? idx : 2 * T - 2 - idx];
}

// adjoint of disc_input_kernel for the generated half: dL/dy_hat[b][t] (+= when accumulate)
__global__ void disc_input_grad_kernel(const float* __restrict__ dx0, int B, int T, int p, int H,
                                       float* __restrict__ dldy, int accumulate) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B * T) return;
  const int b = i / T, t = i - b * T;
  float v = dx0[(size_t)(b * p + t % p) * H + t / p];
  const int j = 2 * T - 2 - t;  // the padded position that mirrors t
  if (t <= T - 2 && j < p * H) v += dx0[(size_t)(b * p + j % p) * H + j / p];
  dldy[i] = accumulate ? dldy[i] + v : v;
}

// ------------------------------------------------------------------------------------------------
// torch.optim.AdamW (amsgrad off): p *= 1 - lr wd; m = lerp(m, g, 1 - b1); v = b2 v + (1 - b2) g^2;
// p -= (lr / bc1) m / (sqrt(v) / sqrt(bc2) + eps)
// ------------------------------------------------------------------------------------------------
__global__ void disc_adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                                  float* __restrict__ v, long long n, float decay, float b1, float b2, float eps,
                                  float step_size, float bc2_sqrt) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float gi = g[i];
  const float mi = fmaf(1.f - b1, gi - m[i], m[i]);
  const float vi = fmaf(1.f - b2, gi * gi, b2 * v[i]);
  m[i] = mi;
  v[i] = vi;
  const float denom = sqrtf(vi) / bc2_sqrt + eps;
  p[i] = p[i] * decay - step_size * (mi / denom);
}

// the all-reduced gradient sum -> the mean over the ranks (torch DDP's averaging)
__global__ void disc_scale_kernel(float* __restrict__ g, long long n, float s) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) g[i] *= s;
}

// ------------------------------------------------------------------------------------------------
// host runtime
// ------------------------------------------------------------------------------------------------
struct Spec {
  int ci, co, k, s, grp, pad;
};
// DiscriminatorS (models.py:981-996) and DiscriminatorP (models.py:1014-1077); conv_post last
constexpr Spec kSpecS[] = {{1, 16, 15, 1, 1, 7},        {16, 64, 41, 4, 4, 20},   {64, 256, 41, 4, 16, 20},
                           {256, 1024, 41, 4, 64, 20},  {1024, 1024, 41, 4, 256, 20},
                           {1024, 1024, 5, 1, 1, 2},    {1024, 1, 3, 1, 1, 1}};
constexpr Spec kSpecP[] = {{1, 32, 5, 3, 1, 2},     {32, 128, 5, 3, 1, 2},     {128, 512, 5, 3, 1, 2},
                           {512, 1024, 5, 3, 1, 2}, {1024, 1024, 5, 1, 1, 2}, {1024, 1, 3, 1, 1, 1}};
constexpr int kPeriodsV1[] = {2, 3, 5, 7, 11, 17};

static bool periods_of(const int* periods, int n_periods, std::vector<int>& out) {
  out.clear();
  if (!periods || n_periods <= 0) {
    out.assign(kPeriodsV1, kPeriodsV1 + 6);
    return true;
  }
  if (n_periods > 16) return false;
  for (int i = 0; i < n_periods; ++i) {
    if (periods[i] < 2 || periods[i] > 64) return false;
    out.push_back(periods[i]);
  }
  return true;
}

static void specs_of(int period, const Spec** s, int* n) {
  *s = period ? kSpecP : kSpecS;
  *n = period ? 6 : 7;
}

struct TensorInfo {
  std::string name;
  int shape[3];
  long long offset, size;
};

static std::vector<TensorInfo> tensor_table(const std::vector<int>& periods) {
  std::vector<TensorInfo> t;
  long long off = 0;
  for (int d = 0; d <= (int)periods.size(); ++d) {
    const Spec* sp;
    int nl;
    specs_of(d ? periods[d - 1] : 0, &sp, &nl);
    for (int li = 0; li < nl; ++li) {
      const std::string base = "discriminators." + std::to_string(d) +
                               (li == nl - 1 ? std::string(".conv_post") : ".convs." + std::to_string(li));
      const int co = sp[li].co, len = sp[li].ci / sp[li].grp * sp[li].k;
      t.push_back({base + ".bias", {co, 1, 1}, off, co});
      off += co;
      t.push_back({base + ".weight_g", {co, 1, 1}, off, co});
      off += co;
      t.push_back({base + ".weight_v", {co, sp[li].ci / sp[li].grp, sp[li].k}, off, (long long)co * len});
      off += (long long)co * len;
    }
  }
  return t;
}

struct LayerRt {
  DLayer L;
  int N = 0;
  int tco = 1, tci = 1, tm = 1, tn = 64;
  int splits = 1, chunk = 0;
  bool gemm_wgrad = false;  // dense layer: disc_gemm_wgrad_kernel (tm = 64 rows x tn = 128 columns)
  bool gemm_fwd = false, gemm_dgrad = false;  // disc_gemm_fwd_kernel / disc_gemm_dgrad_kernel
  long long wt_off = -1;                       // tap-major weight copy of the GEMM kernels
  long long p_bias = 0, p_g = 0, p_v = 0, w_off = 0;
  int len = 0;
  float* a = nullptr;   // output [N][C_out][L_out]
  float* da = nullptr;  // its gradient (then dz in place)
};

struct Net {
  int period = 0, H = 0, N = 0;
  float* x0 = nullptr;
  float* dx0 = nullptr;
  std::vector<LayerRt> layers;
};

static int pick(int n, std::initializer_list<int> opts) {
  for (int o : opts)
    if (n % o == 0) return o;
  return 1;
}

}  // namespace disc
}  // namespace wb

using namespace wb::disc;

struct WubuB200Disc {
  int B = 0, T = 0;
  std::vector<int> periods;
  std::vector<Net> nets;
  long long n_params = 0, n_weff = 0, n_weft = 0;
  float *params = nullptr, *grads = nullptr, *m = nullptr, *v = nullptr, *weff = nullptr, *weft = nullptr;
  float *part = nullptr, *dw = nullptr;
  float *y_dev = nullptr, *yh_dev = nullptr, *dldy_dev = nullptr;
  double* loss_part = nullptr;
  float* losses_dev = nullptr;
  float* losses_host = nullptr;
  LossTerm *terms_d = nullptr, *terms_g = nullptr;
  int n_terms_d = 0, n_terms_g = 0;
  cudaStream_t st = nullptr;
  bool own_stream = false;
  long long step = 0;
  float lr = 1e-4f, b1 = 0.8f, b2 = 0.99f, eps = 1e-9f, wd = 0.01f;
  bool weff_stale = true;
  int launches = 0;
  void* arena = nullptr;
  // data parallelism: the gradient is all-reduced (then averaged) before AdamW
  void* comm = nullptr;
  int rank = 0, world = 1;
  int comm_timeout_ms = 60000;
  bool comm_dead = false;  // aborted after a deadline or an NCCL error: no further step
};

namespace {

int check_launch(WubuB200Disc* d) {
  ++d->launches;
  return cudaGetLastError() == cudaSuccess ? 0 : WUBU_B200_ERR_CUDA;
}

#define DISC_TRY(x)            \
  do {                         \
    const int rc_ = (x);       \
    if (rc_) return rc_;       \
  } while (0)

int launch_fwd(WubuB200Disc* d, const LayerRt& l, const float* in) {
  if (l.L.C_out == 1 && l.L.groups == 1) {
    const size_t smem = (size_t)l.L.C_in * l.L.k * sizeof(float);
    disc_post_fwd_kernel<<<(l.N * l.L.L_out + 31) / 32, 256, smem, d->st>>>(in, d->weff + l.w_off,
                                                                              d->params + l.p_bias, l.a, l.L, l.N);
    return check_launch(d);
  }
  if (l.gemm_fwd) {
    const dim3 g2((l.N * l.L.L_out + kGN - 1) / kGN, l.L.C_out / kGM);
    disc_gemm_fwd_kernel<<<g2, kGT, 0, d->st>>>(in, d->weft + l.wt_off, d->params + l.p_bias, l.a, l.L, l.N);
    return check_launch(d);
  }
  const dim3 grid((l.N * l.L.L_out + kPos - 1) / kPos, l.L.C_out / l.tco);
  const size_t smem = (size_t)l.tco * std::min(kCIC, l.L.C_in / l.L.groups) * l.L.k * sizeof(float);
  const float* w = d->weff + l.w_off;
  const float* b = d->params + l.p_bias;
  switch (l.tco) {
    case 32: disc_conv_fwd_kernel<32><<<grid, kPos, smem, d->st>>>(in, w, b, l.a, l.L, l.N); break;
    case 16: disc_conv_fwd_kernel<16><<<grid, kPos, smem, d->st>>>(in, w, b, l.a, l.L, l.N); break;
    case 4: disc_conv_fwd_kernel<4><<<grid, kPos, smem, d->st>>>(in, w, b, l.a, l.L, l.N); break;
    default: disc_conv_fwd_kernel<1><<<grid, kPos, smem, d->st>>>(in, w, b, l.a, l.L, l.N); break;
  }
  return check_launch(d);
}

// input gradient over n_seq sequences starting at the given (already offset) pointers
int launch_dgrad(WubuB200Disc* d, const LayerRt& l, const float* dz, float* dx, int n_seq) {
  if (l.gemm_dgrad) {
    const int V = (l.L.L_in + l.L.s - 1) / l.L.s;  // positions of the longest phase
    const dim3 g2((n_seq * V + kGN - 1) / kGN, l.L.C_in / kGM, l.L.s);
    disc_gemm_dgrad_kernel<<<g2, kGT, 0, d->st>>>(dz, d->weft + l.wt_off, dx, l.L, n_seq);
    return check_launch(d);
  }
  const dim3 grid((n_seq * l.L.L_in + kPos - 1) / kPos, l.L.C_in / l.tci);
  const size_t smem = (size_t)std::min(kOC, l.L.C_out / l.L.groups) * l.L.k * l.tci * sizeof(float);
  const float* w = d->weff + l.w_off;
  switch (l.tci) {
    case 32: disc_conv_dgrad_kernel<32><<<grid, kPos, smem, d->st>>>(dz, w, dx, l.L, n_seq); break;
    case 4: disc_conv_dgrad_kernel<4><<<grid, kPos, smem, d->st>>>(dz, w, dx, l.L, n_seq); break;
    default: disc_conv_dgrad_kernel<1><<<grid, kPos, smem, d->st>>>(dz, w, dx, l.L, n_seq); break;
  }
  return check_launch(d);
}

// weight, bias and weight-norm (g, v) gradients of one layer from its dz and its input
int launch_wgrad(WubuB200Disc* d, const LayerRt& l, const float* in) {
  const int cols = l.len + 1;
  const dim3 grid((cols + l.tn - 1) / l.tn, l.L.C_out / l.tm, l.splits);
  if (l.gemm_wgrad) {
    disc_gemm_wgrad_kernel<<<grid, kGT, 0, d->st>>>(l.da, in, d->part, l.L, l.N, l.chunk);
  } else switch (l.tm) {
    case 64: disc_conv_wgrad_kernel<64, 64><<<grid, 256, 0, d->st>>>(l.da, in, d->part, l.L, l.N, l.chunk); break;
    case 32: disc_conv_wgrad_kernel<32, 64><<<grid, 256, 0, d->st>>>(l.da, in, d->part, l.L, l.N, l.chunk); break;
    case 16: disc_conv_wgrad_kernel<16, 64><<<grid, 256, 0, d->st>>>(l.da, in, d->part, l.L, l.N, l.chunk); break;
    case 4: disc_conv_wgrad_kernel<4, 256><<<grid, 256, 0, d->st>>>(l.da, in, d->part, l.L, l.N, l.chunk); break;
    default: disc_conv_wgrad_kernel<1, 256><<<grid, 256, 0, d->st>>>(l.da, in, d->part, l.L, l.N, l.chunk); break;
  }
  DISC_TRY(check_launch(d));
  const int n = l.L.C_out * cols;
  disc_wgrad_reduce_kernel<<<(n + 255) / 256, 256, 0, d->st>>>(d->part, l.splits, l.L.C_out, cols, d->dw,
                                                               d->grads + l.p_bias);
  DISC_TRY(check_launch(d));
  disc_wn_bwd_kernel<<<l.L.C_out, 128, 0, d->st>>>(d->params + l.p_v, d->params + l.p_g, d->dw, d->grads + l.p_g,
                                                   d->grads + l.p_v, l.len);
  return check_launch(d);
}

int refresh_weights(WubuB200Disc* d) {
  if (!d->weff_stale) return 0;
  for (auto& net : d->nets)
    for (auto& l : net.layers) {
      disc_wn_fwd_kernel<<<l.L.C_out, 128, 0, d->st>>>(d->params + l.p_v, d->params + l.p_g, d->weff + l.w_off,
                                                       l.wt_off >= 0 ? d->weft + l.wt_off : nullptr, l.len, l.L.k,
                                                       l.L.C_in / l.L.groups);
      DISC_TRY(check_launch(d));
    }
  d->weff_stale = false;
  return 0;
}

int forward(WubuB200Disc* d, const float* y, const float* yh) {
  DISC_TRY(refresh_weights(d));
  for (auto& net : d->nets) {
    const int n = net.N * net.H;
    disc_input_kernel<<<(n + 255) / 256, 256, 0, d->st>>>(y, yh, d->B, d->T, net.period ? net.period : 1, net.H,
                                                        net.x0);
    DISC_TRY(check_launch(d));
    const float* in = net.x0;
    for (auto& l : net.layers) {
      DISC_TRY(launch_fwd(d, l, in));
      in = l.a;
    }
  }
  return 0;
}

int run_losses(WubuB200Disc* d, const LossTerm* terms, int n_terms) {
  disc_loss_partial_kernel<<<dim3(kLossBlocks, n_terms), 256, 0, d->st>>>(terms, d->loss_part);
  DISC_TRY(check_launch(d));
  disc_loss_final_kernel<<<1, 32, 0, d->st>>>(terms, n_terms, d->loss_part, d->losses_dev);
  return check_launch(d);
}

// discriminator loss, its gradient through every layer into the parameter gradients
int backward_d(WubuB200Disc* d) {
  DISC_TRY(run_losses(d, d->terms_d, d->n_terms_d));
  for (auto& net : d->nets) {
    const int nl = (int)net.layers.size();
    LayerRt& post = net.layers[nl - 1];
    const int half = net.N / 2 * post.L.L_out;
    disc_dpost_d_kernel<<<(2 * half + 255) / 256, 256, 0, d->st>>>(post.a, post.da, half, 2.f / (float)half);
    DISC_TRY(check_launch(d));
    for (int li = nl - 1; li >= 0; --li) {
      LayerRt& l = net.layers[li];
      if (l.L.act) {
        const int n = l.N * l.L.C_out * l.L.L_out;
        disc_act_grad_kernel<<<(n + 255) / 256, 256, 0, d->st>>>(l.da, l.a, nullptr, n, 0.f);
        DISC_TRY(check_launch(d));
      }
      const float* in = li ? net.layers[li - 1].a : net.x0;
      DISC_TRY(launch_wgrad(d, l, in));
      if (li) DISC_TRY(launch_dgrad(d, l, l.da, net.layers[li - 1].da, l.N));
    }
  }
  return 0;
}

// generator_loss + feature_loss and their gradient down to the generated waveform (dldy_dev)
int backward_g(WubuB200Disc* d, float* dldy) {
  DISC_TRY(run_losses(d, d->terms_g, d->n_terms_g));
  for (size_t ni = 0; ni < d->nets.size(); ++ni) {
    Net& net = d->nets[ni];
    const int nl = (int)net.layers.size(), hs = net.N / 2;
    LayerRt& post = net.layers[nl - 1];
    const int half = hs * post.L.L_out;
    disc_dpost_g_kernel<<<(half + 255) / 256, 256, 0, d->st>>>(post.a, post.da, half, 2.f / (float)half);
    DISC_TRY(check_launch(d));
    for (int li = nl - 1; li >= 0; --li) {
      LayerRt& l = net.layers[li];
      const size_t off = (size_t)hs * l.L.C_out * l.L.L_out;
      if (l.L.act) {
        const int n = (int)off;
        disc_act_grad_kernel<<<(n + 255) / 256, 256, 0, d->st>>>(l.da + off, l.a + off, l.a, n, 2.f / (float)n);
        DISC_TRY(check_launch(d));
      }
      float* dx = li ? net.layers[li - 1].da + (size_t)hs * l.L.C_in * l.L.L_in : net.dx0 + (size_t)hs * net.H;
      DISC_TRY(launch_dgrad(d, l, l.da + off, dx, hs));
    }
    const int n = d->B * d->T;
    disc_input_grad_kernel<<<(n + 255) / 256, 256, 0, d->st>>>(net.dx0 + (size_t)hs * net.H, d->B, d->T,
                                                              net.period ? net.period : 1, net.H, dldy, ni > 0);
    DISC_TRY(check_launch(d));
  }
  return 0;
}

int adamw(WubuB200Disc* d) {
  d->step += 1;
  const double bc1 = 1.0 - std::pow((double)d->b1, (double)d->step);
  const double bc2 = 1.0 - std::pow((double)d->b2, (double)d->step);
  const long long n = d->n_params;
  disc_adamw_kernel<<<(unsigned)((n + 255) / 256), 256, 0, d->st>>>(
      d->params, d->grads, d->m, d->v, n, 1.f - d->lr * d->wd, d->b1, d->b2, d->eps, (float)(d->lr / bc1),
      (float)std::sqrt(bc2));
  d->weff_stale = true;
  return check_launch(d);
}

int inputs(WubuB200Disc* d, const float* y, const float* yh, int flags, const float** yd, const float** yhd) {
  if (flags & WUBU_B200_DISC_DEVICE) {
    *yd = y;
    *yhd = yh;
    return 0;
  }
  const size_t bytes = (size_t)d->B * d->T * sizeof(float);
  if (cudaMemcpyAsync(d->y_dev, y, bytes, cudaMemcpyHostToDevice, d->st) != cudaSuccess ||
      cudaMemcpyAsync(d->yh_dev, yh, bytes, cudaMemcpyHostToDevice, d->st) != cudaSuccess)
    return WUBU_B200_ERR_CUDA;
  *yd = d->y_dev;
  *yhd = d->yh_dev;
  return 0;
}

// Waits for the context's stream.  With a communicator the wait is bounded: past the deadline (a peer
// that hangs or left mid-step) or on an NCCL error the communicator is aborted, which ends the
// collective waiting on the peer, and the call returns WUBU_B200_ERR_COMM; the context takes no
// further step.
int bounded_sync(WubuB200Disc* d) {
  if (!d->comm) return cudaStreamSynchronize(d->st) == cudaSuccess ? 0 : WUBU_B200_ERR_CUDA;
  const auto t0 = std::chrono::steady_clock::now();
  for (long long spins = 0;; ++spins) {
    const cudaError_t q = cudaStreamQuery(d->st);
    if (q == cudaSuccess) return 0;
    if (q != cudaErrorNotReady) return WUBU_B200_ERR_CUDA;
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
    if (wb::nccl_plain_async_error(d->comm) || ms.count() > d->comm_timeout_ms) {
      fprintf(stderr, "wuburvc_b200: discriminator all-reduce failed or timed out: aborting the communicator\n");
      wb::nccl_plain_abort(d->comm);
      d->comm = nullptr;
      d->comm_dead = true;
      cudaStreamSynchronize(d->st);
      cudaGetLastError();
      return WUBU_B200_ERR_COMM;
    }
    if (spins < 20000) sched_yield();
    else usleep(50);
  }
}

int read_losses(WubuB200Disc* d, float* out, int first, int n) {
  if (!out) return bounded_sync(d);
  if (cudaMemcpyAsync(d->losses_host, d->losses_dev, 4 * sizeof(float), cudaMemcpyDeviceToHost, d->st) != cudaSuccess)
    return WUBU_B200_ERR_CUDA;
  DISC_TRY(bounded_sync(d));
  memcpy(out, d->losses_host + first, n * sizeof(float));
  return 0;
}

}  // namespace

// ------------------------------------------------------------------------------------------------
// C ABI
// ------------------------------------------------------------------------------------------------
extern "C" int wubu_b200_disc_param_count(const int* periods, int n_periods) {
  std::vector<int> per;
  if (!periods_of(periods, n_periods, per)) return WUBU_B200_ERR_ARG;
  return (int)tensor_table(per).size();
}

extern "C" long long wubu_b200_disc_param_total(const int* periods, int n_periods) {
  std::vector<int> per;
  if (!periods_of(periods, n_periods, per)) return WUBU_B200_ERR_ARG;
  const auto t = tensor_table(per);
  return t.back().offset + t.back().size;
}

extern "C" int wubu_b200_disc_param_info(const int* periods, int n_periods, int index, char* name, int name_cap,
                                         int* shape3, long long* offset) {
  std::vector<int> per;
  if (!periods_of(periods, n_periods, per)) return WUBU_B200_ERR_ARG;
  const auto t = tensor_table(per);
  if (index < 0 || index >= (int)t.size()) return WUBU_B200_ERR_ARG;
  const TensorInfo& e = t[index];
  if (name) {
    if (name_cap <= (int)e.name.size()) return WUBU_B200_ERR_ARG;
    memcpy(name, e.name.c_str(), e.name.size() + 1);
  }
  if (shape3) memcpy(shape3, e.shape, sizeof(e.shape));
  if (offset) *offset = e.offset;
  return 0;
}

extern "C" void wubu_b200_disc_destroy(WubuB200Disc* d) {
  if (!d) return;
  if (d->st) cudaStreamSynchronize(d->st);
  if (d->comm) wb::nccl_plain_destroy(d->comm);
  if (d->arena) cudaFree(d->arena);
  if (d->losses_host) cudaFreeHost(d->losses_host);
  if (d->own_stream && d->st) cudaStreamDestroy(d->st);
  delete d;
}

extern "C" WubuB200Disc* wubu_b200_disc_create(int B, int T, const int* periods, int n_periods, void* stream) {
  std::vector<int> per;
  if (B < 1 || B > 4096 || T < 128 || T > (1 << 22) || !periods_of(periods, n_periods, per)) return nullptr;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  auto* d = new WubuB200Disc;
  d->B = B;
  d->T = T;
  d->periods = per;
  const auto tab = tensor_table(per);
  d->n_params = tab.back().offset + tab.back().size;
  // plan: shapes, kernel tiles, weight-gradient splits, and the arena's float counts
  size_t act_floats = 0, part_cap = 0, dw_cap = 0;
  int ti = 0, n_terms_g = 0;
  for (int di = 0; di <= (int)per.size(); ++di) {
    Net net;
    net.period = di ? per[di - 1] : 0;
    const int p = net.period ? net.period : 1;
    net.H = (T + p - 1) / p;
    net.N = 2 * B * p;
    if ((long long)net.N * net.H > (1LL << 30)) {
      delete d;
      return nullptr;
    }
    act_floats += 2 * (size_t)net.N * net.H;  // x0, dx0
    const Spec* sp;
    int nl;
    specs_of(net.period, &sp, &nl);
    int L_in = net.H;
    for (int li = 0; li < nl; ++li) {
      LayerRt l;
      const int L_out = (L_in + 2 * sp[li].pad - sp[li].k) / sp[li].s + 1;
      // element counts and (n, t) positions are int inside the kernels
      if (L_out < 1 || (long long)net.N * sp[li].co * L_out >= (1LL << 31)) {
        delete d;
        return nullptr;
      }
      l.L = {sp[li].ci, sp[li].co, sp[li].k, sp[li].s, sp[li].grp, sp[li].pad, L_in, L_out, li < nl - 1 ? 1 : 0};
      l.N = net.N;
      const int cig = sp[li].ci / sp[li].grp, cog = sp[li].co / sp[li].grp;
      l.tco = pick(cog, {32, 16, 4});
      l.tci = pick(cig, {32, 4});
      l.tm = pick(cog, {64, 32, 16, 4});
      l.tn = l.tm >= 16 ? 64 : 256;
      if (cog % kGM == 0) {
        l.gemm_wgrad = true;
        l.tm = kGM;
        l.tn = kGN;
      }
      l.gemm_fwd = cog % kGM == 0 && cig % kGK == 0;
      l.gemm_dgrad = cig % kGM == 0 && cog % kGK == 0;
      l.len = cig * sp[li].k;
      if (l.gemm_fwd || l.gemm_dgrad) {
        l.wt_off = d->n_weft;
        d->n_weft += (long long)sp[li].co * l.len;
      }
      l.p_bias = tab[ti].offset;
      l.p_g = tab[ti + 1].offset;
      l.p_v = tab[ti + 2].offset;
      ti += 3;
      l.w_off = d->n_weff;
      d->n_weff += (long long)sp[li].co * l.len;
      const int cols = l.len + 1, P = l.N * L_out;
      const int base = (cols + l.tn - 1) / l.tn * (sp[li].co / l.tm);
      int splits = std::max(1, std::min(592 / base, P / 256));
      l.chunk = ((P + splits - 1) / splits + 31) / 32 * 32;
      l.splits = (P + l.chunk - 1) / l.chunk;
      part_cap = std::max(part_cap, (size_t)l.splits * sp[li].co * cols);
      dw_cap = std::max(dw_cap, (size_t)sp[li].co * l.len);
      act_floats += 2 * (size_t)l.N * sp[li].co * L_out;
      net.layers.push_back(l);
      L_in = L_out;
    }
    n_terms_g += 1 + nl;
    d->nets.push_back(std::move(net));
  }
  d->n_terms_d = 2 * (int)d->nets.size();
  d->n_terms_g = n_terms_g;
  // one arena: 256-byte aligned pieces
  size_t bytes = 0;
  auto take = [&](size_t b) {
    const size_t o = bytes;
    bytes += (b + 255) / 256 * 256;
    return o;
  };
  const size_t np = (size_t)d->n_params * sizeof(float);
  const size_t o_params = take(np), o_grads = take(np), o_m = take(np), o_v = take(np);
  const size_t o_weff = take((size_t)d->n_weff * sizeof(float));
  const size_t o_weft = take((size_t)std::max(d->n_weft, 1LL) * sizeof(float));
  const size_t o_part = take(part_cap * sizeof(float)), o_dw = take(dw_cap * sizeof(float));
  const size_t bt = (size_t)B * T * sizeof(float);
  const size_t o_y = take(bt), o_yh = take(bt), o_dldy = take(bt);
  const int max_terms = std::max(d->n_terms_d, d->n_terms_g);
  const size_t o_lp = take((size_t)max_terms * kLossBlocks * sizeof(double));
  const size_t o_l = take(4 * sizeof(float));
  const size_t o_td = take(d->n_terms_d * sizeof(LossTerm)), o_tg = take(d->n_terms_g * sizeof(LossTerm));
  const size_t o_act = take(act_floats * sizeof(float));
  if (cudaMalloc(&d->arena, bytes) != cudaSuccess) {
    d->arena = nullptr;
    cudaGetLastError();
    wubu_b200_disc_destroy(d);
    return nullptr;
  }
  char* A = static_cast<char*>(d->arena);
  d->params = reinterpret_cast<float*>(A + o_params);
  d->grads = reinterpret_cast<float*>(A + o_grads);
  d->m = reinterpret_cast<float*>(A + o_m);
  d->v = reinterpret_cast<float*>(A + o_v);
  d->weff = reinterpret_cast<float*>(A + o_weff);
  d->weft = reinterpret_cast<float*>(A + o_weft);
  d->part = reinterpret_cast<float*>(A + o_part);
  d->dw = reinterpret_cast<float*>(A + o_dw);
  d->y_dev = reinterpret_cast<float*>(A + o_y);
  d->yh_dev = reinterpret_cast<float*>(A + o_yh);
  d->dldy_dev = reinterpret_cast<float*>(A + o_dldy);
  d->loss_part = reinterpret_cast<double*>(A + o_lp);
  d->losses_dev = reinterpret_cast<float*>(A + o_l);
  d->terms_d = reinterpret_cast<LossTerm*>(A + o_td);
  d->terms_g = reinterpret_cast<LossTerm*>(A + o_tg);
  float* act = reinterpret_cast<float*>(A + o_act);
  std::vector<LossTerm> td, tg;
  for (auto& net : d->nets) {
    net.x0 = act;
    act += (size_t)net.N * net.H;
    net.dx0 = act;
    act += (size_t)net.N * net.H;
    const int hs = net.N / 2;
    for (auto& l : net.layers) {
      const size_t n = (size_t)l.N * l.L.C_out * l.L.L_out;
      l.a = act;
      act += n;
      l.da = act;
      act += n;
    }
    const LayerRt& post = net.layers.back();
    const int half = hs * post.L.L_out;
    td.push_back({post.a, nullptr, half, 0, 0, 1.f / half});
    td.push_back({post.a + half, nullptr, half, 1, 0, 1.f / half});
    tg.push_back({post.a + half, nullptr, half, 0, 1, 1.f / half});
    for (auto& l : net.layers) {
      const int c = hs * l.L.C_out * l.L.L_out;
      tg.push_back({l.a + c, l.a, c, 2, 2, 2.f / c});
    }
  }
  bool ok = cudaMemset(d->arena, 0, bytes) == cudaSuccess &&
            cudaMemcpy(d->terms_d, td.data(), td.size() * sizeof(LossTerm), cudaMemcpyHostToDevice) == cudaSuccess &&
            cudaMemcpy(d->terms_g, tg.data(), tg.size() * sizeof(LossTerm), cudaMemcpyHostToDevice) == cudaSuccess &&
            cudaMallocHost(&d->losses_host, 4 * sizeof(float)) == cudaSuccess;
  if (ok) {
    if (stream) {
      d->st = static_cast<cudaStream_t>(stream);
    } else {
      ok = cudaStreamCreateWithFlags(&d->st, cudaStreamNonBlocking) == cudaSuccess;
      d->own_stream = ok;
    }
  }
  if (!ok) {
    cudaGetLastError();
    wubu_b200_disc_destroy(d);
    return nullptr;
  }
  return d;
}

extern "C" long long wubu_b200_disc_n_params(const WubuB200Disc* d) { return d ? d->n_params : WUBU_B200_ERR_ARG; }

static int copy_flat(WubuB200Disc* d, float* dev, const float* src_host, float* dst_host) {
  if (!d || !(src_host || dst_host)) return WUBU_B200_ERR_ARG;
  const size_t bytes = (size_t)d->n_params * sizeof(float);
  const cudaError_t e = src_host ? cudaMemcpyAsync(dev, src_host, bytes, cudaMemcpyHostToDevice, d->st)
                                 : cudaMemcpyAsync(dst_host, dev, bytes, cudaMemcpyDeviceToHost, d->st);
  if (e != cudaSuccess || cudaStreamSynchronize(d->st) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  return 0;
}

extern "C" int wubu_b200_disc_set_params(WubuB200Disc* d, const float* host_flat) {
  if (!d || !host_flat) return WUBU_B200_ERR_ARG;
  d->weff_stale = true;
  return copy_flat(d, d->params, host_flat, nullptr);
}
extern "C" int wubu_b200_disc_get_params(WubuB200Disc* d, float* host_flat) {
  return d ? copy_flat(d, d->params, nullptr, host_flat) : WUBU_B200_ERR_ARG;
}
extern "C" int wubu_b200_disc_get_grads(WubuB200Disc* d, float* host_flat) {
  return d ? copy_flat(d, d->grads, nullptr, host_flat) : WUBU_B200_ERR_ARG;
}

extern "C" int wubu_b200_disc_set_adamw(WubuB200Disc* d, float lr, float b1, float b2, float eps, float wd) {
  if (!d || !(lr >= 0.f) || !(b1 >= 0.f && b1 < 1.f) || !(b2 >= 0.f && b2 < 1.f) || !(eps >= 0.f) || !(wd >= 0.f))
    return WUBU_B200_ERR_ARG;
  d->lr = lr;
  d->b1 = b1;
  d->b2 = b2;
  d->eps = eps;
  d->wd = wd;
  return 0;
}

extern "C" int wubu_b200_disc_step(WubuB200Disc* d, const float* y, const float* y_hat, int flags, float* loss_d) {
  if (!d || !y || !y_hat || (flags & ~(WUBU_B200_DISC_DEVICE | WUBU_B200_DISC_NO_UPDATE))) return WUBU_B200_ERR_ARG;
  if (d->comm_dead) return WUBU_B200_ERR_COMM;
  d->launches = 0;
  const float *yd, *yhd;
  DISC_TRY(inputs(d, y, y_hat, flags, &yd, &yhd));
  DISC_TRY(forward(d, yd, yhd));
  DISC_TRY(backward_d(d));
  if (d->comm) {
    DISC_TRY(wb::nccl_plain_allreduce_sum(d->comm, d->grads, (size_t)d->n_params, d->st));
    disc_scale_kernel<<<(unsigned)((d->n_params + 255) / 256), 256, 0, d->st>>>(d->grads, d->n_params,
                                                                                1.f / (float)d->world);
    DISC_TRY(check_launch(d));
  }
  if (!(flags & WUBU_B200_DISC_NO_UPDATE)) DISC_TRY(adamw(d));
  if (loss_d || !(flags & WUBU_B200_DISC_DEVICE)) return read_losses(d, loss_d, 0, 1);
  return 0;
}

extern "C" int wubu_b200_disc_gen_loss(WubuB200Disc* d, const float* y, const float* y_hat, float* dldy_hat,
                                       int flags, float* losses2) {
  if (!d || !y || !y_hat || !dldy_hat || (flags & ~WUBU_B200_DISC_DEVICE)) return WUBU_B200_ERR_ARG;
  if (d->comm_dead) return WUBU_B200_ERR_COMM;
  d->launches = 0;
  const float *yd, *yhd;
  DISC_TRY(inputs(d, y, y_hat, flags, &yd, &yhd));
  DISC_TRY(forward(d, yd, yhd));
  const bool dev = flags & WUBU_B200_DISC_DEVICE;
  DISC_TRY(backward_g(d, dev ? dldy_hat : d->dldy_dev));
  if (!dev && cudaMemcpyAsync(dldy_hat, d->dldy_dev, (size_t)d->B * d->T * sizeof(float), cudaMemcpyDeviceToHost,
                              d->st) != cudaSuccess)
    return WUBU_B200_ERR_CUDA;
  if (losses2 || !dev) return read_losses(d, losses2, 1, 2);
  return 0;
}

extern "C" void* wubu_b200_disc_stream(WubuB200Disc* d) { return d ? (void*)d->st : nullptr; }

extern "C" int wubu_b200_disc_sync(WubuB200Disc* d) {
  if (!d) return WUBU_B200_ERR_ARG;
  return bounded_sync(d);
}

extern "C" int wubu_b200_disc_attach_comm(WubuB200Disc* d, int rank, int world, const void* id128) {
  if (!d || world < 1 || rank < 0 || rank >= world || (world > 1 && !id128) || d->comm) return WUBU_B200_ERR_ARG;
  d->rank = rank;
  d->world = world;
  if (world == 1) return 0;
  DISC_TRY(wb::nccl_plain_init(&d->comm, rank, world, id128));
  d->comm_dead = false;
  return 0;
}

extern "C" int wubu_b200_disc_set_comm_timeout_ms(WubuB200Disc* d, int ms) {
  if (!d || ms <= 0) return WUBU_B200_ERR_ARG;
  d->comm_timeout_ms = ms;
  return 0;
}

extern "C" int wubu_b200_disc_launches(const WubuB200Disc* d) { return d ? d->launches : WUBU_B200_ERR_ARG; }
