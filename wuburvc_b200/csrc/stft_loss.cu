// stft_loss.cu — multi-scale STFT spectral loss (linear + log magnitude) and its gradient, the
// reference's wubu_stft_loss_grad (src/wubu_train.c:318-446) for B signal pairs at once.
//
// Per scale w in (512, 256, 128)[:n_scales] (hop w/4, Hann window 0.5 - 0.5 cos(2 pi i / (w-1)),
// n_frames = max(1, (n - w) / hop + 1)), per frame:
//   X[k] = sum_t x[t] win[t] e^{-2 pi i k t / w}, k = 0..w/2, for both signals;
//   frame loss = 0.5 (sum_k |ma - mb| + sum_k |log(ma + 1e-10) - log(mb + 1e-10)|) / (w/2 + 1), k >= 1;
//   dm_k = 0.5 (sgn(ma - mb) + clamp(sgn(la - lb) / la, +-10)) / ((w/2 + 1) n_frames n_scales);
//   dL/dx[start + t] += win[t] sum_{k>=1} dm_k (Re_k cos th + Im_k sin th) / ma_k,  th = -2 pi k t / w
//                     = win[t] Re( sum_k Z_k e^{+2 pi i k t / w} ),  Z_k = dm_k (Re_k + i Im_k) / ma_k.
// The reference evaluates both sums as direct DFTs; here both are radix-2 FFTs of the frame in
// shared memory (one block per frame and item), which gives the same values with less rounding.
// Frame gradients go to a scratch buffer and are overlap-added per sample in a fixed order (scale,
// then frame), and the losses are summed in a fixed order, so results are deterministic.
#include "common.cuh"

namespace wb {

namespace {

constexpr int kStftThreads = 256;
constexpr int kStftScales = 3;
__host__ __device__ constexpr int stft_w(int q) { return 512 >> q; }  // window of scale q

__device__ __forceinline__ float stft_warp_sum(float v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// In-place radix-2 FFT of W points (re, im in shared memory, natural order in and out):
// sign = -1 forward (e^{-2 pi i k t / W}), +1 inverse without normalisation.
template <int W>
__device__ void fft_smem(float* re, float* im, float sign) {
  constexpr int LOG = W == 512 ? 9 : W == 256 ? 8 : 7;
  // bit-reversal permutation
  for (int i = threadIdx.x; i < W; i += kStftThreads) {
    const int j = (int)(__brev((unsigned)i) >> (32 - LOG));
    if (i < j) {
      const float r = re[i], m = im[i];
      re[i] = re[j];
      im[i] = im[j];
      re[j] = r;
      im[j] = m;
    }
  }
  __syncthreads();
  for (int len = 2; len <= W; len <<= 1) {
    const int half = len >> 1;
    for (int j = threadIdx.x; j < W / 2; j += kStftThreads) {
      const int pos = j & (half - 1);
      const int i0 = (j - pos) * 2 + pos, i1 = i0 + half;
      float sn, cs;
      sincospif(sign * 2.0f * (float)pos / (float)len, &sn, &cs);
      const float tr = re[i1] * cs - im[i1] * sn, ti = re[i1] * sn + im[i1] * cs;
      re[i1] = re[i0] - tr;
      im[i1] = im[i0] - ti;
      re[i0] += tr;
      im[i0] += ti;
    }
    __syncthreads();
  }
}

// One block per (frame, item): spectra of both signals, the frame's loss, the frame's gradient.
template <int W>
__global__ void __launch_bounds__(kStftThreads) stft_frame_kernel(const float* __restrict__ a,
                                                                   const float* __restrict__ b, int n,
                                                                   int n_frames, float scale_div,
                                                                   float* __restrict__ frame_loss,
                                                                   float* __restrict__ frame_grad) {
  constexpr int NB = W / 2 + 1, HOP = W / 4;
  __shared__ float win[W], ra[W], ia[W], rb[W], ib[W];
  __shared__ float red[2][kStftThreads / 32];
  const int f = blockIdx.x, item = blockIdx.y, tid = threadIdx.x;
  const int start = f * HOP;
  const float* sa = a + (size_t)item * n;
  const float* sb = b + (size_t)item * n;
  for (int i = tid; i < W; i += kStftThreads) {
    // the window exactly as the reference forms it, in single precision
    const float wv = 0.5f - 0.5f * cosf(2.0f * 3.14159265358979f * (float)i / (float)(W - 1));
    const int idx = start + i;
    win[i] = wv;
    ra[i] = (idx < n ? sa[idx] : 0.f) * wv;
    rb[i] = (idx < n ? sb[idx] : 0.f) * wv;
    ia[i] = 0.f;
    ib[i] = 0.f;
  }
  __syncthreads();
  fft_smem<W>(ra, ia, -1.f);
  fft_smem<W>(rb, ib, -1.f);
  // bins k = 1..W/2: loss terms and the gradient coefficients Z_k (into rb / ib), other entries zero
  float dl = 0.f, dg = 0.f;
  const float norm = (float)NB * (float)n_frames * scale_div;
  for (int k = tid; k < W; k += kStftThreads) {
    float zr = 0.f, zi = 0.f;
    if (k >= 1 && k < NB) {
      const float xr = ra[k], xi = ia[k];
      const float ma = sqrtf(xr * xr + xi * xi), mb = sqrtf(rb[k] * rb[k] + ib[k] * ib[k]);
      const float la = ma + 1e-10f, lb = mb + 1e-10f;
      dl += fabsf(ma - mb);
      dg += fabsf(logf(la) - logf(lb));
      const float dlog = fminf(fmaxf((la > lb ? 1.f : -1.f) / la, -10.f), 10.f);
      const float dm = 0.5f * ((ma > mb ? 1.f : -1.f) + dlog) / norm;
      if (ma > 1e-12f) {
        zr = dm * xr / ma;
        zi = dm * xi / ma;
      }
    }
    rb[k] = zr;  // the second signal's spectrum is no longer needed
    ib[k] = zi;
  }
  dl = stft_warp_sum(dl);
  dg = stft_warp_sum(dg);
  if ((tid & 31) == 0) {
    red[0][tid >> 5] = dl;
    red[1][tid >> 5] = dg;
  }
  __syncthreads();
  if (tid == 0) {
    float s0 = 0.f, s1 = 0.f;
    for (int w = 0; w < kStftThreads / 32; ++w) {
      s0 += red[0][w];
      s1 += red[1][w];
    }
    frame_loss[(size_t)item * n_frames + f] = 0.5f * (s0 / (float)NB + s1 / (float)NB);
  }
  fft_smem<W>(rb, ib, 1.f);
  float* g = frame_grad + ((size_t)item * n_frames + f) * W;
  for (int t = tid; t < W; t += kStftThreads) g[t] = rb[t] * win[t];
}

struct StftScales {
  const float* grad[kStftScales];  // [B][n_frames][w]
  const float* loss[kStftScales];  // [B][n_frames]
  int n_frames[kStftScales];
  int n_scales;                    // scales evaluated (at most 3)
  float divisor;                   // the requested scale count (the reference divides by it)
};

// dL/da[item][i]: the frames covering sample i, scale by scale, frame by frame (fixed order)
__global__ void stft_overlap_add_kernel(StftScales s, int n, float* __restrict__ grad) {
  const int item = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float acc = 0.f;
  for (int q = 0; q < s.n_scales; ++q) {
    const int w = stft_w(q), hop = w / 4, nf = s.n_frames[q];
    // frames f with f*hop <= i < f*hop + w
    int f0 = i >= w ? (i - w) / hop + 1 : 0;
    const int f1 = min(nf - 1, i / hop);
    for (int f = f0; f <= f1; ++f) acc += s.grad[q][((size_t)item * nf + f) * w + (i - f * hop)];
  }
  grad[(size_t)item * n + i] = acc;
}

// loss[item] = sum over scales of (sum over frames of the frame loss) / n_frames, / n_scales
__global__ void stft_loss_sum_kernel(StftScales s, float* __restrict__ loss) {
  const int item = blockIdx.x, lane = threadIdx.x;
  float total = 0.f;
  for (int q = 0; q < s.n_scales; ++q) {
    const int nf = s.n_frames[q];
    float acc = 0.f;
    for (int f = lane; f < nf; f += 32) acc += s.loss[q][(size_t)item * nf + f];
    acc = stft_warp_sum(acc);
    total += acc / (float)nf;
  }
  if (lane == 0) loss[item] = total / s.divisor;
}

}  // namespace

int stft_frames(int n, int w) { return n >= w ? (n - w) / (w / 4) + 1 : 1; }

// Scratch: per scale B * n_frames floats of frame losses and B * n_frames * w of frame gradients.
size_t stft_scratch_floats(int B, int n, int n_scales) {
  if (n_scales <= 0) n_scales = 3;
  size_t t = 0;
  for (int q = 0; q < n_scales && q < kStftScales; ++q) {
    const int nf = stft_frames(n, stft_w(q));
    t += (size_t)B * nf * (stft_w(q) + 1);
  }
  return t;
}

// n_scales <= 0 means 3; more than 3 evaluates 3 but divides by the count given (as the reference)
cudaError_t stft_loss_grad(const float* a, const float* b, int B, int n, int n_scales, float* grad, float* loss,
                           float* scratch, cudaStream_t st) {
  if (n_scales <= 0) n_scales = 3;
  StftScales s{};
  s.n_scales = n_scales < kStftScales ? n_scales : kStftScales;
  s.divisor = (float)n_scales;
  float* p = scratch;
  for (int q = 0; q < s.n_scales; ++q) {
    const int w = stft_w(q), nf = stft_frames(n, w);
    s.n_frames[q] = nf;
    float* fl = p;
    float* fg = p + (size_t)B * nf;
    p = fg + (size_t)B * nf * w;
    s.loss[q] = fl;
    s.grad[q] = fg;
    const dim3 grid((unsigned)nf, (unsigned)B);
    if (w == 512) stft_frame_kernel<512><<<grid, kStftThreads, 0, st>>>(a, b, n, nf, s.divisor, fl, fg);
    else if (w == 256) stft_frame_kernel<256><<<grid, kStftThreads, 0, st>>>(a, b, n, nf, s.divisor, fl, fg);
    else stft_frame_kernel<128><<<grid, kStftThreads, 0, st>>>(a, b, n, nf, s.divisor, fl, fg);
  }
  stft_overlap_add_kernel<<<dim3((unsigned)((n + 255) / 256), (unsigned)B), 256, 0, st>>>(s, n, grad);
  stft_loss_sum_kernel<<<B, 32, 0, st>>>(s, loss);
  return cudaGetLastError();
}

}  // namespace wb
