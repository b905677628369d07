// api_noalloc.cu — the Conv1d weight gradient without any device allocation.
//
// wubu_b200_conv1d_wgrad allocates its split-K partial buffer and error word with cudaMalloc on
// every call.  Some callers cannot do that: a host whose device memory is entirely owned by its own
// allocator (a framework's caching allocator that has reserved the HBM), or a host that forbids
// allocation inside its processing callback, because cudaMalloc / cudaFree take the driver's locks
// and cudaFree may synchronise the whole device.  For them this variant keeps its scratch in a
// file-scope __device__ array of fixed size, present on every GPU that loads the library until the
// process exits.  The call still waits for its own stream to finish (it reads back the kernels'
// error word before returning).
#include <mutex>

#include "../../include/wuburvc_b200.h"
#include "conv_plan.h"

namespace wb {

namespace {

// Split-K partials (floats) available to one call; the first 64 floats hold the error word.
constexpr size_t kNoAllocPartFloats = (size_t)4 << 20;  // 16 MiB
constexpr size_t kNoAllocHeadFloats = 64;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocHeadFloats + kNoAllocPartFloats];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
float* g_dev_scratch[kMaxDevices] = {};

// Device address of the scratch array on the current device (the host-side symbol is only a
// stand-in).  Resolved once per device, with that device current.
float* scratch_address(int* rc) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *rc = WUBU_B200_ERR_CUDA;
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_dev_scratch[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      fprintf(stderr, "wuburvc_b200: cudaGetSymbolAddress of the no-alloc scratch failed: %s\n",
              cudaGetErrorString(e));
      *rc = WUBU_B200_ERR_CUDA;
      return nullptr;
    }
    g_dev_scratch[dev] = static_cast<float*>(p);
  }
  return g_dev_scratch[dev];
}

// dw[oc][ic][tap] = sum over splits of part[split][tap * C_out + oc][ic] (fixed order).  A block owns
// one output channel and 32 input channels: it reads each tap's 32 partials as one coalesced row
// (ic fastest, as the weight-gradient kernel wrote them), sums the splits, and writes the
// transposed [ic][tap] tile to dw as one contiguous run through shared memory.
constexpr int kReduceIc = 32;
constexpr int kReduceMaxTaps = 256;

__global__ void noalloc_wgrad_reduce_kernel(const float* __restrict__ part, int splits, long long ld, int c_out,
                                            int c_in, int k, float* __restrict__ dw) {
  extern __shared__ float tile[];  // [kReduceIc][k]
  const int oc = blockIdx.y;
  const int ic0 = blockIdx.x * kReduceIc;
  const int nic = min(kReduceIc, c_in - ic0);
  for (int idx = threadIdx.x; idx < k * kReduceIc; idx += blockDim.x) {
    const int tap = idx / kReduceIc, icl = idx % kReduceIc;
    if (icl >= nic) continue;
    const long long src = ((long long)tap * c_out + oc) * c_in + ic0 + icl;
    float s = 0.f;
    for (int sp = 0; sp < splits; ++sp) s += part[(long long)sp * ld + src];
    tile[icl * k + tap] = s;
  }
  __syncthreads();
  float* out = dw + ((long long)oc * c_in + ic0) * k;
  for (int j = threadIdx.x; j < nic * k; j += blockDim.x) out[j] = tile[j];
}

}  // namespace

}  // namespace wb

using namespace wb;

extern "C" int wubu_b200_conv1d_wgrad_noalloc(const void* dy, const void* x, float* dw, int B, int C_in, int T,
                                              int C_out, int k, int dil, int pad, void* stream) {
  if (!dy || !x || !dw || B < 1 || T < 1 || k < 1 || C_in < 1 || C_out < 1) return WUBU_B200_ERR_ARG;
  if (k > kReduceMaxTaps || C_out > 65535) return WUBU_B200_ERR_SHAPE;
  int rc = WUBU_B200_OK;
  float* base = scratch_address(&rc);
  if (!base) return rc;
  int* err = reinterpret_cast<int*>(base);
  float* part = base + kNoAllocHeadFloats;
  cudaStream_t st = (cudaStream_t)stream;
  ConvGeom g{B, T, T + 2 * pad - dil * (k - 1), C_in, C_out, k, dil, pad};
  WgradLaunch L;
  // shape check with unlimited scratch, then fit the split count into the fixed scratch
  if (!plan_wgrad(L, g, dy, x, part, ~size_t(0), 296, err)) return WUBU_B200_ERR_SHAPE;
  const size_t per_split = (size_t)L.p.n_mtiles * 128 * L.p.n_total;
  if (wgrad_part_floats(L) > kNoAllocPartFloats) {
    const int max_splits = (int)(kNoAllocPartFloats / per_split);
    if (max_splits < 1) {
      fprintf(stderr,
              "wuburvc_b200: conv1d_wgrad_noalloc needs %zu floats of scratch per split, more than the %zu it "
              "holds (C_out*k*C_in too large)\n",
              per_split, kNoAllocPartFloats);
      return WUBU_B200_ERR_SHAPE;
    }
    const int base_ctas = (int)(L.grid.x * L.grid.z);
    if (!plan_wgrad(L, g, dy, x, part, kNoAllocPartFloats, max_splits * base_ctas, err)) return WUBU_B200_ERR_SHAPE;
  }
  // the error word must start at zero; the partials are fully overwritten by every call
  if (cudaMemsetAsync(err, 0, sizeof(int), st) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  if (L.run(st) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  const dim3 rgrid((unsigned)((C_in + kReduceIc - 1) / kReduceIc), (unsigned)C_out);
  noalloc_wgrad_reduce_kernel<<<rgrid, 128, (size_t)kReduceIc * k * sizeof(float), st>>>(
      part, L.splits, (long long)per_split, C_out, C_in, k, dw);
  if (cudaGetLastError() != cudaSuccess) return WUBU_B200_ERR_CUDA;
  int h = 0;
  if (cudaMemcpyAsync(&h, err, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  return h ? WUBU_B200_ERR_TIMEOUT : WUBU_B200_OK;
}
