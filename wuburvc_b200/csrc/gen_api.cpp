// gen_api.cpp — C ABI of the generator training context.
#include <cstdio>
#include <cstring>
#include <vector>

#include "gen_model.h"

namespace wb {
bool gen_setup(Gen& m);
bool gen_forward(Gen& m);
bool gen_backward(Gen& m);
bool gen_adamw(Gen& m, float grad_scale, int bump_noise);
void gen_free(Gen& m);
bool gen_set_operand_format(Gen& m, int bf16);
bool gen_set_forward_only(Gen& m, int on);
int comm_attach(Gen& m, int rank, int world, const void* id128);
int comm_unique_id(void* out128);
int comm_world(Gen& m);
int comm_sync(Gen& m);
bool comm_aborted(Gen& m);
int comm_set_timeout(Gen& m, int ms);
}  // namespace wb

using namespace wb;

struct WubuB200Gen {
  Gen m;
};

namespace {

int check_err(Gen& m) {
  if (comm_world(m) > 1) {  // data parallel: bounded wait on the collectives (comm.cpp)
    const int rc = comm_sync(m);
    if (rc) return rc;
  }
  cudaError_t e = cudaStreamSynchronize(m.stream);
  if (e != cudaSuccess) {
    fprintf(stderr, "wuburvc_b200: CUDA error: %s\n", cudaGetErrorString(e));
    return WUBU_B200_ERR_CUDA;
  }
  int h = 0;
  if (cudaMemcpy(&h, m.err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  if (h) {
    cudaMemset(m.err, 0, sizeof(int));
    if (h == ERR_RANGE) {
      fprintf(stderr, "wuburvc_b200: a forward operand (activation, weight or z) reached 65504, the limit of "
                      "the fp16 operand split\n");
      return WUBU_B200_ERR_RANGE;
    }
    fprintf(stderr, "wuburvc_b200: a kernel's bounded wait expired (code %d)\n", h);
    return WUBU_B200_ERR_TIMEOUT;
  }
  return WUBU_B200_OK;
}

// After a range error (a forward operand reached the fp16 limit of the operand split; the step's
// update was skipped on the device) the context switches to the bf16 pair format for good.  Returns
// true when the caller should recompute the step.
bool range_fallback(Gen& m, int rc) {
  if (rc != WUBU_B200_ERR_RANGE || m.op_bf16) return false;
  fprintf(stderr, "wuburvc_b200: switching this context's forward operands to the bf16 pair format\n");
  return gen_set_operand_format(m, 1);
}

// whole flat buffers between the reference tensor layouts and the device storage layouts
void flat_to_internal(const ParamTable& t, const float* ref, float* dev) {
  memset(dev, 0, sizeof(float) * (size_t)t.total);
  for (const auto& e : t.e) to_internal(e, ref + e.off, dev + e.off);
}
void flat_to_reference(const ParamTable& t, const float* dev, float* ref) {
  memset(ref, 0, sizeof(float) * (size_t)t.total);
  for (const auto& e : t.e) to_reference(e, dev + e.off, ref + e.off);
}

int download_reference(Gen& m, const float* dsrc, float* host_flat) {
  std::vector<float> tmp((size_t)m.table.total);
  if (cudaMemcpyAsync(tmp.data(), dsrc, sizeof(float) * tmp.size(), cudaMemcpyDeviceToHost, m.stream) != cudaSuccess)
    return WUBU_B200_ERR_CUDA;
  const int rc = check_err(m);
  if (rc) return rc;
  flat_to_reference(m.table, tmp.data(), host_flat);
  return 0;
}

int set_noise_stream(Gen& m, unsigned long long s) {
  // pageable source: staged before return, ordered on the model stream
  return cudaMemcpyAsync(&m.state->noise_stream, &s, sizeof(s), cudaMemcpyHostToDevice, m.stream) == cudaSuccess
             ? 0
             : WUBU_B200_ERR_CUDA;
}

// forward + backward (+ bucketed all-reduce) + AdamW, enqueued on the model stream
bool enqueue_step(Gen& m) {
  if (!gen_forward(m) || !gen_backward(m)) return false;
  return gen_adamw(m, 1.f / (float)comm_world(m), 1);
}

int run_step_graph(Gen& m) {
  if (comm_aborted(m)) return WUBU_B200_ERR_COMM;
  if (!m.graph) {
    cudaGraph_t g = nullptr;
    if (cudaStreamBeginCapture(m.stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return WUBU_B200_ERR_CUDA;
    const bool ok = enqueue_step(m);
    const cudaError_t e = cudaStreamEndCapture(m.stream, &g);
    if (!ok || e != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      fprintf(stderr, "wuburvc_b200: step capture failed (%s)\n", cudaGetErrorString(e));
      return WUBU_B200_ERR_CUDA;
    }
    size_t nn = 0;
    cudaGraphGetNodes(g, nullptr, &nn);
    std::vector<cudaGraphNode_t> nodes(nn);
    cudaGraphGetNodes(g, nodes.data(), &nn);
    m.graph_kernels = 0;
    for (auto nd : nodes) {
      cudaGraphNodeType t;
      if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++m.graph_kernels;
    }
    const cudaError_t ie = cudaGraphInstantiate(&m.graph, g, 0);
    cudaGraphDestroy(g);
    if (ie != cudaSuccess) {
      m.graph = nullptr;
      fprintf(stderr, "wuburvc_b200: graph instantiate failed (%s)\n", cudaGetErrorString(ie));
      return WUBU_B200_ERR_CUDA;
    }
  }
  return cudaGraphLaunch(m.graph, m.stream) == cudaSuccess ? 0 : WUBU_B200_ERR_CUDA;
}

int upload(Gen& m, const float* z, const float* f0, const float* g, const float* noise, const float* dldy) {
  const WubuB200GenConfig& c = m.cfg;
  cudaStream_t st = m.stream;
  auto cp = [&](void* d, const void* h, size_t bytes) {
    return cudaMemcpyAsync(d, h, bytes, cudaMemcpyHostToDevice, st) == cudaSuccess;
  };
  if (!z) return WUBU_B200_ERR_ARG;
  if (!cp(m.z, z, sizeof(float) * m.B * c.in_channels * m.F)) return WUBU_B200_ERR_CUDA;
  // dldy may be left out for forward-only use (the previous upload's, zeros at first, stays)
  if (dldy && !cp(m.dldy, dldy, sizeof(float) * m.B * m.T)) return WUBU_B200_ERR_CUDA;
  if (c.gin_channels) {
    if (!g) return WUBU_B200_ERR_ARG;
    if (!cp(m.g, g, sizeof(float) * m.B * c.gin_channels)) return WUBU_B200_ERR_CUDA;
  }
  if (c.nsf) {
    if (!f0) return WUBU_B200_ERR_ARG;
    if (!cp(m.f0, f0, sizeof(float) * m.B * m.F)) return WUBU_B200_ERR_CUDA;
    const bool had = m.has_noise_input;
    m.has_noise_input = noise != nullptr;
    if (noise && !cp(m.noise, noise, sizeof(float) * m.B * m.T * m.dim)) return WUBU_B200_ERR_CUDA;
    if (had != m.has_noise_input && m.graph) {  // the captured step baked the other noise source
      cudaGraphExecDestroy(m.graph);
      m.graph = nullptr;
    }
  }
  return 0;
}

}  // namespace

extern "C" {

WubuB200Gen* wubu_b200_gen_create(const WubuB200GenConfig* cfg, const WubuB200TrainOptions* opt) {
  if (!cfg || !opt || !config_valid(*cfg) || opt->batch < 1 || opt->frames < 1) return nullptr;
  if (opt->precision != WUBU_B200_PRECISION_BF16 && opt->precision != WUBU_B200_PRECISION_FP32) return nullptr;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || opt->device < 0 || opt->device >= ndev) {
    fprintf(stderr, "wuburvc_b200: no CUDA device %d\n", opt ? opt->device : -1);
    return nullptr;
  }
  auto* h = new WubuB200Gen();
  h->m.cfg = *cfg;
  h->m.opt = *opt;
  tc_kernels_init();
  if (!gen_setup(h->m)) {
    gen_free(h->m);
    delete h;
    return nullptr;
  }
  std::vector<float> p((size_t)h->m.table.total), d(p.size());
  init_params(h->m.cfg, h->m.table, 0, p.data());
  flat_to_internal(h->m.table, p.data(), d.data());
  cudaMemcpy(h->m.params, d.data(), d.size() * sizeof(float), cudaMemcpyHostToDevice);
  return h;
}

void wubu_b200_gen_destroy(WubuB200Gen* gen) {
  if (!gen) return;
  cudaSetDevice(gen->m.opt.device);
  gen_free(gen->m);
  delete gen;
}

int wubu_b200_gen_samples(const WubuB200Gen* gen) { return gen ? gen->m.T : WUBU_B200_ERR_ARG; }

void* wubu_b200_gen_stream(WubuB200Gen* gen) { return gen ? (void*)gen->m.stream : nullptr; }

int wubu_b200_gen_set_params(WubuB200Gen* gen, const float* host_flat) {
  if (!gen || !host_flat) return WUBU_B200_ERR_ARG;
  Gen& m = gen->m;
  cudaSetDevice(m.opt.device);
  const size_t bytes = sizeof(float) * (size_t)m.table.total;
  std::vector<float> d((size_t)m.table.total);
  flat_to_internal(m.table, host_flat, d.data());
  if (cudaMemcpyAsync(m.params, d.data(), bytes, cudaMemcpyHostToDevice, m.stream) != cudaSuccess)
    return WUBU_B200_ERR_CUDA;
  // a new parameter set restarts the optimiser
  cudaMemsetAsync(m.adam_m, 0, bytes, m.stream);
  cudaMemsetAsync(m.adam_v, 0, bytes, m.stream);
  cudaMemsetAsync(m.state, 0, sizeof(StepState), m.stream);
  return check_err(m);
}

int wubu_b200_gen_get_params(WubuB200Gen* gen, float* host_flat) {
  if (!gen || !host_flat) return WUBU_B200_ERR_ARG;
  Gen& m = gen->m;
  cudaSetDevice(m.opt.device);
  return download_reference(m, m.params, host_flat);
}

int wubu_b200_gen_get_opt_state(WubuB200Gen* gen, float* m_flat, float* v_flat, long long* step,
                                unsigned long long* noise_stream) {
  if (!gen || !m_flat || !v_flat) return WUBU_B200_ERR_ARG;
  Gen& m = gen->m;
  cudaSetDevice(m.opt.device);
  int rc = download_reference(m, m.adam_m, m_flat);
  if (!rc) rc = download_reference(m, m.adam_v, v_flat);
  if (rc) return rc;
  StepState st{};
  if (cudaMemcpy(&st, m.state, sizeof(st), cudaMemcpyDeviceToHost) != cudaSuccess) return WUBU_B200_ERR_CUDA;
  if (step) *step = st.adam_t;
  if (noise_stream) *noise_stream = st.noise_stream;
  return WUBU_B200_OK;
}

int wubu_b200_gen_set_opt_state(WubuB200Gen* gen, const float* m_flat, const float* v_flat, long long step,
                                unsigned long long noise_stream) {
  if (!gen || !m_flat || !v_flat || step < 0 || step > 0x7fffffffLL) return WUBU_B200_ERR_ARG;
  Gen& m = gen->m;
  cudaSetDevice(m.opt.device);
  const size_t bytes = sizeof(float) * (size_t)m.table.total;
  std::vector<float> dm((size_t)m.table.total), dv(dm.size());
  flat_to_internal(m.table, m_flat, dm.data());
  flat_to_internal(m.table, v_flat, dv.data());
  StepState st{};
  st.adam_t = (int)step;
  st.noise_stream = noise_stream;
  // synchronous copies: the host vectors go out of scope on return
  if (cudaStreamSynchronize(m.stream) != cudaSuccess || cudaMemcpy(m.adam_m, dm.data(), bytes, cudaMemcpyHostToDevice) ||
      cudaMemcpy(m.adam_v, dv.data(), bytes, cudaMemcpyHostToDevice) ||
      cudaMemcpy(m.state, &st, sizeof(st), cudaMemcpyHostToDevice))
    return WUBU_B200_ERR_CUDA;
  return check_err(m);
}

int wubu_b200_gen_get_grads(WubuB200Gen* gen, float* host_flat) {
  if (!gen || !host_flat) return WUBU_B200_ERR_ARG;
  Gen& m = gen->m;
  cudaSetDevice(m.opt.device);
  return download_reference(m, m.grads, host_flat);
}

int wubu_b200_gen_upload(WubuB200Gen* gen, const float* z, const float* f0, const float* g, const float* noise,
                         const float* dldy) {
  if (!gen) return WUBU_B200_ERR_ARG;
  cudaSetDevice(gen->m.opt.device);
  const int rc = upload(gen->m, z, f0, g, noise, dldy);
  return rc ? rc : check_err(gen->m);
}

int wubu_b200_gen_forward(WubuB200Gen* gen, unsigned long long noise_stream, float* audio_out) {
  if (!gen) return WUBU_B200_ERR_ARG;
  Gen& m = gen->m;
  cudaSetDevice(m.opt.device);
  for (int attempt = 0;; ++attempt) {
    if (set_noise_stream(m, noise_stream)) return WUBU_B200_ERR_CUDA;
    if (!gen_forward(m)) return WUBU_B200_ERR_CUDA;
    if (audio_out &&
        cudaMemcpyAsync(audio_out, m.audio, sizeof(float) * m.B * m.T, cudaMemcpyDeviceToHost, m.stream) != cudaSuccess)
      return WUBU_B200_ERR_CUDA;
    const int rc = check_err(m);
    if (attempt == 0 && range_fallback(m, rc)) continue;
    return rc;
  }
}

int wubu_b200_gen_set_forward_only(WubuB200Gen* gen, int on) {
  if (!gen || on < 0 || on > 2) return WUBU_B200_ERR_ARG;
  cudaSetDevice(gen->m.opt.device);
  return gen_set_forward_only(gen->m, on) ? 0 : WUBU_B200_ERR_CUDA;
}

int wubu_b200_gen_backward(WubuB200Gen* gen) {
  if (!gen || gen->m.forward_only) return WUBU_B200_ERR_ARG;
  cudaSetDevice(gen->m.opt.device);
  if (!gen_backward(gen->m)) return WUBU_B200_ERR_CUDA;
  return check_err(gen->m);
}

int wubu_b200_gen_adamw(WubuB200Gen* gen) {
  if (!gen || gen->m.forward_only) return WUBU_B200_ERR_ARG;
  cudaSetDevice(gen->m.opt.device);
  if (!gen_adamw(gen->m, 1.f / (float)comm_world(gen->m), 0)) return WUBU_B200_ERR_CUDA;
  return check_err(gen->m);
}

int wubu_b200_gen_train_step(WubuB200Gen* gen, const float* z, const float* f0, const float* g, const float* noise,
                             const float* dldy, float* audio_out, unsigned long long noise_stream, int flags) {
  if (!gen || gen->m.forward_only) return WUBU_B200_ERR_ARG;
  Gen& m = gen->m;
  cudaSetDevice(m.opt.device);
  if (!(flags & WUBU_B200_INPUTS_RESIDENT)) {
    const int rc = upload(m, z, f0, g, noise, dldy);
    if (rc) return rc;
  }
  for (int attempt = 0;; ++attempt) {
    if (set_noise_stream(m, noise_stream)) return WUBU_B200_ERR_CUDA;
    const int rc = run_step_graph(m);
    if (rc) return rc;
    if (audio_out &&
        cudaMemcpyAsync(audio_out, m.audio, sizeof(float) * m.B * m.T, cudaMemcpyDeviceToHost, m.stream) != cudaSuccess)
      return WUBU_B200_ERR_CUDA;
    const int rc2 = check_err(m);
    // the overflowing step changed nothing (its update was skipped on every rank): recompute it
    if (attempt == 0 && range_fallback(m, rc2)) continue;
    return rc2;
  }
}

int wubu_b200_gen_train_step_async(WubuB200Gen* gen, unsigned long long noise_stream) {
  if (!gen || gen->m.forward_only) return WUBU_B200_ERR_ARG;
  Gen& m = gen->m;
  cudaSetDevice(m.opt.device);
  if (set_noise_stream(m, noise_stream)) return WUBU_B200_ERR_CUDA;
  return run_step_graph(m);
}

int wubu_b200_gen_sync(WubuB200Gen* gen) {
  if (!gen) return WUBU_B200_ERR_ARG;
  cudaSetDevice(gen->m.opt.device);
  const int rc = check_err(gen->m);
  range_fallback(gen->m, rc);  // the skipped steps are reported; later steps use the bf16 format
  return rc;
}

int wubu_b200_gen_graph_kernels(WubuB200Gen* gen) {
  if (!gen) return WUBU_B200_ERR_ARG;
  return gen->m.graph ? gen->m.graph_kernels : -1;
}

int wubu_b200_gen_kernel_bench(WubuB200Gen* gen, int which, int stage, int iters, float* ms_per_launch,
                               double* flops_per_launch) {
  if (!gen || stage < 0 || stage > 3 || iters < 1 || which < 0 || which > 9) return WUBU_B200_ERR_ARG;
  Gen& m = gen->m;
  cudaSetDevice(m.opt.device);
  StageBufs& s = m.sg[stage];
  int j = 0;
  for (int q = 1; q < m.nk; ++q)
    if (m.cfg.resblock_kernels[q] > m.cfg.resblock_kernels[j]) j = q;
  StackBufs& k = s.st[j];
  // algorithmic FLOPs: resblock convs 2 rows C^2 k; ConvTranspose 2 rows_out C Cin k/s (each output
  // sample meets k/s taps); conv_pre 2 B F C0 C_in 7
  double flops = 2.0 * s.rows * (double)s.C * s.C * m.cfg.resblock_kernels[j];
  if (which >= 5 && which <= 7) flops = 2.0 * s.rows * (double)s.C * s.Cin * s.ku / s.su;
  if (which == 8) flops = 2.0 * m.B * m.F * (double)m.cfg.initial_channel * m.cfg.in_channels * 7;
  if (which == 9) flops = 2.0 * s.rows * (double)s.C * s.C * m.cfg.resblock_kernels[j];
  auto launch = [&]() -> bool {
    switch (which) {
      case 0: return k.f1[0].run(m.stream) == cudaSuccess;
      case 1: return k.d1[0].run(m.stream) == cudaSuccess;
      case 2: return k.g1[0].L.run(m.stream) == cudaSuccess;
      case 3: return k.f2[0].run(m.stream) == cudaSuccess;
      case 4: return k.d2[0].run(m.stream) == cudaSuccess;
      case 5: return s.up_fwd.run(m.stream) == cudaSuccess;
      case 6: return s.up_dg.run(m.stream) == cudaSuccess;
      case 7: return s.up_wg.L.run(m.stream) == cudaSuccess;
      case 8: return m.pre_fwd.run(m.stream) == cudaSuccess;
      default: return k.g2[0].L.run(m.stream) == cudaSuccess;
    }
  };
  for (int i = 0; i < 2; ++i)
    if (!launch()) return WUBU_B200_ERR_CUDA;
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  cudaEventRecord(a, m.stream);
  for (int i = 0; i < iters; ++i)
    if (!launch()) return WUBU_B200_ERR_CUDA;
  cudaEventRecord(b, m.stream);
  const int rc = check_err(m);
  float ms = 0.f;
  cudaEventElapsedTime(&ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  if (ms_per_launch) *ms_per_launch = ms / (float)iters;
  if (flops_per_launch) *flops_per_launch = flops;
  return rc;
}

int wubu_b200_nccl_unique_id(void* out128) {
  if (!out128) return WUBU_B200_ERR_ARG;
  return comm_unique_id(out128);
}

int wubu_b200_gen_set_comm_timeout_ms(WubuB200Gen* gen, int ms) {
  if (!gen) return WUBU_B200_ERR_ARG;
  return comm_set_timeout(gen->m, ms);
}

int wubu_b200_gen_attach_comm(WubuB200Gen* gen, int rank, int world, const void* id128) {
  if (!gen) return WUBU_B200_ERR_ARG;
  Gen& m = gen->m;
  cudaSetDevice(m.opt.device);
  cudaStreamSynchronize(m.stream);
  if (m.graph) {  // the captured step did not contain the all-reduce
    cudaGraphExecDestroy(m.graph);
    m.graph = nullptr;
  }
  return comm_attach(m, rank, world, id128);
}

}  // extern "C"
