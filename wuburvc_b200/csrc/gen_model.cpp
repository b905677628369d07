// gen_model.cpp — the generator training step on one GPU: buffers, launch plans, forward,
// backward, AdamW, CUDA-graph capture.
//
// Data layout in HBM: every activation is channels-last [B][T][C].  Residual streams (pair inputs,
// stage sums, their gradients) are fp32.  Forward GEMM operands are fp16 hi + fp16 lo*2^11 pairs
// (three products, fp32-accurate; bf16 pairs after a range error); every activation also keeps a
// bf16 copy, the weight gradient's operand and the LeakyReLU mask source.  Backward operands are
// single bf16, or under fp32 precision bf16 hi + lo pairs: every bf16 operand tensor then has a lo
// companion written by its producer, the input gradients take three products in one kernel and the
// weight gradients three launches summed by one reduction.  Parameters, gradients and AdamW moments
// live in flat fp32 buffers laid out by the parameter table.
#include "gen_model.h"

#include <cmath>
#include <cstdio>
#include <cstring>

#include "small_kernels.cuh"

namespace wb {

// comm.cpp (no-ops without a communicator)
int comm_bucket_ready(Gen& m, int bucket, cudaStream_t producer);
int comm_world(Gen& m);
int comm_join(Gen& m);
void comm_destroy(Gen& m);

namespace {

constexpr size_t kWgBatchBytes = (size_t)24 << 20;  // split-K partials reduced per batch (measured: 24 MB +0.5 % over 48)
constexpr int kWgradCtas = 296;  // 2 waves of 148 SMs for split-K weight gradients

#define CK(x)                                                                                   \
  do {                                                                                          \
    cudaError_t e_ = (x);                                                                       \
    if (e_ != cudaSuccess) {                                                                    \
      fprintf(stderr, "wuburvc_b200: %s failed: %s (%s:%d)\n", #x, cudaGetErrorString(e_), __FILE__, \
              __LINE__);                                                                        \
      return false;                                                                             \
    }                                                                                           \
  } while (0)

template <class T>
bool dalloc(Gen& m, T** p, size_t n) {
  *p = nullptr;
  if (n == 0) return true;
  void* q = nullptr;
  if (cudaMalloc(&q, n * sizeof(T)) != cudaSuccess) {
    fprintf(stderr, "wuburvc_b200: cudaMalloc of %zu bytes failed\n", n * sizeof(T));
    return false;
  }
  cudaMemset(q, 0, n * sizeof(T));
  m.allocs.push_back(q);
  *p = static_cast<T*>(q);
  return true;
}

Epi epi0(float slope) {
  Epi e{};
  e.scale = 1.f;
  e.slope = slope;
  return e;
}

const float* alpha_ptr(Gen& m, const std::string& name) {
  const int i = m.pidx(name);
  return i >= 0 ? m.P(i) : nullptr;
}
float* alpha_grad(Gen& m, const std::string& name) {
  const int i = m.pidx(name);
  return i >= 0 ? m.G(i) : nullptr;
}

// derived weights of one conv param
bool make_weights(Gen& m, ConvWeights& w, const std::string& base, bool resblock, bool convT, int stride) {
  const bool wn = m.cfg.weight_norm && (resblock || convT);
  const std::string vname = resblock ? base + ".weight_v" : (wn ? base + ".weight_v" : base + ".weight");
  w.pv = m.pidx(vname);
  w.pg = wn ? m.pidx(base + ".weight_g") : -1;
  w.pb = m.pidx(base + ".bias");
  if (w.pv < 0 || (wn && w.pg < 0)) {
    fprintf(stderr, "wuburvc_b200: missing parameter %s\n", vname.c_str());
    return false;
  }
  const ParamEntry& p = m.table.e[w.pv];
  w.rows = p.shape[0];
  w.cols = p.shape[1];
  w.k = p.shape[2];
  w.convT = convT;
  w.stride = stride;
  const size_t n = (size_t)p.n;
  if (!dalloc(m, &w.fwd_hi, n) || !dalloc(m, &w.fwd_lo, n) || !dalloc(m, &w.dg, n)) return false;
  if (m.fp32 && !dalloc(m, &w.dg_lo, n)) return false;
  if (wn) {
    if (!dalloc(m, &w.norm, (size_t)w.rows) || !dalloc(m, &w.dW, n)) return false;
  } else {
    w.dW = m.G(w.pv);
  }
  return true;
}

bool make_wgrad_job(Gen& m, WgradJob& j, int layout, int c_out, int k, const ConvWeights& w) {
  j.layout = layout;
  j.c_out = c_out;
  j.k = k;
  j.w = &w;
  j.dW = w.dW;
  // every (oc, tap) must own a partial row
  std::vector<char> seen((size_t)c_out * k, 0);
  for (size_t r = 0; r < j.L.row_tap.size(); ++r)
    if (j.L.row_tap[r] >= 0) seen[(size_t)j.L.row_oc[r] * k + j.L.row_tap[r]] = 1;
  for (char x : seen)
    if (!x) return false;
  const size_t one = wgrad_part_floats(j.L);
  if (!dalloc(m, &j.part, one * j.nl)) return false;
  j.L.p.part = j.part;
  for (int i = 0; i + 1 < j.nl; ++i) {
    if (j.lo[i].splits != j.L.splits || j.lo[i].p.n_mtiles != j.L.p.n_mtiles || j.lo[i].p.n_total != j.L.p.n_total)
      return false;
    j.lo[i].p.part = j.part + one * (i + 1);
  }
  return true;
}

size_t job_part_floats(const WgradJob& j) { return wgrad_part_floats(j.L) * j.nl; }

// Input-gradient GEMM: single bf16 operands, or under fp32 precision bf16 hi + lo pairs (three products).
bool plan_dgrad(Gen& m, ConvOp& op, const ConvGeom& g, const bf16* dy, const bf16* dy_lo, const ConvWeights& w,
                const Epi& e) {
  if (m.fp32 && (!dy_lo || !w.dg_lo)) return false;
  if (!plan_conv_any(op, g, dy, m.fp32 ? dy_lo : nullptr, w.dg, m.fp32 ? w.dg_lo : nullptr, m.fp32, e, m.err))
    return false;
  op.v1.p.split_bf16 = 1;  // gradient pairs are bf16 hi + bf16 lo (no effect without the split)
  op.c2.p.split_bf16 = 1;
  return true;
}

// Weight-gradient GEMM of a Conv1d: one launch, or under fp32 precision three (dy_hi x x_hi, dy_hi x
// x_lo, dy_lo x x_hi) whose split-K partials one reduction sums.
bool plan_wgrad_job(Gen& m, WgradJob& j, const ConvGeom& g, const bf16* dy, const bf16* dy_lo, const bf16* x,
                    const bf16* x_lo, const ConvWeights& w) {
  j.nl = m.fp32 ? 3 : 1;
  if (m.fp32 && (!dy_lo || !x_lo)) return false;
  if (!plan_wgrad(j.L, g, dy, x, nullptr, ~size_t(0), kWgradCtas, m.err)) return false;
  if (m.fp32 && (!plan_wgrad(j.lo[0], g, dy, x_lo, nullptr, ~size_t(0), kWgradCtas, m.err) ||
                 !plan_wgrad(j.lo[1], g, dy_lo, x, nullptr, ~size_t(0), kWgradCtas, m.err)))
    return false;
  return make_wgrad_job(m, j, 0, g.C_out, g.k, w);
}

// The split-K reduction of a weight gradient: partial rows are (tap * C_out + oc) x C_in, so the first
// k*C_out rows of each split are exactly the tap-major device layout of the weight and the sum over
// splits is a plain column reduction.  Under weight norm it lands in the dW temp (then wn backward).
ReduceDesc wgrad_desc(Gen& m, const WgradJob& j) {
  const ConvWeights& w = *j.w;
  ReduceDesc d{};
  d.part = j.part;
  d.out = w.pg >= 0 ? w.dW : m.G(w.pv);
  d.ld = (long long)j.L.p.n_mtiles * 128 * j.L.p.n_total;
  d.n = (long long)j.k * j.c_out * j.L.p.n_total;
  d.nparts = j.L.splits * j.nl;  // the fp32-precision launches' partials follow L's
  return d;
}

WnDesc wn_desc(Gen& m, const ConvWeights& w) {
  WnDesc d{};
  d.dW = w.dW;
  d.v = m.P(w.pv);
  d.g = m.P(w.pg);
  d.norm = w.norm;
  d.dv = m.G(w.pv);
  d.dg = m.G(w.pg);
  d.rows = w.rows;
  d.cols = w.cols;
  d.k = w.k;
  d.is_convT = w.convT;
  return d;
}

ReduceDesc colsum_desc(const float* part, int nparts, int C, float* out) {
  ReduceDesc d{};
  d.part = part;
  d.out = out;
  d.ld = C;
  d.n = C;
  d.nparts = nparts;
  return d;
}

// Uploads a batch of column reductions (with their chunk scratch and counters) for one launch.
bool upload_reduce_table(Gen& m, std::vector<ReduceDesc>& v, ReduceDesc** dev, int* n, int* blocks) {
  size_t sc_total = 0, ct_total = 0;
  int first = 0;
  std::vector<size_t> sc_off(v.size()), ct_off(v.size());
  for (size_t i = 0; i < v.size(); ++i) {
    size_t sf = 0, cn = 0;
    const int nb = reduce_desc_shape(v[i], first, &sf, &cn);
    if (nb < 0) {
      fprintf(stderr, "wuburvc_b200: reduction shape not float4-aligned (n %lld ld %lld)\n", v[i].n, v[i].ld);
      return false;
    }
    first += nb;
    sc_off[i] = sc_total;
    ct_off[i] = ct_total;
    sc_total += sf;
    ct_total += cn;
  }
  float* sc = nullptr;
  unsigned int* ct = nullptr;
  if (sc_total && !dalloc(m, &sc, sc_total)) return false;
  if (ct_total) {
    if (!dalloc(m, &ct, ct_total)) return false;
    CK(cudaMemset(ct, 0, ct_total * sizeof(unsigned int)));
  }
  for (size_t i = 0; i < v.size(); ++i)
    if (v[i].nchunks > 1) {
      v[i].scratch = sc + sc_off[i];
      v[i].counter = ct + ct_off[i];
    }
  *n = (int)v.size();
  *blocks = first;
  if (v.empty()) return true;
  if (!dalloc(m, dev, v.size())) return false;
  CK(cudaMemcpy(*dev, v.data(), v.size() * sizeof(ReduceDesc), cudaMemcpyHostToDevice));
  return true;
}

bool upload_wn_table(Gen& m, std::vector<WnDesc>& v, WnDesc** dev, int* n, int* rows) {
  int first = 0;
  for (WnDesc& d : v) {
    d.first = first;
    first += d.rows;
  }
  *n = (int)v.size();
  *rows = first;
  if (v.empty()) return true;
  if (!dalloc(m, dev, v.size())) return false;
  CK(cudaMemcpy(*dev, v.data(), v.size() * sizeof(WnDesc), cudaMemcpyHostToDevice));
  return true;
}

// split-K partials into the job's own buffer; the batched reductions follow the group's last job
// fork: the side stream waits for everything enqueued on the main stream so far; join: the reverse
bool fork_side(Gen& m) {
  const cudaEvent_t e = m.evs[(size_t)(m.ev_next++) % m.evs.size()];
  CK(cudaEventRecord(e, m.stream));
  CK(cudaStreamWaitEvent(m.side, e, 0));
  return true;
}

bool join_side(Gen& m) {
  const cudaEvent_t e = m.evs[(size_t)(m.ev_next++) % m.evs.size()];
  CK(cudaEventRecord(e, m.side));
  CK(cudaStreamWaitEvent(m.stream, e, 0));
  return true;
}

bool run_wgrad_launches(Gen& m, const WgradJob& j) {
  CK(j.L.run(m.stream));
  for (int i = 0; i + 1 < j.nl; ++i) CK(j.lo[i].run(m.stream));
  return true;
}

bool run_wgrad(Gen& m, StageBufs& s, const WgradJob& j) {
  if (!run_wgrad_launches(m, j)) return false;
  if (j.flush >= 0) {  // the group's reductions overlap the next convolutions
    const WgradBatch& b = s.wg_batches[j.flush];
    if (!fork_side(m)) return false;
    reduce_batched(b.wg_d, b.wg_n, b.wg_blocks, m.side);
    wn_backward_batched(b.wn_d, b.wn_n, b.wn_rows, m.side);
  }
  return true;
}

// conv_pre's weight gradient (kernel + reduction + weight norm; a handful of launches, once per step)
bool run_pre_wgrad(Gen& m) {
  if (!run_wgrad_launches(m, m.pre_wg)) return false;
  const ReduceDesc d = wgrad_desc(m, m.pre_wg);
  col_reduce_ld(d.part, d.nparts, d.n, d.ld, d.out, 0, m.stream);
  const ConvWeights& w = m.wpre;
  if (w.pg >= 0)
    wn_backward(w.dW, m.P(w.pv), m.P(w.pg), w.norm, w.rows, w.cols, w.k, w.convT, m.G(w.pv), m.G(w.pg), m.stream);
  return true;
}


}  // namespace

// =============================================================================================
// setup
// =============================================================================================
bool gen_setup(Gen& m) {
  const WubuB200GenConfig& c = m.cfg;
  m.B = m.opt.batch;
  m.F = m.opt.frames;
  m.nk = c.n_kernels;
  m.nd = c.n_dilations;
  m.upp = 1;
  for (int L = 0; L < 4; ++L) m.upp *= c.upsample_rates[L];
  m.T = m.F * m.upp;
  m.dim = c.harmonic_num + 1;
  const bool snake = c.activation == 1;
  const int B = m.B;
  m.fp32 = m.opt.precision == WUBU_B200_PRECISION_FP32;
  // a bf16 lo companion, allocated under fp32 precision only (left null otherwise)
  auto lo_alloc = [&](bf16** p, size_t n) { return !m.fp32 || dalloc(m, p, n); };
  CK(cudaSetDevice(m.opt.device));
  CK(cudaStreamCreateWithFlags(&m.stream, cudaStreamNonBlocking));
  CK(cudaStreamCreateWithFlags(&m.side, cudaStreamNonBlocking));
  m.evs.resize(64);
  for (auto& e : m.evs) CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  if (!dalloc(m, &m.err, 1) || !dalloc(m, &m.state, 1)) return false;

  m.table = build_param_table(c);
  const size_t P = (size_t)m.table.total;
  // the gradient buffer carries one more slot after the parameters: the data-parallel range flag
  // (summed over ranks in the last all-reduce bucket)
  if (!dalloc(m, &m.params, P) || !dalloc(m, &m.grads, P + 64) || !dalloc(m, &m.adam_m, P) ||
      !dalloc(m, &m.adam_v, P))
    return false;

  // ---- inputs ----
  if (!dalloc(m, &m.z, (size_t)B * c.in_channels * m.F) || !dalloc(m, &m.dldy, (size_t)B * m.T)) return false;
  if (!dalloc(m, &m.z_hi, (size_t)B * m.F * c.in_channels) || !dalloc(m, &m.z_lo, (size_t)B * m.F * c.in_channels) ||
      !dalloc(m, &m.z_bf, (size_t)B * m.F * c.in_channels) || !lo_alloc(&m.z_bflo, (size_t)B * m.F * c.in_channels))
    return false;
  if (c.gin_channels && !dalloc(m, &m.g, (size_t)B * c.gin_channels)) return false;
  if (c.nsf) {
    if (!dalloc(m, &m.f0, (size_t)B * m.F) || !dalloc(m, &m.noise, (size_t)B * m.T * m.dim)) return false;
    if (!dalloc(m, &m.har, (size_t)B * m.T) || !dalloc(m, &m.sw, (size_t)B * m.T * m.dim) ||
        !dalloc(m, &m.d_har, (size_t)B * m.T) || !dalloc(m, &m.nsf_acc, (size_t)B * m.F))
      return false;
    m.nsf_parts = 256;
    if (!dalloc(m, &m.nsf_part, (size_t)(m.nsf_parts + 1) * (m.dim + 1))) return false;
  }

  // ---- stage geometry ----
  const int C0 = c.initial_channel;
  int Tcur = m.F;
  for (int L = 0; L < 4; ++L) {
    StageBufs& s = m.sg[L];
    s.su = c.upsample_rates[L];
    s.ku = c.upsample_kernels[L];
    s.pu = (s.ku - s.su) / 2;
    s.Cin = C0 >> L;
    s.C = C0 >> (L + 1);
    s.T = Tcur * s.su;
    s.rows = B * s.T;
    Tcur = s.T;
    if (L + 1 < 4) {
      int sf = 1;
      for (int i = L + 1; i < 4; ++i) sf *= c.upsample_rates[i];
      s.sn = sf;
      s.kn = 2 * sf;
      s.pn = sf / 2;
    } else {
      s.sn = 1;
      s.kn = 1;
      s.pn = 0;
    }
  }
  if (m.sg[3].T != m.T) return false;

  // ---- derived weights ----
  if (!make_weights(m, m.wpre, "dec.conv_pre", false, false, 1)) return false;
  for (int L = 0; L < 4; ++L) {
    StageBufs& s = m.sg[L];
    if (!make_weights(m, s.wu, "dec.ups." + std::to_string(L), false, true, s.su)) return false;
    for (int j = 0; j < m.nk; ++j)
      for (int cp = 0; cp < m.nd; ++cp) {
        const std::string R = "dec.resblocks." + std::to_string(L * m.nk + j);
        if (!make_weights(m, s.st[j].w1[cp], R + ".convs1." + std::to_string(cp), true, false, 1)) return false;
        if (!make_weights(m, s.st[j].w2[cp], R + ".convs2." + std::to_string(cp), true, false, 1)) return false;
      }
  }

  // ---- activations ----
  const size_t n_pre = (size_t)B * m.F * C0;
  if (!dalloc(m, &m.pre_hi, n_pre) || !dalloc(m, &m.pre_lo, n_pre) || !dalloc(m, &m.pre_bf, n_pre) ||
      !dalloc(m, &m.d_pre_bf, n_pre))
    return false;
  if (snake && !dalloc(m, &m.pre_pre, n_pre)) return false;
  if (!lo_alloc(&m.pre_bflo, n_pre) || !lo_alloc(&m.d_pre_bflo, n_pre) || (snake && !lo_alloc(&m.pre_prelo, n_pre)))
    return false;
  if (c.gin_channels && !dalloc(m, &m.rowadd, (size_t)B * C0)) return false;
  if (!dalloc(m, &m.audio, (size_t)B * m.T)) return false;
  for (int L = 0; L < 4; ++L) {
    StageBufs& s = m.sg[L];
    const size_t n = (size_t)s.rows * s.C;
    if (!dalloc(m, &s.x_in, n) || !dalloc(m, &s.sout, n) || !dalloc(m, &s.sa_hi, n) || !dalloc(m, &s.sa_lo, n) ||
        !dalloc(m, &s.sa_bf, n))
      return false;
    if (!dalloc(m, &s.d_s, n) || !dalloc(m, &s.d_s_bf, n) || !dalloc(m, &s.d_x, n) || !dalloc(m, &s.d_x_bf, n))
      return false;
    if (!lo_alloc(&s.sa_bflo, n) || !lo_alloc(&s.d_s_bflo, n) || !lo_alloc(&s.d_x_bflo, n)) return false;
    const int nxa = snake ? m.nk : 1;
    for (int q = 0; q < nxa; ++q)
      if (!dalloc(m, &s.xa_hi[q], n) || !dalloc(m, &s.xa_lo[q], n) || !dalloc(m, &s.xa_bf[q], n) ||
          !lo_alloc(&s.xa_bflo[q], n))
        return false;
    if (snake && (!dalloc(m, &s.x_pre, n) || !dalloc(m, &s.s_pre, n))) return false;
    if (snake && (!lo_alloc(&s.x_prelo, n) || !lo_alloc(&s.s_prelo, n))) return false;
    const int tiles = B * ((s.T + 127) / 128);
    for (int j = 0; j < m.nk; ++j) {
      StackBufs& k = s.st[j];
      k.tiles = tiles;
      k.p[0] = s.x_in;
      k.a1_hi[0] = s.xa_hi[snake ? j : 0];
      k.a1_lo[0] = s.xa_lo[snake ? j : 0];
      k.a1_bf[0] = s.xa_bf[snake ? j : 0];
      k.a1_pre[0] = s.x_pre;
      k.a1_bflo[0] = s.xa_bflo[snake ? j : 0];
      k.a1_prelo[0] = s.x_prelo;
      for (int cp = 0; cp < m.nd; ++cp) {
        if (cp > 0) {
          if (!dalloc(m, &k.p[cp], n) || !dalloc(m, &k.a1_hi[cp], n) || !dalloc(m, &k.a1_lo[cp], n) ||
              !dalloc(m, &k.a1_bf[cp], n) || !lo_alloc(&k.a1_bflo[cp], n))
            return false;
          if (snake && (!dalloc(m, &k.a1_pre[cp], n) || !lo_alloc(&k.a1_prelo[cp], n))) return false;
        }
        if (!dalloc(m, &k.a2_hi[cp], n) || !dalloc(m, &k.a2_lo[cp], n) || !dalloc(m, &k.a2_bf[cp], n) ||
            !lo_alloc(&k.a2_bflo[cp], n))
          return false;
        if (snake && (!dalloc(m, &k.a2_pre[cp], n) || !lo_alloc(&k.a2_prelo[cp], n))) return false;
        // column-sum partials: one row per tile (general kernel) or per CTA of the persistent kernel,
        // which may split N in two and writes two rows (epilogue groups) per CTA: at most 4 * tiles rows
        if (!dalloc(m, &k.cs_dc1[cp], (size_t)4 * tiles * s.C) || !dalloc(m, &k.cs_dp[cp], (size_t)4 * tiles * s.C))
          return false;
        if (snake &&
            (!dalloc(m, &k.ap1[cp], (size_t)4 * tiles * s.C) || !dalloc(m, &k.ap2[cp], (size_t)4 * tiles * s.C)))
          return false;
      }
      if (!dalloc(m, &k.d_c1, n) || !lo_alloc(&k.d_c1_lo, n)) return false;
      for (int q = 0; q < 2; ++q)
        if (!dalloc(m, &k.pp[q], n) || !dalloc(m, &k.pp_bf[q], n) || !lo_alloc(&k.pp_bflo[q], n)) return false;
    }
    if (c.nsf) {
      s.noise_parts = noise_backward_parts(B, s.T, s.C, s.kn);
      if (!dalloc(m, &s.noise_wt, (size_t)s.C * s.kn)) return false;
      if (!dalloc(m, &s.noise_wpart, (size_t)s.noise_parts * s.C * s.kn)) return false;
      m.noise_scratch_n = std::max(m.noise_scratch_n, (size_t)s.noise_parts * s.C * s.kn);
      if (!dalloc(m, &s.noise_g, (size_t)B * s.T * s.kn)) return false;
      // the noise kernels' shared-memory windows stay within the default 48 KB
      if (noise_act_smem(s.kn, s.sn) > 48 * 1024 || sizeof(float) * ((size_t)127 * s.sn + s.kn) > 30 * 1024) {
        fprintf(stderr, "wuburvc_b200: noise conv of stage %d too large (k=%d stride=%d)\n", L, s.kn, s.sn);
        return false;
      }
    }
  }

  // ---- launch plans ----
  // forward conv_pre
  {
    Epi e = epi0(c.lrelu_slope);
    e.bias = m.P(m.wpre.pb);
    e.rowadd = m.rowadd;
    e.act_hi = m.pre_hi;
    e.act_lo = m.pre_lo;
    e.act_bf = m.pre_bf;
    e.act_bflo = m.pre_bflo;
    e.range_err = m.err;
    e.act_kind = c.activation;
    e.act_alpha = alpha_ptr(m, "dec.ups_act.0.alpha");
    e.pre_hi = m.pre_pre;
    e.pre_lo = m.pre_prelo;
    ConvGeom g{B, m.F, m.F, c.in_channels, C0, 7, 1, 3};
    if (!plan_conv(m.pre_fwd, g, m.z_hi, m.z_lo, m.wpre.fwd_hi, m.wpre.fwd_lo, 1, e, m.err)) return false;
  }
  for (int L = 0; L < 4; ++L) {
    StageBufs& s = m.sg[L];
    const bool last = L == 3;
    const int Tin = (L == 0) ? m.F : m.sg[L - 1].T;
    const f16* in_hi = (L == 0) ? m.pre_hi : m.sg[L - 1].sa_hi;
    const f16* in_lo = (L == 0) ? m.pre_lo : m.sg[L - 1].sa_lo;
    {  // ups forward
      Epi e = epi0(c.lrelu_slope);
      e.bias = m.P(s.wu.pb);
      e.out_f32 = s.x_in;
      if (!plan_convT(s.up_fwd, B, Tin, s.Cin, s.C, s.ku, s.su, s.pu, in_hi, in_lo, s.wu.fwd_hi, s.wu.fwd_lo, 1, e,
                      m.err))
        return false;
    }
    for (int j = 0; j < m.nk; ++j) {
      StackBufs& k = s.st[j];
      const int kk = c.resblock_kernels[j];
      const std::string R = std::to_string(L * m.nk + j);
      for (int cp = 0; cp < m.nd; ++cp) {
        const int dil = c.resblock_dilations[j][cp];
        const std::string P = std::to_string(cp);
        {  // conv1: bias -> act -> a2
          Epi e = epi0(c.lrelu_slope);
          e.bias = m.P(k.w1[cp].pb);
          e.act_hi = k.a2_hi[cp];
          e.act_lo = k.a2_lo[cp];
          e.act_bf = k.a2_bf[cp];
          e.act_bflo = k.a2_bflo[cp];
          e.range_err = m.err;
          e.act_kind = c.activation;
          e.act_alpha = alpha_ptr(m, "dec.resblocks." + R + ".alpha2." + P);
          e.pre_hi = k.a2_pre[cp];
          e.pre_lo = k.a2_prelo[cp];
          ConvGeom g{B, s.T, s.T, s.C, s.C, kk, dil, dil * (kk - 1) / 2};
          if (!plan_conv_any(k.f1[cp], g, k.a1_hi[cp], k.a1_lo[cp], k.w1[cp].fwd_hi, k.w1[cp].fwd_lo, 1, e, m.err))
            return false;
        }
        {  // conv2: bias + residual -> next pair input (+act) or stage sum
          Epi e = epi0(c.lrelu_slope);
          e.bias = m.P(k.w2[cp].pb);
          e.res = k.p[cp];
          e.act_kind = c.activation;
          if (cp + 1 < m.nd) {
            e.out_f32 = k.p[cp + 1];
            e.act_hi = k.a1_hi[cp + 1];
            e.act_lo = k.a1_lo[cp + 1];
            e.act_bf = k.a1_bf[cp + 1];
            e.act_bflo = k.a1_bflo[cp + 1];
            e.range_err = m.err;
            e.act_alpha = alpha_ptr(m, "dec.resblocks." + R + ".alpha1." + std::to_string(cp + 1));
            e.pre_hi = k.a1_pre[cp + 1];
            e.pre_lo = k.a1_prelo[cp + 1];
          } else {
            e.scale = 1.f / (float)m.nk;
            e.out_f32 = s.sout;
            e.accumulate = j > 0;
            if (j == m.nk - 1) {
              e.act_hi = s.sa_hi;
              e.act_lo = s.sa_lo;
              e.act_bf = s.sa_bf;
              e.act_bflo = s.sa_bflo;
              e.range_err = m.err;
              e.pre_hi = s.s_pre;
              e.pre_lo = s.s_prelo;
              e.slope = last ? c.final_slope : c.lrelu_slope;
              e.act_alpha = alpha_ptr(m, last ? "dec.post_act.alpha" : "dec.ups_act." + std::to_string(L + 1) + ".alpha");
            }
          }
          ConvGeom g{B, s.T, s.T, s.C, s.C, kk, 1, (kk - 1) / 2};
          if (!plan_conv_any(k.f2[cp], g, k.a2_hi[cp], k.a2_lo[cp], k.w2[cp].fwd_hi, k.w2[cp].fwd_lo, 1, e, m.err))
            return false;
        }
      }
    }
  }

  // ---- backward plans ----
  // gradient wrt each stage output: produced by conv_post bwd (L=3) or ups L+1 dgrad
  m.post_blocks = post_backward_blocks(B, m.T);
  if (!dalloc(m, &m.post_cs, (size_t)m.post_blocks * m.sg[3].C) ||
      !dalloc(m, &m.post_wpart, (size_t)m.post_blocks * m.sg[3].C * 7))
    return false;
  if (snake && !dalloc(m, &m.post_ap, (size_t)m.post_blocks * m.sg[3].C)) return false;
  m.sg[3].cs_ds = m.post_cs;
  m.sg[3].cs_ds_tiles = m.post_blocks;
  for (int L = 0; L < 4; ++L) {
    StageBufs& s = m.sg[L];
    for (int j = 0; j < m.nk; ++j) {
      StackBufs& k = s.st[j];
      const int kk = c.resblock_kernels[j];
      const std::string R = std::to_string(L * m.nk + j);
      for (int cp = m.nd - 1; cp >= 0; --cp) {
        const int dil = c.resblock_dilations[j][cp];
        const std::string P = std::to_string(cp);
        const float* dp_out_f = (cp == m.nd - 1) ? s.d_s : k.pp[cp % 2];
        const bf16* dp_out_b = (cp == m.nd - 1) ? s.d_s_bf : k.pp_bf[cp % 2];
        const bf16* dp_out_lo = (cp == m.nd - 1) ? s.d_s_bflo : k.pp_bflo[cp % 2];
        (void)dp_out_f;
        {  // conv2 dgrad -> d_c1 (mask of conv1's activation)
          Epi e = epi0(c.lrelu_slope);
          e.act_kind = c.activation;
          e.mask_src = snake ? k.a2_pre[cp] : k.a2_bf[cp];
          e.mask_lo = snake ? k.a2_prelo[cp] : nullptr;
          e.mask_alpha = alpha_ptr(m, "dec.resblocks." + R + ".alpha2." + P);
          e.alpha_part = k.ap2[cp];
          e.out_bf16 = k.d_c1;
          e.out_bf16_lo = k.d_c1_lo;
          e.colsum = k.cs_dc1[cp];
          ConvGeom g{B, s.T, s.T, s.C, s.C, kk, 1, (kk - 1) / 2};
          if (!plan_dgrad(m, k.d2[cp], g, dp_out_b, dp_out_lo, k.w2[cp], e)) return false;
          if (k.d2[cp].partials() > 4 * k.tiles) return false;  // partial buffers hold 4 * tiles rows
        }
        {  // conv2 wgrad
          ConvGeom g{B, s.T, s.T, s.C, s.C, kk, 1, (kk - 1) / 2};
          if (!plan_wgrad_job(m, k.g2[cp], g, dp_out_b, dp_out_lo, k.a2_bf[cp], k.a2_bflo[cp], k.w2[cp]))
            return false;
        }
        {  // conv1 dgrad -> gradient wrt the pair input
          Epi e = epi0(c.lrelu_slope);
          e.act_kind = c.activation;
          e.mask_src = snake ? k.a1_pre[cp] : k.a1_bf[cp];
          e.mask_lo = snake ? k.a1_prelo[cp] : nullptr;
          e.mask_alpha = alpha_ptr(m, "dec.resblocks." + R + ".alpha1." + P);
          e.alpha_part = k.ap1[cp];
          e.res = (cp == m.nd - 1) ? s.d_s : k.pp[cp % 2];
          e.colsum = k.cs_dp[cp];
          if (cp > 0) {
            e.out_f32 = k.pp[(cp - 1) % 2];
            e.out_bf16 = k.pp_bf[(cp - 1) % 2];
            e.out_bf16_lo = k.pp_bflo[(cp - 1) % 2];
          } else {
            e.out_f32 = s.d_x;
            e.accumulate = j > 0;
            e.out_bf16 = (j == m.nk - 1) ? s.d_x_bf : nullptr;
            e.out_bf16_lo = (j == m.nk - 1) ? s.d_x_bflo : nullptr;
          }
          ConvGeom g{B, s.T, s.T, s.C, s.C, kk, dil, dil * (kk - 1) / 2};
          if (!plan_dgrad(m, k.d1[cp], g, k.d_c1, k.d_c1_lo, k.w1[cp], e)) return false;
          if (k.d1[cp].partials() > 4 * k.tiles) return false;
        }
        {  // conv1 wgrad
          ConvGeom g{B, s.T, s.T, s.C, s.C, kk, dil, dil * (kk - 1) / 2};
          if (!plan_wgrad_job(m, k.g1[cp], g, k.d_c1, k.d_c1_lo, k.a1_bf[cp], k.a1_bflo[cp], k.w1[cp])) return false;
        }
      }
    }
    // ups L input gradient -> gradient wrt the previous stage output (or conv_pre output)
    {
      const int Tin = (L == 0) ? m.F : m.sg[L - 1].T;
      Epi e = epi0(c.lrelu_slope);
      e.act_kind = c.activation;
      e.mask_alpha = alpha_ptr(m, "dec.ups_act." + std::to_string(L) + ".alpha");
      const int tiles = B * ((Tin + 127) / 128);
      if (snake && !dalloc(m, &s.ap_up, (size_t)tiles * s.Cin)) return false;
      s.ap_up_tiles = tiles;
      e.alpha_part = s.ap_up;
      if (L > 0) {
        StageBufs& pv = m.sg[L - 1];
        e.mask_src = snake ? pv.s_pre : pv.sa_bf;
        e.mask_lo = snake ? pv.s_prelo : nullptr;
        e.scale = 1.f / (float)m.nk;
        e.out_f32 = pv.d_s;
        e.out_bf16 = pv.d_s_bf;
        e.out_bf16_lo = pv.d_s_bflo;
        if (!dalloc(m, &pv.cs_ds, (size_t)tiles * pv.C)) return false;
        pv.cs_ds_tiles = tiles;
        e.colsum = pv.cs_ds;
      } else {
        e.mask_src = snake ? m.pre_pre : m.pre_bf;
        e.mask_lo = snake ? m.pre_prelo : nullptr;
        e.out_bf16 = m.d_pre_bf;
        e.out_bf16_lo = m.d_pre_bflo;
        if (!dalloc(m, &m.cs_pre, (size_t)tiles * C0)) return false;
        m.cs_pre_tiles = tiles;
        m.pre_tiles_per_item = (Tin + 127) / 128;
        e.colsum = m.cs_pre;
      }
      if (!plan_convT_dgrad(s.up_dg, B, Tin, s.Cin, s.C, s.ku, s.su, s.pu, s.d_x_bf, s.wu.dg,
                            m.fp32 ? s.d_x_bflo : nullptr, m.fp32 ? s.wu.dg_lo : nullptr, e, m.err))
        return false;
      const bf16* xin = (L == 0) ? m.pre_bf : m.sg[L - 1].sa_bf;
      const bf16* xin_lo = (L == 0) ? m.pre_bflo : m.sg[L - 1].sa_bflo;
      WgradJob& j = s.up_wg;
      j.nl = m.fp32 ? 3 : 1;
      if (!plan_convT_wgrad(j.L, B, Tin, s.Cin, s.C, s.ku, s.su, s.pu, xin, s.d_x_bf, nullptr, ~size_t(0),
                            kWgradCtas, m.err))
        return false;
      if (m.fp32 && (!plan_convT_wgrad(j.lo[0], B, Tin, s.Cin, s.C, s.ku, s.su, s.pu, xin_lo, s.d_x_bf, nullptr,
                                       ~size_t(0), kWgradCtas, m.err) ||
                     !plan_convT_wgrad(j.lo[1], B, Tin, s.Cin, s.C, s.ku, s.su, s.pu, xin, s.d_x_bflo, nullptr,
                                       ~size_t(0), kWgradCtas, m.err)))
        return false;
      if (!make_wgrad_job(m, j, 1, s.C, s.ku, s.wu)) return false;
    }
  }
  {  // conv_pre wgrad
    ConvGeom g{B, m.F, m.F, c.in_channels, C0, 7, 1, 3};
    if (!plan_wgrad_job(m, m.pre_wg, g, m.d_pre_bf, m.d_pre_bflo, m.z_bf, m.z_bflo, m.wpre)) return false;
  }
  // ---- batched per-stage reductions ----
  for (int L = 0; L < 4; ++L) {
    StageBufs& s = m.sg[L];
    // the stacks accumulate their input gradients into d_x in order; the last stack's epilogue
    // takes the column sums of the finished sum (the ups bias gradient), the others none
    const int slot = s.st[m.nk - 1].d1[0].partials();
    if (!dalloc(m, &s.cs_dx, (size_t)slot * s.C)) return false;
    for (int j = 0; j < m.nk; ++j) {
      s.st[j].cs_dp[0] = (j == m.nk - 1) ? s.cs_dx : nullptr;
      s.st[j].d1[0].set_colsum(s.st[j].cs_dp[0]);
    }
    // weight gradients in execution order, grouped while their partials fit the L2 budget
    std::vector<WgradJob*> jobs;
    for (int j = 0; j < m.nk; ++j)
      for (int cp = m.nd - 1; cp >= 0; --cp) {
        jobs.push_back(&s.st[j].g2[cp]);
        jobs.push_back(&s.st[j].g1[cp]);
      }
    jobs.push_back(&s.up_wg);
    {
      std::vector<ReduceDesc> wg;
      std::vector<WnDesc> wn;
      size_t bytes = 0;
      for (size_t i = 0; i < jobs.size(); ++i) {
        WgradJob& jb = *jobs[i];
        wg.push_back(wgrad_desc(m, jb));
        if (jb.w->pg >= 0) wn.push_back(wn_desc(m, *jb.w));
        bytes += job_part_floats(jb) * sizeof(float);
        const size_t next = i + 1 < jobs.size() ? job_part_floats(*jobs[i + 1]) * sizeof(float) : 0;
        if (i + 1 == jobs.size() || bytes + next > kWgBatchBytes) {
          WgradBatch bt;
          if (!upload_reduce_table(m, wg, &bt.wg_d, &bt.wg_n, &bt.wg_blocks) ||
              !upload_wn_table(m, wn, &bt.wn_d, &bt.wn_n, &bt.wn_rows))
            return false;
          jb.flush = (int)s.wg_batches.size();
          s.wg_batches.push_back(bt);
          wg.clear();
          wn.clear();
          bytes = 0;
        }
      }
    }
    std::vector<ReduceDesc> cs;
    for (int j = 0; j < m.nk; ++j) {
      StackBufs& k = s.st[j];
      const std::string R = std::to_string(L * m.nk + j);
      for (int cp = m.nd - 1; cp >= 0; --cp) {
        const std::string P = std::to_string(cp);
        cs.push_back(colsum_desc(k.cs_dc1[cp], k.d2[cp].partials(), s.C, m.G(k.w1[cp].pb)));
        if (cp == m.nd - 1)
          cs.push_back(colsum_desc(s.cs_ds, s.cs_ds_tiles, s.C, m.G(k.w2[cp].pb)));
        else
          cs.push_back(colsum_desc(k.cs_dp[cp + 1], k.d1[cp + 1].partials(), s.C, m.G(k.w2[cp].pb)));
        if (snake) {
          cs.push_back(colsum_desc(k.ap1[cp], k.d1[cp].partials(), s.C,
                                   alpha_grad(m, "dec.resblocks." + R + ".alpha1." + P)));
          cs.push_back(colsum_desc(k.ap2[cp], k.d2[cp].partials(), s.C,
                                   alpha_grad(m, "dec.resblocks." + R + ".alpha2." + P)));
        }
      }
    }
    cs.push_back(colsum_desc(s.cs_dx, slot, s.C, m.G(m.pidx("dec.ups." + std::to_string(L) + ".bias"))));
    if (snake)
      cs.push_back(
          colsum_desc(s.ap_up, s.ap_up_tiles, s.Cin, alpha_grad(m, "dec.ups_act." + std::to_string(L) + ".alpha")));
    if (!upload_reduce_table(m, cs, &s.cs_d, &s.cs_n, &s.cs_blocks)) return false;
  }
  m.red_scratch_n = (size_t)4 << 20;
  if (!dalloc(m, &m.red_scratch, m.red_scratch_n)) return false;
  if (m.noise_scratch_n && !dalloc(m, &m.noise_scratch, m.noise_scratch_n)) return false;
  // Programmatic dependent launch for the tensor-core kernels of the step: each waits for its
  // predecessor before touching activations; the persistent resblock kernels also load their weights
  // and epilogue vectors first (prepared at the start of the step, written by no neighbouring kernel)
  for (int L = 0; L < 4; ++L) {
    StageBufs& s = m.sg[L];
    for (int j = 0; j < m.nk; ++j)
      for (int cp = 0; cp < m.nd; ++cp) {
        StackBufs& k = s.st[j];
        k.f1[cp].set_pdl(true);
        k.f2[cp].set_pdl(true);
        k.d1[cp].set_pdl(true);
        k.d2[cp].set_pdl(true);
        for (WgradJob* wj : {&k.g1[cp], &k.g2[cp]}) {
          wj->L.p.pdl = 1;
          wj->lo[0].p.pdl = wj->lo[1].p.pdl = 1;
        }
      }
    s.up_fwd.p.pdl = 1;
    s.up_dg.p.pdl = 1;
    s.up_wg.L.p.pdl = 1;
    s.up_wg.lo[0].p.pdl = s.up_wg.lo[1].p.pdl = 1;
  }
  m.pre_fwd.p.pdl = 1;
  m.pre_wg.L.p.pdl = 1;
  m.pre_wg.lo[0].p.pdl = m.pre_wg.lo[1].p.pdl = 1;
  {  // weight preparation table: every GEMM weight, two launches per step
    std::vector<PrepDesc> d;
    int nb = 0, tb = 0;
    auto add = [&](const ConvWeights& w) -> bool {
      PrepDesc p{};
      p.v = m.P(w.pv);
      p.g = w.pg >= 0 ? m.P(w.pg) : nullptr;
      p.norm = w.norm;
      p.fwd_hi = w.fwd_hi;
      p.fwd_lo = w.fwd_lo;
      p.range_err = m.err;
      p.dg = w.dg;
      p.dg_lo = w.dg_lo;
      p.P = w.convT ? w.cols : w.rows;
      p.Q = w.convT ? w.rows : w.cols;
      p.k = w.k;
      p.is_convT = w.convT;
      p.stride = w.stride;
      if (p.P % 32 || p.Q % 32) {
        fprintf(stderr, "wuburvc_b200: weight %d x %d not a multiple of 32 channels\n", p.P, p.Q);
        return false;
      }
      p.qs = p.Q % 128 == 0 ? 4 : p.Q % 64 == 0 ? 2 : 1;
      p.nchunks = (p.k * p.P + kPrepPairs - 1) / kPrepPairs;
      if (p.g && p.is_convT && !dalloc(m, &p.npart, (size_t)p.nchunks * p.Q)) return false;
      p.norm_first = nb;
      p.tile_first = tb;
      nb += prep_norm_blocks(p);
      tb += prep_tile_blocks(p);
      d.push_back(p);
      m.all_weights.push_back(&w);
      return true;
    };
    if (!add(m.wpre)) return false;
    for (int L = 0; L < 4; ++L) {
      if (!add(m.sg[L].wu)) return false;
      for (int j = 0; j < m.nk; ++j)
        for (int cp = 0; cp < m.nd; ++cp)
          if (!add(m.sg[L].st[j].w1[cp]) || !add(m.sg[L].st[j].w2[cp])) return false;
    }
    m.n_prep = (int)d.size();
    m.prep_norm_blocks = nb;
    m.prep_tile_blocks = tb;
    if (!dalloc(m, &m.prep_descs, d.size())) return false;
    CK(cudaMemcpy(m.prep_descs, d.data(), d.size() * sizeof(PrepDesc), cudaMemcpyHostToDevice));
    m.prep_host = d;
  }
  return true;
}

// Forward operand format of every producer and forward GEMM (see Gen::op_bf16).  The step graph is
// released: the next step captures it again with the new format.
bool gen_set_operand_format(Gen& m, int bf16) {
  m.op_bf16 = bf16 ? 1 : 0;
  if (m.op_bf16) m.fast = 0;  // single fp16 operands have the same range limit: back to the pairs
  auto conv = [&](TcConvParams& p) {
    p.split_bf16 = m.op_bf16;
    p.epi.act_bf16pair = m.op_bf16;
  };
  auto conv2 = [&](TcConv2Params& p) {
    p.split_bf16 = m.op_bf16;
    p.epi.act_bf16pair = m.op_bf16;
  };
  conv(m.pre_fwd.p);
  for (int L = 0; L < 4; ++L) {
    StageBufs& s = m.sg[L];
    conv(s.up_fwd.p);
    for (int j = 0; j < m.nk; ++j)
      for (int cp = 0; cp < m.nd; ++cp)
        for (ConvOp* op : {&s.st[j].f1[cp], &s.st[j].f2[cp]}) {
          conv(op->v1.p);
          conv2(op->c2.p);
        }
  }
  for (auto& d : m.prep_host) d.fmt_bf16 = m.op_bf16;
  CK(cudaStreamSynchronize(m.stream));
  CK(cudaMemcpy(m.prep_descs, m.prep_host.data(), m.prep_host.size() * sizeof(PrepDesc), cudaMemcpyHostToDevice));
  if (m.graph) cudaGraphExecDestroy(m.graph);
  m.graph = nullptr;
  return true;
}

namespace {
// The fast-inference forward plans: the regular forward's epilogues (in their forward-only form) on
// single fp16 operands, the operand's hi half alone (the lo half is neither read nor written).
bool plan_fast(Gen& m) {
  const WubuB200GenConfig& c = m.cfg;
  const int B = m.B, C0 = c.initial_channel;
  auto single = [](TcConvParams& p) { p.single_f16 = 1; };
  {
    Epi e = m.pre_fwd.p.epi;
    e.act_lo = nullptr;
    ConvGeom g{B, m.F, m.F, c.in_channels, C0, 7, 1, 3};
    if (!plan_conv(m.pre_fast, g, m.z_hi, nullptr, m.wpre.fwd_hi, nullptr, 0, e, m.err)) return false;
    single(m.pre_fast.p);
    m.pre_fast.p.pdl = 1;
  }
  for (int L = 0; L < 4; ++L) {
    StageBufs& s = m.sg[L];
    const int Tin = (L == 0) ? m.F : m.sg[L - 1].T;
    const f16* in_hi = (L == 0) ? m.pre_hi : m.sg[L - 1].sa_hi;
    Epi eu = s.up_fwd.p.epi;
    if (!plan_convT(s.up_fast, B, Tin, s.Cin, s.C, s.ku, s.su, s.pu, in_hi, nullptr, s.wu.fwd_hi, nullptr, 0, eu,
                    m.err))
      return false;
    single(s.up_fast.p);
    s.up_fast.p.pdl = 1;
    for (int j = 0; j < m.nk; ++j) {
      StackBufs& k = s.st[j];
      const int kk = c.resblock_kernels[j];
      for (int cp = 0; cp < m.nd; ++cp) {
        const int dil = c.resblock_dilations[j][cp];
        for (int which = 0; which < 2; ++which) {
          ConvOp& src = which ? k.f2[cp] : k.f1[cp];
          ConvOp& dst = which ? k.f2f[cp] : k.f1f[cp];
          Epi e = src.v2 ? src.c2.p.epi : src.v1.p.epi;
          e.act_lo = nullptr;
          const ConvGeom g = which ? ConvGeom{B, s.T, s.T, s.C, s.C, kk, 1, (kk - 1) / 2}
                                   : ConvGeom{B, s.T, s.T, s.C, s.C, kk, dil, dil * (kk - 1) / 2};
          const f16* x = which ? k.a2_hi[cp] : k.a1_hi[cp];
          const ConvWeights& w = which ? k.w2[cp] : k.w1[cp];
          if (!plan_conv_any(dst, g, x, nullptr, w.fwd_hi, nullptr, 0, e, m.err)) return false;
          single(dst.v1.p);
          dst.c2.p.single_f16 = 1;
          dst.set_pdl(true);
        }
      }
    }
  }
  m.fast_planned = true;
  return true;
}
}  // namespace

// Forward-only mode (see Gen::forward_only): the forward plans and the weight preparation stop (or
// resume) writing the tensors only the backward reads; on = 2 also selects the fast-inference plans.
// The step graph is released.
bool gen_set_forward_only(Gen& m, int on) {
  m.forward_only = on ? 1 : 0;
  auto act = [&](Epi& e, bf16* bf, bf16* bflo, bf16* pre, bf16* prelo) {
    e.act_bf = on ? nullptr : bf;
    e.act_bflo = on ? nullptr : bflo;
    e.pre_hi = on ? nullptr : pre;
    e.pre_lo = on ? nullptr : prelo;
  };
  auto both = [&](ConvOp& op, bf16* bf, bf16* bflo, bf16* pre, bf16* prelo) {
    act(op.v1.p.epi, bf, bflo, pre, prelo);
    act(op.c2.p.epi, bf, bflo, pre, prelo);
  };
  act(m.pre_fwd.p.epi, m.pre_bf, m.pre_bflo, m.pre_pre, m.pre_prelo);
  for (int L = 0; L < 4; ++L) {
    StageBufs& s = m.sg[L];
    for (int j = 0; j < m.nk; ++j) {
      StackBufs& k = s.st[j];
      for (int cp = 0; cp < m.nd; ++cp) {
        both(k.f1[cp], k.a2_bf[cp], k.a2_bflo[cp], k.a2_pre[cp], k.a2_prelo[cp]);
        if (cp + 1 < m.nd)
          both(k.f2[cp], k.a1_bf[cp + 1], k.a1_bflo[cp + 1], k.a1_pre[cp + 1], k.a1_prelo[cp + 1]);
        else if (j == m.nk - 1)
          both(k.f2[cp], s.sa_bf, s.sa_bflo, s.s_pre, s.s_prelo);
      }
    }
  }
  CK(cudaStreamSynchronize(m.stream));
  if (m.prep_host.size() != m.all_weights.size()) return false;
  for (size_t i = 0; i < m.prep_host.size(); ++i) {
    m.prep_host[i].dg = on ? nullptr : m.all_weights[i]->dg;
    m.prep_host[i].dg_lo = on ? nullptr : m.all_weights[i]->dg_lo;
  }
  CK(cudaMemcpy(m.prep_descs, m.prep_host.data(), m.prep_host.size() * sizeof(PrepDesc), cudaMemcpyHostToDevice));
  if (m.graph) cudaGraphExecDestroy(m.graph);
  m.graph = nullptr;
  // the fast plans copy the forward-only epilogues above; a context whose operands fell back to bf16
  // pairs after a range error stays on those
  m.fast = 0;
  if (on == 2 && !m.op_bf16) {
    if (!m.fast_planned && !plan_fast(m)) return false;
    m.fast = 1;
  }
  return true;
}

// =============================================================================================
// forward
// =============================================================================================
bool gen_forward(Gen& m) {
  const WubuB200GenConfig& c = m.cfg;
  const bool snake = c.activation == 1;
  cudaStream_t st = m.stream;
  set_reduce_scratch(m.red_scratch, m.red_scratch_n);
  // GEMM weights for this step (weight norm + bf16 hi/lo + transposed layouts)
  prep_weights(m.prep_descs, m.n_prep, m.prep_norm_blocks, m.prep_tile_blocks, st);
  pack_z(m.z, m.B, c.in_channels, m.F, m.z_hi, m.z_lo, m.forward_only ? nullptr : m.z_bf,
         m.forward_only ? nullptr : m.z_bflo, m.err, m.op_bf16, st);
  if (c.nsf) {
    NsfArgs a{};
    a.f0 = m.f0;
    a.noise = m.has_noise_input ? m.noise : nullptr;
    a.lin_w = m.P(m.pidx("dec.m_source.l_linear.weight"));
    a.lin_b = m.P(m.pidx("dec.m_source.l_linear.bias"));
    a.har = m.har;
    a.sw = m.sw;
    a.acc = m.nsf_acc;
    a.B = m.B;
    a.F = m.F;
    a.upp = m.upp;
    a.dim = m.dim;
    a.sr = (float)c.sample_rate;
    a.sine_amp = c.sine_amp;
    a.noise_std = c.noise_std;
    a.seed = m.opt.seed;
    a.stream = &m.state->noise_stream;
    nsf_forward(a, st);
  }
  if (c.gin_channels)
    cond_forward(m.P(m.pidx("dec.cond.weight")), m.P(m.pidx("dec.cond.bias")), m.g, m.B, c.initial_channel,
                 c.gin_channels, m.rowadd, st);
  CK((m.fast ? m.pre_fast : m.pre_fwd).run(st));
  for (int L = 0; L < 4; ++L) {
    StageBufs& s = m.sg[L];
    CK((m.fast ? s.up_fast : s.up_fwd).run(st));
    NoiseActArgs na{};
    na.x = s.x_in;
    na.har = c.nsf ? m.har : nullptr;
    if (c.nsf) {
      transpose_ck(m.P(m.pidx("dec.noise_convs." + std::to_string(L) + ".weight")), s.C, s.kn, s.noise_wt, st);
      na.w = s.noise_wt;
      na.bias = m.P(m.pidx("dec.noise_convs." + std::to_string(L) + ".bias"));
    }
    na.B = m.B;
    na.T = s.T;
    na.C = s.C;
    na.k = s.kn;
    na.stride = s.sn;
    na.pad = s.pn;
    na.T_full = m.T;
    na.act_kind = c.activation;
    na.slope = c.lrelu_slope;
    na.n_act = snake ? m.nk : 1;
    for (int q = 0; q < na.n_act; ++q) {
      na.alpha[q] = snake ? alpha_ptr(m, "dec.resblocks." + std::to_string(L * m.nk + q) + ".alpha1.0") : nullptr;
      na.act_hi[q] = s.xa_hi[q];
      na.act_lo[q] = s.xa_lo[q];
      na.act_bf[q] = m.forward_only ? nullptr : s.xa_bf[q];
      na.act_bflo[q] = m.forward_only ? nullptr : s.xa_bflo[q];
    }
    na.pre = m.forward_only ? nullptr : s.x_pre;
    na.pre_lo = m.forward_only ? nullptr : s.x_prelo;
    na.range_err = m.err;
    na.fmt_bf16 = m.op_bf16;
    noise_add_act(na, st);
    for (int j = 0; j < m.nk; ++j)
      for (int cp = 0; cp < m.nd; ++cp) {
        CK((m.fast ? s.st[j].f1f[cp] : s.st[j].f1[cp]).run(st));
        CK((m.fast ? s.st[j].f2f[cp] : s.st[j].f2[cp]).run(st));
      }
  }
  post_forward(m.sg[3].sa_hi, m.fast ? nullptr : m.sg[3].sa_lo, m.op_bf16, m.P(m.pidx("dec.conv_post.weight")), m.B, m.T, m.sg[3].C, 7, m.audio,
               st);
  return true;
}

// =============================================================================================
// backward
// =============================================================================================
bool gen_backward(Gen& m) {
  m.ev_next = 0;
  const WubuB200GenConfig& c = m.cfg;
  const bool snake = c.activation == 1;
  cudaStream_t st = m.stream;
  const int B = m.B;
  set_reduce_scratch(m.red_scratch, m.red_scratch_n);
  {  // conv_post + tanh backward -> gradient wrt stage 3 output (/nk per stack)
    StageBufs& s3 = m.sg[3];
    PostBwdArgs a{};
    a.dy = m.dldy;
    a.audio = m.audio;
    a.W = m.P(m.pidx("dec.conv_post.weight"));
    a.a_hi = s3.sa_hi;
    a.a_lo = s3.sa_lo;
    a.fmt_bf16 = m.op_bf16;
    a.mask_src = snake ? s3.s_pre : s3.sa_bf;
    a.mask_lo = snake ? s3.s_prelo : nullptr;
    a.alpha = alpha_ptr(m, "dec.post_act.alpha");
    a.act_kind = c.activation;
    a.slope = c.final_slope;
    a.scale = 1.f / (float)m.nk;
    a.B = B;
    a.T = m.T;
    a.C = s3.C;
    a.k = 7;
    a.d_stage = s3.d_s;
    a.d_stage_bf = s3.d_s_bf;
    a.d_stage_bf_lo = s3.d_s_bflo;
    a.colsum_part = m.post_cs;
    a.w_part = m.post_wpart;
    a.alpha_part = m.post_ap;
    post_backward(a, st);
    rows_reduce(m.post_wpart, m.post_blocks, s3.C * 7, m.G(m.pidx("dec.conv_post.weight")), 0, st);
    if (snake) rows_reduce(m.post_ap, m.post_blocks, s3.C, alpha_grad(m, "dec.post_act.alpha"), 0, st);
  }
  for (int L = 3; L >= 0; --L) {
    StageBufs& s = m.sg[L];
    for (int j = 0; j < m.nk; ++j) {
      StackBufs& k = s.st[j];
      for (int cp = m.nd - 1; cp >= 0; --cp) {
        CK(k.d2[cp].run(st));
        if (!run_wgrad(m, s, k.g2[cp])) return false;
        CK(k.d1[cp].run(st));
        if (!run_wgrad(m, s, k.g1[cp])) return false;
      }
    }
    // stage input gradient d_x: noise conv (side stream: it only reads d_x and feeds the source
    // gradient at the end of the backward), ups dgrad / wgrad
    if (c.nsf) {
      const int nw = m.pidx("dec.noise_convs." + std::to_string(L) + ".weight");
      if (!fork_side(m)) return false;
      noise_backward(s.d_x, m.har, s.noise_wt, B, s.T, s.C, s.kn, s.sn, s.pn, m.T, m.d_har, L < 3, s.noise_wpart,
                     s.noise_g, m.side);
      noise_wgrad_reduce(s.noise_wpart, s.noise_parts, s.C, s.kn, m.G(nw), m.noise_scratch, m.noise_scratch_n,
                         m.side);
    }
    CK(s.up_dg.run(st));
    if (!run_wgrad(m, s, s.up_wg)) return false;
    // every bias / Snake-alpha gradient of the stage, on the side stream after the stage's kernels
    if (!fork_side(m)) return false;
    reduce_batched(s.cs_d, s.cs_n, s.cs_blocks, m.side);
    if (c.nsf) {  // the noise conv's bias is added where the ups bias is: same gradient
      const int ub = m.pidx("dec.ups." + std::to_string(L) + ".bias");
      const int nb = m.pidx("dec.noise_convs." + std::to_string(L) + ".bias");
      CK(cudaMemcpyAsync(m.G(nb), m.G(ub), sizeof(float) * s.C, cudaMemcpyDeviceToDevice, m.side));
    }
    // this stage's gradients are final once the side stream gets here (noise-conv weight gradient
    // and everything before the fork are on the main stream, which the side stream waited for)
    if (comm_bucket_ready(m, 3 - L, m.side)) return false;
  }
  // conv_pre, cond, source
  if (!run_pre_wgrad(m)) return false;
  colsum_reduce(m.cs_pre, m.cs_pre_tiles, c.initial_channel, m.G(m.wpre.pb), 0, st);
  if (c.gin_channels)
    cond_backward(m.cs_pre, m.pre_tiles_per_item, B, c.initial_channel, m.g, c.gin_channels,
                  m.G(m.pidx("dec.cond.weight")), m.G(m.pidx("dec.cond.bias")), st);
  if (c.nsf && !join_side(m)) return false;  // d_har is complete on the side stream
  if (c.nsf)
    nsf_backward(m.d_har, m.har, m.sw, B * m.T, m.dim, m.nsf_part, m.nsf_parts,
                 m.G(m.pidx("dec.m_source.l_linear.weight")), m.G(m.pidx("dec.m_source.l_linear.bias")), st);
  if (comm_bucket_ready(m, 4, m.stream) || comm_join(m)) return false;
  return join_side(m);  // AdamW (main stream) needs every reduction
}

bool gen_adamw(Gen& m, float grad_scale, int bump_noise) {
  // under data parallelism the ranks' range flags arrive summed in the slot after the gradients
  const float* flag = comm_world(m) > 1 ? m.grads + m.table.total : nullptr;
  step_bump(m.state, bump_noise, m.err, flag, m.stream);
  adamw(m.params, m.grads, m.adam_m, m.adam_v, m.table.total, m.opt.lr, m.opt.beta1, m.opt.beta2, m.opt.eps,
        m.opt.weight_decay, m.state, grad_scale, m.err, flag, m.stream);
  return cudaGetLastError() == cudaSuccess;
}

void gen_free(Gen& m) {
  if (m.stream) cudaStreamSynchronize(m.stream);
  // the captured step holds the NCCL all-reduces: release it before the communicator
  if (m.graph) cudaGraphExecDestroy(m.graph);
  m.graph = nullptr;
  comm_destroy(m);
  if (m.side) {
    cudaStreamSynchronize(m.side);
    cudaStreamDestroy(m.side);
    m.side = nullptr;
  }
  for (auto e : m.evs) cudaEventDestroy(e);
  m.evs.clear();
  for (void* p : m.allocs) cudaFree(p);
  m.allocs.clear();
  if (m.stream) cudaStreamDestroy(m.stream);
  m.stream = nullptr;
}

}  // namespace wb
