// tc_conv2.cu — persistent, halo-reusing tcgen05 implicit-GEMM for stride-1 Conv1d (forward and
// input-gradient), the MRF resblock convolutions that carry ~97% of the step's FLOPs.
#include "tc_epilogue.cuh"

namespace wb {

namespace {

WB_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

}  // namespace

// Warp roles: 0..7 epilogue (warp w reads TMEM lane quadrant w%4 and column half w/4), 8 TMA producer,
// 9 TMEM allocation + MMA issue.
constexpr int kConv2Threads = 320;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;

// Shared memory: [A stages][W stages or resident W][barriers].  A stage = halo tile (hi[, lo]) of one
// channel chunk (R x KC, swizzled); a weight stage holds `w_group` taps of one chunk, each tap hi[, lo]
// (N x KC, swizzled);
// resident weights hold every (chunk, tap) of the CTA's N tile in the same per-tap layout, loaded once.
template <int KC, bool SPLIT, uint32_t F>
__global__ void __launch_bounds__(kConv2Threads, 1)
    tc_conv2_kernel(const __grid_constant__ TcConv2Maps maps, const __grid_constant__ TcConv2Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ float red[2][128];
  // epilogue vectors of this CTA's N tile, and the groups' running column sums
  __shared__ __align__(16) float s_bias[256], s_aalpha[256], s_malpha[256];
  __shared__ float s_csum[2][256], s_asum[2][256];
  __shared__ uint4 s_stage[8][128];  // per epilogue warp: 32 rows x 64 B of outgoing data

  constexpr int nA = SPLIT ? 2 : 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int N = p.n;
  const int ntaps = p.ntaps, nch = p.n_chunks, G = p.w_group, dil = p.dil;
  const bool resident = p.w_resident != 0;
  const int ngroups = resident ? 1 : (ntaps + G - 1) / G;
  const uint32_t a_sub = p.a_sub_bytes;
  const uint32_t a_stage = nA * a_sub;
  const uint32_t w_sub = (uint32_t)N * KC * 2u;  // one tap, hi or lo
  const uint32_t w_tap = nA * w_sub;
  const uint32_t w_stage = resident ? (uint32_t)(nch * ntaps) * w_tap : (uint32_t)G * w_tap;
  const int AS = p.a_stages, WS = resident ? 1 : p.w_stages;

  uint8_t* a_base = smem;
  uint8_t* w_base = smem + (size_t)AS * a_stage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(w_base + (size_t)WS * w_stage);
  uint64_t* a_full = bars;
  uint64_t* a_empty = a_full + AS;
  uint64_t* w_full = a_empty + AS;
  uint64_t* w_empty = w_full + WS;
  uint64_t* acc_full = w_empty + WS;   // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint64_t* mma_done = acc_empty + 2;  // every MMA of the CTA complete (drained before TMEM is freed)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < AS; ++s) { mbar_init(&a_full[s], 1); mbar_init(&a_empty[s], 1); }
    for (int s = 0; s < WS; ++s) { mbar_init(&w_full[s], 1); mbar_init(&w_empty[s], 1); }
    // an accumulator is free again once every epilogue group that reads it has arrived (see below)
    const uint32_t acc_readers = N >= 64 ? 2u : 1u;
    for (int b = 0; b < 2; ++b) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], acc_readers); }
    mbar_init(mma_done, 1);
    fence_barrier_init();
  }
  if (warp == kMmaWarp) tmem_alloc(tmem_slot, (uint32_t)p.tmem_cols);
  if (threadIdx.x < 256) {
    const int i = threadIdx.x, col = (blockIdx.x % p.n_tiles) * N + i;
    const bool in_tile = i < N;
    s_bias[i] = (in_tile && p.epi.bias) ? p.epi.bias[col] : 0.f;
    s_aalpha[i] = (in_tile && p.epi.act_alpha) ? p.epi.act_alpha[col] : 1.f;
    s_malpha[i] = (in_tile && p.epi.mask_alpha) ? p.epi.mask_alpha[col] : 1.f;
    s_csum[0][i] = s_csum[1][i] = s_asum[0][i] = s_asum[1][i] = 0.f;
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Producer and MMA roles: whole warps with a warp-uniform `ok` flag instead of early exits (a
  // break out of these loops makes the compiler treat the issuing code as divergent, which costs
  // the MMA issue rate); after a timed-out wait the loops run on without issuing anything.
  if (warp == kProducerWarp) {
    // ---------------- TMA producer ----------------
    bool ok = true;
    FillTrack fa, fw;
    const int n0_cta = (blockIdx.x % p.n_tiles) * N;  // every tile of this CTA has this N tile
    // weight stage u of the CTA's weight sequence (chunk u / ngroups, tap group u % ngroups) into slot s,
    // the slot's phase parity ph
    auto load_w = [&](int u, int s, uint32_t ph) {
      const int c = u / ngroups, t0 = (u % ngroups) * G, nt = min(G, ntaps - t0);
      uint8_t* wd = w_base + (size_t)s * w_stage;
      fw.fill(s, ph);
      mbar_expect_tx_warp(&w_full[s], (uint32_t)nt * w_tap);
      for (int j = 0; j < nt; ++j) {
        tma_load_3d_warp(wd + j * w_tap, &maps.w_hi, &w_full[s], c * KC, n0_cta, t0 + j);
        if (SPLIT) tma_load_3d_warp(wd + j * w_tap + w_sub, &maps.w_lo, &w_full[s], c * KC, n0_cta, t0 + j);
      }
    };
    // the weights are not the previous kernel's output: they go out before the dependency wait
    int w_pre = 0;
    if (resident) {
      mbar_expect_tx_warp(&w_full[0], (uint32_t)(nch * ntaps) * w_tap);
      fw.fill(0, 0);
      for (int c = 0; c < nch; ++c)
        for (int t = 0; t < ntaps; ++t) {
          uint8_t* wd = w_base + (size_t)(c * ntaps + t) * w_tap;
          tma_load_3d_warp(wd, &maps.w_hi, &w_full[0], c * KC, n0_cta, t);
          if (SPLIT) tma_load_3d_warp(wd + w_sub, &maps.w_lo, &w_full[0], c * KC, n0_cta, t);
        }
    } else if (blockIdx.x < p.ntiles) {
      w_pre = min(WS, nch * ngroups);
      for (int u = 0; u < w_pre; ++u) load_w(u, u, 0);
    }
    griddep_wait();
    int sa = 0, sw = 0;
    uint32_t aph = 0, wph = 0;
    int a_uses = 0, w_uses = 0;
    for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x) {
      const int mtile = tile / p.n_tiles;
      const int item = mtile / p.tiles_per_item;
      const int q0 = (mtile - item * p.tiles_per_item) * 128;
      for (int c = 0; c < nch; ++c) {
        if (ok && a_uses >= AS) ok = mbar_wait_warp(&a_empty[sa], aph ^ 1u, p.err, ERR_WAIT_EMPTY, p.wait_ns);
        if (ok) {
          // one swizzled box per operand: R rows of KC channels
          uint8_t* ad = a_base + (size_t)sa * a_stage;
          fa.fill(sa, aph);
          mbar_expect_tx_warp(&a_full[sa], nA * (uint32_t)p.halo_rows * KC * 2u);
          tma_load_3d_warp(ad, &maps.a_hi, &a_full[sa], c * KC, q0 + p.halo_start, item);
          if (SPLIT) tma_load_3d_warp(ad + a_sub, &maps.a_lo, &a_full[sa], c * KC, q0 + p.halo_start, item);
        }
        ++a_uses;
        if (++sa == AS) { sa = 0; aph ^= 1u; }
        if (resident) continue;
        for (int g = 0; g < ngroups; ++g) {
          if (w_uses < w_pre) {  // issued before the dependency wait
            ++w_uses;
            if (++sw == WS) { sw = 0; wph ^= 1u; }
            continue;
          }
          if (ok && w_uses >= WS) ok = mbar_wait_warp(&w_empty[sw], wph ^ 1u, p.err, ERR_WAIT_EMPTY, p.wait_ns);
          if (ok) load_w(c * ngroups + g, sw, wph);
          ++w_uses;
          if (++sw == WS) { sw = 0; wph ^= 1u; }
        }
      }
    }
    // no copy of this CTA may land after it exits
    fa.drain(a_full, p.err, p.wait_ns);
    fw.drain(w_full, p.err, p.wait_ns);
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    // The split product as two MMAs per K16 step: A_hi x [W_hi | W_lo] (N = 2N: the tap's hi and lo
    // weight tiles are adjacent rows in shared memory) into accumulator columns [0, 2N), then A_lo x
    // W_hi added to columns [N, 2N); the epilogue sums the two halves (the second one unscaled).  Fewer operand reads from shared memory than
    // three N-wide MMAs, and a wider (more efficient) first MMA.
    // split pairs: fp16 hi / scaled lo (forward) or bf16 hi / lo; single operands are bf16
    const int fmt_bf16 = SPLIT ? p.split_bf16 : (p.single_f16 ? 0 : 1);
    const uint32_t idesc = make_idesc(128, N, 0, 0, fmt_bf16);
    const uint32_t idesc2 = make_idesc(128, 2 * N, 0, 0, fmt_bf16);
    constexpr uint32_t wlayout = (KC == 64) ? 2u : 4u;
    constexpr uint32_t wsbo = (KC == 64) ? 1024u : 512u;
    // A: the halo tile in the swizzled K-major layout TMA writes (rows of KC channels, 8-row swizzle
    // atoms).  The swizzle is a function of the absolute shared-memory address, so a tap's operand is
    // the same tile started tap*dil rows further on (measured exact for any start row).
    // descriptors are built once; a tap / k-step / stage moves the 14-bit start-address field
    const uint64_t da0 = make_sdesc(smem_u32(a_base), 16, wsbo, wlayout);
    const uint64_t dw0 = make_sdesc(smem_u32(w_base), 16, wsbo, wlayout);
    const uint32_t tap_step = (uint32_t)dil * (KC * 2u / 16u);  // 16-byte units per tap (dil rows)
    const uint32_t k_step_a = 2u;                                 // K16 step = 32 bytes along the row
    bool ok = true;
    if (resident) ok = mbar_wait_warp(&w_full[0], 0, p.err, ERR_WAIT_FULL, p.wait_ns);
    int sa = 0, sw = 0, t_it = 0;
    uint32_t aph = 0, wph = 0;
    bool w_ready = false;  // weight stage sw known complete (polled ahead)
    for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x, ++t_it) {
      const int buf = t_it & 1;
      if (ok && t_it >= 2) ok = mbar_wait_warp(&acc_empty[buf], ((t_it >> 1) & 1) ^ 1, p.err, ERR_WAIT_ACC, p.wait_ns);
      tc_fence_after();
      const uint32_t d = tmem + (uint32_t)(buf * N * nA);  // nA = 2: accumulator of 2N columns
      for (int c = 0; c < nch; ++c) {
        if (ok) ok = mbar_wait_warp(&a_full[sa], aph, p.err, ERR_WAIT_FULL, p.wait_ns);
        const uint64_t dah = da0 + (uint64_t)((sa * a_stage) >> 4);
        const uint64_t dal = dah + (uint64_t)(a_sub >> 4);
        // one tap: KC/16 K16 steps, 2 MMAs each under the split (3 products)
        auto issue_tap = [&](uint32_t w_off, int t, uint32_t acc0) {
          const uint64_t dwh = dw0 + (uint64_t)(w_off >> 4);
          const uint64_t dwl = dwh + (uint64_t)(w_sub >> 4);
          const uint32_t at = (uint32_t)t * tap_step;
#pragma unroll
          for (int k = 0; k < KC / 16; ++k) {
            const uint64_t ao = at + (uint32_t)k * k_step_a;
            if (SPLIT) {
              umma_f16_warp(d, dah + ao, dwh + 2u * k, idesc2, k ? 1u : acc0);
              umma_f16_warp(d + (uint32_t)N, dal + ao, dwh + 2u * k, idesc, 1);
            } else {
              umma_f16_warp(d, dah + ao, dwh + 2u * k, idesc, k ? 1u : acc0);
            }
          }
          (void)dwl;
        };
        if (resident) {
          if (ok) {
            const uint32_t wst = (uint32_t)(c * ntaps) * w_tap;
            for (int t = 0; t < ntaps; ++t) issue_tap(wst + (uint32_t)t * w_tap, t, (c | t) ? 1u : 0u);
          }
        } else {
          for (int g = 0; g < ngroups; ++g) {
            const int t0 = g * G, nt = min(G, ntaps - t0);
            if (ok && !w_ready) ok = mbar_wait_warp(&w_full[sw], wph, p.err, ERR_WAIT_FULL, p.wait_ns);
            // look at the next weight stage now, so its (usually complete) wait is off the issue path
            int sw2 = sw + 1;
            uint32_t ph2 = wph;
            if (sw2 == WS) { sw2 = 0; ph2 ^= 1u; }
            w_ready = mbar_poll_warp(&w_full[sw2], ph2);
            if (ok) {
              const uint32_t wst = (uint32_t)sw * w_stage;
              for (int j = 0; j < nt; ++j) issue_tap(wst + (uint32_t)j * w_tap, t0 + j, (c | t0 | j) ? 1u : 0u);
              umma_commit_warp(&w_empty[sw]);
            }
            sw = sw2;
            wph = ph2;
          }
        }
        if (ok) umma_commit_warp(&a_empty[sa]);
        if (++sa == AS) { sa = 0; aph ^= 1u; }
      }
      if (ok) umma_commit_warp(&acc_full[buf]);
    }
    // every MMA this warp issued has completed before TMEM is released (also after a timed-out wait)
    umma_commit_warp(mma_done);
    mbar_wait_warp(mma_done, 0, p.err, ERR_WAIT_ACC, p.wait_ns);
  } else {
    // ---------------- epilogue: two groups of 4 warps (warp w reads TMEM lane quadrant w%4).  With
    // N >= 64 both groups drain every tile, group g the column half g, so a tile's epilogue takes half
    // the time and the last one (which no MMA work hides) ends sooner; with N = 32 (one 32-column
    // chunk) group g drains every other tile, so two tiles' epilogues run concurrently ----------------
    griddep_wait();  // the epilogue inputs and outputs belong to the previous kernels' data
    const int qw = warp & 3, grp = warp >> 2;
    const Epi& e = p.epi;
    const int n0 = (blockIdx.x % p.n_tiles) * N;  // every tile of this CTA has this N tile
    const float* bias = e.bias ? s_bias : nullptr;
    const float* aal = e.act_alpha ? s_aalpha : nullptr;
    const float* mal = e.mask_alpha ? s_malpha : nullptr;
    const bool halves = N >= 64;
    const int c_beg = halves ? grp * (N / 2) : 0, c_end = halves ? c_beg + N / 2 : N;
    int t_it = halves ? 0 : grp;
    bool ok = true;
    for (int tile = blockIdx.x + (halves ? 0 : grp * (int)gridDim.x); tile < p.ntiles;
         tile += (halves ? 1 : 2) * gridDim.x, t_it += halves ? 1 : 2) {
      const int buf = t_it & 1;
      const int mtile = tile / p.n_tiles;
      const int item = mtile / p.tiles_per_item;
      const int q = (mtile - item * p.tiles_per_item) * 128 + qw * 32 + lane;
      const bool valid = q < p.t_rows;
      const size_t row_off = ((size_t)item * p.t_rows + (valid ? q : 0)) * p.n_total + n0;
      const float* ra = e.rowadd ? e.rowadd + (size_t)item * p.n_total + n0 : nullptr;
      const int wrow0 = (mtile - item * p.tiles_per_item) * 128 + qw * 32;  // warp's first output row
      RowOut o;
      o.stage = s_stage[warp];
      o.off0 = ((size_t)item * p.t_rows + wrow0) * p.n_total + n0 + c_beg;
      o.pitch = (size_t)p.n_total;
      o.rows_valid = ok ? max(0, min(32, p.t_rows - wrow0)) : 0;
      o.lane = lane;
      // the first chunk's inputs are in flight while the accumulator is still being computed
      EpiIn in;
      epi_load<F>(e, valid, row_off + c_beg, in);
      if (ok) ok = mbar_wait_warp(&acc_full[buf], (t_it >> 1) & 1, p.err, ERR_WAIT_ACC, p.wait_ns);
      tc_fence_after();
#pragma unroll 1
      for (int c0 = c_beg; c0 < c_end; c0 += 32) {
        float v[32];
        if (ok) {
          const uint32_t ta = tmem + (uint32_t)(buf * N * nA) + ((uint32_t)(qw * 32) << 16) + (uint32_t)c0;
          tmem_ld32(ta, v);
          if (SPLIT) {  // [0, N) holds hi*hi, [N, 2N) hi*lo + lo*hi (scaled by 2^11 in the fp16 format)
            float u[32];
            tmem_ld32(ta + (uint32_t)N, u);
            const float ls = p.split_bf16 ? 1.f : kLoUnscale;
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] += u[i] * ls;
          }
        } else
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0.f;
        // the chunk's named barriers are reached by the whole group whether or not the wait succeeded
        float cs = 0.f, ap = 0.f;
        epi_finish<F>(e, v, in, valid && ok, row_off + c0, 0, ra ? ra + c0 : nullptr, bias ? bias + c0 : nullptr,
                   aal ? aal + c0 : nullptr, mal ? mal + c0 : nullptr, qw, lane, red[grp], &cs, &ap, 1 + grp, true,
                   o, c0 + 32 < c_end, row_off + c0 + 32);
        o.off0 += 32;
        if (qw == 0) {  // column sums accumulate over the group's tiles (warp 0 holds this tile's)
          s_csum[grp][c0 + lane] += cs;
          s_asum[grp][c0 + lane] += ap;
        }
      }
      tc_fence_before();
      asm volatile("bar.sync %0, 128;" ::"r"(3 + grp) : "memory");
      if (qw == 0 && lane == 0) mbar_arrive(&acc_empty[buf]);
    }
    if (qw == 0) {
      // one partial row per group (2 per CTA): its sums in this CTA's N tile (its column half, or
      // every column of its tiles), zeros elsewhere
      const size_t prow = (size_t)(2 * blockIdx.x + grp) * p.n_total;
      for (int c = 0; c < p.n_total; c += 32) {
        const int rel = c - n0;
        const bool mine = rel >= 0 && rel < N;
        if (e.colsum) e.colsum[prow + c + lane] = mine ? s_csum[grp][rel + lane] : 0.f;
        if (e.alpha_part) e.alpha_part[prow + c + lane] = mine ? s_asum[grp][rel + lane] : 0.f;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, (uint32_t)p.tmem_cols);
  }
}

// Instantiated (KC, SPLIT, epilogue feature set) combinations: the forward (split), the fast-inference
// forward (single fp16 operands) and input-gradient epilogues of the resblock convolutions (with and
// without column sums), plus a generic kernel for any other epilogue.
#define WB_CONV2_KERNELS(X)                                                                     \
  X(64, true, kEpiGeneric) X(64, true, kEpiAct) X(64, true, kEpiAct | kEpiSnake)                 \
  X(64, true, kEpiRes | kEpiAct) X(64, true, kEpiRes | kEpiAct | kEpiSnake) X(64, true, kEpiRes)  \
  X(64, true, 0u) X(64, false, kEpiGeneric) X(64, false, kEpiMask | kEpiColsum)                 \
  X(64, false, kEpiMask | kEpiColsum | kEpiSnake) X(64, false, kEpiMask | kEpiRes | kEpiColsum)  \
  X(64, false, kEpiMask | kEpiRes | kEpiColsum | kEpiSnake) X(64, false, kEpiMask | kEpiRes)     \
  X(64, false, kEpiMask | kEpiRes | kEpiSnake) X(64, false, kEpiAct) X(64, false, kEpiRes | kEpiAct) \
  X(64, false, kEpiAct | kEpiSnake) X(64, false, kEpiRes | kEpiAct | kEpiSnake) X(64, false, kEpiRes) \
  X(32, true, kEpiGeneric) X(32, true, kEpiAct) X(32, true, kEpiAct | kEpiSnake)                 \
  X(32, true, kEpiRes | kEpiAct) X(32, true, kEpiRes | kEpiAct | kEpiSnake) X(32, true, kEpiRes)  \
  X(32, true, 0u) X(32, false, kEpiGeneric) X(32, false, kEpiMask | kEpiColsum)                 \
  X(32, false, kEpiMask | kEpiColsum | kEpiSnake) X(32, false, kEpiMask | kEpiRes | kEpiColsum)  \
  X(32, false, kEpiMask | kEpiRes | kEpiColsum | kEpiSnake) X(32, false, kEpiMask | kEpiRes)     \
  X(32, false, kEpiMask | kEpiRes | kEpiSnake) X(32, false, kEpiAct) X(32, false, kEpiRes | kEpiAct) \
  X(32, false, kEpiAct | kEpiSnake) X(32, false, kEpiRes | kEpiAct | kEpiSnake) X(32, false, kEpiRes)

// `lim` = opt-in shared memory minus 1 KB; the kernels' own static shared memory comes off it too
void tc_conv2_set_smem_limit(int lim) {
  int i = 0;
#define WB_SET(kc, sp, f)                                                                          \
  {                                                                                                \
    const void* k = (const void*)tc_conv2_kernel<kc, sp, f>;                                       \
    cudaFuncAttributes fa{};                                                                       \
    cudaError_t e = cudaFuncGetAttributes(&fa, k);                                                 \
    if (e == cudaSuccess)                                                                          \
      e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,                     \
                               lim + 1024 - (int)fa.sharedSizeBytes);                              \
    if (e != cudaSuccess) fprintf(stderr, "wuburvc_b200: tc_conv2 smem limit %d: %s\n", i, cudaGetErrorString(e)); \
    ++i;                                                                                           \
  }
  WB_CONV2_KERNELS(WB_SET)
#undef WB_SET
}

void tc_kernels_init();  // tc_conv.cu

cudaError_t launch_tc_conv2(const TcConv2Maps& maps, const TcConv2Params& p, int kc, int grid, size_t smem,
                            cudaStream_t st) {
  tc_kernels_init();
  const bool split = p.split != 0;
  const uint32_t f = epi_features(p.epi);
  bool done = false;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kConv2Threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = p.pdl ? 1 : 0;
  cudaError_t err = cudaSuccess;
#define WB_LAUNCH(kc_, sp, f_)                                                                     \
  if (!done && kc == kc_ && split == sp && f == (f_)) {                                             \
    err = cudaLaunchKernelEx(&cfg, tc_conv2_kernel<kc_, sp, f_>, maps, p);                         \
    done = true;                                                                                   \
  }
  WB_CONV2_KERNELS(WB_LAUNCH)
#undef WB_LAUNCH
  if (!done) {  // any other epilogue: the generic instantiation
    if (kc == 64) {
      if (split) err = cudaLaunchKernelEx(&cfg, tc_conv2_kernel<64, true, kEpiGeneric>, maps, p);
      else err = cudaLaunchKernelEx(&cfg, tc_conv2_kernel<64, false, kEpiGeneric>, maps, p);
    } else {
      if (split) err = cudaLaunchKernelEx(&cfg, tc_conv2_kernel<32, true, kEpiGeneric>, maps, p);
      else err = cudaLaunchKernelEx(&cfg, tc_conv2_kernel<32, false, kEpiGeneric>, maps, p);
    }
  }
  return err != cudaSuccess ? err : cudaGetLastError();
}

}  // namespace wb
