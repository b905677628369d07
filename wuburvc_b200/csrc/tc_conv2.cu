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

template <int KC>
__global__ void __launch_bounds__(kConv2Threads, 1)
    tc_conv2_kernel(const __grid_constant__ TcConv2Maps maps, const __grid_constant__ TcConv2Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ float red[2][128];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int N = p.n;
  const int nA = p.split ? 2 : 1;
  const uint32_t a_stage = nA * p.a_sub_bytes;
  const uint32_t w_sub = (uint32_t)N * KC * 2u;
  const uint32_t w_stage = nA * w_sub;
  const int AS = p.a_stages, WS = p.w_stages;

  uint8_t* a_base = smem;
  uint8_t* w_base = smem + (size_t)AS * a_stage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(w_base + (size_t)WS * w_stage);
  uint64_t* a_full = bars;
  uint64_t* a_empty = a_full + AS;
  uint64_t* w_full = a_empty + AS;
  uint64_t* w_empty = w_full + WS;
  uint64_t* acc_full = w_empty + WS;   // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  if (threadIdx.x == 0) {
    for (int s = 0; s < AS; ++s) { mbar_init(&a_full[s], 1); mbar_init(&a_empty[s], 1); }
    for (int s = 0; s < WS; ++s) { mbar_init(&w_full[s], 1); mbar_init(&w_empty[s], 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], 1); }
    fence_barrier_init();
  }
  if (warp == kMmaWarp) tmem_alloc(tmem_slot, (uint32_t)p.tmem_cols);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProducerWarp) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int a_it = 0, w_it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.ntiles && ok; tile += gridDim.x) {
        const int mtile = tile / p.n_tiles;
        const int n0 = (tile - mtile * p.n_tiles) * N;
        const int item = mtile / p.tiles_per_item;
        const int q0 = (mtile - item * p.tiles_per_item) * 128;
        for (int c = 0; c < p.n_chunks && ok; ++c) {
          const int sa = a_it % AS;
          if (a_it >= AS && !mbar_wait(&a_empty[sa], ((a_it / AS) & 1) ^ 1, p.err, ERR_WAIT_EMPTY)) { ok = false; break; }
          uint8_t* ad = a_base + (size_t)sa * a_stage;
          mbar_arrive_expect_tx(&a_full[sa], (uint32_t)nA * (uint32_t)p.halo_rows * KC * 2u);
          // one box of R rows x 8 channels per core-matrix column: column j lands at j * R * 16 bytes
          const uint32_t colb = (uint32_t)p.halo_rows * 16u;
#pragma unroll
          for (int j = 0; j < KC / 8; ++j) {
            tma_load_3d(ad + j * colb, &maps.a_hi, &a_full[sa], c * KC + j * 8, q0 + p.halo_start, item);
            if (p.split)
              tma_load_3d(ad + p.a_sub_bytes + j * colb, &maps.a_lo, &a_full[sa], c * KC + j * 8, q0 + p.halo_start,
                          item);
          }
          ++a_it;
          for (int t = 0; t < p.ntaps; ++t) {
            const int sw = w_it % WS;
            if (w_it >= WS && !mbar_wait(&w_empty[sw], ((w_it / WS) & 1) ^ 1, p.err, ERR_WAIT_EMPTY)) { ok = false; break; }
            uint8_t* wd = w_base + (size_t)sw * w_stage;
            mbar_arrive_expect_tx(&w_full[sw], w_stage);
            tma_load_3d(wd, &maps.w_hi, &w_full[sw], c * KC, n0, p.tap_w[t]);
            if (p.split) tma_load_3d(wd + w_sub, &maps.w_lo, &w_full[sw], c * KC, n0, p.tap_w[t]);
            ++w_it;
          }
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = make_idesc_bf16(128, N, 0, 0);
      constexpr uint32_t wlayout = (KC == 64) ? 2u : 4u;
      constexpr uint32_t wsbo = (KC == 64) ? 1024u : 512u;
      const uint32_t a_lbo = (uint32_t)p.halo_rows * 16u;  // stride between 8-channel core-matrix columns
      const uint32_t abase = smem_u32(a_base), wbase = smem_u32(w_base);
      int a_it = 0, w_it = 0, t_it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.ntiles && ok; tile += gridDim.x, ++t_it) {
        const int buf = t_it & 1;
        if (t_it >= 2 && !mbar_wait(&acc_empty[buf], ((t_it >> 1) & 1) ^ 1, p.err, ERR_WAIT_ACC)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * N);
        bool first = true;
        for (int c = 0; c < p.n_chunks && ok; ++c) {
          const int sa = a_it % AS;
          if (!mbar_wait(&a_full[sa], (a_it / AS) & 1, p.err, ERR_WAIT_FULL)) { ok = false; break; }
          tc_fence_after();
          const uint32_t ah = abase + (uint32_t)sa * a_stage;
          const uint32_t al = ah + p.a_sub_bytes;
          for (int t = 0; t < p.ntaps; ++t) {
            const int sw = w_it % WS;
            if (!mbar_wait(&w_full[sw], (w_it / WS) & 1, p.err, ERR_WAIT_FULL)) { ok = false; break; }
            tc_fence_after();
            const uint32_t wh = wbase + (uint32_t)sw * w_stage;
            const uint32_t wl = wh + w_sub;
            const uint32_t toff = (uint32_t)p.tap_off[t] * 16u;
#pragma unroll
            for (int k = 0; k < KC / 16; ++k) {
              const uint32_t aoff = toff + (uint32_t)k * 2u * a_lbo;
              const uint64_t dah = make_sdesc(ah + aoff, a_lbo, 128, 0);
              const uint64_t dwh = make_sdesc(wh + (uint32_t)k * 32u, 16, wsbo, wlayout);
              umma_f16(d, dah, dwh, idesc, first ? 0u : 1u);
              first = false;
              if (p.split) {
                const uint64_t dal = make_sdesc(al + aoff, a_lbo, 128, 0);
                const uint64_t dwl = make_sdesc(wl + (uint32_t)k * 32u, 16, wsbo, wlayout);
                umma_f16(d, dal, dwh, idesc, 1);
                umma_f16(d, dah, dwl, idesc, 1);
              }
            }
            umma_commit(&w_empty[sw]);
            ++w_it;
          }
          umma_commit(&a_empty[sa]);
          ++a_it;
        }
        if (ok) umma_commit(&acc_full[buf]);
      }
    }
  } else {
    // ---------------- epilogue: two groups of 4 warps; group g drains TMEM accumulator g, i.e. every
    // other tile, so two tiles' epilogues run concurrently (warp w reads TMEM lane quadrant w%4) ----------------
    const int qw = warp & 3, grp = warp >> 2;
    // column sums (bias / Snake-alpha gradients) accumulate over the group's tiles: one partial row
    // per group, 2 per CTA
    float cs_acc[8], ap_acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) cs_acc[i] = ap_acc[i] = 0.f;
    int t_it = grp;
    for (int tile = blockIdx.x + grp * gridDim.x; tile < p.ntiles; tile += 2 * gridDim.x, t_it += 2) {
      const int buf = grp;
      const bool ok = mbar_wait(&acc_full[buf], (t_it >> 1) & 1, p.err, ERR_WAIT_ACC);
      tc_fence_after();
      if (!ok) break;
      const int mtile = tile / p.n_tiles;
      const int n0 = (tile - mtile * p.n_tiles) * N;
      const int item = mtile / p.tiles_per_item;
      const int q = (mtile - item * p.tiles_per_item) * 128 + qw * 32 + lane;
      const bool valid = q < p.t_rows;
      const size_t row_off = ((size_t)item * p.t_rows + (valid ? q : 0)) * p.n_total + n0;
      const size_t part_row = (size_t)tile * p.n_total + n0;  // unused: sums accumulate per CTA
      const float* ra = p.epi.rowadd ? p.epi.rowadd + (size_t)item * p.n_total + n0 : nullptr;
#pragma unroll 1
      for (int c0 = 0; c0 < N; c0 += 32) {
        float v[32];
        tmem_ld32(tmem + (uint32_t)(buf * N) + ((uint32_t)(qw * 32) << 16) + (uint32_t)c0, v);
        epi_chunk(p.epi, v, valid, row_off + c0, n0 + c0, part_row + c0, ra ? ra + c0 : nullptr, qw, lane,
                  red[grp], &cs_acc[c0 >> 5], &ap_acc[c0 >> 5], 1 + grp);
      }
      tc_fence_before();
      asm volatile("bar.sync %0, 128;" ::"r"(3 + grp) : "memory");
      if (qw == 0 && lane == 0) mbar_arrive(&acc_empty[buf]);
    }
    if (qw == 0) {
      // every tile of this CTA shares one N tile (the grid is a multiple of n_tiles): the group's partial
      // row holds its sums in that tile's columns and zeros elsewhere
      const int my_n0 = (blockIdx.x % p.n_tiles) * N;
      const size_t prow = (size_t)(2 * blockIdx.x + grp) * p.n_total;
      for (int c = 0; c < p.n_total; c += 32) {
        const int rel = c - my_n0;
        const bool mine = rel >= 0 && rel < N;
        const float cs = mine ? cs_acc[rel >> 5] : 0.f, ap = mine ? ap_acc[rel >> 5] : 0.f;
        if (p.epi.colsum) p.epi.colsum[prow + c + lane] = cs;
        if (p.epi.alpha_part) p.epi.alpha_part[prow + c + lane] = ap;
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

void tc_conv2_set_smem_limit(int lim) {
  const cudaError_t a = cudaFuncSetAttribute(tc_conv2_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  const cudaError_t b = cudaFuncSetAttribute(tc_conv2_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  if (a != cudaSuccess || b != cudaSuccess)
    fprintf(stderr, "wuburvc_b200: tc_conv2 smem limit: %s / %s\n", cudaGetErrorString(a), cudaGetErrorString(b));
}

void tc_kernels_init();  // tc_conv.cu

cudaError_t launch_tc_conv2(const TcConv2Maps& maps, const TcConv2Params& p, int kc, int grid, size_t smem,
                            cudaStream_t st) {
  tc_kernels_init();
  if (kc == 64)
    tc_conv2_kernel<64><<<grid, kConv2Threads, smem, st>>>(maps, p);
  else
    tc_conv2_kernel<32><<<grid, kConv2Threads, smem, st>>>(maps, p);
  return cudaGetLastError();
}

}  // namespace wb
