// tc_conv.cu — tcgen05/TMEM implicit-GEMM kernels (sm_100a).  See tc_conv.cuh.
#include "tc_epilogue.cuh"

namespace wb {

// ---------------------------------------------------------------------------------------------
// tc_conv kernel
// ---------------------------------------------------------------------------------------------
template <int KC>
__global__ void __launch_bounds__(192, 1)
    tc_conv_kernel(const __grid_constant__ TcMaps maps, const __grid_constant__ TcConvParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ float red[128];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int phase = blockIdx.z;
  const int tile = blockIdx.x;
  const int item = tile / p.tiles_per_item;
  const int q0 = (tile % p.tiles_per_item) * 128;
  const int N = p.n_tile;
  const int n0 = blockIdx.y * N;
  const int tap0 = p.tap_start[phase];
  const int ntaps = p.tap_start[phase + 1] - tap0;
  const int ksteps = ntaps * p.n_chunks;
  const int S = p.stages, G = p.kgroup;  // a pipeline stage holds G consecutive (tap, chunk) steps
  const int ngroups = (ksteps + G - 1) / G;
  const int nA = p.split ? 2 : 1;
  constexpr uint32_t a_bytes = 128u * KC * 2u;
  const uint32_t w_bytes = (uint32_t)N * KC * 2u;
  const uint32_t step_bytes = nA * (a_bytes + w_bytes);
  const uint32_t stage_bytes = (uint32_t)G * step_bytes;

  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes);
  uint64_t* empty = full + S;
  uint64_t* accf = empty + S;
  uint64_t* mma_done = accf + 1;  // every MMA of the CTA complete (drained before TMEM is freed)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    mbar_init(accf, 1);
    mbar_init(mma_done, 1);
    fence_barrier_init();
  }
  if (warp == 5) tmem_alloc(tmem_slot, (uint32_t)p.tmem_cols);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();  // every global read and write below follows the previous kernel

  // producer / MMA: converged warps, elect.sync issue, warp-uniform `ok` (no early exits)
  if (warp == 4) {
    // ---------------- TMA producer ----------------
    bool ok = true;
    FillTrack fill;
    int s = 0;
    uint32_t ph = 0;
    for (int g = 0; g < ngroups; ++g) {
      if (ok && g >= S) ok = mbar_wait_warp(&empty[s], ph ^ 1u, p.err, ERR_WAIT_EMPTY, p.wait_ns);
      if (ok) {
        const int ks0 = g * G, nk = min(G, ksteps - ks0);
        uint8_t* st = smem + (size_t)s * stage_bytes;
        fill.fill(s, ph);
        mbar_expect_tx_warp(&full[s], (uint32_t)nk * step_bytes);
        for (int i = 0; i < nk; ++i) {
          const int ks = ks0 + i;
          const int t = ks / p.n_chunks, c = ks - t * p.n_chunks;
          const int ti = tap0 + t;
          const int mi = p.tap_map[ti];
          const int row = q0 + p.tap_shift[ti];
          uint8_t* sd = st + (size_t)i * step_bytes;
          tma_load_3d_warp(sd, &maps.a[mi], &full[s], c * KC, row, item);
          if (p.split) tma_load_3d_warp(sd + a_bytes, &maps.a[p.lo_base + mi], &full[s], c * KC, row, item);
          uint8_t* wd = sd + nA * a_bytes;
          tma_load_3d_warp(wd, &maps.w_hi, &full[s], c * KC, n0, p.tap_w[ti]);
          if (p.split) tma_load_3d_warp(wd + w_bytes, &maps.w_lo, &full[s], c * KC, n0, p.tap_w[ti]);
        }
      }
      if (++s == S) { s = 0; ph ^= 1u; }
    }
    fill.drain(full, p.err, p.wait_ns);  // no copy of this CTA may land after it exits
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    // the split product as A_hi x [W_hi | W_lo] (2N wide: the tiles are adjacent rows) + A_lo x W_hi
    // into the upper N columns; the epilogue adds the halves (the upper one unscaled)
    const int fmt_bf16 = p.split ? p.split_bf16 : (p.single_f16 ? 0 : 1);
    const uint32_t idesc = make_idesc(128, N, 0, 0, fmt_bf16);
    const uint32_t idesc2 = make_idesc(128, 2 * N, 0, 0, fmt_bf16);
    constexpr uint32_t layout = (KC == 64) ? 2u : 4u;        // 128B / 64B swizzle
    constexpr uint32_t sbo = (KC == 64) ? 1024u : 512u;       // 8 rows x row bytes
    const uint64_t d0 = make_sdesc(smem_u32(smem), 16, sbo, layout);
    bool ok = true;
    int s = 0;
    uint32_t ph = 0;
    for (int g = 0; g < ngroups; ++g) {
      if (ok) ok = mbar_wait_warp(&full[s], ph, p.err, ERR_WAIT_FULL, p.wait_ns);
      if (ok) {
        const int nk = min(G, ksteps - g * G);
        for (int i = 0; i < nk; ++i) {
          const uint64_t dah = d0 + (((uint32_t)s * stage_bytes + (uint32_t)i * step_bytes) >> 4);
          const uint64_t dal = dah + (a_bytes >> 4);
          const uint64_t dwh = dah + ((nA * a_bytes) >> 4);
          const uint64_t dwl = dwh + (w_bytes >> 4);
#pragma unroll
          for (int k = 0; k < KC / 16; ++k) {  // K16 step = 32 bytes along the swizzled row
            if (p.split) {
              umma_f16_warp(tmem, dah + 2u * k, dwh + 2u * k, idesc2, (g | i | k) != 0);
              umma_f16_warp(tmem + (uint32_t)N, dal + 2u * k, dwh + 2u * k, idesc, 1);
            } else {
              umma_f16_warp(tmem, dah + 2u * k, dwh + 2u * k, idesc, (g | i | k) != 0);
            }
          }
          (void)dwl;
        }
        umma_commit_warp(&empty[s]);
      }
      if (++s == S) { s = 0; ph ^= 1u; }
    }
    if (ok) umma_commit_warp(accf);
    // every MMA this warp issued has completed before TMEM is released (also after a timed-out wait)
    umma_commit_warp(mma_done);
    mbar_wait_warp(mma_done, 0, p.err, ERR_WAIT_ACC, p.wait_ns);
  } else {
    // ---------------- epilogue (warps 0..3 <-> TMEM lanes 0..127) ----------------
    const bool ok = mbar_wait_warp(accf, 0, p.err, ERR_WAIT_ACC, p.wait_ns);
    tc_fence_after();
    const int q = q0 + warp * 32 + lane;
    const int orow = q * p.out_stride + p.out_off[phase];
    const bool valid = ok && q < p.m_rows && orow >= 0 && orow < p.t_out;
    const size_t row_off = ((size_t)item * p.t_out + (valid ? orow : 0)) * p.n_total + n0;
    const size_t part_row = (size_t)(blockIdx.z * gridDim.x + blockIdx.x) * p.n_total + n0;
    const float* ra = p.epi.rowadd ? p.epi.rowadd + (size_t)item * p.n_total + n0 : nullptr;
    for (int c0 = 0; c0 < N; c0 += 32) {
      float v[32];
      if (ok) {
        tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, v);
        if (p.split) {  // [0, N) holds hi*hi, [N, 2N) hi*lo + lo*hi (scaled by 2^11 in the fp16 format)
          float u[32];
          tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(N + c0), u);
          const float ls = p.split_bf16 ? 1.f : kLoUnscale;
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] += u[i] * ls;
        }
      } else
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0.f;
      // every epilogue warp reaches the chunk's named barriers, whether or not the wait succeeded
      epi_chunk(p.epi, v, valid, row_off + c0, n0 + c0, part_row + c0, ra ? ra + c0 : nullptr, warp, lane, red);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, (uint32_t)p.tmem_cols);
  }
}

// ---------------------------------------------------------------------------------------------
// tc_wgrad kernel: partial dW tiles over a K (time) range.  A pipeline stage holds `kb_group` blocks
// of 64 time rows (every atom of the M tile's dOut views + the activation rows), so the MMA warp
// pays one barrier round trip per kb_group x 4 MMAs.  Producer and MMA run as converged warps with
// elect.sync issue and a warp-uniform `ok` flag.  The partial tile leaves through the (then idle)
// pipeline shared memory as coalesced row pieces.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(192, 1)
    tc_wgrad_kernel(const __grid_constant__ TcWgMaps maps, const __grid_constant__ TcWgParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = blockIdx.x;
  const int split = blockIdx.y;
  const int nbase = blockIdx.z * p.n_in;
  const int kb0 = split * p.kb_per_split;
  const int kb1 = min(p.total_kblocks, kb0 + p.kb_per_split);
  const int nkb = max(0, kb1 - kb0);
  const int G = p.kb_group;
  const int ngroups = (nkb + G - 1) / G;
  const int S = p.stages;
  const int KR = p.kb_rows;  // time rows per K block (64, 128 or 256)
  const uint32_t atom_a_bytes = (uint32_t)KR * (uint32_t)p.atom_m * 2u;
  const uint32_t a_bytes = 128u * (uint32_t)KR * 2u;
  const int atom_n = p.n_in / p.n_atoms;
  const uint32_t atom_b_bytes = (uint32_t)KR * (uint32_t)atom_n * 2u;
  const uint32_t b_bytes = (uint32_t)p.n_in * (uint32_t)KR * 2u;
  const uint32_t kb_bytes = a_bytes + b_bytes;
  const uint32_t stage_bytes = (uint32_t)G * kb_bytes;

  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes);
  uint64_t* empty = full + S;
  uint64_t* accf = empty + S;
  uint64_t* mma_done = accf + 1;  // every MMA of the CTA complete (drained before TMEM is freed)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);

  // this M tile's atoms (dOut view, row shift, first channel), hoisted out of the parameter tables
  int a_map[4], a_shift[4], a_oc0[4];
  bool a_use[4];
  uint32_t kb_load = b_bytes;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    a_use[j] = j < p.m_atoms && p.atom_tap[mt][j] >= 0;
    a_map[j] = p.atom_map[mt][j];
    a_shift[j] = p.atom_shift[mt][j];
    a_oc0[j] = p.atom_oc0[mt][j];
    if (a_use[j]) kb_load += atom_a_bytes;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    mbar_init(accf, 1);
    mbar_init(mma_done, 1);
    fence_barrier_init();
  }
  if (warp == 5) tmem_alloc(tmem_slot, (uint32_t)p.tmem_cols);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();  // every global read and write below follows the previous kernel

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    bool ok = true;
    FillTrack fill;
    int s = 0;
    uint32_t ph = 0;
    for (int g = 0; g < ngroups; ++g) {
      if (ok && g >= S) ok = mbar_wait_warp(&empty[s], ph ^ 1u, p.err, ERR_WAIT_EMPTY, p.wait_ns);
      if (ok) {
        const int kbg = kb0 + g * G, nk = min(G, kb1 - kbg);
        uint8_t* st = smem + (size_t)s * stage_bytes;
        fill.fill(s, ph);
        mbar_expect_tx_warp(&full[s], (uint32_t)nk * kb_load);
        for (int i = 0; i < nk; ++i) {
          const int kb = kbg + i;
          const int item = kb / p.kblocks_per_item;
          const int t0 = (kb - item * p.kblocks_per_item) * KR;
          uint8_t* kd = st + (size_t)i * kb_bytes;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (a_use[j])
              tma_load_3d_warp(kd + j * atom_a_bytes, &maps.d[a_map[j]], &full[s], a_oc0[j], t0 + a_shift[j], item);
          for (int j = 0; j < p.n_atoms; ++j)
            tma_load_3d_warp(kd + a_bytes + j * atom_b_bytes, &maps.x, &full[s], nbase + j * atom_n, t0, item);
        }
      }
      if (++s == S) { s = 0; ph ^= 1u; }
    }
    fill.drain(full, p.err, p.wait_ns);  // no copy of this CTA may land after it exits
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc = make_idesc_bf16(128, p.n_in, 1, 1);
    const uint32_t la = (p.atom_m == 64) ? 2u : 4u, sboa = (uint32_t)p.atom_m * 16u;
    const uint32_t lb = (atom_n == 64) ? 2u : 4u, sbob = (uint32_t)atom_n * 16u;
    // descriptors built once; a k-step / block / stage moves the 14-bit start-address field
    const uint64_t da0 = make_sdesc(smem_u32(smem), atom_a_bytes, sboa, la);
    const uint64_t db0 = make_sdesc(smem_u32(smem) + a_bytes, atom_b_bytes, sbob, lb);
    const uint32_t ka = (2u * sboa) >> 4, kbb = (2u * sbob) >> 4;
    bool ok = true;
    int s = 0;
    uint32_t ph = 0;
    for (int g = 0; g < ngroups; ++g) {
      if (ok) ok = mbar_wait_warp(&full[s], ph, p.err, ERR_WAIT_FULL, p.wait_ns);
      if (ok) {
        const int nk = min(G, kb1 - (kb0 + g * G));
        const uint32_t sbase = ((uint32_t)s * stage_bytes) >> 4;
        for (int i = 0; i < nk; ++i) {
          const uint32_t kbase = sbase + (((uint32_t)i * kb_bytes) >> 4);
          for (int k = 0; k < KR / 16; ++k)  // KR time rows = KR/16 x K16
            umma_f16_warp(tmem, da0 + kbase + k * ka, db0 + kbase + k * kbb, idesc, (g | i | k) != 0);
        }
        umma_commit_warp(&empty[s]);
      }
      if (++s == S) { s = 0; ph ^= 1u; }
    }
    if (ok) umma_commit_warp(accf);
    // every MMA this warp issued has completed before TMEM is released (also after a timed-out wait)
    umma_commit_warp(mma_done);
    mbar_wait_warp(mma_done, 0, p.err, ERR_WAIT_ACC, p.wait_ns);
  } else {
    // ---------------- epilogue: 4 warps, TMEM lane quadrant = warp ----------------
    bool ok = nkb > 0 ? mbar_wait_warp(accf, 0, p.err, ERR_WAIT_ACC, p.wait_ns) : true;
    tc_fence_after();
    // the pipeline buffers are idle once the accumulator is complete: 2 KB staging per warp
    uint4* stage = reinterpret_cast<uint4*>(smem) + warp * 128;
    char* dst = reinterpret_cast<char*>(p.part + ((size_t)split * p.n_mtiles * 128 + (size_t)mt * 128 + warp * 32) *
                                                     p.n_total + nbase);
    for (int c0 = 0; c0 < p.n_in; c0 += 32) {
      float v[32];
      if (nkb > 0 && ok) tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, v);
      else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0.f;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = __float_as_uint(v[16 * h + i]);
        stage_put64(stage, lane, w, dst + (size_t)(c0 + 16 * h) * 4, (size_t)p.n_total * 4, 32);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, (uint32_t)p.tmem_cols);
  }
}

// ---------------------------------------------------------------------------------------------
// tc_wgrad halo kernel (see TcWgParams): per K block of kb_rows time rows ONE dOut halo (the CTA's
// channels x R rows) and one activation tile (MN-major atoms of 64 or 32 channels).
//   pack == 1: CTA = 128 output channels (two SW128 atoms of 64) x tg taps, one accumulator per tap;
//     tap tb + j reads the halo from row (tg - 1 - j) * dil.
//   pack > 1 : CTA = all C_out channels x tg = nacc * pack taps.  Accumulator j holds taps
//     tb + j*pack .. tb + j*pack + pack - 1 in its M atoms pack-1 .. 0 (atom a at halo row
//     (tg - pack*(j+1) + a) * dil): one MMA per K16 step covers `pack` taps.
// Every view stays inside the halo: its last row is (tg-1)*dil + kb_rows - 1 < R.
// ---------------------------------------------------------------------------------------------
constexpr int kHaloKR = 128;  // time rows per K block of the halo weight gradient

template <bool PACKED>
__global__ void __launch_bounds__(192, 1)
    tc_wgrad_halo_kernel(const __grid_constant__ TcWgMaps maps, const __grid_constant__ TcWgParams p) {
  constexpr int kMaxAcc = PACKED ? 8 : 2;  // accumulators per CTA (the planner's limits)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pack = PACKED ? p.pack : 1, tg = p.tg;
  const int oc0 = (blockIdx.x % p.oc_chunks) * 128;
  const int tb = (blockIdx.x / p.oc_chunks) * tg;  // first tap of this CTA
  // accumulators holding at least one real tap
  const int nacc = min(p.nacc, (p.ntaps - tb + pack - 1) / pack);
  const int split = blockIdx.y;
  const int nbase = blockIdx.z * p.n_in;
  const int kb0 = split * p.kb_per_split;
  const int kb1 = min(p.total_kblocks, kb0 + p.kb_per_split);
  const int nkb = max(0, kb1 - kb0);
  const int S = p.stages;
  const int KR = kHaloKR, R = p.halo_rows, N = p.n_in;
  // one M atom's halo row: 128 B (64 channels) or, packed, C_out * 2 B
  const uint32_t a_row = PACKED ? (uint32_t)p.c_out * 2u : 128u;
  const uint32_t a_bytes = (PACKED ? a_row : 256u) * (uint32_t)R;
  const uint32_t x_row = (uint32_t)p.x_atom * 2u;
  const uint32_t atom_b_bytes = (uint32_t)KR * x_row;
  const uint32_t b_bytes = (uint32_t)N * (uint32_t)KR * 2u;
  const uint32_t stage_bytes = a_bytes + b_bytes;

  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes);
  uint64_t* empty = full + S;
  uint64_t* accf = empty + S;
  uint64_t* mma_done = accf + 1;  // every MMA of the CTA complete (drained before TMEM is freed)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    mbar_init(accf, 1);
    mbar_init(mma_done, 1);
    fence_barrier_init();
  }
  if (warp == 5) tmem_alloc(tmem_slot, (uint32_t)p.tmem_cols);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();  // every global read and write below follows the previous kernel

  if (warp == 4) {
    // ---------------- TMA producer ----------------
    bool ok = true;
    FillTrack fill;
    int s = 0;
    uint32_t ph = 0;
    for (int i = 0; i < nkb; ++i) {
      if (ok && i >= S) ok = mbar_wait_warp(&empty[s], ph ^ 1u, p.err, ERR_WAIT_EMPTY, p.wait_ns);
      if (ok) {
        const int kb = kb0 + i;
        const int item = kb / p.kblocks_per_item;
        const int t0 = (kb - item * p.kblocks_per_item) * KR;
        uint8_t* st = smem + (size_t)s * stage_bytes;
        fill.fill(s, ph);
        mbar_expect_tx_warp(&full[s], stage_bytes);
        // dOut rows t0 + pad - (tb + tg - 1) * dil ... : every tap's window, once
        const int hr = t0 + p.pad - (tb + tg - 1) * p.dil;
        if (!PACKED) {  // two 64-channel atoms
          tma_load_3d_warp(st, &maps.d[0], &full[s], oc0, hr, item);
          tma_load_3d_warp(st + a_bytes / 2, &maps.d[0], &full[s], oc0 + 64, hr, item);
        } else {
          tma_load_3d_warp(st, &maps.d[0], &full[s], 0, hr, item);
        }
        for (int j = 0; j < p.n_atoms; ++j)
          tma_load_3d_warp(st + a_bytes + j * atom_b_bytes, &maps.x, &full[s], nbase + j * p.x_atom, t0, item);
      }
      if (++s == S) { s = 0; ph ^= 1u; }
    }
    fill.drain(full, p.err, p.wait_ns);  // no copy of this CTA may land after it exits
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc = make_idesc_bf16(128, N, 1, 1);
    // A: MN-major swizzled atoms (128-B rows: SW128, 8-row groups 1 KB apart; 64-B rows: SW64, 512 B),
    // the next M atom at LBO (the other 64 channels, or the next tap dil rows on).  The swizzle
    // follows the absolute address, so a view may start at any row.  B: MN-major atoms of x_atom
    // channels x KR rows.
    const uint32_t a_layout = a_row == 128u ? 2u : 4u, b_layout = x_row == 128u ? 2u : 4u;
    const uint32_t a_lbo = PACKED ? (uint32_t)p.dil * a_row : (uint32_t)R * 128u;
    const uint64_t da0 = make_sdesc(smem_u32(smem), a_lbo, a_row * 8u, a_layout);
    const uint64_t db0 = make_sdesc(smem_u32(smem) + a_bytes, atom_b_bytes, x_row * 8u, b_layout);
    const uint32_t a_k16 = a_row, b_k16 = x_row;  // K16 step = 16 rows, in 16-byte units
    bool ok = true;
    int s = 0;
    uint32_t ph = 0;
    for (int i = 0; i < nkb; ++i) {
      if (ok) ok = mbar_wait_warp(&full[s], ph, p.err, ERR_WAIT_FULL, p.wait_ns);
      if (ok) {
        const uint32_t sb = ((uint32_t)s * stage_bytes) >> 4;
#pragma unroll
        for (int j = 0; j < kMaxAcc; ++j) {
          if (j < nacc) {
            const int row = PACKED ? (tg - pack * (j + 1)) * p.dil : (tg - 1 - j) * p.dil;
            const uint32_t toff = (uint32_t)row * (a_row >> 4);
            const uint32_t d = tmem + (uint32_t)(j * N);
#pragma unroll
            for (int k = 0; k < kHaloKR / 16; ++k)
              umma_f16_warp(d, da0 + sb + toff + (uint32_t)k * a_k16, db0 + sb + (uint32_t)k * b_k16, idesc,
                            (i | k) != 0);
          }
        }
        umma_commit_warp(&empty[s]);
      }
      if (++s == S) { s = 0; ph ^= 1u; }
    }
    if (ok) umma_commit_warp(accf);
    // every MMA this warp issued has completed before TMEM is released (also after a timed-out wait)
    umma_commit_warp(mma_done);
    mbar_wait_warp(mma_done, 0, p.err, ERR_WAIT_ACC, p.wait_ns);
  } else {
    // ---------------- epilogue: 4 warps, TMEM lane quadrant = warp; 32 partial rows per accumulator ----------------
    const bool ok = nkb > 0 ? mbar_wait_warp(accf, 0, p.err, ERR_WAIT_ACC, p.wait_ns) : true;
    tc_fence_after();
    uint4* stage = reinterpret_cast<uint4*>(smem) + warp * 128;  // pipeline buffers are idle now
    for (int j = 0; j < nacc; ++j) {
      // accumulator row m = 32 * warp + lane: tap and output channel
      int tap, oc;
      if (!PACKED) {
        tap = tb + j;
        oc = oc0 + warp * 32;
      } else {
        const int ap = (warp * 32) / p.c_out;
        tap = tb + j * pack + pack - 1 - ap;
        oc = (warp * 32) % p.c_out;
      }
      if (tap >= p.ntaps) continue;  // warp-uniform
      const size_t row0 = (size_t)split * p.n_mtiles * 128 + (size_t)tap * p.c_out + oc;
      char* dst = reinterpret_cast<char*>(p.part + row0 * p.n_total + nbase);
      for (int c0 = 0; c0 < N; c0 += 32) {
        float v[32];
        if (nkb > 0 && ok) tmem_ld32(tmem + (uint32_t)(j * N) + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, v);
        else
#pragma unroll
          for (int q = 0; q < 32; ++q) v[q] = 0.f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t w[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) w[q] = __float_as_uint(v[16 * h + q]);
          stage_put64(stage, lane, w, dst + (size_t)(c0 + 16 * h) * 4, (size_t)p.n_total * 4, 32);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, (uint32_t)p.tmem_cols);
  }
}

// launch wrappers (host).  The dynamic shared-memory limit is raised once, before any capture.
void tc_conv2_set_smem_limit(int lim);  // tc_conv2.cu

static void raise_smem_limits() {
  static bool done = false;
  if (done) return;
  done = true;
  // opt-in limit minus room for the kernels' static shared memory
  int dev = 0, optin = 227 * 1024;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const int lim = optin - 1024;
  cudaError_t e[3];
  e[0] = cudaFuncSetAttribute(tc_conv_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  e[1] = cudaFuncSetAttribute(tc_conv_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  e[2] = cudaFuncSetAttribute(tc_wgrad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
  for (const void* k : {(const void*)tc_wgrad_halo_kernel<false>, (const void*)tc_wgrad_halo_kernel<true>}) {
    const cudaError_t eh = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    if (eh != cudaSuccess) fprintf(stderr, "wuburvc_b200: smem limit (wgrad halo): %s\n", cudaGetErrorString(eh));
  }
  for (int i = 0; i < 3; ++i)
    if (e[i] != cudaSuccess) fprintf(stderr, "wuburvc_b200: smem limit %d: %s\n", i, cudaGetErrorString(e[i]));
  tc_conv2_set_smem_limit(lim);
  cudaGetLastError();
}

void tc_kernels_init() { raise_smem_limits(); }

namespace {
// launch with programmatic stream serialization when `pdl` (the kernels wait for the previous one
// before their first global access)
template <typename K, typename M, typename P>
cudaError_t launch_192(K kernel, const M& maps, const P& p, dim3 grid, size_t smem, cudaStream_t st, int pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, maps, p);
  return e != cudaSuccess ? e : cudaGetLastError();
}
}  // namespace

cudaError_t launch_tc_conv(const TcMaps& maps, const TcConvParams& p, int kc, dim3 grid, size_t smem,
                           cudaStream_t st) {
  raise_smem_limits();
  if (kc == 64) return launch_192(tc_conv_kernel<64>, maps, p, grid, smem, st, p.pdl);
  return launch_192(tc_conv_kernel<32>, maps, p, grid, smem, st, p.pdl);
}

cudaError_t launch_tc_wgrad(const TcWgMaps& maps, const TcWgParams& p, dim3 grid, size_t smem, cudaStream_t st) {
  raise_smem_limits();
  if (p.halo && p.pack > 1) return launch_192(tc_wgrad_halo_kernel<true>, maps, p, grid, smem, st, p.pdl);
  if (p.halo) return launch_192(tc_wgrad_halo_kernel<false>, maps, p, grid, smem, st, p.pdl);
  return launch_192(tc_wgrad_kernel, maps, p, grid, smem, st, p.pdl);
}

}  // namespace wb
