// tc_epilogue.cuh — the fused epilogue shared by the tcgen05 convolution kernels.
//
// Four epilogue warps own TMEM lanes 0..127 (one output row per thread).  Per 32-column chunk the
// accumulator row is combined with: activation-derivative mask (LeakyReLU sign or Snake), bias,
// cond(g) row-broadcast, fp32 residual, scale, column-sum partials (bias gradients), accumulation
// into an fp32 sum, and written as fp32 / bf16 / the activation as a GEMM operand pair with a bf16
// copy.
#pragma once
#include "tc_conv.cuh"

namespace wb {

// Warp transpose-reduction: on return v[0] of lane l holds the sum over lanes of input v[l].
WB_DEV float warp_colsum32(float* v, int lane) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      float send = upper ? v[i] : v[i + off];
      float keep = upper ? v[i + off] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  return v[0];
}

// bf16 pairs packed in 32-bit words: element 2i in the low half.  Conversions stay in registers
// (no arrays whose address is taken, which would put them on the stack).
WB_DEV float bf16lo_f(uint32_t w) { return __uint_as_float(w << 16); }
WB_DEV float bf16hi_f(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
// two floats -> packed bf16x2 (round to nearest even), one conversion instruction
WB_DEV uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  uint32_t u;
  memcpy(&u, &h, sizeof(u));
  return u;
}

// fp16 pairs the same way (the forward operand split)
WB_DEV float f16lo_f(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xffffu))); }
WB_DEV float f16hi_f(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }
WB_DEV uint32_t pack_f16(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  uint32_t u;
  memcpy(&u, &h, sizeof(u));
  return u;
}

WB_DEV void store_packed16(bf16* p, const uint32_t* w) {  // 16 words = 32 bf16 = 64 bytes
  uint4* q = reinterpret_cast<uint4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) q[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
}

WB_DEV void store_f32x32(float* p, const float* v) {
  float4* q = reinterpret_cast<float4*>(p);
#pragma unroll
  for (int i = 0; i < 8; ++i) q[i] = make_float4(v[i * 4], v[i * 4 + 1], v[i * 4 + 2], v[i * 4 + 3]);
}

// A warp's 32 rows x 64 bytes leave through its 2 KB staging buffer: each lane writes its row
// (16-byte pieces XOR-swizzled by row, conflict-free), then the warp stores 8 rows x 64 B per
// instruction, contiguous where the rows are (512 B when a row is 64 B).  Rows >= rows_valid are
// not stored.  g0 = address of the warp's row 0 at this column piece.  With `add` the pieces are
// fp32 quadruples added to memory (one vector reduction each, resolved in L2) instead of stored.
WB_DEV void stage_put64(uint4* st, int lane, const uint32_t* w, char* g0, size_t pitch_bytes, int rows_valid,
                        bool add = false) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
    st[lane * 4 + (i ^ ((lane >> 1) & 3))] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int r = 8 * j + (lane >> 2), sg = lane & 3;
    const uint4 x = st[r * 4 + (sg ^ ((r >> 1) & 3))];
    if (r < rows_valid) {
      char* g = g0 + (size_t)r * pitch_bytes + sg * 16;
      if (add)
        atomicAdd(reinterpret_cast<float4*>(g),
                  make_float4(__uint_as_float(x.x), __uint_as_float(x.y), __uint_as_float(x.z), __uint_as_float(x.w)));
      else
        *reinterpret_cast<uint4*>(g) = x;
    }
  }
  __syncwarp();
}

// Where the chunk's outputs go: the thread's own row (stage == null), or the warp's staging buffer.
struct RowOut {
  uint4* stage;    // warp's 2 KB staging buffer, or null for direct per-row stores
  size_t off0;     // element offset of the warp's row 0 at this chunk (staged path)
  size_t pitch;    // elements per row
  int rows_valid;  // rows of the warp that exist (staged path)
  int lane;
};

WB_DEV void out_bf16x32(const RowOut& o, bf16* base, size_t off, const uint32_t* w) {
  if (o.stage) stage_put64(o.stage, o.lane, w, reinterpret_cast<char*>(base + o.off0), o.pitch * 2, o.rows_valid);
  else store_packed16(base + off, w);
}

WB_DEV void out_f32x32(const RowOut& o, float* base, size_t off, const float* v, bool add = false) {
  if (o.stage) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t w[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) w[i] = __float_as_uint(v[16 * h + i]);
      stage_put64(o.stage, o.lane, w, reinterpret_cast<char*>(base + o.off0 + 16 * h), o.pitch * 4, o.rows_valid,
                  add);
    }
  } else if (add) {
    float4* q = reinterpret_cast<float4*>(base + off);
#pragma unroll
    for (int i = 0; i < 8; ++i) atomicAdd(q + i, make_float4(v[i * 4], v[i * 4 + 1], v[i * 4 + 2], v[i * 4 + 3]));
  } else {
    store_f32x32(base + off, v);
  }
}

// Column sums of v over the 128 rows of the four epilogue warps; warp 0 lane l gets column l.
// Named barrier 1 synchronises only the 128 epilogue threads.
WB_DEV float cta_colsum32(float* v, float* red /*smem [128]*/, int warp, int lane, int bar) {
  // warp = index within a group of four epilogue warps; named barrier `bar` spans that group only
  const float s = warp_colsum32(v, lane);
  red[warp * 32 + lane] = s;
  asm volatile("bar.sync %0, 128;" ::"r"(bar) : "memory");
  float t = 0.f;
  if (warp == 0) t = red[lane] + red[32 + lane] + red[64 + lane] + red[96 + lane];
  asm volatile("bar.sync %0, 128;" ::"r"(bar) : "memory");
  return t;
}

// Compile-time epilogue feature sets.  A kernel instantiated for a feature set F contains only that
// set's code (smaller code, fewer registers); kEpiGeneric keeps every feature a run-time check.
enum : uint32_t {
  kEpiMask = 1u,     // activation-derivative mask from mask_src
  kEpiSnake = 2u,    // Snake (else LeakyReLU) for the mask and the activation
  kEpiRes = 4u,      // fp32 residual
  kEpiColsum = 8u,   // column-sum partials of the result (bias gradient)
  kEpiAct = 16u,     // activation output: operand pair (fp16 hi + lo * 2^11, or bf16 hi + lo) + bf16 copy
  kEpiLo = 32u,      // fp32 precision: bf16 lo companions of the bf16 outputs and of the Snake mask source
  kEpiGeneric = 1u << 31,
};

// The feature set of an epilogue, as the kernels' template argument expects it.
inline uint32_t epi_features(const Epi& e) {
  const bool snake = e.act_kind == 1 && (e.mask_src || e.act_hi);
  const bool lo = e.out_bf16_lo || e.act_bflo || e.pre_lo || e.mask_lo;
  return (e.mask_src ? kEpiMask : 0u) | (snake ? kEpiSnake : 0u) | (e.res ? kEpiRes : 0u) |
         (e.colsum ? kEpiColsum : 0u) | (e.act_hi ? kEpiAct : 0u) | (lo ? kEpiLo : 0u);
}

#define WB_EPI_HAS(bit, runtime) ((F & kEpiGeneric) ? (runtime) : ((F & (bit)) != 0))

// Per-row inputs of one 32-column chunk, loaded before they are needed (ideally before the
// accumulator is ready) so their memory latency overlaps the wait.
struct EpiIn {
  uint4 m[4];   // mask source (bf16)
  uint4 ml[4];  // its lo companion (fp32-precision Snake masks)
  float4 r[8];  // residual
};

template <uint32_t F>
WB_DEV void epi_load_mask(const Epi& e, bool valid, size_t off, EpiIn& in) {
  if (WB_EPI_HAS(kEpiMask, e.mask_src != nullptr) && valid) {
    const uint4* q = reinterpret_cast<const uint4*>(e.mask_src + off);
#pragma unroll
    for (int i = 0; i < 4; ++i) in.m[i] = __ldcs(q + i);
    if (WB_EPI_HAS(kEpiLo, e.mask_lo != nullptr) && e.mask_lo) {
      const uint4* ql = reinterpret_cast<const uint4*>(e.mask_lo + off);
#pragma unroll
      for (int i = 0; i < 4; ++i) in.ml[i] = __ldcs(ql + i);
    }
  }
}

template <uint32_t F>
WB_DEV void epi_load_res(const Epi& e, bool valid, size_t off, EpiIn& in) {
  if (WB_EPI_HAS(kEpiRes, e.res != nullptr) && valid) {
    const float4* q = reinterpret_cast<const float4*>(e.res + off);
#pragma unroll
    for (int i = 0; i < 8; ++i) in.r[i] = __ldcs(q + i);
  }
}

template <uint32_t F>
WB_DEV void epi_load(const Epi& e, bool valid, size_t off, EpiIn& in) {
  epi_load_mask<F>(e, valid, off, in);
  epi_load_res<F>(e, valid, off, in);
}

// Applies the epilogue to one 32-column chunk of one row (inputs from epi_load).
//   off      element offset of (row, column c0) in every [B][T][n_total] tensor
//   col      global column index of the chunk's first column (bias / alpha index)
//   part_row offset of this tile's row in the [tiles][n_total] partial buffers (+col)
//   bias / act_alpha / mask_alpha: the vectors at `col` (shared-memory copies in the persistent
//   kernel, else e's global vectors offset by col)
//   cs_acc / ap_acc: when non-null (persistent kernels), warp 0 accumulates this tile's column sums
//   there instead of writing a per-tile partial.
//   next / next_off: when `next`, the inputs of the row's next chunk (at next_off) are loaded into
//   `in` as soon as this chunk has consumed them, so their latency overlaps this chunk's work.
// Order: mask, bias, cond row, residual, scale, accumulation into out_f32, outputs, column sums
// (of the final, accumulated value).  An accumulation whose sum nothing else in the epilogue reads
// is a vector reduction into out_f32 (no read of the previous value on the SM).
template <uint32_t F>
WB_DEV void epi_finish(const Epi& e, float* v, EpiIn& in, bool valid, size_t off, size_t part_row,
                       const float* rowadd_row, const float* bias, const float* act_alpha, const float* mask_alpha,
                       int warp, int lane, float* red, float* cs_acc, float* ap_acc, int bar,
                       bool bias16 = false, const RowOut& o = RowOut{}, bool next = false, size_t next_off = 0) {
  const bool has_act = WB_EPI_HAS(kEpiAct, e.act_hi != nullptr);
  const bool has_cs = WB_EPI_HAS(kEpiColsum, e.colsum != nullptr);
  if (WB_EPI_HAS(kEpiMask, e.mask_src != nullptr)) {
    float x[32];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t w[4] = {in.m[i].x, in.m[i].y, in.m[i].z, in.m[i].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        x[8 * i + 2 * j] = valid ? bf16lo_f(w[j]) : 0.f;
        x[8 * i + 2 * j + 1] = valid ? bf16hi_f(w[j]) : 0.f;
      }
    }
    if (WB_EPI_HAS(kEpiLo, e.mask_lo != nullptr) && e.mask_lo && valid) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t w[4] = {in.ml[i].x, in.ml[i].y, in.ml[i].z, in.ml[i].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          x[8 * i + 2 * j] += bf16lo_f(w[j]);
          x[8 * i + 2 * j + 1] += bf16hi_f(w[j]);
        }
      }
    }
    if (next) epi_load_mask<F>(e, valid, next_off, in);
    if (WB_EPI_HAS(kEpiSnake, e.act_kind == 1)) {
      float ga[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        float dx, da;
        snake_grads(x[i], mask_alpha[i], dx, da);
        ga[i] = valid ? v[i] * da : 0.f;
        v[i] *= dx;
      }
      if (e.alpha_part) {
        const float t = cta_colsum32(ga, red, warp, lane, bar);
        if (warp == 0) {
          if (ap_acc) *ap_acc += t;
          else e.alpha_part[part_row + lane] = t;
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] *= (x[i] > 0.f) ? 1.f : e.slope;
    }
  }
  if (bias && bias16) {  // 16-byte aligned copy (the persistent kernel's shared memory)
    const float4* b4 = reinterpret_cast<const float4*>(bias);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 b = b4[i];
      v[4 * i] += b.x;
      v[4 * i + 1] += b.y;
      v[4 * i + 2] += b.z;
      v[4 * i + 3] += b.w;
    }
  } else if (bias) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] += bias[i];
  }
  if (rowadd_row) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] += rowadd_row[i];
  }
  if (WB_EPI_HAS(kEpiRes, e.res != nullptr) && valid) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[4 * i] += in.r[i].x;
      v[4 * i + 1] += in.r[i].y;
      v[4 * i + 2] += in.r[i].z;
      v[4 * i + 3] += in.r[i].w;
    }
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] *= e.scale;
  // accumulation: by reduction when only out_f32 receives the sum, else read + add here
  const bool acc_red = e.accumulate && !e.out_bf16 && !e.pre_hi && !has_act && !has_cs;
  if (e.accumulate && !acc_red && valid) {
    const float4* q = reinterpret_cast<const float4*>(e.out_f32 + off);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 a = __ldcs(q + i);
      v[4 * i] += a.x;
      v[4 * i + 1] += a.y;
      v[4 * i + 2] += a.z;
      v[4 * i + 3] += a.w;
    }
  }
  if (next) epi_load_res<F>(e, valid, next_off, in);
  if (valid || o.stage) {  // (the staged path needs every lane of the warp)
    if (e.out_f32) out_f32x32(o, e.out_f32, off, v, acc_red);
    if (e.out_bf16 || e.pre_hi) {
      uint32_t b[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) b[i] = pack_bf16(v[2 * i], v[2 * i + 1]);
      if (e.out_bf16) out_bf16x32(o, e.out_bf16, off, b);
      if (e.pre_hi) out_bf16x32(o, e.pre_hi, off, b);
      if (WB_EPI_HAS(kEpiLo, e.out_bf16_lo || e.pre_lo) && (e.out_bf16_lo || e.pre_lo)) {
        // lo companions: v - bf16(v), exact in fp32, rounded to bf16
#pragma unroll
        for (int i = 0; i < 16; ++i) b[i] = pack_bf16(v[2 * i] - bf16lo_f(b[i]), v[2 * i + 1] - bf16hi_f(b[i]));
        if (e.out_bf16_lo) out_bf16x32(o, e.out_bf16_lo, off, b);
        if (e.pre_lo) out_bf16x32(o, e.pre_lo, off, b);
      }
    }
    if (has_act) {
      // the activation as the next forward GEMM's operand pair (fp16 hi, fp16 lo * 2^11; or the
      // bf16 pair of the fallback format) and as a bf16 copy (the weight gradient's operand and the
      // LeakyReLU mask source)
      uint32_t h[16], l[16], bw[16], bl[16];
      const bool has_bflo = WB_EPI_HAS(kEpiLo, e.act_bflo != nullptr) && e.act_bflo;
      bool big = false;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float a0, a1;
        if (WB_EPI_HAS(kEpiSnake, e.act_kind == 1)) {
          a0 = snake(v[2 * i], act_alpha[2 * i]);
          a1 = snake(v[2 * i + 1], act_alpha[2 * i + 1]);
        } else {
          a0 = lrelu(v[2 * i], e.slope);
          a1 = lrelu(v[2 * i + 1], e.slope);
        }
        bw[i] = pack_bf16(a0, a1);
        if (has_bflo) bl[i] = pack_bf16(a0 - bf16lo_f(bw[i]), a1 - bf16hi_f(bw[i]));
        if (e.act_bf16pair) {
          h[i] = bw[i];
          l[i] = pack_bf16(a0 - bf16lo_f(h[i]), a1 - bf16hi_f(h[i]));
        } else {
          big |= !(fabsf(a0) < kF16Max) || !(fabsf(a1) < kF16Max);
          h[i] = pack_f16(a0, a1);
          l[i] = pack_f16((a0 - f16lo_f(h[i])) * kLoScale, (a1 - f16hi_f(h[i])) * kLoScale);
        }
      }
      if (big && valid && e.range_err) atomicCAS(e.range_err, 0, ERR_RANGE);
      out_bf16x32(o, reinterpret_cast<bf16*>(e.act_hi), off, h);
      if (e.act_lo) out_bf16x32(o, reinterpret_cast<bf16*>(e.act_lo), off, l);
      if (e.act_bf) out_bf16x32(o, e.act_bf, off, bw);
      if (has_bflo) out_bf16x32(o, e.act_bflo, off, bl);
    }
  }
  if (has_cs) {  // every lane reaches the group's named barriers; v is consumed here
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = valid ? v[i] : 0.f;
    const float t = cta_colsum32(v, red, warp, lane, bar);
    if (warp == 0) {
      if (cs_acc) *cs_acc += t;
      else e.colsum[part_row + lane] = t;
    }
  }
}

// One-shot form (load + finish) with the epilogue's global bias / alpha vectors.
WB_DEV void epi_chunk(const Epi& e, float* v, bool valid, size_t off, int col, size_t part_row, const float* rowadd_row,
                      int warp, int lane, float* red, float* cs_acc = nullptr, float* ap_acc = nullptr,
                      int bar = 1) {
  EpiIn in;
  epi_load<kEpiGeneric>(e, valid, off, in);
  epi_finish<kEpiGeneric>(e, v, in, valid, off, part_row, rowadd_row, e.bias ? e.bias + col : nullptr,
             e.act_alpha ? e.act_alpha + col : nullptr, e.mask_alpha ? e.mask_alpha + col : nullptr, warp, lane, red,
             cs_acc, ap_acc, bar);
}

}  // namespace wb
