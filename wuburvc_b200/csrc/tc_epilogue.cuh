// tc_epilogue.cuh — the fused epilogue shared by the tcgen05 convolution kernels.
//
// Four epilogue warps own TMEM lanes 0..127 (one output row per thread).  Per 32-column chunk the
// accumulator row is combined with: activation-derivative mask (LeakyReLU sign or Snake), bias,
// cond(g) row-broadcast, fp32 residual, scale, column-sum partials (bias gradients), accumulation
// into an fp32 sum, and written as fp32 / bf16 / activated bf16 hi+lo pairs.
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

WB_DEV void load_bf16x32(const bf16* p, float* out) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 u = q[i];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __bfloat1622float2(h[j]);
      out[i * 8 + j * 2] = f.x;
      out[i * 8 + j * 2 + 1] = f.y;
    }
  }
}

WB_DEV void store_bf16x32(bf16* p, const bf16* v) {
  uint4* q = reinterpret_cast<uint4*>(p);
  const uint4* s = reinterpret_cast<const uint4*>(v);
#pragma unroll
  for (int i = 0; i < 4; ++i) q[i] = s[i];
}

WB_DEV void load_f32x32(const float* p, float* out) {
  const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float4 f = q[i];
    out[i * 4] = f.x; out[i * 4 + 1] = f.y; out[i * 4 + 2] = f.z; out[i * 4 + 3] = f.w;
  }
}

WB_DEV void store_f32x32(float* p, const float* v) {
  float4* q = reinterpret_cast<float4*>(p);
#pragma unroll
  for (int i = 0; i < 8; ++i) q[i] = make_float4(v[i * 4], v[i * 4 + 1], v[i * 4 + 2], v[i * 4 + 3]);
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

// Applies the epilogue to one 32-column chunk of one row.
//   off      element offset of (row, column c0) in every [B][T][n_total] tensor
//   col      global column index of the chunk's first column (bias / alpha index)
//   part_row offset of this tile's row in the [tiles][n_total] partial buffers (+col)
//   cs_acc / ap_acc: when non-null (persistent kernels), warp 0 accumulates this tile's column sums
//   there instead of writing a per-tile partial.
WB_DEV void epi_chunk(const Epi& e, float* v, bool valid, size_t off, int col, size_t part_row, const float* rowadd_row,
                      int warp, int lane, float* red, float* cs_acc = nullptr, float* ap_acc = nullptr,
                      int bar = 1) {
  if (e.mask_src) {
    float x[32];
    if (valid) load_bf16x32(e.mask_src + off, x);
    else {
#pragma unroll
      for (int i = 0; i < 32; ++i) x[i] = 0.f;
    }
    if (e.act_kind == 1) {
      float ga[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float a = e.mask_alpha[col + i];
        float sn, cs;
        sincosf(a * x[i], &sn, &cs);
        const float s2 = 2.f * sn * cs;  // sin(2 a x)
        ga[i] = valid ? v[i] * (x[i] * s2 / a - sn * sn / (a * a)) : 0.f;
        v[i] *= 1.f + s2;
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
  if (e.bias) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] += e.bias[col + i];
  }
  if (rowadd_row) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] += rowadd_row[i];
  }
  if (e.res && valid) {
    float r[32];
    load_f32x32(e.res + off, r);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] += r[i];
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] *= e.scale;
  if (e.colsum) {
    float cv[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) cv[i] = valid ? v[i] : 0.f;
    const float t = cta_colsum32(cv, red, warp, lane, bar);
    if (warp == 0) {
      if (cs_acc) *cs_acc += t;
      else e.colsum[part_row + lane] = t;
    }
  }
  if (!valid) return;
  if (e.accumulate) {
    float r[32];
    load_f32x32(e.out_f32 + off, r);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] += r[i];
  }
  if (e.out_f32) store_f32x32(e.out_f32 + off, v);
  if (e.out_bf16 || e.pre_hi) {
    __align__(16) bf16 b[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) b[i] = __float2bfloat16_rn(v[i]);
    if (e.out_bf16) store_bf16x32(e.out_bf16 + off, b);
    if (e.pre_hi) store_bf16x32(e.pre_hi + off, b);
  }
  if (e.act_hi) {
    __align__(16) bf16 h[32];
    __align__(16) bf16 l[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float a = (e.act_kind == 1) ? snake(v[i], e.act_alpha[col + i]) : lrelu(v[i], e.slope);
      split_bf16(a, h[i], l[i]);
    }
    store_bf16x32(e.act_hi + off, h);
    if (e.act_lo) store_bf16x32(e.act_lo + off, l);
  }
}

}  // namespace wb
