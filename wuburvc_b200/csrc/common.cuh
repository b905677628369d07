// common.cuh — shared device helpers for the sm_100a generator kernels.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#define WB_DEV __device__ __forceinline__

namespace wb {

typedef __nv_bfloat16 bf16;
typedef __half f16;

// Forward GEMM operands are fp32 values split into an fp16 high part and an fp16 low part scaled by
// 2^11: x = hi + lo / 2^11 to ~2^-22 relative (11 significant bits each; the scale keeps the low
// part out of fp16's subnormal range for |x| >= 2^-14, and |lo| <= |x| so it cannot overflow where
// hi does not).  Products hi*hi + (hi*lo + lo*hi) / 2^11 are then fp32-accurate; the two sums land
// in separate accumulators and the epilogue applies the 1/2^11.  Values must stay below 65504
// (fp16's largest); producers report larger ones (ERR_RANGE) and the context then falls back to
// bf16 hi + bf16 lo pairs (range-safe, ~2^-17 relative).
constexpr float kLoScale = 2048.f;
constexpr float kLoUnscale = 1.f / 2048.f;
constexpr float kF16Max = 65504.f;

// Error codes written by kernels into the context's device error word.
enum : int {
  ERR_NONE = 0,
  ERR_WAIT_FULL = 1,      // MMA warp gave up waiting for a TMA stage
  ERR_WAIT_EMPTY = 2,     // producer gave up waiting for a free stage
  ERR_WAIT_ACC = 3,       // epilogue gave up waiting for the accumulator
  ERR_BAD_SHAPE = 4,
  ERR_RANGE = 5,          // a forward operand exceeded the fp16 range of the operand split
};

// Default time after which a bounded mbarrier wait gives up and the kernel reports a timeout (ns of
// %globaltimer; far above any legitimate wait, short enough that a broken pipeline ends quickly).
// The kernels take the limit from their launch parameters (wait_ns), set by the planner from
// wubu_b200_set_wait_limit_ns.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

WB_DEV unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

WB_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

WB_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// Programmatic dependent launch: a kernel launched with programmatic stream serialization may start
// before its predecessor has finished (the predecessor's CTAs let it in as they exit); it waits here
// for the predecessor's completion and memory before touching the predecessor's outputs.  A no-op for
// a kernel launched without the attribute.  (An explicit early trigger in the predecessors measured
// no faster and slower for the multi-wave kernels, so none is issued.)
WB_DEV void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

WB_DEV void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

WB_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

WB_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and records `code`) if the phase never flips.
WB_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  while (global_ns() - t0 < kWaitLimitNs)
    if (mbar_try_wait(bar, parity)) return true;
  if (err) atomicCAS(err, 0, code);
  return false;
}

// 3-D tiled TMA load into shared memory, completing on `bar`.
WB_DEV void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

WB_DEV void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- tcgen05 (5th-gen tensor core) -----------------------------------------
WB_DEV void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

WB_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

WB_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
WB_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 in, f32 accumulate).
WB_DEV void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// ---- warp-converged issue ----------------------------------------------------------------------
// The producer and MMA roles run their loops with all 32 lanes converged, so descriptors and
// coordinates are warp-uniform values (uniform registers); one lane chosen by elect.sync (the lowest,
// i.e. always the same lane) issues the asynchronous instruction.  Issuing from a lane-0-only branch
// instead makes every tcgen05.mma pay a register-to-uniform conversion of its operands.
WB_DEV void umma_f16_warp(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

WB_DEV void umma_commit_warp(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

WB_DEV void mbar_expect_tx_warp(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

WB_DEV void tma_load_3d_warp(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];\n\t}" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

WB_DEV void tma_load_4d_warp(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2, int c3) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];\n\t}" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

// Bounded wait by a converged warp; every lane gets the same result.  The spin loop lives inside one
// asm block so the compiler sees no divergent control flow around the issuing code (a C++ loop here
// makes it treat descriptors as per-lane values and every tcgen05.mma pays for uniformising them).
WB_DEV bool mbar_wait_warp(uint64_t* bar, uint32_t parity, int* err, int code,
                           unsigned long long limit_ns = kWaitLimitNs) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t.reg .u64 t0, t1;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "@p bra WB_WAIT_DONE;\n\t"
      "mov.u64 t0, %%globaltimer;\n"
      "WB_WAIT_LOOP:\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "@p bra WB_WAIT_DONE;\n\t"
      "mov.u64 t1, %%globaltimer;\n\t"
      "sub.u64 t1, t1, t0;\n\t"
      "setp.lt.u64 q, t1, %3;\n\t"
      "@q bra WB_WAIT_LOOP;\n"
      "WB_WAIT_DONE:\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity), "l"(limit_ns)
      : "memory");
  const bool ok = __all_sync(0xffffffffu, done != 0);
  if (!ok && err && (threadIdx.x & 31) == 0) atomicCAS(err, 0, code);
  return ok;
}

// The producer's record of its fills: bit s of `issued` = pipeline slot s (< 32) received a TMA fill,
// bit s of `parity` = the phase parity of its last one.  Before the kernel ends the producer waits
// (bounded) for the last fill of every slot, so that even after another warp gave up on a timed-out
// wait no copy lands in shared memory once the CTA has exited.  In a normal run those phases have
// long completed and the drain costs one poll per slot.
struct FillTrack {
  uint32_t issued = 0, parity = 0;
  WB_DEV void fill(int s, uint32_t ph) {
    issued |= 1u << s;
    parity = (parity & ~(1u << s)) | ((ph & 1u) << s);
  }
  WB_DEV void drain(uint64_t* full, int* err, unsigned long long limit_ns) const {
    for (int s = 0; s < 32; ++s)
      if ((issued >> s) & 1u) mbar_wait_warp(&full[s], (parity >> s) & 1u, err, ERR_WAIT_FULL, limit_ns);
  }
};

// Non-blocking test by a converged warp: has the phase with this parity completed?  (One
// mbarrier.test_wait; lets the MMA warp look at the next stage while it issues the current one.)
WB_DEV bool mbar_poll_warp(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return __all_sync(0xffffffffu, done != 0);
}

// Arrive on `bar` once every previously issued tcgen05.mma of this thread completes.
WB_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread (lane) gets its TMEM lane's row.
WB_DEV void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor (tcgen05 "smem descriptor", sm_100 version 1).
//   layout: 0 none, 2 = 128B swizzle, 4 = 64B swizzle, 6 = 32B swizzle.
WB_DEV uint64_t make_sdesc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes, uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  d |= (uint64_t)(layout & 7) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with f32 accumulation; A and B are both bf16 (bf16 = 1) or
// both fp16 (bf16 = 0).
WB_DEV uint32_t make_idesc(int M, int N, int a_mn_major, int b_mn_major, int bf16) {
  uint32_t d = 0;
  d |= 1u << 4;                          // D format f32
  d |= (uint32_t)(bf16 ? 1 : 0) << 7;    // A format: 0 f16, 1 bf16
  d |= (uint32_t)(bf16 ? 1 : 0) << 10;   // B format
  d |= (uint32_t)(a_mn_major & 1) << 15;
  d |= (uint32_t)(b_mn_major & 1) << 16;
  d |= (uint32_t)((N >> 3) & 0x3F) << 17;
  d |= (uint32_t)((M >> 4) & 0x1F) << 24;
  return d;
}
WB_DEV uint32_t make_idesc_bf16(int M, int N, int a_mn_major, int b_mn_major) {
  return make_idesc(M, N, a_mn_major, b_mn_major, 1);
}

// ---- misc -------------------------------------------------------------------
WB_DEV float lrelu(float x, float s) { return x > 0.f ? x : s * x; }

// Snake(alpha) = x + sin^2(alpha x) / alpha, with the SFU sine and a fast divide (absolute error of
// the sine ~1e-6 for the activations' range, far below the bf16 and fp32-mode gradient gates)
WB_DEV float snake(float x, float a) {
  const float s = __sinf(a * x);
  return x + __fdividef(s * s, a);
}
// Snake's derivative 1 + sin(2 alpha x) and its alpha derivative
// x sin(2 alpha x) / alpha - sin^2(alpha x) / alpha^2 (a difference of two ~x^2 terms for small
// arguments), from one sine / cosine pair accurate in RELATIVE terms down to small arguments
WB_DEV void snake_grads(float x, float a, float& dx, float& da) {
  // |alpha x| < 1/4: Taylor series (relative error below 1e-9; the SFU's absolute error would swamp
  // sin^2 of small arguments).  Else Cody-Waite reduction of the argument to [-pi, pi] (2 pi as a
  // float plus its rounding remainder, two FMAs) and the SFU pair, accurate on that interval.
  const float y = a * x, y2 = y * y;
  const float ts = y * (1.f - y2 * (1.f / 6.f - y2 * (1.f / 120.f - y2 * (1.f / 5040.f))));
  const float tc = 1.f - y2 * (0.5f - y2 * (1.f / 24.f - y2 * (1.f / 720.f)));
  const float k = rintf(y * 0.15915494309189535f);
  float r = fmaf(-k, 6.28318548202514648f, y);
  r = fmaf(-k, -1.7484556000744487e-07f, r);
  float sn, cs;
  __sincosf(r, &sn, &cs);
  const bool small = fabsf(y) < 0.25f;
  sn = small ? ts : sn;
  cs = small ? tc : cs;
  const float s2 = 2.f * sn * cs;
  const float ia = __fdividef(1.f, a);
  dx = 1.f + s2;
  da = (x * s2 - sn * sn * ia) * ia;
}

// split an fp32 value into bf16 hi + bf16 lo (hi + lo == x to ~2^-17 relative)
WB_DEV void split_bf16(float x, bf16& hi, bf16& lo) {
  hi = __float2bfloat16_rn(x);
  lo = __float2bfloat16_rn(x - __bfloat162float(hi));
}

// the forward operand split (see kLoScale): x = hi + lo / 2^11
WB_DEV void split_f16(float x, f16& hi, f16& lo) {
  hi = __float2half_rn(x);
  lo = __float2half_rn((x - __half2float(hi)) * kLoScale);
}
WB_DEV float join_f16(f16 hi, f16 lo) { return __half2float(hi) + __half2float(lo) * kLoUnscale; }

// A forward operand stored as 16-bit words in either format: fp16 hi / scaled lo (fmt_bf16 = 0) or
// the range-safe bf16 hi / lo a context falls back to after a range error (fmt_bf16 = 1).
WB_DEV void split_op(float x, int fmt_bf16, f16& hi, f16& lo) {
  if (fmt_bf16) {
    bf16 h, l;
    split_bf16(x, h, l);
    hi = __ushort_as_half(__bfloat16_as_ushort(h));
    lo = __ushort_as_half(__bfloat16_as_ushort(l));
  } else {
    split_f16(x, hi, lo);
  }
}
WB_DEV float join_op(f16 hi, f16 lo, int fmt_bf16) {
  if (fmt_bf16)
    return __bfloat162float(__ushort_as_bfloat16(__half_as_ushort(hi))) +
           __bfloat162float(__ushort_as_bfloat16(__half_as_ushort(lo)));
  return join_f16(hi, lo);
}

}  // namespace wb
