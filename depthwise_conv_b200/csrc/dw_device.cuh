// dw_device.cuh -- sm_100a device helpers for the depthwise engine:
// mbarriers with bounded waits, TMA tile loads, packed fp32x2 FMA and the
// fused epilogue arithmetic.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dwb {

// Error codes a kernel stores in the device error word (first writer wins)
// when one of its bounded waits expires: 1 = stage wait before a tile's
// first step, 2 = stage wait of a step, 3 = producer's free-stage (empty)
// wait, 4 = row-split partial-sum hand-off, 5 = the bounded-wait self-test
// (dwb_selftest_bounded_wait), whose wait nothing ever completes; the
// pointwise GEMM: 6 = producer's free-stage wait, 7 = MMA issuer's operand
// wait, 8 = epilogue's accumulator wait.  The word lives in the launcher's
// translation unit; kernels receive its address.

// ~1 s at 2 GHz: far above any legitimate wait (a row load takes ~1 us).
constexpr long long kWaitLimitCycles = 2000000000LL;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Test the phase.  With SLEEP, a thread whose phase is not complete may be
// suspended (up to kSuspendHintNs) instead of spinning on issue slots; the
// consumers' waits use the plain form, whose wake-up follows the phase
// completion more closely.
constexpr uint32_t kSuspendHintNs = 1000000;  // 1 ms
template <bool SLEEP>
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  if constexpr (SLEEP) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(kSuspendHintNs)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
  }
  return ok != 0;
}

// Non-blocking test of the phase (never suspends).  A consumer issues it for
// the next step's stage before the current step's FMAs and reads the answer
// after them, so the barrier round trip overlaps the arithmetic.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete.  Returns false (and
// records `code` in *err) if it has not completed within `limit` clock cycles
// (kWaitLimitCycles unless a self-test asks for less).
template <bool SLEEP = false>
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err, int code,
                                                  long long limit = kWaitLimitCycles) {
  if (mbar_try_wait<SLEEP>(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait<SLEEP>(bar, parity)) {
    if (clock64() - t0 > limit) {
      atomicCAS(err, 0, code);
      return false;
    }
  }
  return true;
}

// Position in a ring of mbarrier-guarded slots: the slot index and the
// parity of the current use of that slot (flips at every wrap).
struct RingPos {
  int slot = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void next(int n) {
    if (++slot == n) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

// Programmatic dependent launch.  A kernel launched with the programmatic
// stream-serialization attribute may start before the previous kernel of its
// stream has finished; griddep_wait() returns once that kernel has completed
// and its memory is visible, so every global read or write of data another
// kernel may produce comes after it.  griddep_launch_dependents() lets the
// next kernel of the stream start its own set-up early.  Every engine kernel
// calls it right after its own wait, not before: signalled before the wait,
// each waiting kernel let the next one in as well, and a graph of many
// back-to-back launches of a small grid piled up generations of resident,
// waiting CTAs (7x7x1024 k13: 3.8 us per launch in a graph of 50, 6.6 us in
// one of 1000; 3.4 us flat with the call after the wait).  Both are no-ops
// for a kernel launched without the attribute.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Tiled TMA loads (no multicast), completion signalled on an mbarrier.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// ---- packed fp32x2 arithmetic (sm_100: one FFMA2 = two fp32 FMAs) ----------

__device__ __forceinline__ unsigned long long f2_bits(float2 v) {
  return (static_cast<unsigned long long>(__float_as_uint(v.y)) << 32) | __float_as_uint(v.x);
}
__device__ __forceinline__ float2 bits_f2(unsigned long long b) {
  return make_float2(__uint_as_float(static_cast<uint32_t>(b)), __uint_as_float(static_cast<uint32_t>(b >> 32)));
}

// Packed fp32 pairs are kept in 64-bit registers ({lo, hi} = two channels)
// from conversion to epilogue, so no instruction ever repacks them.
typedef unsigned long long f32x2;

// acc += a * b, element-wise on the two lanes, each a single-rounding fp32 FMA.
__device__ __forceinline__ void ffma2(f32x2& acc, f32x2 a, f32x2 b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}

// acc += b, element-wise on the two lanes.
__device__ __forceinline__ void fadd2(f32x2& acc, f32x2 b) {
  asm("add.rn.f32x2 %0, %0, %1;" : "+l"(acc) : "l"(b));
}
__device__ __forceinline__ f32x2 fmul2(f32x2 a, f32x2 b) {
  f32x2 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ f32x2 splat2(float v) {
  const unsigned long long u = __float_as_uint(v);
  return (u << 32) | u;
}

// half2 (two channels) -> packed fp32 pair.
__device__ __forceinline__ f32x2 h2_to_f32x2(__half2 h) {
  f32x2 r;
  const uint32_t u = *reinterpret_cast<const uint32_t*>(&h);
  asm("{\n\t.reg .b16 lo, hi;\n\t.reg .f32 a, b;\n\t"
      "mov.b32 {lo, hi}, %1;\n\tcvt.f32.f16 a, lo;\n\tcvt.f32.f16 b, hi;\n\t"
      "mov.b64 %0, {a, b};\n\t}"
      : "=l"(r)
      : "r"(u));
  return r;
}


// acc.{lo,hi} += h.{lo,hi} with mixed-precision adds (fp16 operand, fp32
// accumulator, one rounding each).
__device__ __forceinline__ void add_h2_to_f32x2(f32x2& acc, __half2 h) {
  const uint32_t u = *reinterpret_cast<const uint32_t*>(&h);
  asm("{\n\t.reg .b16 lo, hi;\n\t.reg .f32 a, b;\n\t"
      "mov.b32 {lo, hi}, %1;\n\tmov.b64 {a, b}, %0;\n\t"
      "add.rn.f32.f16 a, lo, a;\n\tadd.rn.f32.f16 b, hi, b;\n\t"
      "mov.b64 %0, {a, b};\n\t}"
      : "+l"(acc)
      : "r"(u));
}
__device__ __forceinline__ f32x2 f32x2_zero() { return 0ull; }

// ---- epilogue ---------------------------------------------------------------

enum : int { kActNone = 0, kActRelu = 1, kActGelu = 2 };

__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Exact-form GELU, v * Phi(v) = 0.5 v erfc(-v / sqrt 2), with erfc from the
// rational approximation 7.1.26 of Abramowitz & Stegun (Handbook of
// Mathematical Functions, 1964): for a >= 0,
//   erfc(a) = (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) exp(-a^2),
//   t = 1 / (1 + p a),  |error| <= 1.5e-7,
// used directly on the negative side (where the product is small and its
// relative accuracy matters) and as 1 - erfc on the positive side.  Evaluated
// on a packed pair of channels: the polynomial and the products run as fp32x2
// instructions, only the reciprocal and the exponential per lane (two
// special-function ops per value).  The constants are folded so that the
// FMA pipe -- the bound resource of the convolution -- sees 11 packed
// operations per pair: a = |v|/sqrt2 is never formed (p/sqrt2 multiplies |v|
// directly, and exp(-a^2) = 2^(v * v * -log2(e)/2)), and the polynomial's
// coefficients carry the factor 1/2 of v * erfc / 2.  The result is within
// one fp16 ulp of the exact GELU over the whole fp16 range.
__device__ __forceinline__ f32x2 gelu_erf2(f32x2 v) {
  const f32x2 av = v & 0x7fffffff7fffffffull;                                           // |v|
  const float2 d = bits_f2(fma2(av, splat2(0.3275911f * 0.70710678118654752f), splat2(1.0f)));  // 1 + p a
  const f32x2 t = f2_bits(make_float2(rcp_approx(d.x), rcp_approx(d.y)));
  f32x2 poly = fma2(splat2(0.5f * 1.061405429f), t, splat2(0.5f * -1.453152027f));
  poly = fma2(poly, t, splat2(0.5f * 1.421413741f));
  poly = fma2(poly, t, splat2(0.5f * -0.284496736f));
  poly = fma2(poly, t, splat2(0.5f * 0.254829592f));
  poly = fmul2(poly, t);                                                                     // erfc(a) / 2 / exp(-a^2)
  const float2 ea = bits_f2(fmul2(fmul2(v, splat2(-0.5f * 1.4426950408889634f)), v));       // -a^2 log2(e)
  const f32x2 q = fmul2(v, fmul2(poly, f2_bits(make_float2(ex2_approx(ea.x), ex2_approx(ea.y)))));  // v erfc / 2
  const float2 pos = bits_f2(fma2(q, splat2(-1.0f), v));                                     // v (1 - erfc/2)
  const float2 vf = bits_f2(v), qf = bits_f2(q);
  return f2_bits(make_float2(vf.x >= 0.0f ? pos.x : qf.x, vf.y >= 0.0f ? pos.y : qf.y));
}

}  // namespace dwb
