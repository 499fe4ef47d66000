// Device-side building blocks shared by the gdnr kernels (sm_100a).
//
// * mbarrier + cp.async.bulk (the untiled TMA path) with bounded waits;
// * e4m3 / bf16 / fp16 conversions through the hardware cvt instructions;
// * the vblock32 quantiser used by both the standalone codec kernel and the
//   flush branch, so that both produce identical bytes.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/gdnr.h"

namespace gdnr {

constexpr int KD = 128;      // key dim (K)
constexpr int VD = 128;      // value dim (V)
constexpr int VBLOCK = 32;   // value rows per scale
constexpr int MAX_L = 64;    // longest ring the kernels accept
constexpr int MAX_G = 4;     // value heads per key head
constexpr float FP8_MAX = 448.0f;
constexpr float L2_EPS = 1e-6f;             // prototype/gdn_replayssm_fp8_kernel.py:756
constexpr float SOFTPLUS_THRESHOLD = 20.0f; // prototype/gdn_replayssm_fp8_kernel.py:757

// ---------------------------------------------------------------- timing
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier / bulk copy
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Makes mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wall-clock budget of one bounded wait.  A healthy wait here lasts a few
// microseconds; after this budget the kernel records GDNR_DEVERR_WAIT_TIMEOUT
// and the caller skips its computation instead of spinning for ever.
constexpr uint64_t WAIT_LIMIT_NS = 1000000000ull;  // 1 s
constexpr uint32_t WAIT_LIMIT_ITERS = 1u << 26;

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t* err) {
  const uint32_t a = smem_addr(bar);
  if (mbar_try_wait(a, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1; it < WAIT_LIMIT_ITERS; ++it) {
    if (mbar_try_wait(a, parity)) return true;
    if ((it & 255u) == 0 && globaltimer_ns() - t0 > WAIT_LIMIT_NS) break;
  }
  atomicOr(err, GDNR_DEVERR_WAIT_TIMEOUT);
  return false;
}

// Programmatic dependent launch: wait for the preceding grid's memory /
// allow the next grid to start its pre-wait prologue.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Global -> shared bulk copy (untiled TMA).  dst/src 16-byte aligned,
// bytes a multiple of 16.  Completion is signalled on `bar` as tx bytes.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// ---------------------------------------------------------------- conversions
__device__ __forceinline__ float bf16_to_f(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

__device__ __forceinline__ uint16_t f_to_bf16(float x) {
  __nv_bfloat16 h = __float2bfloat16_rn(x);
  return *reinterpret_cast<uint16_t*>(&h);
}

// Two packed bf16 in one 32-bit word -> float2.
__device__ __forceinline__ float2 bf16x2_to_f2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}

// Four e4m3 bytes (little-endian in w) -> four floats (exact).
__device__ __forceinline__ void e4m3x4_to_f4(uint32_t w, float* f) {
  __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w & 0xFFFFu), __NV_E4M3);
  __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(w >> 16), __NV_E4M3);
  float2 a = __half22float2(*reinterpret_cast<__half2*>(&lo));
  float2 b = __half22float2(*reinterpret_cast<__half2*>(&hi));
  f[0] = a.x;
  f[1] = a.y;
  f[2] = b.x;
  f[3] = b.y;
}

// float -> e4m3 with round-to-nearest-even; NaN -> 0x7F.  Inputs are already
// clamped to +-448 by the quantiser, so saturation never triggers.
__device__ __forceinline__ uint32_t f2_to_e4m3x2(float lo, float hi) {
  return static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E4M3));
}

// Scalar loads of small per-head values whose dtype is a runtime choice.
__device__ __forceinline__ float load_scalar(const void* p, int64_t i, int dtype) {
  switch (dtype) {
    case GDNR_F32: return static_cast<const float*>(p)[i];
    case GDNR_BF16: return bf16_to_f(static_cast<const uint16_t*>(p)[i]);
    case GDNR_F16: return __half2float(static_cast<const __half*>(p)[i]);
    default: return 0.0f;
  }
}

__device__ __forceinline__ void store_scalar(void* p, int64_t i, int dtype, float x) {
  switch (dtype) {
    case GDNR_F32: static_cast<float*>(p)[i] = x; break;
    case GDNR_BF16: static_cast<uint16_t*>(p)[i] = f_to_bf16(x); break;
    case GDNR_F16: static_cast<__half*>(p)[i] = __float2half_rn(x); break;
    default: break;
  }
}

// Value as it reads back after a store in `dtype` (the reference rounds g,
// beta, q and k by storing them; later steps read the rounded values).
__device__ __forceinline__ float round_to(float x, int dtype) {
  switch (dtype) {
    case GDNR_BF16: return bf16_to_f(f_to_bf16(x));
    case GDNR_F16: return __half2float(__float2half_rn(x));
    default: return x;
  }
}

// ---------------------------------------------------------------- reductions
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// max that propagates NaN (torch.amax semantics, ref.py:84)
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

__device__ __forceinline__ float warp_max_nan(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmax_nan(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

// ---------------------------------------------------------------- vblock32 quantiser
// Scale rule of quantize_checkpoint(..., "vblock", 32) (ref.py:36-37, :83-94):
//   s32 = amax > 0 ? amax / 448 : 1.0      (NaN amax -> 1.0)
//   stored scale = fp16(s32) (RNE)
//   divisor = s32 (reference oracle) or float(fp16(s32)) (Triton flush, kern.py:231-234)
struct VScale {
  float divisor;
  __half stored;
};

__device__ __forceinline__ VScale vblock_scale(float amax, int rounded_divisor) {
  float s32 = (amax > 0.0f) ? __fdiv_rn(amax, FP8_MAX) : 1.0f;
  VScale r;
  r.stored = __float2half_rn(s32);
  r.divisor = rounded_divisor ? __half2float(r.stored) : s32;
  return r;
}

// INT8 vblock scale ("vblock_int8", ref.py:44-47): amax / 127, 1 for a zero
// (or NaN) amax, stored as f16; the divisor is the f32 value or, with
// rounded_divisor, the stored f16 one.
__device__ __forceinline__ VScale vblock_scale_i8(float amax, int rounded_divisor) {
  const float s32 = (amax > 0.0f) ? __fdiv_rn(amax, 127.0f) : 1.0f;
  VScale r;
  r.stored = __float2half_rn(s32);
  r.divisor = rounded_divisor ? __half2float(r.stored) : s32;
  return r;
}

// INT8 code of x (ref.py:96-97): round-half-even of the IEEE quotient, clamped
// to +-127; NaN gives 0 (the reference's float -> int8 cast on its host).
// `sat` counts |x / divisor| > 127.
__device__ __forceinline__ uint32_t quant_i8(float x, float divisor, uint32_t& sat) {
  const float y = __fdiv_rn(x, divisor);
  sat += fabsf(y) > 127.0f ? 1u : 0u;
  const float c = y != y ? 0.0f : fminf(fmaxf(rintf(y), -127.0f), 127.0f);
  return uint32_t(__float2int_rn(c)) & 0xFFu;
}

// x / divisor with IEEE division, then clamp to +-448 keeping NaN (torch.clamp
// semantics, ref.py:99), returned as the pre-cast float.
__device__ __forceinline__ float quant_normalize(float x, float divisor) {
  float y = __fdiv_rn(x, divisor);
  y = (y > FP8_MAX) ? FP8_MAX : y;
  y = (y < -FP8_MAX) ? -FP8_MAX : y;
  return y;
}

// Quantise 16 consecutive values of one row with a known divisor; returns the
// 16 e4m3 bytes packed little-endian in a uint4 and counts saturated entries.
__device__ __forceinline__ uint4 quantize16(const float* x, float divisor, uint32_t& sat) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float y0 = __fdiv_rn(x[4 * i + 0], divisor);
    float y1 = __fdiv_rn(x[4 * i + 1], divisor);
    float y2 = __fdiv_rn(x[4 * i + 2], divisor);
    float y3 = __fdiv_rn(x[4 * i + 3], divisor);
    sat += (fabsf(y0) > FP8_MAX) + (fabsf(y1) > FP8_MAX) + (fabsf(y2) > FP8_MAX) + (fabsf(y3) > FP8_MAX);
    y0 = (y0 > FP8_MAX) ? FP8_MAX : ((y0 < -FP8_MAX) ? -FP8_MAX : y0);
    y1 = (y1 > FP8_MAX) ? FP8_MAX : ((y1 < -FP8_MAX) ? -FP8_MAX : y1);
    y2 = (y2 > FP8_MAX) ? FP8_MAX : ((y2 < -FP8_MAX) ? -FP8_MAX : y2);
    y3 = (y3 > FP8_MAX) ? FP8_MAX : ((y3 < -FP8_MAX) ? -FP8_MAX : y3);
    w[i] = f2_to_e4m3x2(y0, y1) | (f2_to_e4m3x2(y2, y3) << 16);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}


// ---------------------------------------------------------------- fast exact quantiser
// y = x / divisor computed as x * (1/divisor); that product is within 2.5 ulp
// of the IEEE quotient, so the e4m3 rounding of the two can differ only when
// y lies within a few ulp of an e4m3 rounding midpoint (mantissa bits below
// the 3 kept ones == 0x80000) or in the e4m3 subnormal range; those elements
// take the IEEE division instead, and so do quotients within a few ulp of 448
// (where the saturation count |x/divisor| > 448 is decided).  `fast_ok` is false when the divisor or its
// reciprocal is not a normal float (then every element is divided exactly).
__device__ __forceinline__ float quant_quotient(float x, float divisor, float rcp, bool fast_ok) {
  float y = x * rcp;
  const uint32_t u = __float_as_uint(y) & 0x7FFFFFFFu;
  const bool near_mid = ((u & 0xFFFFFu) - 0x7FFF8u) <= 16u;
  const bool near_max = (u - 0x43DFFFF8u) <= 16u;              // |y| within 8 ulp of 448 (saturation test)
  const bool subnormal_e4m3 = (u != 0u) && (u < 0x3C800000u);  // |y| < 2^-6
  if (!fast_ok || near_mid || near_max || subnormal_e4m3) y = __fdiv_rn(x, divisor);
  return y;
}

__device__ __forceinline__ bool quant_fast_ok(float divisor, float rcp) {
  return isfinite(divisor) && isfinite(rcp) && divisor >= 1.17549435e-38f && rcp >= 1.17549435e-38f;
}

// ---------------------------------------------------------------- division-free exact quantiser
// A float with the same e4m3 rounding (RNE, satfinite) as the IEEE quotient
// q = RN(x / d), from y = RN(x * rcp) without a division.
//
// The e4m3 grid has 8 values per binade on [2^-6, 448] and steps of 2^-9 on
// [0, 2^-6) -- the spacing of [2^-6, 2^-5), so that range is located by
// shifting it up by 2^-6 (round-toward-zero keeps the shifted value below 2^-5).
// y falls in the grid interval of the exact quotient, or -- when the quotient
// is next to a grid value, far from any midpoint -- in a neighbouring one.  Let
// m be the midpoint of y's interval (at most 5 significant bits, an even f32
// mantissa) and u its f32 ulp.  Then q rounds (in e4m3) to the upper grid
// neighbour of m iff q > m, i.e. iff x/d > m + u/2 (at exactly m + u/2 the f32
// rounding ties to m); to the lower iff x/d < m - u/2; otherwise q == m and
// the e4m3 tie goes to even.  r = fma(-m, d, x) is x - m d exactly whenever
// |x/d - m| is within a few ulp (the difference then fits in 24 bits), and
// otherwise has the right sign and is far from the thresholds +-(u/2) d, so
// the two comparisons are exact; the result is m, or m moved one f32 ulp up or
// down, which the e4m3 conversion rounds to the same grid value as q.  (The
// lower threshold at m = 2^-10, a power of two, would be u/4 d; there both
// outcomes are the grid value 0.)  NaN stays NaN.  Requires d, 1/d in
// [2^-60, 2^60] (quant_exact_ok), so that no threshold leaves the normal range;
// kd = quant_exact_kd(d) puts (u/2) d in bits as (bits(m) & exponent) + kd.
__device__ __forceinline__ bool quant_exact_ok(float d, float rcp) {
  return d >= 8.6736174e-19f && d <= 1.1529215e18f && rcp >= 8.6736174e-19f && rcp <= 1.1529215e18f;  // 2^-60, 2^60
}

__device__ __forceinline__ uint32_t quant_exact_kd(float d) { return __float_as_uint(d) - (151u << 23); }

__device__ __forceinline__ float quant_exact(float x, float d, float rcp, uint32_t kd) {
  const float y = x * rcp;
  const uint32_t sy = __float_as_uint(y) & 0x80000000u;
  const float a = fabsf(y);
  const bool sub = a < 0.015625f;
  const float t = sub ? __fadd_rz(a, 0.015625f) : a;
  const float mt = __uint_as_float((__float_as_uint(t) & 0xFFF00000u) | 0x00080000u);
  const float ma = sub ? mt - 0.015625f : mt;  // |m|, exact
  const uint32_t mb = __float_as_uint(ma) | sy;
  const float r = fmaf(__uint_as_float(mb), -d, x);                      // x - m d
  const float hd = __uint_as_float((__float_as_uint(ma) & 0x7F800000u) + kd);  // (u/2) d
  const float rr = __uint_as_float(__float_as_uint(r) ^ sy);             // > 0: |q| beyond |m|
  return __uint_as_float(mb + (rr > hd ? 1u : 0u) - (rr < -hd ? 1u : 0u));
}

// Two quotients as e4m3 bytes (low byte = x0); `ok` = quant_exact_ok(d, rcp),
// otherwise the IEEE division.
__device__ __forceinline__ uint32_t quant_e4m3x2(float x0, float x1, float d, float rcp, uint32_t kd, bool ok) {
  const float y0 = ok ? quant_exact(x0, d, rcp, kd) : __fdiv_rn(x0, d);
  const float y1 = ok ? quant_exact(x1, d, rcp, kd) : __fdiv_rn(x1, d);
  return f2_to_e4m3x2(y0, y1);
}

// The exact path of quant_pairs_warp, out of line: it is rare, and one copy of it
// instead of one per pair keeps the re-quantisation loops small in the
// instruction cache (flush step 69.6 -> 68.5 us at B = 64, L = 16).
static __device__ __noinline__ uint32_t quant_e4m3x2_slow(float x0, float x1, float d, float rcp, uint32_t kd, bool ok) {
  return quant_e4m3x2(x0, x1, d, rcp, kd, ok);
}

// e4m3 codes of RN(x / d) for NP pairs, the common case without a division and
// without the per-element work of quant_exact.  y = RN(x * rcp) is within one
// ulp of the IEEE quotient RN(x / d) (rcp = RN(1 / d) has relative error at
// most 2^-24, so |x rcp - x / d| < ulp), and RN(y (1 -+ 2^-23)) lie at least one
// ulp below / above y, so they bracket the quotient (for a normal y; a subnormal
// y and its quotient both convert to +-0).  When both brackets convert to the
// same e4m3 value, so does the quotient (the conversion is monotonic) and cvt(y)
// is exact; otherwise -- near a rounding midpoint, about 6e-5 of the values of a
// flushed checkpoint -- the pair is redone with quant_e4m3x2 behind one
// warp-uniform branch.  All lanes of the warp call it together.
template <int NP>
__device__ __forceinline__ void quant_pairs_warp(const float* x, uint32_t* c, float d, float rcp, uint32_t kd,
                                                 bool ok) {
  const float lo = __uint_as_float(0x3F7FFFFEu), hi = __uint_as_float(0x3F800001u);  // 1 -+ 2^-23
  uint32_t amb = ok ? 0u : 0xFFFFFFFFu;
#pragma unroll
  for (int j = 0; j < NP; ++j) {
    const float y0 = x[2 * j] * rcp, y1 = x[2 * j + 1] * rcp;
    c[j] = f2_to_e4m3x2(y0, y1);
    const uint32_t ca = f2_to_e4m3x2(y0 * lo, y1 * lo), cb = f2_to_e4m3x2(y0 * hi, y1 * hi);
    amb |= uint32_t(ca != cb) << j;
  }
  if (__any_sync(0xffffffffu, amb != 0u)) {
#pragma unroll
    for (int j = 0; j < NP; ++j)
      if ((amb >> j) & 1u) c[j] = quant_e4m3x2_slow(x[2 * j], x[2 * j + 1], d, rcp, kd, ok);
  }
}

// e4m3 pair with satfinite: RNE, then |y| > 448 -> 448 and NaN -> NaN, which
// equals clamp(+-448) followed by the cast (ref.py:99).
__device__ __forceinline__ uint32_t e4m3x2_sat(float lo, float hi) { return f2_to_e4m3x2(lo, hi); }

// 16 values (all lanes of the warp together; exact, see quant_pairs_warp); with
// count_sat, also counts |x/divisor| > 448 from the IEEE quotient.
__device__ __forceinline__ uint4 quantize16_fast(const float* x, float divisor, float rcp, bool count_sat,
                                                 uint32_t& sat) {
  uint32_t c[8];
  quant_pairs_warp<8>(x, c, divisor, rcp, quant_exact_kd(divisor), quant_exact_ok(divisor, rcp));
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = c[2 * i] | (c[2 * i + 1] << 16);
  if (count_sat) {
    const bool fast = quant_fast_ok(divisor, rcp);
#pragma unroll
    for (int i = 0; i < 16; ++i) sat += fabsf(quant_quotient(x[i], divisor, rcp, fast)) > FP8_MAX;
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// ---------------------------------------------------------------- tensor-core helpers (mma.sync m16n8k16)
// Fragment layout (g = lane/4, t4 = lane%4):
//   A: a0 = (row g, k 2t4..+1), a1 = (row g+8, k 2t4..+1), a2 = (row g, k 2t4+8..+9), a3 = (row g+8, k 2t4+8..+9)
//   B: b0 = (k 2t4..+1, col g), b1 = (k 2t4+8..+9, col g)
//   C: c0,c1 = (row g, col 2t4..+1), c2,c3 = (row g+8, col 2t4..+1)
__device__ __forceinline__ void mma16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// two e4m3 bytes (low byte = lower index) -> f16x2 (exact)
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two_bytes) {
  __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two_bytes & 0xFFFFu), __NV_E4M3);
  return uint32_t(h.x) | (uint32_t(h.y) << 16);
}

// bf16x2 -> f16x2 (RNE; exact for the normalised keys except magnitudes < 2^-14)
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t w) {
  const float2 f = bf16x2_to_f2(w);
  return pack_f16x2(f.x, f.y);
}

__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}


__device__ __forceinline__ void mma16816_bf16(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// power of two p with max_abs * p in [2^13, 2^14) (1 when max_abs is 0 or not finite);
// scaling f16 operands by it keeps them in the normal range without rounding
__device__ __forceinline__ float pow2_scale_for(float max_abs) {
  if (!(max_abs > 0.0f) || !isfinite(max_abs)) return 1.0f;
  int e;
  frexpf(max_abs, &e);  // max_abs in [2^(e-1), 2^e)
  // clamped so that the scale itself stays a normal float (values below
  // 2^-110 contribute nothing representable either way)
  const int k = 14 - e;
  return ldexpf(1.0f, k > 124 ? 124 : (k < -124 ? -124 : k));
}


// m16n8k32 with e4m3 A and B (A fragment: a0 = (row g, k 4t4..+3), a1 = (row g+8, ..),
// a2 = (row g, k 16+4t4..+3), a3 = (row g+8, ..); B: b0 = (k 4t4..+3, col g), b1 = (k 16+4t4.., col g))
__device__ __forceinline__ void mma16832_e4m3(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma16832_s8(int32_t* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// two int8 codes (low byte first) as f32 / f16x2 (exact: |code| <= 128)
__device__ __forceinline__ float2 i8x2_to_f2(uint32_t w) {
  return make_float2(float(int8_t(uint8_t(w))), float(int8_t(uint8_t(w >> 8))));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return uint32_t(f_to_bf16(lo)) | (uint32_t(f_to_bf16(hi)) << 16);
}

// e4m3 byte -> float (exact)
__device__ __forceinline__ float e4m3_to_f(uint32_t byte) {
  const uint32_t h = e4m3x2_to_f16x2(byte & 0xFFu);
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h & 0xFFFFu)));
}


// ---------------------------------------------------------------- cp.async (LDGSTS)
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace gdnr
