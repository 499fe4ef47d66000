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

}  // namespace gdnr
