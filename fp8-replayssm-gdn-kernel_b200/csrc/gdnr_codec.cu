// Standalone vblock32 FP8 codec kernels.
//
// quantize: float32 state [B,HV,V,K] -> e4m3 payload + one fp16 scale per 32
// value rows, bit-exact with quantize_checkpoint(state, "vblock", 32)
// (prototype/gdn_replay_fp8_reference.py:40-106).  It shares vblock_scale /
// quantize16 with the flush branch of the step kernel, so the flush writes
// exactly what this kernel writes for the same float32 state.
//
// dequantize: payload * scale[row/32] (ref.py:109-134).
//
// INT8 payloads ("vblock_int8", ref.py:44-47, :96-97): scale amax/127 (1 for a
// zero block), code = round-half-even(x / divisor) clamped to +-127 -- the
// IEEE quotient, then the integer rounding, as the reference's
// `(source / scale).round().clamp(-127, 127)` does.
#include "gdnr_device.cuh"
#include "gdnr_internal.h"

namespace gdnr {

// One CTA per vblock (32 rows x 128 columns = 4096 values); thread t owns
// row t/8, columns 16*(t%8) .. +15.
__global__ void __launch_bounds__(256) quantize_kernel(const __grid_constant__ CodecParams p) {
  __shared__ float red[8];
  __shared__ uint32_t sred[8];
  const int vb = blockIdx.x & 3;
  const int bh = blockIdx.x >> 2;
  const int b = bh / p.HV, hv = bh - b * p.HV;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = vb * VBLOCK + (tid >> 3), c = tid & 7;
  const float4* src =
      reinterpret_cast<const float4*>(p.state + int64_t(b) * p.st_sb + int64_t(hv) * p.st_sh + int64_t(r) * 128 + c * 16);
  float x[16];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 v = src[i];
    x[4 * i] = v.x;
    x[4 * i + 1] = v.y;
    x[4 * i + 2] = v.z;
    x[4 * i + 3] = v.w;
  }
  float am = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) am = fmax_nan(am, fabsf(x[i]));
  am = warp_max_nan(am);
  if (lane == 0) red[warp] = am;
  __syncthreads();
  am = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) am = fmax_nan(am, red[w]);
  uint32_t sat = 0;
  VScale vs;
  uint4 q;
  if (p.int8) {
    vs = vblock_scale_i8(am, p.quant_rounded);
    uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i >> 2] |= quant_i8(x[i], vs.divisor, sat) << (8 * (i & 3));
    q = make_uint4(w[0], w[1], w[2], w[3]);
  } else {
    vs = vblock_scale(am, p.quant_rounded);
    const float rcp = __fdiv_rn(1.0f, vs.divisor);
    q = quantize16_fast(x, vs.divisor, rcp, p.sat != nullptr, sat);
  }
  *reinterpret_cast<uint4*>(p.payload + int64_t(b) * p.pl_sb + int64_t(hv) * p.pl_sh + int64_t(r) * 128 + c * 16) = q;
  if (tid == 0) {
    const int64_t si = int64_t(b) * p.sc_sb + int64_t(hv) * p.sc_sh + int64_t(vb) * p.sc_sv;
    if (p.sc_dt == GDNR_F16)
      static_cast<__half*>(p.sc)[si] = vs.stored;
    else
      static_cast<float*>(p.sc)[si] = __half2float(vs.stored);
  }
  if (p.sat) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sat += __shfl_xor_sync(0xffffffffu, sat, o);
    if (lane == 0) sred[warp] = sat;
    __syncthreads();
    if (tid == 0) {
      uint32_t tot = 0;
#pragma unroll
      for (int w = 0; w < 8; ++w) tot += sred[w];
      if (tot) atomicAdd(p.sat, tot);
    }
  }
}

__global__ void __launch_bounds__(256) dequantize_kernel(const __grid_constant__ CodecParams p) {
  const int vb = blockIdx.x & 3;
  const int bh = blockIdx.x >> 2;
  const int b = bh / p.HV, hv = bh - b * p.HV;
  const int tid = threadIdx.x;
  const int r = vb * VBLOCK + (tid >> 3), c = tid & 7;
  const int64_t si = int64_t(b) * p.sc_sb + int64_t(hv) * p.sc_sh + int64_t(vb) * p.sc_sv;
  const float sc = load_scalar(p.sc, si, p.sc_dt);
  const uint4 w =
      *reinterpret_cast<const uint4*>(p.payload + int64_t(b) * p.pl_sb + int64_t(hv) * p.pl_sh + int64_t(r) * 128 + c * 16);
  float f[16];
  if (p.int8) {
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 16; ++i) f[i] = float(int8_t(uint8_t(wv[i >> 2] >> (8 * (i & 3)))));
  } else {
    e4m3x4_to_f4(w.x, f);
    e4m3x4_to_f4(w.y, f + 4);
    e4m3x4_to_f4(w.z, f + 8);
    e4m3x4_to_f4(w.w, f + 12);
  }
  float4* dst = reinterpret_cast<float4*>(p.state + int64_t(b) * p.st_sb + int64_t(hv) * p.st_sh + int64_t(r) * 128 + c * 16);
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[i] = make_float4(f[4 * i] * sc, f[4 * i + 1] * sc, f[4 * i + 2] * sc, f[4 * i + 3] * sc);
}

cudaError_t launch_quantize(const CodecParams& p, cudaStream_t stream) {
  const int64_t blocks = int64_t(p.B) * p.HV * 4;
  quantize_kernel<<<dim3(unsigned(blocks)), 256, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_dequantize(const CodecParams& p, cudaStream_t stream) {
  const int64_t blocks = int64_t(p.B) * p.HV * 4;
  dequantize_kernel<<<dim3(unsigned(blocks)), 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace gdnr
