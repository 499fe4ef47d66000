// The GDN decode step on an FP8 checkpoint + ring (sm_100a).
//
// One CTA owns one (sequence b, key head h) pair and the G value heads that
// share that key head, for a tile of `rows` value rows (128 = whole head).
// Everything one step needs is pulled into shared memory with bulk TMA copies
// (cp.async.bulk, one per ring slot row and one per checkpoint tile) while the
// CTA runs the prep stage; then either
//
//  * non-flush: the backward ("adjoint") replay of the ring
//      T <- q;  for t = n-1..0: c_t = beta_t (k_t . T); T <- exp(g_t)(T - c_t k_t)
//      o = sum_t c_t v_t + (S_fp8 * scale) T;  o *= K^-1/2
//    (prototype/gdn_replayssm_fp8_kernel.py:121-176), or
//  * flush: the forward rebuild S <- exp(g)S; S += beta (v - S k) k^T over the
//    ring (kern.py:177-228), the readout from the rebuilt state, and the
//    vblock32 re-quantisation written back in place (ref.py:40-106).
//
// In fused mode the prep stage (q/k L2 norm, gates, ring append of slot pos;
// kern.py:453-576) runs inside the same CTA and the token it appends takes
// part in this step's replay straight from shared memory.
#include <cstdio>

#include "gdnr_device.cuh"
#include "gdnr_internal.h"

namespace gdnr {

// K^-1/2 for K = 128, as float32 (prototype/gdn_replayssm_fp8_kernel.py:175)
constexpr float KSCALE = 0.08838834764831845f;

// All threads of the CTA wait on `bar`; the CTA agrees on failure so that it
// takes one uniform exit path.
__device__ __forceinline__ bool cta_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
  bool ok = mbar_wait_bounded(bar, parity, err);
  return __syncthreads_or(!ok) == 0;
}

template <bool FUSED, bool F32CK, int G>
__global__ void __launch_bounds__(256) step_kernel(const __grid_constant__ StepParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int ESZ = F32CK ? 4 : 1;
  const int h = blockIdx.x, b = blockIdx.y, z = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int R = p.rows;
  const int row0 = z * R;
  const int L = p.L;
  const SmemLayout S = step_smem_layout(G, L, R, ESZ);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S.bar);  // [0] ring, [1+j] checkpoint head j
  uint8_t* ck_s = smem + S.ck;
  uint16_t* kr_s = reinterpret_cast<uint16_t*>(smem + S.kr);  // [L][K]
  uint16_t* vr_s = reinterpret_cast<uint16_t*>(smem + S.vr);  // [G][L][R]
  float* gr_s = reinterpret_cast<float*>(smem + S.gr);        // [G][L]
  float* br_s = reinterpret_cast<float*>(smem + S.br);        // [G][L]
  float* tq_s = reinterpret_cast<float*>(smem + S.tq);        // [G][K]
  float* cf_s = reinterpret_cast<float*>(smem + S.cf);        // [G][L]
  float* orng_s = reinterpret_cast<float*>(smem + S.orng);    // [G][R]
  float* ofin_s = reinterpret_cast<float*>(smem + S.ofin);    // [G][R]
  float* qs_s = reinterpret_cast<float*>(smem + S.qs);        // [K]
  float* red_s = reinterpret_cast<float*>(smem + S.red);      // [8]

  // ---- per-sequence control (uniform over the CTA)
  int n_mem, n, pslot = -1;
  bool do_flush;
  if constexpr (FUSED) {
    const int pv = p.pos[int64_t(b) * p.pos_s];
    if (pv < 0 || pv >= L) {
      if (tid == 0) atomicOr(p.err, GDNR_DEVERR_BAD_POS);
      return;
    }
    pslot = pv;
    n_mem = pv;
    n = pv + 1;
    do_flush = (n == L);
  } else {
    int v = p.valid_len[int64_t(b) * p.vl_s];
    v = v < 0 ? 0 : (v > L ? L : v);
    n_mem = n = v;
    do_flush = (p.fl_dt == GDNR_I32) ? (static_cast<const int32_t*>(p.flush)[int64_t(b) * p.fl_s] != 0)
                                     : (static_cast<const uint8_t*>(p.flush)[int64_t(b) * p.fl_s] != 0);
  }

  if (tid == 0) {
#pragma unroll
    for (int i = 0; i < 1 + G; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  __syncthreads();

  // ---- bulk copies: ring rows (slots 0..n_mem-1), then the checkpoint tiles
  const uint32_t ring_bytes = uint32_t(n_mem) * (128 * 2 + G * R * 2);
  const uint32_t ck_bytes = uint32_t(R) * 128 * ESZ;
  if (warp == 0) {
    if (lane == 0) {
      if (ring_bytes) mbar_arrive_expect_tx(&bars[0], ring_bytes);
#pragma unroll
      for (int j = 0; j < G; ++j) mbar_arrive_expect_tx(&bars[1 + j], ck_bytes);
    }
    __syncwarp();
    if (lane < G) {
      const int hv = h * G + lane;
      const uint8_t* src = static_cast<const uint8_t*>(p.ck) +
                           (int64_t(b) * p.ck_sb + int64_t(hv) * p.ck_sh + int64_t(row0) * 128) * ESZ;
      bulk_g2s(ck_s + size_t(lane) * R * 128 * ESZ, src, ck_bytes, &bars[1 + lane]);
    }
    for (int t = lane; t < n_mem; t += 32) {
      const uint16_t* ksrc = p.kr + int64_t(b) * p.kr_sb + int64_t(t) * p.kr_st + int64_t(h) * p.kr_sh;
      bulk_g2s(kr_s + t * 128, ksrc, 128 * 2, &bars[0]);
#pragma unroll
      for (int j = 0; j < G; ++j) {
        const uint16_t* vsrc =
            p.vr + int64_t(b) * p.vr_sb + int64_t(t) * p.vr_st + int64_t(h * G + j) * p.vr_sh + row0;
        bulk_g2s(vr_s + (j * L + t) * R, vsrc, uint32_t(R) * 2, &bars[0]);
      }
    }
  }

  // ---- gates of the slots read from memory
  for (int i = tid; i < G * n_mem; i += blockDim.x) {
    const int j = i / n_mem, t = i - j * n_mem, hv = h * G + j;
    gr_s[j * L + t] = load_scalar(p.gr, int64_t(b) * p.gr_sb + int64_t(t) * p.gr_st + int64_t(hv) * p.gr_sh, p.gr_dt);
    br_s[j * L + t] = load_scalar(p.br, int64_t(b) * p.br_sb + int64_t(t) * p.br_st + int64_t(hv) * p.br_sh, p.br_dt);
  }

  // ---- prep (fused) or the query (replay)
  if constexpr (FUSED) {
    const int64_t mrow = int64_t(b) * p.mx_sb;
    if (warp < 2) {
      // warp 0: q, warp 1: k -- x / sqrt(sum(x^2) + 1e-6)  (kern.py:505-515)
      const int64_t off = mrow + (warp == 0 ? 0 : int64_t(p.H) * 128) + int64_t(h) * 128 + lane * 4;
      float x[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) x[i] = load_scalar(p.mixed, off + i, p.mx_dt);
      const float ss = warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]);
      const float nrm = sqrtf(ss + L2_EPS);
      if (warp == 0) {
        const int qdt = p.q_out ? p.qo_dt : GDNR_BF16;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float y = round_to(__fdiv_rn(x[i], nrm), qdt);
          qs_s[lane * 4 + i] = y;
          if (p.q_out && z == 0)
            store_scalar(p.q_out, int64_t(b) * p.qo_sb + int64_t(h) * p.qo_sh + lane * 4 + i, qdt, y);
        }
      } else {
        uint16_t kb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) kb[i] = f_to_bf16(__fdiv_rn(x[i], nrm));
        const uint2 kw = make_uint2(uint32_t(kb[0]) | (uint32_t(kb[1]) << 16), uint32_t(kb[2]) | (uint32_t(kb[3]) << 16));
        *reinterpret_cast<uint2*>(kr_s + pslot * 128 + lane * 4) = kw;
        if (z == 0)
          *reinterpret_cast<uint2*>(p.kr + int64_t(b) * p.kr_sb + int64_t(pslot) * p.kr_st + int64_t(h) * p.kr_sh +
                                    lane * 4) = kw;
      }
    } else if (warp < 2 + G) {
      // warps 2..2+G-1: value head j -- v copy and gates (kern.py:534-576)
      const int j = warp - 2, hv = h * G + j;
      const int64_t vin = mrow + 2 * int64_t(p.H) * 128 + int64_t(hv) * 128 + row0;
      uint16_t* vdst = p.vr + int64_t(b) * p.vr_sb + int64_t(pslot) * p.vr_st + int64_t(hv) * p.vr_sh + row0;
      for (int r = lane; r < R; r += 32) {
        const uint16_t vb = (p.mx_dt == GDNR_BF16) ? static_cast<const uint16_t*>(p.mixed)[vin + r]
                                                   : f_to_bf16(static_cast<const float*>(p.mixed)[vin + r]);
        vr_s[(j * L + pslot) * R + r] = vb;
        vdst[r] = vb;
      }
      if (lane == 0) {
        const float av = load_scalar(p.a, int64_t(b) * p.a_sb + int64_t(hv) * p.a_sh, p.a_dt);
        const float bv = load_scalar(p.bb, int64_t(b) * p.b_sb + int64_t(hv) * p.b_sh, p.b_dt);
        const float x = av + p.dt_bias[int64_t(hv) * p.db_s];
        const float sp = (x <= SOFTPLUS_THRESHOLD) ? logf(1.0f + expf(x)) : x;
        const float g = round_to(-expf(p.a_log[int64_t(hv) * p.al_s]) * sp, p.gr_dt);
        const float beta = round_to(1.0f / (1.0f + expf(-bv)), p.br_dt);
        gr_s[j * L + pslot] = g;
        br_s[j * L + pslot] = beta;
        if (z == 0) {
          store_scalar(p.gr, int64_t(b) * p.gr_sb + int64_t(pslot) * p.gr_st + int64_t(hv) * p.gr_sh, p.gr_dt, g);
          store_scalar(p.br, int64_t(b) * p.br_sb + int64_t(pslot) * p.br_st + int64_t(hv) * p.br_sh, p.br_dt, beta);
        }
      }
    }
    if (p.pos_out && h == 0 && z == 0 && tid == 0) p.pos_out[int64_t(b) * p.po_s] = (pslot + 1) % L;
  } else {
    if (warp == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        qs_s[lane * 4 + i] = load_scalar(p.q, int64_t(b) * p.q_sb + int64_t(h) * p.q_sh + lane * 4 + i, p.q_dt);
    }
  }
  __syncthreads();

  bool ok = true;
  if (ring_bytes) ok = cta_wait(&bars[0], 0, p.err);

  if (!do_flush) {
    // ---- backward T-chain, one warp per value head
    if (ok && warp < G) {
      const int j = warp;
      float T[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) T[i] = qs_s[lane * 4 + i];
      for (int t = n - 1; t >= 0; --t) {
        const uint2 kw = *reinterpret_cast<const uint2*>(kr_s + t * 128 + lane * 4);
        const float2 k01 = bf16x2_to_f2(kw.x), k23 = bf16x2_to_f2(kw.y);
        float d = T[0] * k01.x;
        d = fmaf(T[1], k01.y, d);
        d = fmaf(T[2], k23.x, d);
        d = fmaf(T[3], k23.y, d);
        d = warp_sum(d);
        const float c = br_s[j * L + t] * d;
        if (lane == 0) cf_s[j * L + t] = c;
        const float gam = expf(gr_s[j * L + t]);
        T[0] = gam * (T[0] - c * k01.x);
        T[1] = gam * (T[1] - c * k01.y);
        T[2] = gam * (T[2] - c * k23.x);
        T[3] = gam * (T[3] - c * k23.y);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) tq_s[j * 128 + lane * 4 + i] = T[i];
    }
    __syncthreads();
    // ---- ring part of the output: sum_t c_t v_t
    if (ok) {
      for (int i = tid; i < G * R; i += blockDim.x) {
        const int j = i / R, r = i - j * R;
        float acc = 0.0f;
        for (int t = n - 1; t >= 0; --t) acc = fmaf(cf_s[j * L + t], bf16_to_f(vr_s[(j * L + t) * R + r]), acc);
        orng_s[i] = acc;
      }
    }
    // ---- checkpoint readout: (S_fp8 . T) * scale, 8 lanes per row, one vblock per warp pass
#pragma unroll
    for (int j = 0; j < G; ++j) ok = cta_wait(&bars[1 + j], 0, p.err) && ok;
    if (ok) {
      const int vb_per_head = R / VBLOCK;
      const int c = lane & 7;
      for (int vb = warp; vb < G * vb_per_head; vb += 8) {
        const int j = vb / vb_per_head, rb = (vb - j * vb_per_head) * VBLOCK, hv = h * G + j;
        float sc = 1.0f;
        if constexpr (!F32CK)
          sc = load_scalar(p.sc, int64_t(b) * p.sc_sb + int64_t(hv) * p.sc_sh + int64_t((row0 + rb) / VBLOCK) * p.sc_sv,
                           p.sc_dt);
        float Tl[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) Tl[i] = tq_s[j * 128 + c * 16 + i];
#pragma unroll 2
        for (int it = 0; it < VBLOCK / 4; ++it) {
          const int r = rb + it * 4 + (lane >> 3);
          float acc = 0.0f;
          if constexpr (!F32CK) {
            const uint4 w = *reinterpret_cast<const uint4*>(ck_s + (size_t(j) * R + r) * 128 + c * 16);
            float f[16];
            e4m3x4_to_f4(w.x, f);
            e4m3x4_to_f4(w.y, f + 4);
            e4m3x4_to_f4(w.z, f + 8);
            e4m3x4_to_f4(w.w, f + 12);
#pragma unroll
            for (int i = 0; i < 16; ++i) acc = fmaf(f[i], Tl[i], acc);
          } else {
            const float4* rp = reinterpret_cast<const float4*>(ck_s + ((size_t(j) * R + r) * 128 + c * 16) * 4);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float4 v = rp[i];
              acc = fmaf(v.x, Tl[4 * i + 0], acc);
              acc = fmaf(v.y, Tl[4 * i + 1], acc);
              acc = fmaf(v.z, Tl[4 * i + 2], acc);
              acc = fmaf(v.w, Tl[4 * i + 3], acc);
            }
          }
          acc += __shfl_xor_sync(0xffffffffu, acc, 1);
          acc += __shfl_xor_sync(0xffffffffu, acc, 2);
          acc += __shfl_xor_sync(0xffffffffu, acc, 4);
          if (c == 0) ofin_s[j * R + r] = (orng_s[j * R + r] + acc * sc) * KSCALE;
        }
      }
    }
  } else {
    // ---- flush: forward rebuild per vblock, 32 rows x 8 lanes (16 columns each)
#pragma unroll
    for (int j = 0; j < G; ++j) ok = cta_wait(&bars[1 + j], 0, p.err) && ok;
    if (ok) {
      const int c = tid & 7, rl = tid >> 3;
      const int vb_per_head = R / VBLOCK;
      float ql[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) ql[i] = qs_s[c * 16 + i];
      for (int vb = 0; vb < G * vb_per_head; ++vb) {
        const int j = vb / vb_per_head, rb = (vb - j * vb_per_head) * VBLOCK, hv = h * G + j;
        const int r = rb + rl;
        float Sv[16];
        if constexpr (!F32CK) {
          const float sc =
              load_scalar(p.sc, int64_t(b) * p.sc_sb + int64_t(hv) * p.sc_sh + int64_t((row0 + rb) / VBLOCK) * p.sc_sv,
                          p.sc_dt);
          const uint4 w = *reinterpret_cast<const uint4*>(ck_s + (size_t(j) * R + r) * 128 + c * 16);
          e4m3x4_to_f4(w.x, Sv);
          e4m3x4_to_f4(w.y, Sv + 4);
          e4m3x4_to_f4(w.z, Sv + 8);
          e4m3x4_to_f4(w.w, Sv + 12);
#pragma unroll
          for (int i = 0; i < 16; ++i) Sv[i] *= sc;  // exact: 4-bit x 11-bit significands
        } else {
          const float4* rp = reinterpret_cast<const float4*>(ck_s + ((size_t(j) * R + r) * 128 + c * 16) * 4);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4 v = rp[i];
            Sv[4 * i + 0] = v.x;
            Sv[4 * i + 1] = v.y;
            Sv[4 * i + 2] = v.z;
            Sv[4 * i + 3] = v.w;
          }
        }
        for (int t = 0; t < n; ++t) {
          const float gam = expf(gr_s[j * L + t]);
          const uint4 k0 = *reinterpret_cast<const uint4*>(kr_s + t * 128 + c * 16);
          const uint4 k1 = *reinterpret_cast<const uint4*>(kr_s + t * 128 + c * 16 + 8);
          float kk[16];
          {
            float2 f;
            f = bf16x2_to_f2(k0.x); kk[0] = f.x; kk[1] = f.y;
            f = bf16x2_to_f2(k0.y); kk[2] = f.x; kk[3] = f.y;
            f = bf16x2_to_f2(k0.z); kk[4] = f.x; kk[5] = f.y;
            f = bf16x2_to_f2(k0.w); kk[6] = f.x; kk[7] = f.y;
            f = bf16x2_to_f2(k1.x); kk[8] = f.x; kk[9] = f.y;
            f = bf16x2_to_f2(k1.y); kk[10] = f.x; kk[11] = f.y;
            f = bf16x2_to_f2(k1.z); kk[12] = f.x; kk[13] = f.y;
            f = bf16x2_to_f2(k1.w); kk[14] = f.x; kk[15] = f.y;
          }
          float d = 0.0f;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            Sv[i] *= gam;
            d = fmaf(Sv[i], kk[i], d);
          }
          d += __shfl_xor_sync(0xffffffffu, d, 1);
          d += __shfl_xor_sync(0xffffffffu, d, 2);
          d += __shfl_xor_sync(0xffffffffu, d, 4);
          const float corr = (bf16_to_f(vr_s[(j * L + t) * R + r]) - d) * br_s[j * L + t];
#pragma unroll
          for (int i = 0; i < 16; ++i) Sv[i] = fmaf(corr, kk[i], Sv[i]);
        }
        // readout from the rebuilt state (kern.py:227)
        float o = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) o = fmaf(Sv[i], ql[i], o);
        o += __shfl_xor_sync(0xffffffffu, o, 1);
        o += __shfl_xor_sync(0xffffffffu, o, 2);
        o += __shfl_xor_sync(0xffffffffu, o, 4);
        if (c == 0) ofin_s[j * R + r] = o * KSCALE;
        const int64_t row_el = int64_t(b) * p.ck_sb + int64_t(hv) * p.ck_sh + int64_t(row0 + r) * 128 + c * 16;
        if constexpr (F32CK) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.ck) + row_el);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_float4(Sv[4 * i], Sv[4 * i + 1], Sv[4 * i + 2], Sv[4 * i + 3]);
        } else {
          // vblock amax (NaN-propagating, like torch.amax) across the 256 threads
          float am = 0.0f;
#pragma unroll
          for (int i = 0; i < 16; ++i) am = fmax_nan(am, fabsf(Sv[i]));
          am = warp_max_nan(am);
          if (lane == 0) red_s[warp] = am;
          __syncthreads();
          am = red_s[0];
#pragma unroll
          for (int w = 1; w < 8; ++w) am = fmax_nan(am, red_s[w]);
          __syncthreads();
          const VScale vs = vblock_scale(am, p.quant_rounded);
          uint32_t sat = 0;
          const uint4 qb = quantize16(Sv, vs.divisor, sat);
          *reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.ck) + row_el) = qb;
          if (tid == 0) {
            const int64_t si = int64_t(b) * p.sc_sb + int64_t(hv) * p.sc_sh + int64_t((row0 + rb) / VBLOCK) * p.sc_sv;
            if (p.sc_dt == GDNR_F16)
              static_cast<__half*>(p.sc)[si] = vs.stored;
            else
              static_cast<float*>(p.sc)[si] = __half2float(vs.stored);
          }
        }
      }
    }
  }
  __syncthreads();
  // ---- output rows (coalesced)
  if (ok) {
    for (int i = tid; i < G * R; i += blockDim.x) {
      const int j = i / R, r = i - j * R;
      store_scalar(p.out, int64_t(b) * p.o_sb + int64_t(h * G + j) * p.o_sh + int64_t(row0 + r) * p.o_sv, p.o_dt,
                   ofin_s[i]);
    }
  }
}

template <bool FUSED, bool F32CK, int G>
static cudaError_t launch_t(const StepParams& p, cudaStream_t stream) {
  const int esz = F32CK ? 4 : 1;
  const SmemLayout s = step_smem_layout(G, p.L, p.rows, esz);
  auto kern = step_kernel<FUSED, F32CK, G>;
  static DynSmemCache smem_cache;  // per device: dynamic smem already allowed for this instance
  cudaError_t e = ensure_dyn_smem(reinterpret_cast<const void*>(kern), int(s.total), smem_cache);
  if (e != cudaSuccess) return e;
  dim3 grid(p.H, p.B, 128 / p.rows);
  kern<<<grid, 256, s.total, stream>>>(p);
  return cudaGetLastError();
}

template <bool FUSED, bool F32CK>
static cudaError_t launch_g(const StepParams& p, int group, cudaStream_t stream) {
  switch (group) {
    case 1: return launch_t<FUSED, F32CK, 1>(p, stream);
    case 2: return launch_t<FUSED, F32CK, 2>(p, stream);
    case 4: return launch_t<FUSED, F32CK, 4>(p, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_step(const StepParams& p, bool fused, bool f32ck, int group, cudaStream_t stream) {
  if (step5_eligible(p, fused, f32ck)) return launch_step5(p, fused, p.pdl != 0, stream);
  if (p.sidx) return cudaErrorNotSupported;  // slot indirection: the persistent kernel only
  if (!f32ck && p.L <= STEP2_MAX_L) return launch_step2(p, fused, stream);
  if (p.ck_i8) return cudaErrorNotSupported;  // INT8 checkpoints: rings of L <= 16 only (checked by the API)
  if (fused) return f32ck ? launch_g<true, true>(p, group, stream) : launch_g<true, false>(p, group, stream);
  return f32ck ? launch_g<false, true>(p, group, stream) : launch_g<false, false>(p, group, stream);
}

}  // namespace gdnr
