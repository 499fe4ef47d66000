// The GDN decode step on an FP8 (E4M3) or INT8 checkpoint + ring, B200 path for
// rings of L <= 16 that the persistent kernel (gdnr_step5.cu) does not take:
// L < 4, rows or rings not 16-byte aligned, and the flush-capable calls on
// INT8 checkpoints.
//
// One CTA owns one (sequence b, value head hv) and `rows` value rows
// (128 = the whole head); warp w owns value rows [32w, 32w+32) -- exactly one
// vblock, i.e. one scale.
//
//  * The warp's 4 KiB of checkpoint is prefetched into registers with
//    coalesced 16-byte loads issued first thing, then parked in shared memory
//    in a 16-byte XOR swizzle (conflict-free tensor-core fragment reads).
//  * The ring (k rows and this tile's v rows) arrives by bulk TMA copies into
//    row-padded shared memory.
//  * Non-flush: warp 0 runs the backward T-chain in Gram form
//    (prototype/gdn_replayssm_fp8_kernel.py:121-176); the readout
//      o = scale (S . T) + sum_t c_t v_t        (then * K^-1/2)
//    is one tensor-core product per 16-row tile straight from the 8-bit tile:
//    E4M3 against T split into five power-of-two-scaled e4m3 terms, INT8
//    against four int8 limbs (integer MMA, exact s32 sums), plus V^T c as a
//    bf16 product (gdnr_head.cuh).
//  * Flush (ring full): the state rebuild runs in WY/Gram form on tensor
//    cores (mma.sync m16n8k16, f32 accumulate):
//      E = S0 [K;q]^T,  G = K K^T
//      r_t = a_t E_t + sum_{j<t} u_j M[j][t],  u_t = beta_t (v_t - r_t)
//      S_L = a_{n-1} S0 + W K,   W_t = u_t d_t
//    with a_t = prod_{m<=t} gamma_m, d_t = prod_{m>t} gamma_m,
//    M[j][t] = prod_{j<m<=t} gamma_m G[j][t] -- algebraically the reference's
//    token loop S <- gamma S; S += beta (v - S k) k^T (ref.py:137-163).  The
//    E accumulators become, after the per-row recurrence, the A fragments of
//    the S_L product in registers.  S_L is re-quantised per vblock in the
//    checkpoint's format (ref.py:40-106; int8: ref.py:44-47, :96-97) and
//    written back in place.
// In fused mode the prep stage (q/k L2 norm, gates, ring append,
// kern.py:453-576) runs first and the new token joins this step's replay.
#include "gdnr_device.cuh"
#include "gdnr_head.cuh"
#include "gdnr_internal.h"

namespace gdnr {

struct Smem2 {
  uint32_t bar, kr, vr, gr, br, qs, cf, tb, cb, ow, misc, qb, t8, gram, mg, ad, kx, s0, total;
  int vstr;
};

__host__ __device__ inline Smem2 step2_smem(int L, int rows) {
  Smem2 s;
  uint32_t o = 0;
  const int W = rows / 32;
  s.vstr = rows + 8;
  s.bar = smem_take(o, 16);
  s.kr = smem_take(o, uint32_t(L) * KSTR * 2);
  s.vr = smem_take(o, uint32_t(L) * s.vstr * 2);
  s.gr = smem_take(o, 16 * 4);                // g_t
  s.br = smem_take(o, 16 * 4);                // beta_t
  s.qs = smem_take(o, 128 * 4);               // q (f32)
  s.cf = smem_take(o, 16 * 4);                // c_t
  s.tb = smem_take(o, 2 * 128 * 2);           // [T_hi; T_lo] f16
  s.cb = smem_take(o, 3 * 16 * 2);            // [c_hi; c_mid; c_lo] bf16
  s.ow = smem_take(o, uint32_t(W) * 32 * 4);  // per-warp output rows
  s.misc = smem_take(o, 16);                  // 1/T scale
  s.qb = smem_take(o, 3 * 128 * 2);           // non-flush: q split into 3 bf16 rows
  s.t8 = smem_take(o, 8 * T8STR);             // non-flush: T split into e4m3 terms (rows 5..7 zero)
  s.gram = smem_take(o, 16 * 24 * 4);         // flush: Gram [t][s], kq in col 16/17
  s.mg = smem_take(o, 16 * 16 * 4);           // flush: M[j][t]
  s.ad = smem_take(o, 4 * 16 * 4);            // flush: gamma_t, a_t, d_t, kq_t
  // flush: k16 ([18][KSTR] f16: 16 keys, q_hi, q_lo; scaled by 256) for E / Gram,
  // later reused as K^T ([128][KTSTR] f16, scaled by 256) for the S_L product
  s.kx = smem_take(o, KX_BYTES);
  s.s0 = smem_take(o, uint32_t(rows) * 128);  // checkpoint tile (swizzled e4m3)
  s.total = o;
  return s;
}

__device__ __forceinline__ bool cta_wait2(uint64_t* bar, uint32_t parity, uint32_t* err) {
  bool ok = mbar_wait_bounded(bar, parity, err);
  return __syncthreads_or(!ok) == 0;
}

// I8: the checkpoint holds int8 codes ("vblock_int8"); see gdnr_head.cuh.
// CTAs per SM the register budget is sized for (6 x 128 threads: 80 registers; the
// int8 variants then spill a few bytes in the flush, which costs less than the lower
// occupancy of a larger budget -- 22 vs 26.5 us non-flush, 99 vs 108 us flush, same-box A/B)
constexpr int S2_MIN_BLOCKS = 6;

template <bool FUSED, bool I8>
__global__ void __launch_bounds__(128, S2_MIN_BLOCKS) step2_kernel(const __grid_constant__ StepParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int hv = blockIdx.x, b = blockIdx.y, z = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c8 = lane & 7;
  const int R = p.rows;
  const int row0 = z * R;
  const int G = p.HV / p.H, h = hv / G;
  const int L = p.L;
  const Smem2 S = step2_smem(L, R);
  const int VSTR = S.vstr;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + S.bar);
  uint16_t* kr_s = reinterpret_cast<uint16_t*>(smem + S.kr);
  uint16_t* vr_s = reinterpret_cast<uint16_t*>(smem + S.vr);
  float* gr_s = reinterpret_cast<float*>(smem + S.gr);
  float* br_s = reinterpret_cast<float*>(smem + S.br);
  float* qs_s = reinterpret_cast<float*>(smem + S.qs);
  uint8_t* s0 = smem + S.s0;

  // ---- per-sequence control (CTA-uniform)
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

  // ---- 1. checkpoint prefetch: warp w, rows 32w + 4it + lane/8, 16-byte chunk lane%8
  const uint8_t* ck_head =
      static_cast<const uint8_t*>(p.ck) + int64_t(b) * p.ck_sb + int64_t(hv) * p.ck_sh + int64_t(row0) * 128;
  uint4 ck[8];
#pragma unroll
  for (int it = 0; it < 8; ++it) ck[it] = ldg_stream_v4(ck_head + (32 * warp + 4 * it + (lane >> 3)) * 128 + c8 * 16);

  // ---- 2. ring via bulk TMA (slots 0..n_mem-1)
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  const uint32_t ring_bytes = uint32_t(n_mem) * (128 * 2 + R * 2);
  if (warp == 0) {
    if (lane == 0 && ring_bytes) mbar_arrive_expect_tx(bar, ring_bytes);
    __syncwarp();
    for (int t = lane; t < n_mem; t += 32) {
      bulk_g2s(kr_s + t * KSTR, p.kr + int64_t(b) * p.kr_sb + int64_t(t) * p.kr_st + int64_t(h) * p.kr_sh, 256, bar);
      bulk_g2s(vr_s + t * VSTR, p.vr + int64_t(b) * p.vr_sb + int64_t(t) * p.vr_st + int64_t(hv) * p.vr_sh + row0,
               uint32_t(R) * 2, bar);
    }
  }
  for (int t = tid; t < n_mem; t += blockDim.x) {
    gr_s[t] = load_scalar(p.gr, int64_t(b) * p.gr_sb + int64_t(t) * p.gr_st + int64_t(hv) * p.gr_sh, p.gr_dt);
    br_s[t] = load_scalar(p.br, int64_t(b) * p.br_sb + int64_t(t) * p.br_st + int64_t(hv) * p.br_sh, p.br_dt);
  }

  // ---- 3. prep (fused) or query load (replay)
  if constexpr (FUSED) {
    const int64_t mrow = int64_t(b) * p.mx_sb;
    const bool owner = (hv % G) == 0 && z == 0;  // one CTA per key head writes k / q_out
    if (warp < 2) {
      const int64_t off = mrow + (warp == 0 ? 0 : int64_t(p.H) * 128) + int64_t(h) * 128 + lane * 4;
      float x[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) x[i] = load_scalar(p.mixed, off + i, p.mx_dt);
      const float nrm = sqrtf(warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]) + L2_EPS);
      if (warp == 0) {
        const int qdt = p.q_out ? p.qo_dt : GDNR_BF16;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float y = round_to(__fdiv_rn(x[i], nrm), qdt);
          qs_s[lane * 4 + i] = y;
          if (p.q_out && owner) store_scalar(p.q_out, int64_t(b) * p.qo_sb + int64_t(h) * p.qo_sh + lane * 4 + i, qdt, y);
        }
      } else {
        uint16_t kb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) kb[i] = f_to_bf16(__fdiv_rn(x[i], nrm));
        const uint2 kw = make_uint2(uint32_t(kb[0]) | (uint32_t(kb[1]) << 16), uint32_t(kb[2]) | (uint32_t(kb[3]) << 16));
        *reinterpret_cast<uint2*>(kr_s + pslot * KSTR + lane * 4) = kw;
        if (owner)
          *reinterpret_cast<uint2*>(p.kr + int64_t(b) * p.kr_sb + int64_t(pslot) * p.kr_st + int64_t(h) * p.kr_sh +
                                    lane * 4) = kw;
      }
    } else if (warp == 2) {
      const int64_t vin = mrow + 2 * int64_t(p.H) * 128 + int64_t(hv) * 128 + row0;
      uint16_t* vdst = p.vr + int64_t(b) * p.vr_sb + int64_t(pslot) * p.vr_st + int64_t(hv) * p.vr_sh + row0;
      for (int r = lane; r < R; r += 32) {
        const uint16_t vb = (p.mx_dt == GDNR_BF16) ? static_cast<const uint16_t*>(p.mixed)[vin + r]
                                                   : f_to_bf16(static_cast<const float*>(p.mixed)[vin + r]);
        vr_s[pslot * VSTR + r] = vb;
        vdst[r] = vb;
      }
    } else if (warp == 3 && lane == 0) {
      const float av = load_scalar(p.a, int64_t(b) * p.a_sb + int64_t(hv) * p.a_sh, p.a_dt);
      const float bv = load_scalar(p.bb, int64_t(b) * p.b_sb + int64_t(hv) * p.b_sh, p.b_dt);
      const float x = av + p.dt_bias[int64_t(hv) * p.db_s];
      const float sp = (x <= SOFTPLUS_THRESHOLD) ? logf(1.0f + expf(x)) : x;
      const float g = round_to(-expf(p.a_log[int64_t(hv) * p.al_s]) * sp, p.gr_dt);
      const float beta = round_to(1.0f / (1.0f + expf(-bv)), p.br_dt);
      gr_s[pslot] = g;
      br_s[pslot] = beta;
      if (z == 0) {
        store_scalar(p.gr, int64_t(b) * p.gr_sb + int64_t(pslot) * p.gr_st + int64_t(hv) * p.gr_sh, p.gr_dt, g);
        store_scalar(p.br, int64_t(b) * p.br_sb + int64_t(pslot) * p.br_st + int64_t(hv) * p.br_sh, p.br_dt, beta);
      }
    }
    if (p.pos_out && hv == 0 && z == 0 && tid == 0) p.pos_out[int64_t(b) * p.po_s] = (pslot + 1) % L;
  } else {
    if (warp == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        qs_s[lane * 4 + i] = load_scalar(p.q, int64_t(b) * p.q_sb + int64_t(h) * p.q_sh + lane * 4 + i, p.q_dt);
    }
  }
  // park this warp's checkpoint rows in the swizzled tile
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int r = 32 * warp + 4 * it + (lane >> 3);
    *reinterpret_cast<uint4*>(s0 + s0_off(r, c8)) = ck[it];
  }
  // one thread waits for the ring copies; the barrier publishes the result
  // (and the prep stage's shared-memory writes) to the whole CTA
  bool mine = true;
  if (ring_bytes && tid == 0) mine = mbar_wait_bounded(bar, 0, p.err);
  const bool ok = __syncthreads_or(!mine) == 0;
  if (!ok) {
    // give copies still in flight a second bounded window before the CTA's
    // shared memory is released
    mbar_wait_bounded(bar, 0, p.err);
    return;
  }

  const int64_t sc_idx = int64_t(b) * p.sc_sb + int64_t(hv) * p.sc_sh + int64_t((row0 + 32 * warp) / VBLOCK) * p.sc_sv;
  const float sc = load_scalar(p.sc, sc_idx, p.sc_dt);
  const int rw0 = 32 * warp;  // first tile row of this warp
  float* misc = reinterpret_cast<float*>(smem + S.misc);
  float* ow = reinterpret_cast<float*>(smem + S.ow) + warp * 32;

  const HeadTile T{s0, kr_s, vr_s, gr_s, br_s, VSTR};
  const HeadScratch X{qs_s,
                      reinterpret_cast<float*>(smem + S.cf),
                      reinterpret_cast<uint16_t*>(smem + S.cb),
                      reinterpret_cast<uint16_t*>(smem + S.qb),
                      smem + S.t8,
                      reinterpret_cast<float*>(smem + S.gram),
                      reinterpret_cast<float*>(smem + S.mg),
                      reinterpret_cast<float*>(smem + S.ad),
                      reinterpret_cast<uint16_t*>(smem + S.kx),
                      reinterpret_cast<float*>(smem + S.ow),
                      misc};
  if (!do_flush) {
    head_nonflush<I8>(T, X, n, sc, warp, lane, CtaSync{});
  } else {
    uint8_t* ck_tile = static_cast<uint8_t*>(p.ck) + int64_t(b) * p.ck_sb + int64_t(hv) * p.ck_sh + int64_t(row0) * 128;
    head_flush<I8>(T, X, n, sc, p.quant_rounded, ck_tile, p.sc, sc_idx, p.sc_dt, warp, lane, tid, blockDim.x, CtaSync{});
  }
  // ---- 12. output rows of this warp
  store_scalar(p.out, int64_t(b) * p.o_sb + int64_t(hv) * p.o_sh + int64_t(row0 + rw0 + lane) * p.o_sv, p.o_dt,
               ow[lane]);
}

template <bool FUSED, bool I8>
static cudaError_t launch_step2_t(const StepParams& p, cudaStream_t stream) {
  const Smem2 s = step2_smem(p.L, p.rows);
  static DynSmemCache smem_cache;  // per device: dynamic smem already allowed for this instance
  cudaError_t e = ensure_dyn_smem(reinterpret_cast<const void*>(step2_kernel<FUSED, I8>), int(s.total), smem_cache);
  if (e != cudaSuccess) return e;
  step2_kernel<FUSED, I8><<<dim3(p.HV, p.B, 128 / p.rows), p.rows, s.total, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_step2(const StepParams& p, bool fused, cudaStream_t stream) {
  if (p.ck_i8) return fused ? launch_step2_t<true, true>(p, stream) : launch_step2_t<false, true>(p, stream);
  return fused ? launch_step2_t<true, false>(p, stream) : launch_step2_t<false, false>(p, stream);
}

}  // namespace gdnr
