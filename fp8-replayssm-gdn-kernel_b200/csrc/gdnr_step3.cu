// Persistent, software-pipelined GDN decode step (sm_100a), the B200 path for
// E4M3 checkpoints with rings of L <= 16.
//
// One CTA per SM, three independent pipelines of four warps.  The value
// heads (b, hv) are dealt to the SMs round-robin (head u goes to CTA
// u mod gridDim.x), and inside an SM the pipelines claim that list through a
// shared-memory counter, so every SM does 13-14 of the 2048 heads of a B=64
// step and the pipelines stay balanced.
//
// Each pipeline keeps two stages.  While it computes head i from stage s it
// has head i+1 streaming into stage s^1 with cp.async (LDGSTS): the 16 KiB
// checkpoint tile (written straight into the 16-byte XOR swizzle the tensor
// core reads conflict-free), the ring rows of the slots the head replays,
// their gates, the four vblock scales and the raw q/k/v rows of this token.
// HBM therefore always has the next heads' bytes in flight while the
// current heads run their latency-bound chains; the per-head math
// (gdnr_head.cuh) is the same as the one-CTA-per-head kernel.
//
// Per-head scalars (ring position / valid length, flush flag, a, b, A_log,
// dt_bias) of the SM's heads are read once into a shared table at start.
#include "gdnr_device.cuh"
#include "gdnr_head.cuh"
#include "gdnr_internal.h"

namespace gdnr {

constexpr int S3_GROUPS = 3;
constexpr int S3_THREADS = 128 * S3_GROUPS;
constexpr int S3_VSTR = 136;  // padded v-ring row (bf16 elements)

struct HeadRec {
  int ninfo;  // fused: ring slot pos (-1 = invalid); replay: clamped valid_len
  int flush;  // replay: flush flag
  float a, b, alog, dtb;
};

struct S3Stage {
  uint32_t s0, kr, vr, gr, br, sc, in;
};

struct S3Group {
  S3Stage st[2];
  uint32_t qs, cf, cb, qb, t8, gram, mg, ad, kx, ow, misc, claim, bytes;
};

struct S3Layout {
  uint32_t ctr, table, group0, group_bytes, total;
};

__host__ __device__ inline S3Stage s3_stage(int L, uint32_t& o) {
  S3Stage s;
  s.s0 = smem_take(o, 128 * 128);
  s.kr = smem_take(o, uint32_t(L) * KSTR * 2);
  s.vr = smem_take(o, uint32_t(L) * S3_VSTR * 2);
  s.gr = smem_take(o, 16 * 4);
  s.br = smem_take(o, 16 * 4);
  s.sc = smem_take(o, 16);
  s.in = smem_take(o, 3 * 512);
  return s;
}

__host__ __device__ inline S3Group s3_group(int L) {
  S3Group G;
  uint32_t o = 0;
  G.st[0] = s3_stage(L, o);
  G.st[1] = s3_stage(L, o);
  G.qs = smem_take(o, 128 * 4);
  G.cf = smem_take(o, 16 * 4);
  G.cb = smem_take(o, 3 * 16 * 2);
  G.qb = smem_take(o, 3 * 128 * 2);
  G.t8 = smem_take(o, 8 * T8STR);
  G.gram = smem_take(o, 16 * 24 * 4);
  G.mg = smem_take(o, 16 * 16 * 4);
  G.ad = smem_take(o, 4 * 16 * 4);
  G.kx = smem_take(o, KX_BYTES);
  G.ow = smem_take(o, 4 * 32 * 4);
  G.misc = smem_take(o, 16);
  G.claim = smem_take(o, 16);
  G.bytes = o;
  return G;
}

__host__ __device__ inline S3Layout s3_layout(int L, int max_heads) {
  S3Layout s;
  uint32_t o = 0;
  s.ctr = smem_take(o, 16);
  s.table = smem_take(o, uint32_t(max_heads) * uint32_t(sizeof(HeadRec)));
  s.group0 = o;
  s.group_bytes = s3_group(L).bytes;
  s.total = o + S3_GROUPS * s.group_bytes;
  return s;
}

template <bool FUSED>
__global__ void __launch_bounds__(S3_THREADS, 1) step3_kernel(const __grid_constant__ StepParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, group = tid >> 7, gtid = tid & 127, warp = gtid >> 5, lane = tid & 31;
  const int c8 = lane & 7;
  const int L = p.L, G = p.HV / p.H;
  const int total = p.B * p.HV;
  const int nh = (total > int(blockIdx.x)) ? (total - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x) : 0;
  const int max_heads = (total + int(gridDim.x) - 1) / int(gridDim.x);
  const S3Layout lay = s3_layout(L, max_heads);
  const S3Group GL = s3_group(L);
  int* ctr = reinterpret_cast<int*>(smem + lay.ctr);
  HeadRec* table = reinterpret_cast<HeadRec*>(smem + lay.table);
  uint8_t* gb = smem + lay.group0 + uint32_t(group) * GL.bytes;
  const GroupSync gsync{1 + group};

  // ---- per-head scalars of this SM's heads
  if (tid == 0) *ctr = 0;
  for (int i = tid; i < nh; i += blockDim.x) {
    const int u = int(blockIdx.x) + i * int(gridDim.x);
    const int b = u / p.HV, hv = u - b * p.HV;
    HeadRec r;
    r.flush = 0;
    r.a = r.b = r.alog = r.dtb = 0.0f;
    if constexpr (FUSED) {
      const int pv = p.pos[int64_t(b) * p.pos_s];
      if (pv < 0 || pv >= L) {
        r.ninfo = -1;
        atomicOr(p.err, GDNR_DEVERR_BAD_POS);
      } else {
        r.ninfo = pv;
      }
      r.a = load_scalar(p.a, int64_t(b) * p.a_sb + int64_t(hv) * p.a_sh, p.a_dt);
      r.b = load_scalar(p.bb, int64_t(b) * p.b_sb + int64_t(hv) * p.b_sh, p.b_dt);
      r.alog = p.a_log[int64_t(hv) * p.al_s];
      r.dtb = p.dt_bias[int64_t(hv) * p.db_s];
    } else {
      int v = p.valid_len[int64_t(b) * p.vl_s];
      r.ninfo = v < 0 ? 0 : (v > L ? L : v);
      r.flush = (p.fl_dt == GDNR_I32) ? (static_cast<const int32_t*>(p.flush)[int64_t(b) * p.fl_s] != 0)
                                      : (static_cast<const uint8_t*>(p.flush)[int64_t(b) * p.fl_s] != 0);
    }
    table[i] = r;
  }
  __syncthreads();

  const int esz_in = FUSED ? (p.mx_dt == GDNR_BF16 ? 2 : 4) : (p.q_dt == GDNR_BF16 ? 2 : 4);

  // ---- stage fill: head i of this SM into stage s of this pipeline (all 128 threads)
  auto prefetch = [&](int i, int s) {
    const HeadRec r = table[i];
    if (r.ninfo < 0) return;
    const int u = int(blockIdx.x) + i * int(gridDim.x);
    const int b = u / p.HV, hv = u - b * p.HV, h = hv / G;
    const S3Stage& S = GL.st[s];
    const int n_mem = r.ninfo;
    const uint8_t* ckh = static_cast<const uint8_t*>(p.ck) + int64_t(b) * p.ck_sb + int64_t(hv) * p.ck_sh;
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int row = 32 * warp + 4 * it + (lane >> 3);
      cp_async16(gb + S.s0 + s0_off(row, c8), ckh + row * 128 + c8 * 16);
    }
    for (int idx = gtid; idx < n_mem * 32; idx += 128) {
      const int t = idx >> 5, w = idx & 31;
      if (w < 16)
        cp_async16(gb + S.kr + (t * KSTR + w * 8) * 2,
                   p.kr + int64_t(b) * p.kr_sb + int64_t(t) * p.kr_st + int64_t(h) * p.kr_sh + w * 8);
      else
        cp_async16(gb + S.vr + (t * S3_VSTR + (w - 16) * 8) * 2,
                   p.vr + int64_t(b) * p.vr_sb + int64_t(t) * p.vr_st + int64_t(hv) * p.vr_sh + (w - 16) * 8);
    }
    if (gtid < n_mem)
      cp_async4(gb + S.gr + gtid * 4, static_cast<const float*>(p.gr) + int64_t(b) * p.gr_sb + int64_t(gtid) * p.gr_st +
                                          int64_t(hv) * p.gr_sh);
    else if (gtid >= 32 && gtid - 32 < n_mem)
      cp_async4(gb + S.br + (gtid - 32) * 4, static_cast<const float*>(p.br) + int64_t(b) * p.br_sb +
                                                 int64_t(gtid - 32) * p.br_st + int64_t(hv) * p.br_sh);
    else if (gtid == 64) {
      const int64_t si = int64_t(b) * p.sc_sb + int64_t(hv) * p.sc_sh;
      if (p.sc_dt == GDNR_F32)
        cp_async16(gb + S.sc, static_cast<const float*>(p.sc) + si);
      else
        cp_async8(gb + S.sc, static_cast<const __half*>(p.sc) + si);
    }
    const int chunks = 8 * esz_in;  // 16-byte pieces of one 128-element row
    if constexpr (FUSED) {
      for (int idx = gtid; idx < 3 * chunks; idx += 128) {
        const int row = idx / chunks, w = idx - row * chunks;
        const int64_t off = row == 0 ? int64_t(h) * 128 : (row == 1 ? int64_t(p.H + h) * 128 : 2 * int64_t(p.H) * 128 + int64_t(hv) * 128);
        cp_async16(gb + S.in + row * 512 + w * 16,
                   static_cast<const uint8_t*>(p.mixed) + (int64_t(b) * p.mx_sb + off) * esz_in + w * 16);
      }
    } else {
      if (gtid < chunks)
        cp_async16(gb + S.in + gtid * 16,
                   static_cast<const uint8_t*>(p.q) + (int64_t(b) * p.q_sb + int64_t(h) * p.q_sh) * esz_in + gtid * 16);
    }
  };

  auto in_value = [&](const uint8_t* row, int i) -> float {
    return esz_in == 2 ? bf16_to_f(reinterpret_cast<const uint16_t*>(row)[i]) : reinterpret_cast<const float*>(row)[i];
  };

  // ---- one head from stage s
  auto compute = [&](int i, int s) {
    const HeadRec r = table[i];
    if (r.ninfo < 0) return;
    const int u = int(blockIdx.x) + i * int(gridDim.x);
    const int b = u / p.HV, hv = u - b * p.HV, h = hv / G;
    const S3Stage& S = GL.st[s];
    const HeadTile T{gb + S.s0, reinterpret_cast<uint16_t*>(gb + S.kr), reinterpret_cast<uint16_t*>(gb + S.vr),
                     reinterpret_cast<float*>(gb + S.gr), reinterpret_cast<float*>(gb + S.br), S3_VSTR};
    const HeadScratch X{reinterpret_cast<float*>(gb + GL.qs),    reinterpret_cast<float*>(gb + GL.cf),
                        reinterpret_cast<uint16_t*>(gb + GL.cb), reinterpret_cast<uint16_t*>(gb + GL.qb),
                        gb + GL.t8,                              reinterpret_cast<float*>(gb + GL.gram),
                        reinterpret_cast<float*>(gb + GL.mg),    reinterpret_cast<float*>(gb + GL.ad),
                        reinterpret_cast<uint16_t*>(gb + GL.kx), reinterpret_cast<float*>(gb + GL.ow),
                        reinterpret_cast<float*>(gb + GL.misc)};
    const uint8_t* in = gb + S.in;
    int n;
    bool do_flush;
    if constexpr (FUSED) {
      const int pslot = r.ninfo;
      n = pslot + 1;
      do_flush = (n == L);
      const bool owner = (hv % G) == 0;  // one head per key head writes k / q_out
      if (warp < 2) {
        float x[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) x[k] = in_value(in + warp * 512, lane * 4 + k);
        const float nrm = sqrtf(warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]) + L2_EPS);
        if (warp == 0) {
          const int qdt = p.q_out ? p.qo_dt : GDNR_BF16;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float y = round_to(__fdiv_rn(x[k], nrm), qdt);
            X.qs[lane * 4 + k] = y;
            if (p.q_out && owner)
              store_scalar(p.q_out, int64_t(b) * p.qo_sb + int64_t(h) * p.qo_sh + lane * 4 + k, qdt, y);
          }
        } else {
          uint16_t kb[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) kb[k] = f_to_bf16(__fdiv_rn(x[k], nrm));
          const uint2 kw =
              make_uint2(uint32_t(kb[0]) | (uint32_t(kb[1]) << 16), uint32_t(kb[2]) | (uint32_t(kb[3]) << 16));
          *reinterpret_cast<uint2*>(T.kr + pslot * KSTR + lane * 4) = kw;
          if (owner)
            *reinterpret_cast<uint2*>(p.kr + int64_t(b) * p.kr_sb + int64_t(pslot) * p.kr_st + int64_t(h) * p.kr_sh +
                                      lane * 4) = kw;
        }
      } else if (warp == 2) {
        uint16_t* vdst = p.vr + int64_t(b) * p.vr_sb + int64_t(pslot) * p.vr_st + int64_t(hv) * p.vr_sh;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int rr = lane + 32 * k;
          const uint16_t vb = esz_in == 2 ? reinterpret_cast<const uint16_t*>(in + 1024)[rr]
                                          : f_to_bf16(reinterpret_cast<const float*>(in + 1024)[rr]);
          T.vr[pslot * S3_VSTR + rr] = vb;
          vdst[rr] = vb;
        }
      } else if (lane == 0) {
        const float x = r.a + r.dtb;
        const float sp = (x <= SOFTPLUS_THRESHOLD) ? logf(1.0f + expf(x)) : x;
        const float g = round_to(-expf(r.alog) * sp, p.gr_dt);
        const float beta = round_to(1.0f / (1.0f + expf(-r.b)), p.br_dt);
        T.gr[pslot] = g;
        T.br[pslot] = beta;
        store_scalar(p.gr, int64_t(b) * p.gr_sb + int64_t(pslot) * p.gr_st + int64_t(hv) * p.gr_sh, p.gr_dt, g);
        store_scalar(p.br, int64_t(b) * p.br_sb + int64_t(pslot) * p.br_st + int64_t(hv) * p.br_sh, p.br_dt, beta);
      }
      if (p.pos_out && hv == 0 && gtid == 0) p.pos_out[int64_t(b) * p.po_s] = (pslot + 1) % L;
    } else {
      n = r.ninfo;
      do_flush = r.flush != 0;
      if (warp == 0) {
#pragma unroll
        for (int k = 0; k < 4; ++k) X.qs[lane * 4 + k] = in_value(in, lane * 4 + k);
      }
    }
    gsync();
    const float sc = p.sc_dt == GDNR_F32 ? reinterpret_cast<const float*>(gb + S.sc)[warp]
                                         : __half2float(reinterpret_cast<const __half*>(gb + S.sc)[warp]);
    if (!do_flush) {
      head_nonflush(T, X, n, sc, warp, lane, gsync);
    } else {
      uint8_t* ck_tile = static_cast<uint8_t*>(p.ck) + int64_t(b) * p.ck_sb + int64_t(hv) * p.ck_sh;
      head_flush(T, X, n, sc, p.quant_rounded, ck_tile, p.sc,
                 int64_t(b) * p.sc_sb + int64_t(hv) * p.sc_sh + int64_t(warp) * p.sc_sv, p.sc_dt, warp, lane, gtid, 128,
                 gsync);
    }
    store_scalar(p.out, int64_t(b) * p.o_sb + int64_t(hv) * p.o_sh + int64_t(32 * warp + lane) * p.o_sv, p.o_dt,
                 X.ow[32 * warp + lane]);
  };

  // ---- pipeline: claim, prefetch the next head, compute the current one
  int* claim = reinterpret_cast<int*>(gb + GL.claim);
  if (gtid == 0) *claim = atomicAdd(ctr, 1);
  gsync();
  int cur = *claim;
  int st = 0;
  if (cur < nh) prefetch(cur, 0);
  cp_async_commit();
  while (cur < nh) {
    gsync();  // every thread has read *claim
    if (gtid == 0) *claim = atomicAdd(ctr, 1);
    gsync();
    const int nxt = *claim;
    if (nxt < nh) prefetch(nxt, st ^ 1);
    cp_async_commit();
    cp_async_wait<1>();  // this thread's copies of `cur` have landed
    gsync();             // ... and everybody's
    compute(cur, st);
    gsync();             // stage st is free again
    cur = nxt;
    st ^= 1;
  }
  cp_async_wait<0>();
}

static int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return n;
}

bool step3_eligible(const StepParams& p, bool fused, bool f32ck) {
  if (f32ck || p.L > STEP2_MAX_L || p.rows != 128) return false;
  if (p.gr_dt != GDNR_F32 || p.br_dt != GDNR_F32) return false;
  if (p.sc_sv != 1 || p.sc_sb % 4 || p.sc_sh % 4) return false;
  const uintptr_t sc_align = p.sc_dt == GDNR_F32 ? 16 : 8;
  if (reinterpret_cast<uintptr_t>(p.sc) % sc_align) return false;
  if (fused) {
    const int esz = p.mx_dt == GDNR_BF16 ? 2 : 4;
    if (reinterpret_cast<uintptr_t>(p.mixed) % 16 || (p.mx_sb * esz) % 16) return false;
  } else {
    const int esz = p.q_dt == GDNR_BF16 ? 2 : 4;
    if (reinterpret_cast<uintptr_t>(p.q) % 16 || (p.q_sb * esz) % 16 || (p.q_sh * esz) % 16) return false;
  }
  const int nsm = sm_count();
  if (nsm <= 0) return false;
  const int64_t total = int64_t(p.B) * p.HV;
  const int grid = int(total < nsm ? total : nsm);
  const int max_heads = int((total + grid - 1) / grid);
  return s3_layout(p.L, max_heads).total <= MAX_DYN_SMEM;
}

cudaError_t launch_step3(const StepParams& p, bool fused, cudaStream_t stream) {
  const int nsm = sm_count();
  const int64_t total = int64_t(p.B) * p.HV;
  const int grid = int(total < nsm ? total : nsm);
  const int max_heads = int((total + grid - 1) / grid);
  const S3Layout lay = s3_layout(p.L, max_heads);
  auto kern = fused ? step3_kernel<true> : step3_kernel<false>;
  static int configured[2] = {0, 0};
  int& conf = configured[fused ? 1 : 0];
  if (int(lay.total) > conf) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(lay.total));
    if (e != cudaSuccess) return e;
    conf = int(lay.total);
  }
  kern<<<grid, S3_THREADS, lay.total, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace gdnr
