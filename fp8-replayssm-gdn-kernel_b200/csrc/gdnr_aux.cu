// Mirrors of the reference's auxiliary operators:
//
// * gdnr_prep_ring    -- standalone prep (kern.py:453-576, wrapper :710-795);
// * gdnr_replay_split -- two-phase replay into caller T / coefficient buffers
//                        (precompute kern.py:798-896, apply :899-1018,
//                        wrapper :1129-1235);
// * gdnr_bf16_step    -- one-token GDN step on a bf16 state, the same-box
//                        read-modify-write control (kern.py:245-341, :408-450).
//
// These are API-completeness paths; the decode hot path is gdnr_fused_step.
#include <cstring>
#include <mutex>

#include "gdnr_device.cuh"
#include "gdnr_internal.h"

namespace gdnr {

constexpr float KSCALE_AUX = 0.08838834764831845f;  // 128^-1/2

// ------------------------------------------------------------------ prep
struct PrepParams {
  const void* mixed;
  int64_t mx_sb;
  int32_t mx_dt;
  const void* a;
  int64_t a_sb, a_sh;
  int32_t a_dt;
  const void* bb;
  int64_t b_sb, b_sh;
  int32_t b_dt;
  const float* a_log;
  int64_t al_s;
  const float* dt_bias;
  int64_t db_s;
  const int32_t* pos;
  int64_t pos_s;
  void* q_out;
  int64_t qo_sb, qo_sh;
  int32_t qo_dt;
  uint16_t* kr;
  int64_t kr_sb, kr_st, kr_sh;
  uint16_t* vr;
  int64_t vr_sb, vr_st, vr_sh;
  void* gr;
  int64_t gr_sb, gr_st, gr_sh;
  int32_t gr_dt;
  void* br;
  int64_t br_sb, br_st, br_sh;
  int32_t br_dt;
  int32_t B, H, HV, L;
  uint32_t* err;
};

// grid (H + HV, B), one warp: programs [0,H) do q/k, [H,H+HV) do v + gates.
__global__ void __launch_bounds__(32) prep_kernel(const __grid_constant__ PrepParams p) {
  const int pid = blockIdx.x, b = blockIdx.y, lane = threadIdx.x;
  const int pv = p.pos[int64_t(b) * p.pos_s];
  if (pv < 0 || pv >= p.L) {
    if (lane == 0 && pid == 0) atomicOr(p.err, GDNR_DEVERR_BAD_POS);
    return;
  }
  const int64_t mrow = int64_t(b) * p.mx_sb;
  if (pid < p.H) {
    const int h = pid;
    float q[4], k[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      q[i] = load_scalar(p.mixed, mrow + int64_t(h) * 128 + lane * 4 + i, p.mx_dt);
      k[i] = load_scalar(p.mixed, mrow + int64_t(p.H + h) * 128 + lane * 4 + i, p.mx_dt);
    }
    const float qn = sqrtf(warp_sum(q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3]) + L2_EPS);
    const float kn = sqrtf(warp_sum(k[0] * k[0] + k[1] * k[1] + k[2] * k[2] + k[3] * k[3]) + L2_EPS);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      store_scalar(p.q_out, int64_t(b) * p.qo_sb + int64_t(h) * p.qo_sh + lane * 4 + i, p.qo_dt, __fdiv_rn(q[i], qn));
      p.kr[int64_t(b) * p.kr_sb + int64_t(pv) * p.kr_st + int64_t(h) * p.kr_sh + lane * 4 + i] =
          f_to_bf16(__fdiv_rn(k[i], kn));
    }
  } else {
    const int hv = pid - p.H;
    const int64_t vin = mrow + 2 * int64_t(p.H) * 128 + int64_t(hv) * 128;
    uint16_t* vdst = p.vr + int64_t(b) * p.vr_sb + int64_t(pv) * p.vr_st + int64_t(hv) * p.vr_sh;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = lane * 4 + i;
      vdst[r] = (p.mx_dt == GDNR_BF16) ? static_cast<const uint16_t*>(p.mixed)[vin + r]
                                       : f_to_bf16(static_cast<const float*>(p.mixed)[vin + r]);
    }
    if (lane == 0) {
      const float x = load_scalar(p.a, int64_t(b) * p.a_sb + int64_t(hv) * p.a_sh, p.a_dt) + p.dt_bias[hv * p.db_s];
      const float sp = (x <= SOFTPLUS_THRESHOLD) ? logf(1.0f + expf(x)) : x;
      const float g = -expf(p.a_log[hv * p.al_s]) * sp;
      const float beta = 1.0f / (1.0f + expf(-load_scalar(p.bb, int64_t(b) * p.b_sb + int64_t(hv) * p.b_sh, p.b_dt)));
      store_scalar(p.gr, int64_t(b) * p.gr_sb + int64_t(pv) * p.gr_st + int64_t(hv) * p.gr_sh, p.gr_dt, g);
      store_scalar(p.br, int64_t(b) * p.br_sb + int64_t(pv) * p.br_st + int64_t(hv) * p.br_sh, p.br_dt, beta);
    }
  }
}

// ------------------------------------------------------------------ split replay
struct SplitParams {
  const uint8_t* ck;  // e4m3 [B,HV,V,K] rows packed
  int64_t ck_sb, ck_sh;
  const void* sc;
  int64_t sc_sb, sc_sh, sc_sv;
  int32_t sc_dt;
  const void* q;
  int64_t q_sb, q_sh;
  int32_t q_dt;
  const uint16_t* kr;
  int64_t kr_sb, kr_st, kr_sh;
  const uint16_t* vr;
  int64_t vr_sb, vr_st, vr_sh;
  const void* gr;
  int64_t gr_sb, gr_st, gr_sh;
  int32_t gr_dt;
  const void* br;
  int64_t br_sb, br_st, br_sh;
  int32_t br_dt;
  const int32_t* valid_len;
  int64_t vl_s;
  float* tq;
  int64_t tq_sb, tq_sh, tq_sk;
  float* coef;
  int64_t co_sb, co_sh, co_st;
  void* out;
  int64_t o_sb, o_sh, o_sv;
  int32_t o_dt;
  int32_t B, H, HV, L, G, rows;
};

// grid (H, B), one warp per value head of the key head (kern.py:1021-1126
// grouped form): T-chain, c_t -> coef[b,hv,t] for t < valid_len, T -> tq.
__global__ void __launch_bounds__(128) split_precompute_kernel(const __grid_constant__ SplitParams p) {
  const int h = blockIdx.x, b = blockIdx.y;
  const int j = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hv = h * p.G + j;  // the block has 32 G threads
  int n = p.valid_len[int64_t(b) * p.vl_s];
  n = n < 0 ? 0 : (n > p.L ? p.L : n);
  // the key head's ring rows (4 elements per lane; shared by the G warps) and each
  // warp's betas and decays of slots t < n, all loaded before the backward chain so
  // that the chain waits on no global load
  __shared__ uint2 ks[MAX_L][32];
  __shared__ float bs[MAX_G][MAX_L], gs[MAX_G][MAX_L];
  for (int t = j; t < n; t += p.G) {
    const uint16_t* kp = p.kr + int64_t(b) * p.kr_sb + int64_t(t) * p.kr_st + int64_t(h) * p.kr_sh + lane * 4;
    ks[t][lane] = make_uint2(uint32_t(kp[0]) | (uint32_t(kp[1]) << 16), uint32_t(kp[2]) | (uint32_t(kp[3]) << 16));
  }
  for (int t = lane; t < n; t += 32) {
    bs[j][t] = load_scalar(p.br, int64_t(b) * p.br_sb + int64_t(t) * p.br_st + int64_t(hv) * p.br_sh, p.br_dt);
    gs[j][t] = expf(load_scalar(p.gr, int64_t(b) * p.gr_sb + int64_t(t) * p.gr_st + int64_t(hv) * p.gr_sh, p.gr_dt));
  }
  float T[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) T[i] = load_scalar(p.q, int64_t(b) * p.q_sb + int64_t(h) * p.q_sh + lane * 4 + i, p.q_dt);
  __syncthreads();
  for (int t = n - 1; t >= 0; --t) {
    const uint2 kw = ks[t][lane];
    const float2 k01 = bf16x2_to_f2(kw.x), k23 = bf16x2_to_f2(kw.y);
    const float k[4] = {k01.x, k01.y, k23.x, k23.y};
    float d = T[0] * k[0];
    d = fmaf(T[1], k[1], d);
    d = fmaf(T[2], k[2], d);
    d = fmaf(T[3], k[3], d);
    d = warp_sum(d);
    const float c = bs[j][t] * d;
    if (lane == 0) p.coef[int64_t(b) * p.co_sb + int64_t(hv) * p.co_sh + int64_t(t) * p.co_st] = c;
    const float gam = gs[j][t];
#pragma unroll
    for (int i = 0; i < 4; ++i) T[i] = gam * (T[i] - c * k[i]);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) p.tq[int64_t(b) * p.tq_sb + int64_t(hv) * p.tq_sh + int64_t(lane * 4 + i) * p.tq_sk] = T[i];
}

// grid (HV, B, 128/rows), 256 threads: out = sum_t c_t v_t + (S_fp8 . T) * scale, * K^-1/2.
__global__ void __launch_bounds__(256) split_apply_kernel(const __grid_constant__ SplitParams p) {
  __shared__ float tq_s[128];
  __shared__ float cf_s[MAX_L];
  __shared__ float sc_s[4];
  __shared__ uint16_t vr_s[MAX_L][128];  // value-ring rows [z rows, (z + 1) rows) of every slot
  const int hv = blockIdx.x, b = blockIdx.y, z = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Every load of the block goes out before the one barrier: the valid length,
  // T, all L coefficients (those at t >= n are masked after the barrier), the four
  // vblock scales, the value-ring rows of all L slots and each warp's checkpoint
  // rows (at most 4 passes of 4 rows, 8 lanes per row).
  const int nraw = p.valid_len[int64_t(b) * p.vl_s];
  const float tqv = tid < 128 ? p.tq[int64_t(b) * p.tq_sb + int64_t(hv) * p.tq_sh + int64_t(tid) * p.tq_sk] : 0.0f;
  const float cfv = tid < p.L ? p.coef[int64_t(b) * p.co_sb + int64_t(hv) * p.co_sh + int64_t(tid) * p.co_st] : 0.0f;
  if (tid < 4) sc_s[tid] = load_scalar(p.sc, int64_t(b) * p.sc_sb + int64_t(hv) * p.sc_sh + int64_t(tid) * p.sc_sv, p.sc_dt);
  for (int idx = tid; idx < p.L * p.rows; idx += 256) {
    const int t = idx / p.rows, rr = idx - t * p.rows;
    vr_s[t][rr] = p.vr[int64_t(b) * p.vr_sb + int64_t(t) * p.vr_st + int64_t(hv) * p.vr_sh + z * p.rows + rr];
  }
  constexpr int NP = 4;
  const int c = lane & 7;
  const int rl0 = warp * 4 + (lane >> 3);  // row within the block's rows
  const int npass = p.rows / 32;
  uint4 w[NP];
#pragma unroll
  for (int k = 0; k < NP; ++k)
    if (k < npass)
      w[k] = *reinterpret_cast<const uint4*>(p.ck + int64_t(b) * p.ck_sb + int64_t(hv) * p.ck_sh +
                                             int64_t(z * p.rows + rl0 + 32 * k) * 128 + c * 16);
  const int n = nraw < 0 ? 0 : (nraw > p.L ? p.L : nraw);
  if (tid < 128) tq_s[tid] = tqv;
  if (tid < p.L) cf_s[tid] = tid < n ? cfv : 0.0f;
  __syncthreads();
  float Tl[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) Tl[i] = tq_s[c * 16 + i];
#pragma unroll
  for (int k = 0; k < NP; ++k) {
    if (k >= npass) break;
    const int rl = rl0 + 32 * k, r = z * p.rows + rl;
    float f[16];
    e4m3x4_to_f4(w[k].x, f);
    e4m3x4_to_f4(w[k].y, f + 4);
    e4m3x4_to_f4(w[k].z, f + 8);
    e4m3x4_to_f4(w[k].w, f + 12);
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) acc = fmaf(f[i], Tl[i], acc);
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    acc += __shfl_xor_sync(0xffffffffu, acc, 4);
    // V^T c of this row: the row's 8 lanes take the slots t = c (mod 8), then reduce
    float ring = 0.0f;
    for (int t = c; t < n; t += 8) ring = fmaf(cf_s[t], bf16_to_f(vr_s[t][rl]), ring);
    ring += __shfl_xor_sync(0xffffffffu, ring, 1);
    ring += __shfl_xor_sync(0xffffffffu, ring, 2);
    ring += __shfl_xor_sync(0xffffffffu, ring, 4);
    if (c == 0)
      store_scalar(p.out, int64_t(b) * p.o_sb + int64_t(hv) * p.o_sh + int64_t(r) * p.o_sv, p.o_dt,
                   fmaf(acc, sc_s[r / VBLOCK], ring) * KSCALE_AUX);
  }
}

// ------------------------------------------------------------------ bf16 step
struct Bf16StepParams {
  uint16_t* state;
  int64_t s_sb, s_sh;
  const void* q;
  int64_t q_sb, q_sh;
  int32_t q_dt;
  const void* k;
  int64_t k_sb, k_sh;
  int32_t k_dt;
  const void* v;
  int64_t v_sb, v_sh, v_sv;
  int32_t v_dt;
  const void* g;
  int64_t g_sb, g_sh;
  int32_t g_dt;
  const void* beta;
  int64_t be_sb, be_sh;
  int32_t be_dt;
  void* out;
  int64_t o_sb, o_sh, o_sv;
  int32_t o_dt;
  int32_t B, H, HV;
};

// grid (HV, B, 256 / NT), NT threads: 8 lanes x 16 columns per row, NT / 8
// rows per pass, 4 passes (NT / 2 rows per CTA).  A thread issues the loads of
// all four of its rows (128 bytes) before it computes the first one, and k / q
// sit in shared memory rather than registers, so that 768 threads fit on an SM
// and keep enough of the state stream in flight to run at HBM speed.
constexpr int BF16_PASSES = 4;
constexpr int BF16_NT = 64;  // threads per CTA (64: 36.5 us, 128: 36.8, 256: 39.0 at B=64, same-box A/B)

template <int NT>
__global__ void __launch_bounds__(NT, 768 / NT) bf16_step_kernel(const __grid_constant__ Bf16StepParams p) {
  __shared__ __align__(16) float kq_s[2][128];
  const int hv = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int h = hv / (p.HV / p.H);
  const int c = tid & 7, r0 = blockIdx.z * (NT / 2) + (tid >> 3);
  uint16_t* head = p.state + int64_t(b) * p.s_sb + int64_t(hv) * p.s_sh + c * 16;
  uint4 w[BF16_PASSES][2];
#pragma unroll
  for (int j = 0; j < BF16_PASSES; ++j) {
    const uint4* src = reinterpret_cast<const uint4*>(head + int64_t(r0 + (NT / 8) * j) * 128);
    w[j][0] = src[0];
    w[j][1] = src[1];
  }
  float vv[BF16_PASSES];
#pragma unroll
  for (int j = 0; j < BF16_PASSES; ++j)
    vv[j] = load_scalar(p.v, int64_t(b) * p.v_sb + int64_t(hv) * p.v_sh + int64_t(r0 + (NT / 8) * j) * p.v_sv,
                        p.v_dt);
  for (int i = tid; i < 256; i += NT) {
    if (i < 128)
      kq_s[0][i] = load_scalar(p.k, int64_t(b) * p.k_sb + int64_t(h) * p.k_sh + i, p.k_dt);
    else
      kq_s[1][i - 128] = load_scalar(p.q, int64_t(b) * p.q_sb + int64_t(h) * p.q_sh + i - 128, p.q_dt);
  }
  const float gam = expf(load_scalar(p.g, int64_t(b) * p.g_sb + int64_t(hv) * p.g_sh, p.g_dt));
  const float be = load_scalar(p.beta, int64_t(b) * p.be_sb + int64_t(hv) * p.be_sh, p.be_dt);
  __syncthreads();
  const float4* kk4 = reinterpret_cast<const float4*>(kq_s[0] + c * 16);
  const float4* qq4 = reinterpret_cast<const float4*>(kq_s[1] + c * 16);
#pragma unroll
  for (int j = 0; j < BF16_PASSES; ++j) {
    const int r = r0 + (NT / 8) * j;
    const uint32_t ws[8] = {w[j][0].x, w[j][0].y, w[j][0].z, w[j][0].w, w[j][1].x, w[j][1].y, w[j][1].z, w[j][1].w};
    float s[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float2 f = bf16x2_to_f2(ws[i]);
      s[2 * i] = f.x * gam;
      s[2 * i + 1] = f.y * gam;
    }
    float kk[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 k4 = kk4[i];
      kk[4 * i] = k4.x;
      kk[4 * i + 1] = k4.y;
      kk[4 * i + 2] = k4.z;
      kk[4 * i + 3] = k4.w;
    }
    float d = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) d = fmaf(s[i], kk[i], d);
    d += __shfl_xor_sync(0xffffffffu, d, 1);
    d += __shfl_xor_sync(0xffffffffu, d, 2);
    d += __shfl_xor_sync(0xffffffffu, d, 4);
    const float corr = (vv[j] - d) * be;
    float o = 0.0f;
    uint32_t wo[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 q4 = qq4[i];
      const float qv[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        s[4 * i + e] = fmaf(corr, kk[4 * i + e], s[4 * i + e]);
        o = fmaf(s[4 * i + e], qv[e], o);
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) wo[i] = uint32_t(f_to_bf16(s[2 * i])) | (uint32_t(f_to_bf16(s[2 * i + 1])) << 16);
    uint4* dst = reinterpret_cast<uint4*>(head + int64_t(r) * 128);
    dst[0] = make_uint4(wo[0], wo[1], wo[2], wo[3]);
    dst[1] = make_uint4(wo[4], wo[5], wo[6], wo[7]);
    o += __shfl_xor_sync(0xffffffffu, o, 1);
    o += __shfl_xor_sync(0xffffffffu, o, 2);
    o += __shfl_xor_sync(0xffffffffu, o, 4);
    if (c == 0) store_scalar(p.out, int64_t(b) * p.o_sb + int64_t(hv) * p.o_sh + int64_t(r) * p.o_sv, p.o_dt, o * KSCALE_AUX);
  }
}

// ---------------------------------------------------------------- static-scratch split replay
// gdnr_replay_split needs two caller buffers (T and c).  This variant keeps
// them in one file-scope device array so that a caller which cannot allocate
// device memory when it calls the replay can still use the split path; the
// array is sized for GDNR_SPLIT_STATIC_MAX_PAIRS (sequence, value head) pairs
// and rings of up to MAX_L slots: 4096 x (128 + 64) floats = 3 MiB per device.
static_assert(GDNR_SPLIT_STATIC_MAX_L == MAX_L, "static scratch is sized for MAX_L ring slots");
constexpr int64_t SPLIT_STATIC_TQ = int64_t(GDNR_SPLIT_STATIC_MAX_PAIRS) * 128;
constexpr int64_t SPLIT_STATIC_FLOATS = int64_t(GDNR_SPLIT_STATIC_MAX_PAIRS) * (128 + MAX_L);
static __device__ __align__(256) float g_split_scratch[SPLIT_STATIC_FLOATS];

constexpr int SPLIT_STATIC_MAX_DEVICES = 64;
static float* g_split_scratch_ptr[SPLIT_STATIC_MAX_DEVICES] = {};
static std::mutex g_split_scratch_mu;

// Device address of the scratch array on the current device, looked up once
// per device (with that device current) and cached.
static int split_scratch_for_current_device(float** out) {
  int dev = -1;
  int rc = cuda_status(cudaGetDevice(&dev), "gdnr_replay_split_static: cudaGetDevice");
  if (rc != GDNR_OK) return rc;
  if (dev < 0 || dev >= SPLIT_STATIC_MAX_DEVICES)
    return set_error(GDNR_ERR_UNSUPPORTED, "gdnr_replay_split_static: device index %d above %d", dev,
                     SPLIT_STATIC_MAX_DEVICES - 1);
  std::lock_guard<std::mutex> lock(g_split_scratch_mu);
  if (!g_split_scratch_ptr[dev]) {
    void* ptr = nullptr;
    rc = cuda_status(cudaGetSymbolAddress(&ptr, g_split_scratch), "gdnr_replay_split_static: cudaGetSymbolAddress");
    if (rc != GDNR_OK) return rc;
    g_split_scratch_ptr[dev] = static_cast<float*>(ptr);
  }
  *out = g_split_scratch_ptr[dev];
  return GDNR_OK;
}

}  // namespace gdnr

using namespace gdnr;

namespace {
const int A_F32[] = {GDNR_F32};
const int A_I32[] = {GDNR_I32};
const int A_BF16[] = {GDNR_BF16};
const int A_E4M3[] = {GDNR_E4M3};
const int A_SCALE[] = {GDNR_F16, GDNR_F32};
const int A_ACT[] = {GDNR_BF16, GDNR_F32};
const int A_GATE[] = {GDNR_F32, GDNR_BF16, GDNR_F16};
#define CK(expr)                    \
  do {                              \
    int _rc = (expr);               \
    if (_rc != GDNR_OK) return _rc; \
  } while (0)
}  // namespace

extern "C" {

int gdnr_prep_ring(const gdnr_prep_args* a, void* stream) {
  if (!a) return set_error(GDNR_ERR_ARG, "args: null pointer");
  PrepParams p;
  memset(&p, 0, sizeof(p));
  CK(check_tensor(a->k_ring, "k_ring", 4, A_BF16, 1, nullptr));
  const int64_t B = a->k_ring.shape[0], L = a->k_ring.shape[1], H = a->k_ring.shape[2];
  if (a->k_ring.shape[3] != 128) return set_error(GDNR_ERR_UNSUPPORTED, "only K = 128 is implemented");
  CK(check_tensor(a->v_ring, "v_ring", 4, A_BF16, 1, nullptr));
  const int64_t HV = a->v_ring.shape[2];
  const int64_t want_v[4] = {B, L, HV, 128};
  CK(check_tensor(a->v_ring, "v_ring", 4, A_BF16, 1, want_v));
  if (L < 1 || H < 1 || HV < 1 || HV % H) return set_error(GDNR_ERR_ARG, "inconsistent ring geometry");
  const int64_t want_g[3] = {B, L, HV};
  CK(check_tensor(a->g_ring, "g_ring", 3, A_GATE, 3, want_g));
  CK(check_tensor(a->beta_ring, "beta_ring", 3, A_GATE, 3, want_g));
  const int64_t want_m[2] = {B, 2 * H * 128 + HV * 128};
  CK(check_tensor(a->mixed_qkv, "mixed_qkv", 2, A_ACT, 2, want_m));
  CK(check_inner_contiguous(a->mixed_qkv, "mixed_qkv"));
  const int64_t want_ab[2] = {B, HV};
  CK(check_tensor(a->a, "a", 2, A_GATE, 3, want_ab));
  CK(check_tensor(a->b, "b", 2, A_GATE, 3, want_ab));
  const int64_t want_hv[1] = {HV};
  CK(check_tensor(a->a_log, "A_log", 1, A_F32, 1, want_hv));
  CK(check_tensor(a->dt_bias, "dt_bias", 1, A_F32, 1, want_hv));
  const int64_t want_b[1] = {B};
  CK(check_tensor(a->pos, "pos", 1, A_I32, 1, want_b));
  const int64_t want_q[3] = {B, H, 128};
  CK(check_tensor(a->q_out, "q_out", 3, A_ACT, 2, want_q));
  CK(check_inner_contiguous(a->q_out, "q_out"));
  CK(check_inner_contiguous(a->k_ring, "k_ring"));
  CK(check_inner_contiguous(a->v_ring, "v_ring"));
  if (B > 65535 || H + HV > 2147483647LL) return set_error(GDNR_ERR_UNSUPPORTED, "grid too large");
  p.mixed = a->mixed_qkv.data; p.mx_sb = a->mixed_qkv.stride[0]; p.mx_dt = a->mixed_qkv.dtype;
  p.a = a->a.data; p.a_sb = a->a.stride[0]; p.a_sh = a->a.stride[1]; p.a_dt = a->a.dtype;
  p.bb = a->b.data; p.b_sb = a->b.stride[0]; p.b_sh = a->b.stride[1]; p.b_dt = a->b.dtype;
  p.a_log = static_cast<const float*>(a->a_log.data); p.al_s = a->a_log.stride[0];
  p.dt_bias = static_cast<const float*>(a->dt_bias.data); p.db_s = a->dt_bias.stride[0];
  p.pos = static_cast<const int32_t*>(a->pos.data); p.pos_s = a->pos.stride[0];
  p.q_out = a->q_out.data; p.qo_sb = a->q_out.stride[0]; p.qo_sh = a->q_out.stride[1]; p.qo_dt = a->q_out.dtype;
  p.kr = static_cast<uint16_t*>(a->k_ring.data);
  p.kr_sb = a->k_ring.stride[0]; p.kr_st = a->k_ring.stride[1]; p.kr_sh = a->k_ring.stride[2];
  p.vr = static_cast<uint16_t*>(a->v_ring.data);
  p.vr_sb = a->v_ring.stride[0]; p.vr_st = a->v_ring.stride[1]; p.vr_sh = a->v_ring.stride[2];
  p.gr = a->g_ring.data; p.gr_sb = a->g_ring.stride[0]; p.gr_st = a->g_ring.stride[1]; p.gr_sh = a->g_ring.stride[2];
  p.gr_dt = a->g_ring.dtype;
  p.br = a->beta_ring.data; p.br_sb = a->beta_ring.stride[0]; p.br_st = a->beta_ring.stride[1];
  p.br_sh = a->beta_ring.stride[2]; p.br_dt = a->beta_ring.dtype;
  p.B = int(B); p.H = int(H); p.HV = int(HV); p.L = int(L);
  p.err = a->error_flag ? a->error_flag : default_error_word();
  if (!p.err) return set_error(GDNR_ERR_CUDA, "no device error word available");
  if (B == 0) return GDNR_OK;
  prep_kernel<<<dim3(unsigned(H + HV), unsigned(B)), 32, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return cuda_status(cudaGetLastError(), "gdnr_prep_ring launch");
}

int gdnr_replay_split(const gdnr_replay_split_args* a, void* stream) {
  if (!a) return set_error(GDNR_ERR_ARG, "args: null pointer");
  SplitParams p;
  memset(&p, 0, sizeof(p));
  CK(check_tensor(a->k_ring, "k_ring", 4, A_BF16, 1, nullptr));
  const int64_t B = a->k_ring.shape[0], L = a->k_ring.shape[1], H = a->k_ring.shape[2];
  CK(check_tensor(a->v_ring, "v_ring", 4, A_BF16, 1, nullptr));
  const int64_t HV = a->v_ring.shape[2];
  if (a->k_ring.shape[3] != 128 || a->v_ring.shape[3] != 128)
    return set_error(GDNR_ERR_UNSUPPORTED, "only K = V = 128 is implemented");
  if (L < 1 || L > MAX_L) return set_error(GDNR_ERR_UNSUPPORTED, "ring length outside [1, %d]", MAX_L);
  if (H < 1 || HV % H || HV / H > 4) return set_error(GDNR_ERR_UNSUPPORTED, "HV/H must be 1, 2 or 4");
  const int64_t want_v[4] = {B, L, HV, 128};
  CK(check_tensor(a->v_ring, "v_ring", 4, A_BF16, 1, want_v));
  const int64_t want_g[3] = {B, L, HV};
  CK(check_tensor(a->g_ring, "g_ring", 3, A_GATE, 3, want_g));
  CK(check_tensor(a->beta_ring, "beta_ring", 3, A_GATE, 3, want_g));
  const int64_t want_ck[4] = {B, HV, 128, 128};
  CK(check_tensor(a->checkpoint, "checkpoint", 4, A_E4M3, 1, want_ck));
  if (a->checkpoint.stride[3] != 1 || a->checkpoint.stride[2] != 128)
    return set_error(GDNR_ERR_LAYOUT, "checkpoint: rows must be packed");
  CK(check_aligned16(a->checkpoint, "checkpoint", 0));
  const int64_t want_s[3] = {B, HV, 4};
  CK(check_tensor(a->scale, "scale", 3, A_SCALE, 2, want_s));
  const int64_t want_q[3] = {B, H, 128};
  CK(check_tensor(a->q, "q", 3, A_ACT, 2, want_q));
  CK(check_inner_contiguous(a->q, "q"));
  CK(check_inner_contiguous(a->k_ring, "k_ring"));
  const int64_t want_b[1] = {B};
  CK(check_tensor(a->valid_len, "valid_len", 1, A_I32, 1, want_b));
  const int64_t want_tq[3] = {B, HV, 128};
  CK(check_tensor(a->tq, "tq", 3, A_F32, 1, want_tq));
  const int64_t want_co[3] = {B, HV, L};
  CK(check_tensor(a->coef, "coef", 3, A_F32, 1, want_co));
  const int64_t want_o[3] = {B, HV, 128};
  CK(check_tensor(a->out, "out", 3, A_ACT, 2, want_o));
  if (overlaps(a->tq, a->coef)) return set_error(GDNR_ERR_ALIAS, "tq and coef overlap");
  int rows = a->block_v ? a->block_v : 128;
  if (rows != 32 && rows != 64 && rows != 128) return set_error(GDNR_ERR_ARG, "block_v must be 32, 64 or 128");
  if (B > 65535) return set_error(GDNR_ERR_UNSUPPORTED, "B above 65535");
  p.ck = static_cast<const uint8_t*>(a->checkpoint.data);
  p.ck_sb = a->checkpoint.stride[0]; p.ck_sh = a->checkpoint.stride[1];
  p.sc = a->scale.data; p.sc_sb = a->scale.stride[0]; p.sc_sh = a->scale.stride[1]; p.sc_sv = a->scale.stride[2];
  p.sc_dt = a->scale.dtype;
  p.q = a->q.data; p.q_sb = a->q.stride[0]; p.q_sh = a->q.stride[1]; p.q_dt = a->q.dtype;
  p.kr = static_cast<const uint16_t*>(a->k_ring.data);
  p.kr_sb = a->k_ring.stride[0]; p.kr_st = a->k_ring.stride[1]; p.kr_sh = a->k_ring.stride[2];
  p.vr = static_cast<const uint16_t*>(a->v_ring.data);
  p.vr_sb = a->v_ring.stride[0]; p.vr_st = a->v_ring.stride[1]; p.vr_sh = a->v_ring.stride[2];
  p.gr = a->g_ring.data; p.gr_sb = a->g_ring.stride[0]; p.gr_st = a->g_ring.stride[1]; p.gr_sh = a->g_ring.stride[2];
  p.gr_dt = a->g_ring.dtype;
  p.br = a->beta_ring.data; p.br_sb = a->beta_ring.stride[0]; p.br_st = a->beta_ring.stride[1];
  p.br_sh = a->beta_ring.stride[2]; p.br_dt = a->beta_ring.dtype;
  p.valid_len = static_cast<const int32_t*>(a->valid_len.data); p.vl_s = a->valid_len.stride[0];
  p.tq = static_cast<float*>(a->tq.data); p.tq_sb = a->tq.stride[0]; p.tq_sh = a->tq.stride[1]; p.tq_sk = a->tq.stride[2];
  p.coef = static_cast<float*>(a->coef.data);
  p.co_sb = a->coef.stride[0]; p.co_sh = a->coef.stride[1]; p.co_st = a->coef.stride[2];
  p.out = a->out.data; p.o_sb = a->out.stride[0]; p.o_sh = a->out.stride[1]; p.o_sv = a->out.stride[2];
  p.o_dt = a->out.dtype;
  p.B = int(B); p.H = int(H); p.HV = int(HV); p.L = int(L); p.G = int(HV / H); p.rows = rows;
  if (B == 0) return GDNR_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the persistent step kernel in replay mode, writing T and c as it goes, where it
  // takes the layout; else the precompute + apply kernels below
  {
    const int64_t tq_s[3] = {a->tq.stride[0], a->tq.stride[1], a->tq.stride[2]};
    const int64_t co_s[3] = {a->coef.stride[0], a->coef.stride[1], a->coef.stride[2]};
    int done = 0;
    CK(replay_split_step5(a->checkpoint, a->scale, a->q, a->k_ring, a->v_ring, a->g_ring, a->beta_ring, a->valid_len,
                          a->out, p.tq, tq_s, p.coef, co_s, static_cast<uint32_t*>(a->error_flag), st, &done));
    if (done) return GDNR_OK;
  }
  split_precompute_kernel<<<dim3(unsigned(H), unsigned(B)), 32 * p.G, 0, st>>>(p);
  CK(cuda_status(cudaGetLastError(), "gdnr_replay_split precompute launch"));
  split_apply_kernel<<<dim3(unsigned(HV), unsigned(B), unsigned(128 / rows)), 256, 0, st>>>(p);
  return cuda_status(cudaGetLastError(), "gdnr_replay_split apply launch");
}

int gdnr_replay_split_static(const gdnr_replay_split_static_args* a, void* stream) {
  if (!a) return set_error(GDNR_ERR_ARG, "args: null pointer");
  if (a->k_ring.ndim != 4 || a->v_ring.ndim != 4)
    return set_error(GDNR_ERR_ARG, "k_ring and v_ring must be 4-D [B,L,H,K] / [B,L,HV,V]");
  const int64_t B = a->k_ring.shape[0], L = a->k_ring.shape[1], HV = a->v_ring.shape[2];
  if (B < 0 || HV < 0) return set_error(GDNR_ERR_ARG, "gdnr_replay_split_static: negative extent");
  // each factor is bounded before the product is formed, so B*HV cannot overflow
  if (B > GDNR_SPLIT_STATIC_MAX_PAIRS || HV > GDNR_SPLIT_STATIC_MAX_PAIRS || B * HV > GDNR_SPLIT_STATIC_MAX_PAIRS)
    return set_error(GDNR_ERR_UNSUPPORTED,
                     "gdnr_replay_split_static: B = %lld, HV = %lld exceed the static scratch's %d (sequence, value "
                     "head) pairs; use gdnr_replay_split with caller buffers",
                     static_cast<long long>(B), static_cast<long long>(HV), GDNR_SPLIT_STATIC_MAX_PAIRS);
  if (L < 1 || L > GDNR_SPLIT_STATIC_MAX_L)
    return set_error(GDNR_ERR_UNSUPPORTED, "gdnr_replay_split_static: ring length %lld outside [1, %d]",
                     static_cast<long long>(L), GDNR_SPLIT_STATIC_MAX_L);
  float* scratch = nullptr;
  CK(split_scratch_for_current_device(&scratch));
  gdnr_replay_split_args s;
  memset(&s, 0, sizeof(s));
  s.checkpoint = a->checkpoint;
  s.scale = a->scale;
  s.q = a->q;
  s.k_ring = a->k_ring;
  s.v_ring = a->v_ring;
  s.g_ring = a->g_ring;
  s.beta_ring = a->beta_ring;
  s.valid_len = a->valid_len;
  s.out = a->out;
  s.block_v = a->block_v;
  s.error_flag = a->error_flag;
  // T [B,HV,128] then c [B,HV,L], both contiguous, inside the scratch; every
  // element the apply phase reads is written by the precompute phase of the
  // same call, so nothing has to start at zero
  s.tq.data = scratch;
  s.tq.dtype = GDNR_F32;
  s.tq.ndim = 3;
  s.tq.shape[0] = B; s.tq.shape[1] = HV; s.tq.shape[2] = 128;
  s.tq.stride[0] = HV * 128; s.tq.stride[1] = 128; s.tq.stride[2] = 1;
  s.coef.data = scratch + SPLIT_STATIC_TQ;
  s.coef.dtype = GDNR_F32;
  s.coef.ndim = 3;
  s.coef.shape[0] = B; s.coef.shape[1] = HV; s.coef.shape[2] = L;
  s.coef.stride[0] = HV * L; s.coef.stride[1] = L; s.coef.stride[2] = 1;
  return gdnr_replay_split(&s, stream);
}

int gdnr_bf16_step(const gdnr_bf16_step_args* a, void* stream) {
  if (!a) return set_error(GDNR_ERR_ARG, "args: null pointer");
  Bf16StepParams p;
  memset(&p, 0, sizeof(p));
  CK(check_tensor(a->state, "state", 4, A_BF16, 1, nullptr));
  const int64_t B = a->state.shape[0], HV = a->state.shape[1];
  if (a->state.shape[2] != 128 || a->state.shape[3] != 128)
    return set_error(GDNR_ERR_UNSUPPORTED, "only V = K = 128 is implemented");
  if (a->state.stride[3] != 1 || a->state.stride[2] != 128)
    return set_error(GDNR_ERR_LAYOUT, "state: rows must be packed");
  CK(check_aligned16(a->state, "state", 0));
  CK(check_tensor(a->q, "q", 3, A_ACT, 2, nullptr));
  const int64_t H = a->q.shape[1];
  if (H < 1 || HV % H) return set_error(GDNR_ERR_ARG, "HV must be a multiple of H");
  const int64_t want_qk[3] = {B, H, 128};
  CK(check_tensor(a->q, "q", 3, A_ACT, 2, want_qk));
  CK(check_tensor(a->k, "k", 3, A_ACT, 2, want_qk));
  const int64_t want_v[3] = {B, HV, 128};
  CK(check_tensor(a->v, "v", 3, A_ACT, 2, want_v));
  CK(check_tensor(a->out, "out", 3, A_ACT, 2, want_v));
  const int64_t want_g[2] = {B, HV};
  CK(check_tensor(a->g, "g", 2, A_GATE, 3, want_g));
  CK(check_tensor(a->beta, "beta", 2, A_GATE, 3, want_g));
  CK(check_inner_contiguous(a->q, "q"));
  CK(check_inner_contiguous(a->k, "k"));
  if (B > 65535) return set_error(GDNR_ERR_UNSUPPORTED, "B above 65535");
  p.state = static_cast<uint16_t*>(a->state.data); p.s_sb = a->state.stride[0]; p.s_sh = a->state.stride[1];
  p.q = a->q.data; p.q_sb = a->q.stride[0]; p.q_sh = a->q.stride[1]; p.q_dt = a->q.dtype;
  p.k = a->k.data; p.k_sb = a->k.stride[0]; p.k_sh = a->k.stride[1]; p.k_dt = a->k.dtype;
  p.v = a->v.data; p.v_sb = a->v.stride[0]; p.v_sh = a->v.stride[1]; p.v_sv = a->v.stride[2]; p.v_dt = a->v.dtype;
  p.g = a->g.data; p.g_sb = a->g.stride[0]; p.g_sh = a->g.stride[1]; p.g_dt = a->g.dtype;
  p.beta = a->beta.data; p.be_sb = a->beta.stride[0]; p.be_sh = a->beta.stride[1]; p.be_dt = a->beta.dtype;
  p.out = a->out.data; p.o_sb = a->out.stride[0]; p.o_sh = a->out.stride[1]; p.o_sv = a->out.stride[2];
  p.o_dt = a->out.dtype;
  p.B = int(B); p.H = int(H); p.HV = int(HV);
  if (B == 0) return GDNR_OK;
  bf16_step_kernel<BF16_NT>
      <<<dim3(unsigned(HV), unsigned(B), 256 / BF16_NT), BF16_NT, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return cuda_status(cudaGetLastError(), "gdnr_bf16_step launch");
}

}  // extern "C"
