// extern "C" entry points of libgdnr: argument validation (shape, dtype,
// stride, alignment, aliasing) and the launch of the kernels.  Nothing here
// allocates device memory or synchronises, except gdnr_read_device_error.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "gdnr_device.cuh"
#include "gdnr_internal.h"

namespace gdnr {

static thread_local std::string g_last_error;

// Library-owned error word used when a call passes error_flag == NULL.
__device__ uint32_t g_device_error;

int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

uint32_t* default_error_word() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return static_cast<uint32_t*>(p);
}

int dtype_size(int dt) {
  switch (dt) {
    case GDNR_F32: case GDNR_I32: return 4;
    case GDNR_F16: case GDNR_BF16: return 2;
    case GDNR_E4M3: case GDNR_U8: case GDNR_I8: return 1;
    default: return 0;
  }
}

static const char* dtype_name(int dt) {
  switch (dt) {
    case GDNR_F32: return "f32";
    case GDNR_F16: return "f16";
    case GDNR_BF16: return "bf16";
    case GDNR_E4M3: return "e4m3";
    case GDNR_I32: return "i32";
    case GDNR_U8: return "u8";
    case GDNR_I8: return "i8";
    default: return "?";
  }
}

int check_tensor(const gdnr_tensor& t, const char* name, int ndim, const int* dtypes, int ndtypes,
                 const int64_t* want) {
  if (t.data == nullptr) return set_error(GDNR_ERR_ARG, "%s: null data pointer", name);
  if (t.ndim != ndim) return set_error(GDNR_ERR_ARG, "%s: expected rank %d, got %d", name, ndim, t.ndim);
  bool dt_ok = false;
  for (int i = 0; i < ndtypes; ++i) dt_ok |= (t.dtype == dtypes[i]);
  if (!dt_ok) {
    std::string allowed;
    for (int i = 0; i < ndtypes; ++i) {
      if (i) allowed += "|";
      allowed += dtype_name(dtypes[i]);
    }
    return set_error(GDNR_ERR_DTYPE, "%s: dtype %s not supported (want %s)", name, dtype_name(t.dtype), allowed.c_str());
  }
  for (int i = 0; i < ndim; ++i) {
    if (t.shape[i] < 0) return set_error(GDNR_ERR_ARG, "%s: negative extent in dim %d", name, i);
    if (want && want[i] >= 0 && t.shape[i] != want[i])
      return set_error(GDNR_ERR_ARG, "%s: dim %d is %lld, expected %lld", name, i, (long long)t.shape[i],
                       (long long)want[i]);
  }
  return GDNR_OK;
}

int check_inner_contiguous(const gdnr_tensor& t, const char* name) {
  if (t.ndim > 0 && t.shape[t.ndim - 1] > 1 && t.stride[t.ndim - 1] != 1)
    return set_error(GDNR_ERR_LAYOUT, "%s: innermost stride must be 1 (got %lld)", name,
                     (long long)t.stride[t.ndim - 1]);
  return GDNR_OK;
}

// Base address and the strides of dims [first, ndim-1) must be 16-byte multiples.
int check_aligned16(const gdnr_tensor& t, const char* name, int first) {
  const int es = dtype_size(t.dtype);
  if (reinterpret_cast<uintptr_t>(t.data) % 16)
    return set_error(GDNR_ERR_LAYOUT, "%s: base address must be 16-byte aligned", name);
  for (int i = first; i < t.ndim - 1; ++i)
    if (t.shape[i] > 1 && (t.stride[i] * es) % 16)
      return set_error(GDNR_ERR_LAYOUT, "%s: stride of dim %d (%lld elements) is not a multiple of 16 bytes", name, i,
                       (long long)t.stride[i]);
  return GDNR_OK;
}

// Conservative byte-range overlap test.
bool overlaps(const gdnr_tensor& a, const gdnr_tensor& b) {
  if (!present(a) || !present(b)) return false;
  auto span = [](const gdnr_tensor& t, uintptr_t& lo, uintptr_t& hi) {
    int64_t last = 0;
    for (int i = 0; i < t.ndim; ++i)
      if (t.shape[i] > 0) last += (t.shape[i] - 1) * (t.stride[i] < 0 ? -t.stride[i] : t.stride[i]);
    lo = reinterpret_cast<uintptr_t>(t.data);
    hi = lo + uintptr_t(last + 1) * dtype_size(t.dtype);
  };
  uintptr_t alo, ahi, blo, bhi;
  span(a, alo, ahi);
  span(b, blo, bhi);
  return alo < bhi && blo < ahi;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return GDNR_OK;
  return set_error(GDNR_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

}  // namespace gdnr

using namespace gdnr;

namespace {

const int DT_F32[] = {GDNR_F32};
const int DT_I32[] = {GDNR_I32};
const int DT_BF16[] = {GDNR_BF16};
const int DT_PAYLOAD[] = {GDNR_E4M3, GDNR_I8};
const int DT_CK[] = {GDNR_E4M3, GDNR_F32, GDNR_I8};
const int DT_SCALE[] = {GDNR_F16, GDNR_F32};
const int DT_ACT[] = {GDNR_BF16, GDNR_F32};
const int DT_GATE[] = {GDNR_F32, GDNR_BF16, GDNR_F16};
const int DT_FLAG[] = {GDNR_U8, GDNR_I32};

#define CHECK(expr)               \
  do {                            \
    int _rc = (expr);             \
    if (_rc != GDNR_OK) return _rc; \
  } while (0)

// Shared validation of the persistent state tuple (checkpoint, scale, rings).
// Fills B, H, HV, L and the StepParams fields of those tensors.
int validate_state(const gdnr_tensor& ck, const gdnr_tensor& sc, const gdnr_tensor& kr, const gdnr_tensor& vr,
                   const gdnr_tensor& gr, const gdnr_tensor& br, StepParams& p, bool& f32ck, int& group) {
  CHECK(check_tensor(kr, "k_ring", 4, DT_BF16, 1, nullptr));
  const int64_t B = kr.shape[0], L = kr.shape[1], H = kr.shape[2], K = kr.shape[3];
  CHECK(check_tensor(vr, "v_ring", 4, DT_BF16, 1, nullptr));
  const int64_t HV = vr.shape[2], V = vr.shape[3];
  if (K != 128 || V != 128)
    return set_error(GDNR_ERR_UNSUPPORTED, "head dims K=%lld V=%lld: only K = V = 128 is implemented", (long long)K,
                     (long long)V);
  if (L < 1 || L > MAX_L) return set_error(GDNR_ERR_UNSUPPORTED, "ring length L=%lld outside [1, %d]", (long long)L, MAX_L);
  if (H < 1 || HV % H) return set_error(GDNR_ERR_ARG, "HV=%lld is not a multiple of H=%lld", (long long)HV, (long long)H);
  group = int(HV / H);
  if (group != 1 && group != 2 && group != 4)
    return set_error(GDNR_ERR_UNSUPPORTED, "HV/H = %d: only 1, 2 or 4 value heads per key head", group);
  if (B > 65535 || H > 65535) return set_error(GDNR_ERR_UNSUPPORTED, "B or H above 65535");
  const int64_t want_v[4] = {B, L, HV, V};
  CHECK(check_tensor(vr, "v_ring", 4, DT_BF16, 1, want_v));
  const int64_t want_g[3] = {B, L, HV};
  CHECK(check_tensor(gr, "g_ring", 3, DT_GATE, 3, want_g));
  CHECK(check_tensor(br, "beta_ring", 3, DT_GATE, 3, want_g));
  const int64_t want_ck[4] = {B, HV, V, K};
  CHECK(check_tensor(ck, "checkpoint", 4, DT_CK, 3, want_ck));
  f32ck = ck.dtype == GDNR_F32;
  p.ck_i8 = ck.dtype == GDNR_I8 ? 1 : 0;
  if (p.ck_i8 && L > STEP2_MAX_L)
    return set_error(GDNR_ERR_UNSUPPORTED, "INT8 checkpoint: ring length L=%lld above %d", (long long)L, STEP2_MAX_L);
  CHECK(check_inner_contiguous(kr, "k_ring"));
  CHECK(check_inner_contiguous(vr, "v_ring"));
  CHECK(check_inner_contiguous(ck, "checkpoint"));
  if (ck.stride[2] != K && V > 1)
    return set_error(GDNR_ERR_LAYOUT, "checkpoint: rows of one head must be packed (stride[2] == K)");
  CHECK(check_aligned16(kr, "k_ring", 0));
  CHECK(check_aligned16(vr, "v_ring", 0));
  CHECK(check_aligned16(ck, "checkpoint", 0));
  if (!f32ck) {
    const int64_t want_s[3] = {B, HV, V / VBLOCK};
    CHECK(check_tensor(sc, "scale", 3, DT_SCALE, 2, want_s));
    p.sc = sc.data;
    p.sc_sb = sc.stride[0];
    p.sc_sh = sc.stride[1];
    p.sc_sv = sc.stride[2];
    p.sc_dt = sc.dtype;
  } else {
    if (present(sc)) return set_error(GDNR_ERR_ARG, "scale must be absent for a float32 checkpoint");
  }
  p.ck = ck.data;
  p.ck_sb = ck.stride[0];
  p.ck_sh = ck.stride[1];
  p.kr = static_cast<uint16_t*>(kr.data);
  p.kr_sb = kr.stride[0];
  p.kr_st = kr.stride[1];
  p.kr_sh = kr.stride[2];
  p.vr = static_cast<uint16_t*>(vr.data);
  p.vr_sb = vr.stride[0];
  p.vr_st = vr.stride[1];
  p.vr_sh = vr.stride[2];
  p.gr = gr.data;
  p.gr_sb = gr.stride[0];
  p.gr_st = gr.stride[1];
  p.gr_sh = gr.stride[2];
  p.gr_dt = gr.dtype;
  p.br = br.data;
  p.br_sb = br.stride[0];
  p.br_st = br.stride[1];
  p.br_sh = br.stride[2];
  p.br_dt = br.dtype;
  p.B = int(B);
  p.H = int(H);
  p.HV = int(HV);
  p.L = int(L);
  return GDNR_OK;
}

int validate_out(const gdnr_tensor& out, StepParams& p) {
  const int64_t want[3] = {p.B, p.HV, 128};
  CHECK(check_tensor(out, "out", 3, DT_ACT, 2, want));
  p.out = out.data;
  p.o_sb = out.stride[0];
  p.o_sh = out.stride[1];
  p.o_sv = out.stride[2];
  p.o_dt = out.dtype;
  return GDNR_OK;
}

int check_launch_opts(int32_t hint, int32_t flags, StepParams& p) {
  if (hint != GDNR_FLUSH_AUTO && hint != GDNR_FLUSH_NONE && hint != GDNR_FLUSH_ALL)
    return set_error(GDNR_ERR_ARG, "flush_hint must be GDNR_FLUSH_AUTO, _NONE or _ALL (got %d)", hint);
  if (flags & ~GDNR_LAUNCH_PDL) return set_error(GDNR_ERR_ARG, "unknown launch_flags bits 0x%x", flags);
  p.flush_hint = hint;
  p.pdl = (flags & GDNR_LAUNCH_PDL) ? 1 : 0;
  return GDNR_OK;
}

// Picks the row tile: the requested one, shrunk until the CTA's shared
// memory fits (only the float32 checkpoint variant ever needs that).
int pick_rows(int requested, int group, int L, bool f32ck, int& rows) {
  if (requested == 0) requested = 128;
  if (requested != 32 && requested != 64 && requested != 128)
    return set_error(GDNR_ERR_ARG, "block_v must be 32, 64 or 128 (got %d)", requested);
  rows = requested;
  while (step_smem_layout(group, L, rows, f32ck ? 4 : 1).total > MAX_DYN_SMEM && rows > 32) rows >>= 1;
  if (step_smem_layout(group, L, rows, f32ck ? 4 : 1).total > MAX_DYN_SMEM)
    return set_error(GDNR_ERR_UNSUPPORTED, "shared memory for G=%d L=%d exceeds 227 KiB", group, L);
  return GDNR_OK;
}

}  // namespace

int gdnr::replay_split_step5(const gdnr_tensor& ck, const gdnr_tensor& sc, const gdnr_tensor& q, const gdnr_tensor& kr,
                       const gdnr_tensor& vr, const gdnr_tensor& gr, const gdnr_tensor& br, const gdnr_tensor& vl,
                       const gdnr_tensor& out, float* tq, const int64_t* tq_s, float* co, const int64_t* co_s,
                       uint32_t* err, cudaStream_t st, int* done) {
  *done = 0;
  StepParams p;
  memset(&p, 0, sizeof(p));
  bool f32ck = false;
  int group = 0;
  CHECK(validate_state(ck, sc, kr, vr, gr, br, p, f32ck, group));
  if (f32ck || tq_s[2] != 1) return GDNR_OK;
  CHECK(validate_out(out, p));
  p.q = q.data;
  p.q_sb = q.stride[0];
  p.q_sh = q.stride[1];
  p.q_dt = q.dtype;
  p.valid_len = static_cast<const int32_t*>(vl.data);
  p.vl_s = vl.stride[0];
  p.flush = nullptr;  // no flush input: every unit replays
  p.rows = 128;
  p.err = err ? err : default_error_word();
  if (!p.err) return GDNR_OK;
  p.flush_hint = GDNR_FLUSH_NONE;
  p.tqo = tq;
  p.tqo_sb = tq_s[0];
  p.tqo_sh = tq_s[1];
  p.coo = co;
  p.coo_sb = co_s[0];
  p.coo_sh = co_s[1];
  p.coo_st = co_s[2];
  if (!step5_eligible(p, false, false)) return GDNR_OK;
  *done = 1;
  if (p.B == 0) return GDNR_OK;
  return cuda_status(launch_step5(p, false, false, st), "gdnr_replay_split launch");
}


extern "C" {

const char* gdnr_last_error(void) { return g_last_error.c_str(); }

const char* gdnr_version(void) { return "gdnr 0.1.0 (sm_100a)"; }

int gdnr_abi_version(void) { return GDNR_ABI_VERSION; }

int gdnr_read_device_error(uint32_t* value, int clear) {
  if (!value) return set_error(GDNR_ERR_ARG, "value: null pointer");
  CHECK(cuda_status(cudaMemcpyFromSymbol(value, g_device_error, sizeof(uint32_t)), "read device error word"));
  if (clear) {
    const uint32_t zero = 0;
    CHECK(cuda_status(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(uint32_t)), "clear device error word"));
  }
  return GDNR_OK;
}

int gdnr_replay(const gdnr_replay_args* a, void* stream) {
  if (!a) return set_error(GDNR_ERR_ARG, "args: null pointer");
  StepParams p;
  memset(&p, 0, sizeof(p));
  bool f32ck = false;
  int group = 0;
  CHECK(validate_state(a->checkpoint, a->scale, a->k_ring, a->v_ring, a->g_ring, a->beta_ring, p, f32ck, group));
  const int64_t want_q[3] = {p.B, p.H, 128};
  CHECK(check_tensor(a->q, "q", 3, DT_ACT, 2, want_q));
  CHECK(check_inner_contiguous(a->q, "q"));
  const int64_t want_b[1] = {p.B};
  CHECK(check_tensor(a->valid_len, "valid_len", 1, DT_I32, 1, want_b));
  CHECK(check_tensor(a->flush, "flush", 1, DT_FLAG, 2, want_b));
  CHECK(validate_out(a->out, p));
  int rows = 128;
  CHECK(pick_rows(a->block_v, group, p.L, f32ck, rows));
  if (a->quant_divisor != 0 && a->quant_divisor != 1)
    return set_error(GDNR_ERR_ARG, "quant_divisor must be 0 or 1");
  p.q = a->q.data;
  p.q_sb = a->q.stride[0];
  p.q_sh = a->q.stride[1];
  p.q_dt = a->q.dtype;
  p.valid_len = static_cast<const int32_t*>(a->valid_len.data);
  p.vl_s = a->valid_len.stride[0];
  p.flush = a->flush.data;
  p.fl_s = a->flush.stride[0];
  p.fl_dt = a->flush.dtype;
  p.rows = rows;
  p.quant_rounded = a->quant_divisor;
  p.err = a->error_flag ? a->error_flag : default_error_word();
  if (!p.err) return set_error(GDNR_ERR_CUDA, "no device error word available");
  CHECK(check_launch_opts(a->flush_hint, a->launch_flags, p));
  if (p.B == 0) return GDNR_OK;
  return cuda_status(launch_step(p, false, f32ck, group, static_cast<cudaStream_t>(stream)), "gdnr_replay launch");
}

int gdnr_fused_step(const gdnr_step_args* a, void* stream) {
  if (!a) return set_error(GDNR_ERR_ARG, "args: null pointer");
  StepParams p;
  memset(&p, 0, sizeof(p));
  bool f32ck = false;
  int group = 0;
  CHECK(validate_state(a->checkpoint, a->scale, a->k_ring, a->v_ring, a->g_ring, a->beta_ring, p, f32ck, group));
  const int64_t width = 2 * int64_t(p.H) * 128 + int64_t(p.HV) * 128;
  const int64_t want_m[2] = {p.B, width};
  CHECK(check_tensor(a->mixed_qkv, "mixed_qkv", 2, DT_ACT, 2, want_m));
  CHECK(check_inner_contiguous(a->mixed_qkv, "mixed_qkv"));
  const int64_t want_ab[2] = {p.B, p.HV};
  CHECK(check_tensor(a->a, "a", 2, DT_GATE, 3, want_ab));
  CHECK(check_tensor(a->b, "b", 2, DT_GATE, 3, want_ab));
  const int64_t want_hv[1] = {p.HV};
  CHECK(check_tensor(a->a_log, "A_log", 1, DT_F32, 1, want_hv));
  CHECK(check_tensor(a->dt_bias, "dt_bias", 1, DT_F32, 1, want_hv));
  const int64_t want_b[1] = {p.B};
  CHECK(check_tensor(a->pos, "pos", 1, DT_I32, 1, want_b));
  if (present(a->pos_out)) {
    CHECK(check_tensor(a->pos_out, "pos_out", 1, DT_I32, 1, want_b));
    if (overlaps(a->pos, a->pos_out)) return set_error(GDNR_ERR_ALIAS, "pos_out must not overlap pos");
    p.pos_out = static_cast<int32_t*>(a->pos_out.data);
    p.po_s = a->pos_out.stride[0];
  }
  if (present(a->q_out)) {
    const int64_t want_q[3] = {p.B, p.H, 128};
    CHECK(check_tensor(a->q_out, "q_out", 3, DT_ACT, 2, want_q));
    CHECK(check_inner_contiguous(a->q_out, "q_out"));
    p.q_out = a->q_out.data;
    p.qo_sb = a->q_out.stride[0];
    p.qo_sh = a->q_out.stride[1];
    p.qo_dt = a->q_out.dtype;
  }
  CHECK(validate_out(a->out, p));
  if (a->quant_divisor != 0 && a->quant_divisor != 1)
    return set_error(GDNR_ERR_ARG, "quant_divisor must be 0 or 1");
  int rows = 128;
  CHECK(pick_rows(128, group, p.L, f32ck, rows));
  p.mixed = a->mixed_qkv.data;
  p.mx_sb = a->mixed_qkv.stride[0];
  p.mx_dt = a->mixed_qkv.dtype;
  p.a = a->a.data;
  p.a_sb = a->a.stride[0];
  p.a_sh = a->a.stride[1];
  p.a_dt = a->a.dtype;
  p.bb = a->b.data;
  p.b_sb = a->b.stride[0];
  p.b_sh = a->b.stride[1];
  p.b_dt = a->b.dtype;
  p.a_log = static_cast<const float*>(a->a_log.data);
  p.al_s = a->a_log.stride[0];
  p.dt_bias = static_cast<const float*>(a->dt_bias.data);
  p.db_s = a->dt_bias.stride[0];
  p.pos = static_cast<const int32_t*>(a->pos.data);
  p.pos_s = a->pos.stride[0];
  p.rows = rows;
  p.quant_rounded = a->quant_divisor;
  p.err = a->error_flag ? a->error_flag : default_error_word();
  if (!p.err) return set_error(GDNR_ERR_CUDA, "no device error word available");
  CHECK(check_launch_opts(a->flush_hint, a->launch_flags, p));
  if (p.B == 0) return GDNR_OK;
  return cuda_status(launch_step(p, true, f32ck, group, static_cast<cudaStream_t>(stream)), "gdnr_fused_step launch");
}

// The serving engine's decode call over a state-slot pool (see include/gdnr.h):
// gdnr_fused_step with every state tensor indexed through state_indices.
int gdnr_packed_decode(const gdnr_packed_decode_args* a, void* stream) {
  if (!a) return set_error(GDNR_ERR_ARG, "args: null pointer");
  StepParams p;
  memset(&p, 0, sizeof(p));
  bool f32ck = false;
  int group = 0;
  CHECK(validate_state(a->checkpoint, a->scale, a->k_ring, a->v_ring, a->g_ring, a->beta_ring, p, f32ck, group));
  if (f32ck || p.ck_i8) return set_error(GDNR_ERR_UNSUPPORTED, "packed decode: E4M3 checkpoints only");
  const int32_t slots = p.B;
  CHECK(check_tensor(a->mixed_qkv, "mixed_qkv", 2, DT_ACT, 2, nullptr));
  const int64_t B = a->mixed_qkv.shape[0];
  if (B > 65535) return set_error(GDNR_ERR_UNSUPPORTED, "batch above 65535");
  p.B = int32_t(B);
  p.S = slots;
  const int64_t width = 2 * int64_t(p.H) * 128 + int64_t(p.HV) * 128;
  const int64_t want_m[2] = {B, width};
  CHECK(check_tensor(a->mixed_qkv, "mixed_qkv", 2, DT_ACT, 2, want_m));
  CHECK(check_inner_contiguous(a->mixed_qkv, "mixed_qkv"));
  const int64_t want_ab[2] = {B, p.HV};
  CHECK(check_tensor(a->a, "a", 2, DT_GATE, 3, want_ab));
  CHECK(check_tensor(a->b, "b", 2, DT_GATE, 3, want_ab));
  const int64_t want_hv[1] = {p.HV};
  CHECK(check_tensor(a->a_log, "A_log", 1, DT_F32, 1, want_hv));
  CHECK(check_tensor(a->dt_bias, "dt_bias", 1, DT_F32, 1, want_hv));
  const int64_t want_b[1] = {B};
  CHECK(check_tensor(a->state_indices, "state_indices", 1, DT_I32, 1, want_b));
  const int64_t want_s[1] = {slots};
  CHECK(check_tensor(a->pos, "pos", 1, DT_I32, 1, want_s));
  if (present(a->pos_out)) {
    CHECK(check_tensor(a->pos_out, "pos_out", 1, DT_I32, 1, want_s));
    if (overlaps(a->pos, a->pos_out)) return set_error(GDNR_ERR_ALIAS, "pos_out must not overlap pos");
    p.pos_out = static_cast<int32_t*>(a->pos_out.data);
    p.po_s = a->pos_out.stride[0];
  }
  // out [B,1,HV,V] (the production layout) or [B,HV,V]
  gdnr_tensor out = a->out;
  if (out.ndim == 4) {
    if (out.shape[1] != 1) return set_error(GDNR_ERR_ARG, "out: dim 1 of a rank-4 out must be 1");
    out.ndim = 3;
    out.shape[1] = out.shape[2];
    out.shape[2] = out.shape[3];
    out.stride[1] = out.stride[2];
    out.stride[2] = out.stride[3];
    out.shape[3] = 0;
    out.stride[3] = 0;
  }
  CHECK(validate_out(out, p));
  if (a->use_qk_l2norm != 1)
    return set_error(GDNR_ERR_UNSUPPORTED, "use_qk_l2norm_in_kernel must be true (the kernel always normalises q, k)");
  const float kscale = 0.08838834764831845f;  // 128^-1/2
  if (!(fabsf(a->qk_scale - kscale) <= 1e-6f * kscale))
    return set_error(GDNR_ERR_UNSUPPORTED, "scale must be head_k_dim^-1/2 = %.9g (got %.9g)", double(kscale),
                     double(a->qk_scale));
  if (a->quant_divisor != 0 && a->quant_divisor != 1)
    return set_error(GDNR_ERR_ARG, "quant_divisor must be 0 or 1");
  p.mixed = a->mixed_qkv.data;
  p.mx_sb = a->mixed_qkv.stride[0];
  p.mx_dt = a->mixed_qkv.dtype;
  p.a = a->a.data;
  p.a_sb = a->a.stride[0];
  p.a_sh = a->a.stride[1];
  p.a_dt = a->a.dtype;
  p.bb = a->b.data;
  p.b_sb = a->b.stride[0];
  p.b_sh = a->b.stride[1];
  p.b_dt = a->b.dtype;
  p.a_log = static_cast<const float*>(a->a_log.data);
  p.al_s = a->a_log.stride[0];
  p.dt_bias = static_cast<const float*>(a->dt_bias.data);
  p.db_s = a->dt_bias.stride[0];
  p.pos = static_cast<const int32_t*>(a->pos.data);
  p.pos_s = a->pos.stride[0];
  p.sidx = static_cast<const int32_t*>(a->state_indices.data);
  p.si_s = a->state_indices.stride[0];
  p.rows = 128;
  p.quant_rounded = a->quant_divisor;
  p.err = a->error_flag ? a->error_flag : default_error_word();
  if (!p.err) return set_error(GDNR_ERR_CUDA, "no device error word available");
  CHECK(check_launch_opts(a->flush_hint, a->launch_flags, p));
  if (!step5_eligible(p, true, false))
    return set_error(GDNR_ERR_UNSUPPORTED,
                     "packed decode: layout outside the persistent step kernel (16-byte aligned rows and rings, "
                     "HV/H = 1 or even, 4 <= L <= 16)");
  if (p.B == 0) return GDNR_OK;
  return cuda_status(launch_step(p, true, false, group, static_cast<cudaStream_t>(stream)),
                     "gdnr_packed_decode launch");
}

static int validate_codec(const gdnr_codec_args* a, CodecParams& p) {
  if (!a) return set_error(GDNR_ERR_ARG, "args: null pointer");
  CHECK(check_tensor(a->state, "state", 4, DT_F32, 1, nullptr));
  const int64_t B = a->state.shape[0], HV = a->state.shape[1], V = a->state.shape[2], K = a->state.shape[3];
  if (K != 128 || V != 128) return set_error(GDNR_ERR_UNSUPPORTED, "only V = K = 128 is implemented");
  const int64_t want[4] = {B, HV, V, K};
  CHECK(check_tensor(a->payload, "payload", 4, DT_PAYLOAD, 2, want));
  const int64_t want_s[3] = {B, HV, V / VBLOCK};
  CHECK(check_tensor(a->scale, "scale", 3, DT_SCALE, 2, want_s));
  CHECK(check_inner_contiguous(a->state, "state"));
  CHECK(check_inner_contiguous(a->payload, "payload"));
  if (a->state.stride[2] != 128 || a->payload.stride[2] != 128)
    return set_error(GDNR_ERR_LAYOUT, "state/payload: rows of one head must be packed (stride[2] == K)");
  CHECK(check_aligned16(a->state, "state", 0));
  CHECK(check_aligned16(a->payload, "payload", 0));
  if (overlaps(a->state, a->payload)) return set_error(GDNR_ERR_ALIAS, "state and payload overlap");
  if (a->quant_divisor != 0 && a->quant_divisor != 1) return set_error(GDNR_ERR_ARG, "quant_divisor must be 0 or 1");
  if (B * HV * 4 > 0x7fffffffLL) return set_error(GDNR_ERR_UNSUPPORTED, "too many vblocks for one launch");
  p.state = static_cast<float*>(a->state.data);
  p.st_sb = a->state.stride[0];
  p.st_sh = a->state.stride[1];
  p.payload = static_cast<uint8_t*>(a->payload.data);
  p.pl_sb = a->payload.stride[0];
  p.pl_sh = a->payload.stride[1];
  p.sc = a->scale.data;
  p.sc_sb = a->scale.stride[0];
  p.sc_sh = a->scale.stride[1];
  p.sc_sv = a->scale.stride[2];
  p.sc_dt = a->scale.dtype;
  p.B = int(B);
  p.HV = int(HV);
  p.quant_rounded = a->quant_divisor;
  p.sat = a->saturation_count;
  p.int8 = a->payload.dtype == GDNR_I8 ? 1 : 0;
  return GDNR_OK;
}

int gdnr_quantize_vblock32(const gdnr_codec_args* a, void* stream) {
  CodecParams p;
  memset(&p, 0, sizeof(p));
  CHECK(validate_codec(a, p));
  if (p.B == 0 || p.HV == 0) return GDNR_OK;
  return cuda_status(launch_quantize(p, static_cast<cudaStream_t>(stream)), "gdnr_quantize_vblock32 launch");
}

int gdnr_dequantize_vblock32(const gdnr_codec_args* a, void* stream) {
  CodecParams p;
  memset(&p, 0, sizeof(p));
  CHECK(validate_codec(a, p));
  if (p.B == 0 || p.HV == 0) return GDNR_OK;
  return cuda_status(launch_dequantize(p, static_cast<cudaStream_t>(stream)), "gdnr_dequantize_vblock32 launch");
}

}  // extern "C"
