// Internal (non-ABI) declarations shared by the gdnr translation units:
// kernel parameter blocks, the shared-memory layout of the step kernel and
// the host-side argument validation helpers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>
#include <string>

#include "../../include/gdnr.h"

namespace gdnr {

// ---------------------------------------------------------------- step kernel
// One parameter block serves both the replay mirror (gdnr_replay) and the
// fused full-contract step (gdnr_fused_step).  Strides are in elements.
struct StepParams {
  void* ck;  // checkpoint [B,HV,V,K] (rows of K contiguous)
  int64_t ck_sb, ck_sh;
  void* sc;  // scales [B,HV,V/32]
  int64_t sc_sb, sc_sh, sc_sv;
  int32_t sc_dt;
  const void* q;  // replay mode: normalised q [B,H,K]
  int64_t q_sb, q_sh;
  int32_t q_dt;
  uint16_t* kr;  // k ring [B,L,H,K] bf16
  int64_t kr_sb, kr_st, kr_sh;
  uint16_t* vr;  // v ring [B,L,HV,V] bf16
  int64_t vr_sb, vr_st, vr_sh;
  void* gr;  // g ring [B,L,HV]
  int64_t gr_sb, gr_st, gr_sh;
  int32_t gr_dt;
  void* br;  // beta ring [B,L,HV]
  int64_t br_sb, br_st, br_sh;
  int32_t br_dt;
  const int32_t* valid_len;  // replay mode
  int64_t vl_s;
  const void* flush;
  int64_t fl_s;
  int32_t fl_dt;
  const int32_t* pos;  // fused mode
  int64_t pos_s;
  int32_t* pos_out;
  int64_t po_s;
  const void* mixed;  // fused mode: [B, 2HK + HV V]
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
  void* q_out;
  int64_t qo_sb, qo_sh;
  int32_t qo_dt;
  void* out;  // [B,HV,V]
  int64_t o_sb, o_sh, o_sv;
  int32_t o_dt;
  int32_t B, H, HV, L;
  int32_t rows;  // value rows per CTA (32/64/128)
  int32_t quant_rounded;
  uint32_t* err;
  int32_t flush_hint;   // GDNR_FLUSH_*
  int32_t pdl;          // launch with programmatic stream serialization
  // packed decode: batch row b uses state slot sidx[b * si_s] of every state
  // tensor (S slots; an index <= 0 is the null slot); null = the state is indexed by b
  const int32_t* sidx;
  int64_t si_s;
  int32_t S;
  // the checkpoint holds int8 codes ("vblock_int8"); launched on the
  // one-CTA-per-head kernel (gdnr_step2.cu) only
  int32_t ck_i8;
  // persistent step without the flush path: the gate rings are read by TMA
  // (set by its launcher when their layout allows)
  int32_t gtma;
  // persistent step: one value head per work unit even when two share a key head
  // (set by its launcher for steps without the flush path on small batches)
  int32_t hpu1;
  // split replay (gdnr_replay_split): the persistent kernel also writes the
  // transformed query T [B,HV,K] (innermost contiguous) and the coefficients c_t
  // (t < valid_len) [B,HV,L] to these caller buffers; null otherwise
  float* tqo;
  int64_t tqo_sb, tqo_sh;
  float* coo;
  int64_t coo_sb, coo_sh, coo_st;
};

struct SmemLayout {
  uint32_t bar, ck, kr, vr, gr, br, tq, cf, orng, ofin, qs, red, total;
};

__host__ __device__ inline uint32_t smem_take(uint32_t& off, uint32_t bytes) {
  uint32_t r = off;
  off = (off + bytes + 127u) & ~127u;
  return r;
}

__host__ __device__ inline SmemLayout step_smem_layout(int G, int L, int rows, int ck_esize) {
  SmemLayout s;
  uint32_t o = 0;
  s.bar = smem_take(o, 8 * 8);
  s.ck = smem_take(o, uint32_t(G) * rows * 128 * ck_esize);
  s.kr = smem_take(o, uint32_t(L) * 128 * 2);
  s.vr = smem_take(o, uint32_t(G) * L * rows * 2);
  s.gr = smem_take(o, uint32_t(G) * L * 4);
  s.br = smem_take(o, uint32_t(G) * L * 4);
  s.tq = smem_take(o, uint32_t(G) * 128 * 4);
  s.cf = smem_take(o, uint32_t(G) * L * 4);
  s.orng = smem_take(o, uint32_t(G) * rows * 4);
  s.ofin = smem_take(o, uint32_t(G) * rows * 4);
  s.qs = smem_take(o, 128 * 4);
  s.red = smem_take(o, 8 * 4 * 4);
  s.total = o;
  return s;
}

// Largest dynamic shared memory one CTA may use on sm_100 (227 KiB).
constexpr uint32_t MAX_DYN_SMEM = 227u * 1024u;

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) acts on the current device
// only, so the size a kernel has been allowed is cached per device ordinal;
// one cache object per kernel instantiation.  Raising is serialised by a
// mutex (the attribute is only ever raised, never lowered); the fast path is
// one acquire load.
struct DynSmemCache {
  static constexpr int kMaxDevices = 64;
  std::atomic<int> allowed[kMaxDevices] = {};
  std::mutex mu;
};

inline cudaError_t ensure_dyn_smem(const void* func, int bytes, DynSmemCache& c) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const bool cached = dev >= 0 && dev < DynSmemCache::kMaxDevices;
  if (cached && c.allowed[dev].load(std::memory_order_acquire) >= bytes) return cudaSuccess;
  std::lock_guard<std::mutex> lock(c.mu);
  if (cached && c.allowed[dev].load(std::memory_order_relaxed) >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  if (cached) c.allowed[dev].store(bytes, std::memory_order_release);
  return cudaSuccess;
}

cudaError_t launch_step(const StepParams& p, bool fused, bool f32ck, int group, cudaStream_t stream);
// B200 path for E4M3 or INT8 checkpoints and rings of L <= 16 (one CTA per value head)
cudaError_t launch_step2(const StepParams& p, bool fused, cudaStream_t stream);
constexpr int STEP2_MAX_L = 16;
// persistent warp-specialised path for the heads that do not flush (gdnr_step5.cu)
bool step5_eligible(const StepParams& p, bool fused, bool f32ck);
cudaError_t launch_step5(const StepParams& p, bool fused, bool pdl, cudaStream_t stream);

// ---------------------------------------------------------------- codec kernel
struct CodecParams {
  float* state;
  int64_t st_sb, st_sh;  // rows of K contiguous, row stride K
  uint8_t* payload;
  int64_t pl_sb, pl_sh;
  void* sc;
  int64_t sc_sb, sc_sh, sc_sv;
  int32_t sc_dt;
  int32_t B, HV;
  int32_t quant_rounded;
  uint32_t* sat;
  int32_t int8;  // payload: int8 codes with amax/127 scales ("vblock_int8"), else e4m3
};

cudaError_t launch_quantize(const CodecParams& p, cudaStream_t stream);
cudaError_t launch_dequantize(const CodecParams& p, cudaStream_t stream);

// ---------------------------------------------------------------- host helpers
int set_error(int code, const char* fmt, ...);
uint32_t* default_error_word();
// The split replay through the persistent step kernel (replay without flush that
// also writes T and c); *done = 0 when the layout is not one it takes.
int replay_split_step5(const gdnr_tensor& ck, const gdnr_tensor& sc, const gdnr_tensor& q, const gdnr_tensor& kr,
                       const gdnr_tensor& vr, const gdnr_tensor& gr, const gdnr_tensor& br, const gdnr_tensor& vl,
                       const gdnr_tensor& out, float* tq, const int64_t* tq_s, float* co, const int64_t* co_s,
                       uint32_t* err, cudaStream_t st, int* done);

inline bool present(const gdnr_tensor& t) { return t.ndim > 0 && t.data != nullptr; }

int dtype_size(int dt);

// Checks rank, dtype membership and (when want[i] >= 0) exact extents.
int check_tensor(const gdnr_tensor& t, const char* name, int ndim, const int* dtypes, int ndtypes,
                 const int64_t* want);

int check_inner_contiguous(const gdnr_tensor& t, const char* name);
int check_aligned16(const gdnr_tensor& t, const char* name, int first_dim_to_check);
bool overlaps(const gdnr_tensor& a, const gdnr_tensor& b);
int cuda_status(cudaError_t e, const char* what);

}  // namespace gdnr
