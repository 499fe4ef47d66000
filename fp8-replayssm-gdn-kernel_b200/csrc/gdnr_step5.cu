// Persistent warp-specialised GDN decode step (sm_100a) for E4M3 checkpoints
// with rings of 4 <= L <= 16: every head whose ring is not full.  INT8
// checkpoints (template flag I8) run the variant without the flush path: the
// team readout on the integer tensor path against T in int8 limbs.
//
// Work unit: the (up to) two value heads of one key head that share the key
// ring and the query (G = HV/H value heads per key head; a unit holds
// hpu = min(G, 2) of them).  One CTA per SM owns units blockIdx.x,
// blockIdx.x + gridDim.x, ...  Three warp roles run concurrently:
//
//  * producer (warp 0): streams each unit's checkpoint tiles (ONE tensor-map
//    TMA request of 128 x 128 x hpu bytes, 128-byte swizzle = the layout the
//    tensor-core fragments read conflict-free) and value-ring rows (boxes of
//    8 slots) through S5_STAGES shared-memory stages, in unit order.
//  * chain warps (S5_NCW): one warp per unit runs everything that does not
//    touch the checkpoint -- prep of this token (q/k L2 norm, gates, ring
//    append; kern.py:453-576), the Gram matrix of the key ring on tensor
//    cores, the triangular solve for the replay coefficients c and the
//    transformed query T of the backward chain (kern.py:121-176 in Gram
//    form) -- for both heads of the unit at once.  A unit's chain needs only
//    its key ring (4 KB, loaded by the chain warp's own TMA), so all chains of
//    the SM run while the checkpoints are still streaming in.
//  * readout (S5_NRW warps): consumes the stages in order; in the variant
//    without the flush path two groups of four warps take alternate units, each
//    warp two 32-row vblocks of its unit, on tensor cores: S_fp8 . T as an e4m3
//    MMA against T split into five e4m3 terms, V^T c as a bf16 MMA into the
//    spare accumulator columns, plus this token's value row (rank one).
//
// Units whose ring is full (flush) take the same stages: their chain warp
// hands the decayed Gram matrix and gates to the flush-task workers (the
// readout warps; when every unit of the CTA flushes, also chain warps 1..4),
// which rebuild the state in WY form on tensor cores one vblock of 32 rows at a time
// (E = S0 [K; q]^T, the u recurrence, S_L = a S0 + W K), re-quantise it into
// the stage (vblock32 scales, ref.py:40-106) and write both heads back with one
// tensor-map store.  With GDNR_FLUSH_NONE they are skipped and reported.
#include <cuda.h>

#include "gdnr_device.cuh"
#include "gdnr_head.cuh"
#include "gdnr_internal.h"

namespace gdnr {

constexpr int S5_NS = 4;    // checkpoint / value-ring stages
constexpr int S5_PF = 4;    // units beyond the stages kept prefetched into L2
constexpr int S5_NCW = 7;   // chain warps
constexpr int S5_NRW = 8;   // readout warps
constexpr int S5_TEAM = S5_NRW / S5_NS;  // readout warps per stage
constexpr int S5_THREADS = 32 * (1 + S5_NCW + S5_NRW);
constexpr int S5_GSTR = 20;  // Gram scratch row (floats): 16 key columns + 3 query terms + pad
// Readout structure.  The flush-capable variant with two-head units ("TC")
// shares a flush unit's eight vblock tasks among all readout warps (task w: head
// w / 4, rows 32 (w % 4) ..; their rebuilt state parks in tensor memory) and
// reads the other units out with groups of four warps that claim them in order.
// The flush-capable variant with one-head units uses a team of S5_TEAM warps per
// stage, four units at a time.
template <int HPU, bool FLUSH>
__host__ __device__ constexpr bool s5_tc() {
  return HPU == 2 && FLUSH;
}
// In that variant the entries that do not flush are read out either on the
// tensor cores through tensor memory (S5_VBF 0) or, with S5_VBF, by the
// register-fragment vblock readout of the variant without the flush path (four
// warps per entry, two 32-row vblocks each); the flush entries, the claims and
// the tensor-memory stash of the flush tasks are the same in both.
#ifndef S5_VBF
#define S5_VBF 1
#endif
template <int HPU, bool FLUSH>
__host__ __device__ constexpr bool s5_tcr() {
  return s5_tc<HPU, FLUSH>() && !S5_VBF;
}
// Readout of the variant without the flush path ("vblock readout"): every
// readout warp takes one 32-row vblock of a unit (warp w: head w / 4, rows
// 32 (w % 4) ..), so that a unit is read out by 4 x hpu warps at once (one-head
// units: two groups of 4 warps alternate over the units) and stages free up
// one unit at a time.  The team readout (S5_TEAM warps per stage, four units
// at a time) stays for the flush-capable variant with one-head units.
template <bool FLUSH>
__host__ __device__ constexpr bool s5_vb() {
  return !FLUSH;
}
#ifndef S5_VB_VPW
#define S5_VB_VPW 2
#endif
// vblock readout: vblocks per warp and unit (two-head units: S5_VB_VPW, so that
// 8 / S5_VB_VPW warps read a unit out and S5_VB_VPW units are in flight; one-head
// units: 1, four warps per unit, two units in flight)
template <int HPU>
__host__ __device__ constexpr int s5_vpw() {
  return HPU == 2 ? S5_VB_VPW : 1;
}
template <int HPU, bool FLUSH>
__host__ __device__ constexpr int s5_rpu() {  // readout warps per unit
  return s5_tc<HPU, FLUSH>() ? S5_NRW : (s5_vb<FLUSH>() ? 4 * HPU / s5_vpw<HPU>() : S5_TEAM);
}
// Tensor memory of the tensor-memory readout: columns 0..127 the readout's
// accumulators (stages x heads x 16); from S5_TM_STASH, 128 columns per readout
// warp of a lane quarter (two per quarter), then 128 for the chain warp of the
// quarter among chain warps 1..4, where a flush task parks its rebuilt state
// between the amax and the re-quantisation pass.
constexpr uint32_t S5_TM_STASH = 128;
constexpr uint32_t S5_TMEM_COLS = 512;  // power of two >= S5_TM_STASH + 3 x 128
static_assert(S5_TMEM_COLS >= S5_TM_STASH + 3 * 128, "tensor memory: stash of two readout warps and a chain warp per quarter");
// A chain warp's result area: T terms of a non-flush unit (2 x 8 x T8STR), or the
// flush data of a flush unit -- q split as f16 x 256 [2][128], then per head
// (float offsets) a_t [16] at S5_FA, beta_t [16] at S5_FB, 1 / (operand scale) at
// S5_FINV, the head's four vblock scales at S5_FSC, and from S5_FN the f16 operand
// rows [T diag(d) | z]^T: hi [17][16], then lo [17][16] (the chain's N [16][16]
// f32 scratch before that).
constexpr uint32_t S5_FQ16 = 0, S5_FHEAD = 512;
constexpr int S5_FA = 0, S5_FB = 16, S5_FINV = 32, S5_FSC = 36, S5_FN = 40, S5_TB_LO = 17 * 16;
constexpr uint32_t S5_FHEAD_BYTES = S5_FN * 4 + 1088;  // max(N: 1024, operand rows: 2 x 17 x 16 x 2)
constexpr uint32_t S5_T8_BYTES = S5_FHEAD + 2 * S5_FHEAD_BYTES;
static_assert(S5_T8_BYTES >= 2 * 8 * T8STR, "flush data overlay smaller than the T terms");
constexpr float S5_LOG2E = 1.4426950408889634f;

struct S5Geo {
  int hpu;  // value heads per unit (1 or 2)
  int upk;  // units per key head (G / hpu)
  int rb;   // ring slots per TMA request (8, or 4 when L < 8)
};

__host__ __device__ inline S5Geo s5_geo(int H, int HV, int L, bool one_head = false) {
  S5Geo g;
  const int G = HV / H;
  g.hpu = G >= 2 && !one_head ? 2 : 1;
  g.upk = G / g.hpu;
  g.rb = L >= 8 ? 8 : 4;
  return g;
}

// Shared memory.  Ring regions hold 16 slots of 256 bytes (the fragment loads
// always cover 16 slots; slots >= n are masked).
//   [barriers | table] [stages: ck (hpu x 16 KB) | vr (hpu x 4 KB)] x S5_NS
//   [kbuf: key ring (4 KB)] x S5_NCW
//   [res: t8 x hpu | cb x hpu | misc x hpu | vnew x hpu] x S5_NCW  (the t8 area
//        doubles as the chain's q-split / Gram scratch before T is written)
//   [ost: 128 floats] x S5_NRW
struct S5Layout {
  uint32_t full, empty, kfull, cbar, rbar, abort, vword, vdone, mmab, tmem, table, tdone, gwords;
  uint32_t stage0, stage_bytes, ck, vr;
  uint32_t kbuf0;
  uint32_t res0, res_bytes, t8, cb, cf, misc, vnew;
  uint32_t qb, gram;  // chain scratch inside res (aliases t8)
  uint32_t ost0, zb;
  uint32_t gbuf0;  // variant without the flush path: per chain warp, its unit's gate rings (g, beta; 256 B each)
  uint32_t total;
};

__host__ __device__ inline S5Layout s5_layout(const S5Geo& g, int max_units, bool flush) {
  S5Layout s;
  uint32_t o = 0;
  s.full = smem_take(o, S5_NS * 8);
  s.empty = smem_take(o, S5_NS * 8);
  s.kfull = smem_take(o, S5_NCW * 8);
  s.cbar = smem_take(o, S5_NCW * 8);
  s.rbar = smem_take(o, S5_NCW * 8);
  s.abort = smem_take(o, 16);
  s.vword = smem_take(o, S5_NS * 4);
  s.vdone = smem_take(o, S5_NS * 4);
  s.mmab = smem_take(o, S5_NS * 8);
  s.tmem = smem_take(o, 16);
  s.table = smem_take(o, uint32_t(max_units) * 4u);
  s.tdone = smem_take(o, uint32_t(max_units) * 4u);
  // readout groups (tensor-memory variant): [0] flush entries, [1] claim counter,
  // [2..7] per group a double-buffered claimed rank, [8..15] the claimable entries
  s.gwords = smem_take(o, 16u * 4u);
  o = (o + 1023u) & ~1023u;
  s.stage0 = o;
  s.ck = 0;
  s.vr = uint32_t(g.hpu) * 16384u;
  s.stage_bytes = s.vr + uint32_t(g.hpu) * 4096u;
  o += S5_NS * s.stage_bytes;
  s.kbuf0 = o;
  o += S5_NCW * 4096u;
  uint32_t r = 0;
  // t8: the T terms (tensor-memory readout: the tensor-core B operand, 1 KB per
  // head in K-major 8 x 16-byte core matrices; team readout: rows of T8STR), the
  // chain's q-split / Gram scratch before that, or a flush unit's data
  s.t8 = smem_take(r, flush ? S5_T8_BYTES : 2u * 8u * uint32_t(T8STR));
  s.cb = smem_take(r, 2u * 3u * 16u * 2u);
  s.cf = smem_take(r, 2u * 16u * 4u);
  s.misc = smem_take(r, 2u * 16u);
  s.vnew = smem_take(r, 2u * 128u * 2u);
  s.res_bytes = r;
  r = 0;
  s.qb = smem_take(r, 3u * 128u * 2u);
  s.gram = smem_take(r, 16u * S5_GSTR * 4u);  // qb + gram fit in the t8 area (2048 bytes)
  s.res0 = o;
  o += S5_NCW * s.res_bytes;
  s.ost0 = o;
  o += (S5_NRW + (flush ? 4u : 0u)) * 512u;  // flush-capable: also chain warps 1..4 (flush tasks)
  s.zb = smem_take(o, 1024u);  // zeros: rows 8..15 of every T operand (N = 16)
  s.gbuf0 = smem_take(o, flush ? 0u : S5_NCW * 512u);
  s.total = o;
  return s;
}

// ---------------------------------------------------------------- device helpers
__device__ __forceinline__ void s5_ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ void s5_ldsm_x4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ void s5_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void s5_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Relaxed arrive / add, for releases that only end reads whose values have
// already been consumed (nothing to order behind them).
// Arrivals counting `n` (a readout group of 4 warps owes the 8 arrivals of a unit
// that all 8 readout warps would otherwise make).
__device__ __forceinline__ void s5_arrive_n(uint64_t* bar, uint32_t n) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(n) : "memory");
}

__device__ __forceinline__ void s5_arrive_relaxed_n(uint64_t* bar, uint32_t n) {
  asm volatile("mbarrier.arrive.relaxed.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(n) : "memory");
}

__device__ __forceinline__ void s5_arrive_relaxed(uint64_t* bar) {
  asm volatile("mbarrier.arrive.relaxed.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void s5_add_relaxed(uint32_t* p, uint32_t v) {
  asm volatile("red.relaxed.cta.shared::cta.add.u32 [%0], %1;" ::"r"(smem_addr(p)), "r"(v) : "memory");
}

__device__ __forceinline__ void s5_tma4(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                        uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
      "%5}], [%6];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void s5_tma3(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(bar))
      : "memory");
}

// Heads per 16-byte row of a gate-ring tensor-map box (the box starts at a
// multiple of it, the TMA alignment rule for the innermost coordinate)
__device__ __forceinline__ int s5_gate_hb(int dtype) { return dtype == GDNR_F32 ? 4 : 8; }

__device__ __forceinline__ void s5_tma5(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3, int c4,
                                        uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, "
      "%6}], [%7];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(smem_addr(bar))
      : "memory");
}

// Non-blocking test of an mbarrier phase (try_wait may suspend the thread for a
// while before it reports an incomplete phase).
__device__ __forceinline__ bool s5_test_wait(const uint64_t* bar, uint32_t parity) {
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

// L2 prefetch of a tensor-map box (no shared memory, no completion signal).
__device__ __forceinline__ void s5_prefetch4(const CUtensorMap* map, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}

__device__ __forceinline__ void s5_prefetch5(const CUtensorMap* map, int c0, int c1, int c2, int c3, int c4) {
  asm volatile("cp.async.bulk.prefetch.tensor.5d.L2.global.tile [%0, {%1, %2, %3, %4, %5}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
               : "memory");
}

// ---------------------------------------------------------------- tensor memory (tcgen05)
// Shared-memory matrix descriptors of tcgen05.mma (version 1):
//   K-major with 128-byte swizzle -- the layout the checkpoint tiles land in (8-row
//   atoms of 1 KB; leading offset unused (1), stride 1024 bytes), advanced along K
//   by adding the byte offset to the start address;
//   K-major 8 x 16-byte core matrices without swizzle -- lbo: next 16-byte K chunk,
//   sbo: next group of 8 rows.
__device__ __forceinline__ uint64_t s5_desc_sw128(uint32_t addr) {
  return uint64_t((addr >> 4) & 0x3FFFu) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) | (uint64_t(1) << 46) |
         (uint64_t(2) << 61);
}

__device__ __forceinline__ uint64_t s5_desc_cm(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return uint64_t((addr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46);
}

// Instruction descriptor: f32 accumulator, e4m3 A and B, both K-major, N = 16, M = 128.
constexpr uint32_t S5_IDESC_E4M3_M128_N16 = (1u << 4) | ((16u >> 3) << 17) | ((128u >> 4) << 24);

__device__ __forceinline__ void s5_umma_e4m3(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
  const uint32_t z = 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(S5_IDESC_E4M3_M128_N16), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
      : "memory");
}

// arrives on `bar` once every tcgen05 operation this thread issued so far has completed
__device__ __forceinline__ void s5_umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

// 16 consecutive 32-bit columns of this thread's tensor-memory lane (32x32b shape)
__device__ __forceinline__ void s5_tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 consecutive 32-bit columns of this thread's tensor-memory lane (32x32b shape)
__device__ __forceinline__ void s5_tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 16 consecutive 32-bit columns of this thread's lane, stored (32x32b shape)
__device__ __forceinline__ void s5_tmem_st16(uint32_t taddr, const float* x) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "f"(x[0]), "f"(x[1]), "f"(x[2]), "f"(x[3]), "f"(x[4]), "f"(x[5]), "f"(x[6]), "f"(x[7]), "f"(x[8]), "f"(x[9]),
      "f"(x[10]), "f"(x[11]), "f"(x[12]), "f"(x[13]), "f"(x[14]), "f"(x[15])
      : "memory");
}

__device__ __forceinline__ void s5_tc_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void s5_tc_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Bounded mbarrier wait that also gives up once another warp has recorded a
// failure in *abort (then every later wait returns at once).
// (The waiting part is one out-of-line copy: every inlined copy of it would
// cost instruction-cache space next to the hot code.)
static __device__ __noinline__ bool s5_wait_slow(uint64_t* bar, uint32_t parity, uint32_t* err, volatile int* abort) {
  const uint32_t a = smem_addr(bar);
  if (*abort) return false;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1; it < WAIT_LIMIT_ITERS; ++it) {
    if (mbar_try_wait(a, parity)) return true;
    if ((it & 63u) == 0) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) break;
    }
  }
  *abort = 1;
  atomicOr(err, GDNR_DEVERR_WAIT_TIMEOUT);
  return false;
}

// Abort path only: a bounded wait for an mbarrier phase that ignores *abort, so
// that copies and tensor-core work this CTA has already issued are finished
// before it releases its tensor memory or exits.
static __device__ __noinline__ bool s5_drain_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_addr(bar);
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1; it < WAIT_LIMIT_ITERS; ++it) {
    if (mbar_try_wait(a, parity)) return true;
    if ((it & 63u) == 0 && globaltimer_ns() - t0 > WAIT_LIMIT_NS) return false;
  }
  return false;
}

// Abort path only: the stage loads of the last min(issued, S5_NS) units, the
// only ones that can still be in flight (a stage is reloaded only after its
// previous load was waited for, and no load is issued once *abort is set).
static __device__ __noinline__ void s5_drain_stages(uint64_t* full, int issued) {
  for (int u = issued > S5_NS ? issued - S5_NS : 0; u < issued; ++u)
    s5_drain_wait(&full[u % S5_NS], uint32_t((u / S5_NS) & 1));
}

__device__ __forceinline__ bool s5_wait(uint64_t* bar, uint32_t parity, uint32_t* err, volatile int* abort) {
  if (s5_test_wait(bar, parity)) return true;
  return s5_wait_slow(bar, parity, err, abort);
}

__device__ __forceinline__ bool s5_warp_wait(uint64_t* bar, uint32_t parity, uint32_t* err, volatile int* abort,
                                             int lane) {
  int ok = 1;
  if (lane == 0) ok = s5_wait(bar, parity, err, abort) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// Byte offset of element (slot t, column col) in a ring region written by the
// 128-byte-swizzled ring boxes: slot t is two 128-byte lines R = 2t + col/64,
// and 16-byte chunk c of line R sits at chunk c ^ (R & 7).
__device__ __forceinline__ uint32_t s5_ring_off(int t, int col) {
  const int R = 2 * t + (col >> 6);
  const int c = (col & 63) >> 3;
  return uint32_t(R) * 128u + (uint32_t(c ^ (R & 7)) << 4) + uint32_t(col & 7) * 2u;
}

// Four consecutive elements of a bf16 or f32 row, kept raw until used.  Both
// widths load into the same registers under a predicate, so nothing waits for
// the data before it is unpacked.
__device__ __forceinline__ uint4 s5_load4(const void* base, int64_t idx, bool bf16) {
  uint4 r;
  const char* pb = static_cast<const char*>(base) + idx * (bf16 ? 2 : 4);
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.u32 p, %4, 0;\n\t"
      "@p ld.global.v2.u32 {%0, %1}, [%5];\n\t"
      "@!p ld.global.v4.u32 {%0, %1, %2, %3}, [%5];\n\t}"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "r"(bf16 ? 1u : 0u), "l"(pb));
  return r;
}

__device__ __forceinline__ void s5_unpack4(uint4 w, bool bf16, float* x) {
  if (bf16) {
    const float2 a = bf16x2_to_f2(w.x), b = bf16x2_to_f2(w.y);
    x[0] = a.x;
    x[1] = a.y;
    x[2] = b.x;
    x[3] = b.y;
  } else {
    x[0] = __uint_as_float(w.x);
    x[1] = __uint_as_float(w.y);
    x[2] = __uint_as_float(w.z);
    x[3] = __uint_as_float(w.w);
  }
}

// Unit descriptor in the table: bits 0-7 slots replayed (this token included),
// 8-15 slots read from memory, bit 16 skip (a bad position, or a flush the
// caller ruled out), bit 17 flush (state rebuild + re-quantisation here).
__device__ __forceinline__ int s5_n(int code) { return code & 0xff; }
__device__ __forceinline__ int s5_nmem(int code) { return (code >> 8) & 0xff; }
__device__ __forceinline__ bool s5_skip(int code) { return (code >> 16) & 1; }
// bit 17: the unit flushes here (rebuild + re-quantisation in this kernel)
__device__ __forceinline__ bool s5_flush(int code) { return (code >> 17) & 1; }
// Table entries also carry, in bits 24-31, the CTA-local index of the unit they
// describe (units bid + index * gridDim.x); entry i is the i-th unit processed.
__device__ __forceinline__ int s5_uidx(int entry) { return int(uint32_t(entry) >> 24); }

// A unit: batch row b, key head h, pair pp of its value heads (first value head
// hv0); s: the row's state slot -- b, or under packed decode state_indices[b],
// with -1 for a null slot (index <= 0, the production op's NULL_BLOCK_ID test,
// fused_recurrent.py:292-297) and -2 for an index >= S (both skipped; their
// output rows are written as zeros).
struct S5Unit {
  int b, h, pp, hv0, s;
};

template <bool SIDX>
__device__ __forceinline__ S5Unit s5_unit(int u, const StepParams& p, int G, const S5Geo& g) {
  S5Unit x;
  const int per_b = p.H * g.upk;
  x.b = u / per_b;
  const int r = u - x.b * per_b;
  x.h = r / g.upk;
  x.pp = r - x.h * g.upk;
  x.hv0 = x.h * G + x.pp * g.hpu;
  x.s = x.b;
  if constexpr (SIDX) {
    const int v = __ldg(p.sidx + int64_t(x.b) * p.si_s);
    x.s = v <= 0 ? -1 : (v >= p.S ? -2 : v);
  }
  return x;
}

__device__ __forceinline__ float s5_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^(14 - e) for m in [2^(e-1), 2^e), clamped to 2^[-124, 124]; 1 for m not
// finite-positive (so that max |x| * scale lies in [2^13, 2^14))
__device__ __forceinline__ float s5_pow2_scale(float m) {
  if (!(m > 0.0f) || !(m <= 3.402823466e38f)) return 1.0f;
  const int e = int((__float_as_uint(m) >> 23) & 0xffu) - 126;
  int k = 14 - e;
  k = k > 124 ? 124 : (k < -124 ? -124 : k);
  return __uint_as_float(uint32_t(k + 127) << 23);
}

// Two heads' T (4 elements per lane each: 4 lane .. 4 lane + 3) -> five e4m3
// terms per head, rows 0..4 of an 8-row operand (rows 5..7 zero):
// T sigma = sum_i term_i 16^-i, max |T sigma| in [128, 256); misc[0] = 1/sigma.
// Tensor-memory readout: head h's operand at t8 + 1024 h as K-major 8 x 16-byte
// core matrices (byte k of row j at 128 (k / 16) + 16 j + k % 16); team readout:
// row j of head h at t8 + T8STR (8 h + j).
template <bool TC>
__device__ __forceinline__ uint32_t s5_t8_off(int h, int j, int lane) {
  if constexpr (TC) return uint32_t(h * 1024 + (lane >> 2) * 128 + j * 16 + (lane & 3) * 4);
  return uint32_t((h * 8 + j) * T8STR + lane * 4);
}

// I8 (int8 checkpoint, team readout only): four int8 limbs per head instead,
// T sigma = sum_j limb_j 128^-j with max |T sigma| in [32, 64) (x - rint(x) is
// exact, so every residual times 128 stays within +-64), rows 4..7 zero.
template <int HPU, bool TC, bool I8 = false>
__device__ __forceinline__ void s5_tsplit(const float (*Tq)[4], uint8_t* t8, float* misc, int lane) {
  float m[HPU];
#pragma unroll
  for (int h = 0; h < HPU; ++h)
    m[h] = fmaxf(fmaxf(fabsf(Tq[h][0]), fabsf(Tq[h][1])), fmaxf(fabsf(Tq[h][2]), fabsf(Tq[h][3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int h = 0; h < HPU; ++h) m[h] = fmaxf(m[h], __shfl_xor_sync(0xffffffffu, m[h], o));
  if constexpr (I8) {
    static_assert(!TC, "int8 limbs feed the team readout only");
    float x[HPU][4], sig[HPU];
#pragma unroll
    for (int h = 0; h < HPU; ++h) {
      sig[h] = s5_pow2_scale(m[h]) * (1.0f / 256.0f);
#pragma unroll
      for (int i = 0; i < 4; ++i) x[h][i] = Tq[h][i] * sig[h];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int h = 0; h < HPU; ++h) {
        uint32_t w = 0u;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float r = rintf(x[h][i]);
          w |= (uint32_t(__float2int_rn(r)) & 0xFFu) << (8 * i);
          x[h][i] = (x[h][i] - r) * 128.0f;
        }
        *reinterpret_cast<uint32_t*>(t8 + s5_t8_off<TC>(h, j, lane)) = w;
      }
    }
#pragma unroll
    for (int h = 0; h < HPU; ++h) {
#pragma unroll
      for (int j = 4; j < 8; ++j) *reinterpret_cast<uint32_t*>(t8 + s5_t8_off<TC>(h, j, lane)) = 0u;
      if (lane == 0) misc[h * 4] = 1.0f / sig[h];
    }
    return;
  }
  float x[HPU][4], sig[HPU];
#pragma unroll
  for (int h = 0; h < HPU; ++h) {
    sig[h] = s5_pow2_scale(m[h]) * (1.0f / 64.0f);
#pragma unroll
    for (int i = 0; i < 4; ++i) x[h][i] = Tq[h][i] * sig[h];
  }
#pragma unroll
  for (int j = 0; j < 5; ++j) {
#pragma unroll
    for (int h = 0; h < HPU; ++h) {
      const uint32_t p01 = e4m3x2_sat(x[h][0], x[h][1]);
      const uint32_t p23 = e4m3x2_sat(x[h][2], x[h][3]);
      *reinterpret_cast<uint32_t*>(t8 + s5_t8_off<TC>(h, j, lane)) = p01 | (p23 << 16);
      {
        const uint32_t h01 = e4m3x2_to_f16x2(p01), h23 = e4m3x2_to_f16x2(p23);
        const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&h01));
        const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&h23));
        x[h][0] = (x[h][0] - f01.x) * 16.0f;
        x[h][1] = (x[h][1] - f01.y) * 16.0f;
        x[h][2] = (x[h][2] - f23.x) * 16.0f;
        x[h][3] = (x[h][3] - f23.y) * 16.0f;
      }
    }
  }
#pragma unroll
  for (int h = 0; h < HPU; ++h) {
#pragma unroll
    for (int j = 5; j < 8; ++j) *reinterpret_cast<uint32_t*>(t8 + s5_t8_off<TC>(h, j, lane)) = 0u;
    if (lane == 0) misc[h * 4] = 1.0f / sig[h];
  }
}

// Raw bits of one element of a F32 / BF16 / F16 tensor: the load completes
// in the background; s5_cvt turns it into a float where it is first needed.
__device__ __forceinline__ uint32_t s5_ld_raw(const void* p, int64_t i, int dtype) {
  uint32_t r;
  const bool w32 = dtype == GDNR_F32;
  const char* pb = static_cast<const char*>(p) + i * (w32 ? 4 : 2);
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "@p ld.global.u32 %0, [%2];\n\t"
      "@!p ld.global.u16 %0, [%2];\n\t}"
      : "=r"(r)
      : "r"(w32 ? 1u : 0u), "l"(pb));
  return r;
}

// an I32 or U8 flag, raw
__device__ __forceinline__ int s5_ld_flag(const void* p, int64_t i, int dtype) {
  uint32_t r;
  const bool w32 = dtype == GDNR_I32;
  const char* pb = static_cast<const char*>(p) + i * (w32 ? 4 : 1);
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "@p ld.global.u32 %0, [%2];\n\t"
      "@!p ld.global.u8 %0, [%2];\n\t}"
      : "=r"(r)
      : "r"(w32 ? 1u : 0u), "l"(pb));
  return int(r);
}

__device__ __forceinline__ float s5_cvt(uint32_t raw, int dtype) {
  if (dtype == GDNR_F32) return __uint_as_float(raw);
  if (dtype == GDNR_BF16) return bf16_to_f(uint16_t(raw));
  return __half2float(__ushort_as_half(uint16_t(raw)));
}

// Per-lane raw inputs of one unit for its chain warp (lane 16 e + t: head e,
// ring slot t), issued as soon as the unit is known and consumed only inside
// the chain, so that no warp stalls on them early.
struct S5In {
  uint4 q, k;         // query / key rows, 4 elements per lane
  uint4 v0, v1;       // this token's value rows of heads 0 and 1 (fused)
  uint32_t g, beta;   // gates of (head e, slot min(t, L-1))
  uint32_t a, bb;     // this token's gate inputs of head e (fused)
  float alog, dtb;
  int pos, flag;      // ring position (fused) / valid_len and flush (replay)
  uint32_t scr;       // vblock scale (head e, vblock t % 4), flush-capable variant
};

template <bool FUSED, int HPU, bool FLUSH>
__device__ __forceinline__ S5In s5_fetch(const StepParams& p, const S5Unit& U, int lane) {
  S5In in;
  const int e = lane >> 4, t = lane & 15;
  const int hv = U.hv0 + (e < HPU ? e : 0);
  const int ts = t < p.L ? t : p.L - 1;
  // a null or bad slot (U.s < 0, packed decode) reads slot 0's gates and scales:
  // the unit is skipped, the values are never used, and no load leaves the tensors
  const int64_t sl = U.s < 0 ? 0 : U.s;
  if (!FLUSH && p.gtma) {  // in shared memory (gate-ring TMA with the key ring)
    in.g = in.beta = 0u;
  } else {
    in.g = s5_ld_raw(p.gr, sl * p.gr_sb + int64_t(ts) * p.gr_st + int64_t(hv) * p.gr_sh, p.gr_dt);
    in.beta = s5_ld_raw(p.br, sl * p.br_sb + int64_t(ts) * p.br_st + int64_t(hv) * p.br_sh, p.br_dt);
  }
  in.scr = FLUSH ? s5_ld_raw(p.sc, sl * p.sc_sb + int64_t(hv) * p.sc_sh + int64_t(t & 3) * p.sc_sv, p.sc_dt)
                 : 0u;
  if constexpr (FUSED) {
    const bool bf = p.mx_dt == GDNR_BF16;
    const int64_t row = int64_t(U.b) * p.mx_sb;
    in.q = s5_load4(p.mixed, row + int64_t(U.h) * KD + 4 * lane, bf);
    in.k = s5_load4(p.mixed, row + int64_t(p.H + U.h) * KD + 4 * lane, bf);
    const int64_t vrow = row + 2 * int64_t(p.H) * KD + int64_t(U.hv0) * VD + 4 * lane;
    in.v0 = s5_load4(p.mixed, vrow, bf);
    in.v1 = s5_load4(p.mixed, vrow + (HPU == 2 ? VD : 0), bf);
    in.a = s5_ld_raw(p.a, int64_t(U.b) * p.a_sb + int64_t(hv) * p.a_sh, p.a_dt);
    in.bb = s5_ld_raw(p.bb, int64_t(U.b) * p.b_sb + int64_t(hv) * p.b_sh, p.b_dt);
    in.alog = p.a_log[int64_t(hv) * p.al_s];
    in.dtb = p.dt_bias[int64_t(hv) * p.db_s];
    in.pos = U.s >= 0 ? p.pos[int64_t(U.s) * p.pos_s] : INT_MIN;  // null / bad slot: skipped
    in.flag = 0;
  } else {
    in.q = s5_load4(p.q, int64_t(U.b) * p.q_sb + int64_t(U.h) * p.q_sh + 4 * lane, p.q_dt == GDNR_BF16);
    in.k = in.v0 = in.v1 = make_uint4(0u, 0u, 0u, 0u);
    in.a = in.bb = 0u;
    in.alog = in.dtb = 0.0f;
    in.pos = p.valid_len[int64_t(U.b) * p.vl_s];
    in.flag = p.flush ? s5_ld_flag(p.flush, int64_t(U.b) * p.fl_s, p.fl_dt) : 0;
  }
  return in;
}

// Unit descriptor (see s5_n / s5_nmem / s5_skip) from its raw position inputs.
// here: flush units are rebuilt in this kernel (bit 17); otherwise they are
// skipped (bit 16) -- the caller promised none (GDNR_FLUSH_NONE).
template <bool FUSED>
__device__ __forceinline__ int s5_code(int raw, int flag, int L, bool here) {
  const int fl = here ? (1 << 17) : (1 << 16);
  if constexpr (FUSED) {
    if (raw < 0 || raw >= L) return 1 << 16;
    return (raw + 1) | (raw << 8) | (raw == L - 1 ? fl : 0);
  } else {
    const int v = raw < 0 ? 0 : (raw > L ? L : raw);
    return v | (v << 8) | (flag != 0 ? fl : 0);
  }
}

// This token's ring append and query output (fused), written to HBM after
// the chain has handed its results to the readout.
struct S5Append {
  uint2 kw;        // normalised key (bf16), 4 elements per lane
  uint2 vw[2];     // value rows of heads 0 and 1 (bf16)
  float g, beta;   // gates of (head lane/16, slot pos) on lane pos
  float qv[4];     // normalised query
};

template <bool FUSED, int HPU>
__device__ __forceinline__ void s5_append(const StepParams& p, const S5Unit& U, int code, const S5Append& a,
                                          int lane) {
  if constexpr (FUSED) {
    const int pos = s5_nmem(code);
    const int e = lane >> 4, t = lane & 15;
    const bool owner = U.pp == 0;
    if (owner) {
      *reinterpret_cast<uint2*>(p.kr + int64_t(U.s) * p.kr_sb + int64_t(pos) * p.kr_st + int64_t(U.h) * p.kr_sh +
                                4 * lane) = a.kw;
      if (p.q_out) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          store_scalar(p.q_out, int64_t(U.b) * p.qo_sb + int64_t(U.h) * p.qo_sh + 4 * lane + i, p.qo_dt, a.qv[i]);
      }
    }
#pragma unroll
    for (int h = 0; h < HPU; ++h)
      *reinterpret_cast<uint2*>(p.vr + int64_t(U.s) * p.vr_sb + int64_t(pos) * p.vr_st +
                                int64_t(U.hv0 + h) * p.vr_sh + 4 * lane) = a.vw[h];
    if (t == pos && e < HPU) {
      const int hv = U.hv0 + e;
      store_scalar(p.gr, int64_t(U.s) * p.gr_sb + int64_t(pos) * p.gr_st + int64_t(hv) * p.gr_sh, p.gr_dt, a.g);
      store_scalar(p.br, int64_t(U.s) * p.br_sb + int64_t(pos) * p.br_st + int64_t(hv) * p.br_sh, p.br_dt, a.beta);
      if (p.pos_out && hv == 0) p.pos_out[int64_t(U.s) * p.po_s] = (pos + 1) % p.L;
    }
  }
}

// Triangular solve and transformed query of both heads (lane 16 e + t), with
// NSTEP = 8 or 16 ring slots (slots >= n carry zero gates and keys, so the
// steps run unconditionally).  em[j] = M[t][j] for the lane's row t.
__device__ __forceinline__ void s5_solve(const float* em, float bsel, float& acc, float& cval, int t) {
#pragma unroll
  for (int j = 15; j >= 0; --j) {
    const float cj = __shfl_sync(0xffffffffu, bsel * acc, j, 16);
    if (t == j) cval = cj;
    if (t < j) acc = fmaf(-cj, em[j], acc);
  }
}

template <int HPU>
__device__ __forceinline__ void s5_tloop(const uint8_t* kbuf, float wj, int n, float (*T)[4], int lane) {
  const int half = lane >> 4, c16 = (lane & 15) >> 1;
  const uint8_t* kbase = kbuf + half * 128 + (lane & 1) * 8;
#pragma unroll 1
  for (int j0 = 0; j0 < n; j0 += 4) {
    float w[HPU][4];
    uint2 kw[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int j = j0 + q;
#pragma unroll
      for (int h = 0; h < HPU; ++h) w[h][q] = __shfl_sync(0xffffffffu, wj, 16 * h + (j & 15));
      const int R = 2 * j + half;
      kw[q] = *reinterpret_cast<const uint2*>(kbase + (j & 15) * 256 + ((c16 ^ (R & 7)) << 4));
      if (j >= n) kw[q] = make_uint2(0u, 0u);  // stale slot (its weight is zero too)
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 k01 = bf16x2_to_f2(kw[q].x), k23 = bf16x2_to_f2(kw[q].y);
#pragma unroll
      for (int h = 0; h < HPU; ++h) {
        T[h][0] = fmaf(-w[h][q], k01.x, T[h][0]);
        T[h][1] = fmaf(-w[h][q], k01.y, T[h][1]);
        T[h][2] = fmaf(-w[h][q], k23.x, T[h][2]);
        T[h][3] = fmaf(-w[h][q], k23.y, T[h][3]);
      }
    }
  }
}

// The chain of one unit (one warp, both heads).  kbuf: the unit's key ring
// (swizzled, slots < nmem loaded); res: this warp's result block.
// WT: also write T (fp32, before its split) and the replay coefficients c_t of the
// slots t < n to the split replay's buffers (StepParams::tqo / coo)
template <bool FUSED, int HPU, bool FLUSH, bool I8 = false, bool WT = false>
__device__ __forceinline__ S5Append s5_chain(const StepParams& p, const S5Unit& U, int code, const S5In& in,
                                             uint8_t* kbuf, const uint8_t* gbuf, uint8_t* res, const S5Layout& lay,
                                             int lane) {
  S5Append ap{};
  const int g8 = lane >> 2, t4 = lane & 3;
  const int e = lane >> 4, t = lane & 15;
  const int n = s5_n(code), nmem = s5_nmem(code);
  uint16_t* qb = reinterpret_cast<uint16_t*>(res + lay.t8 + lay.qb);
  float* gram = reinterpret_cast<float*>(res + lay.t8 + lay.gram);
  float* misc = reinterpret_cast<float*>(res + lay.misc);
  uint32_t graw = in.g, braw = in.beta;
  if (!FLUSH && p.gtma) {
    // the gate-ring boxes: slot-major rows of 16 bytes, heads from hv0 rounded down
    const int ts = t < p.L ? t : p.L - 1;
    const int hv = U.hv0 + (e < HPU ? e : 0);
    const int ig = ts * s5_gate_hb(p.gr_dt) + (hv & (s5_gate_hb(p.gr_dt) - 1));
    const int ib = ts * s5_gate_hb(p.br_dt) + (hv & (s5_gate_hb(p.br_dt) - 1));
    graw = p.gr_dt == GDNR_F32 ? reinterpret_cast<const uint32_t*>(gbuf)[ig]
                               : uint32_t(reinterpret_cast<const uint16_t*>(gbuf)[ig]);
    braw = p.br_dt == GDNR_F32 ? reinterpret_cast<const uint32_t*>(gbuf + 256)[ib]
                               : uint32_t(reinterpret_cast<const uint16_t*>(gbuf + 256)[ib]);
  }
  float g_own = s5_cvt(graw, p.gr_dt), beta_own = s5_cvt(braw, p.br_dt);  // gates of (head e, slot t)
  float qv[4];
  if constexpr (FUSED) {
    const int pos = nmem;
    const bool bf = p.mx_dt == GDNR_BF16;
    // this token's gates for head e (every lane; slot pos keeps them)
    {
      const float xg = s5_cvt(in.a, p.a_dt) + in.dtb;
      const float sp = (xg <= SOFTPLUS_THRESHOLD) ? logf(1.0f + expf(xg)) : xg;
      const float gn = round_to(-expf(in.alog) * sp, p.gr_dt);
      const float bn = round_to(1.0f / (1.0f + expf(-s5_cvt(in.bb, p.b_dt))), p.br_dt);
      if (t == pos) {
        g_own = gn;
        beta_own = bn;
      }
    }
    float x[4], y[4];
    s5_unpack4(in.q, bf, x);
    s5_unpack4(in.k, bf, y);
    // q, k <- x / sqrt(sum x^2 + eps)  (kern.py:514-515): one correctly rounded
    // reciprocal of the norm, then products
    const float qs2 = warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]);
    const float ks2 = warp_sum(y[0] * y[0] + y[1] * y[1] + y[2] * y[2] + y[3] * y[3]);
    const float qi = __frcp_rn(sqrtf(qs2 + L2_EPS)), ki = __frcp_rn(sqrtf(ks2 + L2_EPS));
    const int qdt = p.q_out ? p.qo_dt : GDNR_BF16;
#pragma unroll
    for (int i = 0; i < 4; ++i) qv[i] = round_to(x[i] * qi, qdt);
    const uint2 kw = make_uint2(pack_bf16x2(y[0] * ki, y[1] * ki), pack_bf16x2(y[2] * ki, y[3] * ki));
    *reinterpret_cast<uint2*>(kbuf + s5_ring_off(pos, 4 * lane)) = kw;
    ap.kw = kw;
    // this token's value rows: the readout's rank-one term (HBM ring slot later)
#pragma unroll
    for (int h = 0; h < HPU; ++h) {
      float vv[4];
      s5_unpack4(h == 0 ? in.v0 : in.v1, bf, vv);
      const uint2 vw = make_uint2(pack_bf16x2(vv[0], vv[1]), pack_bf16x2(vv[2], vv[3]));
      *reinterpret_cast<uint2*>(res + lay.vnew + h * 256 + 8 * lane) = vw;
      ap.vw[h] = vw;
    }
    ap.g = g_own;
    ap.beta = beta_own;
#pragma unroll
    for (int i = 0; i < 4; ++i) ap.qv[i] = qv[i];
  } else {
    s5_unpack4(in.q, p.q_dt == GDNR_BF16, qv);
  }
  // q split into three bf16 rows (the Gram's query columns)
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float q = qv[i];
    const uint16_t q0 = f_to_bf16(q);
    const float r1 = q - bf16_to_f(q0);
    const uint16_t q1 = f_to_bf16(r1);
    const uint16_t q2 = f_to_bf16(r1 - bf16_to_f(q1));
    qb[4 * lane + i] = q0;
    qb[128 + 4 * lane + i] = q1;
    qb[256 + 4 * lane + i] = q2;
  }
  __syncwarp();

  // ---- Gram G = K [K; q]^T on tensor cores (slots >= n masked to zero)
  {
    const uint32_t kr_addr = smem_addr(kbuf);
    const uint32_t m_lo = g8 < n ? 0xffffffffu : 0u, m_hi = g8 + 8 < n ? 0xffffffffu : 0u;
    float gacc[3][4];
#pragma unroll
    for (int nt = 0; nt < 3; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) gacc[nt][i] = 0.0f;
    const int mi = lane >> 3;
    const int trow = (lane & 7) + 8 * (mi & 1);
#pragma unroll 2
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t a[4];
      s5_ldsm_x4(kr_addr + s5_ring_off(trow, 16 * ks + 8 * (mi >> 1)), a);
      a[0] &= m_lo;
      a[2] &= m_lo;
      a[1] &= m_hi;
      a[3] &= m_hi;
      mma16816_bf16(gacc[0], a, a[0], a[2]);
      mma16816_bf16(gacc[1], a, a[1], a[3]);
      const int col = 16 * ks + 2 * t4;
      const uint32_t b0 = g8 < 3 ? *reinterpret_cast<const uint32_t*>(qb + g8 * 128 + col) : 0u;
      const uint32_t b1 = g8 < 3 ? *reinterpret_cast<const uint32_t*>(qb + g8 * 128 + col + 8) : 0u;
      mma16816_bf16(gacc[2], a, b0, b1);
    }
#pragma unroll
    for (int nt = 0; nt < 3; ++nt) {
      if (nt < 2 || t4 < 2) {
        const int col = 8 * nt + 2 * t4;
        *reinterpret_cast<float2*>(gram + g8 * S5_GSTR + col) = make_float2(gacc[nt][0], gacc[nt][1]);
        *reinterpret_cast<float2*>(gram + (g8 + 8) * S5_GSTR + col) = make_float2(gacc[nt][2], gacc[nt][3]);
      }
    }
  }
  __syncwarp();
  // lane (e, t) holds row t of G (the same rows in both half-warps)
  float grow[16];
  float kq;
  {
    const float4* gr4 = reinterpret_cast<const float4*>(gram + t * S5_GSTR);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 v = gr4[i];
      grow[4 * i] = v.x;
      grow[4 * i + 1] = v.y;
      grow[4 * i + 2] = v.z;
      grow[4 * i + 3] = v.w;
    }
    const float4 v = gr4[4];
    kq = v.x + v.y + v.z;
  }
  // ---- decays in log2 space per head (16-lane segment), gl_m = g_m log2(e):
  // a_t = 2^(sum_{m<=t} gl_m), and the ratios d_t = 2^(sum_{t<m<n} gl_m) and
  // M[t][j] = 2^(sum_{t<m<=j} gl_m) G[t][j] (t < j) from running sums over (t, j]
  // -- not as differences of two prefix sums, which would carry the rounding of
  // the whole prefix (~|prefix| eps, large under strong decay) into every ratio.
  const float gl = t < n ? g_own * S5_LOG2E : 0.0f;
  float Lg = gl;
#pragma unroll
  for (int o = 1; o < 16; o <<= 1) {
    const float up = __shfl_up_sync(0xffffffffu, Lg, o, 16);
    if (t >= o) Lg += up;
  }
  const float Llast = __shfl_sync(0xffffffffu, Lg, 15, 16);  // slots >= n add nothing
  const float a_own = s5_ex2(Lg);
  float em[16], dsum = 0.0f;
  {
    float run = 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float gj = __shfl_sync(0xffffffffu, gl, j, 16);
      if (j > t) run += gj;
      em[j] = s5_ex2(run) * grow[j];  // used for j > t only
      if (j == n - 1) dsum = run;
    }
  }
  if (FLUSH && s5_flush(code)) {
    // flush unit: hand the rebuild's inputs to the readout team (the T chain
    // is not needed: the flush output comes from the rebuilt state)
    __syncwarp();  // q-split / Gram scratch is dead from here on
    uint8_t* fd = res + lay.t8;
    // q split as f16 x 256 (B operand of E = S0 [K; q]^T)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float hq = __half2float(__float2half_rn(qv[i] * KPOW));
      reinterpret_cast<__half*>(fd + S5_FQ16)[4 * lane + i] = __float2half_rn(hq);
      reinterpret_cast<__half*>(fd + S5_FQ16)[128 + 4 * lane + i] = __float2half_rn(qv[i] * KPOW - hq);
    }
    {
      // per head (16-lane segment e): a_t, beta_t; N[j][m] = M[j][m] beta_m (j < m)
      // with w_j = d_j kq_j on its diagonal; then lane t solves column t of
      // T = (I + N)^-1 and (redundantly) z = T w by back substitution
      float* fh = reinterpret_cast<float*>(fd + S5_FHEAD + (e < HPU ? e : 0) * S5_FHEAD_BYTES);
      float* nm = fh + S5_FN;
      const bool live = t < n, wr = e < HPU;
      const float bt = live ? beta_own : 0.0f;
      const float dt = live ? s5_ex2(dsum) : 0.0f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {  // row t of N
        const float mj = em[j];
        const float bj = __shfl_sync(0xffffffffu, bt, j, 16);
        if (wr) nm[t * 16 + j] = j > t ? (live ? mj * bj : 0.0f) : (j == t ? dt * kq : 0.0f);
      }
      if (wr) {
        fh[S5_FA + t] = live ? a_own : 0.0f;
        fh[S5_FB + t] = bt;
        if (t < 4) fh[S5_FSC + t] = s5_cvt(in.scr, p.sc_dt);
      }
      __syncwarp();
      float tc[16], z[16];
#pragma unroll
      for (int j = 15; j >= 0; --j) {
        float row[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 v = reinterpret_cast<const float4*>(nm + j * 16)[q];
          row[4 * q] = v.x;
          row[4 * q + 1] = v.y;
          row[4 * q + 2] = v.z;
          row[4 * q + 3] = v.w;
        }
        float at = j == t ? 1.0f : 0.0f, az = row[j];
#pragma unroll
        for (int m = j + 1; m < 16; ++m) {
          at = fmaf(-row[m], tc[m], at);
          az = fmaf(-row[m], z[m], az);
        }
        tc[j] = at;
        z[j] = az;
      }
      // B operand of U = R [T diag(d) | z]: row t = column t of T diag(d), row 16 = z,
      // as f16 hi / lo after a power-of-two scale
      float mx = 0.0f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        tc[j] *= dt;
        mx = fmaxf(mx, fmaxf(fabsf(tc[j]), fabsf(z[j])));
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float ts = s5_pow2_scale(mx);
      __syncwarp();  // N is read; the operand rows overwrite it
      __half* tb = reinterpret_cast<__half*>(nm);
      auto put_row = [&](int r, const float* x) {
        uint32_t hw[8], lw[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float x0 = x[2 * c] * ts, x1 = x[2 * c + 1] * ts;
          const float h0 = __half2float(__float2half_rn(x0)), h1 = __half2float(__float2half_rn(x1));
          hw[c] = pack_f16x2(h0, h1);
          lw[c] = pack_f16x2(x0 - h0, x1 - h1);
        }
        uint4* dh = reinterpret_cast<uint4*>(tb + r * 16);
        uint4* dl = reinterpret_cast<uint4*>(tb + S5_TB_LO + r * 16);
        dh[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        dh[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
        dl[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        dl[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
      };
      if (wr) {
        put_row(t, tc);
        if (t == 0) {
          put_row(16, z);
          fh[S5_FINV] = 1.0f / ts;
        }
      }
    }
    __syncwarp();
    // key ring in place to f16 x 256 (slots >= n zero): B operand of E and of W K
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = lane + 32 * i;  // 16-byte chunk; its 128-byte line is c / 8, its slot c / 16
      uint4 w = reinterpret_cast<const uint4*>(kbuf)[c];
      const bool live = (c >> 4) < n;
      uint32_t* wv = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 f = bf16x2_to_f2(wv[h]);
        wv[h] = live ? pack_f16x2(f.x * KPOW, f.y * KPOW) : 0u;
      }
      reinterpret_cast<uint4*>(kbuf)[c] = w;
    }
    return ap;
  }
  const float bsel = t < n ? beta_own : 0.0f;
  float acc = t < n ? s5_ex2(dsum) * kq : 0.0f;
  float cval = 0.0f;
  // ---- triangular solve, j = n-1 .. 0: c_j = beta_j (d_j kq_j - sum_{m>j} c_m M[j][m])
  s5_solve(em, bsel, acc, cval, t);
  // ---- c -> [c_hi; c_mid; c_lo] bf16 over the slots read from memory (ring
  // columns of the readout); this token's own slot is a rank-one term
  constexpr bool TC = s5_tcr<HPU, FLUSH>();
  if (TC && e < HPU) reinterpret_cast<float*>(res + lay.cf)[e * 16 + t] = t < nmem ? cval : 0.0f;
  if (!TC && e < HPU) {
    uint16_t* cb = reinterpret_cast<uint16_t*>(res + lay.cb + e * 96);
    const float cc = t < nmem ? cval : 0.0f;
    const uint16_t chi = f_to_bf16(cc);
    const float r1 = cc - bf16_to_f(chi);
    const uint16_t cmid = f_to_bf16(r1);
    const uint16_t clo = f_to_bf16(r1 - bf16_to_f(cmid));
    cb[t] = chi;
    cb[16 + t] = cmid;
    cb[32 + t] = clo;
  }
  {
    // coefficient of this token's own slot (fused): one writer per head
    const float cp = __shfl_sync(0xffffffffu, cval, (lane & 16) + (nmem & 15));
    if (t == 0 && e < HPU) misc[e * 4 + 1] = FUSED ? cp : 0.0f;
  }
  // ---- T_e = a_{n-1} q - sum_j c_j a_j k_j  (lane: elements 4 lane .. 4 lane + 3)
  const float wj = cval * a_own;  // 0 for slots >= n
  float T[HPU][4];
#pragma unroll
  for (int h = 0; h < HPU; ++h) {
    const float al = s5_ex2(__shfl_sync(0xffffffffu, Llast, 16 * h));
#pragma unroll
    for (int i = 0; i < 4; ++i) T[h][i] = al * qv[i];
  }
  s5_tloop<HPU>(kbuf, wj, n, T, lane);
  if constexpr (WT) {
#pragma unroll
    for (int h = 0; h < HPU; ++h)
#pragma unroll
      for (int i = 0; i < 4; ++i)
        p.tqo[int64_t(U.b) * p.tqo_sb + int64_t(U.hv0 + h) * p.tqo_sh + 4 * lane + i] = T[h][i];
    if (e < HPU && t < n) p.coo[int64_t(U.b) * p.coo_sb + int64_t(U.hv0 + e) * p.coo_sh + int64_t(t) * p.coo_st] = cval;
  }
  __syncwarp();  // q-split / Gram scratch (aliases t8) is dead from here on
  s5_tsplit<HPU, s5_tcr<HPU, FLUSH>(), I8>(T, res + lay.t8, misc, lane);
  return ap;
}

// Readout of MW m-tiles (rows rbase .. rbase + 16 MW - 1) of one head by one
// warp: pre-scale o(row) = (S_fp8 . T) / sigma * scale(row) + V^T c into ost[row].
// Lane sc_base + v of sc holds the scale of vblock v of these rows.
// I8: the tile holds int8 codes and t8 four int8 limbs of T (s5_tsplit): the
// tile product runs on the integer tensor path (exact s32 sums, below 2^24 so
// they convert to f32 exactly) and the ring product into its own f32 accumulator.
// REG: o of row rbase + 32 pr + s5_rd_row(lane) goes to ost[pr] (registers once
// inlined) instead of shared memory.
__device__ __forceinline__ int s5_rd_row(int lane) {
  const int g8 = lane >> 2, t4 = lane & 3;
  return 16 * (t4 & 1) + g8 + 8 * (t4 >> 1);
}
template <int MW, bool I8 = false, bool REG = false>
__device__ __forceinline__ void s5_readout(const uint8_t* ck_s, const uint8_t* vr_s, const uint8_t* t8,
                                           const uint16_t* cb, float inv_sig, float sc, int sc_base, int rbase,
                                           int nmem, float* ost, int lane) {
  const int g8 = lane >> 2, t4 = lane & 3;
  uint32_t bt[4][2];
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    bt[ks][0] = g8 < 5 ? *reinterpret_cast<const uint32_t*>(t8 + g8 * T8STR + 32 * ks + 4 * t4) : 0u;
    bt[ks][1] = g8 < 5 ? *reinterpret_cast<const uint32_t*>(t8 + g8 * T8STR + 32 * ks + 16 + 4 * t4) : 0u;
  }
  const bool rcol = g8 >= 5;
  const uint32_t rb0 = rcol ? *reinterpret_cast<const uint32_t*>(cb + (g8 - 5) * 16 + 2 * t4) : 0u;
  const uint32_t rb1 = rcol ? *reinterpret_cast<const uint32_t*>(cb + (g8 - 5) * 16 + 8 + 2 * t4) : 0u;
  // value-ring slots >= nmem hold stale or unloaded data: mask them in the A fragments
  const int t0 = 2 * t4, t1 = 2 * t4 + 8;
  const uint32_t mk0 = (t0 < nmem ? 0x0000ffffu : 0u) | (t0 + 1 < nmem ? 0xffff0000u : 0u);
  const uint32_t mk1 = (t1 < nmem ? 0x0000ffffu : 0u) | (t1 + 1 < nmem ? 0xffff0000u : 0u);
  const uint32_t ck_addr = smem_addr(ck_s), vr_addr = smem_addr(vr_s);
  const int mi = lane >> 3, r8 = lane & 7;
  // m-tiles in pairs (one vblock of 32 rows per pair)
#pragma unroll(REG ? MW / 2 : (MW == 4 ? 2 : 1))
  for (int pr = 0; pr < MW / 2; ++pr) {
    const int rp = rbase + 32 * pr;
    float acc[2][4];
    int32_t iacc[2][4];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[m][i] = 0.0f;
        iacc[m][i] = 0;
      }
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        uint32_t a[4];
        s5_ldsm_x4(ck_addr + s0_off(rp + 16 * m + r8 + 8 * (mi & 1), 2 * ks + (mi >> 1)), a);
        if constexpr (I8)
          mma16832_s8(iacc[m], a, bt[ks][0], bt[ks][1]);
        else
          mma16832_e4m3(acc[m], a, bt[ks][0], bt[ks][1]);
      }
    }
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      uint32_t a[4];
      s5_ldsm_x4_t(vr_addr + s5_ring_off(r8 + 8 * (mi >> 1), rp + 16 * m + 8 * (mi & 1)), a);
      a[0] &= mk0;
      a[1] &= mk0;
      a[2] &= mk1;
      a[3] &= mk1;
      mma16816_bf16(acc[m], a, rb0, rb1);
    }
    // column weights: t4 = 0 -> terms 0,1; 1 -> terms 2,3; 2 -> term 4, ring; 3 -> ring, ring
    const float wsc = inv_sig * __shfl_sync(0xffffffffu, sc, sc_base + pr);
    float v0, v1, v2, v3;
    if constexpr (I8) {
      // limb weights: t4 = 0 -> limbs 0, 1; 1 -> limbs 2, 3; the ring columns (t4 >= 2) are in acc
      const float w0 = t4 == 0 ? wsc : (t4 == 1 ? wsc * (1.0f / 16384.0f) : 0.0f);
      const float w1 = t4 == 0 ? wsc * (1.0f / 128.0f) : (t4 == 1 ? wsc * (1.0f / 2097152.0f) : 0.0f);
      v0 = fmaf(float(iacc[0][1]), w1, float(iacc[0][0]) * w0) + (acc[0][0] + acc[0][1]);
      v1 = fmaf(float(iacc[0][3]), w1, float(iacc[0][2]) * w0) + (acc[0][2] + acc[0][3]);
      v2 = fmaf(float(iacc[1][1]), w1, float(iacc[1][0]) * w0) + (acc[1][0] + acc[1][1]);
      v3 = fmaf(float(iacc[1][3]), w1, float(iacc[1][2]) * w0) + (acc[1][2] + acc[1][3]);
    } else {
      const float w0 = t4 == 0 ? wsc : (t4 == 1 ? wsc * (1.0f / 256.0f) : (t4 == 2 ? wsc * (1.0f / 65536.0f) : 1.0f));
      const float w1 = t4 == 0 ? wsc * (1.0f / 16.0f) : (t4 == 1 ? wsc * (1.0f / 4096.0f) : 1.0f);
      // v = (m0 row g8, m0 row g8+8, m1 row g8, m1 row g8+8)
      v0 = fmaf(acc[0][1], w1, acc[0][0] * w0);
      v1 = fmaf(acc[0][3], w1, acc[0][2] * w0);
      v2 = fmaf(acc[1][1], w1, acc[1][0] * w0);
      v3 = fmaf(acc[1][3], w1, acc[1][2] * w0);
    }
    // summed over the quad as a transpose-reduce: lane t4 ends with m-tile t4 & 1, row half t4 >> 1
    const bool odd = t4 & 1;
    float x0 = odd ? v2 : v0, x1 = odd ? v3 : v1;
    x0 += __shfl_xor_sync(0xffffffffu, odd ? v0 : v2, 1);
    x1 += __shfl_xor_sync(0xffffffffu, odd ? v1 : v3, 1);
    const bool hi = t4 & 2;
    float r = hi ? x1 : x0;
    r += __shfl_xor_sync(0xffffffffu, hi ? x0 : x1, 2);
    if constexpr (REG)
      ost[pr] = r;
    else
      ost[32 * pr + s5_rd_row(lane)] = r;
  }
}

// ---------------------------------------------------------------- flush (rebuild + re-quantisation)
// One vblock (rows rb .. rb + 31 of a head) of a flush unit, by one warp, in WY form
// (the token loop of ref.py:137-163, kern.py:200-240):
//   E = S0 [K; q]^T                      (f16 MMA: S0 from the e4m3 tile, K and q as f16 x 256)
//   R_t = beta_t (v_t - a_t E_t)         (accumulator layout, slots t < n)
//   [W | y] = R [T diag(d) | z]          (f16 hi / lo MMA; T = (I + N)^-1 and z = T (d kq)
//                                         from the chain warp, so u = R T solves
//                                         u_t = R_t - sum_{j<t} u_j beta_t M[j][t])
//   o = a_{n-1} (S0 q) + y,  S_L = a_{n-1} S0 + W K,
// then the vblock32 re-quantisation (ref.py:40-106) written into the tile in place.
// tile: the head's e4m3 tile (swizzled); vr: its value ring; vnew: this token's
// value row (slot nmem) or null; kf: the unit's key ring as f16 x 256; fq: q split
// [2][128] f16 x 256; fh: the head's flush block.  o(row rb + i) (before K^-1/2) -> ost[i].
// STASH: the tensor memory at `stash` (this warp's lane quarter, 128 columns)
// holds the rebuilt state between the two passes; otherwise the second pass
// rebuilds it again.
template <bool STASH>
__device__ __forceinline__ void s5_flush_vblock(uint8_t* tile, const uint8_t* vr, const uint16_t* vnew,
                                                const uint8_t* kf, const __half* fq, const float* fh, int rb,
                                                int n, int nmem, float sc, int quant_rounded, void* scale_ptr,
                                                int64_t sc_index, int sc_dt, float* ost, uint32_t stash, int lane) {
  const int g8 = lane >> 2, t4 = lane & 3;
  const float* av = fh + S5_FA;
  const float* bv = fh + S5_FB;
  const __half* tb = reinterpret_cast<const __half*>(fh + S5_FN);
  const uint32_t kf_addr = smem_addr(kf), vr_addr = smem_addr(vr);
  const int mi = lane >> 3;
  const float alast = n > 0 ? av[n - 1] : 1.0f;
  const float asc = alast * sc;
  const float esc = sc * INV_KPOW;
  // ---- E = S0 [K; q]^T for both m-tiles (rows rb + 16 mt + g8 (+8))
  float e[2][3][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 3; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) e[mt][nt][i] = 0.0f;
#pragma unroll 2
  for (int ks = 0; ks < 8; ++ks) {
    uint32_t bk[4];
    s5_ldsm_x4(kf_addr + s5_ring_off((lane & 7) + 8 * (mi & 1), 16 * ks + 8 * (mi >> 1)), bk);
    const uint32_t q0 = g8 < 2 ? *reinterpret_cast<const uint32_t*>(fq + g8 * 128 + 16 * ks + 2 * t4) : 0u;
    const uint32_t q1 = g8 < 2 ? *reinterpret_cast<const uint32_t*>(fq + g8 * 128 + 16 * ks + 8 + 2 * t4) : 0u;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      uint32_t a[4];
      s0_afrag_f16(tile, rb + 16 * mt, ks, g8, t4, a);
      mma16816(e[mt][0], a, bk[0], bk[2]);
      mma16816(e[mt][1], a, bk[1], bk[3]);
      mma16816(e[mt][2], a, q0, q1);
    }
  }
  // ---- the operand rows (n-tiles 0, 1: T diag(d); n-tile 2: z in column 0)
  uint32_t bh[3][2], bl[3][2];
#pragma unroll
  for (int nt = 0; nt < 3; ++nt) {
    const int r = 8 * nt + g8;
    const bool ok = r < 17;
    bh[nt][0] = ok ? *reinterpret_cast<const uint32_t*>(tb + r * 16 + 2 * t4) : 0u;
    bh[nt][1] = ok ? *reinterpret_cast<const uint32_t*>(tb + r * 16 + 8 + 2 * t4) : 0u;
    bl[nt][0] = ok ? *reinterpret_cast<const uint32_t*>(tb + S5_TB_LO + r * 16 + 2 * t4) : 0u;
    bl[nt][1] = ok ? *reinterpret_cast<const uint32_t*>(tb + S5_TB_LO + r * 16 + 8 + 2 * t4) : 0u;
  }
  const float tinv = fh[S5_FINV];
  // lane's slots: t = 8 nt + 2 t4 + j (accumulator columns)
  float at[2][2], bt[2][2];
  bool lv[2][2], nw[2][2];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int t = 8 * nt + 2 * t4 + j;
      at[nt][j] = av[t] * esc;
      bt[nt][j] = bv[t];
      lv[nt][j] = t < n;
      nw[nt][j] = vnew != nullptr && t == nmem;
    }
  uint32_t ahi[2][4], alo[2][4];
  float dsc[2];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
    // value-ring A fragment: (row g8 / g8+8, slots 2t4.. / 8+2t4..) as bf16 pairs
    uint32_t va[4];
    s5_ldsm_x4_t(vr_addr + s5_ring_off((lane & 7) + 8 * (mi >> 1), rb + 16 * mt + 8 * (mi & 1)), va);
    const float vn0 = vnew != nullptr ? bf16_to_f(vnew[rb + 16 * mt + g8]) : 0.0f;
    const float vn1 = vnew != nullptr ? bf16_to_f(vnew[rb + 16 * mt + g8 + 8]) : 0.0f;
    float rr[2][4];  // [n-tile][c]: row g8 + 8 (c >> 1), slot 8 nt + 2 t4 + (c & 1)
    float rmax = 0.0f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const float2 v2 = bf16x2_to_f2(va[2 * nt + hf]);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          float v = j ? v2.y : v2.x;
          v = nw[nt][j] ? (hf ? vn1 : vn0) : v;
          const float r = bt[nt][j] * (v - at[nt][j] * e[mt][nt][2 * hf + j]);
          rr[nt][2 * hf + j] = lv[nt][j] ? r : 0.0f;
          rmax = fmaxf(rmax, fabsf(rr[nt][2 * hf + j]));
        }
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, o));
    const float rs = s5_pow2_scale(rmax);
    uint32_t rh[4], rl[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {  // A fragment c: (n-tile c >> 1, row half c & 1)
      const float x0 = rr[c >> 1][2 * (c & 1)] * rs, x1 = rr[c >> 1][2 * (c & 1) + 1] * rs;
      const float h0 = __half2float(__float2half_rn(x0)), h1 = __half2float(__float2half_rn(x1));
      rh[c] = pack_f16x2(h0, h1);
      rl[c] = pack_f16x2(x0 - h0, x1 - h1);
    }
    float u[3][4];
#pragma unroll
    for (int nt = 0; nt < 3; ++nt) {
#pragma unroll
      for (int i = 0; i < 4; ++i) u[nt][i] = 0.0f;
      mma16816(u[nt], rh, bh[nt][0], bh[nt][1]);
      mma16816(u[nt], rh, bl[nt][0], bl[nt][1]);
      mma16816(u[nt], rl, bh[nt][0], bh[nt][1]);
    }
    const float us = tinv / rs;
    // output o = a_{n-1} (S0 q) + y: column 0 of n-tile 2 / E columns q_hi, q_lo (lanes t4 == 0)
    if (t4 == 0) {
#pragma unroll
      for (int hf = 0; hf < 2; ++hf)
        ost[16 * mt + g8 + 8 * hf] =
            fmaf(asc * INV_KPOW, e[mt][2][2 * hf] + e[mt][2][2 * hf + 1], u[2][2 * hf] * us);
    }
    // W (A operand of W K), split hi / lo after a power-of-two scale
    float wmax = 0.0f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        u[nt][i] *= us;
        wmax = fmaxf(wmax, fabsf(u[nt][i]));
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) wmax = fmaxf(wmax, __shfl_xor_sync(0xffffffffu, wmax, o));
    const float wp = s5_pow2_scale(wmax);
    dsc[mt] = INV_KPOW / wp;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float x0 = u[c >> 1][2 * (c & 1)] * wp, x1 = u[c >> 1][2 * (c & 1) + 1] * wp;
      const float h0 = __half2float(__float2half_rn(x0)), h1 = __half2float(__float2half_rn(x1));
      ahi[mt][c] = pack_f16x2(h0, h1);
      alo[mt][c] = pack_f16x2(x0 - h0, x1 - h1);
    }
  }
  // ---- S_L = a_{n-1} sc S0 + W K over columns 16 np .. 16 np + 15: x[i], i =
  // ((h * 2 + mt) * 2 + hf) * 2 + j  <->  row rb + 16 mt + 8 hf + g8, column
  // 16 np + 8 h + 2 t4 + j; its tile byte: row * 128 + 16 (np ^ g8) + 8 h + 2 t4 + j.
  // S0 enters through an e4m3 MMA against an identity slice (exact, and in the
  // accumulator layout): n-tile 2 np + h takes key columns 8 (2 (np & 1) + h) ..
  // of the 32-column slice np / 2, i.e. B[k][c] = 1 for k = 8 (2 (np & 1) + h) + c.
  uint8_t* const trow = tile + (rb + g8) * 128 + 2 * t4;
  const uint32_t tile_addr = smem_addr(tile);
  const uint32_t id0 = ((g8 >> 2) == t4) ? (0x38u << (8 * (g8 & 3))) : 0u;        // e4m3 1.0 at k = g8
  const uint32_t id1 = (((8 + g8) >> 2) == t4) ? (0x38u << (8 * (g8 & 3))) : 0u;  // at k = 8 + g8
  auto sl_cols = [&](int np, float* x) {
    uint32_t bkt[4];  // n-tile 2np: (bkt[0], bkt[2]); 2np + 1: (bkt[1], bkt[3])
    s5_ldsm_x4_t(kf_addr + s5_ring_off((lane & 7) + 8 * (mi >> 1), 16 * np + 8 * (mi & 1)), bkt);
    const bool odd = np & 1;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      uint32_t as[4];  // e4m3 A fragment of rows rb + 16 mt .., key columns 32 (np / 2) ..
      s5_ldsm_x4(tile_addr + s0_off(rb + 16 * mt + (lane & 7) + 8 * (mi & 1), 2 * (np >> 1) + (mi >> 1)), as);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f}, sv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        mma16816(acc, ahi[mt], bkt[h], bkt[2 + h]);
        mma16816(acc, alo[mt], bkt[h], bkt[2 + h]);
        const uint32_t id = h ? id1 : id0;
        mma16832_e4m3(sv, as, odd ? 0u : id, odd ? id : 0u);
#pragma unroll
        for (int c = 0; c < 4; ++c) x[((h * 2 + mt) * 2 + (c >> 1)) * 2 + (c & 1)] = fmaf(acc[c], dsc[mt], asc * sv[c]);
      }
    }
  };
  float amax = 0.0f;
#pragma unroll 1
  for (int np = 0; np < 8; ++np) {
    float x[16];
    sl_cols(np, x);
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmax_nan(amax, fabsf(x[i]));
    if constexpr (STASH) s5_tmem_st16(stash + 16u * uint32_t(np), x);
  }
  if constexpr (STASH) asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
  amax = warp_max_nan(amax);
  const VScale vs = vblock_scale(amax, quant_rounded);
  const float rcp = __fdiv_rn(1.0f, vs.divisor);
  const bool qok = quant_exact_ok(vs.divisor, rcp);
  const uint32_t qkd = quant_exact_kd(vs.divisor);
  __syncwarp();
#pragma unroll 1
  for (int np = 0; np < 8; ++np) {
    float x[16];
    if constexpr (STASH) {
      uint32_t xr[16];
      s5_tmem_ld16(stash + 16u * uint32_t(np), xr);
#pragma unroll
      for (int i = 0; i < 16; ++i) x[i] = __uint_as_float(xr[i]);
    } else {
      sl_cols(np, x);
    }
    uint32_t cq[8];
    quant_pairs_warp<8>(x, cq, vs.divisor, rcp, qkd, qok);
    uint8_t* cp = trow + 16 * (np ^ g8);
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf)
          *reinterpret_cast<uint16_t*>(cp + (16 * mt + 8 * hf) * 128 + 8 * h) =
              static_cast<uint16_t>(cq[(h * 2 + mt) * 2 + hf]);
  }
  __syncwarp();
  if (lane == 0) {
    if (sc_dt == GDNR_F16)
      static_cast<__half*>(scale_ptr)[sc_index] = vs.stored;
    else
      static_cast<float*>(scale_ptr)[sc_index] = __half2float(vs.stored);
  }
}

__device__ __forceinline__ void s5_tma_store4(const CUtensorMap* map, const void* src, int c0, int c1, int c2,
                                              int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_addr(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ uint32_t s5_ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_addr(p)) : "memory");
  return v;
}

__device__ __forceinline__ void s5_st_release(uint32_t* p, uint32_t v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_addr(p)), "r"(v) : "memory");
}

// Abort path only (tensor-memory readout): the scheduler publishes how many
// unit commits it issued when it stops; the commit of the last one arrives
// once every tensor-core operation of the CTA has completed.  Bounded waits
// for both, ignoring *abort, before the tensor memory is released.
static __device__ __noinline__ void s5_drain_mma(uint64_t* mmab, const uint32_t* ncommit) {
  const uint64_t t0 = globaltimer_ns();
  uint32_t n = s5_ld_acquire(ncommit);
  for (uint32_t it = 1; n == 0xffffffffu && it < WAIT_LIMIT_ITERS; ++it) {
    __nanosleep(64);
    n = s5_ld_acquire(ncommit);
    if ((it & 63u) == 0 && globaltimer_ns() - t0 > WAIT_LIMIT_NS) break;
  }
  if (n == 0xffffffffu || n == 0u) return;
  s5_drain_wait(&mmab[(n - 1) % S5_NS], ((n - 1) / S5_NS) & 1u);
}

__device__ __forceinline__ void s5_add_release(uint32_t* p, uint32_t v) {
  asm volatile("red.release.cta.shared::cta.add.u32 [%0], %1;" ::"r"(smem_addr(p)), "r"(v) : "memory");
}

// add with acquire-release semantics; returns the previous value
__device__ __forceinline__ uint32_t s5_add_acq_rel(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], %2;" : "=r"(old) : "r"(smem_addr(p)), "r"(v) : "memory");
  return old;
}

// Bounded wait (by lane 0, broadcast) for a shared counter to reach `target`.
__device__ __forceinline__ bool s5_warp_wait_count(const uint32_t* c, uint32_t target, uint32_t* err,
                                                   volatile int* abort, int lane) {
  int ok = 1;
  if (lane == 0 && s5_ld_acquire(c) < target) {
    ok = 0;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1; it < WAIT_LIMIT_ITERS; ++it) {
      __nanosleep(32);
      if (s5_ld_acquire(c) >= target) {
        ok = 1;
        break;
      }
      if ((it & 63u) == 0) {
        if (*abort) break;
        if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) {
          *abort = 1;
          atomicOr(err, GDNR_DEVERR_WAIT_TIMEOUT);
          break;
        }
      }
    }
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
}

// ---------------------------------------------------------------- flush task pool
// A flush unit's vblocks (4 per head) are tasks that the readout team of the
// unit's stage shares out: the team publishes the unit in the stage's task word
// (unit << 8 | next task) and each warp claims tasks with compare-and-swap until
// none is left, so the work balances between the two warps whatever the
// per-task times.  A claim for another unit never succeeds.
__device__ __forceinline__ int s5_claim(uint32_t* vword, int unit, int ntask, int lane) {
  int t = -1;
  if (lane == 0) {
    uint32_t w = s5_ld_acquire(vword);
    while ((w >> 8) == uint32_t(unit) && int(w & 0xffu) < ntask) {
      const uint32_t prev = atomicCAS(vword, w, w + 1u);
      if (prev == w) {
        t = int(w & 0xffu);
        break;
      }
      w = prev;
    }
  }
  return __shfl_sync(0xffffffffu, t, 0);
}

// Task `task` of flush unit U (stage s, chain results of chain warp ccw): head
// task / 4 (two-head units), vblock task % 4.  Its 32 outputs go through
// `stage` (32 floats of the executing warp) to HBM; its rows of the tile are
// re-quantised in place and made visible to the tensor-map store.
template <bool FUSED, int HPU>
__device__ __forceinline__ void s5_flush_task(const StepParams& p, uint8_t* smem, const S5Layout& lay,
                                              const S5Unit& U, int s, int ccw, int code, int task, float* stage,
                                              uint32_t stash, int lane) {
  const int head = HPU == 2 ? task >> 2 : 0, v = task & 3;
  uint8_t* sb = smem + lay.stage0 + s * lay.stage_bytes;
  const uint8_t* res = smem + lay.res0 + ccw * lay.res_bytes;
  const uint8_t* fd = res + lay.t8;
  const float* fh = reinterpret_cast<const float*>(fd + S5_FHEAD + head * S5_FHEAD_BYTES);
  const int hv = U.hv0 + head;
  s5_flush_vblock<s5_tc<HPU, true>()>(sb + lay.ck + head * 16384, sb + lay.vr + head * 4096,
                  FUSED ? reinterpret_cast<const uint16_t*>(res + lay.vnew + head * 256) : nullptr,
                  smem + lay.kbuf0 + ccw * 4096, reinterpret_cast<const __half*>(fd + S5_FQ16), fh, VBLOCK * v,
                  s5_n(code), s5_nmem(code), fh[S5_FSC + v], p.quant_rounded, p.sc,
                  int64_t(U.s) * p.sc_sb + int64_t(hv) * p.sc_sh + int64_t(v) * p.sc_sv, p.sc_dt, stage, stash,
                  lane);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp();
  store_scalar(p.out, int64_t(U.b) * p.o_sb + int64_t(hv) * p.o_sh + int64_t(VBLOCK * v + lane) * p.o_sv, p.o_dt,
               stage[lane] * KSCALE_H);
  __syncwarp();
}

// SIDX: packed decode (state slots through StepParams::sidx)
// I8: int8 checkpoint codes ("vblock_int8"); the variant without the flush path only
// WT: the split replay (replay mode, no flush): T and c also go to the caller's buffers
template <bool FUSED, int HPU, bool FLUSH, bool SIDX, bool I8 = false, bool WT = false>
__global__ void __launch_bounds__(S5_THREADS, 1)
    step5_kernel(const __grid_constant__ StepParams p, const __grid_constant__ CUtensorMap ck_map,
                 const __grid_constant__ CUtensorMap kr_map, const __grid_constant__ CUtensorMap vr_map,
                 const __grid_constant__ CUtensorMap gr_map, const __grid_constant__ CUtensorMap br_map) {
  static_assert(!(I8 && (FLUSH || SIDX)), "int8 checkpoints: the non-flush, slot-free variant only");
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr bool TC = s5_tc<HPU, FLUSH>();
  constexpr bool TCR = s5_tcr<HPU, FLUSH>();  // non-flush entries on the tensor cores
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int L = p.L, G = p.HV / p.H;
  const S5Geo geo = s5_geo(p.H, p.HV, L, p.hpu1 != 0);
  const int total = p.B * p.H * geo.upk;
  const int grid = int(gridDim.x), bid = int(blockIdx.x);
  const int nu = total > bid ? (total - bid + grid - 1) / grid : 0;
  const int max_units = (total + grid - 1) / grid;
  const S5Layout lay = s5_layout(geo, max_units, FLUSH);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + lay.full);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + lay.empty);
  uint64_t* kfull = reinterpret_cast<uint64_t*>(smem + lay.kfull);
  // per chain warp, one phase per unit: its chain is finished (cbar), its
  // readout warps are finished with it (rbar)
  uint64_t* cbar = reinterpret_cast<uint64_t*>(smem + lay.cbar);
  uint64_t* rbar = reinterpret_cast<uint64_t*>(smem + lay.rbar);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + lay.abort);
  uint32_t* vword = reinterpret_cast<uint32_t*>(smem + lay.vword);  // flush task word per stage
  uint32_t* vdone = reinterpret_cast<uint32_t*>(smem + lay.vdone);  // flush tasks finished per stage
  uint64_t* mmab = reinterpret_cast<uint64_t*>(smem + lay.mmab);    // tensor-core readout of a stage done
  int* table = reinterpret_cast<int*>(smem + lay.table);
  uint32_t* tdone = reinterpret_cast<uint32_t*>(smem + lay.tdone);  // flush tasks done per unit (tensor-memory readout)
  // self-check of the launch: the swizzled TMA boxes need 1024-byte alignment, and
  // the layout must fit the dynamic shared memory the launch was given
  uint32_t dyn_smem;
  asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn_smem));
  if ((smem_addr(smem) & 1023u) != 0 || lay.total > dyn_smem || geo.hpu != HPU) {
    if (tid == 0) atomicOr(p.err, GDNR_DEVERR_LAYOUT);
    return;
  }
  const uint32_t box_bytes = uint32_t(geo.rb) * 256u;
  const uint32_t ck_bytes = uint32_t(HPU) * 16384u;

  if (warp == 1 && lane < 3) {  // the tensor maps' descriptors, ahead of their first copies
    const CUtensorMap* m = lane == 0 ? &kr_map : (lane == 1 ? &ck_map : &vr_map);
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
  }
  if (tid == 0) {
    for (int s = 0; s < S5_NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], s5_rpu<HPU, FLUSH>());
      mbar_init(&mmab[s], 1);
    }
    for (int c = 0; c < S5_NCW; ++c) {
      mbar_init(&kfull[c], 1);
      mbar_init(&cbar[c], 1);
      mbar_init(&rbar[c], s5_rpu<HPU, FLUSH>());
    }
    for (int st = 0; st < S5_NS; ++st) {
      vword[st] = 0xffffffffu;
      vdone[st] = 0u;
    }
    *abort = 0;
    reinterpret_cast<volatile int*>(smem + lay.tmem)[1] = -1;  // commits issued, published by the scheduler at exit
    fence_mbar_init();
  }
  __syncthreads();
  // two-head units: the first readout warp allocates the readout's tensor
  // memory (released by the same warp at the end); the other readout warps see
  // the address after barrier 1
  if (TC && warp == 1 + S5_NCW) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(smem + lay.tmem)),
                 "r"(S5_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    s5_tc_before_sync();
  }

  // Checkpoint tiles of the first stages: decode state, not output of the
  // preceding kernel (see GDNR_LAUNCH_PDL), so under programmatic dependent
  // launch they stream while that kernel drains.
  const int npro = nu < S5_NS ? nu : S5_NS;
  auto prologue = [&]() {
    for (int i = 0; i < npro; ++i) {
      const S5Unit U = s5_unit<SIDX>(bid + i * grid, p, G, geo);
      s5_expect_tx(&full[i], ck_bytes);
      s5_tma4(smem + lay.stage0 + i * lay.stage_bytes + lay.ck, &ck_map, 0, 0, U.hv0, U.s, &full[i]);
    }
  };
  if (p.pdl && !p.sidx && warp == 0 && lane == 0) prologue();  // slots come from an input
  griddep_wait();
  // Chain warps: the first unit's inputs and whole key ring (small, on the
  // critical path), alongside the checkpoint stream.
  const int cw = warp - 1;
  const bool chain_warp = warp >= 1 && warp <= S5_NCW;
  const int nreq_k = (L + geo.rb - 1) / geo.rb;
  uint8_t* kbuf = smem + lay.kbuf0 + (chain_warp ? cw : 0) * 4096;
  uint8_t* gbuf = smem + lay.gbuf0 + (chain_warp ? cw : 0) * 512;
  // gate rings of unit U with its key ring (variant without the flush path)
  const bool gtma = !FLUSH && p.gtma;
  const uint32_t gate_bytes = gtma ? 2u * 16u * uint32_t(L) : 0u;
  auto issue_gates = [&](const S5Unit& U) {
    s5_tma3(gbuf, &gr_map, U.hv0 & ~(s5_gate_hb(p.gr_dt) - 1), 0, U.s, &kfull[cw]);
    s5_tma3(gbuf + 256, &br_map, U.hv0 & ~(s5_gate_hb(p.br_dt) - 1), 0, U.s, &kfull[cw]);
  };
  S5In in0;
  if (chain_warp) {
    const int i0 = cw < nu ? cw : 0;
    const S5Unit U = s5_unit<SIDX>(bid + i0 * grid, p, G, geo);
    if (lane == 0) {
      const int nr = cw < nu && U.s >= 0 ? nreq_k : 0;
      mbar_arrive_expect_tx(&kfull[cw], uint32_t(nr) * box_bytes + (nr > 0 ? gate_bytes : 0u));
      for (int j = 0; j < nr; ++j) s5_tma5(kbuf + j * box_bytes, &kr_map, 0, 0, U.h, j * geo.rb, U.s, &kfull[cw]);
      if (gtma && nr > 0) issue_gates(U);
    }
    in0 = s5_fetch<FUSED, HPU, FLUSH>(p, U, lane);
    // the key rings and these loads go out first; the producer starts the
    // checkpoint stream once the ring positions (issued alongside) are back
    // (barriers 3 and 2): DRAM serves a running stream before scattered loads
    asm volatile("bar.arrive 3, %0;" ::"n"(32 * (1 + S5_NCW)) : "memory");
  } else if (warp == 0) {
    asm volatile("bar.sync 3, %0;" ::"n"(32 * (1 + S5_NCW)) : "memory");
  }
  // readout warps: vblock scales of their first units, raw until used.
  // Vblock readout: lane l holds unit l's scale of the warp's head and vblock.
  // One-head units (teams): lane l holds team unit l / (2 HPU), vblock l % (2 HPU)
  // of the warp's rows.
  constexpr bool VB = s5_vb<FLUSH>();
  constexpr int VBW = 2 * HPU;  // vblocks per readout warp and unit (teams)
  constexpr int VPW = s5_vpw<HPU>();              // vblock readout: vblocks per warp and unit
  constexpr int WPU = 4 * HPU / VPW;             // vblock readout: warps per unit
  constexpr int SC_UNITS = VB ? 32 / VPW : 32 / VBW;  // units with a prefetched scale
  uint32_t scl_raw = 0u;
  const int rw = warp - 1 - S5_NCW;
  const int team = rw / S5_TEAM, mem = rw % S5_TEAM;
  const int vq = (rw % WPU) * VPW;  // vblock readout: the warp's first vblock of a unit (0..4 HPU - 1)
  const int head_r = TC ? (HPU == 2 ? (rw >> 2) : 0) : (VB ? vq / 4 : (HPU == 2 ? mem : 0));
  const int rbase = VB ? 32 * (vq % 4) : (HPU == 2 ? 0 : 64 * mem);
  if (warp > S5_NCW) {
    if constexpr (TC) {  // the zero rows of the tensor-core T operands
      reinterpret_cast<uint32_t*>(smem + lay.zb)[tid - 32 * (1 + S5_NCW)] = 0u;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    } else if constexpr (VB) {
      // lane l: unit l / VPW, the warp's vblock l % VPW
      const int i = lane / VPW < nu ? lane / VPW : 0;
      const S5Unit U = s5_unit<SIDX>(bid + i * grid, p, G, geo);
      scl_raw = s5_ld_raw(p.sc, int64_t(U.s < 0 ? 0 : U.s) * p.sc_sb + int64_t(U.hv0 + head_r) * p.sc_sh +
                                    int64_t(rbase / VBLOCK + lane % VPW) * p.sc_sv,
                          p.sc_dt);
    } else {
      int i = team + S5_NS * (lane / VBW);
      i = i < nu ? i : 0;
      const S5Unit U = s5_unit<SIDX>(bid + i * grid, p, G, geo);
      const int vb = rbase / VBLOCK + lane % VBW;
      scl_raw = s5_ld_raw(p.sc, int64_t(U.s < 0 ? 0 : U.s) * p.sc_sb + int64_t(U.hv0 + head_r) * p.sc_sh +
                                    int64_t(vb) * p.sc_sv,
                          p.sc_dt);
    }
  }
  // ring positions of this CTA's units for the producer and the readout, read
  // by the threads from the top of the block down (the producer is busy
  // issuing the checkpoint stream, which blocks at the SM's share of HBM)
  const int ti = S5_THREADS - 1 - tid;
  int raw0 = 0, raw1 = 0;
  if (ti < nu) {
    const S5Unit U = s5_unit<SIDX>(bid + ti * grid, p, G, geo);
    if constexpr (FUSED) {
      raw0 = U.s >= 0 ? p.pos[int64_t(U.s) * p.pos_s] : INT_MIN;  // null / bad slot: skipped
    } else {
      raw0 = p.valid_len[int64_t(U.b) * p.vl_s];
      raw1 = p.flush ? s5_ld_flag(p.flush, int64_t(U.b) * p.fl_s, p.fl_dt) : 0;
    }
  }
  if (tid == S5_THREADS - 1) griddep_launch();
  if (ti < nu) {
    const S5Unit U = s5_unit<SIDX>(bid + ti * grid, p, G, geo);
    const int code = s5_code<FUSED>(raw0, raw1, L, FLUSH);
    if (FUSED && s5_n(code) == 0 && U.s >= 0 && U.h == 0 && U.pp == 0) atomicOr(p.err, GDNR_DEVERR_BAD_POS);
    if (U.s == -2 && U.h == 0 && U.pp == 0) atomicOr(p.err, GDNR_DEVERR_BAD_SLOT);
    if constexpr (SIDX) {
      if (U.s < 0) {  // null / bad slot: a zero output row, as the production op stores
        for (int e = 0; e < geo.hpu; ++e)
          for (int r = 0; r < VD; ++r)
            store_scalar(p.out, int64_t(U.b) * p.o_sb + int64_t(U.hv0 + e) * p.o_sh + int64_t(r) * p.o_sv, p.o_dt, 0.f);
      }
    }
    if (s5_n(code) > 0 && s5_skip(code) && p.flush_hint == GDNR_FLUSH_NONE && U.h == 0 && U.pp == 0)
      atomicOr(p.err, GDNR_DEVERR_BAD_HINT);
    if (!FUSED && s5_skip(code) && p.flush_hint == GDNR_FLUSH_NONE && U.h == 0 && U.pp == 0)
      atomicOr(p.err, GDNR_DEVERR_BAD_HINT);
    raw0 = code;
  }
  // Processing order.  In the tensor-memory variant, when every unit of the CTA has
  // a chain warp of its own (nu <= S5_NCW, so the chain phases impose no order)
  // and no checkpoint was requested ahead by the PDL prologue, the flush units go
  // first: their vblock tasks then overlap the other units' chains instead of
  // trailing the CTA's last readout.  The units' entries are then all in the
  // last warp (ti = 31 - lane).  Otherwise unit order.
  // Claim mode (tensor-memory variant, every unit with a chain warp of its own, no
  // PDL prologue): the flush units take entries whose stage no later entry reuses
  // (the last entries of the first round of stages, then the last entries), so
  // that their long rebuild holds no stage another unit waits for; the other
  // units fill the remaining entries in order, and readout groups claim those in
  // order (the chain warps 1..4, whose single units are done early, forming a
  // third group).  All the CTA's units are then in the last warp (ti = 31 - lane).
  const bool claim = TC && nu <= S5_NCW && !p.pdl;
  if (ti < 32 && warp == (S5_THREADS / 32) - 1) {
    int at = ti;
    if (claim) {
      const uint32_t fu = __brev(__ballot_sync(0xffffffffu, ti < nu && s5_flush(raw0)));  // bit ti: unit ti flushes
      const int nf = __popc(fu);
      uint32_t fp = 0u;  // entries of the flush units
      int cnt = 0;
      const int first_round = nu < S5_NS ? nu : S5_NS;
      for (int q = first_round - 1; q >= 0 && q + S5_NS >= nu && cnt < nf; --q, ++cnt) fp |= 1u << q;
      for (int q = nu - 1; q >= 0 && cnt < nf; --q)
        if (!((fp >> q) & 1u)) {
          fp |= 1u << q;
          ++cnt;
        }
      const bool fl = ti < nu && ((fu >> ti) & 1u);
      // k-th flush unit -> k-th flush entry; k-th other unit -> k-th other entry
      const int k = __popc((fl ? fu : ~fu) & ((1u << ti) - 1u));
      const uint32_t pool = fl ? fp : (~fp & ((1u << nu) - 1u));
      int seen = -1;
      for (int q = 0; q < 32 && seen < k; ++q)
        if ((pool >> q) & 1u) {
          ++seen;
          at = q;
        }
      uint32_t* gw = reinterpret_cast<uint32_t*>(smem + lay.gwords);
      if (ti < nu && !fl) gw[8 + k] = uint32_t(at);  // claimable entries, in order
      if (lane == 0) {
        gw[0] = uint32_t(nf);
        gw[1] = 0u;  // next claimable entry (rank)
      }
    }
    if (ti < nu) {
      table[at] = raw0 | (ti << 24);
      tdone[at] = 0u;
    }
  } else if (ti < nu) {
    table[ti] = raw0 | (ti << 24);
    tdone[ti] = 0u;
  }
  // The table is for the producer and the readout warps: the readout warps
  // sync on it (barrier 1) and signal it to the producer (barrier 2), which
  // joins once it has issued the checkpoint stream.  Chain warps decode their
  // own units.
  if (warp > S5_NCW) {
    asm volatile("bar.arrive 2, %0;" ::"n"(32 * (1 + S5_NRW)) : "memory");
    asm volatile("bar.sync 1, %0;" ::"n"(32 * S5_NRW) : "memory");
    // the chain warps of the third readout group read the table after their chains
    if (claim) asm volatile("bar.arrive 10, %0;" ::"n"(32 * (S5_NRW + 4)) : "memory");
  } else if (warp == 0) {
    asm volatile("bar.sync 2, %0;" ::"n"(32 * (1 + S5_NRW)) : "memory");
  }

  if (warp == 0) {
    // =================== producer / scheduler ===================
    if (lane != 0) return;
    // stage loads of entry i (stage i % S5_NS, free once its previous unit is read out)
    int pf_next = S5_NS;  // next entry to prefetch into L2
    auto load_unit = [&](int i) {
      const int s = i % S5_NS;
      const int code = table[i];
      const S5Unit U = s5_unit<SIDX>(bid + s5_uidx(code) * grid, p, G, geo);
      uint8_t* sb = smem + lay.stage0 + s * lay.stage_bytes;
      const bool skip = s5_skip(code);
      const int nreq = skip ? 0 : (s5_nmem(code) + geo.rb - 1) / geo.rb;
      const bool ck = i >= (p.pdl && !p.sidx ? npro : 0) && !skip;  // not already requested before griddepcontrol.wait
      mbar_arrive_expect_tx(&full[s], (ck ? ck_bytes : 0u) + uint32_t(nreq * HPU) * box_bytes);
      if (ck) s5_tma4(sb + lay.ck, &ck_map, 0, 0, U.hv0, U.s, &full[s]);
      for (int j = 0; j < nreq; ++j)
#pragma unroll
        for (int e = 0; e < HPU; ++e)
          s5_tma5(sb + lay.vr + e * 4096 + j * box_bytes, &vr_map, 0, 0, U.hv0 + e, j * geo.rb, U.s, &full[s]);
      if (i >= S5_NS - 1) {
        // the next S5_PF units waiting for a free stage: their tiles and rings into
        // L2 now, so that their stage loads later are served from L2 (a bounded
        // window: prefetching every remaining unit of a large batch would overrun L2)
        for (; pf_next < nu && pf_next <= i + S5_PF; ++pf_next) {
          const int cu = table[pf_next];
          if (s5_skip(cu)) continue;
          const S5Unit V = s5_unit<SIDX>(bid + s5_uidx(cu) * grid, p, G, geo);
          s5_prefetch4(&ck_map, 0, 0, V.hv0, V.s);
          const int nr = (s5_nmem(cu) + geo.rb - 1) / geo.rb;
          for (int j = 0; j < nr; ++j)
#pragma unroll
            for (int e = 0; e < HPU; ++e) s5_prefetch5(&vr_map, 0, 0, V.hv0 + e, j * geo.rb, V.s);
        }
      }
    };
    if constexpr (TCR) {
      // Tensor-memory readout: this thread also issues each unit's tensor-core readout
      // as soon as its stage has landed and its chain is done -- per head 4 x
      // tcgen05.mma (M = 128 rows, N = 16: five T terms + zeros, K = 32) from the
      // stage tile and the chain's T operand into the stage's 32 tensor-memory
      // columns -- and commits it to mmab[s], one commit per unit (none issued
      // for a flush or skipped unit: the commit then arrives at once), so that
      // mmab[s] completes one phase per unit of the stage.  The columns are free:
      // a stage's next load needs all readout warps to release it first.
      // Nothing here blocks: loads and readouts progress as stages free up and
      // chains finish.
      int nl = 0, nm = 0;
      const uint64_t t0 = globaltimer_ns();
      for (uint32_t it = 0; (nl < nu || nm < nu) && it < WAIT_LIMIT_ITERS; ++it) {
        bool progress = false;
        while (nl < nu && (nl < S5_NS || s5_test_wait(&empty[nl % S5_NS], uint32_t(((nl / S5_NS) - 1) & 1))) &&
               !*abort) {
          load_unit(nl++);
          progress = true;
        }
        // flush entries: their commit (no MMAs: it arrives at once, keeping mmab's
        // phases one per entry) once their stage has landed; every other entry's
        // MMAs and commit are issued by the readout group that takes it
        // (tc_group_entry), several entries at a time
        while (nm < nl) {
          const int cu = table[nm];
          if (FLUSH && s5_flush(cu)) {
            if (!s5_test_wait(&full[nm % S5_NS], uint32_t((nm / S5_NS) & 1))) break;
            s5_umma_commit(&mmab[nm % S5_NS]);
          }
          ++nm;
          progress = true;
        }
        if (!progress) {
          if ((it & 63u) == 0 && (*abort || globaltimer_ns() - t0 > 4 * WAIT_LIMIT_NS)) break;
          __nanosleep(32);
        }
      }
      if (nl < nu || nm < nu) {
        if (!*abort) atomicOr(p.err, GDNR_DEVERR_WAIT_TIMEOUT);
        *abort = 1;
      }
      // the readout's tensor-memory release waits for the last commit issued
      s5_st_release(reinterpret_cast<uint32_t*>(smem + lay.tmem) + 1, uint32_t(nm));
      if (*abort) s5_drain_stages(full, nl);
    } else {
      int nl = 0;
      for (; nl < nu; ++nl) {
        if (nl >= S5_NS && !s5_wait(&empty[nl % S5_NS], ((nl / S5_NS) - 1) & 1, p.err, abort)) break;
        if (*abort) break;  // read after the wait: a stage released under abort may still be loading
        load_unit(nl);
      }
      if (*abort) s5_drain_stages(full, nl);
    }
    return;
  }

  // ---- tensor-memory readout of one entry that does not flush, by one warp of a
  // readout group (4 warps, one per tensor-memory lane quarter qd = warp % 4): both
  // heads of the rows 32 qd .. 32 qd + 31.  The scheduler thread has issued the
  // entry's MMAs (five T terms per head into stage s's 32 columns: head h at
  // 16 h); per row: the terms' weighted sum, V^T c over the ring slots, this
  // token's own slot, K^-1/2, one store per head.  The group owes the unit's 8
  // stage and chain-result arrivals: 2 per warp.
  auto tc_group_entry = [&](int i, int code) {
    const int s = i % S5_NS;
    const uint32_t par = (i / S5_NS) & 1;
    const int ui = s5_uidx(code);
    const int ccw = ui % S5_NCW, k = ui / S5_NCW;
    const int qd = warp & 3, row = 32 * qd + lane;
    const S5Unit U = s5_unit<SIDX>(bid + ui * grid, p, G, geo);
    const bool skip = s5_skip(code);
    // this quarter's vblock scale of both heads, issued before the waits
    uint32_t scr[2] = {0u, 0u};
    if (!skip) {
#pragma unroll
      for (int h = 0; h < 2; ++h)
        scr[h] = s5_ld_raw(p.sc, int64_t(U.s) * p.sc_sb + int64_t(U.hv0 + h) * p.sc_sh + int64_t(qd) * p.sc_sv,
                           p.sc_dt);
    }
    bool ok = s5_warp_wait(&full[s], par, p.err, abort, lane);
    ok = s5_warp_wait(&cbar[ccw], uint32_t(k & 1), p.err, abort, lane) && ok;
    const bool mma = ok && !skip;
    const uint8_t* sb = smem + lay.stage0 + s * lay.stage_bytes;
    const uint8_t* res = smem + lay.res0 + ccw * lay.res_bytes;
    // the group's first thread issues the entry's readout on the tensor cores -- per
    // head 4 x tcgen05.mma (M = 128 rows, N = 16: the five T terms and zeros, K =
    // 32) from the stage tile and the chain's T operand into the stage's 32 columns
    // -- and its commit (one per entry, also without MMAs, so that mmab[s]
    // completes one phase per entry of the stage)
    const bool leader = (warp & 3) == 0 && lane == 0;
    if (leader) {
      if (mma) {
        s5_tc_after_sync();
        const uint32_t tm = *reinterpret_cast<volatile uint32_t*>(smem + lay.tmem);
        const uint32_t zb = smem_addr(smem + lay.zb);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint32_t bs = smem_addr(res + lay.t8 + h * 1024) + 256 * ks;
            s5_umma_e4m3(tm + uint32_t(s * 32 + h * 16), s5_desc_sw128(smem_addr(sb + lay.ck + h * 16384) + 32 * ks),
                         s5_desc_cm(bs, 128, zb - bs), ks > 0 ? 1u : 0u);
          }
      }
      s5_umma_commit(&mmab[s]);
    }
    float ov[2] = {0.0f, 0.0f};
    if (mma) {
      // V^T c: all 16 slots loaded unconditionally (the region is always
      // allocated), the slots >= nmem (stale or unloaded data) selected away
      const int nmem = s5_nmem(code);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint8_t* vr = sb + lay.vr + h * 4096;
        const float4* cf = reinterpret_cast<const float4*>(res + lay.cf) + h * 4;
        uint16_t vraw[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) vraw[t] = *reinterpret_cast<const uint16_t*>(vr + s5_ring_off(t, row));
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 c4 = cf[q];
          const float cq[4] = {c4.x, c4.y, c4.z, c4.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int t = 4 * q + j;
            ov[h] = fmaf(cq[j], t < nmem ? bf16_to_f(vraw[t]) : 0.0f, ov[h]);
          }
        }
        if constexpr (FUSED) {
          const float* misc = reinterpret_cast<const float*>(res + lay.misc) + h * 4;
          ov[h] = fmaf(misc[1], bf16_to_f(reinterpret_cast<const uint16_t*>(res + lay.vnew + h * 256)[row]), ov[h]);
        }
      }
    }
    const bool mok = s5_warp_wait(&mmab[s], par, p.err, abort, lane);
    // abort: the MMAs this thread issued finish before the tensor memory is released
    if (!mok && leader) s5_drain_wait(&mmab[s], par);
    float o[2] = {0.0f, 0.0f};
    if (mma) {
      s5_tc_after_sync();
      const uint32_t tm = *reinterpret_cast<volatile uint32_t*>(smem + lay.tmem);
      uint32_t d[32];
      s5_tmem_ld32(tm + (uint32_t(32 * qd) << 16) + uint32_t(s * 32), d);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float* misc = reinterpret_cast<const float*>(res + lay.misc) + h * 4;
        float ot = __uint_as_float(d[16 * h + 4]) * (1.0f / 16.0f);
        ot = (ot + __uint_as_float(d[16 * h + 3])) * (1.0f / 16.0f);
        ot = (ot + __uint_as_float(d[16 * h + 2])) * (1.0f / 16.0f);
        ot = (ot + __uint_as_float(d[16 * h + 1])) * (1.0f / 16.0f);
        ot = ot + __uint_as_float(d[16 * h]);
        o[h] = mok ? fmaf(ot, misc[0] * s5_cvt(scr[h], p.sc_dt), ov[h]) : 0.0f;
      }
    }
    // release the stage and the chain's results before the output stores: every
    // read of them has been consumed, so relaxed releases suffice after an MMA
    s5_tc_before_sync();
    __syncwarp();
    if (lane == 0) {
      if (mma) {
        s5_arrive_relaxed_n(&empty[s], 2u);
        s5_arrive_relaxed_n(&rbar[ccw], 2u);
      } else {
        s5_arrive_n(&empty[s], 2u);
        s5_arrive_n(&rbar[ccw], 2u);
      }
    }
    if (mma) {
#pragma unroll
      for (int h = 0; h < 2; ++h)
        store_scalar(p.out, int64_t(U.b) * p.o_sb + int64_t(U.hv0 + h) * p.o_sh + int64_t(row) * p.o_sv, p.o_dt,
                     o[h] * KSCALE_H);
    }
  };
  // ---- vblock readout of one entry that does not flush (S5_VBF), by one warp of a
  // readout group of 4: warp position q = warp % 4 reads the two 32-row vblocks
  // 2q, 2q + 1 of the unit (head q / 2) as the variant without the flush path
  // does; the group's 4 warps owe the 8 arrivals of the entry (2 each).
  auto vb_group_entry = [&](int i, int code) {
    constexpr int VP = s5_vpw<HPU>();
    const int s = i % S5_NS;
    const uint32_t par = (i / S5_NS) & 1;
    const int ui = s5_uidx(code);
    const int ccw = ui % S5_NCW, k = ui / S5_NCW;
    const int vqw = (warp & 3) * VP;
    const int hr = vqw / 4, rb = 32 * (vqw % 4);
    const S5Unit U = s5_unit<SIDX>(bid + ui * grid, p, G, geo);
    const bool skip = s5_skip(code);
    // lane v < VP: the scale of vblock rb / 32 + v, issued before the waits
    uint32_t scr = 0u;
    if (!skip && lane < VP)
      scr = s5_ld_raw(p.sc, int64_t(U.s) * p.sc_sb + int64_t(U.hv0 + hr) * p.sc_sh + int64_t(rb / VBLOCK + lane) * p.sc_sv,
                      p.sc_dt);
    int okw = 1;
    if (lane == 0) {
      okw = s5_wait(&full[s], par, p.err, abort) ? 1 : 0;
      okw = (s5_wait(&cbar[ccw], uint32_t(k & 1), p.err, abort) && okw) ? 1 : 0;
    }
    const bool ok = __shfl_sync(0xffffffffu, okw, 0) != 0;
    if (ok && !skip) {
      const uint8_t* sb = smem + lay.stage0 + s * lay.stage_bytes;
      const uint8_t* res = smem + lay.res0 + ccw * lay.res_bytes;
      const float* misc = reinterpret_cast<const float*>(res + lay.misc) + hr * 4;
      const int orow = rb + s5_rd_row(lane);
      float o[VP];
      s5_readout<2 * VP, I8, true>(sb + lay.ck + hr * 16384, sb + lay.vr + hr * 4096, res + lay.t8 + hr * 8 * T8STR,
                                   reinterpret_cast<const uint16_t*>(res + lay.cb + hr * 96), misc[0],
                                   s5_cvt(scr, p.sc_dt), 0, rb, s5_nmem(code), o, lane);
      if (FUSED) {
        const uint16_t* vnew = reinterpret_cast<const uint16_t*>(res + lay.vnew + hr * 256);
        const float c1 = misc[1];
#pragma unroll
        for (int r = 0; r < VP; ++r) o[r] = fmaf(c1, bf16_to_f(vnew[orow + 32 * r]), o[r]);
      }
      __syncwarp();
      if (lane == 0) {
        s5_arrive_relaxed_n(&empty[s], 2u);
        s5_arrive_relaxed_n(&rbar[ccw], 2u);
      }
      const int64_t ob = int64_t(U.b) * p.o_sb + int64_t(U.hv0 + hr) * p.o_sh;
#pragma unroll
      for (int r = 0; r < VP; ++r) store_scalar(p.out, ob + int64_t(orow + 32 * r) * p.o_sv, p.o_dt, o[r] * KSCALE_H);
    } else {
      __syncwarp();
      if (lane == 0) {
        s5_arrive_n(&empty[s], 2u);
        s5_arrive_n(&rbar[ccw], 2u);
      }
    }
  };
  // Claim mode: the group's first warp claims the next entry after the flush
  // entries (a shared counter), the group syncs on a named barrier of its own and
  // reads the claim (double-buffered, so that a claim is never overwritten before
  // the whole group has read it); a claim past the last entry ends the loop.
  auto tc_claim_loop = [&](int grp) {
    uint32_t* gw = reinterpret_cast<uint32_t*>(smem + lay.gwords);
    const int ncl = nu - int(gw[0]);
    for (int round = 0;; ++round) {
      volatile uint32_t* slot = gw + 2 + 2 * grp + (round & 1);
      if ((warp & 3) == 0 && lane == 0) *slot = atomicAdd(&gw[1], 1u);
      asm volatile("bar.sync %0, %1;" ::"r"(12 + grp), "n"(128) : "memory");
      const int r = int(*slot);
      if (r >= ncl) break;
      const int i = int(gw[8 + r]);
      if constexpr (TCR)
        tc_group_entry(i, table[i]);
      else
        vb_group_entry(i, table[i]);
    }
  };

  if (chain_warp) {
    // =================== chain warps ===================
    uint8_t* res = smem + lay.res0 + cw * lay.res_bytes;
    for (int i = cw, k = 0; i < nu; i += S5_NCW, ++k) {
      const S5Unit U = s5_unit<SIDX>(bid + i * grid, p, G, geo);
      bool ok = true;
      if (k > 0) {
        // the key ring and result block are free once both readout warps of
        // this warp's previous unit are done with them
        ok = s5_warp_wait(&rbar[cw], uint32_t((k - 1) & 1), p.err, abort, lane);
        if (!ok) break;  // abort: this warp issues no further loads
        // every lane's earlier generic accesses to kbuf, ordered before the
        // copy engine overwrites it
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          const int nr = U.s >= 0 ? nreq_k : 0;
          mbar_arrive_expect_tx(&kfull[cw], uint32_t(nr) * box_bytes + (nr > 0 ? gate_bytes : 0u));
          for (int j = 0; j < nr; ++j)
            s5_tma5(kbuf + j * box_bytes, &kr_map, 0, 0, U.h, j * geo.rb, U.s, &kfull[cw]);
          if (gtma && nr > 0) issue_gates(U);
        }
        in0 = s5_fetch<FUSED, HPU, FLUSH>(p, U, lane);
      }
      ok = s5_warp_wait(&kfull[cw], k & 1, p.err, abort, lane) && ok;
      if (!ok) {  // abort: the key-ring load of this unit may still be in flight
        if (lane == 0) s5_drain_wait(&kfull[cw], uint32_t(k & 1));
        __syncwarp();
        break;
      }
      const int code = s5_code<FUSED>(in0.pos, in0.flag, L, FLUSH);
      const bool work = ok && !s5_skip(code);
      S5Append ap{};
      if (work) ap = s5_chain<FUSED, HPU, FLUSH, I8, WT>(p, U, code, in0, kbuf, gbuf, res, lay, lane);
      // the T operand is read by the tensor cores (async proxy)
      if (TCR) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) s5_arrive(&cbar[cw]);
      if (work) s5_append<FUSED, HPU>(p, U, code, ap, lane);
    }
    if constexpr (TC) {
      // claim mode: chain warps 1..4 (lane quarters 1, 2, 3, 0) are readout group 2
      // (they continue into the readout below, so that one copy of its code serves
      // all three groups)
      if (!(claim && warp <= 4)) return;
      asm volatile("bar.sync 10, %0;" ::"n"(32 * (S5_NRW + 4)) : "memory");
    } else {
      return;
    }
  }

  if constexpr (TC) {
    // =================== readout through tensor memory ===================
    // Flush entries are read out by all S5_NRW readout warps, one vblock task each
    // (warp w: head w / 4, rows 32 (w % 4) ..); the other entries by readout groups
    // of 4 warps, one per tensor-memory lane quarter, both heads (tc_group_entry):
    // group 0 = readout warps 0..3, group 1 = 4..7, and in claim mode group 2 =
    // chain warps 1..4 once their chains are done.  Claim mode (flush entries
    // first): after the flush entries, the groups claim the remaining entries in
    // order, so that a group that is free takes the next one.  Otherwise groups 0
    // and 1 alternate over the non-flush entries in order.
    s5_tc_after_sync();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + lay.tmem);
    const int qd = warp & 3;
    // this warp's flush stash: its lane quarter, 128 columns (two warps share a quarter)
    // Flush-task workers: the readout warps (worker rw), and in claim mode when
    // every unit of the CTA flushes (no entries to claim) also chain warps 1..4
    // (workers 8..11); a worker takes task (f S5_NRW + t) mod workers of the f-th
    // flush entry, entries in order, so every wait is on an earlier entry.
    const bool allflush = claim && int(reinterpret_cast<const uint32_t*>(smem + lay.gwords)[0]) == nu;
    const int nwk = allflush ? S5_NRW + 4 : S5_NRW;
    const int wk = chain_warp ? S5_NRW + (warp - 1) : rw;
    // the worker's flush stash: its lane quarter, 128 columns (readout warps: two
    // per quarter from S5_TM_STASH; chain warps 1..4: one per quarter after them)
    const uint32_t stash = tmem + (uint32_t(32 * qd) << 16) + S5_TM_STASH +
                           (chain_warp ? 256u : 128u * uint32_t(rw >> 2));
    float* ost = reinterpret_cast<float*>(smem + lay.ost0 + wk * 512);
    auto flush_entry = [&](int i, int task) {
      const int s = i % S5_NS;
      const uint32_t par = (i / S5_NS) & 1;
      const int code = table[i];
      const int ui = s5_uidx(code);
      const int ccw = ui % S5_NCW, k = ui / S5_NCW;
      bool ok = s5_warp_wait(&full[s], par, p.err, abort, lane);
      ok = s5_warp_wait(&cbar[ccw], uint32_t(k & 1), p.err, abort, lane) && ok;
      uint8_t* sb = smem + lay.stage0 + s * lay.stage_bytes;
      const S5Unit U = s5_unit<SIDX>(bid + ui * grid, p, G, geo);
      if constexpr (TCR) s5_warp_wait(&mmab[s], par, p.err, abort, lane);  // keeps the commits in step (none issued for it)
      // The unit's 4 x 2 vblock tasks, one per worker (task `task`), then one
      // tensor-map store by the warp whose acquire-release increment of the unit's
      // done count completes it (the other tasks' released rows are visible to
      // it); the others release the stage now (it is reloaded only after all have).
      static_assert(4 * HPU == S5_NRW, "one flush task per readout warp");
      int last = 0;
      if (ok) {
        s5_flush_task<FUSED, HPU>(p, smem, lay, U, s, ccw, code, task, ost, stash, lane);
        if (lane == 0 && s5_add_acq_rel(&tdone[i], 1u) == uint32_t(S5_NRW - 1)) last = 1;
      }
      if (__shfl_sync(0xffffffffu, last, 0) && lane == 0 && *abort == 0) {
        s5_tma_store4(&ck_map, sb + lay.ck, 0, 0, U.hv0, U.s);
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
      }
      s5_tc_before_sync();
      __syncwarp();
      if (lane == 0) {
        s5_arrive(&empty[s]);
        s5_arrive(&rbar[ccw]);
      }
    };
    // claim mode: chain warps 1..4 arrive here as group 2 (flush tasks too when
    // every unit of the CTA flushes; there is then nothing to claim)
    const int g = chain_warp ? 2 : (rw >> 2);
    if (claim) {
      if (!chain_warp || allflush) {
        int fo = 0;  // flush entries so far
        for (int i = 0; i < nu; ++i)
          if (FLUSH && s5_flush(table[i])) {
            const int t = ((wk - fo * S5_NRW) % nwk + nwk) % nwk;
            if (t < S5_NRW) flush_entry(i, t);
            ++fo;
          }
      }
      tc_claim_loop(g);
    } else {
      int rank = 0;
      for (int i = 0; i < nu; ++i) {
        const int code = table[i];
        if (FLUSH && s5_flush(code)) {
          flush_entry(i, rw);
        } else {
          if ((rank & 1) == g) {
            if constexpr (TCR)
              tc_group_entry(i, code);
            else
              vb_group_entry(i, code);
          }
          ++rank;
        }
      }
    }
    // the last commit covers every MMA this CTA issued: complete before the
    // tensor memory is released (and the third group is done with it)
    if (TCR && rw == 0 && nu > 0 &&
        !s5_warp_wait(&mmab[(nu - 1) % S5_NS], uint32_t(((nu - 1) / S5_NS) & 1), p.err, abort, lane) && lane == 0)
      s5_drain_mma(mmab, reinterpret_cast<const uint32_t*>(smem + lay.tmem) + 1);
    s5_tc_before_sync();
    if (claim)
      asm volatile("bar.sync 11, %0;" ::"n"(32 * (S5_NRW + 4)) : "memory");
    else
      asm volatile("bar.sync 1, %0;" ::"n"(32 * S5_NRW) : "memory");
    if (rw == 0) {
      s5_tc_after_sync();
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(S5_TMEM_COLS) : "memory");
    }
  } else if constexpr (VB) {
  // =================== vblock readout ===================
  // The readout warps form NG groups of WPU warps; group g reads out the units
  // i = g (mod NG), warp q of a group the VPW vblocks (32 rows each) from vblock
  // q VPW of the unit (heads in order); the unit's WPU warps release its stage
  // and chain results as they finish.
  constexpr int NG = S5_NRW / WPU;  // readout groups (units in flight)
  const float sc_pre = s5_cvt(scl_raw, p.sc_dt);
  const int orow = rbase + s5_rd_row(lane);  // the lane's rows: orow + 32 v, v < VPW
  for (int i = rw / WPU; i < nu; i += NG) {
    const int s = i % S5_NS;
    const int ccw = i % S5_NCW, k = i / S5_NCW;
    const int code = table[i];
    float sc = sc_pre;
    int sc_base = i * VPW;
    if (i >= SC_UNITS) {  // beyond the prefetched units: lane v < VPW holds vblock v
      sc = 1.0f;
      sc_base = 0;
      if (lane < VPW && !s5_skip(code)) {
        const S5Unit U = s5_unit<SIDX>(bid + i * grid, p, G, geo);
        sc = load_scalar(p.sc, int64_t(U.s) * p.sc_sb + int64_t(U.hv0 + head_r) * p.sc_sh +
                                   int64_t(rbase / VBLOCK + lane) * p.sc_sv,
                         p.sc_dt);
      }
    }
    // the unit's indices ahead of the waits (integer divisions)
    const S5Unit U = s5_unit<SIDX>(bid + i * grid, p, G, geo);
    int okw = 1;
    if (lane == 0) {
      okw = s5_wait(&full[s], (i / S5_NS) & 1, p.err, abort) ? 1 : 0;
      okw = (s5_wait(&cbar[ccw], uint32_t(k & 1), p.err, abort) && okw) ? 1 : 0;
    }
    const bool ok = __shfl_sync(0xffffffffu, okw, 0) != 0;
    uint8_t* sb = smem + lay.stage0 + s * lay.stage_bytes;
    if (ok && !s5_skip(code)) {
      const uint8_t* res = smem + lay.res0 + ccw * lay.res_bytes;
      const float* misc = reinterpret_cast<const float*>(res + lay.misc) + head_r * 4;
      float o[VPW];
      s5_readout<2 * VPW, I8, true>(sb + lay.ck + head_r * 16384, sb + lay.vr + head_r * 4096,
                                    res + lay.t8 + head_r * 8 * T8STR,
                                    reinterpret_cast<const uint16_t*>(res + lay.cb + head_r * 96), misc[0], sc,
                                    sc_base, rbase, s5_nmem(code), o, lane);
      // this token's own slot (fused) as a rank-one term
      if (FUSED) {
        const uint16_t* vnew = reinterpret_cast<const uint16_t*>(res + lay.vnew + head_r * 256);
        const float c1 = misc[1];
#pragma unroll
        for (int r = 0; r < VPW; ++r) o[r] = fmaf(c1, bf16_to_f(vnew[orow + 32 * r]), o[r]);
      }
      __syncwarp();
      // every read of the stage and the chain's results has returned its value (all
      // of them feed o, which every lane holds after the warp barrier): relaxed
      // arrivals suffice
      if (lane == 0) {
        s5_arrive_relaxed(&empty[s]);
        s5_arrive_relaxed(&rbar[ccw]);
      }
      const int64_t ob = int64_t(U.b) * p.o_sb + int64_t(U.hv0 + head_r) * p.o_sh;
#pragma unroll
      for (int r = 0; r < VPW; ++r) store_scalar(p.out, ob + int64_t(orow + 32 * r) * p.o_sv, p.o_dt, o[r] * KSCALE_H);
    } else {
      __syncwarp();
      if (lane == 0) {
        s5_arrive(&empty[s]);
        s5_arrive(&rbar[ccw]);
      }
    }
  }
  } else {
  // =================== readout teams ===================
  // Team j (2 warps) reads out the units of stage j in order; with two heads
  // per unit each warp takes one head (8 m-tiles), with one head each warp
  // takes 64 of its rows.
  constexpr int MW = 4 * HPU;
  constexpr int ROWS = 16 * MW;
  float* ost = reinterpret_cast<float*>(smem + lay.ost0 + rw * 512);
  const int esz_o = p.o_dt == GDNR_BF16 ? 2 : 4;
  const bool vec_out = p.o_sv == 1 && (reinterpret_cast<uintptr_t>(p.out) % 16) == 0 &&
                       ((p.o_sb * esz_o) % 16) == 0 && ((p.o_sh * esz_o) % 16) == 0;
  for (int i = team, ul = 0; i < nu; i += S5_NS, ++ul) {
    const int s = i % S5_NS;  // == team
    const int ccw = i % S5_NCW, k = i / S5_NCW;
    const int code = table[i];
    float sc = s5_cvt(scl_raw, p.sc_dt);
    int sc_base = ul * VBW;
    if (ul >= SC_UNITS) {  // beyond the prefetched units
      sc = 1.0f;
      sc_base = 0;
      if (lane < VBW && !s5_skip(code)) {
        const S5Unit U = s5_unit<SIDX>(bid + i * grid, p, G, geo);
        sc = load_scalar(p.sc, int64_t(U.s) * p.sc_sb + int64_t(U.hv0 + head_r) * p.sc_sh +
                                   int64_t(rbase / VBLOCK + lane) * p.sc_sv,
                         p.sc_dt);
      }
    }
    bool ok = s5_warp_wait(&full[s], (i / S5_NS) & 1, p.err, abort, lane);
    ok = s5_warp_wait(&cbar[ccw], uint32_t(k & 1), p.err, abort, lane) && ok;
    const bool flush = FLUSH && s5_flush(code);
    uint8_t* sb = smem + lay.stage0 + s * lay.stage_bytes;
    if (flush) {
      // publish the unit's vblock tasks, take them, then write the re-quantised
      // tiles back with one tensor-map store
      constexpr int NT = 4 * HPU;
      if (mem == 0 && lane == 0) {
        vdone[s] = 0u;
        __threadfence_block();
        atomicExch(&vword[s], uint32_t(i) << 8);
      }
      asm volatile("bar.sync %0, %1;" ::"r"(4 + team), "n"(32 * S5_TEAM) : "memory");
      const S5Unit U = s5_unit<SIDX>(bid + i * grid, p, G, geo);
      if (ok) {
        for (;;) {
          const int t = s5_claim(&vword[s], i, NT, lane);
          if (t < 0) break;
          s5_flush_task<FUSED, HPU>(p, smem, lay, U, s, ccw, code, t, ost, 0u, lane);
          if (lane == 0) s5_add_release(&vdone[s], 1u);
        }
      }
      s5_warp_wait_count(&vdone[s], uint32_t(NT), p.err, abort, lane);
      if (mem == 0 && lane == 0 && *abort == 0) {
        s5_tma_store4(&ck_map, sb + lay.ck, 0, 0, U.hv0, U.s);
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
      }
    } else if (ok && !s5_skip(code)) {
      const S5Unit U = s5_unit<SIDX>(bid + i * grid, p, G, geo);
      const uint8_t* res = smem + lay.res0 + ccw * lay.res_bytes;
      const float* misc = reinterpret_cast<const float*>(res + lay.misc) + head_r * 4;
      s5_readout<MW, I8>(sb + lay.ck + head_r * 16384, sb + lay.vr + head_r * 4096, res + lay.t8 + head_r * 8 * T8STR,
                     reinterpret_cast<const uint16_t*>(res + lay.cb + head_r * 96), misc[0], sc, sc_base, rbase,
                     s5_nmem(code), ost, lane);
      __syncwarp();
      // this token's own slot (fused) as a rank-one term, K^-1/2, coalesced store
      constexpr int RPL = ROWS / 32;  // rows per lane: 4 or 2
      const int r0 = RPL * lane;
      float o[RPL];
#pragma unroll
      for (int q = 0; q < RPL; ++q) o[q] = ost[r0 + q];
      if (FUSED) {
        const float cpos = misc[1];
        const uint16_t* vnew = reinterpret_cast<const uint16_t*>(res + lay.vnew + head_r * 256) + rbase;
#pragma unroll
        for (int q = 0; q < RPL; ++q) o[q] = fmaf(cpos, bf16_to_f(vnew[r0 + q]), o[q]);
      }
      const int64_t obase = int64_t(U.b) * p.o_sb + int64_t(U.hv0 + head_r) * p.o_sh;
      if (vec_out) {
        if (esz_o == 2) {
          if constexpr (RPL == 4)
            *reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.out) + obase + rbase + r0) =
                make_uint2(pack_bf16x2(o[0] * KSCALE_H, o[1] * KSCALE_H), pack_bf16x2(o[2] * KSCALE_H, o[3] * KSCALE_H));
          else
            *reinterpret_cast<uint32_t*>(static_cast<uint16_t*>(p.out) + obase + rbase + r0) =
                pack_bf16x2(o[0] * KSCALE_H, o[1] * KSCALE_H);
        } else {
          if constexpr (RPL == 4)
            *reinterpret_cast<float4*>(static_cast<float*>(p.out) + obase + rbase + r0) =
                make_float4(o[0] * KSCALE_H, o[1] * KSCALE_H, o[2] * KSCALE_H, o[3] * KSCALE_H);
          else
            *reinterpret_cast<float2*>(static_cast<float*>(p.out) + obase + rbase + r0) =
                make_float2(o[0] * KSCALE_H, o[1] * KSCALE_H);
        }
      } else {
#pragma unroll
        for (int q = 0; q < RPL; ++q)
          store_scalar(p.out, obase + int64_t(rbase + r0 + q) * p.o_sv, p.o_dt, o[q] * KSCALE_H);
      }
    }
    __syncwarp();
    if (lane == 0) {
      s5_arrive(&empty[s]);
      s5_arrive(&rbar[ccw]);
    }
  }
  }
  // the checkpoint stores are complete before the kernel ends
  if (FLUSH && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// ---------------------------------------------------------------- host side
static int s5_sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return n;
}

static bool s5_grid(const StepParams& p, int& grid, S5Layout& lay) {
  const bool flush = p.flush_hint != GDNR_FLUSH_NONE;
  const int nsm = s5_sm_count();
  if (nsm <= 0) return false;
  const S5Geo g = s5_geo(p.H, p.HV, p.L, p.hpu1 != 0);
  const int64_t total = int64_t(p.B) * p.H * g.upk;
  if (total <= 0 || total > (int64_t(1) << 30)) return false;
  grid = int(total < nsm ? total : nsm);
  const int max_units = int((total + grid - 1) / grid);
  if (max_units > 32 * S5_NRW) return false;  // the unit table is filled in one pass by the readout warps
  lay = s5_layout(g, max_units, flush);
  return true;
}

// The split replay's kernel instantiations (WT) are compiled in a translation unit
// of their own (gdnr_step5_split.cu includes this file with GDNR_S5_SPLIT_TU):
// kept in the same module they shift the code of the flush-capable kernel and
// slow it down (68.3 -> 71.5 us per flush launch, same box).
cudaError_t launch_step5_split(const StepParams& q, const CUtensorMap& ck, const CUtensorMap& kr,
                               const CUtensorMap& vr, const CUtensorMap& gm, const CUtensorMap& bm, int hpu, int grid,
                               uint32_t smem, bool pdl, cudaStream_t stream);

#ifndef GDNR_S5_SPLIT_TU
bool step5_eligible(const StepParams& p, bool fused, bool f32ck) {
  if (f32ck || p.L < 4 || p.L > STEP2_MAX_L) return false;
  // int8 checkpoints: the non-flush variant only (a flush-capable call runs the
  // one-CTA-per-head kernel), and no slot indirection
  if (p.ck_i8 && (p.flush_hint != GDNR_FLUSH_NONE || p.sidx)) return false;
  const int G = p.HV / p.H;
  if (G != 1 && G % 2 != 0) return false;
  if (p.ck_sb % 16 || p.ck_sh % 16 || reinterpret_cast<uintptr_t>(p.ck) % 16) return false;
  // ring tensor maps: 16-byte aligned base and strides
  if (reinterpret_cast<uintptr_t>(p.kr) % 16 || (p.kr_sb * 2) % 16 || (p.kr_st * 2) % 16 || (p.kr_sh * 2) % 16)
    return false;
  if (reinterpret_cast<uintptr_t>(p.vr) % 16 || (p.vr_sb * 2) % 16 || (p.vr_st * 2) % 16 || (p.vr_sh * 2) % 16)
    return false;
  if (fused) {
    const int esz = p.mx_dt == GDNR_BF16 ? 2 : 4;
    if (reinterpret_cast<uintptr_t>(p.mixed) % 16 || (p.mx_sb * esz) % 16) return false;
  } else {
    const int esz = p.q_dt == GDNR_BF16 ? 2 : 4;
    if (reinterpret_cast<uintptr_t>(p.q) % 16 || (p.q_sb * esz) % 16 || (p.q_sh * esz) % 16) return false;
  }
  int grid;
  S5Layout lay;
  if (!s5_grid(p, grid, lay)) return false;
  return lay.total <= MAX_DYN_SMEM;
}
#endif  // GDNR_S5_SPLIT_TU

using S5EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static S5EncodeFn s5_encode_fn() {
  static S5EncodeFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<S5EncodeFn>(ptr);
  }
  return fn;
}

template <bool FUSED, int HPU, bool FLUSH, bool SIDX = false, bool I8 = false, bool WT = false>
static cudaError_t s5_launch(const StepParams& p, const CUtensorMap& ck, const CUtensorMap& kr,
                             const CUtensorMap& vr, const CUtensorMap& gm, const CUtensorMap& bm, int grid,
                             uint32_t smem, bool pdl, cudaStream_t stream) {
  auto kern = step5_kernel<FUSED, HPU, FLUSH, SIDX, I8, WT>;
  static DynSmemCache smem_cache;  // per device: dynamic smem already allowed for this instance
  cudaError_t e = ensure_dyn_smem(reinterpret_cast<const void*>(kern), int(smem), smem_cache);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(S5_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p, ck, kr, vr, gm, bm);
}

#ifndef GDNR_S5_SPLIT_TU
cudaError_t launch_step5(const StepParams& p_in, bool fused, bool pdl, cudaStream_t stream) {
  S5EncodeFn enc = s5_encode_fn();
  if (!enc) return cudaErrorNotSupported;
  // Steps without the flush path on a batch of at most 4 value heads per SM: one
  // value head per unit (twice the units, each chain half as long), which is
  // slightly shorter there (B = 1 / 4 / 16, L = 16: 0.16-0.30 / 0.06-0.59 /
  // 0.14-0.34 us less per launch, two boxes); with more value heads (B = 64:
  // 14.4 -> 22.2 us) or with the flush path (one-head units use the team
  // readout: 17.0 -> 22.8 us at B = 1) the two-head units are faster.
  StepParams p = p_in;
  p.hpu1 = (p.flush_hint == GDNR_FLUSH_NONE && p.HV >= 2 * p.H &&
            int64_t(p.B) * p.HV <= 4 * int64_t(s5_sm_count()))
               ? 1
               : 0;
  const S5Geo g = s5_geo(p.H, p.HV, p.L, p.hpu1 != 0);
  int grid;
  S5Layout lay;
  if (!s5_grid(p, grid, lay)) return cudaErrorInvalidValue;
  CUtensorMap ck, kr, vr;
  const int nst = p.sidx ? p.S : p.B;  // state slots (packed decode: the pool's)
  {
    // checkpoint [slots][HV][V][K] e4m3: box = hpu whole 128 x 128 head tiles
    const cuuint64_t dims[4] = {128, 128, cuuint64_t(p.HV), cuuint64_t(nst)};
    const cuuint64_t strides[3] = {128, cuuint64_t(p.ck_sh), cuuint64_t(p.ck_sb)};
    const cuuint32_t box[4] = {128, 128, cuuint32_t(g.hpu), 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    if (enc(&ck, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, p.ck, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  // rings [B][L][heads][128] bf16 viewed as [B][L][heads][2][64]: a box of rb
  // slots lands as rb x 256-byte rows, each 128-byte half swizzled
  auto ring_map = [&](CUtensorMap* m, void* base, int heads, int64_t s_head, int64_t s_slot, int64_t s_b) {
    const cuuint64_t dims[5] = {64, 2, cuuint64_t(heads), cuuint64_t(p.L), cuuint64_t(nst)};
    const cuuint64_t strides[4] = {128, cuuint64_t(s_head * 2), cuuint64_t(s_slot * 2), cuuint64_t(s_b * 2)};
    const cuuint32_t box[5] = {64, 2, 1, cuuint32_t(g.rb), 1};
    const cuuint32_t es[5] = {1, 1, 1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 5, base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  };
  if (ring_map(&kr, p.kr, p.H, p.kr_sh, p.kr_st, p.kr_sb) != CUDA_SUCCESS) return cudaErrorInvalidValue;
  if (ring_map(&vr, p.vr, p.HV, p.vr_sh, p.vr_st, p.vr_sb) != CUDA_SUCCESS) return cudaErrorInvalidValue;
  // gate rings [slots][L][HV] (heads contiguous) for the variant without the flush
  // path: a box of 16 bytes of heads x L slots per ring, read by TMA with the key ring
  StepParams q = p;
  CUtensorMap gm, bm;
  memset(&gm, 0, sizeof(gm));
  memset(&bm, 0, sizeof(bm));
  q.gtma = 0;
  if (p.flush_hint == GDNR_FLUSH_NONE) {
    auto gate_map = [&](CUtensorMap* m, void* base, int dt, int64_t s_slot, int64_t s_b, int64_t s_head) {
      const int esz = dt == GDNR_F32 ? 4 : 2, hb = 16 / esz;
      if (s_head != 1 || p.HV < hb || reinterpret_cast<uintptr_t>(base) % 16 || (s_slot * esz) % 16 ||
          (s_b * esz) % 16)
        return false;
      const cuuint64_t dims[3] = {cuuint64_t(p.HV), cuuint64_t(p.L), cuuint64_t(nst)};
      const cuuint64_t strides[2] = {cuuint64_t(s_slot * esz), cuuint64_t(s_b * esz)};
      const cuuint32_t box[3] = {cuuint32_t(hb), cuuint32_t(p.L), 1};
      const cuuint32_t es[3] = {1, 1, 1};
      return enc(m, esz == 4 ? CU_TENSOR_MAP_DATA_TYPE_UINT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, base, dims, strides,
                 box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    };
    q.gtma = gate_map(&gm, p.gr, p.gr_dt, p.gr_st, p.gr_sb, p.gr_sh) &&
             gate_map(&bm, p.br, p.br_dt, p.br_st, p.br_sb, p.br_sh);
  }
  // GDNR_FLUSH_NONE: the variant without the flush path (flushing units are
  // skipped and reported); otherwise the flush-capable one
  const bool flush = p.flush_hint != GDNR_FLUSH_NONE;
  const uint32_t sm = lay.total;
  if (p.ck_i8) {  // int8 checkpoints: GDNR_FLUSH_NONE steps only (step5_eligible)
    if (flush || p.sidx) return cudaErrorNotSupported;
    if (fused)
      return g.hpu == 2 ? s5_launch<true, 2, false, false, true>(q, ck, kr, vr, gm, bm, grid, sm, pdl, stream)
                        : s5_launch<true, 1, false, false, true>(q, ck, kr, vr, gm, bm, grid, sm, pdl, stream);
    return g.hpu == 2 ? s5_launch<false, 2, false, false, true>(q, ck, kr, vr, gm, bm, grid, sm, pdl, stream)
                      : s5_launch<false, 1, false, false, true>(q, ck, kr, vr, gm, bm, grid, sm, pdl, stream);
  }
  if (fused && p.sidx) {
    if (g.hpu == 2)
      return flush ? s5_launch<true, 2, true, true>(q, ck, kr, vr, gm, bm, grid, sm, pdl, stream)
                   : s5_launch<true, 2, false, true>(q, ck, kr, vr, gm, bm, grid, sm, pdl, stream);
    return flush ? s5_launch<true, 1, true, true>(q, ck, kr, vr, gm, bm, grid, sm, pdl, stream)
                 : s5_launch<true, 1, false, true>(q, ck, kr, vr, gm, bm, grid, sm, pdl, stream);
  }
  if (p.sidx) return cudaErrorNotSupported;  // packed decode: fused steps only
  if (p.tqo) {  // split replay: replay mode, no flush
    if (fused || flush || p.ck_i8) return cudaErrorNotSupported;
    return launch_step5_split(q, ck, kr, vr, gm, bm, g.hpu, grid, sm, pdl, stream);
  }
  if (fused) {
    if (g.hpu == 2)
      return flush ? s5_launch<true, 2, true>(q, ck, kr, vr, gm, bm, grid, sm, pdl, stream)
                   : s5_launch<true, 2, false>(q, ck, kr, vr, gm, bm, grid, sm, pdl, stream);
    return flush ? s5_launch<true, 1, true>(q, ck, kr, vr, gm, bm, grid, sm, pdl, stream)
                 : s5_launch<true, 1, false>(q, ck, kr, vr, gm, bm, grid, sm, pdl, stream);
  }
  if (g.hpu == 2)
    return flush ? s5_launch<false, 2, true>(q, ck, kr, vr, gm, bm, grid, sm, pdl, stream)
                 : s5_launch<false, 2, false>(q, ck, kr, vr, gm, bm, grid, sm, pdl, stream);
  return flush ? s5_launch<false, 1, true>(q, ck, kr, vr, gm, bm, grid, sm, pdl, stream)
               : s5_launch<false, 1, false>(q, ck, kr, vr, gm, bm, grid, sm, pdl, stream);
}

#else   // GDNR_S5_SPLIT_TU
cudaError_t launch_step5_split(const StepParams& q, const CUtensorMap& ck, const CUtensorMap& kr,
                               const CUtensorMap& vr, const CUtensorMap& gm, const CUtensorMap& bm, int hpu, int grid,
                               uint32_t smem, bool pdl, cudaStream_t stream) {
  return hpu == 2 ? s5_launch<false, 2, false, false, false, true>(q, ck, kr, vr, gm, bm, grid, smem, pdl, stream)
                  : s5_launch<false, 1, false, false, false, true>(q, ck, kr, vr, gm, bm, grid, smem, pdl, stream);
}
#endif  // GDNR_S5_SPLIT_TU

}  // namespace gdnr

// ---------------------------------------------------------------- bounded-wait self-test
#ifndef GDNR_S5_SPLIT_TU
namespace gdnr {

// One CTA, two warps, exercising the error path of the persistent kernel's
// waits (s5_wait / s5_wait_slow, the code every wait of step5_kernel runs):
// warp 0 holds 32 tensor-memory columns and waits on an mbarrier that nothing
// ever arrives on, warp 1 waits on another one.  Warp 0's wait gives up after
// WAIT_LIMIT_NS, records GDNR_DEVERR_WAIT_TIMEOUT and sets the CTA's abort
// word; warp 1's wait then returns at its next poll of that word.  Warp 0
// releases its tensor memory before the kernel returns.  report[0..3]: the two
// waits' results (0 = gave up) and the nanoseconds each waited.
__global__ void __launch_bounds__(64, 1) s5_wait_selftest_kernel(uint32_t* err, unsigned long long* report) {
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ int abort_word;
  __shared__ uint32_t tmem_addr;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    abort_word = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 32;" ::"r"(smem_addr(&tmem_addr))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  volatile int* abort = &abort_word;
  if (lane == 0) {
    const uint64_t t0 = globaltimer_ns();
    const bool ok = s5_wait(&bars[warp], 0u, err, abort);
    const uint64_t t1 = globaltimer_ns();
    report[warp] = ok ? 1ull : 0ull;
    report[2 + warp] = t1 - t0;
    if (warp == 1 && !ok) return;  // an early exit of one warp: the other still releases its tensor memory
  }
  if (warp == 0) {
    __syncwarp();
    s5_tc_before_sync();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 32;" ::"r"(tmem_addr) : "memory");
  }
}

}  // namespace gdnr

extern "C" int gdnr_selftest_wait_timeout(uint32_t* error_flag, unsigned long long* report, void* stream) {
  using namespace gdnr;
  if (!report) return set_error(GDNR_ERR_ARG, "report: null pointer");
  uint32_t* err = error_flag ? error_flag : default_error_word();
  if (!err) return set_error(GDNR_ERR_CUDA, "device error word unavailable");
  s5_wait_selftest_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(err, report);
  return cuda_status(cudaGetLastError(), "gdnr_selftest_wait_timeout launch");
}
#endif  // GDNR_S5_SPLIT_TU
