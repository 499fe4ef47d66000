/*
 * gdnr.h -- C ABI of the B200-native FP8-checkpoint replay GDN decode path.
 *
 * Every entry point takes plain pointers + shapes + strides (gdnr_tensor),
 * never allocates, never synchronises, and enqueues its work on the CUDA
 * stream it is given (a cudaStream_t passed as void*; NULL = legacy default
 * stream).  Return value: GDNR_OK (0) or a negative gdnr_status; the message
 * of the last failure on the calling thread is gdnr_last_error().
 *
 * Reference interfaces replaced (paths inside zz774ever/fp8-replayssm-gdn-kernel):
 *   gdnr_replay          <- gdn_replay_fp8           prototype/gdn_replayssm_fp8_kernel.py:344-405
 *   gdnr_replay_split    <- gdn_replay_fp8_split     prototype/gdn_replayssm_fp8_kernel.py:1129-1235
 *   gdnr_prep_ring       <- gdn_prep_ring            prototype/gdn_replayssm_fp8_kernel.py:710-795
 *   gdnr_bf16_step       <- gdn_bf16_step            prototype/gdn_replayssm_fp8_kernel.py:408-450
 *   gdnr_quantize_vblock32   <- quantize_checkpoint(state, "vblock", 32)
 *                                                   prototype/gdn_replay_fp8_reference.py:40-106
 *   gdnr_dequantize_vblock32 <- dequantize_checkpoint prototype/gdn_replay_fp8_reference.py:109-134
 *   gdnr_fused_step      <- gdn_prep_ring + gdn_replay_fp8 (+ flush) as one call, the
 *                          full-contract step of prototype/bench_gdn_full_contract.py:138-308
 *
 * Geometry supported by the kernels: K = V = 128 (Qwen3.5 GDN head dims),
 * HV = G*H with G in {1,2,4}, ring length L in [1, 64], one scale per
 * 32 value rows ("vblock32").
 */
#ifndef GDNR_H
#define GDNR_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GDNR_ABI_VERSION 2 /* 2: adds gdnr_packed_decode (the other structs are unchanged) */

typedef enum {
  GDNR_DT_NONE = 0,
  GDNR_F32 = 1,
  GDNR_F16 = 2,
  GDNR_BF16 = 3,
  GDNR_E4M3 = 4, /* float8_e4m3fn, one byte */
  GDNR_I32 = 5,
  GDNR_U8 = 6,   /* torch.bool / uint8 */
  GDNR_I8 = 7
} gdnr_dtype;

typedef enum {
  GDNR_OK = 0,
  GDNR_ERR_ARG = -1,         /* null pointer, wrong rank, inconsistent shapes */
  GDNR_ERR_DTYPE = -2,       /* unsupported dtype for that argument */
  GDNR_ERR_LAYOUT = -3,      /* stride / 16-byte alignment requirement not met */
  GDNR_ERR_ALIAS = -4,       /* two buffers that must be distinct overlap */
  GDNR_ERR_UNSUPPORTED = -5, /* geometry outside what the kernels implement */
  GDNR_ERR_CUDA = -6         /* launch failed (message has the CUDA error) */
} gdnr_status;

/* Bits of the device error word (see error_flag below). */
#define GDNR_DEVERR_WAIT_TIMEOUT 0x1u /* a bounded mbarrier wait gave up */
#define GDNR_DEVERR_BAD_POS 0x2u      /* fused step: pos[b] outside [0, L) */
#define GDNR_DEVERR_BAD_HINT 0x4u     /* flush_hint NONE but a sequence's ring was full */
#define GDNR_DEVERR_BAD_SLOT 0x8u     /* packed decode: state_indices[i] >= slots */
#define GDNR_DEVERR_LAYOUT 0x10u      /* a kernel's shared memory did not fit its layout (a launch
                                         configuration fault of the library): nothing was done */

/* flush_hint: what the caller knows about which sequences flush in this call */
#define GDNR_FLUSH_AUTO 0 /* unknown: every head is checked on the device */
#define GDNR_FLUSH_NONE 1 /* no sequence flushes (a full ring is reported as GDNR_DEVERR_BAD_HINT) */
#define GDNR_FLUSH_ALL 2  /* every sequence may flush */

/* launch_flags */
#define GDNR_LAUNCH_PDL 0x1 /* programmatic dependent launch: the kernel may start while the
                               preceding kernel on the stream drains and read this call's
                               checkpoint before that kernel completes.  Only valid when the
                               preceding kernel does not write this call's checkpoint. */

/* Strided view of a device (or, for validation only, any) buffer. */
typedef struct {
  void* data;
  int32_t dtype; /* gdnr_dtype */
  int32_t ndim;  /* 0 = absent (optional argument) */
  int64_t shape[4];
  int64_t stride[4]; /* in elements */
} gdnr_tensor;

/* ---- gdnr_replay: mirror of gdn_replay_fp8 ---------------------------- */
typedef struct {
  gdnr_tensor checkpoint; /* [B,HV,V,K] E4M3, I8 ("vblock_int8" codes, L <= 16; the flush
                             re-quantises to I8), or F32 for the full-precision variant; in/out */
  gdnr_tensor scale;      /* [B,HV,V/32] F16|F32 (absent for an F32 checkpoint); in/out */
  gdnr_tensor q;          /* [B,H,K] BF16|F32, already L2-normalised */
  gdnr_tensor k_ring;     /* [B,L,H,K] BF16 */
  gdnr_tensor v_ring;     /* [B,L,HV,V] BF16 */
  gdnr_tensor g_ring;     /* [B,L,HV] F32|BF16 (log decay) */
  gdnr_tensor beta_ring;  /* [B,L,HV] F32|BF16 */
  gdnr_tensor valid_len;  /* [B] I32: slots 0..valid_len-1 are replayed (clamped to [0,L]) */
  gdnr_tensor flush;      /* [B] U8|I32: nonzero -> rebuild + re-quantise in place */
  gdnr_tensor out;        /* [B,HV,V] BF16|F32 */
  int32_t block_v;        /* value rows per CTA: 32, 64 or 128 (0 -> 128) */
  int32_t quant_divisor;  /* 0: x/(amax/448) like ref.py:94; 1: x/fp16(amax/448) like kern.py:234 */
  uint32_t* error_flag;   /* optional device word, OR-ed with GDNR_DEVERR_* */
  int32_t flush_hint;     /* GDNR_FLUSH_* */
  int32_t launch_flags;   /* GDNR_LAUNCH_* */
} gdnr_replay_args;

int gdnr_replay(const gdnr_replay_args* args, void* stream);

/* ---- gdnr_replay_split: mirror of gdn_replay_fp8_split ----------------- */
typedef struct {
  gdnr_tensor checkpoint, scale, q, k_ring, v_ring, g_ring, beta_ring, valid_len;
  gdnr_tensor tq;   /* [B,HV,K] F32 caller buffer: receives the transformed query */
  gdnr_tensor coef; /* [B,HV,L] F32 caller buffer: receives c_t for t < valid_len */
  gdnr_tensor out;  /* [B,HV,V] BF16|F32 */
  int32_t block_v;
  uint32_t* error_flag;
} gdnr_replay_split_args;

int gdnr_replay_split(const gdnr_replay_split_args* args, void* stream);

/* ---- gdnr_replay_split_static: gdnr_replay_split without caller scratch --
 * No counterpart in the reference.  The split replay needs T [B,HV,K] and
 * c [B,HV,L] scratch; this entry point keeps them in a library-owned device
 * array instead, for callers that cannot allocate device memory when they
 * call the replay (e.g. a serving runtime that reserves all device memory for
 * its state pool up front, or code inside an allocator callback that must not
 * re-enter the allocator).  It allocates nothing.
 *
 * Limits: B*HV <= GDNR_SPLIT_STATIC_MAX_PAIRS and L <= GDNR_SPLIT_STATIC_MAX_L
 * (3 MiB of scratch per device); larger calls fail with GDNR_ERR_UNSUPPORTED.
 * The first call on a device looks up the scratch address (cudaGetSymbolAddress,
 * with that device current) and caches it: make that first call before any
 * stream capture.  All calls on a device share the one scratch, so calls that
 * overlap in time (concurrent streams or host threads) race on it; serialise
 * them.  Nothing in the scratch needs to start at zero. */
#define GDNR_SPLIT_STATIC_MAX_PAIRS 4096
#define GDNR_SPLIT_STATIC_MAX_L 64
typedef struct {
  gdnr_tensor checkpoint, scale, q, k_ring, v_ring, g_ring, beta_ring, valid_len; /* as gdnr_replay_split */
  gdnr_tensor out;
  int32_t block_v;
  uint32_t* error_flag;
} gdnr_replay_split_static_args;

int gdnr_replay_split_static(const gdnr_replay_split_static_args* args, void* stream);

/* ---- gdnr_prep_ring: mirror of gdn_prep_ring --------------------------- */
typedef struct {
  gdnr_tensor mixed_qkv; /* [B, 2*H*K + HV*V] BF16|F32, inner stride 1 */
  gdnr_tensor a, b;      /* [B,HV] BF16|F32 */
  gdnr_tensor a_log;     /* [HV] F32 */
  gdnr_tensor dt_bias;   /* [HV] F32 */
  gdnr_tensor pos;       /* [B] I32 ring slot written */
  gdnr_tensor q_out;     /* [B,H,K] BF16|F32 */
  gdnr_tensor k_ring, v_ring, g_ring, beta_ring;
  uint32_t* error_flag;
} gdnr_prep_args;

int gdnr_prep_ring(const gdnr_prep_args* args, void* stream);

/* ---- gdnr_fused_step: prep + ring append + replay + flush, one launch -- */
typedef struct {
  gdnr_tensor mixed_qkv, a, b, a_log, dt_bias; /* as gdnr_prep_args */
  gdnr_tensor pos;        /* [B] I32: slot of this token; the step flushes when pos == L-1 */
  gdnr_tensor pos_out;    /* optional [B] I32 (distinct from pos): receives (pos+1) % L */
  gdnr_tensor checkpoint; /* [B,HV,V,K] E4M3 | I8 (L <= 16) | F32, in/out */
  gdnr_tensor scale;      /* [B,HV,V/32] F16|F32 (absent for F32 checkpoint), in/out */
  gdnr_tensor k_ring, v_ring, g_ring, beta_ring; /* in/out: slot pos is written */
  gdnr_tensor out;        /* [B,HV,V] BF16|F32 */
  gdnr_tensor q_out;      /* optional [B,H,K]: normalised q as the reference's prep writes it */
  int32_t quant_divisor;
  uint32_t* error_flag;
  int32_t flush_hint;     /* GDNR_FLUSH_* */
  int32_t launch_flags;   /* GDNR_LAUNCH_* */
} gdnr_step_args;

int gdnr_fused_step(const gdnr_step_args* args, void* stream);

/* ---- gdnr_packed_decode: the production decode call over a state-slot pool --
 * Replaces the serving engine's decode call
 *   fused_recurrent_gated_delta_rule_packed_decode(mixed_qkv, a, b, A_log, dt_bias, scale,
 *       initial_state, out, ssm_state_indices, use_qk_l2norm_in_kernel=True)
 * as the reference drives it (prototype/bench_gdn_full_contract.py:157-170; contract notes
 * findings.md:37-45), with the bf16 state cache [slots,HV,V,K] replaced by the FP8
 * checkpoint + ring pool below: batch row i uses slot state_indices[i] of every state
 * tensor.  An index <= 0 is the null slot (the serving engine's padding; the production
 * kernel's NULL_BLOCK_ID test, vLLM fused_recurrent.py:292-297): no state is read or written
 * for that row and its out rows are written as zeros, as the production op does.  An index
 * >= slots is treated the same way and reported as GDNR_DEVERR_BAD_SLOT.  The non-null
 * indices of one call must be distinct (one row per sequence, as in the production
 * contract): two rows on one slot race on its state within the launch and the result is
 * undefined; nothing checks for it.  q and k are
 * always L2-normalised in the kernel and the output is scaled by K^-1/2: the production
 * call's use_qk_l2norm_in_kernel and scale arguments must be 1 and K^-1/2.  The step is
 * gdnr_fused_step's (prep + ring append + replay, and the flush when a slot's pos is L-1);
 * pos_out (optional, [slots]) receives (pos+1) % L for the slots of the batch.  E4M3
 * checkpoints only, in the layout gdnr_fused_step's persistent kernel takes (16-byte
 * aligned rows and rings, HV/H = 1 or even, 4 <= L <= 16); anything else fails with
 * GDNR_ERR_UNSUPPORTED. */
typedef struct {
  gdnr_tensor mixed_qkv, a, b, a_log, dt_bias; /* [B,...] as gdnr_step_args */
  gdnr_tensor state_indices; /* [B] I32: slot of each batch row */
  gdnr_tensor pos;        /* [slots] I32: ring slot of this token, per state slot */
  gdnr_tensor pos_out;    /* optional [slots] I32 (distinct from pos) */
  gdnr_tensor checkpoint; /* [slots,HV,V,K] E4M3, in/out */
  gdnr_tensor scale;      /* [slots,HV,V/32] F16|F32, in/out */
  gdnr_tensor k_ring, v_ring, g_ring, beta_ring; /* [slots,L,...] in/out */
  gdnr_tensor out;        /* [B,HV,V] or [B,1,HV,V] BF16|F32 */
  float qk_scale;         /* must be K^-1/2 */
  int32_t use_qk_l2norm;  /* must be 1 */
  int32_t quant_divisor;
  uint32_t* error_flag;
  int32_t flush_hint;     /* GDNR_FLUSH_* */
  int32_t launch_flags;   /* GDNR_LAUNCH_*; GDNR_LAUNCH_PDL is accepted, but the early
                             checkpoint requests wait for griddepcontrol.wait here (the
                             slots come from state_indices, an input) */
} gdnr_packed_decode_args;

int gdnr_packed_decode(const gdnr_packed_decode_args* args, void* stream);

/* ---- FP8 vblock32 codec ------------------------------------------------ */
typedef struct {
  gdnr_tensor state;      /* [B,HV,V,K] F32 (quantize: in; dequantize: out) */
  gdnr_tensor payload;    /* [B,HV,V,K] E4M3 */
  gdnr_tensor scale;      /* [B,HV,V/32] F16|F32 */
  int32_t quant_divisor;  /* as gdnr_replay_args */
  uint32_t* saturation_count; /* optional device counter: += #{|x/divisor| > 448} */
} gdnr_codec_args;

int gdnr_quantize_vblock32(const gdnr_codec_args* args, void* stream);
int gdnr_dequantize_vblock32(const gdnr_codec_args* args, void* stream);

/* ---- gdnr_bf16_step: mirror of gdn_bf16_step (bf16 state RMW control) -- */
typedef struct {
  gdnr_tensor state; /* [B,HV,V,K] BF16, in/out */
  gdnr_tensor q, k;  /* [B,H,K] BF16|F32 */
  gdnr_tensor v;     /* [B,HV,V] BF16|F32 */
  gdnr_tensor g, beta; /* [B,HV] BF16|F32 */
  gdnr_tensor out;   /* [B,HV,V] BF16|F32 */
} gdnr_bf16_step_args;

int gdnr_bf16_step(const gdnr_bf16_step_args* args, void* stream);

/* ---- misc --------------------------------------------------------------- */
const char* gdnr_last_error(void);
const char* gdnr_version(void);
int gdnr_abi_version(void);
/* Library-owned device error word used when a call passes error_flag = NULL.
 * Reads it (synchronously, on the current device) and optionally clears it. */
int gdnr_read_device_error(uint32_t* value, int clear);

/* Diagnostic, no counterpart in the reference: one tiny launch that runs the
 * persistent step kernel's bounded-wait code into its time limit (a barrier
 * nothing arrives on, held with 32 tensor-memory columns allocated) and
 * returns cleanly.  After it completes (about one second of GPU time), the
 * error word has GDNR_DEVERR_WAIT_TIMEOUT set and report (device memory,
 * 4 x u64) holds: both waits' results (0 = gave up), then the nanoseconds
 * each waited; the second wait ends through the abort word the first one set.
 * Used by the tests to show that a timed-out wait leaves the context usable. */
int gdnr_selftest_wait_timeout(uint32_t* error_flag, unsigned long long* report, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GDNR_H */
