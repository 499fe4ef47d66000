"""Operator API -- drop-in mirror of the reference prototype's call contract.

Same names, argument order, argument meaning and in-place side effects as
``prototype/gdn_replayssm_fp8_kernel.py`` (zz774ever/fp8-replayssm-gdn-kernel):

* :func:`gdn_replay_fp8`        <- ``gdn_replay_fp8``        (:344-405)
* :func:`gdn_replay_fp8_split`  <- ``gdn_replay_fp8_split``  (:1129-1235)
* :func:`gdn_prep_ring`         <- ``gdn_prep_ring``         (:710-795)
* :func:`gdn_bf16_step`         <- ``gdn_bf16_step``         (:408-450)

plus the fused full-contract step (:func:`gdn_fused_step`, prep + replay +
flush in one launch) and the GPU vblock32 codec (:func:`quantize_checkpoint`,
:func:`dequantize_checkpoint`, mirrors of
``prototype/gdn_replay_fp8_reference.py:40-134``).

All work runs in libgdnr (hand-written sm_100a CUDA) on the current torch
stream; nothing falls back to the CPU.  Triton-specific tuning knobs
(``num_warps``, ``num_stages``, ``block_kc``, ``precompute_grouped``,
``fused``) are accepted for signature compatibility and ignored.
Invalid arguments raise ``ValueError`` (``GdnrValueError``).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib

_DIVISOR = {"oracle": 0, "rounded": 1}


def _divisor(mode: str | int) -> int:
    if isinstance(mode, int):
        return mode
    try:
        return _DIVISOR[mode]
    except KeyError:
        raise ValueError(f"quant_divisor must be one of {sorted(_DIVISOR)}") from None


_FLUSH_HINT = {"auto": 0, "none": 1, "all": 2}
LAUNCH_PDL = 0x1


def _flush_hint(hint: str) -> int:
    try:
        return _FLUSH_HINT[hint]
    except KeyError:
        raise ValueError(f"flush_hint must be one of {sorted(_FLUSH_HINT)}") from None


def _as_bhv(out: torch.Tensor) -> torch.Tensor:
    # accept the production layout [B,1,HV,V] as well as [B,HV,V]
    if out.dim() == 4 and out.shape[1] == 1:
        return out.squeeze(1)
    return out


def _err_ptr(error_flag: torch.Tensor | None) -> int | None:
    if error_flag is None:
        return None
    if error_flag.dtype not in (torch.int32, torch.uint32) or error_flag.numel() < 1 or error_flag.device.type != "cuda":
        raise ValueError("error_flag must be a CUDA int32 tensor with at least one element")
    return error_flag.data_ptr()


def gdn_replay_fp8(
    checkpoint: torch.Tensor,
    checkpoint_scale: torch.Tensor | None,
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    g_cache: torch.Tensor,
    beta_cache: torch.Tensor,
    valid_len: torch.Tensor,
    flush: torch.Tensor,
    block_v: int = 32,
    num_warps: int = 4,
    out: torch.Tensor | None = None,
    quant_divisor: str = "oracle",
    error_flag: torch.Tensor | None = None,
    flush_hint: str = "auto",
    pdl: bool = False,
) -> torch.Tensor:
    """Replay (and, where ``flush[b]``, rebuild + re-quantise in place).

    checkpoint [B,HV,V,K] float8_e4m3fn, int8 (the "vblock_int8" option,
    rings of L <= 16) or float32 (full-precision variant),
    checkpoint_scale [B,HV,V/32] float16|float32, q [B,H,K], rings
    k [B,L,H,K] / v [B,L,HV,V] bf16, g/beta [B,L,HV], valid_len [B] int32,
    flush [B] bool.  Returns out [B,HV,V] in q's dtype unless ``out`` given.

    ``flush_hint`` -- what the caller knows about ``flush``: "auto" (nothing),
    "none" (no sequence flushes: one launch; a set flag is reported in the
    device error word as ``GDNR_DEVERR_BAD_HINT`` and that sequence is left
    unprocessed) or "all".  ``pdl`` launches with programmatic dependent
    launch; only valid when the preceding kernel on the stream does not write
    this call's checkpoint or scales.
    """
    del num_warps
    batch, _, _, _ = k_cache.shape
    value_heads, value_dim = v_cache.shape[2], v_cache.shape[3]
    if out is None:
        out = torch.empty(batch, value_heads, value_dim, dtype=q.dtype, device=q.device)
    args = _lib.ReplayArgs()
    args.checkpoint = _lib.tensor_desc(checkpoint)
    args.scale = _lib.tensor_desc(checkpoint_scale if checkpoint.dtype != torch.float32 else None)
    args.q = _lib.tensor_desc(q)
    args.k_ring = _lib.tensor_desc(k_cache)
    args.v_ring = _lib.tensor_desc(v_cache)
    args.g_ring = _lib.tensor_desc(g_cache)
    args.beta_ring = _lib.tensor_desc(beta_cache)
    args.valid_len = _lib.tensor_desc(valid_len)
    args.flush = _lib.tensor_desc(flush)
    args.out = _lib.tensor_desc(_as_bhv(out))
    args.block_v = int(block_v)
    args.quant_divisor = _divisor(quant_divisor)
    args.error_flag = _err_ptr(error_flag)
    args.flush_hint = _flush_hint(flush_hint)
    args.launch_flags = LAUNCH_PDL if pdl else 0
    _lib.call("gdnr_replay", args, q.device)
    return out


def gdn_replay_fp8_split(
    checkpoint: torch.Tensor,
    checkpoint_scale: torch.Tensor,
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    g_cache: torch.Tensor,
    beta_cache: torch.Tensor,
    valid_len: torch.Tensor,
    transformed_query_buffer: torch.Tensor,
    coefficient_buffer: torch.Tensor,
    block_v: int = 32,
    num_warps: int = 4,
    block_kc: int = 128,
    precompute_grouped: bool = True,
    num_stages: int = 2,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Non-flush replay as precompute + apply (kern.py:1129-1235).

    ``transformed_query_buffer`` [B,HV,K] float32 and ``coefficient_buffer``
    [B,HV,L] float32 are caller-owned and receive T and c_t (t < valid_len).
    """
    del num_warps, block_kc, precompute_grouped, num_stages
    batch = k_cache.shape[0]
    value_heads, value_dim = v_cache.shape[2], v_cache.shape[3]
    if out is None:
        out = torch.empty(batch, value_heads, value_dim, dtype=q.dtype, device=q.device)
    args = _lib.ReplaySplitArgs()
    args.checkpoint = _lib.tensor_desc(checkpoint)
    args.scale = _lib.tensor_desc(checkpoint_scale)
    args.q = _lib.tensor_desc(q)
    args.k_ring = _lib.tensor_desc(k_cache)
    args.v_ring = _lib.tensor_desc(v_cache)
    args.g_ring = _lib.tensor_desc(g_cache)
    args.beta_ring = _lib.tensor_desc(beta_cache)
    args.valid_len = _lib.tensor_desc(valid_len)
    args.tq = _lib.tensor_desc(transformed_query_buffer)
    args.coef = _lib.tensor_desc(coefficient_buffer)
    args.out = _lib.tensor_desc(_as_bhv(out))
    args.block_v = int(block_v)
    _lib.call("gdnr_replay_split", args, q.device)
    return out


def gdn_replay_fp8_split_static(
    checkpoint: torch.Tensor,
    checkpoint_scale: torch.Tensor,
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    g_cache: torch.Tensor,
    beta_cache: torch.Tensor,
    valid_len: torch.Tensor,
    out: torch.Tensor,
    block_v: int = 32,
) -> torch.Tensor:
    """:func:`gdn_replay_fp8_split` without caller scratch (no reference counterpart).

    For callers that cannot allocate device memory when they call the replay:
    T and c live in a library-owned 3 MiB device array (B*HV <= 4096, L <= 64;
    larger calls raise), and ``out`` must be given.  The first call on a device
    sets the array up (make it before any stream capture); calls that overlap
    in time share the array and must be serialised.
    """
    args = _lib.ReplaySplitStaticArgs()
    args.checkpoint = _lib.tensor_desc(checkpoint)
    args.scale = _lib.tensor_desc(checkpoint_scale)
    args.q = _lib.tensor_desc(q)
    args.k_ring = _lib.tensor_desc(k_cache)
    args.v_ring = _lib.tensor_desc(v_cache)
    args.g_ring = _lib.tensor_desc(g_cache)
    args.beta_ring = _lib.tensor_desc(beta_cache)
    args.valid_len = _lib.tensor_desc(valid_len)
    args.out = _lib.tensor_desc(_as_bhv(out))
    args.block_v = int(block_v)
    _lib.call("gdnr_replay_split_static", args, q.device)
    return out


def gdn_prep_ring(
    mixed_qkv: torch.Tensor,
    a: torch.Tensor,
    b: torch.Tensor,
    a_log: torch.Tensor,
    dt_bias: torch.Tensor,
    pos: torch.Tensor,
    q_out: torch.Tensor,
    k_ring: torch.Tensor,
    v_ring: torch.Tensor,
    g_ring: torch.Tensor,
    beta_ring: torch.Tensor,
    num_warps: int = 1,
    fused: bool = True,
    error_flag: torch.Tensor | None = None,
) -> None:
    """q/k L2 norm, gating, ring append of slot ``pos[b]`` (kern.py:710-795)."""
    del num_warps, fused
    args = _lib.PrepArgs()
    for name, t in (("mixed_qkv", mixed_qkv), ("a", a), ("b", b), ("a_log", a_log), ("dt_bias", dt_bias),
                    ("pos", pos), ("q_out", q_out), ("k_ring", k_ring), ("v_ring", v_ring), ("g_ring", g_ring),
                    ("beta_ring", beta_ring)):
        setattr(args, name, _lib.tensor_desc(t))
    args.error_flag = _err_ptr(error_flag)
    _lib.call("gdnr_prep_ring", args, mixed_qkv.device)


def gdn_fused_step(
    mixed_qkv: torch.Tensor,
    a: torch.Tensor,
    b: torch.Tensor,
    a_log: torch.Tensor,
    dt_bias: torch.Tensor,
    pos: torch.Tensor,
    checkpoint: torch.Tensor,
    checkpoint_scale: torch.Tensor | None,
    k_ring: torch.Tensor,
    v_ring: torch.Tensor,
    g_ring: torch.Tensor,
    beta_ring: torch.Tensor,
    out: torch.Tensor | None = None,
    q_out: torch.Tensor | None = None,
    pos_out: torch.Tensor | None = None,
    quant_divisor: str = "oracle",
    error_flag: torch.Tensor | None = None,
    flush_hint: str = "auto",
    pdl: bool = False,
) -> torch.Tensor:
    """One full-contract decode step.

    Appends this token (prep of ``mixed_qkv``/``a``/``b``) to ring slot
    ``pos[b]``, replays slots ``0..pos[b]`` against the FP8 checkpoint, writes
    ``out`` [B,HV,V] (or [B,1,HV,V]), and when ``pos[b] == L-1`` rebuilds the
    state and re-quantises the checkpoint in place.  ``pos_out`` (optional,
    distinct from ``pos``) receives ``(pos+1) % L``.  The checkpoint is
    float8_e4m3fn, int8 (the "vblock_int8" option, L <= 16: re-quantised to
    int8 on a flush) or float32 (full precision, no scales).

    ``flush_hint``: "auto" (some sequences may be at ``L-1``: the
    flush-capable kernel decides per sequence on the device), "none" (no
    ``pos[b] == L-1``: the kernel without the flush path, the fastest when it
    holds; a violation is reported in the device error word as
    ``GDNR_DEVERR_BAD_HINT`` and that sequence is left unprocessed) or "all"
    (the flush-capable kernel, as "auto").  ``pdl`` as in
    :func:`gdn_replay_fp8`.
    """
    batch = mixed_qkv.shape[0]
    value_heads = v_ring.shape[2]
    if out is None:
        out = torch.empty(batch, value_heads, v_ring.shape[3], dtype=mixed_qkv.dtype, device=mixed_qkv.device)
    args = _lib.StepArgs()
    args.mixed_qkv = _lib.tensor_desc(mixed_qkv)
    args.a = _lib.tensor_desc(a)
    args.b = _lib.tensor_desc(b)
    args.a_log = _lib.tensor_desc(a_log)
    args.dt_bias = _lib.tensor_desc(dt_bias)
    args.pos = _lib.tensor_desc(pos)
    args.pos_out = _lib.tensor_desc(pos_out)
    args.checkpoint = _lib.tensor_desc(checkpoint)
    args.scale = _lib.tensor_desc(checkpoint_scale if checkpoint.dtype != torch.float32 else None)
    args.k_ring = _lib.tensor_desc(k_ring)
    args.v_ring = _lib.tensor_desc(v_ring)
    args.g_ring = _lib.tensor_desc(g_ring)
    args.beta_ring = _lib.tensor_desc(beta_ring)
    args.out = _lib.tensor_desc(_as_bhv(out))
    args.q_out = _lib.tensor_desc(q_out)
    args.quant_divisor = _divisor(quant_divisor)
    args.error_flag = _err_ptr(error_flag)
    args.flush_hint = _flush_hint(flush_hint)
    args.launch_flags = LAUNCH_PDL if pdl else 0
    _lib.call("gdnr_fused_step", args, mixed_qkv.device)
    return out


KEY_SCALE = 128 ** -0.5  # the output scale head_k_dim^-1/2 the kernels apply


def fused_recurrent_gated_delta_rule_packed_decode(
    mixed_qkv: torch.Tensor,
    a: torch.Tensor,
    b: torch.Tensor,
    A_log: torch.Tensor,
    dt_bias: torch.Tensor,
    scale: float,
    initial_state,
    out: torch.Tensor,
    ssm_state_indices: torch.Tensor,
    use_qk_l2norm_in_kernel: bool = True,
    *,
    quant_divisor: str = "oracle",
    error_flag: torch.Tensor | None = None,
    flush_hint: str = "auto",
    pdl: bool = False,
) -> torch.Tensor:
    """The serving engine's GDN decode call over a pool of FP8 replay states.

    Same arguments as the production operator the reference swaps out
    (``fused_recurrent_gated_delta_rule_packed_decode`` at vLLM's
    ``_forward_core_decode_non_spec`` call site; reference
    prototype/bench_gdn_full_contract.py:157-170, contract notes
    findings.md:37-45), except that ``initial_state`` is a
    :class:`gdnr.ReplayState` whose leading dimension is the slot pool instead
    of the bf16 state cache ``[slots, HV, V, K]``.  Batch row ``i`` runs one
    fused decode step (prep, ring append, replay, and the flush when the slot's
    ring position is ``L-1``) on slot ``ssm_state_indices[i]`` of every state
    tensor and advances that slot's ring position.  An index ``<= 0`` is the
    null slot (padding rows, the production kernel's ``NULL_BLOCK_ID`` test):
    no state is read or written for it and its ``out`` rows are set to zero,
    as the production op does; an index ``>= slots`` is treated the same way
    and reported in the device error word as ``GDNR_DEVERR_BAD_SLOT``.
    The non-null indices of one call must be distinct, as in the production
    contract (one batch row per sequence): two rows on the same slot would
    both read-modify-write that slot's checkpoint, rings and position in the
    same launch, and the result is undefined (nothing checks for it).
    ``out`` is ``[B, 1, HV, V]`` (or ``[B, HV, V]``).  q and k are always
    L2-normalised in the kernel and the output is scaled by ``K^-1/2``:
    ``use_qk_l2norm_in_kernel`` must be true and ``scale`` must be
    ``head_k_dim ** -0.5``.  The other keywords as in :func:`gdn_fused_step`.
    """
    if not use_qk_l2norm_in_kernel:
        raise _lib.GdnrValueError(_lib.ERR_UNSUPPORTED,
                                  "use_qk_l2norm_in_kernel must be True: the kernel always normalises q and k")
    if abs(float(scale) - KEY_SCALE) > 1e-6 * KEY_SCALE:
        raise _lib.GdnrValueError(_lib.ERR_UNSUPPORTED,
                                  f"scale must be head_k_dim ** -0.5 = {KEY_SCALE!r} (got {scale!r})")
    st = initial_state
    # the ring positions advance through a staging copy: the kernel reads
    # st.pos and writes the batch's slots of pos_next, then st.pos takes it
    pos_next = getattr(st, "_pos_next", None)
    if pos_next is None or pos_next.shape != st.pos.shape or pos_next.device != st.pos.device:
        pos_next = torch.empty_like(st.pos)
        st._pos_next = pos_next
    pos_next.copy_(st.pos)
    args = _lib.PackedDecodeArgs()
    for name, t in (("mixed_qkv", mixed_qkv), ("a", a), ("b", b), ("a_log", A_log), ("dt_bias", dt_bias),
                    ("state_indices", ssm_state_indices), ("pos", st.pos), ("pos_out", pos_next),
                    ("checkpoint", st.checkpoint), ("scale", st.scale), ("k_ring", st.k_ring), ("v_ring", st.v_ring),
                    ("g_ring", st.g_ring), ("beta_ring", st.beta_ring), ("out", out)):
        setattr(args, name, _lib.tensor_desc(t))
    args.qk_scale = float(scale)
    args.use_qk_l2norm = 1
    args.quant_divisor = _divisor(quant_divisor)
    args.error_flag = _err_ptr(error_flag)
    args.flush_hint = _flush_hint(flush_hint)
    args.launch_flags = LAUNCH_PDL if pdl else 0
    _lib.call("gdnr_packed_decode", args, mixed_qkv.device)
    st.pos.copy_(pos_next)
    return out


def gdn_bf16_step(state, q, k, v, g, beta) -> torch.Tensor:
    """One-token GDN step on a bf16 state, read-modify-write (kern.py:408-450)."""
    batch, value_heads, value_dim, _ = state.shape
    out = torch.empty(batch, value_heads, value_dim, dtype=q.dtype, device=q.device)
    args = _lib.Bf16StepArgs()
    for name, t in (("state", state), ("q", q), ("k", k), ("v", v), ("g", g), ("beta", beta), ("out", out)):
        setattr(args, name, _lib.tensor_desc(t))
    _lib.call("gdnr_bf16_step", args, q.device)
    return out


@dataclass
class QuantizedCheckpoint:
    """Mirror of ``QuantizedCheckpoint`` (ref.py:21-33), on the GPU."""

    payload: torch.Tensor
    scale: torch.Tensor
    granularity: str
    tile_size: int
    saturation_fraction: float

    @property
    def storage_bytes(self) -> int:
        return self.payload.numel() * self.payload.element_size() + self.scale.numel() * self.scale.element_size()


def quantize_checkpoint(
    state: torch.Tensor,
    granularity: str = "vblock",
    tile_size: int = 32,
    scale_dtype: torch.dtype = torch.float16,
    quant_divisor: str = "oracle",
    payload: torch.Tensor | None = None,
    scale: torch.Tensor | None = None,
    compute_saturation: bool = True,
) -> QuantizedCheckpoint:
    """GPU vblock32 quantiser, bit-exact with ``quantize_checkpoint(state, granularity, 32)``
    for ``granularity`` "vblock" (FP8 E4M3 payload) and "vblock_int8" (int8
    payload, scales amax/127; ref.py:44-47, :96-97).

    ``state`` [B,HV,V,K] float32 on CUDA.  ``compute_saturation`` reads the
    saturation count back (one synchronisation), like the reference's
    ``.item()`` at ref.py:95.  An int8 payload also runs through
    :func:`gdn_replay_fp8` and :func:`gdn_fused_step` (rings of L <= 16; the
    flush re-quantises it to int8); the packed decode and the split replay
    take E4M3 payloads only.
    """
    if granularity not in ("vblock", "vblock_int8") or tile_size != 32:
        raise ValueError("the GPU codec implements granularity 'vblock' / 'vblock_int8' with tile_size=32 only")
    int8 = granularity == "vblock_int8"
    state = state if state.dtype == torch.float32 else state.float()
    b, hv, v, k = state.shape
    if payload is None:
        payload = torch.empty(b, hv, v, k, dtype=torch.int8 if int8 else torch.float8_e4m3fn, device=state.device)
    if scale is None:
        scale = torch.empty(b, hv, v // 32, dtype=scale_dtype, device=state.device)
    sat = torch.zeros(1, dtype=torch.int32, device=state.device) if compute_saturation else None
    args = _lib.CodecArgs()
    args.state = _lib.tensor_desc(state)
    args.payload = _lib.tensor_desc(payload)
    args.scale = _lib.tensor_desc(scale)
    args.quant_divisor = _divisor(quant_divisor)
    args.saturation_count = sat.data_ptr() if sat is not None else None
    _lib.call("gdnr_quantize_vblock32", args, state.device)
    frac = float(sat.item()) / max(state.numel(), 1) if sat is not None else 0.0
    return QuantizedCheckpoint(payload, scale, granularity, 32, frac)


def dequantize_checkpoint(ckpt: QuantizedCheckpoint, out: torch.Tensor | None = None) -> torch.Tensor:
    """payload * scale[row/32] as float32 (ref.py:109-134), on the GPU (E4M3 or int8 payload)."""
    if ckpt.granularity not in ("vblock", "vblock_int8") or ckpt.tile_size != 32:
        raise ValueError("the GPU codec implements granularity 'vblock' / 'vblock_int8' with tile_size=32 only")
    if out is None:
        out = torch.empty(ckpt.payload.shape, dtype=torch.float32, device=ckpt.payload.device)
    args = _lib.CodecArgs()
    args.state = _lib.tensor_desc(out)
    args.payload = _lib.tensor_desc(ckpt.payload)
    args.scale = _lib.tensor_desc(ckpt.scale)
    _lib.call("gdnr_dequantize_vblock32", args, out.device)
    return out


def read_device_error(clear: bool = True) -> int:
    """Read (and clear) the library's default device error word (synchronous)."""
    v = ctypes.c_uint32(0)
    _lib.check(_lib.load().gdnr_read_device_error(ctypes.byref(v), int(clear)))
    return int(v.value)
