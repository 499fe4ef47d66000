"""numpy restatement of the reference's FP8-checkpoint replay GDN algorithm.

TEST INFRASTRUCTURE ONLY -- the checker for the CUDA path and the timed CPU
baseline.  The product package never imports this module.

Every function cites the reference line it restates (paths are relative to
the reference project zz774ever/fp8-replayssm-gdn-kernel):

* ``prototype/gdn_replay_fp8_reference.py`` -- codec, recurrence, replay chain
  (abbreviated ``ref.py`` below);
* ``prototype/gdn_replayssm_fp8_kernel.py`` -- prep stage and the backward
  replay form of the Triton kernel (abbreviated ``kern.py`` below).

Arithmetic is float32 throughout, like the reference (torch float32 on CPU).
Summation order differs from torch's, so float results agree to ~1e-6
relative; the FP8/fp16/bf16 codecs are bit-exact given identical inputs.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

__all__ = [
    "FP8_MAX",
    "INT8_MAX",
    "L2_EPS",
    "SOFTPLUS_THRESHOLD",
    "bf16_round",
    "bf16_bits",
    "bf16_from_bits",
    "fp16_round",
    "e4m3_encode",
    "e4m3_decode",
    "QuantizedCheckpoint",
    "safe_scale",
    "quantize_checkpoint",
    "dequantize_checkpoint",
    "run_kernel",
    "baseline_decode",
    "replay_decode",
    "replay_adjoint",
    "error_metrics",
    "relative_l2",
    "prep",
    "fused_step",
    "replay_step",
    "quantize_vblock32",
    "RingState",
    "algorithmic_bytes",
    "reference_traffic_bytes",
]

FP8_MAX = 448.0  # torch.finfo(torch.float8_e4m3fn).max, ref.py:17-18
INT8_MAX = 127.0  # ref.py:46
L2_EPS = 1e-6  # kern.py:756 (L2_EPS constexpr passed by gdn_prep_ring)
SOFTPLUS_THRESHOLD = 20.0  # kern.py:757

_F32 = np.float32


# --------------------------------------------------------------------------
# scalar codecs (bit-level restatements; RNE everywhere)
# --------------------------------------------------------------------------

def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit pattern, round-to-nearest-even, NaN kept quiet.

    This is what torch's ``.to(torch.bfloat16)`` (and Triton's store into a
    bf16 pointer) does to the q/k/v/g/beta values the reference writes.
    """
    x = np.ascontiguousarray(x, dtype=_F32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        r = np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)
    return r


def bf16_from_bits(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(_F32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (returned as float32)."""
    return bf16_from_bits(bf16_bits(x))


def fp16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> float16 (RNE, as torch ``.to(torch.float16)``)."""
    with np.errstate(over="ignore"):
        return np.asarray(x, _F32).astype(np.float16)


def _e4m3_table() -> np.ndarray:
    codes = np.arange(256, dtype=np.int64)
    sign = np.where(codes & 0x80, -1.0, 1.0)
    e = (codes >> 3) & 0xF
    m = codes & 0x7
    val = np.where(e == 0, m / 8.0 * 2.0**-6, (1.0 + m / 8.0) * 2.0 ** (e - 7.0))
    val = sign * val
    val[(codes & 0x7F) == 0x7F] = np.nan  # e4m3fn: only S.1111.111 is NaN
    return val.astype(_F32)


_E4M3_VALUES = _e4m3_table()


def e4m3_decode(codes: np.ndarray) -> np.ndarray:
    """float8_e4m3fn byte -> float32 value (exact)."""
    return _E4M3_VALUES[np.asarray(codes, np.uint8)]


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """float32 -> float8_e4m3fn byte with round-to-nearest-even.

    Restates the semantics of torch's ``.to(torch.float8_e4m3fn)`` used at
    ref.py:99 (the reference clamps to +-448 first, so the saturating edge
    never matters there):

    * |x| >= 2**-6 (normal range): round the 3-bit mantissa half-to-even,
      carrying into the exponent; anything that rounds past 448 becomes the
      NaN code 0x7F (e4m3fn has no infinity).
    * |x| < 2**-6: subnormal grid of 2**-9, rounded half-to-even.
    * NaN -> 0x7F with the input's sign bit (torch CPU produces 0xFF for the
      negative default NaN of ``0/0``; a GPU produces 0x7F).
    """
    x = np.ascontiguousarray(x, dtype=_F32)
    sign = ((x.view(np.uint32) >> 31).astype(np.uint8)) << 7
    a = np.abs(x.astype(np.float64))
    out = np.zeros(x.shape, dtype=np.uint8)

    normal = a >= 2.0**-6
    with np.errstate(all="ignore"):
        frac, ex = np.frexp(np.where(normal, a, 1.0))  # a = frac * 2**ex, frac in [0.5,1)
        e = ex.astype(np.int64) - 1
        mq = np.rint((frac * 2.0 - 1.0) * 8.0).astype(np.int64)  # half-to-even
        carry = mq == 8
        e = np.where(carry, e + 1, e)
        mq = np.where(carry, 0, mq)
        big = (e + 7 > 15) | ((e + 7 == 15) & (mq == 7)) | np.isinf(a)
        code_n = np.where(big, 0x7F, ((e + 7) << 3) | mq)
        code_d = np.rint(np.where(normal, 0.0, a) * 512.0).astype(np.int64)
    out = np.where(normal, code_n, code_d).astype(np.uint8)
    out = np.where(np.isnan(x), np.uint8(0x7F), out)
    return out | sign


# --------------------------------------------------------------------------
# checkpoint codec (ref.py:21-134)
# --------------------------------------------------------------------------

@dataclass
class QuantizedCheckpoint:
    """Mirror of ``QuantizedCheckpoint`` (ref.py:21-33).

    ``payload`` holds raw float8_e4m3fn bytes (uint8) or int8 codes;
    ``scale`` is float16 like the reference.
    """

    payload: np.ndarray
    scale: np.ndarray
    granularity: str
    tile_size: int
    saturation_fraction: float

    @property
    def storage_bytes(self) -> int:  # ref.py:29-33
        return int(self.payload.size * self.payload.itemsize + self.scale.size * self.scale.itemsize)


def safe_scale(amax: np.ndarray, quant_max: float) -> np.ndarray:
    """ref.py:36-37: amax/quant_max where amax > 0, else 1.0 (NaN amax -> 1.0)."""
    amax = np.asarray(amax, _F32)
    with np.errstate(invalid="ignore"):
        return np.where(amax > 0, amax / _F32(quant_max), _F32(1.0)).astype(_F32)


def _nan_amax(x: np.ndarray, axis) -> np.ndarray:
    # torch.amax propagates NaN; numpy's max does too.
    return np.max(np.abs(x), axis=axis, keepdims=True)


def quantize_checkpoint(state: np.ndarray, granularity: str, tile_size: int) -> QuantizedCheckpoint:
    """Restatement of ``quantize_checkpoint`` (ref.py:40-106).

    Note the reference's divisor: for ``tile`` and ``vblock`` the payload is
    ``x / (amax/448)`` with the *unrounded* float32 scale (ref.py:69, :86,
    :94), while the stored scale is that value rounded to float16 (ref.py:87,
    :91).  ``head`` and ``row`` divide by the float16-rounded scale
    (ref.py:92-93).
    """
    source = np.asarray(state, _F32)
    is_int8 = granularity.endswith("_int8")
    base = granularity[: -len("_int8")] if is_int8 else granularity
    qmax = INT8_MAX if is_int8 else FP8_MAX
    if base == "head":
        scale = safe_scale(_nan_amax(source, (-2, -1)), qmax)
        expanded = None
    elif base == "row":
        scale = safe_scale(_nan_amax(source, -1), qmax)
        expanded = None
    elif base == "tile":
        vd, kd = source.shape[-2:]
        if vd % tile_size or kd % tile_size:
            raise ValueError("tile granularity requires dimensions divisible by tile_size")
        blocks = source.reshape(*source.shape[:-2], vd // tile_size, tile_size, kd // tile_size, tile_size)
        bscale = safe_scale(_nan_amax(blocks, (-3, -1)), qmax)
        expanded = np.broadcast_to(bscale, blocks.shape).reshape(source.shape)
        scale = bscale.squeeze(-1).squeeze(-2)
    elif base == "vblock":
        vd, kd = source.shape[-2:]
        if vd % tile_size:
            raise ValueError("vblock granularity requires value_dim divisible by tile_size")
        blocks = source.reshape(*source.shape[:-2], vd // tile_size, tile_size, kd)
        bscale = safe_scale(_nan_amax(blocks, (-2, -1)), qmax)
        expanded = np.broadcast_to(bscale, blocks.shape).reshape(source.shape)
        scale = bscale.squeeze(-1).squeeze(-1)
    else:
        raise ValueError(f"unsupported granularity: {granularity}")
    scale16 = fp16_round(scale)
    if expanded is None:
        expanded = scale16.astype(_F32)
    with np.errstate(all="ignore"):
        normalized = (source / expanded.astype(_F32)).astype(_F32)
        saturation = float(np.mean(np.abs(normalized) > qmax))
        clamped = np.where(normalized > qmax, _F32(qmax), normalized)
        clamped = np.where(clamped < -qmax, _F32(-qmax), clamped)  # NaN passes, like torch.clamp
    if is_int8:
        with np.errstate(invalid="ignore"):
            payload = np.rint(clamped).astype(np.int8)
    else:
        payload = e4m3_encode(clamped)
    return QuantizedCheckpoint(payload, scale16, granularity, tile_size, saturation)


def dequantize_checkpoint(ckpt: QuantizedCheckpoint) -> np.ndarray:
    """Restatement of ``dequantize_checkpoint`` (ref.py:109-134)."""
    base = ckpt.granularity[: -len("_int8")] if ckpt.granularity.endswith("_int8") else ckpt.granularity
    if ckpt.payload.dtype == np.int8:
        values = ckpt.payload.astype(_F32)
    else:
        values = e4m3_decode(ckpt.payload)
    s = ckpt.scale.astype(_F32)
    ts = ckpt.tile_size
    if base in ("head", "row"):
        return (values * s).astype(_F32)
    vd, kd = values.shape[-2:]
    if base == "tile":
        blocks = values.reshape(*values.shape[:-2], vd // ts, ts, kd // ts, ts)
        return (blocks * s[..., :, None, :, None]).reshape(values.shape).astype(_F32)
    blocks = values.reshape(*values.shape[:-2], vd // ts, ts, kd)
    return (blocks * s[..., :, None, None]).reshape(values.shape).astype(_F32)


# --------------------------------------------------------------------------
# recurrence (ref.py:137-244)
# --------------------------------------------------------------------------

def run_kernel(state, q, k, v, g, beta):
    """Exact per-token GDN recurrence (ref.py:137-163).

    state [B,HV,V,K]; q,k [B,T,H,K]; v [B,T,HV,V]; g,beta [B,T,HV].
    Returns (outputs [B,T,HV,V], final state).  Per token::

        S = exp(g) * S; r = S k; S += beta (v - r) k^T; o = (S q) * K**-0.5
    """
    scratch = np.array(state, dtype=_F32, copy=True)
    hv_n = v.shape[2]
    group = hv_n // k.shape[2]
    scale = _F32(q.shape[-1] ** -0.5)
    outs = []
    for t in range(q.shape[1]):
        qt = np.repeat(np.asarray(q[:, t], _F32), group, axis=1)
        kt = np.repeat(np.asarray(k[:, t], _F32), group, axis=1)
        vt = np.asarray(v[:, t], _F32)
        decay = np.exp(np.asarray(g[:, t], _F32))[..., None, None]
        bt = np.asarray(beta[:, t], _F32)[..., None]
        scratch = scratch * decay
        retrieved = (scratch * kt[:, :, None, :]).sum(axis=-1, dtype=_F32)
        correction = (vt - retrieved) * bt
        scratch = scratch + correction[..., None] * kt[:, :, None, :]
        outs.append(((scratch * qt[:, :, None, :]).sum(axis=-1, dtype=_F32) * scale)[:, None])
    return np.concatenate(outs, axis=1).astype(_F32), scratch.astype(_F32)


def baseline_decode(initial_state, q, k, v, g, beta):
    """Per-token recurrence, one token per call (ref.py:166-186)."""
    state = np.array(initial_state, _F32, copy=True)
    outs = []
    for t in range(q.shape[1]):
        o, state = run_kernel(state, q[:, t:t + 1], k[:, t:t + 1], v[:, t:t + 1], g[:, t:t + 1], beta[:, t:t + 1])
        outs.append(o)
    return np.concatenate(outs, axis=1), state


def replay_decode(initial_state, q, k, v, g, beta, window, granularity, tile_size):
    """Replay chain with an optional quantised checkpoint (ref.py:189-244)."""
    checkpoint = np.array(initial_state, _F32, copy=True)
    quantized = quantize_checkpoint(checkpoint, granularity, tile_size) if granularity is not None else None
    max_sat = 0.0
    outs = []
    ring_start = 0
    reconstructed = checkpoint
    for t in range(q.shape[1]):
        if quantized is not None:
            checkpoint = dequantize_checkpoint(quantized)
        sl = slice(ring_start, t + 1)
        o, reconstructed = run_kernel(checkpoint, q[:, sl], k[:, sl], v[:, sl], g[:, sl], beta[:, sl])
        outs.append(o[:, -1:])
        if t - ring_start + 1 == window:
            checkpoint = reconstructed
            if granularity is not None:
                quantized = quantize_checkpoint(checkpoint, granularity, tile_size)
                max_sat = max(max_sat, quantized.saturation_fraction)
            ring_start = t + 1
    final_state = reconstructed
    if quantized is not None and ring_start == q.shape[1]:
        final_state = dequantize_checkpoint(quantized)
    ckpt_bytes = quantized.storage_bytes if quantized is not None else checkpoint.size * 4
    return np.concatenate(outs, axis=1), final_state, max_sat, ckpt_bytes


def replay_adjoint(state, q, k_ring, v_ring, g_ring, beta_ring, valid_len):
    """Backward ("adjoint") replay of the Triton kernel's non-flush branch.

    kern.py:121-176.  state [B,HV,V,K] (already dequantised); q [B,H,K];
    rings [B,L,...]; valid_len [B].  Per (b, hv)::

        T <- q; o <- 0
        for t = n-1 .. 0: c = beta_t (k_t . T); o += c v_t; T <- exp(g_t)(T - c k_t)
        o += S T;  o *= K**-0.5
    """
    state = np.asarray(state, _F32)
    b_n, hv_n, vd, kd = state.shape
    group = hv_n // k_ring.shape[2]
    out = np.zeros((b_n, hv_n, vd), _F32)
    scale = _F32(kd ** -0.5)
    for b in range(b_n):
        n = int(min(max(int(valid_len[b]), 0), k_ring.shape[1]))
        for hv in range(hv_n):
            h = hv // group
            tq = np.asarray(q[b, h], _F32).copy()
            o = np.zeros(vd, _F32)
            for t in range(n - 1, -1, -1):
                kt = np.asarray(k_ring[b, t, h], _F32)
                c = _F32(beta_ring[b, t, hv]) * np.dot(kt, tq).astype(_F32)
                o = o + c * np.asarray(v_ring[b, t, hv], _F32)
                tq = (np.exp(_F32(g_ring[b, t, hv])) * (tq - c * kt)).astype(_F32)
            o = o + state[b, hv] @ tq
            out[b, hv] = o * scale
    return out


def relative_l2(actual, expected) -> float:
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    return float(np.linalg.norm((a - e).ravel()) / max(np.linalg.norm(e.ravel()), 1e-12))


def error_metrics(actual, expected) -> dict[str, float]:
    """ref.py:247-259 (max/mean abs, relative L2, cosine)."""
    a = np.asarray(actual, np.float64).ravel()
    e = np.asarray(expected, np.float64).ravel()
    d = a - e
    cos = float(np.dot(a, e) / max(np.linalg.norm(a) * np.linalg.norm(e), 1e-8))
    return {
        "max_abs": float(np.abs(d).max()) if d.size else 0.0,
        "mean_abs": float(np.abs(d).mean()) if d.size else 0.0,
        "relative_l2": relative_l2(a, e),
        "cosine": cos,
    }


# --------------------------------------------------------------------------
# prep stage and the full-contract step (kern.py:453-795, bench_gdn_full_contract.py)
# --------------------------------------------------------------------------

def _store_round(x, dtype: str):
    if dtype == "bf16":
        return bf16_round(x)
    if dtype == "f32":
        return np.asarray(x, _F32)
    if dtype == "f16":
        return fp16_round(x).astype(_F32)
    raise ValueError(dtype)


def prep(mixed_qkv, a, b, a_log, dt_bias, heads: int, key_dim: int, value_heads: int, value_dim: int,
         q_dtype="bf16", k_dtype="bf16", v_dtype="bf16", gate_dtype="bf16"):
    """Restatement of ``_gdn_prep_fused_kernel`` (kern.py:453-576).

    mixed_qkv [B, 2*H*K + HV*V] holds raw q | k | v; a, b [B,HV];
    a_log, dt_bias [HV].  Returns q_out [B,H,K], k [B,H,K], v [B,HV,V],
    g [B,HV], beta [B,HV], each rounded to the dtype it is stored in::

        q, k <- x / sqrt(sum(x*x) + 1e-6)                 (kern.py:514-515)
        g    <- -exp(A_log) * (x <= 20 ? log(1+exp(x)) : x),  x = a + dt_bias
        beta <- sigmoid(b)                                 (kern.py:558-561)
    """
    mixed = np.asarray(mixed_qkv, _F32)
    bsz = mixed.shape[0]
    hk = heads * key_dim
    q = mixed[:, :hk].reshape(bsz, heads, key_dim)
    k = mixed[:, hk:2 * hk].reshape(bsz, heads, key_dim)
    v = mixed[:, 2 * hk:2 * hk + value_heads * value_dim].reshape(bsz, value_heads, value_dim)
    eps = _F32(L2_EPS)
    qn = q / np.sqrt((q * q).sum(-1, dtype=_F32, keepdims=True) + eps)
    kn = k / np.sqrt((k * k).sum(-1, dtype=_F32, keepdims=True) + eps)
    x = np.asarray(a, _F32) + np.asarray(dt_bias, _F32)[None, :]
    with np.errstate(over="ignore"):
        sp = np.where(x <= _F32(SOFTPLUS_THRESHOLD), np.log(_F32(1.0) + np.exp(x)), x).astype(_F32)
        g = (-np.exp(np.asarray(a_log, _F32))[None, :] * sp).astype(_F32)
        beta = (_F32(1.0) / (_F32(1.0) + np.exp(-np.asarray(b, _F32)))).astype(_F32)
    return (
        _store_round(qn, q_dtype),
        _store_round(kn, k_dtype),
        _store_round(v, v_dtype),
        _store_round(g, gate_dtype),
        _store_round(beta, gate_dtype),
    )


@dataclass
class RingState:
    """Persistent per-sequence state of the replay scheme (kern.py:344-405 args).

    payload [B,HV,V,K] e4m3 bytes, int8 codes (the 'vblock_int8' option) or
    float32 for the full-precision variant; scale [B,HV,V/32] float16 (None
    for float32); rings
    k [B,L,H,K], v [B,L,HV,V], g/beta [B,L,HV] as float32 arrays holding
    values already rounded to their storage dtype.
    """

    payload: np.ndarray
    scale: np.ndarray | None
    k_ring: np.ndarray
    v_ring: np.ndarray
    g_ring: np.ndarray
    beta_ring: np.ndarray

    def copy(self) -> "RingState":
        return RingState(*(None if x is None else x.copy() for x in
                           (self.payload, self.scale, self.k_ring, self.v_ring, self.g_ring, self.beta_ring)))

    def dequantized(self) -> np.ndarray:
        if self.scale is None:
            return np.asarray(self.payload, _F32)
        return dequantize_checkpoint(QuantizedCheckpoint(self.payload, self.scale, "vblock", 32, 0.0))


def replay_step(st: RingState, qn, pos, out_dtype="bf16", quant_divisor="oracle"):
    """Replay half of one full-contract step, on a ring that already holds
    this token in slot ``pos`` (mutates ``st`` on flush); returns out.

    Output = exact recurrence from the dequantised checkpoint over slots
    ``0..pos`` read out with ``qn`` (ref.py:137-163, :208-219); when
    ``pos == L-1`` the rebuilt state is re-quantised in place (ref.py:220-229).
    """
    value_heads, value_dim = st.v_ring.shape[2], st.v_ring.shape[3]
    ring_len = st.k_ring.shape[1]
    bsz = qn.shape[0]
    out = np.zeros((bsz, value_heads, value_dim), _F32)
    for i in range(bsz):
        n = int(pos[i]) + 1
        sl = slice(i, i + 1)
        if st.scale is None:
            s0 = np.asarray(st.payload[sl], _F32)
        else:
            s0 = dequantize_checkpoint(QuantizedCheckpoint(st.payload[sl], st.scale[sl], "vblock", 32, 0.0))
        qrep = np.repeat(np.asarray(qn[sl], _F32)[:, None], n, axis=1)
        o, s_new = run_kernel(s0, qrep, st.k_ring[sl, :n], st.v_ring[sl, :n], st.g_ring[sl, :n], st.beta_ring[sl, :n])
        out[i] = o[0, -1]
        if n == ring_len:
            if st.scale is None:
                st.payload[i] = s_new[0]
            else:
                # an int8 payload stays int8 (the 'vblock_int8' codec, ref.py:44-47, :96-97)
                qc = quantize_vblock32(s_new, divisor=quant_divisor, int8=st.payload.dtype == np.int8)
                st.payload[i] = qc.payload[0]
                st.scale[i] = qc.scale[0]
    return _store_round(out, out_dtype)


def fused_step(st: RingState, mixed_qkv, a, b, a_log, dt_bias, pos, heads, key_dim,
               out_dtype="bf16", gate_dtype="bf16", quant_divisor="oracle"):
    """One full-contract decode step on ``st`` (mutated in place); returns (out, q_out).

    Semantics of the reference's cycle (bench_gdn_full_contract.py:138-154,
    :225-308 and ref.py:189-244): prep writes ring slot ``pos``; the output
    is the exact recurrence from the dequantised checkpoint over slots
    ``0..pos`` read out with this token's q; when ``pos == L-1`` the ring is
    full and the rebuilt state is re-quantised in place (vblock32).

    ``quant_divisor='oracle'`` divides by the unrounded scale (ref.py:94);
    ``'rounded'`` divides by the float16-rounded one like the Triton flush
    (kern.py:231-236).
    """
    value_heads, value_dim = st.v_ring.shape[2], st.v_ring.shape[3]
    qn, kn, v, g, beta = prep(mixed_qkv, a, b, a_log, dt_bias, heads, key_dim, value_heads, value_dim,
                              gate_dtype=gate_dtype)
    for i in range(qn.shape[0]):
        p = int(pos[i])
        st.k_ring[i, p] = kn[i]
        st.v_ring[i, p] = v[i]
        st.g_ring[i, p] = g[i]
        st.beta_ring[i, p] = beta[i]
    return replay_step(st, qn, pos, out_dtype, quant_divisor), qn


def quantize_vblock32(state, divisor="oracle", int8=False) -> QuantizedCheckpoint:
    """vblock32 quantiser (FP8 E4M3, or int8 with ``int8``) with a selectable
    divisor convention.

    ``divisor='oracle'`` is exactly ``quantize_checkpoint(state,'vblock',32)``
    (``'vblock_int8'`` with ``int8``, ref.py:44-47, :96-97); ``'rounded'``
    divides by float32(float16(scale)) as kern.py:231-236 does (but keeps the
    oracle's amax==0 -> 1.0 rule of ref.py:36-37).
    """
    gran = "vblock_int8" if int8 else "vblock"
    if divisor == "oracle":
        return quantize_checkpoint(state, gran, 32)
    qmax = INT8_MAX if int8 else FP8_MAX
    source = np.asarray(state, _F32)
    vd, kd = source.shape[-2:]
    blocks = source.reshape(*source.shape[:-2], vd // 32, 32, kd)
    s16 = fp16_round(safe_scale(_nan_amax(blocks, (-2, -1)), qmax))
    with np.errstate(all="ignore"):
        normalized = (blocks / s16.astype(_F32)).astype(_F32)
        sat = float(np.mean(np.abs(normalized) > qmax))
        c = np.where(normalized > qmax, _F32(qmax), normalized)
        c = np.where(c < -qmax, _F32(-qmax), c)
    if int8:
        with np.errstate(invalid="ignore"):
            payload = np.rint(c).astype(np.int8).reshape(source.shape)
    else:
        payload = e4m3_encode(c).reshape(source.shape)
    return QuantizedCheckpoint(payload, s16.squeeze(-1).squeeze(-1), gran, 32, sat)


# --------------------------------------------------------------------------
# byte accounting
# --------------------------------------------------------------------------

def reference_traffic_bytes(batch, window, heads, value_heads, key_dim, value_dim, block_v):
    """The reference's byte model (prototype/bench_gdn_replayssm.py:45-87)."""
    tiles = value_dim // block_v
    checkpoint = batch * value_heads * value_dim * key_dim
    scales = batch * value_heads * tiles * 2
    query = batch * heads * key_dim * 2
    ring_key = batch * window * heads * key_dim * 2
    ring_value = batch * window * value_heads * value_dim * 2
    ring_scalars = batch * window * value_heads * 4
    return {
        "replay_logical": checkpoint + scales + query + ring_key + ring_value + ring_scalars,
        "replay_actual": checkpoint + scales + tiles * (query + ring_key) + ring_value + ring_scalars,
        "flush_actual": 2 * checkpoint + 2 * scales + tiles * ring_key + ring_value + ring_scalars,
        "bf16_baseline": batch * value_heads * value_dim * key_dim * 4,
    }


def algorithmic_bytes(batch, ring_fill, ring_len, heads=16, value_heads=32, key_dim=128, value_dim=128,
                      scale_bytes=2, gate_bytes=4, ab_bytes=2, out_bytes=2, fused=True):
    """Unique bytes one decode step must move (each tensor counted once).

    ``fused=True``: one full-contract fused step at ring fill ``ring_fill``
    (1..ring_len; the step at fill == ring_len flushes).  ``fused=False``:
    the core replay of a ring already holding ``ring_fill`` slots.
    """
    ckpt = batch * value_heads * value_dim * key_dim
    scales = batch * value_heads * (value_dim // 32) * scale_bytes
    k_slot = batch * heads * key_dim * 2
    v_slot = batch * value_heads * value_dim * 2
    gb_slot = batch * value_heads * 2 * gate_bytes
    out = batch * value_heads * value_dim * out_bytes
    if not fused:
        q = batch * heads * key_dim * 2
        return ckpt + scales + q + ring_fill * (k_slot + v_slot + gb_slot) + out
    mixed = batch * (2 * heads * key_dim + value_heads * value_dim) * 2
    ab = batch * value_heads * 2 * ab_bytes
    params = value_heads * 2 * 4
    prev = (ring_fill - 1) * (k_slot + v_slot + gb_slot)
    append = k_slot + v_slot + gb_slot
    total = mixed + ab + params + ckpt + scales + prev + append + out
    if ring_fill == ring_len:
        total += ckpt + scales
    return total
