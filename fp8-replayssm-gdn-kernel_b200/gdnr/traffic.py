"""Algorithmic HBM bytes of one decode step (the roofline's numerator).

Every tensor the step must touch is counted once, at its storage width: the
FP8 checkpoint and its vblock32 scales, the ring slots replayed, this token's
raw inputs, the ring append, the output, and on a flush the checkpoint and
scale write.  Key-ring bytes are counted per key head (the value heads of a
key head share its ring).  This is the byte accounting of the reference's
benchmark (prototype/bench_gdn_replayssm.py:45-87) extended to the fused
full-contract step (prep + append + replay + flush).
"""

from __future__ import annotations

KD = VD = 128


def step_bytes(batch: int, ring_fill: int, ring_len: int, heads: int = 16, value_heads: int = 32,
               scale_bytes: int = 4, gate_bytes: int = 4, ab_bytes: int = 2, out_bytes: int = 2,
               fused: bool = True) -> int:
    """Bytes of one launch over ``batch`` sequences.

    ``fused``: the full-contract step of a token that lands in ring slot
    ``ring_fill - 1`` (the launch at ``ring_fill == ring_len`` flushes).
    Otherwise the core replay of a ring that already holds ``ring_fill`` slots
    (query given, no append, no flush).
    """
    ck = batch * value_heads * VD * KD
    sc = batch * value_heads * (VD // 32) * scale_bytes
    slot = batch * (heads * KD * 2 + value_heads * VD * 2 + value_heads * 2 * gate_bytes)
    out = batch * value_heads * VD * out_bytes
    if not fused:
        return ck + sc + batch * heads * KD * 2 + ring_fill * slot + out
    raw = batch * ((2 * heads * KD + value_heads * VD) * 2 + value_heads * 2 * ab_bytes) + value_heads * 2 * 4
    total = raw + ck + sc + ring_fill * slot + out
    if ring_fill == ring_len:
        total += ck + sc
    return total


def cycle_bytes(batch: int, ring_len: int, **kw) -> float:
    """Mean bytes per launch over one ring cycle (fills 1..L, the flush included)."""
    return sum(step_bytes(batch, n, ring_len, **kw) for n in range(1, ring_len + 1)) / ring_len


def state_bytes(batch: int, ring_len: int, heads: int = 16, value_heads: int = 32, scale_bytes: int = 4,
                gate_bytes: int = 4) -> int:
    """Resident decode state of ``batch`` sequences of one layer."""
    return batch * (value_heads * VD * KD + value_heads * (VD // 32) * scale_bytes +
                    ring_len * (heads * KD * 2 + value_heads * VD * 2 + value_heads * 2 * gate_bytes) + 4)
