"""Timed CPU baseline: the oracle port of the reference's replay chain.

TEST INFRASTRUCTURE / BASELINE ONLY -- used by ``bench.py``'s CPU-baseline
leg and ``--impl reference`` arm, never by the product path.

One *unit* is one full-contract decode step of one sequence of one GDN layer
(H=16, HV=32, K=V=128): prep of the raw token, ring append, replay from the
dequantised FP8 checkpoint over the ring (the O(n.V.K) per-token recurrence
of ``replay_decode``, ref.py:189-244) and, when the ring is full, the
vblock32 re-quantisation.  Each worker process owns one sequence state and
walks it through its ring cycle, so a sample of units covers ring fills
1..L (and the flush) in proportion.
"""

from __future__ import annotations

import os
import time

import numpy as np

from . import gdn_oracle as O

_STATE = {}


def _init(seed: int, ring_len: int, heads: int = 16, value_heads: int = 32, dim: int = 128) -> None:
    rng = np.random.default_rng(seed)
    s0 = (0.02 * rng.standard_normal((1, value_heads, dim, dim))).astype(np.float32)
    q0 = O.quantize_checkpoint(s0, "vblock", 32)
    st = O.RingState(q0.payload, q0.scale, np.zeros((1, ring_len, heads, dim), np.float32),
                     np.zeros((1, ring_len, value_heads, dim), np.float32), np.zeros((1, ring_len, value_heads), np.float32),
                     np.zeros((1, ring_len, value_heads), np.float32))
    _STATE.update(rng=rng, st=st, pos=0, L=ring_len, H=heads, HV=value_heads, D=dim,
                  a_log=np.log(rng.uniform(1, 16, value_heads)).astype(np.float32),
                  dt_bias=(0.5 * rng.standard_normal(value_heads)).astype(np.float32))


def worker_init(seed: int, ring_len: int) -> None:
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    _init(seed + os.getpid() % 9973, ring_len)


def run_units(n: int) -> tuple[int, float]:
    """Run ``n`` units in this process; returns (units, seconds)."""
    s = _STATE
    t0 = time.perf_counter()
    for _ in range(n):
        rng = s["rng"]
        width = 2 * s["H"] * s["D"] + s["HV"] * s["D"]
        mixed = O.bf16_round(rng.standard_normal((1, width)).astype(np.float32))
        a = O.bf16_round(rng.standard_normal((1, s["HV"])).astype(np.float32))
        b = O.bf16_round(rng.standard_normal((1, s["HV"])).astype(np.float32))
        O.fused_step(s["st"], mixed, a, b, s["a_log"], s["dt_bias"], np.array([s["pos"]]), s["H"], s["D"],
                     gate_dtype="f32")
        s["pos"] = (s["pos"] + 1) % s["L"]
    return n, time.perf_counter() - t0
