"""Seeded synthetic inputs with the reference's shapes and distributions.

The reference measures on synthetic inputs (and on a real Qwen3.5-4B decode
capture that is not shipped).  These generators reproduce its distributions:

* raw full-contract inputs (prototype/bench_gdn_full_contract.py:56-77):
  q, k, v ~ N(0,1) bf16 packed as ``mixed_qkv``; a, b ~ N(0,1);
  ``A_log = log U(1,16)`` and ``dt_bias ~ N(0,0.5)`` (the benchmark
  configuration's gate parameters); state ~ N(0, sigma) float32;
* core-replay rings (prototype/gdn_replayssm_fp8_kernel.py:1238-1289):
  normalised q/k bf16, v ~ N(0,1) bf16, gates from a/dt_bias, beta=sigmoid.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def raw_step_inputs(batch: int, steps: int, heads: int = 16, value_heads: int = 32, key_dim: int = 128,
                    value_dim: int = 128, seed: int = 0, device="cuda", ab_dtype=torch.bfloat16,
                    state_sigma: float = 0.02) -> dict:
    """Per-step raw inputs [B, steps, ...] plus gate parameters and an initial state."""
    g = _gen(seed, device)
    width = 2 * heads * key_dim + value_heads * value_dim
    mixed = torch.randn(batch, steps, width, generator=g, device=device).to(torch.bfloat16)
    a = torch.randn(batch, steps, value_heads, generator=g, device=device).to(ab_dtype)
    b = torch.randn(batch, steps, value_heads, generator=g, device=device).to(ab_dtype)
    a_log = torch.log(1.0 + 15.0 * torch.rand(value_heads, generator=g, device=device))
    dt_bias = 0.5 * torch.randn(value_heads, generator=g, device=device)
    state = state_sigma * torch.randn(batch, value_heads, value_dim, key_dim, generator=g, device=device)
    return {"mixed_qkv": mixed, "a": a, "b": b, "a_log": a_log.float(), "dt_bias": dt_bias.float(),
            "state": state.float()}


def drift_gate_inputs(batch: int, steps: int, value_heads: int = 32, seed: int = 0, device="cuda",
                      alpha_lo: float = 0.9, alpha_hi: float = 0.999) -> dict:
    """Gates with alpha = exp(g) ~ U(alpha_lo, alpha_hi): A_log = 0 and
    softplus(a + dt_bias) = -log(alpha) solved for a (dt_bias = 0)."""
    g = _gen(seed + 1, device)
    alpha = alpha_lo + (alpha_hi - alpha_lo) * torch.rand(batch, steps, value_heads, generator=g, device=device)
    y = -torch.log(alpha)  # softplus(x) = y  ->  x = log(expm1(y))
    a = torch.log(torch.expm1(y))
    return {"a": a.float(), "a_log": torch.zeros(value_heads, device=device),
            "dt_bias": torch.zeros(value_heads, device=device)}


def replay_ring_inputs(batch: int, ring_len: int, heads: int = 16, value_heads: int = 32, key_dim: int = 128,
                       value_dim: int = 128, seed: int = 0, device="cuda", gate_dtype=torch.float32,
                       state_sigma: float = 0.05) -> dict:
    """A full ring of already-prepped tokens (core replay)."""
    g = _gen(seed, device)
    bf = torch.bfloat16
    q = F.normalize(torch.randn(batch, heads, key_dim, generator=g, device=device), dim=-1).to(bf)
    k = F.normalize(torch.randn(batch, ring_len, heads, key_dim, generator=g, device=device), dim=-1).to(bf)
    v = torch.randn(batch, ring_len, value_heads, value_dim, generator=g, device=device).to(bf)
    a = torch.randn(batch, ring_len, value_heads, generator=g, device=device)
    a_log = torch.rand(value_heads, generator=g, device=device)
    dt_bias = torch.rand(value_heads, generator=g, device=device) - 4.0
    gates = (-a_log.exp() * F.softplus(a + dt_bias)).to(gate_dtype)
    beta = torch.sigmoid(torch.randn(batch, ring_len, value_heads, generator=g, device=device)).to(gate_dtype)
    state = state_sigma * torch.randn(batch, value_heads, value_dim, key_dim, generator=g, device=device)
    return {"q": q, "k": k, "v": v, "g": gates, "beta": beta, "state": state.float()}


def key_scale(key_dim: int = 128) -> float:
    return key_dim ** -0.5 if key_dim else math.nan
