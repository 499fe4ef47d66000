"""Shared helpers of the GPU parity tests: seeded numpy inputs (so the oracle
and the CUDA path see identical values) and host<->device conversions."""

from __future__ import annotations

import numpy as np
import torch

import oracle as O

# tolerances (relative L2), stated once
TOL_OUT_BF16 = 2e-3  # bf16 output vs the fp32 oracle
TOL_FULL_PRECISION = 1e-5  # float32 checkpoint replay vs per-token recurrence
TOL_F32_KERNEL = 1e-5  # float32 outputs vs the oracle on identical inputs


def to_dev(x: np.ndarray, dtype: torch.dtype, device="cuda") -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(x))
    return t.to(device=device).to(dtype)


def to_np(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).cpu().numpy()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.float().cpu().numpy()
    return t.cpu().numpy()


def e4m3_dev(codes: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(codes, np.uint8)).to(device).view(torch.float8_e4m3fn)


def ring_inputs(rng, B, L, H, HV, K=128, sigma=0.05, gate="f32"):
    """Prepped ring contents + q + a float32 state, values exactly representable
    in their storage dtypes."""
    f32 = np.float32
    q = O.bf16_round(_normalize(rng.standard_normal((B, H, K)).astype(f32)))
    k = O.bf16_round(_normalize(rng.standard_normal((B, L, H, K)).astype(f32)))
    v = O.bf16_round(rng.standard_normal((B, L, HV, K)).astype(f32))
    a = rng.standard_normal((B, L, HV)).astype(f32)
    a_log = rng.uniform(0, 1, HV).astype(f32)
    dt_bias = (rng.uniform(0, 1, HV) - 4.0).astype(f32)
    g = (-np.exp(a_log) * np.log1p(np.exp(a + dt_bias))).astype(f32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((B, L, HV))))).astype(f32)
    if gate == "bf16":
        g, beta = O.bf16_round(g), O.bf16_round(beta)
    state = (sigma * rng.standard_normal((B, HV, K, K))).astype(f32)
    return dict(q=q, k=k, v=v, g=g, beta=beta, state=state)


def _normalize(x):
    return (x / np.sqrt((x * x).sum(-1, keepdims=True))).astype(np.float32)


def raw_inputs(rng, B, H, HV, K=128):
    """Raw full-contract inputs for one step (BASELINE config 1 distributions)."""
    f32 = np.float32
    mixed = O.bf16_round(rng.standard_normal((B, 2 * H * K + HV * K)).astype(f32))
    a = O.bf16_round(rng.standard_normal((B, HV)).astype(f32))
    b = O.bf16_round(rng.standard_normal((B, HV)).astype(f32))
    return mixed, a, b


def gate_params(rng, HV):
    a_log = np.log(rng.uniform(1, 16, HV)).astype(np.float32)
    dt_bias = (0.5 * rng.standard_normal(HV)).astype(np.float32)
    return a_log, dt_bias


def oracle_replay_out(state_f32, q, k, v, g, beta, valid):
    """Last-token output of run_kernel over slots 0..valid[b]-1 (forward form)."""
    B, HV = state_f32.shape[:2]
    out = np.zeros((B, HV, state_f32.shape[2]), np.float32)
    states = np.array(state_f32, copy=True)
    for b in range(B):
        n = int(valid[b])
        if n == 0:
            out[b] = np.einsum("hvk,hk->hv", state_f32[b], np.repeat(q[b], HV // q.shape[1], 0)) * np.float32(
                q.shape[-1] ** -0.5)
            continue
        o, s = O.run_kernel(state_f32[b:b + 1], np.repeat(q[b:b + 1, None], n, 1), k[b:b + 1, :n], v[b:b + 1, :n],
                            g[b:b + 1, :n], beta[b:b + 1, :n])
        out[b] = o[0, -1]
        states[b] = s[0]
    return out, states


def check_prep_and_sync(host, dev, mixed, a, b, a_log, dt_bias, pos, H, gate_name, q_out):
    """Compare this step's prep outputs (ring slot ``pos``, q_out) with the
    oracle's prep, then copy the device's slot into the host ring so that the
    replay comparison runs on identical inputs.  Returns the device q."""
    B, HV = a.shape
    qn, kn, v, g, be = O.prep(mixed, a, b, a_log, dt_bias, H, 128, HV, 128, gate_dtype=gate_name)
    qd = to_np(q_out)
    # x/||x|| is rounded to bf16; a last-bit difference needs a value within
    # ~1e-7 of a rounding midpoint
    assert np.mean(qd != qn) < 1e-2 and np.allclose(qd, qn, rtol=8e-3, atol=1e-6)
    for i in range(B):
        p = pos[i]
        kd = to_np(dev.k_ring[i, p])
        assert np.mean(kd != kn[i]) < 1e-2 and np.allclose(kd, kn[i], rtol=8e-3, atol=1e-6)
        np.testing.assert_array_equal(to_np(dev.v_ring[i, p]), v[i])
        gtol = 1e-5 if gate_name == "f32" else 8e-3
        np.testing.assert_allclose(to_np(dev.g_ring[i, p]), g[i], rtol=gtol, atol=1e-6)
        np.testing.assert_allclose(to_np(dev.beta_ring[i, p]), be[i], rtol=gtol, atol=1e-6)
        host.k_ring[i, p] = kd
        host.v_ring[i, p] = v[i]
        host.g_ring[i, p] = to_np(dev.g_ring[i, p])
        host.beta_ring[i, p] = to_np(dev.beta_ring[i, p])
    return qd
