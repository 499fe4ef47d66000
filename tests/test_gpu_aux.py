"""Mirrors of gdn_prep_ring, gdn_replay_fp8_split and gdn_bf16_step."""

import numpy as np
import pytest
import torch

import gdnr
import oracle as O
from helpers import TOL_F32_KERNEL, e4m3_dev, gate_params, oracle_replay_out, raw_inputs, ring_inputs, to_dev, to_np

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("gate_dtype", [torch.float32, torch.bfloat16])
def test_prep_ring_matches_oracle(cuda_device, gate_dtype):
    rng = np.random.default_rng(21)
    B, H, HV, L = 5, 16, 32, 8
    a_log, dt_bias = gate_params(rng, HV)
    mixed, a, b = raw_inputs(rng, B, H, HV)
    a[0, :4] = [-30.0, 19.75, 20.0, 24.0]  # around the softplus threshold
    pos = np.array([0, 7, 3, 3, 5], np.int32)
    q_out = torch.zeros(B, H, 128, dtype=torch.bfloat16, device="cuda")
    k_ring = torch.zeros(B, L, H, 128, dtype=torch.bfloat16, device="cuda")
    v_ring = torch.zeros(B, L, HV, 128, dtype=torch.bfloat16, device="cuda")
    g_ring = torch.zeros(B, L, HV, dtype=gate_dtype, device="cuda")
    b_ring = torch.zeros(B, L, HV, dtype=gate_dtype, device="cuda")
    gdnr.gdn_prep_ring(to_dev(mixed, torch.bfloat16), to_dev(a, torch.float32), to_dev(b, torch.float32),
                       to_dev(a_log, torch.float32), to_dev(dt_bias, torch.float32), to_dev(pos, torch.int32), q_out,
                       k_ring, v_ring, g_ring, b_ring)
    gname = "f32" if gate_dtype == torch.float32 else "bf16"
    qn, kn, v, g, be = O.prep(mixed, a, b, a_log, dt_bias, H, 128, HV, 128, gate_dtype=gname)
    assert np.allclose(to_np(q_out), qn, rtol=8e-3, atol=1e-6) and np.mean(to_np(q_out) != qn) < 1e-2
    for i in range(B):
        p = pos[i]
        assert np.allclose(to_np(k_ring[i, p]), kn[i], rtol=8e-3, atol=1e-6)
        np.testing.assert_array_equal(to_np(v_ring[i, p]), v[i])
        tol = 1e-5 if gname == "f32" else 8e-3
        np.testing.assert_allclose(to_np(g_ring[i, p]), g[i], rtol=tol, atol=1e-6)
        np.testing.assert_allclose(to_np(b_ring[i, p]), be[i], rtol=tol, atol=1e-6)
        other = [t for t in range(L) if t != p]
        assert torch.count_nonzero(k_ring[i, other]) == 0  # only slot pos written


@pytest.mark.parametrize("block_v", [32, 128])
def test_replay_split_matches_replay(cuda_device, block_v):
    rng = np.random.default_rng(22)
    B, H, HV, L = 3, 2, 4, 8
    d = ring_inputs(rng, B, L, H, HV)
    ck = O.quantize_checkpoint(d["state"], "vblock", 32)
    valid = np.array([8, 0, 5], np.int32)
    tq = torch.full((B, HV, 128), -7.0, device="cuda")
    coef = torch.full((B, HV, L), -7.0, device="cuda")
    out = torch.empty(B, HV, 128, dtype=torch.float32, device="cuda")
    gdnr.gdn_replay_fp8_split(e4m3_dev(ck.payload), to_dev(ck.scale.astype(np.float32), torch.float16),
                              to_dev(d["q"], torch.bfloat16), to_dev(d["k"], torch.bfloat16),
                              to_dev(d["v"], torch.bfloat16), to_dev(d["g"], torch.float32),
                              to_dev(d["beta"], torch.float32), to_dev(valid, torch.int32), tq, coef, block_v=block_v,
                              out=out)
    ref, _ = oracle_replay_out(O.dequantize_checkpoint(ck), d["q"], d["k"], d["v"], d["g"], d["beta"], valid)
    assert O.relative_l2(to_np(out), ref) < TOL_F32_KERNEL
    # coefficients only for t < valid_len (kern.py:878-885 masks the store)
    c = to_np(coef)
    assert np.all(c[1] == -7.0) and np.all(c[2, :, 5:] == -7.0) and np.all(c[2, :, :5] != -7.0)


def test_bf16_step_matches_fp32_reference(cuda_device):
    rng = np.random.default_rng(23)
    B, H, HV = 4, 2, 4
    d = ring_inputs(rng, B, 1, H, HV, sigma=0.02)
    state = O.bf16_round(d["state"])
    st = to_dev(state, torch.bfloat16)
    q = to_dev(d["q"], torch.bfloat16)
    k = to_dev(d["k"][:, 0], torch.bfloat16)
    v = to_dev(d["v"][:, 0], torch.bfloat16)
    g = to_dev(d["g"][:, 0], torch.float32)
    be = to_dev(d["beta"][:, 0], torch.float32)
    out = gdnr.gdn_bf16_step(st, q, k, v, g, be)
    ref_out, ref_state = O.run_kernel(state, d["q"][:, None], d["k"][:, :1], d["v"][:, :1], d["g"][:, :1],
                                      d["beta"][:, :1])
    assert O.relative_l2(to_np(out), ref_out[:, 0]) < 2e-3
    assert O.relative_l2(to_np(st), ref_state) < 4e-3
