"""gdn_fused_step (prep + ring append + replay + flush in one launch) vs the
full-contract step oracle (bench_gdn_full_contract.py:138-308 semantics,
ref.py:189-244 chain)."""

import numpy as np
import pytest
import torch

import gdnr
import oracle as O
from helpers import TOL_F32_KERNEL, TOL_FULL_PRECISION, TOL_OUT_BF16, check_prep_and_sync, e4m3_dev, gate_params, \
    raw_inputs, to_dev, to_np

pytestmark = pytest.mark.gpu


def make_state(rng, B, H, HV, L, gate_dtype, scale_dtype, f32ck=False):
    s0 = (0.02 * rng.standard_normal((B, HV, 128, 128))).astype(np.float32)
    if f32ck:
        host = O.RingState(s0.copy(), None, np.zeros((B, L, H, 128), np.float32), np.zeros((B, L, HV, 128), np.float32),
                           np.zeros((B, L, HV), np.float32), np.zeros((B, L, HV), np.float32))
        dev = gdnr.ReplayState.allocate(B, H, HV, L, checkpoint_dtype=torch.float32, gate_dtype=gate_dtype)
        dev.checkpoint.copy_(to_dev(s0, torch.float32))
        return host, dev
    q0 = O.quantize_checkpoint(s0, "vblock", 32)
    host = O.RingState(q0.payload.copy(), q0.scale.copy(), np.zeros((B, L, H, 128), np.float32),
                       np.zeros((B, L, HV, 128), np.float32), np.zeros((B, L, HV), np.float32),
                       np.zeros((B, L, HV), np.float32))
    dev = gdnr.ReplayState.allocate(B, H, HV, L, scale_dtype=scale_dtype, gate_dtype=gate_dtype)
    dev.checkpoint.copy_(e4m3_dev(q0.payload))
    dev.scale.copy_(to_dev(q0.scale.astype(np.float32), scale_dtype))
    return host, dev


def _gname(dt):
    return {torch.float32: "f32", torch.bfloat16: "bf16"}[dt]


@pytest.mark.parametrize("heads", [(2, 4), (4, 4)])
@pytest.mark.parametrize("flush_hint", ["auto", "all"])
@pytest.mark.parametrize("gate_dtype,scale_dtype", [(torch.float32, torch.float32), (torch.bfloat16, torch.float16)])
def test_fused_cycles_match_oracle(cuda_device, gate_dtype, scale_dtype, flush_hint, heads):
    rng = np.random.default_rng(11)
    (H, HV), B, L, T = heads, 4, 4, 10
    a_log, dt_bias = gate_params(rng, HV)
    host, dev = make_state(rng, B, H, HV, L, gate_dtype, scale_dtype)
    # heterogeneous ring positions: sequences are at different points of their cycle
    pos = np.array([0, 1, 3, 2], np.int32)
    dev.pos.copy_(to_dev(pos, torch.int32))
    pos_next = torch.empty_like(dev.pos)
    for t in range(T):
        mixed, a, b = raw_inputs(rng, B, H, HV)
        out = torch.empty(B, HV, 128, dtype=torch.float32, device="cuda")
        q_out = torch.empty(B, H, 128, dtype=torch.bfloat16, device="cuda")
        dev.step(to_dev(mixed, torch.bfloat16), to_dev(a, torch.bfloat16), to_dev(b, torch.bfloat16),
                 to_dev(a_log, torch.float32), to_dev(dt_bias, torch.float32), out=out, pos_out=pos_next, q_out=q_out,
                 flush_hint=flush_hint)
        np.testing.assert_array_equal(to_np(pos_next), (pos + 1) % L)
        qd = check_prep_and_sync(host, dev, mixed, a, b, a_log, dt_bias, pos, H, _gname(gate_dtype), q_out)
        ref_out = O.replay_step(host, qd, pos, out_dtype="f32")
        assert O.relative_l2(to_np(out), ref_out) < TOL_F32_KERNEL, t
        flushed = pos == L - 1
        if flushed.any():
            got_payload = to_np(dev.checkpoint)
            got_scale = dev.scale.float().cpu().numpy()
            for i in np.nonzero(flushed)[0]:
                assert np.mean(got_payload[i] != host.payload[i]) < 1e-3
                assert np.allclose(got_scale[i], host.scale[i].astype(np.float32), rtol=2e-3)
            host.payload[:] = got_payload
            host.scale[:] = got_scale.astype(np.float16)
        dev.pos.copy_(pos_next)
        pos = (pos + 1) % L


def test_fused_bf16_output_tolerance(cuda_device):
    rng = np.random.default_rng(12)
    B, H, HV, L = 8, 16, 32, 16
    a_log, dt_bias = gate_params(rng, HV)
    host, dev = make_state(rng, B, H, HV, L, torch.float32, torch.float32)
    pos = np.arange(B, dtype=np.int32) * 2 % L  # 0,2,..,14: includes fill 15 (flush at pos 15 never here)
    pos[-1] = L - 1  # one sequence flushes
    dev.pos.copy_(to_dev(pos, torch.int32))
    # pre-fill the ring slots below pos with prepped tokens (same on both sides)
    for t in range(L):
        mixed, a, b = raw_inputs(rng, B, H, HV)
        qn, kn, v, g, be = O.prep(mixed, a, b, a_log, dt_bias, H, 128, HV, 128, gate_dtype="f32")
        host.k_ring[:, t], host.v_ring[:, t], host.g_ring[:, t], host.beta_ring[:, t] = kn, v, g, be
    dev.k_ring.copy_(to_dev(host.k_ring, torch.bfloat16))
    dev.v_ring.copy_(to_dev(host.v_ring, torch.bfloat16))
    dev.g_ring.copy_(to_dev(host.g_ring, torch.float32))
    dev.beta_ring.copy_(to_dev(host.beta_ring, torch.float32))
    mixed, a, b = raw_inputs(rng, B, H, HV)
    q_out = torch.empty(B, H, 128, dtype=torch.bfloat16, device="cuda")
    out = dev.step(to_dev(mixed, torch.bfloat16), to_dev(a, torch.bfloat16), to_dev(b, torch.bfloat16),
                   to_dev(a_log, torch.float32), to_dev(dt_bias, torch.float32), q_out=q_out)
    assert out.dtype == torch.bfloat16
    qd = check_prep_and_sync(host, dev, mixed, a, b, a_log, dt_bias, pos, H, "f32", q_out)
    ref_out = O.replay_step(host, qd, pos, out_dtype="f32")
    assert O.relative_l2(to_np(out), ref_out) < TOL_OUT_BF16


def test_fused_full_precision_equals_recurrence(cuda_device):
    """float32 checkpoint variant over 3 windows == per-token recurrence (1e-5)."""
    rng = np.random.default_rng(13)
    B, H, HV, L, T = 2, 2, 4, 4, 11
    a_log, dt_bias = gate_params(rng, HV)
    s0 = (0.02 * rng.standard_normal((B, HV, 128, 128))).astype(np.float32)
    dev = gdnr.ReplayState.allocate(B, H, HV, L, checkpoint_dtype=torch.float32)
    dev.checkpoint.copy_(to_dev(s0, torch.float32))
    qs, ks, vs, gs, bs, outs = [], [], [], [], [], []
    for t in range(T):
        mixed, a, b = raw_inputs(rng, B, H, HV)
        out = torch.empty(B, HV, 128, dtype=torch.float32, device="cuda")
        q_out = torch.empty(B, H, 128, dtype=torch.float32, device="cuda")
        nxt = torch.empty_like(dev.pos)
        dev.step(to_dev(mixed, torch.bfloat16), to_dev(a, torch.bfloat16), to_dev(b, torch.bfloat16),
                 to_dev(a_log, torch.float32), to_dev(dt_bias, torch.float32), out=out, q_out=q_out, pos_out=nxt)
        dev.pos.copy_(nxt)
        outs.append(to_np(out))
        p = t % L
        qs.append(to_np(q_out))
        ks.append(to_np(dev.k_ring[:, p]))
        vs.append(to_np(dev.v_ring[:, p]))
        gs.append(to_np(dev.g_ring[:, p]))
        bs.append(to_np(dev.beta_ring[:, p]))
    st = lambda xs: np.stack(xs, 1)
    base_out, base_state = O.baseline_decode(s0, st(qs), st(ks), st(vs), st(gs), st(bs))
    assert O.relative_l2(st(outs), base_out) < TOL_FULL_PRECISION
    # after T=11 tokens the checkpoint holds the state after the flush at t=7
    ref_ck = O.baseline_decode(s0, st(qs)[:, :8], st(ks)[:, :8], st(vs)[:, :8], st(gs)[:, :8], st(bs)[:, :8])[1]
    assert O.relative_l2(to_np(dev.checkpoint), ref_ck) < TOL_FULL_PRECISION


def test_fused_bad_pos_sets_error_flag(cuda_device):
    rng = np.random.default_rng(14)
    B, H, HV, L = 3, 2, 4, 4
    a_log, dt_bias = gate_params(rng, HV)
    host, dev = make_state(rng, B, H, HV, L, torch.float32, torch.float32)
    dev.pos.copy_(torch.tensor([0, 7, -1], dtype=torch.int32))
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    mixed, a, b = raw_inputs(rng, B, H, HV)
    out = torch.full((B, HV, 128), 123.0, dtype=torch.float32, device="cuda")
    ring_before = dev.k_ring.clone()
    dev.step(to_dev(mixed, torch.bfloat16), to_dev(a, torch.bfloat16), to_dev(b, torch.bfloat16),
             to_dev(a_log, torch.float32), to_dev(dt_bias, torch.float32), out=out, error_flag=err)
    assert int(err.item()) & gdnr._lib.DEVERR_BAD_POS
    # sequences with a bad position are left untouched
    assert torch.all(out[1:] == 123.0)
    assert torch.equal(dev.k_ring[1:], ring_before[1:])
    assert not torch.all(out[0] == 123.0)


@pytest.mark.parametrize("gate_dtype", [torch.float32, torch.bfloat16])
def test_fused_flush_hint_none_is_identical(cuda_device, gate_dtype):
    """With no sequence at L-1, hint "none" (one launch) writes exactly what
    hint "auto" writes, bit for bit, and sets no error bit."""
    rng = np.random.default_rng(15)
    B, H, HV, L = 6, 2, 4, 8
    a_log, dt_bias = gate_params(rng, HV)
    _, dev = make_state(rng, B, H, HV, L, gate_dtype, torch.float16)
    dev.pos.copy_(torch.tensor([0, 1, 3, 6, 5, 2], dtype=torch.int32))
    for t in range(L):  # fill all ring slots with prepped tokens
        mixed, a, b = raw_inputs(rng, B, H, HV)
        dev.pos.fill_(t)
        dev.step(to_dev(mixed, torch.bfloat16), to_dev(a, torch.bfloat16), to_dev(b, torch.bfloat16),
                 to_dev(a_log, torch.float32), to_dev(dt_bias, torch.float32), flush_hint="auto")
    dev.pos.copy_(torch.tensor([0, 1, 3, 6, 5, 2], dtype=torch.int32))
    twin = dev.snapshot()
    mixed, a, b = raw_inputs(rng, B, H, HV)
    args = (to_dev(mixed, torch.bfloat16), to_dev(a, torch.bfloat16), to_dev(b, torch.bfloat16),
            to_dev(a_log, torch.float32), to_dev(dt_bias, torch.float32))
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out_auto = dev.step(*args, flush_hint="auto", error_flag=err)
    state_auto = dev.snapshot()
    dev.restore(twin)
    out_none = dev.step(*args, flush_hint="none", error_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(out_auto, out_none)
    for name in ("checkpoint", "scale", "k_ring", "v_ring", "g_ring", "beta_ring"):
        assert torch.equal(getattr(dev, name), getattr(state_auto, name)), name


@pytest.mark.parametrize("positions", ["all_flush", "mixed"])
def test_fused_flush_hint_auto_matches_all(cuda_device, positions):
    """hint "auto" and hint "all" write the same output and state (one launch
    that rebuilds the flushing heads and reads out the others either way)."""
    rng = np.random.default_rng(17)
    B, H, HV, L = 8, 4, 8, 8
    a_log, dt_bias = gate_params(rng, HV)
    _, dev = make_state(rng, B, H, HV, L, torch.float32, torch.float16)
    for t in range(L - 1):  # fill slots 0..L-2
        mixed, a, b = raw_inputs(rng, B, H, HV)
        dev.pos.fill_(t)
        dev.step(to_dev(mixed, torch.bfloat16), to_dev(a, torch.bfloat16), to_dev(b, torch.bfloat16),
                 to_dev(a_log, torch.float32), to_dev(dt_bias, torch.float32), flush_hint="auto")
    pos = np.full(B, L - 1, np.int32) if positions == "all_flush" else np.arange(B, dtype=np.int32) % L
    dev.pos.copy_(to_dev(pos, torch.int32))
    twin = dev.snapshot()
    mixed, a, b = raw_inputs(rng, B, H, HV)
    args = (to_dev(mixed, torch.bfloat16), to_dev(a, torch.bfloat16), to_dev(b, torch.bfloat16),
            to_dev(a_log, torch.float32), to_dev(dt_bias, torch.float32))
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out_auto = dev.step(*args, out=torch.empty(B, HV, 128, device="cuda"), flush_hint="auto", error_flag=err)
    state_auto = dev.snapshot()
    dev.restore(twin)
    out_all = dev.step(*args, out=torch.empty(B, HV, 128, device="cuda"), flush_hint="all", error_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(out_auto, out_all)
    for name in ("checkpoint", "scale", "k_ring", "v_ring", "g_ring", "beta_ring"):
        assert torch.equal(getattr(state_auto, name), getattr(dev, name)), name


def test_fused_flush_hint_none_violation_is_reported(cuda_device):
    rng = np.random.default_rng(16)
    B, H, HV, L = 3, 2, 4, 4
    a_log, dt_bias = gate_params(rng, HV)
    _, dev = make_state(rng, B, H, HV, L, torch.float32, torch.float32)
    dev.pos.copy_(torch.tensor([0, L - 1, 1], dtype=torch.int32))
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    mixed, a, b = raw_inputs(rng, B, H, HV)
    out = torch.full((B, HV, 128), 123.0, dtype=torch.float32, device="cuda")
    ck_before = dev.checkpoint.clone()
    dev.step(to_dev(mixed, torch.bfloat16), to_dev(a, torch.bfloat16), to_dev(b, torch.bfloat16),
             to_dev(a_log, torch.float32), to_dev(dt_bias, torch.float32), out=out, error_flag=err, flush_hint="none")
    assert int(err.item()) & gdnr._lib.DEVERR_BAD_HINT
    assert torch.all(out[1] == 123.0)  # the flushing sequence is left unprocessed
    assert not torch.all(out[0] == 123.0) and not torch.all(out[2] == 123.0)
    assert torch.equal(dev.checkpoint, ck_before)


def test_fused_full_size_subset_parity(cuda_device):
    """BASELINE shape (B=64, H=16, HV=32, L=16) through a whole cycle; outputs of
    a random subset of sequences checked against the oracle, and every output
    against a float32 torch recurrence on the GPU."""
    rng = np.random.default_rng(15)
    B, H, HV, L = 64, 16, 32, 16
    a_log, dt_bias = gate_params(rng, HV)
    s0 = (0.02 * rng.standard_normal((B, HV, 128, 128))).astype(np.float32)
    dev = gdnr.ReplayState.allocate(B, H, HV, L)
    dev.load_state(to_dev(s0, torch.float32))
    ck0 = to_np(dev.checkpoint).copy()
    sc0 = dev.scale.cpu().numpy().copy()
    subset = [0, 37]
    host = O.RingState(ck0[subset].copy(), sc0[subset].astype(np.float16), np.zeros((2, L, H, 128), np.float32),
                       np.zeros((2, L, HV, 128), np.float32), np.zeros((2, L, HV), np.float32),
                       np.zeros((2, L, HV), np.float32))
    # torch float32 recurrence from the dequantised checkpoint (exact fp32 path)
    S = gdnr.dequantize_checkpoint(gdnr.QuantizedCheckpoint(dev.checkpoint, dev.scale, "vblock", 32, 0.0)).clone()
    worst = 0.0
    for t in range(L + 2):
        mixed, a, b = raw_inputs(rng, B, H, HV)
        nxt = torch.empty_like(dev.pos)
        md, ad, bd = to_dev(mixed, torch.bfloat16), to_dev(a, torch.bfloat16), to_dev(b, torch.bfloat16)
        q_out = torch.empty(B, H, 128, dtype=torch.bfloat16, device="cuda")
        out = dev.step(md, ad, bd, to_dev(a_log, torch.float32), to_dev(dt_bias, torch.float32), pos_out=nxt,
                       q_out=q_out)
        p = t % L
        # float32 torch reference of the same step
        qn = q_out.float().repeat_interleave(2, 1)
        kn = dev.k_ring[:, p].float().repeat_interleave(2, 1)
        vv = dev.v_ring[:, p].float()
        gg = dev.g_ring[:, p].float()
        bb = dev.beta_ring[:, p].float()
        S = S * torch.exp(gg)[..., None, None]
        r = (S * kn[:, :, None, :]).sum(-1)
        S = S + ((vv - r) * bb[..., None])[..., None] * kn[:, :, None, :]
        o_ref = (S * qn[:, :, None, :]).sum(-1) * (128 ** -0.5)
        err = (out.float() - o_ref).norm() / o_ref.norm()
        worst = max(worst, float(err))
        host.k_ring[:] = to_np(dev.k_ring)[subset]
        host.v_ring[:] = to_np(dev.v_ring)[subset]
        host.g_ring[:] = to_np(dev.g_ring)[subset]
        host.beta_ring[:] = to_np(dev.beta_ring)[subset]
        ref_out = O.replay_step(host, to_np(q_out)[subset], np.full(2, p, np.int32), out_dtype="f32")
        assert O.relative_l2(to_np(out)[subset], ref_out) < TOL_OUT_BF16, t
        if p == L - 1:
            host.payload[:] = to_np(dev.checkpoint)[subset]
            host.scale[:] = dev.scale.cpu().numpy()[subset].astype(np.float16)
            # the fp32 chain continues from the re-quantised checkpoint, like the replay scheme
            S = gdnr.dequantize_checkpoint(gdnr.QuantizedCheckpoint(dev.checkpoint, dev.scale, "vblock", 32, 0.0)).clone()
        dev.pos.copy_(nxt)
    assert worst < TOL_OUT_BF16
