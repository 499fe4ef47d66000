"""INT8 checkpoints ("vblock_int8", ref.py:44-47, :96-97) through the replay and
the fused step: the readout of the int8 codes against the oracle on the same
dequantised checkpoint, and the flush's int8 re-quantisation against the
oracle's quantiser applied to the oracle's rebuilt state -- the same checks the
E4M3 path gets (kern.py:1292-1357 validation pattern), with the tolerances
written below."""

import numpy as np
import pytest
import torch

import gdnr
import oracle as O
from helpers import TOL_F32_KERNEL, TOL_OUT_BF16, check_prep_and_sync, gate_params, oracle_replay_out, raw_inputs, \
    ring_inputs, to_dev, to_np

pytestmark = pytest.mark.gpu

# a rebuilt float32 state agrees with the oracle's to ~1e-7, so an int8 code
# may differ only where x / scale sits that close to a half-integer
TOL_CODE_MISMATCH = 1e-3


def setup_case(seed, B, L, H=2, HV=4, scale_dtype=torch.float16):
    rng = np.random.default_rng(seed)
    d = ring_inputs(rng, B, L, H, HV)
    ck = O.quantize_checkpoint(d["state"], "vblock_int8", 32)
    assert ck.payload.dtype == np.int8
    dev = dict(
        checkpoint=to_dev(ck.payload, torch.int8),
        scale=to_dev(ck.scale.astype(np.float32), scale_dtype),
        q=to_dev(d["q"], torch.bfloat16),
        k=to_dev(d["k"], torch.bfloat16),
        v=to_dev(d["v"], torch.bfloat16),
        g=to_dev(d["g"], torch.float32),
        beta=to_dev(d["beta"], torch.float32),
    )
    return d, ck, dev


@pytest.mark.parametrize("block_v", [32, 128])
def test_int8_replay_nonflush_matches_oracle(cuda_device, block_v):
    B, L = 4, 16
    d, ck, dev = setup_case(41, B, L)
    valid = np.array([L, 1, 0, 9], np.int32)
    args = (dev["checkpoint"], dev["scale"], dev["q"], dev["k"], dev["v"], dev["g"], dev["beta"],
            to_dev(valid, torch.int32), torch.zeros(B, dtype=torch.bool, device="cuda"))
    ref, _ = oracle_replay_out(O.dequantize_checkpoint(ck), d["q"], d["k"], d["v"], d["g"], d["beta"], valid)
    out = gdnr.gdn_replay_fp8(*args, block_v=block_v)
    assert O.relative_l2(to_np(out), ref) < TOL_OUT_BF16
    out32 = torch.empty(B, 4, 128, dtype=torch.float32, device="cuda")
    gdnr.gdn_replay_fp8(*args, block_v=block_v, out=out32)
    for b in range(B):
        assert O.relative_l2(to_np(out32)[b], ref[b]) < TOL_F32_KERNEL, b
    assert np.array_equal(to_np(dev["checkpoint"]), ck.payload)


@pytest.mark.parametrize("divisor", ["oracle", "rounded"])
def test_int8_replay_flush_matches_oracle(cuda_device, divisor):
    B, L = 4, 8
    d, ck, dev = setup_case(42, B, L, H=2, HV=4)
    valid = np.array([L, 3, 0, L], np.int32)
    flush = np.array([1, 1, 1, 0], np.bool_)
    out = torch.empty(B, 4, 128, dtype=torch.float32, device="cuda")
    gdnr.gdn_replay_fp8(dev["checkpoint"], dev["scale"], dev["q"], dev["k"], dev["v"], dev["g"], dev["beta"],
                        to_dev(valid, torch.int32), to_dev(flush, torch.bool), out=out, quant_divisor=divisor)
    ref_out, ref_states = oracle_replay_out(O.dequantize_checkpoint(ck), d["q"], d["k"], d["v"], d["g"], d["beta"],
                                            valid)
    assert O.relative_l2(to_np(out), ref_out) < TOL_F32_KERNEL
    got_payload = to_np(dev["checkpoint"])
    got_scale = dev["scale"].float().cpu().numpy()
    assert got_payload.dtype == np.int8
    for b in range(B):
        if flush[b]:
            refq = O.quantize_vblock32(ref_states[b:b + 1], divisor=divisor, int8=True)
            mism = got_payload[b] != refq.payload[0]
            assert np.mean(mism) < TOL_CODE_MISMATCH, b
            # where a code differs it is by one step (a rounding-midpoint flip)
            assert np.all(np.abs(got_payload[b].astype(np.int32) - refq.payload[0].astype(np.int32)) <= 1)
            assert np.allclose(got_scale[b], refq.scale[0].astype(np.float32), rtol=2e-3)  # <= 1 fp16 ulp
            assert np.all(np.abs(got_payload[b].astype(np.int32)) <= 127)
        else:
            assert np.array_equal(got_payload[b], ck.payload[b])


@pytest.mark.parametrize("heads,L,gate_dtype,scale_dtype", [
    ((2, 4), 4, torch.float32, torch.float32),
    ((2, 2), 3, torch.bfloat16, torch.float16),
    ((1, 4), 8, torch.float32, torch.float16),
])
def test_int8_fused_cycles_match_oracle(cuda_device, heads, L, gate_dtype, scale_dtype):
    rng = np.random.default_rng(43)
    (H, HV), B = heads, 4
    T = 2 * L + 2
    gname = "f32" if gate_dtype == torch.float32 else "bf16"
    a_log, dt_bias = gate_params(rng, HV)
    s0 = (0.02 * rng.standard_normal((B, HV, 128, 128))).astype(np.float32)
    q0 = O.quantize_checkpoint(s0, "vblock_int8", 32)
    host = O.RingState(q0.payload.copy(), q0.scale.copy(), np.zeros((B, L, H, 128), np.float32),
                       np.zeros((B, L, HV, 128), np.float32), np.zeros((B, L, HV), np.float32),
                       np.zeros((B, L, HV), np.float32))
    dev = gdnr.ReplayState.allocate(B, H, HV, L, scale_dtype=scale_dtype, gate_dtype=gate_dtype,
                                    checkpoint_dtype=torch.int8)
    dev.load_state(to_dev(s0, torch.float32))
    np.testing.assert_array_equal(to_np(dev.checkpoint), q0.payload)  # the GPU int8 codec, bit-exact
    pos = np.array([0, 1, L - 1, L // 2], np.int32)
    dev.pos.copy_(to_dev(pos, torch.int32))
    pos_next = torch.empty_like(dev.pos)
    flushes = 0
    for t in range(T):
        mixed, a, b = raw_inputs(rng, B, H, HV)
        out = torch.empty(B, HV, 128, dtype=torch.float32, device="cuda")
        q_out = torch.empty(B, H, 128, dtype=torch.bfloat16, device="cuda")
        dev.step(to_dev(mixed, torch.bfloat16), to_dev(a, torch.bfloat16), to_dev(b, torch.bfloat16),
                 to_dev(a_log, torch.float32), to_dev(dt_bias, torch.float32), out=out, pos_out=pos_next, q_out=q_out)
        qd = check_prep_and_sync(host, dev, mixed, a, b, a_log, dt_bias, pos, H, gname, q_out)
        ref_out = O.replay_step(host, qd, pos, out_dtype="f32")
        assert O.relative_l2(to_np(out), ref_out) < TOL_F32_KERNEL, t
        flushed = pos == L - 1
        if flushed.any():
            flushes += int(flushed.sum())
            got_payload = to_np(dev.checkpoint)
            got_scale = dev.scale.float().cpu().numpy()
            assert host.payload.dtype == np.int8
            for i in np.nonzero(flushed)[0]:
                assert np.mean(got_payload[i] != host.payload[i]) < TOL_CODE_MISMATCH
                assert np.allclose(got_scale[i], host.scale[i].astype(np.float32), rtol=2e-3)
            host.payload[:] = got_payload
            host.scale[:] = got_scale.astype(np.float16)
        dev.pos.copy_(pos_next)
        pos = (pos + 1) % L
    assert flushes >= B


def test_int8_checkpoint_rejected_where_not_built(cuda_device):
    d, ck, dev = setup_case(44, 1, 32, H=1, HV=1)
    with pytest.raises(gdnr.GdnrValueError, match="INT8"):  # rings above 16 slots
        gdnr.gdn_replay_fp8(dev["checkpoint"], dev["scale"], dev["q"], dev["k"], dev["v"], dev["g"], dev["beta"],
                            torch.full((1,), 32, dtype=torch.int32, device="cuda"),
                            torch.zeros(1, dtype=torch.bool, device="cuda"))
    pool = gdnr.ReplayState.allocate(3, 2, 4, 4, checkpoint_dtype=torch.int8)
    rng = np.random.default_rng(45)
    mixed, a, b = raw_inputs(rng, 2, 2, 4)
    a_log, dt_bias = gate_params(rng, 4)
    with pytest.raises(gdnr.GdnrValueError, match="E4M3"):  # the packed decode takes E4M3 pools only
        gdnr.fused_recurrent_gated_delta_rule_packed_decode(
            to_dev(mixed, torch.bfloat16), to_dev(a, torch.bfloat16), to_dev(b, torch.bfloat16),
            to_dev(a_log, torch.float32), to_dev(dt_bias, torch.float32), 128 ** -0.5, pool,
            torch.empty(2, 1, 4, 128, dtype=torch.bfloat16, device="cuda"),
            torch.tensor([1, 2], dtype=torch.int32, device="cuda"))


@pytest.mark.parametrize("heads", [(2, 4), (2, 2)])
def test_int8_replay_nonflush_persistent_matches_oracle(cuda_device, heads):
    """flush_hint="none" runs the persistent kernel's int8 variant (integer
    tensor-core team readout); "auto" runs the one-CTA-per-head kernel."""
    H, HV = heads
    B, L = 5, 16
    d, ck, dev = setup_case(46, B, L, H=H, HV=HV)
    valid = np.array([L, 1, 0, 9, 4], np.int32)
    ref, _ = oracle_replay_out(O.dequantize_checkpoint(ck), d["q"], d["k"], d["v"], d["g"], d["beta"], valid)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    outs = {}
    for hint in ("none", "auto"):
        out = torch.empty(B, HV, 128, dtype=torch.float32, device="cuda")
        gdnr.gdn_replay_fp8(dev["checkpoint"], dev["scale"], dev["q"], dev["k"], dev["v"], dev["g"], dev["beta"],
                            to_dev(valid, torch.int32), torch.zeros(B, dtype=torch.bool, device="cuda"), out=out,
                            flush_hint=hint, error_flag=err)
        outs[hint] = to_np(out)
        for b in range(B):
            assert O.relative_l2(outs[hint][b], ref[b]) < TOL_F32_KERNEL, (hint, b)
    assert int(err.item()) == 0
    assert np.array_equal(to_np(dev["checkpoint"]), ck.payload)


@pytest.mark.parametrize("heads", [(2, 4), (2, 2)])
def test_int8_fused_persistent_cycles_match_oracle(cuda_device, heads):
    """Ring cycles with every sequence at the same position: the non-flush steps
    pass flush_hint="none" (the persistent kernel's int8 variant), the flush
    step "auto" (the one-CTA-per-head kernel)."""
    rng = np.random.default_rng(47)
    (H, HV), B, L = heads, 4, 4
    a_log, dt_bias = gate_params(rng, HV)
    s0 = (0.02 * rng.standard_normal((B, HV, 128, 128))).astype(np.float32)
    q0 = O.quantize_checkpoint(s0, "vblock_int8", 32)
    host = O.RingState(q0.payload.copy(), q0.scale.copy(), np.zeros((B, L, H, 128), np.float32),
                       np.zeros((B, L, HV, 128), np.float32), np.zeros((B, L, HV), np.float32),
                       np.zeros((B, L, HV), np.float32))
    dev = gdnr.ReplayState.allocate(B, H, HV, L, scale_dtype=torch.float32, gate_dtype=torch.float32,
                                    checkpoint_dtype=torch.int8)
    dev.load_state(to_dev(s0, torch.float32))
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    pos_next = torch.empty_like(dev.pos)
    for t in range(2 * L + 1):
        p = t % L
        pos = np.full(B, p, np.int32)
        dev.pos.copy_(to_dev(pos, torch.int32))
        mixed, a, b = raw_inputs(rng, B, H, HV)
        out = torch.empty(B, HV, 128, dtype=torch.float32, device="cuda")
        q_out = torch.empty(B, H, 128, dtype=torch.bfloat16, device="cuda")
        dev.step(to_dev(mixed, torch.bfloat16), to_dev(a, torch.bfloat16), to_dev(b, torch.bfloat16),
                 to_dev(a_log, torch.float32), to_dev(dt_bias, torch.float32), out=out, pos_out=pos_next, q_out=q_out,
                 error_flag=err, flush_hint="auto" if p == L - 1 else "none")
        qd = check_prep_and_sync(host, dev, mixed, a, b, a_log, dt_bias, pos, H, "f32", q_out)
        ref_out = O.replay_step(host, qd, pos, out_dtype="f32")
        assert O.relative_l2(to_np(out), ref_out) < TOL_F32_KERNEL, t
        if p == L - 1:
            got_payload = to_np(dev.checkpoint)
            got_scale = dev.scale.float().cpu().numpy()
            for i in range(B):
                assert np.mean(got_payload[i] != host.payload[i]) < TOL_CODE_MISMATCH
                assert np.allclose(got_scale[i], host.scale[i].astype(np.float32), rtol=2e-3)
            host.payload[:] = got_payload
            host.scale[:] = got_scale.astype(np.float16)
    assert int(err.item()) == 0
