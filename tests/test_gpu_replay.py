"""gdn_replay_fp8 (mirror of kern.py:344-405) vs the oracle.

The reference's own validation (kern.py:1292-1357) compares the kernel's
non-flush output with run_kernel on the dequantised checkpoint, and the
flushed checkpoint with quantize(run_kernel's final state).  Same here, with
asserted tolerances."""

import numpy as np
import pytest
import torch

import gdnr
import oracle as O
from helpers import TOL_F32_KERNEL, TOL_FULL_PRECISION, TOL_OUT_BF16, e4m3_dev, oracle_replay_out, ring_inputs, \
    to_dev, to_np

pytestmark = pytest.mark.gpu


def setup_case(seed, B, L, H=2, HV=4, gate="f32", scale_dtype=torch.float16):
    rng = np.random.default_rng(seed)
    d = ring_inputs(rng, B, L, H, HV, gate=gate)
    ck = O.quantize_checkpoint(d["state"], "vblock", 32)
    gdt = torch.float32 if gate == "f32" else torch.bfloat16
    dev = dict(
        checkpoint=e4m3_dev(ck.payload),
        scale=to_dev(ck.scale.astype(np.float32), scale_dtype),
        q=to_dev(d["q"], torch.bfloat16),
        k=to_dev(d["k"], torch.bfloat16),
        v=to_dev(d["v"], torch.bfloat16),
        g=to_dev(d["g"], gdt),
        beta=to_dev(d["beta"], gdt),
    )
    return d, ck, dev


@pytest.mark.parametrize("block_v", [32, 64, 128])
@pytest.mark.parametrize("gate", ["f32", "bf16"])
def test_replay_nonflush_matches_oracle(cuda_device, block_v, gate):
    B, L = 4, 8
    d, ck, dev = setup_case(1, B, L, gate=gate)
    valid = np.array([L, 1, 0, 5], np.int32)
    out = gdnr.gdn_replay_fp8(dev["checkpoint"], dev["scale"], dev["q"], dev["k"], dev["v"], dev["g"], dev["beta"],
                              to_dev(valid, torch.int32), torch.zeros(B, dtype=torch.bool, device="cuda"),
                              block_v=block_v)
    assert out.dtype == torch.bfloat16 and out.shape == (B, 4, 128)
    ref, _ = oracle_replay_out(O.dequantize_checkpoint(ck), d["q"], d["k"], d["v"], d["g"], d["beta"], valid)
    assert O.relative_l2(to_np(out), ref) < TOL_OUT_BF16
    # float32 output isolates the kernel arithmetic from bf16 output rounding
    out32 = torch.empty(B, 4, 128, dtype=torch.float32, device="cuda")
    gdnr.gdn_replay_fp8(dev["checkpoint"], dev["scale"], dev["q"], dev["k"], dev["v"], dev["g"], dev["beta"],
                        to_dev(valid, torch.int32), torch.zeros(B, dtype=torch.bool, device="cuda"),
                        block_v=block_v, out=out32)
    for b in range(B):
        assert O.relative_l2(to_np(out32)[b], ref[b]) < TOL_F32_KERNEL, b
    # checkpoint untouched by a non-flush replay
    assert np.array_equal(to_np(dev["checkpoint"]), ck.payload)


def test_replay_matches_adjoint_oracle(cuda_device):
    B, L = 2, 16
    d, ck, dev = setup_case(2, B, L, H=1, HV=2)
    valid = np.array([16, 11], np.int32)
    out32 = torch.empty(B, 2, 128, dtype=torch.float32, device="cuda")
    gdnr.gdn_replay_fp8(dev["checkpoint"], dev["scale"], dev["q"], dev["k"], dev["v"], dev["g"], dev["beta"],
                        to_dev(valid, torch.int32), torch.zeros(B, dtype=torch.bool, device="cuda"), out=out32)
    ref = O.replay_adjoint(O.dequantize_checkpoint(ck), d["q"], d["k"], d["v"], d["g"], d["beta"], valid)
    assert O.relative_l2(to_np(out32), ref) < TOL_F32_KERNEL


@pytest.mark.parametrize("heads", [(2, 4), (2, 2)])
@pytest.mark.parametrize("divisor", ["oracle", "rounded"])
def test_replay_flush_matches_oracle(cuda_device, divisor, heads):
    B, L = 4, 6
    H, HV = heads
    d, ck, dev = setup_case(3, B, L, H=H, HV=HV)
    valid = np.array([L, 3, 0, L], np.int32)
    flush = np.array([1, 1, 1, 0], np.bool_)
    out = torch.empty(B, HV, 128, dtype=torch.float32, device="cuda")
    gdnr.gdn_replay_fp8(dev["checkpoint"], dev["scale"], dev["q"], dev["k"], dev["v"], dev["g"], dev["beta"],
                        to_dev(valid, torch.int32), to_dev(flush, torch.bool), out=out, quant_divisor=divisor)
    ref_out, ref_states = oracle_replay_out(O.dequantize_checkpoint(ck), d["q"], d["k"], d["v"], d["g"], d["beta"],
                                            valid)
    assert O.relative_l2(to_np(out), ref_out) < TOL_F32_KERNEL
    got_payload = to_np(dev["checkpoint"])
    got_scale = dev["scale"].float().cpu().numpy()
    for b in range(B):
        if flush[b]:
            refq = O.quantize_vblock32(ref_states[b:b + 1], divisor=divisor)
            # the rebuilt float32 states agree to ~1e-7, so a byte may differ
            # only where a value sits within that of an e4m3 rounding midpoint
            mism = np.mean(got_payload[b] != refq.payload[0])
            assert mism < 1e-3, (b, mism)
            assert np.allclose(got_scale[b], refq.scale[0].astype(np.float32), rtol=2e-3)  # <= 1 fp16 ulp
            got_state = O.dequantize_checkpoint(O.QuantizedCheckpoint(got_payload[b:b + 1], got_scale[b:b + 1].astype(
                np.float16), "vblock", 32, 0.0))
            assert O.relative_l2(got_state, O.dequantize_checkpoint(refq)) < 5e-3
        else:
            assert np.array_equal(got_payload[b], ck.payload[b])


def test_replay_on_strided_ring_slices(cuda_device):
    """The reference's validators pass ring[:, :window] views of a longer ring
    (bench_gdn_full_contract.py:201-212)."""
    B, L_total, L = 3, 8, 4
    d, ck, dev = setup_case(4, B, L_total)
    valid = np.array([4, 2, 3], np.int32)
    sl = slice(0, L)
    out = torch.empty(B, 4, 128, dtype=torch.float32, device="cuda")
    gdnr.gdn_replay_fp8(dev["checkpoint"], dev["scale"], dev["q"], dev["k"][:, sl], dev["v"][:, sl], dev["g"][:, sl],
                        dev["beta"][:, sl], to_dev(valid, torch.int32), torch.zeros(B, dtype=torch.bool, device="cuda"),
                        out=out)
    ref, _ = oracle_replay_out(O.dequantize_checkpoint(ck), d["q"], d["k"][:, sl], d["v"][:, sl], d["g"][:, sl],
                               d["beta"][:, sl], valid)
    assert O.relative_l2(to_np(out), ref) < TOL_F32_KERNEL


def test_full_precision_checkpoint_replay(cuda_device):
    """float32 checkpoint (no quantisation): replay + flush over several windows
    equals the per-token recurrence (ref.py:166-186) within 1e-5."""
    rng = np.random.default_rng(5)
    B, H, HV, L, T = 2, 2, 4, 4, 10
    d = ring_inputs(rng, B, T, H, HV)
    qs = O.bf16_round(d["k"][:, :, :, :] * np.float32(0) + d["q"][:, None])  # same q every token
    base_out, _ = O.baseline_decode(d["state"], qs, d["k"], d["v"], d["g"], d["beta"])
    ck = to_dev(d["state"], torch.float32)
    kd, vd = to_dev(d["k"], torch.bfloat16), to_dev(d["v"], torch.bfloat16)
    gd, bd = to_dev(d["g"], torch.float32), to_dev(d["beta"], torch.float32)
    qd = to_dev(d["q"], torch.bfloat16)
    outs = []
    start = 0
    for t in range(T):
        n = t - start + 1
        sl = slice(start, start + L)
        kr, vr, gr, br = kd[:, sl], vd[:, sl], gd[:, sl], bd[:, sl]
        if kr.shape[1] < L:  # pad the ring view to L slots (unused slots are never read)
            pad = L - kr.shape[1]
            kr = torch.cat([kr, torch.zeros_like(kd[:, :pad])], 1)
            vr = torch.cat([vr, torch.zeros_like(vd[:, :pad])], 1)
            gr = torch.cat([gr, torch.zeros_like(gd[:, :pad])], 1)
            br = torch.cat([br, torch.zeros_like(bd[:, :pad])], 1)
        out = torch.empty(B, HV, 128, dtype=torch.float32, device="cuda")
        flush = torch.full((B,), n == L, dtype=torch.bool, device="cuda")
        gdnr.gdn_replay_fp8(ck, None, qd, kr.contiguous(), vr.contiguous(), gr.contiguous(), br.contiguous(),
                            torch.full((B,), n, dtype=torch.int32, device="cuda"), flush, out=out)
        outs.append(to_np(out))
        if n == L:
            start = t + 1
    assert O.relative_l2(np.stack(outs, 1), base_out) < TOL_FULL_PRECISION
