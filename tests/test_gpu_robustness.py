"""Error paths that must leave the CUDA context usable, and a second device.

* A bounded wait that times out: gdnr_selftest_wait_timeout runs the
  persistent step kernel's wait code (s5_wait) on a barrier that nothing ever
  arrives on, with tensor memory held; the wait gives up after its limit,
  records GDNR_DEVERR_WAIT_TIMEOUT, the second wait of the CTA ends through the
  abort word, the tensor memory is released and the kernel returns.  Then the
  flush-capable step (which allocates the whole tensor memory of every SM it
  runs on) must still run and match the oracle.
* The kernels' shared-memory attribute is configured per device: a step on
  cuda:1 after one on cuda:0 (only where two GPUs are visible).
"""

import numpy as np
import pytest
import torch

import gdnr
import oracle as O
from gdnr import _lib
from helpers import TOL_F32_KERNEL, gate_params, raw_inputs, to_dev, to_np

pytestmark = pytest.mark.gpu


def _step_vs_oracle(device, seed, B=8, H=16, HV=32, L=4):
    """One fused step per ring position over a cycle on ``device`` (flush-capable
    hint, heterogeneous positions), f32 outputs vs the oracle."""
    rng = np.random.default_rng(seed)
    a_log, dt_bias = gate_params(rng, HV)
    s0 = (0.02 * rng.standard_normal((B, HV, 128, 128))).astype(np.float32)
    dev = gdnr.ReplayState.allocate(B, H, HV, L, device=device)
    dev.load_state(torch.from_numpy(s0).to(device))
    host = O.RingState(to_np(dev.checkpoint), dev.scale.float().cpu().numpy().astype(np.float16),
                       np.zeros((B, L, H, 128), np.float32), np.zeros((B, L, HV, 128), np.float32),
                       np.zeros((B, L, HV), np.float32), np.zeros((B, L, HV), np.float32))
    pos = (np.arange(B) % L).astype(np.int32)
    dev.pos.copy_(torch.from_numpy(pos).to(device))
    al, db = torch.from_numpy(a_log).to(device), torch.from_numpy(dt_bias).to(device)
    err = torch.zeros(1, dtype=torch.int32, device=device)
    for t in range(L):
        mixed, a, b = raw_inputs(rng, B, H, HV)
        out = torch.empty(B, HV, 128, dtype=torch.float32, device=device)
        q_out = torch.empty(B, H, 128, dtype=torch.bfloat16, device=device)
        nxt = torch.empty_like(dev.pos)
        dev.step(torch.from_numpy(mixed).to(device, torch.bfloat16), torch.from_numpy(a).to(device, torch.bfloat16),
                 torch.from_numpy(b).to(device, torch.bfloat16), al, db, out=out, q_out=q_out, pos_out=nxt,
                 error_flag=err)
        for i in range(B):
            p = pos[i]
            host.k_ring[i, p] = to_np(dev.k_ring[i, p])
            host.v_ring[i, p] = to_np(dev.v_ring[i, p])
            host.g_ring[i, p] = to_np(dev.g_ring[i, p])
            host.beta_ring[i, p] = to_np(dev.beta_ring[i, p])
        ref = O.replay_step(host, to_np(q_out), pos, out_dtype="f32")
        assert O.relative_l2(to_np(out), ref) < TOL_F32_KERNEL, (device, t)
        for i in np.nonzero(pos == L - 1)[0]:  # continue from the device's checkpoint (judged elsewhere)
            host.payload[i] = to_np(dev.checkpoint[i])
            host.scale[i] = dev.scale[i].float().cpu().numpy().astype(np.float16)
        dev.pos.copy_(nxt)
        pos = (pos + 1) % L
    assert int(err.item()) == 0


def test_bounded_wait_times_out_and_returns(cuda_device):
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    report = torch.full((4,), 7, dtype=torch.int64, device="cuda")
    rc = _lib.load().gdnr_selftest_wait_timeout(err.data_ptr(), report.data_ptr(), _lib.stream_handle())
    assert rc == _lib.OK
    torch.cuda.synchronize()
    assert int(err.item()) & _lib.DEVERR_WAIT_TIMEOUT
    ok0, ok1, ns0, ns1 = report.cpu().tolist()
    assert ok0 == 0 and ok1 == 0  # both waits gave up
    assert 0.9e9 <= ns0 <= 5e9, ns0  # the 1 s limit, measured on the device's global timer
    assert ns1 <= ns0 + 0.5e9, (ns0, ns1)  # the second wait ended through the abort word
    # the context is healthy and every SM's tensor memory is free again
    _step_vs_oracle("cuda:0", seed=71, B=64)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two visible GPUs")
def test_second_device_after_first(cuda_device):
    _step_vs_oracle("cuda:0", seed=72)
    _step_vs_oracle("cuda:1", seed=73)
    _step_vs_oracle("cuda:0", seed=74)
