"""gdnr_replay_split_static (the split replay with library-owned scratch,
through the C ABI) against gdnr_replay_split with caller buffers and against
the oracle's backward replay (kern.py:121-176), and a check that a call
allocates no device memory.

Collected last on purpose: it must also pass after every other test has run
in the same process (and alone, in a fresh process, where its first call sets
up the scratch address).
"""

import numpy as np
import pytest
import torch

import gdnr
import oracle as O
from helpers import TOL_F32_KERNEL, e4m3_dev, ring_inputs, to_dev, to_np

pytestmark = pytest.mark.gpu


def _case(seed, B, L, H, HV, valid=None):
    rng = np.random.default_rng(seed)
    d = ring_inputs(rng, B, L, H, HV)
    ck = O.quantize_checkpoint(d["state"], "vblock", 32)
    if valid is None:
        valid = rng.integers(0, L + 1, size=B).astype(np.int32)
    args = (e4m3_dev(ck.payload), to_dev(ck.scale.astype(np.float32), torch.float16), to_dev(d["q"], torch.float32),
            to_dev(d["k"], torch.bfloat16), to_dev(d["v"], torch.bfloat16), to_dev(d["g"], torch.float32),
            to_dev(d["beta"], torch.float32), to_dev(valid, torch.int32))
    want = O.replay_adjoint(O.dequantize_checkpoint(ck), d["q"], d["k"], d["v"], d["g"], d["beta"], valid)
    return args, want


def test_split_static_matches_split_and_oracle_twice_in_a_row(cuda_device):
    B, L, H, HV = 6, 8, 2, 4
    for call, seed in enumerate((41, 42)):  # two calls in a row on the shared scratch
        args, want = _case(seed, B, L, H, HV)
        tq = torch.empty(B, HV, 128, dtype=torch.float32, device="cuda")
        coef = torch.empty(B, HV, L, dtype=torch.float32, device="cuda")
        ref = torch.empty(B, HV, 128, dtype=torch.float32, device="cuda")
        gdnr.gdn_replay_fp8_split(*args, tq, coef, out=ref)
        got = torch.full((B, HV, 128), float("nan"), dtype=torch.float32, device="cuda")
        gdnr.gdn_replay_fp8_split_static(*args, out=got)
        torch.cuda.synchronize()
        # same kernels on the same inputs: identical up to nothing but buffer placement
        assert torch.isfinite(got).all(), call
        assert O.relative_l2(to_np(got), to_np(ref)) < 1e-6, call
        # and the oracle's backward replay on the dequantised checkpoint
        assert O.relative_l2(to_np(got), want) < TOL_F32_KERNEL, call


def test_split_static_allocates_nothing(cuda_device):
    B, L, H, HV = 6, 8, 2, 4
    args, want = _case(44, B, L, H, HV)
    out = torch.empty(B, HV, 128, dtype=torch.float32, device="cuda")
    gdnr.gdn_replay_fp8_split_static(*args, out=out)  # first call on this device: scratch set-up, kernel loading
    torch.cuda.synchronize()
    torch_before = torch.cuda.memory_allocated()
    free_before, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        gdnr.gdn_replay_fp8_split_static(*args, out=out)
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert torch.cuda.memory_allocated() == torch_before
    assert free_after == free_before, f"device free memory changed by {free_before - free_after} bytes"
    assert O.relative_l2(to_np(out), want) < TOL_F32_KERNEL


def test_split_static_empty_chains(cuda_device):
    """valid_len = 0 everywhere: o = S q K^-1/2 from the checkpoint alone."""
    B, L, H, HV = 3, 4, 2, 4
    args, want = _case(45, B, L, H, HV, valid=np.zeros(3, np.int32))
    out = torch.full((B, HV, 128), float("nan"), dtype=torch.float32, device="cuda")
    gdnr.gdn_replay_fp8_split_static(*args, out=out)
    torch.cuda.synchronize()
    assert O.relative_l2(to_np(out), want) < TOL_F32_KERNEL


def test_split_static_rejects_oversized_batch(cuda_device):
    B, L, H, HV = 1, 4, 2, 4
    args, _ = _case(43, B, L, H, HV)
    # a ring claiming more (sequence, value head) pairs than the scratch holds
    k = torch.zeros(1100, L, H, 128, dtype=torch.bfloat16, device="cuda")
    v = torch.zeros(1100, L, HV, 128, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(1100, HV, 128, dtype=torch.float32, device="cuda")
    with pytest.raises(gdnr.GdnrError, match="static scratch"):
        gdnr.gdn_replay_fp8_split_static(args[0], args[1], args[2], k, v, args[5], args[6], args[7], out=out)


def test_split_static_rejects_huge_head_count_without_overflow(cuda_device):
    """B = 4 and HV = 2^62 claimed in the descriptors: B*HV wraps a 64-bit
    product; each extent is bounded before the product is formed, so the call
    is rejected before anything is read or launched."""
    import ctypes

    from gdnr import _lib

    args, _ = _case(46, 1, 4, 2, 4)
    out = torch.empty(1, 4, 128, dtype=torch.float32, device="cuda")
    a = _lib.ReplaySplitStaticArgs()
    for name, t in zip(("checkpoint", "scale", "q", "k_ring", "v_ring", "g_ring", "beta_ring", "valid_len"), args):
        setattr(a, name, _lib.tensor_desc(t))
    a.out = _lib.tensor_desc(out)
    a.block_v = 32
    a.k_ring.shape[0] = 4
    a.v_ring.shape[2] = 1 << 62
    rc = _lib.load().gdnr_replay_split_static(ctypes.byref(a), _lib.stream_handle())
    assert rc == _lib.ERR_UNSUPPORTED
    assert b"static scratch" in _lib.load().gdnr_last_error()
