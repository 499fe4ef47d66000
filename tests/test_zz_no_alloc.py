"""gdnr_replay_split_static (the split replay with library-owned scratch) vs
gdnr_replay_split with caller buffers, through the C ABI.

Collected last on purpose: it must also pass after every other test has run
in the same process (and alone, in a fresh process, where its first call sets
up the scratch address).
"""

import numpy as np
import pytest
import torch

import gdnr
import oracle as O
from helpers import e4m3_dev, ring_inputs, to_dev, to_np

pytestmark = pytest.mark.gpu


def _case(seed, B, L, H, HV):
    rng = np.random.default_rng(seed)
    d = ring_inputs(rng, B, L, H, HV)
    ck = O.quantize_checkpoint(d["state"], "vblock", 32)
    valid = rng.integers(0, L + 1, size=B).astype(np.int32)
    args = (e4m3_dev(ck.payload), to_dev(ck.scale.astype(np.float32), torch.float16), to_dev(d["q"], torch.float32),
            to_dev(d["k"], torch.bfloat16), to_dev(d["v"], torch.bfloat16), to_dev(d["g"], torch.float32),
            to_dev(d["beta"], torch.float32), to_dev(valid, torch.int32))
    return args


def test_split_static_matches_split_twice_in_a_row(cuda_device):
    B, L, H, HV = 6, 8, 2, 4
    for call, seed in enumerate((41, 42)):  # two calls in a row on the shared scratch
        args = _case(seed, B, L, H, HV)
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


def test_split_static_rejects_oversized_batch(cuda_device):
    B, L, H, HV = 1, 4, 2, 4
    args = list(_case(43, B, L, H, HV))
    # a ring claiming more (sequence, value head) pairs than the scratch holds
    k = torch.zeros(1100, L, H, 128, dtype=torch.bfloat16, device="cuda")
    v = torch.zeros(1100, L, HV, 128, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(1100, HV, 128, dtype=torch.float32, device="cuda")
    with pytest.raises(gdnr.GdnrError, match="static scratch"):
        gdnr.gdn_replay_fp8_split_static(args[0], args[1], args[2], k, v, args[5], args[6], args[7], out=out)
