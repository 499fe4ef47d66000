"""gdnr_packed_decode (the serving engine's decode call over a state-slot pool,
bench_gdn_full_contract.py:157-170 call shape) against gdn_fused_step on the
same slots gathered into a contiguous batch: bit-identical outputs and state;
null rows (index <= 0, the production op's NULL_BLOCK_ID test) and rows with an
index >= slots get zero outputs and leave every slot's state untouched."""

import numpy as np
import pytest
import torch

import gdnr
from helpers import gate_params, raw_inputs, to_dev

pytestmark = pytest.mark.gpu

STATE = ("checkpoint", "scale", "k_ring", "v_ring", "g_ring", "beta_ring", "pos")


def raw(t):
    """Byte view of an e4m3 tensor (indexing and comparisons on the codes)."""
    return t.view(torch.uint8) if t.dtype == torch.float8_e4m3fn else t


def make_pool(rng, S, H, HV, L):
    """S slots with random checkpoints, rings filled by L plain fused steps and
    distinct ring positions."""
    pool = gdnr.ReplayState.allocate(S, H, HV, L, scale_dtype=torch.float32, gate_dtype=torch.float32)
    pool.load_state(to_dev((0.02 * rng.standard_normal((S, HV, 128, 128))).astype(np.float32), torch.float32))
    a_log, dt_bias = gate_params(rng, HV)
    for t in range(L - 1):
        mixed, a, b = raw_inputs(rng, S, H, HV)
        pool.pos.fill_(t)
        pool.step(to_dev(mixed, torch.bfloat16), to_dev(a, torch.bfloat16), to_dev(b, torch.bfloat16),
                  to_dev(a_log, torch.float32), to_dev(dt_bias, torch.float32), flush_hint="none")
    pool.pos.copy_(to_dev(rng.integers(0, L, S).astype(np.int32), torch.int32))
    return pool, a_log, dt_bias


def gather(pool, slots):
    sub = gdnr.ReplayState.allocate(len(slots), pool.k_ring.shape[2], pool.v_ring.shape[2], pool.k_ring.shape[1],
                                    scale_dtype=pool.scale.dtype, gate_dtype=pool.g_ring.dtype)
    idx = torch.tensor(slots, dtype=torch.long, device="cuda")
    for name in STATE:
        raw(getattr(sub, name)).copy_(raw(getattr(pool, name)).index_select(0, idx))
    return sub


@pytest.mark.parametrize("heads", [(2, 4), (2, 2)])
@pytest.mark.parametrize("pdl", [False, True])
def test_packed_decode_matches_fused_step_on_gathered_slots(cuda_device, heads, pdl):
    rng = np.random.default_rng(31)
    H, HV = heads
    S, L = 7, 4
    rows = [3, 0, 5, 1, 6, -1]  # rows 1 and 5 are padding (null: index <= 0)
    active = [i for i, s in enumerate(rows) if s > 0]
    pool, a_log, dt_bias = make_pool(rng, S, H, HV, L)
    ref = gather(pool, [rows[i] for i in active])
    untouched = {name: raw(getattr(pool, name))[[0, 2, 4]].clone() for name in STATE}
    sidx = torch.tensor(rows, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    al, db = to_dev(a_log, torch.float32), to_dev(dt_bias, torch.float32)
    for _ in range(L + 2):  # crosses a flush of every slot
        mixed, a, b = raw_inputs(rng, len(rows), H, HV)
        m, aa, bb = to_dev(mixed, torch.bfloat16), to_dev(a, torch.bfloat16), to_dev(b, torch.bfloat16)
        out = torch.full((len(rows), 1, HV, 128), 7.0, dtype=torch.bfloat16, device="cuda")
        gdnr.fused_recurrent_gated_delta_rule_packed_decode(m, aa, bb, al, db, 128 ** -0.5, pool, out, sidx,
                                                            use_qk_l2norm_in_kernel=True, error_flag=err, pdl=pdl)
        nxt = torch.empty_like(ref.pos)
        want = ref.step(m[active], aa[active], bb[active], al, db,
                        out=torch.empty(len(active), HV, 128, dtype=torch.bfloat16, device="cuda"), pos_out=nxt)
        ref.pos.copy_(nxt)
        torch.cuda.synchronize()
        assert torch.equal(out[active].view(len(active), HV, 128), want)
        assert torch.all(out[1] == 0) and torch.all(out[5] == 0)  # padding rows: zeros, as the production op
    assert int(err.item()) == 0
    for name in STATE:
        assert torch.equal(raw(getattr(pool, name))[[rows[i] for i in active]], raw(getattr(ref, name))), name
        assert torch.equal(raw(getattr(pool, name))[[0, 2, 4]], untouched[name]), name


def test_packed_decode_out_of_range_slot_is_reported_and_skipped(cuda_device):
    rng = np.random.default_rng(32)
    H, HV, S, L = 2, 4, 4, 4
    pool, a_log, dt_bias = make_pool(rng, S, H, HV, L)
    before = {name: raw(getattr(pool, name)).clone() for name in STATE}
    sidx = torch.tensor([2, 9], dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    mixed, a, b = raw_inputs(rng, 2, H, HV)
    out = torch.full((2, HV, 128), 5.0, dtype=torch.float32, device="cuda")
    gdnr.fused_recurrent_gated_delta_rule_packed_decode(
        to_dev(mixed, torch.bfloat16), to_dev(a, torch.bfloat16), to_dev(b, torch.bfloat16),
        to_dev(a_log, torch.float32), to_dev(dt_bias, torch.float32), 128 ** -0.5, pool, out, sidx, error_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) & gdnr._lib.DEVERR_BAD_SLOT
    assert torch.all(out[1] == 0) and not torch.all(out[0] == 0)
    assert int(pool.pos[2]) == (int(before["pos"][2]) + 1) % L
    for s in (0, 1, 3):
        for name in STATE:
            assert torch.equal(raw(getattr(pool, name))[s], before[name][s]), (s, name)
