"""Multi-rank host logic on CPU (gloo, world size 2): the batch shards of the
sequence-sharded path, the max-over-ranks timing reduction, and that sharding
does not change any sequence's result.  The numpy oracle stands in for the
per-rank device step (no GPU here); failures are made on the host."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from gdnr.shard import ShardPlan, gather_shards, max_over_ranks, shard_range


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _global_case(B, T, H=2, HV=4, L=4, seed=5):
    """Seeded global inputs of a full-contract run: initial ring state + T steps of raw inputs."""
    rng = np.random.default_rng(seed)
    s0 = (0.02 * rng.standard_normal((B, HV, 128, 128))).astype(np.float32)
    q0 = O.quantize_checkpoint(s0, "vblock", 32)
    st = O.RingState(q0.payload.copy(), q0.scale.copy(), np.zeros((B, L, H, 128), np.float32),
                     np.zeros((B, L, HV, 128), np.float32), np.zeros((B, L, HV), np.float32),
                     np.zeros((B, L, HV), np.float32))
    width = 2 * H * 128 + HV * 128
    mixed = O.bf16_round(rng.standard_normal((T, B, width)).astype(np.float32))
    a = O.bf16_round(rng.standard_normal((T, B, HV)).astype(np.float32))
    b = O.bf16_round(rng.standard_normal((T, B, HV)).astype(np.float32))
    a_log = np.log(1.0 + 15.0 * rng.random(HV)).astype(np.float32)
    dt_bias = (0.5 * rng.standard_normal(HV)).astype(np.float32)
    pos0 = rng.integers(0, L, B).astype(np.int32)
    return st, mixed, a, b, a_log, dt_bias, pos0, H, L


def _run(st, mixed, a, b, a_log, dt_bias, pos0, H, L, rows):
    """T oracle steps of sequences ``rows``; returns outputs [T, n, HV, V] and the final payload."""
    sub = O.RingState(*(x[rows].copy() for x in (st.payload, st.scale, st.k_ring, st.v_ring, st.g_ring,
                                                 st.beta_ring)))
    pos = pos0[rows].copy()
    outs = []
    for t in range(mixed.shape[0]):
        out, _ = O.fused_step(sub, mixed[t, rows], a[t, rows], b[t, rows], a_log, dt_bias, pos, H, 128,
                              out_dtype="f32", gate_dtype="f32")
        outs.append(out)
        pos = (pos + 1) % L
    return np.stack(outs), sub.payload


def _worker_sharded(rank, world, port, B, T, q):
    _init(rank, world, port)
    try:
        case = _global_case(B, T)
        plan = ShardPlan(B, world)
        rows = np.arange(B)[plan.local(rank).start:plan.local(rank).stop]
        out, payload = _run(*case, rows)
        got_out = gather_shards(torch.from_numpy(np.moveaxis(out, 1, 0).copy()), plan)
        got_pay = gather_shards(torch.from_numpy(payload), plan)
        slowest = max_over_ranks(1.0 + rank)
        if rank == 0:
            ref_out, ref_pay = _run(*case, np.arange(B))
            q.put((np.array_equal(got_out.numpy(), np.moveaxis(ref_out, 1, 0)),
                   np.array_equal(got_pay.numpy(), ref_pay), slowest))
    finally:
        dist.destroy_process_group()


def _worker_failing(rank, world, port):
    _init(rank, world, port, timeout_s=5)
    try:
        if rank == 1:
            raise RuntimeError("rank 1 fails before the timing reduction")
        max_over_ranks(1.0)  # rank 0 waits for a peer that never comes
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("B,world", [(5, 2), (64, 2), (7, 3), (2, 4), (0, 2), (148, 8)])
def test_shard_ranges_partition_the_batch(B, world):
    rgs = [shard_range(B, world, r) for r in range(world)]
    assert [i for rg in rgs for i in rg] == list(range(B))
    assert max(map(len, rgs)) - min(map(len, rgs)) <= 1
    plan = ShardPlan(B, world)
    for s in range(B):
        assert s in plan.local(plan.owner(s))
    x = torch.arange(B * 3).reshape(B, 3)
    assert torch.equal(torch.cat([plan.take(x, r) for r in range(world)]), x)


def test_shard_plan_rejects_bad_arguments():
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)
    with pytest.raises(ValueError):
        ShardPlan(4, 2).take(torch.zeros(5, 1), 0)
    with pytest.raises(ValueError):
        ShardPlan(4, 2).owner(4)


def test_gloo_two_ranks_sharded_run_equals_unsharded():
    """Two ranks run uneven shards (3 + 2 sequences) of a 6-step full-contract run
    crossing a flush; the gathered outputs and re-quantised checkpoints equal the
    single-process run bit for bit, and the timing reduction returns the max."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.spawn(_worker_sharded, args=(2, _free_port(), 5, 6, q), nprocs=2, join=True)
    out_ok, pay_ok, slowest = q.get(timeout=60)
    assert out_ok and pay_ok
    assert slowest == 2.0


def test_gloo_failed_rank_ends_the_collective_with_an_error():
    """A rank that raises before the timing reduction: the other rank's
    collective ends with an error within the process-group timeout instead of
    waiting for ever, and the launcher reports the failure."""
    with pytest.raises(Exception):
        mp.spawn(_worker_failing, args=(2, _free_port()), nprocs=2, join=True)
