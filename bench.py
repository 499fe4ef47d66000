#!/usr/bin/env python
"""Benchmark of the fused FP8-replay GDN decode step on B200.

Workload (BASELINE config 3 at the metric's point, batch 64, L = 16): one
*step* is one decode token through a stack of NL independent GDN layers,
each a single ``gdn_fused_step`` launch (prep + ring append + replay, and the
flush/re-quantisation on the L-th token of the ring cycle) at batch 64,
H = 16, HV = 32, K = V = 128.  Steps walk the ring cycle, so the flush cost
is amortised exactly as in the reference's cycle model
(prototype/bench_gdn_full_contract.py:225-308).  NL layers x ~46 MB of state
(> 2x the 126 MB L2) keep every launch reading its state from HBM.

The metric is decode steps.seq/s per GDN layer: (steps x NL x batch) / time.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU: one process per GPU (torchrun), each rank runs its own batch of
64 sequences (weak scaling over independent sequence shards); no collective
on the data path -- only the barrier and the max-over-ranks of the timing.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import pathlib
import statistics
import sys
import threading
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "fp8-replayssm-gdn-kernel_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "GDN decode steps·seq/s @batch64 L=16; achieved HBM GB/s vs B200 peak"
UNIT = "steps·seq/s"
H, HV, KD = 16, 32, 128
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1024)
    ap.add_argument("--warmup", type=int, default=32)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ring", type=int, default=16)
    ap.add_argument("--layers", type=int, default=8, help="independent layer states (default 8: 368 MB > 2x L2)")
    ap.add_argument("--e2e-steps", type=int, default=64)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-core", action="store_true", help="skip the core-replay (config 2) measurement")
    ap.add_argument("--profile", type=int, default=None, metavar="POS",
                    help="profiling driver for ncu: a few untimed launches of one layer's step at ring position "
                         "POS (no timing, no JSON line)")
    ap.add_argument("--checkpoint", choices=["e4m3", "int8"], default="e4m3",
                    help="checkpoint payload of the --profile driver (int8: the 'vblock_int8' option)")
    return ap.parse_args()


# ---------------------------------------------------------------- helpers

def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profile_traffic():
    """dram bytes per launch of the step kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "step5_kernel_b64_l16.md"
    try:
        for line in p.read_text().splitlines():
            if line.startswith("dram_bytes_per_launch_cycle_avg"):
                return int(float(line.split("=")[1].strip()))
    except Exception:
        pass
    return None


class ClockSampler:
    """NVML sampling of SM clock and clock-event reasons during the timed region."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int):
        self.samples, self.reasons, self.ok = [], set(), False
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = self._handle(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # no NVML: report that instead of numbers
            self.err = repr(e)

    def _handle(self, idx):
        import torch

        pynvml = self.nvml
        try:
            props = torch.cuda.get_device_properties(idx)
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except Exception:
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            phys = int(vis.split(",")[idx]) if vis else idx
            return pynvml.nvmlDeviceGetHandleByIndex(phys)

    def _run(self):
        n = self.nvml
        while not self._stop.is_set():
            try:
                self.samples.append(n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM))
                try:
                    r = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                except AttributeError:
                    r = n.nvmlDeviceGetCurrentClocksThrottleReasons(self.handle)
                for bit, name in self.REASONS.items():
                    if r & bit and bit != 0x1:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": f"NVML unavailable: {self.err}"}
        med = statistics.median(self.samples) if self.samples else None
        return {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


def dist_init():
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    from gdnr.shard import max_over_ranks as reduce_max

    return reduce_max(x)


def barrier(world: int):
    import torch

    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


# ---------------------------------------------------------------- CPU baseline (oracle port)

def cpu_units(units_per_worker: int, workers: int, seed: int, ring_len: int):
    """Run the oracle port on `workers` spawned processes; returns (units, seconds)."""
    import multiprocessing as mp

    from oracle import cpu_bench

    ctx = mp.get_context("spawn")
    with ctx.Pool(workers, initializer=cpu_bench.worker_init, initargs=(seed, ring_len)) as pool:
        pool.map(cpu_bench.run_units, [1] * workers)  # warm the workers
        t0 = time.perf_counter()
        res = pool.map(cpu_bench.run_units, [units_per_worker] * workers)
        wall = time.perf_counter() - t0
    return sum(r[0] for r in res), wall


def cpu_workers():
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:
        return max(1, os.cpu_count() or 1)


def cpu_baseline(seed: int, ring_len: int, target_s: float = 15.0):
    workers = cpu_workers()
    _, probe = cpu_units(1, workers, seed, ring_len)  # one unit per worker: sizes the sample
    per_unit = max(probe, 1e-3)
    n = max(ring_len, int(target_s / per_unit))
    n = (n + ring_len - 1) // ring_len * ring_len  # whole ring cycles (the flush included)
    units, wall = cpu_units(n, workers, seed, ring_len)
    return {"value": units / wall, "unit": UNIT, "cores": workers, "kind": "port",
            "sample": f"{units} sequence-layer steps ({workers} processes x {n} steps = whole L={ring_len} ring "
                      f"cycles incl. the flush) of the numpy oracle port of replay_decode, {wall:.1f} s wall"}


def run_reference(args, world, rank):
    """--impl reference: the reference's CPU implementation of the path (oracle port)."""
    if rank != 0:
        return
    workers = cpu_workers()
    # size each step's sample so the whole run stays within a few minutes:
    # one unit per worker per step; cap total steps timed by the budget
    budget_s = 150.0
    probe_units, probe_wall = cpu_units(1, workers, args.seed, args.ring)
    per_step = probe_wall if probe_wall > 0 else 0.05
    steps = args.steps
    units_per_step = workers
    while steps * per_step > budget_s and steps > 1:
        steps //= 2
    t_units, t_wall = cpu_units(max(1, steps), workers, args.seed, args.ring)
    value = t_units / t_wall
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": steps,
        "warmup": 1,
        "ms_per_step": 1e3 * t_wall / max(1, steps),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded, BASELINE config 1/3 distributions)",
        "config": {"workload": f"config3 full-contract step, one GDN layer, L={args.ring}, CPU sample",
                   "global_batch": units_per_step, "seq_len": args.ring, "parallelism": f"{workers} processes"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": workers, "kind": "port",
                         "sample": f"{t_units} sequence-layer steps ({units_per_step} sequences per step, "
                                   f"{steps} steps) of the numpy oracle port of replay_decode"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference is a Python/Triton prototype that cannot be installed (no setup.py/pyproject); "
                "its CPU path (ref.py replay_decode) is timed through the repo's numpy restatement",
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU arm

def build_stack(args, device, rank: int = 0, world: int = 1, checkpoint_dtype=None):
    """This rank's shard of the job: sequences ShardPlan(B * world, world).local(rank)
    of every layer, each rank with its own seeded inputs and state (weak scaling)."""
    import torch

    import gdnr
    from gdnr import inputs as gin
    from gdnr.shard import ShardPlan

    B, L, NL = args.batch, args.ring, args.layers
    shard = ShardPlan(B * world, world).local(rank)
    assert len(shard) == B
    layers, step_inputs = [], []
    for li in range(NL):
        st = gdnr.ReplayState.allocate(B, H, HV, L, device=device, scale_dtype=torch.float32,
                                       gate_dtype=torch.float32,
                                       checkpoint_dtype=checkpoint_dtype or torch.float8_e4m3fn)
        raw = gin.raw_step_inputs(B, L, seed=(args.seed * 1000 + li) * 4096 + shard.start, device=device)
        st.load_state(raw["state"])
        layers.append({"state": st, "a_log": raw["a_log"], "dt_bias": raw["dt_bias"],
                       "out": torch.empty(B, HV, KD, dtype=torch.bfloat16, device=device)})
        # distinct raw inputs per (layer, ring position), resident in HBM
        step_inputs.append([(raw["mixed_qkv"][:, s].contiguous(), raw["a"][:, s].contiguous(),
                             raw["b"][:, s].contiguous()) for s in range(L)])
        del raw
    pos = [torch.full((B,), s, dtype=torch.int32, device=device) for s in range(L)]
    err = torch.zeros(1, dtype=torch.int32, device=device)
    return layers, step_inputs, pos, err


def flush_hint_for(s: int, L: int) -> str:
    """All sequences share the ring position here, so whether this step flushes
    is known on the host: no sequence ("none") or every sequence ("all")."""
    return "all" if s == L - 1 else "none"


def launch_position(layers, step_inputs, pos, err, s):
    import gdnr

    L = len(pos)
    for li, lay in enumerate(layers):
        st = lay["state"]
        mixed, a, b = step_inputs[li][s]
        gdnr.gdn_fused_step(mixed, a, b, lay["a_log"], lay["dt_bias"], pos[s], st.checkpoint, st.scale, st.k_ring,
                            st.v_ring, st.g_ring, st.beta_ring, out=lay["out"], error_flag=err,
                            flush_hint=flush_hint_for(s, L))


def run_profile(args, local):
    """A few eager launches of one layer's fused step at one ring position (ncu target)."""
    import torch

    args.layers = 1
    device = torch.device("cuda", local)
    layers, step_inputs, pos, err = build_stack(
        args, device, checkpoint_dtype=torch.int8 if args.checkpoint == "int8" else None)
    s = args.profile % args.ring
    for _ in range(3):
        launch_position(layers, step_inputs, pos, err, s)
    torch.cuda.synchronize()
    print(f"profile: 3 launches at ring position {s}, device error word {int(err.item())}", flush=True)


def run_ours(args, world, rank, local):
    import torch

    import gdnr
    from oracle import gdn_oracle as O

    device = torch.device("cuda", local)
    B, L, NL = args.batch, args.ring, args.layers
    cpu_line = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_line = cpu_baseline(args.seed, L)  # spawn pool; GPU untouched so far

    layers, step_inputs, pos, err = build_stack(args, device, rank, world)
    stream = torch.cuda.Stream(device)
    torch.cuda.synchronize()
    # one graph per ring position: NL fused launches
    graphs = []
    with torch.cuda.stream(stream):
        for s in range(L):  # eager pass: lazy loading + smem attribute before capture
            launch_position(layers, step_inputs, pos, err, s)
    torch.cuda.synchronize()
    for s in range(L):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            launch_position(layers, step_inputs, pos, err, s)
        graphs.append(g)
    torch.cuda.synchronize()

    step_idx = 0
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graphs[step_idx % L].replay()
            step_idx += 1
    barrier(world)
    # one event between consecutive graph replays: per-position durations give
    # each kernel's average launch time (non-flush positions -> the persistent
    # step kernel; the flush position -> the flush kernel)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    positions = []
    sampler = ClockSampler(local)
    with sampler:
        with torch.cuda.stream(stream):
            evs[0].record(stream)
            for i in range(args.steps):
                positions.append(step_idx % L)
                graphs[step_idx % L].replay()
                step_idx += 1
                evs[i + 1].record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms = evs[0].elapsed_time(evs[-1])
    ms_max = max_over_ranks(ms, world)
    dev_err = int(err.item())
    step_ms = [evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]

    launches = args.steps * NL
    units = launches * B * world
    value = units / (ms_max / 1e3)
    # algorithmic bytes, averaged over the ring cycle actually timed
    cyc = [O.algorithmic_bytes(B, p + 1, L, scale_bytes=4, gate_bytes=4, ab_bytes=2) for p in positions]
    bytes_per_launch = sum(cyc) / len(cyc)
    peak, peak_kind = measured_peak()
    kernels = {}
    for name, sel in (("step5_kernel<flush=false> (non-flush steps)", lambda p: p != L - 1),
                      ("step5_kernel<flush=true> (flush step)", lambda p: p == L - 1)):
        idx = [i for i, p in enumerate(positions) if sel(p)]
        if not idx:
            continue
        t = sum(step_ms[i] for i in idx) / (len(idx) * NL) / 1e3
        b = sum(cyc[i] for i in idx) / len(idx)
        kernels[name] = {"launches": len(idx) * NL, "us_per_launch": t * 1e6, "algorithmic_bytes_per_launch": b,
                         "achieved_GB_s": b / t / 1e9, "frac_of_peak": b / t / 1e9 / peak}
    dom = max(kernels, key=lambda k: kernels[k]["launches"] * kernels[k]["us_per_launch"])
    achieved = kernels[dom]["achieved_GB_s"]

    # ---- end to end through the public API with host buffers (pinned), per layer-step
    e2e = run_e2e(args, layers, step_inputs, pos, stream, world) if args.e2e_steps > 0 else None

    core = None
    widened = None
    if not args.no_core and world == 1:
        core = run_core(args, device, stream)
        widened = run_widened(args, device, stream)
        widened["comparators"] = run_comparators(args, device, stream, 1e3 * ms_max / launches)

    del graphs
    torch.cuda.synchronize()
    if rank != 0:
        return
    line = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_max / args.steps,
        "us_per_layer_step": 1e3 * ms_max / launches,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "e4m3/f32",
        "data": "synthetic (seeded; BASELINE config 1/3 distributions; random state N(0,0.02))",
        "config": {
            "workload": f"config3 fused full-contract step (prep+ring append+replay, flush every {L}), "
                        f"batch {B}/GPU, L={L}, cycle-amortised; one step = one token through {NL} independent "
                        "GDN layers (one launch each)",
            "global_batch": B * world, "seq_len": L, "parallelism": f"sequence-shard x{world} (no collective)",
            "heads": H, "value_heads": HV, "head_dim": KD, "layers": NL,
            "l2": f"inputs larger than L2: {NL} layer states x {layers[0]['state'].nbytes() / 1e6:.1f} MB",
        },
        "gpu_launches": launches,
        "device_error_word": dev_err,
        "clocks": sampler.summary(),
        "roofline": {
            "bound": "hbm",
            "kernel": dom,
            "achieved": achieved,
            "peak": peak,
            "peak_kind": peak_kind,
            "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": profile_traffic(),
            "algorithmic_bytes_per_launch": kernels[dom]["algorithmic_bytes_per_launch"],
            "note": "achieved = the kernel's algorithmic bytes per launch (averaged over the positions it ran) / "
                    "its average launch time from CUDA events between graph replays on the launch stream",
        },
        "kernels": kernels,
        "cycle_algorithmic_bytes_per_launch": bytes_per_launch,
    }
    if e2e is not None:
        line["e2e"] = e2e
    if core is not None:
        line["core_replay"] = core
    if widened is not None:
        line.update(widened)
    if cpu_line is not None:
        line["cpu_baseline"] = cpu_line
    print(json.dumps(line), flush=True)


def run_e2e(args, layers, step_inputs, pos, stream, world):
    """Public-API step with the step's inputs copied from pinned host memory and
    the output read back to pinned host memory, inside the timed region.

    The way a serving loop runs it: per ring position one CUDA graph, captured
    through the public API (gdnr.gdn_fused_step), holding for every layer one
    host-to-device copy of the step's packed raw inputs (q/k/v projections and
    the two gate inputs) from pinned memory, the step kernel, and one
    device-to-host copy of its output to pinned memory.  The copies run on
    their own streams (forked and joined inside the capture), so the PCIe
    traffic of one layer overlaps the kernels of the others; every step's copies
    are inside the timed region.  The input copies alternate between two
    streams: one stream's pinned copies reach ~24 GB/s on the B200 box, two
    concurrent ones ~32-35 GB/s."""
    import torch

    import gdnr

    B, L = args.batch, args.ring
    dev = layers[0]["out"].device
    parts = [(t.dtype, tuple(t.shape), t.numel() * t.element_size()) for t in step_inputs[0][0]]
    nbytes = sum(n for _, _, n in parts)
    assert all(n % 16 == 0 for _, _, n in parts)

    def pack(ts):
        return torch.cat([t.contiguous().view(-1).view(torch.uint8) for t in ts]).cpu().pin_memory()

    def views(buf):
        out, off = [], 0
        for dt, shape, n in parts:
            out.append(buf[off:off + n].view(dt).view(shape))
            off += n
        return out

    nl = len(layers)
    host_in = [[pack(step_inputs[li][s]) for s in range(L)] for li in range(nl)]
    dev_in = [torch.empty(nbytes, dtype=torch.uint8, device=dev) for _ in range(nl)]
    dev_views = [views(b) for b in dev_in]
    dev_out = [torch.empty(B, HV, KD, dtype=torch.bfloat16, device=dev) for _ in range(nl)]
    host_out = [torch.empty(B, HV, KD, dtype=torch.bfloat16).pin_memory() for _ in range(nl)]
    d2h = host_out[0].numel() * host_out[0].element_size()
    s_ins, s_out = (torch.cuda.Stream(), torch.cuda.Stream()), torch.cuda.Stream()

    def step_body(s):
        for s_in in s_ins:
            s_in.wait_stream(stream)
        s_out.wait_stream(stream)
        for li, lay in enumerate(layers):
            ev_in, ev_k = torch.cuda.Event(), torch.cuda.Event()
            s_in = s_ins[li % 2]
            with torch.cuda.stream(s_in):
                dev_in[li].copy_(host_in[li][s], non_blocking=True)
                ev_in.record(s_in)
            stream.wait_event(ev_in)
            mixed, a, b = dev_views[li]
            st = lay["state"]
            with torch.cuda.stream(stream):
                gdnr.gdn_fused_step(mixed, a, b, lay["a_log"], lay["dt_bias"], pos[s], st.checkpoint, st.scale,
                                    st.k_ring, st.v_ring, st.g_ring, st.beta_ring, out=dev_out[li],
                                    flush_hint=flush_hint_for(s, L))
                ev_k.record(stream)
            s_out.wait_event(ev_k)
            with torch.cuda.stream(s_out):
                host_out[li].copy_(dev_out[li], non_blocking=True)
        for s_in in s_ins:
            stream.wait_stream(s_in)
        stream.wait_stream(s_out)

    # eager pass over the ring (warms up every path), then one graph per position
    for s in range(L):
        with torch.cuda.stream(stream):
            step_body(s)
    torch.cuda.synchronize()
    graphs = []
    for s in range(L):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step_body(s)
        graphs.append(g)
    with torch.cuda.stream(stream):
        for i in range(L):
            graphs[i % L].replay()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(args.e2e_steps):
            graphs[i % L].replay()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    del graphs
    units = args.e2e_steps * nl * B * world
    return {"value": units / (ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": nbytes * nl,
            "d2h_bytes_per_step": d2h * nl, "steps": args.e2e_steps,
            "path": "gdnr.gdn_fused_step (Python) -> libgdnr C ABI, captured per ring position in a CUDA graph "
                    "with, per layer, one pinned H2D copy of the packed raw inputs and one pinned D2H copy of the "
                    "output on forked streams (input copies alternate between two streams; copies overlap other layers' "
                    "kernels)"}


def _graph_us(fn, stream, reps):
    """Mean device time of ``fn`` (captured once in a CUDA graph) over ``reps`` replays."""
    import torch

    with torch.cuda.stream(stream):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn()
    with torch.cuda.stream(stream):
        for _ in range(3):
            g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    del g
    return 1e3 * e0.elapsed_time(e1) / reps


def run_widened(args, device, stream):
    """The rows beyond the core path, measured like it: the packed decode
    (serving call over a slot pool, one random slot per batch row) and the
    fused step on an INT8 checkpoint, each through a whole ring cycle, and the
    vblock32 codec (E4M3 and INT8) on a BASELINE-size state."""
    import torch

    import gdnr
    from gdnr import inputs as gin

    B, L, NL = args.batch, args.ring, min(args.layers, 4)
    S = 2 * B + 1
    gen = torch.Generator().manual_seed(args.seed + 17)
    pools = []
    for li in range(NL):
        pool = gdnr.ReplayState.allocate(S, H, HV, L, device=device, scale_dtype=torch.float32,
                                         gate_dtype=torch.float32)
        raw = gin.raw_step_inputs(S, L, seed=(args.seed * 1000 + li) * 4096 + 7, device=device)
        pool.load_state(raw["state"])
        idx = (torch.randperm(S - 1, generator=gen)[:B] + 1).to(torch.int32).to(device)
        posf = [torch.zeros(S, dtype=torch.int32, device=device).index_fill_(0, idx.long(), s) for s in range(L)]
        inputs = [(raw["mixed_qkv"][:B, s].contiguous(), raw["a"][:B, s].contiguous(), raw["b"][:B, s].contiguous())
                  for s in range(L)]
        pools.append((pool, idx, posf, inputs, raw["a_log"], raw["dt_bias"],
                      torch.empty(B, 1, HV, KD, dtype=torch.bfloat16, device=device)))
        del raw
    total = 0.0
    for s in range(L):
        def step(s=s):
            for pool, idx, posf, inputs, a_log, dt_bias, out in pools:
                pool.pos.copy_(posf[s])
                m, a, b = inputs[s]
                gdnr.fused_recurrent_gated_delta_rule_packed_decode(
                    m, a, b, a_log, dt_bias, KD ** -0.5, pool, out, idx, flush_hint=flush_hint_for(s, L))
        total += _graph_us(step, stream, 10) / NL
    packed_us = total / L
    del pools
    res = {"packed_decode": {
        "us_per_layer_step": packed_us, "steps_seq_per_s": B / (packed_us * 1e-6),
        "workload": f"fused_recurrent_gated_delta_rule_packed_decode: batch {B} rows on random slots of a "
                    f"{S}-slot pool (slot 0 null), {NL} layers, one ring cycle (flush at position {L - 1}); "
                    "includes the wrapper's position copies"}}
    # the INT8 checkpoint option ("vblock_int8") through the fused step, one ring cycle
    layers8 = []
    for li in range(NL):
        st = gdnr.ReplayState.allocate(B, H, HV, L, device=device, scale_dtype=torch.float32,
                                       gate_dtype=torch.float32, checkpoint_dtype=torch.int8)
        raw = gin.raw_step_inputs(B, L, seed=(args.seed * 1000 + li) * 4096 + 13, device=device)
        st.load_state(raw["state"])
        inputs = [(raw["mixed_qkv"][:, s].contiguous(), raw["a"][:, s].contiguous(), raw["b"][:, s].contiguous())
                  for s in range(L)]
        posf = [torch.full((B,), s, dtype=torch.int32, device=device) for s in range(L)]
        layers8.append((st, inputs, posf, raw["a_log"], raw["dt_bias"],
                        torch.empty(B, HV, KD, dtype=torch.bfloat16, device=device)))
        del raw
    total = 0.0
    for s in range(L):
        def step8(s=s):
            for st, inputs, posf, a_log, dt_bias, out in layers8:
                st.pos.copy_(posf[s])
                m, a, b = inputs[s]
                st.step(m, a, b, a_log, dt_bias, out=out, flush_hint=flush_hint_for(s, L))
        total += _graph_us(step8, stream, 10) / NL
    int8_us = total / L
    del layers8
    res["int8_checkpoint_step"] = {
        "us_per_layer_step": int8_us, "steps_seq_per_s": B / (int8_us * 1e-6),
        "workload": f"gdn_fused_step on an int8 ('vblock_int8') checkpoint, batch {B}, L={L}, {NL} layers, one "
                    "ring cycle (flush re-quantises to int8); one-CTA-per-head kernel with the integer "
                    "tensor-core readout; includes a position copy per layer"}
    # codec: [B, HV, V, K] float32 state (134 MB > L2)
    state = torch.randn(B, HV, KD, KD, generator=gen).mul_(0.05).to(device)
    codec = {}
    n = state.numel()
    for gran, pdt, pbytes in (("vblock", torch.float8_e4m3fn, 1), ("vblock_int8", torch.int8, 1)):
        payload = torch.empty(B, HV, KD, KD, dtype=pdt, device=device)
        scale = torch.empty(B, HV, KD // 32, dtype=torch.float16, device=device)
        q_us = _graph_us(lambda: gdnr.quantize_checkpoint(state, gran, payload=payload, scale=scale,
                                                          compute_saturation=False), stream, 20)
        ck = gdnr.QuantizedCheckpoint(payload, scale, gran, 32, 0.0)
        out = torch.empty_like(state)
        d_us = _graph_us(lambda: gdnr.dequantize_checkpoint(ck, out=out), stream, 20)
        moved = n * (4 + pbytes) + scale.numel() * 2
        codec[gran] = {"quantize_us": q_us, "quantize_GB_s": moved / (q_us * 1e-6) / 1e9,
                       "dequantize_us": d_us, "dequantize_GB_s": moved / (d_us * 1e-6) / 1e9}
    codec["shape"] = [B, HV, KD, KD]
    res["codec"] = codec
    return res


def run_comparators(args, device, stream, ours_us):
    """Same-box comparators for the reference's speed-up table
    (bench_gdn_vs_production.py:279-292, bench_gdn_full_contract.py:225-308):
    the production operator the reference swaps out -- vLLM's FLA
    ``fused_recurrent_gated_delta_rule_packed_decode`` (a Triton kernel shipped
    in this image; bf16 state read-modify-write through ``ssm_state_indices``)
    -- and this library's sm_100a bf16 read-modify-write step (kern.py:245-341),
    both at the bench's batch over 4 layers of state (> 2x L2).  ``ours_us`` is
    the cycle-amortised fused step per layer measured above."""
    import torch

    import gdnr
    from gdnr import inputs as gin

    B, NL = args.batch, 4
    state_bytes = 2 * B * HV * KD * KD * 2  # bf16 state read + write per layer step
    res = {"ours_us_per_layer_step": ours_us}
    sets = []
    for li in range(NL):
        d = gin.replay_ring_inputs(B, 1, seed=args.seed * 11 + li, device=device)
        sets.append((d["state"].to(torch.bfloat16), d["q"], d["k"][:, 0].contiguous(), d["v"][:, 0].contiguous(),
                     d["g"][:, 0].contiguous(), d["beta"][:, 0].contiguous()))
        del d

    def bf16_step():
        for st, q, k, v, g, be in sets:
            gdnr.gdn_bf16_step(st, q, k, v, g, be)
    us = _graph_us(bf16_step, stream, 20) / NL
    res["bf16_step_sm100a"] = {"us_per_layer_step": us, "state_GB_s": state_bytes / (us * 1e-6) / 1e9,
                               "speedup_of_ours": us / ours_us}
    del sets
    try:
        from vllm.model_executor.layers.fla.ops.fused_recurrent import \
            fused_recurrent_gated_delta_rule_packed_decode as fla_decode
    except Exception as e:  # the comparator is optional: the image may lack vLLM or Triton
        res["fla_packed_decode"] = {"unavailable": f"{type(e).__name__}: {e}"[:200]}
        return res
    gen = torch.Generator().manual_seed(args.seed + 23)
    layers = []
    for li in range(NL):
        raw = gin.raw_step_inputs(B, 1, seed=(args.seed * 1000 + li) * 4096 + 11, device=device)
        pool = torch.zeros(B + 1, HV, KD, KD, dtype=torch.bfloat16, device=device)  # slot 0 = null
        pool[1:] = raw["state"].to(torch.bfloat16)
        idx = (torch.randperm(B, generator=gen) + 1).to(torch.int32).to(device)
        layers.append((raw["mixed_qkv"][:, 0].contiguous(), raw["a"][:, 0].contiguous(), raw["b"][:, 0].contiguous(),
                       raw["a_log"], raw["dt_bias"], pool, torch.empty(B, 1, HV, KD, dtype=torch.bfloat16,
                                                                       device=device), idx))
        del raw

    def fla_step():
        for m, a, b, al, db, pool, out, idx in layers:
            fla_decode(m, a, b, al, db, KD ** -0.5, pool, out, idx, use_qk_l2norm_in_kernel=True)
    us = _graph_us(fla_step, stream, 20) / NL
    res["fla_packed_decode"] = {
        "us_per_layer_step": us, "state_GB_s": state_bytes / (us * 1e-6) / 1e9, "speedup_of_ours": us / ours_us,
        "workload": f"vLLM FLA packed decode (Triton, JIT-compiled for this GPU), batch {B}, bf16 state pool of "
                    f"{B + 1} slots, random slot order, {NL} layers"}
    del layers
    return res


def run_core(args, device, stream):
    """core replay (non-flush) of a full L=16 ring, block-V sweep."""
    import torch

    import gdnr
    from gdnr import inputs as gin
    from oracle import gdn_oracle as O

    B, L, NL = args.batch, args.ring, args.layers
    sets = []
    for li in range(NL):
        d = gin.replay_ring_inputs(B, L, seed=args.seed * 7 + li, device=device)
        ck = gdnr.quantize_checkpoint(d["state"], scale_dtype=torch.float32, compute_saturation=False)
        sets.append((ck, d, torch.full((B,), L, dtype=torch.int32, device=device),
                     torch.zeros(B, dtype=torch.bool, device=device),
                     torch.empty(B, HV, KD, dtype=torch.bfloat16, device=device)))
    res = {}
    nbytes = O.algorithmic_bytes(B, L, L, scale_bytes=4, gate_bytes=4, fused=False)

    def run():
        for ck, d, vl, fl, out in sets:
            gdnr.gdn_replay_fp8(ck.payload, ck.scale, d["q"], d["k"], d["v"], d["g"], d["beta"], vl, fl, out=out,
                                flush_hint="none")
    with torch.cuda.stream(stream):
        run()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        run()
    reps = 50
    with torch.cuda.stream(stream):
        for _ in range(5):
            g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    us = 1e3 * e0.elapsed_time(e1) / (reps * NL)
    res.update({"us_per_launch": us, "GB_s": nbytes / (us * 1e-6) / 1e9, "steps_seq_per_s": B / (us * 1e-6),
                "frac_of_peak": nbytes / (us * 1e-6) / 1e9 / measured_peak()[0]})
    del g
    res["algorithmic_bytes_per_launch"] = nbytes
    res["workload"] = "config2: gdn_replay_fp8 non-flush, B=64, full L=16 ring, f32 scales/gates"
    return res


def main():
    args = parse_args()
    world, rank, local = dist_init() if args.impl == "ours" else (
        int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        elif args.profile is not None:
            run_profile(args, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        if args.impl == "ours" and world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
