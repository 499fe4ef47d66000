#!/usr/bin/env python
"""Benchmark of the fused FP8-replay GDN decode step on B200.

Headline workload (BASELINE config 3 at the metric's point, batch 64 per GPU,
L = 16): one *step* is one decode token through a stack of NL independent GDN
layers, each a single ``gdn_fused_step`` launch (prep + ring append + replay,
and the flush / re-quantisation on the L-th token of the ring cycle) at
batch 64, H = 16, HV = 32, K = V = 128.  The W warm-up steps end on a ring
boundary, so the K timed steps walk the ring from position 0; ``value`` is
cycle-exact: the per-position mean step times weighted so that the flush is
exactly 1/L of the steps, whatever K is (K >= L), as in the reference's cycle
model (prototype/bench_gdn_full_contract.py:225-308).  NL layers x ~46 MB of
state (> 2x the 126 MB L2) keep every launch reading its state from HBM.

The metric is decode steps.seq/s per GDN layer: (NL x batch) / (cycle-mean
time of one step).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Other keys of the JSON line (each measured the same way, one CUDA graph per
ring position, CUDA events between replays):
  sweep          BASELINE config 3: B in {1,4,16,64,256} x L in {4,8,16}
  heterogeneous  B=64, L=16 with ring positions spread over 0..L-1 (1/L of the
                 sequences flush on every step), default "auto" hint
  config5        BASELINE config 5: 24 layers x 1024 sequences split over the
                 ranks (strong scaling), 256 steps, per-rank times
  comparators    the production op (vLLM FLA packed decode), the sm_100a bf16
                 step, and the reference's own Triton kernels when a copy of
                 the reference's prototype/ directory sits in baseline/_ref/
  e2e            the public Python API with pinned host buffers, host<->device
                 copies inside the timed region

Multi-GPU: one process per GPU (torchrun); the headline runs batch 64 per
rank (weak scaling over independent sequence shards), config5 splits a fixed
job; no collective on the data path -- only barriers and the max over ranks
of the timings.
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
W_MIXED = 2 * H * KD + HV * KD
FALLBACK_HBM_GBS = 6650.0
L2_BYTES = 126e6
REF_DIR = ROOT / "baseline" / "_ref" / "prototype"  # optional copy of the reference's prototype/ (not committed)


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
    ap.add_argument("--no-core", action="store_true",
                    help="skip the single-GPU extras (core replay, widened rows, comparators, sweep, heterogeneous)")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-config5", action="store_true")
    ap.add_argument("--config5-steps", type=int, default=256)
    ap.add_argument("--drift", action="store_true",
                    help="BASELINE config 4 instead of the benchmark: drift of the FP8 replay chain vs an fp32 "
                         "recurrence (one JSON line)")
    ap.add_argument("--drift-steps", type=int, default=4096)
    ap.add_argument("--drift-layers", type=int, default=4)
    ap.add_argument("--drift-rings", default="4,16,64")
    ap.add_argument("--drift-stride", type=int, default=256)
    ap.add_argument("--profile", type=int, default=None, metavar="POS",
                    help="profiling driver for ncu: a few untimed launches of one layer's step at ring position "
                         "POS (no timing, no JSON line)")
    ap.add_argument("--profile-batch", type=int, default=None,
                    help="batch of the --profile driver (default --batch)")
    ap.add_argument("--profile-hetero", action="store_true",
                    help="--profile with ring positions spread over 0..L-1 and the 'auto' hint")
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


def profile_traffic_ratio():
    """(dram bytes / algorithmic bytes, capture note) of the committed ncu summary
    of the non-flush step kernel."""
    p = ROOT / "profiles" / "step5_kernel_b64_l16.md"
    dram = alg = None
    try:
        for line in p.read_text().splitlines():
            if line.startswith("dram_bytes_per_launch_fill8"):
                dram = float(line.split("=")[1].strip())
            if line.startswith("algorithmic_bytes_per_launch_fill8"):
                alg = float(line.split("=")[1].strip())
    except Exception:
        pass
    if dram and alg:
        return dram / alg, "ncu capture at ring fill 8 (profiles/step5_kernel_b64_l16.md), scaled by algorithmic bytes"
    return None, "no ncu capture"


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


def gather_over_ranks(x: float, world: int) -> list:
    if world == 1:
        return [x]
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(x)], dtype=torch.float64, device=torch.device("cuda", torch.cuda.current_device()))
    out = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(o.item()) for o in out]


def barrier(world: int):
    import torch

    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


# ---------------------------------------------------------------- CPU baseline and the reference arm

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


def reference_torch_cpu(args):
    """The reference's own CPU path, when a copy of its prototype/ sits in
    baseline/_ref/: ``replay_decode`` of gdn_replay_fp8_reference.py
    (ref.py:189-244: dequantise, replay the ring from the checkpoint with the
    per-token recurrence, keep the last output, re-quantise when the ring is
    full) at batch 64, H=16, HV=32, on all host threads.  One step = one decode
    token of the batch; steps walk whole L-cycles.  Returns None without the copy."""
    if not (REF_DIR / "gdn_replay_fp8_reference.py").exists():
        return None
    import torch

    sys.path.insert(0, str(REF_DIR))
    import gdn_replay_fp8_reference as ref  # noqa: E402  (the reference's own module)

    threads = cpu_workers()
    torch.set_num_threads(threads)
    B, L = args.batch, args.ring
    gen = torch.Generator().manual_seed(args.seed)
    state = 0.02 * torch.randn(B, HV, KD, KD, generator=gen)

    def inputs(T):
        q = torch.nn.functional.normalize(torch.randn(B, T, H, KD, generator=gen), dim=-1)
        k = torch.nn.functional.normalize(torch.randn(B, T, H, KD, generator=gen), dim=-1)
        v = torch.randn(B, T, HV, KD, generator=gen)
        g = -torch.rand(B, T, HV, generator=gen) * 0.1
        beta = torch.sigmoid(torch.randn(B, T, HV, generator=gen))
        return q, k, v, g, beta

    # replay_decode(T tokens) runs all T steps of the chain; one cycle = L steps.
    # Warm-up: --warmup single steps (untimed); then whole cycles, as many as
    # --steps asks for within about a minute of host time.
    warm = max(1, args.warmup)
    t0 = time.perf_counter()
    for _ in range(warm):
        q, k, v, g, beta = inputs(1)
        ref.replay_decode(state, q, k, v, g, beta, L, "vblock", 32)
    one = (time.perf_counter() - t0) / warm  # one step at fill 1: sizes the sample
    cycles = max(1, min(args.steps // L, int(60.0 / max(one * L * (L + 1) / 2, 1e-3))))
    t0 = time.perf_counter()
    q, k, v, g, beta = inputs(L * cycles)
    ref.replay_decode(state, q, k, v, g, beta, L, "vblock", 32)
    wall = time.perf_counter() - t0
    steps = L * cycles
    value = steps * B / wall
    return {"value": value, "unit": UNIT, "cores": threads, "kind": "reference", "steps": steps, "warmup": warm,
            "sample": f"the reference's replay_decode (gdn_replay_fp8_reference.py, torch on CPU, {threads} threads) "
                      f"over {steps} decode steps (whole L={L} cycles incl. the flush) of batch {B}, H={H}, HV={HV}; "
                      f"{wall:.1f} s wall after {warm} warm-up step(s) of {one:.2f} s each"}


def run_reference(args, world, rank):
    """--impl reference: the reference's CPU implementation of the path on the
    host cores (its own replay_decode when baseline/_ref holds a copy of its
    prototype/, else the numpy oracle port of it)."""
    if rank != 0:
        return
    ref = None
    try:
        ref = reference_torch_cpu(args)
    except Exception as e:  # a broken copy falls back to the port, with the reason
        ref_err = f"{type(e).__name__}: {e}"[:200]
    else:
        ref_err = None
    if ref is not None:
        value, steps, ms = ref["value"], ref["steps"], 1e3 * args.batch / ref["value"]
        warm = ref["warmup"]
        cpu = {k: ref[k] for k in ("value", "unit", "cores", "kind", "sample")}
        cfg_batch, note = args.batch, "the reference's own torch replay_decode, imported from baseline/_ref"
    else:
        workers = cpu_workers()
        budget_s = 150.0
        _, probe_wall = cpu_units(1, workers, args.seed, args.ring)
        per_step = probe_wall if probe_wall > 0 else 0.05
        steps = args.steps
        while steps * per_step > budget_s and steps > 1:
            steps //= 2
        t_units, t_wall = cpu_units(max(1, steps), workers, args.seed, args.ring)
        value, ms, cfg_batch = t_units / t_wall, 1e3 * t_wall / max(1, steps), workers
        warm = 1
        cpu = {"value": value, "unit": UNIT, "cores": workers, "kind": "port",
               "sample": f"{t_units} sequence-layer steps ({workers} sequences per step, {steps} steps) of the numpy "
                         "oracle port of replay_decode"}
        note = ("no copy of the reference's prototype/ in baseline/_ref" + (f" ({ref_err})" if ref_err else "") +
                "; its CPU path (ref.py replay_decode) is timed through the repo's numpy restatement")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": steps,
        "warmup": warm,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded, BASELINE config 1/3 distributions)",
        "config": {"workload": f"one GDN layer's decode step (replay chain + flush every {args.ring}), L={args.ring}, "
                               "CPU sample", "global_batch": cfg_batch, "seq_len": args.ring,
                   "parallelism": f"{cpu['cores']} host threads"},
        "cpu_baseline": cpu,
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": note,
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- workload construction

class LayerStack:
    """NL independent GDN layers of B sequences each: one pooled decode state
    (the layers are consecutive batch ranges of it) and resident raw inputs per
    (layer, ring position), seeded per layer with the config-1 distributions
    (q, k, v, a, b ~ N(0,1) bf16; A_log = log U(1,16); dt_bias ~ N(0,0.5);
    state ~ N(0, 0.02) quantised to the checkpoint)."""

    def __init__(self, B, L, NL, seed_of, device, checkpoint_dtype=None, out_dtype=None):
        import torch

        import gdnr

        bf = torch.bfloat16
        self.B, self.L, self.NL = B, L, NL
        self.pool = gdnr.ReplayState.allocate(NL * B, H, HV, L, device=device, scale_dtype=torch.float32,
                                              gate_dtype=torch.float32,
                                              checkpoint_dtype=checkpoint_dtype or torch.float8_e4m3fn)
        self.mixed = torch.empty(NL, L, B, W_MIXED, dtype=bf, device=device)
        self.a = torch.empty(NL, L, B, HV, dtype=bf, device=device)
        self.b = torch.empty(NL, L, B, HV, dtype=bf, device=device)
        self.a_log = torch.empty(NL, HV, dtype=torch.float32, device=device)
        self.dt_bias = torch.empty(NL, HV, dtype=torch.float32, device=device)
        self.out = torch.empty(NL, B, HV, KD, dtype=out_dtype or bf, device=device)
        self.views = []
        for li in range(NL):
            g = torch.Generator(device=device)
            g.manual_seed(int(seed_of(li)))
            self.mixed[li] = torch.randn(L, B, W_MIXED, generator=g, device=device)
            self.a[li] = torch.randn(L, B, HV, generator=g, device=device)
            self.b[li] = torch.randn(L, B, HV, generator=g, device=device)
            self.a_log[li] = torch.log(1.0 + 15.0 * torch.rand(HV, generator=g, device=device))
            self.dt_bias[li] = 0.5 * torch.randn(HV, generator=g, device=device)
            sl = slice(li * B, (li + 1) * B)
            p = self.pool
            view = gdnr.ReplayState(p.checkpoint[sl], None if p.scale is None else p.scale[sl], p.k_ring[sl],
                                    p.v_ring[sl], p.g_ring[sl], p.beta_ring[sl], p.pos[sl])
            view.load_state(0.02 * torch.randn(B, HV, KD, KD, generator=g, device=device))
            self.views.append(view)
        # the shapes bench's e2e path consumes
        self.layers = [{"state": self.views[li], "a_log": self.a_log[li], "dt_bias": self.dt_bias[li],
                        "out": self.out[li]} for li in range(NL)]
        self.step_inputs = [[(self.mixed[li, s], self.a[li, s], self.b[li, s]) for s in range(L)] for li in range(NL)]

    def state_nbytes(self):
        return self.pool.nbytes()

    def launch(self, s, pos, hint, err=None):
        """Every layer's fused step with this step's inputs of ring position s."""
        import gdnr

        for li, st in enumerate(self.views):
            gdnr.gdn_fused_step(self.mixed[li, s], self.a[li, s], self.b[li, s], self.a_log[li], self.dt_bias[li], pos,
                                st.checkpoint, st.scale, st.k_ring, st.v_ring, st.g_ring, st.beta_ring,
                                out=self.out[li], error_flag=err, flush_hint=hint)


def flush_hint_for(s: int, L: int) -> str:
    """All sequences share the ring position here, so whether this step flushes
    is known on the host: no sequence ("none") or every sequence ("all")."""
    return "all" if s == L - 1 else "none"


def uniform_positions(B, L, device):
    import torch

    return [torch.full((B,), s, dtype=torch.int32, device=device) for s in range(L)]


def spread_positions(B, L, device):
    """Step offset s: sequence b at ring position (b + s) % L (1/L of them flush)."""
    import torch

    base = torch.arange(B, dtype=torch.int32, device=device)
    return [((base + s) % L).to(torch.int32) for s in range(L)]


def capture_positions(fn, L, stream):
    """One CUDA graph per ring position s of fn(s) (after one eager pass).
    Everything the default stream has enqueued (the inputs' initialisation)
    completes first: the launches go to a side stream."""
    import torch

    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for s in range(L):
            fn(s)
    torch.cuda.synchronize()
    graphs = []
    for s in range(L):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            fn(s)
        graphs.append(g)
    torch.cuda.synchronize()
    return graphs


def time_cycles(graphs, stream, cycles, warm=1):
    """Mean device ms of each position's graph over `cycles` whole ring cycles
    (events between consecutive replays on the launch stream)."""
    import torch

    L = len(graphs)
    with torch.cuda.stream(stream):
        for _ in range(warm):
            for g in graphs:
                g.replay()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(cycles * L + 1)]
    with torch.cuda.stream(stream):
        ev[0].record(stream)
        for c in range(cycles):
            for s, g in enumerate(graphs):
                g.replay()
                ev[c * L + s + 1].record(stream)
    torch.cuda.synchronize()
    per = [0.0] * L
    for c in range(cycles):
        for s in range(L):
            per[s] += ev[c * L + s].elapsed_time(ev[c * L + s + 1]) / cycles
    return per


# ---------------------------------------------------------------- GPU arm

def build_stack(args, device, rank: int = 0, world: int = 1, checkpoint_dtype=None, batch=None, layers=None):
    """This rank's shard of the headline job: sequences ShardPlan(B * world,
    world).local(rank) of every layer, each rank with its own seeded inputs and
    state (weak scaling)."""
    from gdnr.shard import ShardPlan

    B = batch or args.batch
    NL = layers or args.layers
    shard = ShardPlan(B * world, world).local(rank)
    assert len(shard) == B
    return LayerStack(B, args.ring, NL, lambda li: (args.seed * 1000 + li) * 4096 + shard.start, device,
                      checkpoint_dtype=checkpoint_dtype)


def run_profile(args, local):
    """A few eager launches of one layer's fused step at one ring position (ncu target)."""
    import torch

    device = torch.device("cuda", local)
    B, L = args.profile_batch or args.batch, args.ring
    stack = build_stack(args, device, batch=B, layers=1,
                        checkpoint_dtype=torch.int8 if args.checkpoint == "int8" else None)
    err = torch.zeros(1, dtype=torch.int32, device=device)
    s = args.profile % L
    if args.profile_hetero:
        pos, hint = spread_positions(B, L, device)[s], "auto"
    else:
        pos, hint = uniform_positions(B, L, device)[s], flush_hint_for(s, L)
    for _ in range(3):
        stack.launch(s, pos, hint, err)
    torch.cuda.synchronize()
    print(f"profile: 3 launches at ring position {s} (batch {B}, hint {hint}), device error word {int(err.item())}",
          flush=True)


def run_ours(args, world, rank, local):
    import torch

    from gdnr import traffic

    device = torch.device("cuda", local)
    B, L, NL = args.batch, args.ring, args.layers
    cpu_line = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_line = cpu_baseline(args.seed, L)  # spawn pool; GPU untouched so far

    stack = build_stack(args, device, rank, world)
    err = torch.zeros(1, dtype=torch.int32, device=device)
    pos = uniform_positions(B, L, device)
    stream = torch.cuda.Stream(device)
    graphs = capture_positions(lambda s: stack.launch(s, pos[s], flush_hint_for(s, L), err), L, stream)

    # warm-up steps end on a ring boundary: the timed steps start at position 0
    step_idx = (-args.warmup) % L
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graphs[step_idx % L].replay()
            step_idx += 1
    barrier(world)
    # one event between consecutive graph replays: per-position step times
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
    ms_window = evs[0].elapsed_time(evs[-1])
    step_ms = [evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]
    by_pos = {}
    for p, t in zip(positions, step_ms):
        by_pos.setdefault(p, []).append(t)
    cycle_exact = len(by_pos) == L
    if cycle_exact:  # each ring position weighted 1/L: the flush is exactly 1/L of the steps
        ms_cycle_step = sum(statistics.fmean(by_pos[p]) for p in range(L)) / L
    else:  # fewer timed steps than ring positions: the window as measured
        ms_cycle_step = ms_window / args.steps
    ms_step = max_over_ranks(ms_cycle_step, world)
    ms_window_max = max_over_ranks(ms_window, world)
    dev_err = int(err.item())

    launches = args.steps * NL
    value = NL * B * world / (ms_step / 1e3)
    peak, peak_kind = measured_peak()
    fill_bytes = {p: traffic.step_bytes(B, p + 1, L) for p in range(L)}
    kernels = {}
    for name, sel in (("step5_kernel<flush=false> (non-flush steps)", lambda p: p != L - 1),
                      ("step5_kernel<flush=true> (flush step)", lambda p: p == L - 1)):
        ps = [p for p in by_pos if sel(p)]
        if not ps:
            continue
        t = statistics.fmean(statistics.fmean(by_pos[p]) for p in ps) / NL / 1e3
        b = statistics.fmean(fill_bytes[p] for p in ps)
        kernels[name] = {"launches": sum(len(by_pos[p]) for p in ps) * NL, "us_per_launch": t * 1e6,
                         "algorithmic_bytes_per_launch": b, "achieved_GB_s": b / t / 1e9,
                         "frac_of_peak": b / t / 1e9 / peak}
    dom = max(kernels, key=lambda k: kernels[k]["launches"] * kernels[k]["us_per_launch"])
    achieved = kernels[dom]["achieved_GB_s"]
    cyc_bytes = traffic.cycle_bytes(B, L)
    ratio, traffic_note = profile_traffic_ratio()

    # ---- end to end through the public API with host buffers (pinned), per layer-step
    e2e = run_e2e(args, stack.layers, stack.step_inputs, pos, stream, world) if args.e2e_steps > 0 else None
    del graphs
    torch.cuda.synchronize()

    extras = {}
    if not args.no_core and world == 1:
        extras["core_replay"] = run_core(args, device, stream)
        extras["heterogeneous"] = run_heterogeneous(args, stack, device, stream, 1e3 * ms_step / NL)
        extras.update(run_widened(args, device, stream))
        extras["comparators"] = run_comparators(args, device, stream, 1e3 * ms_step / NL)
        if not args.no_sweep:
            extras["sweep"] = run_sweep(args, device, stream)
    del stack
    torch.cuda.empty_cache()
    if not args.no_config5:
        extras["config5"] = run_config5(args, world, rank, device, stream)

    if rank != 0:
        return
    line = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_window_max / args.steps,
        "us_per_layer_step": 1e3 * ms_step / NL,
        "cycle_exact": cycle_exact,
        "value_timed_window": NL * B * world * args.steps / (ms_window_max / 1e3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "e4m3/f32",
        "data": "synthetic (seeded; BASELINE config 1/3 distributions; random state N(0,0.02))",
        "config": {
            "workload": f"config3 fused full-contract step (prep+ring append+replay, flush every {L}), "
                        f"batch {B}/GPU, L={L}, cycle-exact (each ring position weighted 1/L); one step = one token "
                        f"through {NL} independent GDN layers (one launch each)",
            "global_batch": B * world, "seq_len": L, "parallelism": f"sequence-shard x{world} (no collective)",
            "heads": H, "value_heads": HV, "head_dim": KD, "layers": NL,
            "l2": f"inputs larger than L2: {NL} layer states, {stack_bytes(B, L, NL) / 1e6:.0f} MB",
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
            "traffic": None if ratio is None else ratio * kernels[dom]["algorithmic_bytes_per_launch"],
            "traffic_source": traffic_note,
            "algorithmic_bytes_per_launch": kernels[dom]["algorithmic_bytes_per_launch"],
            "cycle": {"algorithmic_bytes_per_launch": cyc_bytes, "us_per_launch": 1e3 * ms_step / NL,
                      "achieved": cyc_bytes / (ms_step / NL / 1e3) / 1e9,
                      "frac": cyc_bytes / (ms_step / NL / 1e3) / 1e9 / peak},
            "note": "achieved = the kernel's algorithmic bytes per launch (averaged over the ring positions it ran) / "
                    "its average launch time from CUDA events between graph replays on the launch stream; cycle = "
                    "the same over a whole ring cycle (flush included)",
        },
        "kernels": kernels,
        "per_position_us_per_launch": [1e3 * statistics.fmean(by_pos[p]) / NL for p in sorted(by_pos)],
    }
    if e2e is not None:
        line["e2e"] = e2e
    line.update(extras)
    if cpu_line is not None:
        line["cpu_baseline"] = cpu_line
    print(json.dumps(line), flush=True)


def stack_bytes(B, L, NL):
    from gdnr import traffic

    return NL * traffic.state_bytes(B, L)


def run_heterogeneous(args, stack, device, stream, uniform_us):
    """The headline stack with ring positions spread evenly over 0..L-1 (step
    offset s: sequence b at position (b + s) % L, so 1/L of the sequences flush
    on every step), default "auto" hint; µs per layer-step over a cycle of offsets."""
    import torch

    B, L, NL = stack.B, stack.L, stack.NL
    pos = spread_positions(B, L, device)
    err = torch.zeros(1, dtype=torch.int32, device=device)
    graphs = capture_positions(lambda s: stack.launch(s, pos[s], "auto", err), L, stream)
    per = time_cycles(graphs, stream, cycles=4)
    del graphs
    us = 1e3 * statistics.fmean(per) / NL
    # the uniform cycle again under the default hint ("auto" on every step: the
    # flush-capable kernel also on the steps where no sequence flushes)
    upos = uniform_positions(B, L, device)
    graphs = capture_positions(lambda s: stack.launch(s, upos[s], "auto", err), L, stream)
    uper = time_cycles(graphs, stream, cycles=4)
    del graphs
    auto_us = 1e3 * statistics.fmean(uper) / NL
    return {"us_per_layer_step": us, "steps_seq_per_s": B / (us * 1e-6), "uniform_cycle_us_per_layer_step": uniform_us,
            "ratio_to_uniform": us / uniform_us, "device_error_word": int(err.item()),
            "uniform_cycle_default_hint": {"us_per_layer_step": auto_us, "steps_seq_per_s": B / (auto_us * 1e-6),
                                           "us_nonflush": 1e3 * statistics.fmean(uper[:-1]) / NL,
                                           "us_flush": 1e3 * uper[-1] / NL},
            "workload": f"batch {B}, L={L}, {NL} layers, sequence b at ring position (b + s) % L on step s (1/L flush "
                        "on every step), flush_hint 'auto', 4 cycles; uniform_cycle_default_hint: the headline's "
                        "uniform positions with flush_hint 'auto' on every step"}


def run_sweep(args, device, stream):
    """B in {1,4,16,64,256} x L in {4,8,16}, each cell a whole
    ring cycle (fills 1..L, the flush on the last) with uniform positions, over
    enough layer states to exceed 2x L2; plus the production op (vLLM FLA packed
    decode) per batch, as the reference's speed-up table does
    (bench_gdn_full_contract.py:225-308)."""
    import torch

    from gdnr import traffic

    peak, _ = measured_peak()
    cells = []
    fla = {}
    for B in (1, 4, 16, 64, 256):
        for L in (4, 8, 16):
            NL = max(1, min(512, math.ceil(2.2 * L2_BYTES / traffic.state_bytes(B, L))))
            print(f"bench: sweep cell B={B} L={L} ({NL} layers)", file=sys.stderr, flush=True)
            stack = LayerStack(B, L, NL, lambda li: (args.seed * 7919 + B * 131 + L) * 4096 + li, device)
            torch.cuda.synchronize()
            pos = uniform_positions(B, L, device)
            err = torch.zeros(1, dtype=torch.int32, device=device)
            graphs = capture_positions(lambda s: stack.launch(s, pos[s], flush_hint_for(s, L), err), L, stream)
            per = time_cycles(graphs, stream, cycles=4)
            del graphs
            us = 1e3 * statistics.fmean(per) / NL
            cb = traffic.cycle_bytes(B, L)
            cells.append({"batch": B, "ring": L, "layers": NL, "us_per_layer_step": us,
                          "steps_seq_per_s": B / (us * 1e-6), "GB_s": cb / (us * 1e-6) / 1e9,
                          "frac_of_peak": cb / (us * 1e-6) / 1e9 / peak,
                          "us_nonflush": 1e3 * statistics.fmean(per[:-1]) / NL, "us_flush": 1e3 * per[-1] / NL,
                          "device_error_word": int(err.item())})
            del stack
        fla[B] = fla_packed_decode_us(B, args.seed, device, stream)
        for c in cells:
            if c["batch"] == B and isinstance(fla[B], float):
                c["production_us"] = fla[B]
                c["speedup_vs_production"] = fla[B] / c["us_per_layer_step"]
    return {"cells": cells, "workload": "gdn_fused_step cycle-averaged per layer-step (one CUDA graph per ring "
                                        "position over >2x L2 of layer states); production_us: vLLM FLA packed decode "
                                        "on a bf16 state pool, same batch"}


def fla_packed_decode_us(B, seed, device, stream):
    """µs per layer-step of the production operator (vLLM's FLA packed decode,
    bf16 state pool of B + 1 slots, random slot order) over > 2x L2 of state."""
    import torch

    try:
        from vllm.model_executor.layers.fla.ops.fused_recurrent import \
            fused_recurrent_gated_delta_rule_packed_decode as fla_decode
    except Exception as e:  # optional: the image may lack vLLM or Triton
        return f"unavailable: {type(e).__name__}: {e}"[:200]
    per_layer = (B + 1) * HV * KD * KD * 2
    NL = max(1, min(512, math.ceil(2.2 * L2_BYTES / per_layer)))
    gen = torch.Generator().manual_seed(seed + 23 + B)
    pools = torch.zeros(NL, B + 1, HV, KD, KD, dtype=torch.bfloat16, device=device)
    pools[:, 1:].normal_(0.0, 0.02)
    mixed = torch.randn(NL, B, W_MIXED, device=device).to(torch.bfloat16)
    a = torch.randn(NL, B, HV, device=device).to(torch.bfloat16)
    b = torch.randn(NL, B, HV, device=device).to(torch.bfloat16)
    a_log = torch.log(1.0 + 15.0 * torch.rand(HV, device=device))
    dt_bias = 0.5 * torch.randn(HV, device=device)
    out = torch.empty(NL, B, 1, HV, KD, dtype=torch.bfloat16, device=device)
    idx = (torch.randperm(B, generator=gen) + 1).to(torch.int32).to(device)

    def step(s=0):
        for li in range(NL):
            fla_decode(mixed[li], a[li], b[li], a_log, dt_bias, KD ** -0.5, pools[li], out[li], idx,
                       use_qk_l2norm_in_kernel=True)
    graphs = capture_positions(step, 1, stream)
    per = time_cycles(graphs, stream, cycles=8)
    del graphs, pools
    return 1e3 * per[0] / NL


def run_drift(args, local):
    """long-sequence drift of the FP8 checkpoint + replay
    scheme against an fp32 per-token recurrence run alongside on the GPU, by the
    reference's dual-chain method (prototype/qwen35_drift_study.py:341-379): the
    true state evolves token by token in fp32; each arm (ring length L) keeps the
    checkpoint + ring that gdn_fused_step maintains, its output is the kernel's,
    and its reconstructed state (the recurrence from the dequantised checkpoint
    over the ring, restarted from the kernel's re-quantised checkpoint at every
    flush) is compared with the true state after every token.  Synthetic
    inputs: q, k, v ~ N(0,1) bf16, A_log = 0 and a solved so that
    alpha = exp(g) ~ U(0.9, 0.999), b ~ N(0,1), state ~ N(0, 0.02).  Both chains
    consume the same prepped q, k, v, g, beta (the kernel's ring contents).
    Reports mean / final state and output relative L2 per arm, a curve every
    `--drift-stride` steps, and the steady-state µs per layer-step of each arm."""
    import torch

    import gdnr
    from gdnr import inputs as gin

    device = torch.device("cuda", local)
    torch.backends.cuda.matmul.allow_tf32 = False
    NLy, B, T = args.drift_layers, args.batch, args.drift_steps
    rings = [int(x) for x in args.drift_rings.split(",")]
    NB = NLy * B  # the layers as independent batch ranges of one state
    gen = torch.Generator(device=device)
    gen.manual_seed(args.seed * 4099 + 4)
    s0 = 0.02 * torch.randn(NB, HV, KD, KD, generator=gen, device=device)
    truth = s0.clone()
    arms = {}
    for L in rings:
        st = gdnr.ReplayState.allocate(NB, H, HV, L, device=device)
        st.load_state(s0)
        recon = gdnr.dequantize_checkpoint(gdnr.QuantizedCheckpoint(st.checkpoint, st.scale, "vblock", 32, 0.0)).clone()
        arms[L] = {"state": st, "recon": recon, "sd": [], "od": [], "curve": []}
    gates = gin.drift_gate_inputs(NB, T, HV, seed=args.seed * 4099 + 5, device=device)
    a_log, dt_bias = gates["a_log"], gates["dt_bias"]
    out = torch.empty(NB, HV, KD, dtype=torch.float32, device=device)
    q_out = torch.empty(NB, H, KD, dtype=torch.bfloat16, device=device)  # q as the production step keeps it
    nxt = torch.empty(NB, dtype=torch.int32, device=device)
    scale = KD ** -0.5
    G = HV // H

    def rel(a, b):
        return float(torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b).clamp_min(1e-30))

    def recur(S, q, k, v, g, beta):  # one fp32 token (ref.py:137-163), exact products
        Sv = S.view(NB * HV, KD, KD)
        Sv.mul_(torch.exp(g).view(-1, 1, 1))
        kk = k.repeat_interleave(G, 1).reshape(NB * HV, KD, 1)
        r = torch.bmm(Sv, kk)
        u = (v.reshape(NB * HV, KD, 1) - r) * beta.reshape(NB * HV, 1, 1)
        Sv.baddbmm_(u, kk.transpose(1, 2))
        qq = q.repeat_interleave(G, 1).reshape(NB * HV, KD, 1)
        return (torch.bmm(Sv, qq).view(NB, HV, KD) * scale)

    for t in range(T):
        mixed = torch.randn(NB, W_MIXED, generator=gen, device=device).to(torch.bfloat16)
        a = gates["a"][:, t].contiguous()
        b = torch.randn(NB, HV, generator=gen, device=device)
        true_o = None
        for L, arm in arms.items():
            st = arm["state"]
            p = t % L
            st.step(mixed, a, b, a_log, dt_bias, out=out, q_out=q_out, pos_out=nxt)
            q = q_out.float()
            k = st.k_ring[:, p].float()
            v = st.v_ring[:, p].float()
            g = st.g_ring[:, p].float()
            be = st.beta_ring[:, p].float()
            if true_o is None:  # every arm prepped the same token: the truth consumes it once
                true_o = recur(truth, q, k, v, g, be)
            recur(arm["recon"], q, k, v, g, be)
            if p == L - 1:  # flush: the reconstruction restarts from the kernel's re-quantised checkpoint
                arm["recon"].copy_(gdnr.dequantize_checkpoint(
                    gdnr.QuantizedCheckpoint(st.checkpoint, st.scale, "vblock", 32, 0.0)))
            arm["sd"].append(rel(arm["recon"], truth))
            arm["od"].append(rel(out, true_o))
            if t % args.drift_stride == 0 or t == T - 1:
                arm["curve"].append([t, round(arm["sd"][-1], 6), round(arm["od"][-1], 6)])
            st.pos.copy_(nxt)
    res = {"metric": "drift (relative L2 vs an fp32 per-token recurrence)", "layers": NLy, "batch": B, "steps": T,
           "alpha": [0.9, 0.999], "arms": {}}
    # steady-state time per layer-step of each arm: NLy layers of B sequences, one cycle
    stream = torch.cuda.Stream(device)
    for L, arm in arms.items():
        stack = LayerStack(B, L, NLy, lambda li: args.seed * 7 + li, device)
        pos = uniform_positions(B, L, device)
        graphs = capture_positions(lambda s: stack.launch(s, pos[s], flush_hint_for(s, L)), L, stream)
        per = time_cycles(graphs, stream, cycles=max(1, 64 // L))
        del graphs, stack
        sd, od = arm["sd"], arm["od"]
        res["arms"][f"L{L}"] = {
            "state_drift_mean": statistics.fmean(sd), "state_drift_final": sd[-1],
            "output_drift_mean": statistics.fmean(od), "output_drift_final": od[-1],
            "us_per_layer_step": 1e3 * statistics.fmean(per) / NLy,
            "kernel": "step5_kernel (persistent)" if L <= 16 else "step_kernel (CUDA cores, rings of L > 16)",
            "curve_step_state_output": arm["curve"]}
    print(json.dumps(res), flush=True)


def run_config5(args, world, rank, device, stream):
    """a fixed job of 24 GDN layers x 1024 sequences, L=16,
    split evenly over the ranks (strong scaling), config5_steps decode steps
    (whole ring cycles, a flush every 16) after one warm-up cycle; each rank
    times its own shard with CUDA events; value = all sequence-layer steps /
    the slowest rank's time."""
    import torch

    from gdnr.shard import ShardPlan

    GB_, NL, L = 1024, 24, 16
    shard = ShardPlan(GB_, world).local(rank)
    B = len(shard)
    steps = max(L, (args.config5_steps + L - 1) // L * L)
    stack = LayerStack(B, L, NL, lambda li: (args.seed * 1000003 + li) * 65536 + shard.start, device)
    pos = uniform_positions(B, L, device)
    err = torch.zeros(1, dtype=torch.int32, device=device)
    graphs = capture_positions(lambda s: stack.launch(s, pos[s], flush_hint_for(s, L), err), L, stream)
    with torch.cuda.stream(stream):
        for s in range(L):
            graphs[s].replay()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(steps):
            graphs[i % L].replay()
        e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = e0.elapsed_time(e1)
    per_rank = gather_over_ranks(ms, world)
    del graphs, stack
    torch.cuda.empty_cache()
    ms_max = max(per_rank)
    return {"value": GB_ * NL * steps / (ms_max / 1e3), "unit": UNIT, "scaling": "strong", "n_gpus": world,
            "sequences": GB_, "layers": NL, "ring": L, "steps": steps, "ms_max": ms_max,
            "per_rank_ms": per_rank, "per_rank_sequences": [len(r) for r in ShardPlan(GB_, world).ranges],
            "device_error_word": int(err.item()),
            "workload": f"24 layers x 1024 sequences split over {world} GPU(s) (rank r owns a contiguous 1024/N "
                        f"range), L=16, {steps} steps; per rank one CUDA graph per ring position; no collective"}


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

    # eager pass over the ring (warms up every path), then one graph per position;
    # the buffers above are initialised on the default stream: let that finish first
    torch.cuda.synchronize()
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
    """Mean device time of ``fn`` (captured once in a CUDA graph) over ``reps`` replays
    (after the default stream's pending work, which initialises fn's inputs)."""
    import torch

    torch.cuda.synchronize()
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
    res["triton_reference"] = run_triton_reference(args, device, stream)
    tr = res["triton_reference"].get(f"L{args.ring}", {})
    if "full_contract_us_per_layer_step" in tr:
        tr["speedup_of_ours_full_contract"] = tr["full_contract_us_per_layer_step"] / ours_us
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


def run_triton_reference(args, device, stream):
    """Same-box bar: the reference's own Triton kernels (gdn_prep_ring,
    gdn_replay_fp8, gdn_replay_fp8_split of prototype/gdn_replayssm_fp8_kernel.py
    :710, :344, :1129) as its stock wrappers launch them, when baseline/_ref/
    holds a copy of the reference's prototype/ directory (it is not part of this
    repository).  Batch 64, L in {4, 8, 16}, bf16 rings and fp16 scales as in the
    reference's full-contract benchmark, over > 2x L2 of layer states, one CUDA
    graph per ring position.  Per layer-step, amortised over a cycle like
    bench_gdn_full_contract.py:225-308: core = (sum of the non-flush replays at
    fills 1..L-1, best block_v of 32/64/128, + the flush at block_v 32) / L;
    full = core + prep."""
    if not (REF_DIR / "gdn_replayssm_fp8_kernel.py").exists():
        return {"unavailable": "no copy of the reference's prototype/ in baseline/_ref"}
    import torch

    import gdnr
    from gdnr import traffic

    try:
        sys.path.insert(0, str(REF_DIR))
        import gdn_replayssm_fp8_kernel as rk  # noqa: E402  (the reference's own module)
    except Exception as e:
        return {"unavailable": f"{type(e).__name__}: {e}"[:200]}
    bf = torch.bfloat16
    B = args.batch
    res = {"batch": B}
    for L in (4, 8, 16):
        NL = max(1, math.ceil(2.2 * L2_BYTES / traffic.state_bytes(B, L, scale_bytes=2, gate_bytes=2)))
        gen = torch.Generator(device=device)
        gen.manual_seed(args.seed * 97 + L)
        lay = []
        for li in range(NL):
            ck = gdnr.quantize_checkpoint(0.02 * torch.randn(B, HV, KD, KD, generator=gen, device=device), "vblock",
                                          scale_dtype=torch.float16, compute_saturation=False)
            lay.append({
                "ck": ck.payload, "sc": ck.scale,
                "mixed": torch.randn(L, B, W_MIXED, generator=gen, device=device).to(bf),
                "a": torch.randn(L, B, HV, generator=gen, device=device),
                "b": torch.randn(L, B, HV, generator=gen, device=device),
                "q": torch.empty(B, H, KD, dtype=bf, device=device),
                "k": torch.zeros(B, L, H, KD, dtype=bf, device=device),
                "v": torch.zeros(B, L, HV, KD, dtype=bf, device=device),
                "g": torch.zeros(B, L, HV, dtype=bf, device=device),
                "beta": torch.zeros(B, L, HV, dtype=bf, device=device),
                "out": torch.empty(B, HV, KD, dtype=bf, device=device),
                "tq": torch.empty(B, HV, KD, dtype=torch.float32, device=device),
                "cf": torch.empty(B, HV, L, dtype=torch.float32, device=device),
            })
        a_log = torch.rand(HV, generator=gen, device=device)
        dt_bias = torch.rand(HV, generator=gen, device=device) - 4.0
        pos = uniform_positions(B, L, device)
        valid = [torch.full((B,), s + 1, dtype=torch.int32, device=device) for s in range(L)]
        no_flush = torch.zeros(B, dtype=torch.bool, device=device)
        flush = torch.ones(B, dtype=torch.bool, device=device)

        def prep(s):
            for d in lay:
                rk.gdn_prep_ring(d["mixed"][s], d["a"][s], d["b"][s], a_log, dt_bias, pos[s], d["q"], d["k"], d["v"],
                                 d["g"], d["beta"])

        def replay(s, block_v):
            for d in lay:
                rk.gdn_replay_fp8(d["ck"], d["sc"], d["q"], d["k"], d["v"], d["g"], d["beta"], valid[s],
                                  flush if s == L - 1 else no_flush, block_v=block_v, out=d["out"])

        def split(s):
            for d in lay:
                rk.gdn_replay_fp8_split(d["ck"], d["sc"], d["q"], d["k"], d["v"], d["g"], d["beta"], valid[s],
                                        d["tq"], d["cf"], out=d["out"])
        try:
            prep_us = 1e3 * statistics.fmean(time_cycles(capture_positions(prep, L, stream), stream, 4)) / NL
            nonflush = {}
            for bv in (32, 64, 128):
                per = time_cycles(capture_positions(lambda s, bv=bv: replay(s, bv), L - 1, stream), stream, 4)
                nonflush[bv] = [1e3 * t / NL for t in per]
            best = [min(nonflush[bv][i] for bv in nonflush) for i in range(L - 1)]
            flush_us = 1e3 * time_cycles(capture_positions(lambda s: replay(L - 1, 32), 1, stream), stream, 4)[0] / NL
            split_us = 1e3 * time_cycles(capture_positions(lambda s: split(L - 2), 1, stream), stream, 4)[0] / NL
        except Exception as e:
            res[f"L{L}"] = {"error": f"{type(e).__name__}: {e}"[:300]}
            continue
        core = (sum(best) + flush_us) / L
        res[f"L{L}"] = {"layers": NL, "prep_us": prep_us, "replay_us_by_fill": best,
                        "replay_us_full_ring_nonflush": best[-1], "flush_us": flush_us,
                        "split_us_fill_L_minus_1": split_us, "core_us_per_layer_step": core,
                        "full_contract_us_per_layer_step": core + prep_us,
                        "best_block_v_by_fill": [min(nonflush, key=lambda bv: nonflush[bv][i]) for i in range(L - 1)]}
        del lay
        torch.cuda.empty_cache()
    return res


def run_core(args, device, stream):
    """core replay (non-flush) of a full L=16 ring, block-V sweep."""
    import torch

    import gdnr
    from gdnr import inputs as gin
    from gdnr import traffic

    B, L, NL = args.batch, args.ring, args.layers
    sets = []
    for li in range(NL):
        d = gin.replay_ring_inputs(B, L, seed=args.seed * 7 + li, device=device)
        ck = gdnr.quantize_checkpoint(d["state"], scale_dtype=torch.float32, compute_saturation=False)
        sets.append((ck, d, torch.full((B,), L, dtype=torch.int32, device=device),
                     torch.zeros(B, dtype=torch.bool, device=device),
                     torch.empty(B, HV, KD, dtype=torch.bfloat16, device=device)))
    res = {}
    nbytes = traffic.step_bytes(B, L, L, fused=False)

    def run():
        for ck, d, vl, fl, out in sets:
            gdnr.gdn_replay_fp8(ck.payload, ck.scale, d["q"], d["k"], d["v"], d["g"], d["beta"], vl, fl, out=out,
                                flush_hint="none")

    # gdn_replay_fp8_split (kern.py:1129-1235): precompute + apply launches, caller T / c
    # buffers; and the variant without caller scratch (library-owned static buffers)
    tq = torch.empty(B, HV, KD, dtype=torch.float32, device=device)
    coef = torch.empty(B, HV, L, dtype=torch.float32, device=device)

    def run_split():
        for ck, d, vl, fl, out in sets:
            gdnr.gdn_replay_fp8_split(ck.payload, ck.scale, d["q"], d["k"], d["v"], d["g"], d["beta"], vl, tq, coef,
                                      out=out)

    def run_split_static():
        for ck, d, vl, fl, out in sets:
            gdnr.gdn_replay_fp8_split_static(ck.payload, ck.scale, d["q"], d["k"], d["v"], d["g"], d["beta"], vl, out)

    def graph_us(fn):
        torch.cuda.synchronize()  # the inputs above come from the default stream
        with torch.cuda.stream(stream):
            fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            fn()
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
        del g
        return 1e3 * e0.elapsed_time(e1) / (reps * NL)

    us = graph_us(run)
    res.update({"us_per_launch": us, "GB_s": nbytes / (us * 1e-6) / 1e9, "steps_seq_per_s": B / (us * 1e-6),
                "frac_of_peak": nbytes / (us * 1e-6) / 1e9 / measured_peak()[0]})
    res["algorithmic_bytes_per_launch"] = nbytes
    res["workload"] = "config2: gdn_replay_fp8 non-flush, B=64, full L=16 ring, f32 scales/gates"
    us_split = graph_us(run_split)
    us_static = graph_us(run_split_static)
    res["split"] = {"us_per_call": us_split, "static_us_per_call": us_static,
                    "ratio_to_fused_replay": us_split / us,
                    "workload": "gdn_replay_fp8_split (precompute + apply, caller T [B,HV,K] / c [B,HV,L] f32 "
                                "buffers) and gdn_replay_fp8_split_static (no caller scratch), same inputs"}
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
        elif args.drift:
            run_drift(args, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        if args.impl == "ours" and world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
