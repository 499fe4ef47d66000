"""bench.py's reference arm (`--impl reference`) on the host: one JSON line in
the bench contract, the reference's own CPU replay when a copy of its
prototype sits in baseline/_ref (else the numpy port), the requested warm-up
and whole ring cycles.  CPU only; a tiny configuration so it runs in seconds."""

import json
import pathlib
import subprocess
import sys

ROOT = pathlib.Path(__file__).resolve().parents[1]


def test_reference_arm_line():
    cmd = [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--batch", "2", "--ring", "4",
           "--steps", "8", "--warmup", "2"]
    run = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert run.returncode == 0, run.stderr[-2000:]
    lines = [ln for ln in run.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, run.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["unit"] == "steps·seq/s"
    cpu = d["cpu_baseline"]
    assert cpu["kind"] in ("reference", "port") and cpu["cores"] >= 1
    assert cpu["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    if cpu["kind"] == "reference":
        # the reference's replay_decode: the requested warm-up steps, then whole L = 4 cycles
        assert d["warmup"] == 2
        assert d["steps"] % 4 == 0 and 4 <= d["steps"] <= 8
