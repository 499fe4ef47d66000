"""Real-decode captures as inputs of the replay step.

A capture is what the reference's recorder writes while a serving engine
decodes (prototype/qwen35_capture_raw.py:100-131): a dict keyed by GDN layer
index whose records hold, per decode step of one sequence (batch 1),

* ``mixed_qkv``: list of [1, 2*H*K + HV*V] bf16 (the raw projection output),
* ``a``, ``b``: lists of [1, HV] float32,
* ``production_out``: list of [1, HV*V] bf16 (the production op's output),
* ``state``: [1, HV, V, K] float32, the layer's state before the first step,
* ``a_log``, ``dt_bias``: [HV] float32, ``scale``: float,
  ``use_qk_l2norm_in_kernel``: bool.

:func:`captured_inputs` turns one layer's window into the batch the fused step
takes, replicated across the batch as the reference's full-contract bench does
(prototype/bench_gdn_full_contract.py:83-110: the capture is batch 1; the
kernel has no data-dependent control flow, so replication is sound for timing,
and it keeps the checkpoint and ring self-consistent for validation).  Replay it
with :class:`gdnr.ReplayState`::

    rec = gdnr.capture.load_capture("capture.pt")
    d = gdnr.capture.captured_inputs(rec, batch=64, layer=0, steps=16, device="cuda")
    st = gdnr.ReplayState.allocate(64, d["heads"], d["value_heads"], ring_len=16)
    st.load_state(d["state"])
    for t in range(d["steps"]):
        st.pos.fill_(t % 16)
        out = st.step(d["mixed_qkv"][:, t], d["a"][:, t], d["b"][:, t], d["a_log"], d["dt_bias"])
        err = gdnr.capture.relative_l2_vs_production(out[0], d["production_out"][t])

The capture files are not shipped with the reference (its results README notes
that they need the engine and the model weights to record).
"""

from __future__ import annotations

import torch

REQUIRED = ("mixed_qkv", "a", "b", "production_out", "state", "a_log", "dt_bias")


def load_capture(path: str) -> dict:
    """Load a capture file (tensors, lists, numbers only: no pickled code is run)."""
    records = torch.load(path, map_location="cpu", weights_only=True)
    if not isinstance(records, dict) or not records:
        raise ValueError(f"{path}: not a capture (expected a non-empty dict of layer records)")
    return records


def capture_geometry(record: dict) -> dict:
    """Heads and dims of one layer record: H, HV, K, V and the steps recorded."""
    missing = [k for k in REQUIRED if k not in record or record[k] is None]
    if missing:
        raise ValueError(f"capture record lacks {missing}")
    state = record["state"]
    if state.dim() != 4 or state.shape[0] != 1:
        raise ValueError(f"capture state must be [1, HV, V, K], got {tuple(state.shape)}")
    _, hv, v, k = state.shape
    width = record["mixed_qkv"][0].shape[-1]
    qk = width - hv * v
    if qk <= 0 or qk % (2 * k):
        raise ValueError(f"mixed_qkv width {width} does not split into q, k (H x {k}) and v ({hv} x {v})")
    steps = len(record["mixed_qkv"])
    for name in ("a", "b", "production_out"):
        if len(record[name]) != steps:
            raise ValueError(f"capture lists differ in length: mixed_qkv {steps}, {name} {len(record[name])}")
    return {"heads": qk // (2 * k), "value_heads": hv, "key_dim": k, "value_dim": v, "steps": steps}


def captured_inputs(records: dict, batch: int, layer: int, steps: int, device="cpu") -> dict:
    """One layer's first ``steps`` decode steps, replicated across ``batch``:
    ``mixed_qkv`` [batch, steps, W] bf16, ``a``/``b`` [batch, steps, HV] float32,
    ``state`` [batch, HV, V, K] float32, ``a_log``/``dt_bias`` [HV],
    ``production_out`` [steps, HV, V] bf16, plus the geometry."""
    if layer not in records:
        raise ValueError(f"layer {layer} not in the capture (layers {sorted(records)})")
    record = records[layer]
    geo = capture_geometry(record)
    steps = min(steps, geo["steps"])
    if steps < 1 or batch < 1:
        raise ValueError("need at least one step and one batch row")
    hv, v = geo["value_heads"], geo["value_dim"]

    def stacked(name, dtype):
        return torch.stack([x.reshape(-1) for x in record[name][:steps]]).to(dtype)

    def replicate(x):
        return x.unsqueeze(0).expand(batch, *x.shape).contiguous().to(device)

    out = {
        "mixed_qkv": replicate(stacked("mixed_qkv", torch.bfloat16)),
        "a": replicate(stacked("a", torch.float32)),
        "b": replicate(stacked("b", torch.float32)),
        "state": replicate(record["state"][0].float()),
        "a_log": record["a_log"].float().reshape(-1).to(device),
        "dt_bias": record["dt_bias"].float().reshape(-1).to(device),
        "production_out": stacked("production_out", torch.bfloat16).reshape(steps, hv, v).to(device),
        "scale": float(record.get("scale", geo["key_dim"] ** -0.5)),
        "use_qk_l2norm_in_kernel": bool(record.get("use_qk_l2norm_in_kernel", True)),
    }
    out.update(geo)
    out["steps"] = steps
    return out


def relative_l2_vs_production(out: torch.Tensor, production_out: torch.Tensor) -> float:
    """||out - production|| / ||production|| over one step's [HV, V] output."""
    a = out.float().reshape(-1).cpu()
    b = production_out.float().reshape(-1).cpu()
    return float(torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b).clamp_min(1e-30))
