"""Generate the golden vectors that pin the numpy oracle to the reference.

Run in a container where the reference project is mounted (it is read, never
modified)::

    python tests/golden/make_golden.py --reference <path-to-reference-checkout>

It imports the reference's own ``prototype/gdn_replay_fp8_reference.py``
(pure torch, runs on CPU) and records inputs and outputs of its public
functions on small seeded cases:

* ``codec.npz``     -- ``quantize_checkpoint`` for every granularity plus
  ``dequantize_checkpoint``, on a state that holds the edge cases (all-zero
  vblock, a vblock whose scale underflows float16, one that overflows it,
  exact e4m3 ties, a NaN vblock);
* ``e4m3.npz``      -- torch's float32 -> float8_e4m3fn cast on ties,
  subnormals and random values (the cast the reference uses at ref.py:99);
* ``recurrence.npz`` -- ``run_kernel``, ``baseline_decode`` and
  ``replay_decode`` (full precision and vblock32, full and ragged windows).

The GPU box never runs this script; the tests only read the ``.npz`` files.
"""

from __future__ import annotations

import argparse
import pathlib
import sys

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent


def _np(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy().copy()
    if t.dtype == torch.bfloat16:
        return t.float().numpy().copy()
    return t.numpy().copy()


def codec_state() -> torch.Tensor:
    g = torch.Generator().manual_seed(1234)
    state = torch.randn(2, 3, 128, 64, generator=g) * 0.05
    state[0, 0, 0:32] = 0.0  # amax == 0 -> scale 1.0 (ref.py:36-37)
    state[0, 1, 32:64] *= 1e-6  # amax/448 underflows float16 -> scale 0
    state[0, 2, 64:96] *= 1e9  # amax/448 overflows float16 -> scale inf
    state[1, 0, 0:32, 0] = 1.0  # amax exactly 1 with ties below it
    state[1, 0, 0:32, 1:9] = torch.tensor([0.5, 0.53125, 0.5625, 0.59375, 0.0078125, 0.0087890625,
                                           0.01708984375, 0.002197265625]).mul(1 / 448.0 * 448.0)
    state[1, 1, 96:128, 5] = float("nan")  # NaN vblock (torch.amax propagates NaN)
    return state


def make_codec(ref) -> dict:
    state = codec_state()
    out = {"state": _np(state)}
    for gran in ("vblock", "head", "row", "tile", "vblock_int8"):
        q = ref.quantize_checkpoint(state, gran, 32)
        out[f"{gran}_payload"] = _np(q.payload)
        out[f"{gran}_scale"] = q.scale.numpy().view(np.uint16).copy()
        out[f"{gran}_saturation"] = np.float64(q.saturation_fraction)
        if gran in ("vblock", "tile"):
            out[f"{gran}_dequant"] = _np(ref.dequantize_checkpoint(q))
    # a clean state (no NaN/inf) for dequant-path comparisons
    clean = torch.randn(1, 2, 64, 128, generator=torch.Generator().manual_seed(7)) * 0.02
    qc = ref.quantize_checkpoint(clean, "vblock", 32)
    out["clean_state"] = _np(clean)
    out["clean_payload"] = _np(qc.payload)
    out["clean_scale"] = qc.scale.numpy().view(np.uint16).copy()
    out["clean_saturation"] = np.float64(qc.saturation_fraction)
    out["clean_storage_bytes"] = np.int64(qc.storage_bytes)
    return out


def make_e4m3() -> dict:
    g = torch.Generator().manual_seed(99)
    vals = [torch.randn(3000, generator=g) * s for s in (1e-4, 1e-2, 1.0, 30.0, 200.0)]
    # every e4m3 value, every midpoint between neighbours, and +-1 ulp around each midpoint
    table = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float()
    finite = table[torch.isfinite(table)].unique()
    mids = (finite[1:] + finite[:-1]) / 2
    ulp_up = torch.nextafter(mids, torch.full_like(mids, float("inf")))
    ulp_dn = torch.nextafter(mids, torch.full_like(mids, -float("inf")))
    x = torch.cat(vals + [finite, mids, ulp_up, ulp_dn, -mids]).clamp(-448, 448)
    x = torch.cat([x, torch.tensor([0.0, -0.0, 448.0, -448.0, 2.0**-9, 2.0**-10, 3 * 2.0**-11])])
    return {"x": x.numpy().copy(), "code": x.to(torch.float8_e4m3fn).view(torch.uint8).numpy().copy()}


def recurrence_inputs(seed, batch, tokens, heads, value_heads, key_dim, value_dim):
    g = torch.Generator().manual_seed(seed)
    bf = torch.bfloat16
    q = torch.nn.functional.normalize(torch.randn(batch, tokens, heads, key_dim, generator=g), dim=-1).to(bf)
    k = torch.nn.functional.normalize(torch.randn(batch, tokens, heads, key_dim, generator=g), dim=-1).to(bf)
    v = torch.randn(batch, tokens, value_heads, value_dim, generator=g).to(bf)
    a = torch.randn(batch, tokens, value_heads, generator=g)
    a_log = torch.rand(value_heads, generator=g)
    dt_bias = torch.rand(value_heads, generator=g) - 4.0
    gate = (-a_log.exp() * torch.nn.functional.softplus(a + dt_bias)).to(bf)
    beta = torch.sigmoid(torch.randn(batch, tokens, value_heads, generator=g)).to(bf)
    state = torch.randn(batch, value_heads, value_dim, key_dim, generator=g) * 0.02
    return q.float(), k.float(), v.float(), gate.float(), beta.float(), state


def make_recurrence(ref) -> dict:
    out = {}
    cases = {
        "small": dict(seed=11, batch=2, tokens=8, heads=2, value_heads=4, key_dim=64, value_dim=64),
        "prod": dict(seed=12, batch=1, tokens=6, heads=1, value_heads=2, key_dim=128, value_dim=128),
    }
    for name, cfg in cases.items():
        q, k, v, gate, beta, state = recurrence_inputs(**cfg)
        for key, t in zip(("q", "k", "v", "g", "beta", "state"), (q, k, v, gate, beta, state)):
            out[f"{name}_{key}"] = _np(t)
        o, s = ref.run_kernel(state, q, k, v, gate, beta)
        out[f"{name}_run_out"], out[f"{name}_run_state"] = _np(o), _np(s)
        o, s = ref.baseline_decode(state, q, k, v, gate, beta)
        out[f"{name}_base_out"], out[f"{name}_base_state"] = _np(o), _np(s)
        for window in (4, 3):
            for gran in (None, "vblock"):
                o, s, sat, nbytes = ref.replay_decode(state, q, k, v, gate, beta, window, gran, 32)
                tag = f"{name}_replay_w{window}_{gran or 'fp32'}"
                out[f"{tag}_out"] = _np(o)
                if (window, gran) in ((4, None), (3, "vblock")):
                    out[f"{tag}_state"] = _np(s)
                out[f"{tag}_sat"], out[f"{tag}_bytes"] = np.float64(sat), np.int64(nbytes)
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="root of a checkout of the reference project (its prototype/ directory is imported)")
    args = ap.parse_args()
    sys.path.insert(0, str(pathlib.Path(args.reference) / "prototype"))
    import gdn_replay_fp8_reference as ref  # noqa: E402  (the reference's own oracle)

    torch.set_num_threads(1)
    np.savez_compressed(HERE / "codec.npz", **make_codec(ref))
    np.savez_compressed(HERE / "e4m3.npz", **make_e4m3())
    np.savez_compressed(HERE / "recurrence.npz", **make_recurrence(ref))
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
