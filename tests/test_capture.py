"""Capture loader (real-decode captures, prototype/qwen35_capture_raw.py:100-131
record format) on a synthetic capture written in that format: geometry,
replication across the batch as bench_gdn_full_contract.py:83-110 does, and the
errors for malformed records.  CPU only: no kernel runs here."""

import pytest
import torch

import gdnr


def synthetic_capture(steps=5, H=2, HV=4, K=128, V=128, layers=(0, 3), seed=0):
    g = torch.Generator().manual_seed(seed)
    records = {}
    for layer in layers:
        records[layer] = {
            "mixed_qkv": [torch.randn(1, 2 * H * K + HV * V, generator=g).to(torch.bfloat16) for _ in range(steps)],
            "a": [torch.randn(1, HV, generator=g) for _ in range(steps)],
            "b": [torch.randn(1, HV, generator=g) for _ in range(steps)],
            "production_out": [torch.randn(1, HV * V, generator=g).to(torch.bfloat16) for _ in range(steps)],
            "state": 0.02 * torch.randn(1, HV, V, K, generator=g),
            "a_log": torch.rand(HV, generator=g),
            "dt_bias": torch.randn(HV, generator=g),
            "scale": K ** -0.5,
            "use_qk_l2norm_in_kernel": True,
        }
    return records


def test_load_and_replicate(tmp_path):
    rec = synthetic_capture()
    path = tmp_path / "capture.pt"
    torch.save(rec, path)
    loaded = gdnr.capture.load_capture(str(path))
    d = gdnr.capture.captured_inputs(loaded, batch=3, layer=3, steps=4)
    assert (d["heads"], d["value_heads"], d["key_dim"], d["value_dim"], d["steps"]) == (2, 4, 128, 128, 4)
    assert d["mixed_qkv"].shape == (3, 4, 2 * 2 * 128 + 4 * 128) and d["mixed_qkv"].dtype == torch.bfloat16
    assert d["a"].shape == (3, 4, 4) and d["b"].dtype == torch.float32
    assert d["state"].shape == (3, 4, 128, 128) and d["production_out"].shape == (4, 4, 128)
    for i in range(3):  # every batch row is the recorded sequence
        assert torch.equal(d["mixed_qkv"][i, 2], rec[3]["mixed_qkv"][2][0])
        assert torch.equal(d["a"][i, 1], rec[3]["a"][1][0])
        assert torch.equal(d["state"][i], rec[3]["state"][0])
    assert torch.equal(d["production_out"][0].reshape(-1), rec[3]["production_out"][0][0])
    assert d["scale"] == 128 ** -0.5 and d["use_qk_l2norm_in_kernel"]


def test_steps_clamped_to_recording():
    d = gdnr.capture.captured_inputs(synthetic_capture(steps=3), batch=1, layer=0, steps=16)
    assert d["steps"] == 3 and d["mixed_qkv"].shape[1] == 3


def test_malformed_records_raise():
    rec = synthetic_capture()
    with pytest.raises(ValueError, match="layer 7"):
        gdnr.capture.captured_inputs(rec, 1, 7, 2)
    bad = dict(rec[0], state=None)  # the recorder stores no state when the layer's first call had none
    with pytest.raises(ValueError, match="state"):
        gdnr.capture.capture_geometry(bad)
    bad = dict(rec[0], a=rec[0]["a"][:-1])
    with pytest.raises(ValueError, match="differ in length"):
        gdnr.capture.capture_geometry(bad)
    bad = dict(rec[0], mixed_qkv=[torch.zeros(1, 4 * 128 + 100)])
    with pytest.raises(ValueError, match="does not split"):
        gdnr.capture.capture_geometry(bad)


def test_relative_l2_vs_production():
    p = torch.ones(4, 128, dtype=torch.bfloat16)
    assert gdnr.capture.relative_l2_vs_production(p.float(), p) == 0.0
    assert abs(gdnr.capture.relative_l2_vs_production(1.01 * p.float(), p) - 0.01) < 1e-6
