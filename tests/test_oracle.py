"""The numpy oracle against the reference's own outputs (golden vectors) and
against itself (algebraic identities the reference relies on)."""

import numpy as np
import pytest

import oracle as O


def _load(golden_dir, name):
    return np.load(golden_dir / name)


# ---------------------------------------------------------------- codecs

def test_e4m3_encode_matches_torch_cast(golden_dir):
    g = _load(golden_dir, "e4m3.npz")
    enc = O.e4m3_encode(g["x"])
    assert np.array_equal(enc, g["code"])


def test_e4m3_decode_roundtrip():
    codes = np.arange(256, dtype=np.uint8)
    finite = (codes & 0x7F) != 0x7F
    vals = O.e4m3_decode(codes[finite])
    assert np.array_equal(O.e4m3_encode(vals), codes[finite])
    assert np.isnan(O.e4m3_decode(np.array([0x7F, 0xFF], np.uint8))).all()
    assert O.e4m3_decode(np.array([0x7E], np.uint8))[0] == 448.0
    assert O.e4m3_decode(np.array([0x01], np.uint8))[0] == 2.0**-9


def test_bf16_round_matches_torch():
    import torch

    x = np.random.default_rng(0).standard_normal(100000).astype(np.float32) * np.float32(3.0)
    x = np.concatenate([x, np.array([0.0, -0.0, 1e-40, 3.4e38, np.inf, -np.inf], np.float32)])
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(O.bf16_round(x), ref)


@pytest.mark.parametrize("gran", ["vblock", "head", "row", "tile", "vblock_int8"])
def test_quantize_checkpoint_bit_exact(golden_dir, gran):
    g = _load(golden_dir, "codec.npz")
    q = O.quantize_checkpoint(g["state"], gran, 32)
    ref_payload = g[f"{gran}_payload"]
    got = q.payload.view(np.uint8)
    ref = ref_payload.view(np.uint8)
    if gran.endswith("_int8"):
        # NaN -> int8 is implementation defined in both torch and numpy; the
        # reference test state holds one NaN vblock
        nan_rows = np.isnan(g["state"])
        assert np.array_equal(got[~nan_rows], ref[~nan_rows])
    else:
        # NaN codes: 0x7F or 0xFF (the sign of a generated NaN is platform dependent)
        both_nan = ((got & 0x7F) == 0x7F) & ((ref & 0x7F) == 0x7F)
        assert np.array_equal(got[~both_nan], ref[~both_nan])
    assert np.array_equal(q.scale.view(np.uint16), g[f"{gran}_scale"])
    # the reference takes the mean in float32
    assert q.saturation_fraction == pytest.approx(float(g[f"{gran}_saturation"]), rel=1e-6, abs=1e-9)


def test_quantize_edge_cases_present(golden_dir):
    """The codec fixture really holds the edge cases it claims to."""
    g = _load(golden_dir, "codec.npz")
    scale = g["vblock_scale"].view(np.float16).astype(np.float32)
    assert scale[0, 0, 0] == 1.0  # amax == 0
    assert scale[0, 1, 1] == 0.0  # fp16 underflow
    assert np.isinf(scale[0, 2, 2])  # fp16 overflow
    assert scale[1, 1, 3] == 1.0  # NaN amax -> 1.0 (torch.where(amax > 0, ...))


@pytest.mark.parametrize("gran", ["vblock", "tile"])
def test_dequantize_matches_reference(golden_dir, gran):
    g = _load(golden_dir, "codec.npz")
    q = O.quantize_checkpoint(g["state"], gran, 32)
    d = O.dequantize_checkpoint(q)
    ref = g[f"{gran}_dequant"]
    assert np.array_equal(np.isnan(d), np.isnan(ref))
    fin = ~np.isnan(ref)
    assert np.array_equal(d[fin], ref[fin])


def test_clean_storage_bytes(golden_dir):
    g = _load(golden_dir, "codec.npz")
    q = O.quantize_checkpoint(g["clean_state"], "vblock", 32)
    assert np.array_equal(q.payload, g["clean_payload"])
    assert q.storage_bytes == int(g["clean_storage_bytes"])


# ---------------------------------------------------------------- recurrence

@pytest.mark.parametrize("case", ["small", "prod"])
def test_recurrence_matches_reference(golden_dir, case):
    g = _load(golden_dir, "recurrence.npz")
    q, k, v, gt, b, s = (g[f"{case}_{x}"] for x in ("q", "k", "v", "g", "beta", "state"))
    o, st = O.run_kernel(s, q, k, v, gt, b)
    assert O.relative_l2(o, g[f"{case}_run_out"]) < 1e-6
    assert O.relative_l2(st, g[f"{case}_run_state"]) < 1e-6
    o, st = O.baseline_decode(s, q, k, v, gt, b)
    assert O.relative_l2(o, g[f"{case}_base_out"]) < 1e-6
    assert O.relative_l2(st, g[f"{case}_base_state"]) < 1e-6
    for window in (4, 3):
        for gran in (None, "vblock"):
            tag = f"{case}_replay_w{window}_{gran or 'fp32'}"
            o, st, sat, nbytes = O.replay_decode(s, q, k, v, gt, b, window, gran, 32)
            assert O.relative_l2(o, g[f"{tag}_out"]) < 1e-6, tag
            if f"{tag}_state" in g:
                assert O.relative_l2(st, g[f"{tag}_state"]) < 1e-6, tag
            assert nbytes == int(g[f"{tag}_bytes"])


@pytest.mark.parametrize("window", [2, 3, 4, 8])
def test_full_precision_replay_equals_recurrence(window):
    """ref.py:189-244 with granularity None is exactly the per-token recurrence."""
    rng = np.random.default_rng(window)
    b, t, h, hv, d = 2, 9, 2, 4, 32
    q = O.bf16_round(rng.standard_normal((b, t, h, d)).astype(np.float32) / np.float32(6))
    k = O.bf16_round(rng.standard_normal((b, t, h, d)).astype(np.float32) / np.float32(6))
    v = O.bf16_round(rng.standard_normal((b, t, hv, d)).astype(np.float32))
    gt = O.bf16_round(-np.abs(rng.standard_normal((b, t, hv)).astype(np.float32)))
    bt = O.bf16_round(rng.uniform(0, 1, (b, t, hv)).astype(np.float32))
    s = (rng.standard_normal((b, hv, d, d)) * 0.02).astype(np.float32)
    o1, s1 = O.baseline_decode(s, q, k, v, gt, bt)
    o2, s2, _, _ = O.replay_decode(s, q, k, v, gt, bt, window, None, 32)
    assert O.relative_l2(o2, o1) == 0.0
    assert O.relative_l2(s2, s1) == 0.0


def test_adjoint_replay_equals_forward():
    """The backward T-chain of kern.py:121-176 reproduces run_kernel's last output."""
    rng = np.random.default_rng(5)
    b, L, h, hv, d = 2, 6, 2, 4, 32
    q = O.bf16_round(rng.standard_normal((b, h, d)).astype(np.float32) / np.float32(6))
    k = O.bf16_round(rng.standard_normal((b, L, h, d)).astype(np.float32) / np.float32(6))
    v = O.bf16_round(rng.standard_normal((b, L, hv, d)).astype(np.float32))
    gt = -np.abs(rng.standard_normal((b, L, hv)).astype(np.float32))
    bt = rng.uniform(0, 1, (b, L, hv)).astype(np.float32)
    s = (rng.standard_normal((b, hv, d, d)) * 0.05).astype(np.float32)
    valid = np.array([L, 3])
    got = O.replay_adjoint(s, q, k, v, gt, bt, valid)
    for i in range(b):
        n = valid[i]
        o, _ = O.run_kernel(s[i:i + 1], np.repeat(q[i:i + 1, None], n, 1), k[i:i + 1, :n], v[i:i + 1, :n],
                            gt[i:i + 1, :n], bt[i:i + 1, :n])
        assert O.relative_l2(got[i], o[0, -1]) < 1e-5


@pytest.mark.parametrize("gran", ["vblock", "vblock_int8"])
def test_fused_step_cycle_equals_replay_decode(gran):
    """Driving the full-contract step oracle over T tokens reproduces the
    reference replay chain (ref.py:189-244) on the prepped inputs, for the
    E4M3 and the int8 checkpoint (the flush keeps the payload's format)."""
    rng = np.random.default_rng(3)
    B, T, H, HV, K, L = 2, 7, 1, 2, 128, 3
    mixed = O.bf16_round(rng.standard_normal((T, B, 2 * H * K + HV * K)).astype(np.float32))
    a = rng.standard_normal((T, B, HV)).astype(np.float32)
    bb = rng.standard_normal((T, B, HV)).astype(np.float32)
    a_log = np.log(rng.uniform(1, 16, HV)).astype(np.float32)
    dt_bias = (0.5 * rng.standard_normal(HV)).astype(np.float32)
    s0 = (0.02 * rng.standard_normal((B, HV, K, K))).astype(np.float32)
    q0 = O.quantize_checkpoint(s0, gran, 32)
    st = O.RingState(q0.payload.copy(), q0.scale.copy(), np.zeros((B, L, H, K), np.float32),
                     np.zeros((B, L, HV, K), np.float32), np.zeros((B, L, HV), np.float32),
                     np.zeros((B, L, HV), np.float32))
    outs, qs, ks, vs, gs, bs = [], [], [], [], [], []
    for t in range(T):
        pos = np.full(B, t % L)
        o, qn = O.fused_step(st, mixed[t], a[t], bb[t], a_log, dt_bias, pos, H, K, out_dtype="f32", gate_dtype="f32")
        outs.append(o)
        qn2, kn, v, g, be = O.prep(mixed[t], a[t], bb[t], a_log, dt_bias, H, K, HV, K, gate_dtype="f32")
        qs.append(qn2); ks.append(kn); vs.append(v); gs.append(g); bs.append(be)
    stack = lambda xs: np.stack(xs, axis=1)
    ref_out, ref_state, _, _ = O.replay_decode(s0, stack(qs), stack(ks), stack(vs), stack(gs), stack(bs), L,
                                               gran, 32)
    assert O.relative_l2(np.stack(outs, 1), ref_out) < 1e-6
    # after T=7 tokens with L=3 the ring holds one token past the last flush at t=5
    assert st.payload.dtype == q0.payload.dtype
    assert O.relative_l2(st.dequantized(), O.dequantize_checkpoint(O.quantize_checkpoint(
        O.replay_decode(s0, stack(qs)[:, :6], stack(ks)[:, :6], stack(vs)[:, :6], stack(gs)[:, :6],
                        stack(bs)[:, :6], L, gran, 32)[1], gran, 32))) < 1e-6


def test_prep_formula():
    rng = np.random.default_rng(1)
    B, H, HV, K = 3, 2, 4, 128
    mixed = rng.standard_normal((B, 2 * H * K + HV * K)).astype(np.float32)
    a = np.array([[-30, 0, 19.9, 25.0]] * B, np.float32)
    b = rng.standard_normal((B, HV)).astype(np.float32)
    a_log = np.zeros(HV, np.float32)
    dt_bias = np.zeros(HV, np.float32)
    qn, kn, v, g, beta = O.prep(mixed, a, b, a_log, dt_bias, H, K, HV, K, q_dtype="f32", k_dtype="f32",
                                v_dtype="f32", gate_dtype="f32")
    assert np.allclose(np.linalg.norm(qn, axis=-1), 1.0, atol=1e-5)
    assert np.allclose(np.linalg.norm(kn, axis=-1), 1.0, atol=1e-5)
    assert g[0, 3] == np.float32(-25.0)  # above the softplus threshold: identity
    assert g[0, 1] == pytest.approx(-np.log(2.0), rel=1e-6)
    assert np.allclose(beta, 1 / (1 + np.exp(-b)), rtol=1e-6)
    assert np.array_equal(v, mixed[:, 2 * H * K:].reshape(B, HV, K))


def test_algorithmic_bytes_match_documented_figures():
    # core replay, full ring, B=64, L=16, f32 scales and gates
    assert O.algorithmic_bytes(64, 16, 16, scale_bytes=4, fused=False) == 47_218_688
    cycle = sum(O.algorithmic_bytes(64, n, 16, scale_bytes=4) for n in range(1, 17))
    assert cycle == 705_466_368
    assert cycle // 16 == 44_091_648


def test_package_byte_model_equals_oracle():
    """gdnr.traffic (used by bench.py) and the oracle's byte model agree."""
    from gdnr import traffic

    for B in (1, 4, 64, 256):
        for L in (4, 8, 16, 64):
            for n in range(1, L + 1):
                assert traffic.step_bytes(B, n, L) == O.algorithmic_bytes(B, n, L, scale_bytes=4, gate_bytes=4)
                assert traffic.step_bytes(B, n, L, fused=False) == O.algorithmic_bytes(
                    B, n, L, scale_bytes=4, gate_bytes=4, fused=False)
    assert traffic.cycle_bytes(64, 16) == 44_091_648
