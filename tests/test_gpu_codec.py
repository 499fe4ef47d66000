"""GPU vblock32 codec vs the oracle: bit-exact payload bytes and scales given
an identical float32 state (the quantizer contract of ref.py:40-106)."""

import numpy as np
import pytest
import torch

import gdnr
import oracle as O
from helpers import to_dev, to_np

pytestmark = pytest.mark.gpu


def edge_state(rng, B=3, HV=4):
    s = (0.05 * rng.standard_normal((B, HV, 128, 128))).astype(np.float32)
    s[0, 0, 0:32] = 0.0  # amax 0 -> scale 1
    s[0, 1, 32:64] *= np.float32(1e-6)  # fp16 scale underflow -> x/0
    s[0, 2, 64:96] *= np.float32(1e9)  # fp16 scale overflow -> x/inf
    s[1, 0, 0:32, 0] = 1.0
    s[1, 0, 0:32, 1:9] = [0.5, 0.53125, 0.5625, 0.59375, 0.0078125, 0.0087890625, 0.01708984375, 0.002197265625]
    s[1, 1, 96:128, 5] = np.nan  # NaN vblock
    s[2, 3, 32:64, 7] = np.inf
    # values sitting exactly on e4m3 rounding midpoints after division by amax/448
    s[2, 0, 0:32] = (np.float32(1.0 / 448.0) * np.float32(1.0)) * rng.integers(-900, 900, (32, 128)).astype(np.float32) / np.float32(2.0)
    s[2, 0, 0, 0] = np.float32(448.0 / 448.0)
    return s


def compare_payload(got, ref):
    both_nan = ((got & 0x7F) == 0x7F) & ((ref & 0x7F) == 0x7F)
    return int(((got != ref) & ~both_nan).sum())


@pytest.mark.parametrize("divisor", ["oracle", "rounded"])
@pytest.mark.parametrize("scale_dtype", [torch.float16, torch.float32])
def test_quantize_bit_exact(cuda_device, divisor, scale_dtype):
    rng = np.random.default_rng(42)
    s = edge_state(rng)
    q = gdnr.quantize_checkpoint(to_dev(s, torch.float32), scale_dtype=scale_dtype, quant_divisor=divisor)
    ref = O.quantize_vblock32(s, divisor=divisor)
    assert compare_payload(to_np(q.payload), ref.payload) == 0
    got_scale = q.scale.float().cpu().numpy()
    ref_scale = ref.scale.astype(np.float32)
    assert np.array_equal(np.nan_to_num(got_scale, posinf=7e7), np.nan_to_num(ref_scale, posinf=7e7))
    assert q.saturation_fraction == pytest.approx(ref.saturation_fraction, rel=1e-6, abs=1e-12)


def test_quantize_random_large(cuda_device):
    """Bit-exact on a large state ([16,32,128,128] = 8.4M values, N(0,0.05))."""
    rng = np.random.default_rng(7)
    s = (0.05 * rng.standard_normal((16, 32, 128, 128))).astype(np.float32)
    q = gdnr.quantize_checkpoint(to_dev(s, torch.float32))
    ref = O.quantize_checkpoint(s, "vblock", 32)
    assert np.array_equal(to_np(q.payload), ref.payload)
    assert np.array_equal(q.scale.cpu().numpy().view(np.uint16), ref.scale.view(np.uint16))


def test_dequantize_exact(cuda_device):
    rng = np.random.default_rng(3)
    s = (0.05 * rng.standard_normal((2, 8, 128, 128))).astype(np.float32)
    ref = O.quantize_checkpoint(s, "vblock", 32)
    ck = gdnr.QuantizedCheckpoint(to_dev(ref.payload, torch.uint8).view(torch.float8_e4m3fn),
                                  to_dev(ref.scale, torch.float16), "vblock", 32, 0.0)
    d = gdnr.dequantize_checkpoint(ck)
    assert np.array_equal(to_np(d), O.dequantize_checkpoint(ref))


def test_quantize_strided_views(cuda_device):
    """Non-contiguous batch/head strides (a slice of a larger cache)."""
    rng = np.random.default_rng(9)
    big = (0.05 * rng.standard_normal((4, 6, 128, 128))).astype(np.float32)
    state = to_dev(big, torch.float32)[1:3, ::2]
    payload = torch.empty(4, 6, 128, 128, dtype=torch.float8_e4m3fn, device="cuda")[1:3, ::2]
    scale = torch.empty(4, 6, 4, dtype=torch.float16, device="cuda")[1:3, ::2]
    gdnr.quantize_checkpoint(state, payload=payload, scale=scale)
    ref = O.quantize_checkpoint(big[1:3, ::2], "vblock", 32)
    assert np.array_equal(to_np(payload.contiguous()), ref.payload)
    assert np.array_equal(scale.cpu().numpy().view(np.uint16), ref.scale.view(np.uint16))


def _e4m3_midpoints():
    vals = [k * 2.0 ** -9 for k in range(8)]
    vals += [2.0 ** e * (1 + m / 8) for e in range(-6, 9) for m in range(8) if 2.0 ** e * (1 + m / 8) <= 448.0]
    vals = np.array(sorted(vals))
    return ((vals[:-1] + vals[1:]) / 2).astype(np.float32)  # at most 5 significant bits: exact


@pytest.mark.parametrize("divisor", ["oracle", "rounded"])
def test_quantize_near_midpoints(cuda_device, divisor):
    """Quotients on, and a few ulp around, every e4m3 rounding midpoint (normal
    and subnormal range, both signs), for many divisors: bytes equal the IEEE
    division's rounding, ties to even."""
    rng = np.random.default_rng(21)
    mids = _e4m3_midpoints()
    B, HV = 4, 8
    s = (0.1 * rng.standard_normal((B, HV, 128, 128))).astype(np.float32)
    for b in range(B):
        for hv in range(HV):
            for vb in range(4):
                amax = np.float32(10.0 ** rng.uniform(-4, 4))
                d = np.float32(amax / np.float32(448.0))
                if divisor == "rounded":
                    d = np.float32(np.float16(d))
                block = s[b, hv, 32 * vb:32 * vb + 32].reshape(-1)
                x0 = (mids.astype(np.float64) * np.float64(d)).astype(np.float32)
                vals = []
                for k in range(-3, 4):
                    xk = x0.copy()
                    for _ in range(abs(k)):
                        xk = np.nextafter(xk, np.float32(np.inf) if k > 0 else np.float32(0), dtype=np.float32)
                    vals.append(xk)
                v = np.concatenate(vals)
                v = np.concatenate([v, -v])
                v = v[np.abs(v) <= amax]
                block[:] = np.float32(0.01) * amax * rng.standard_normal(block.size).astype(np.float32)
                block[1:1 + v.size] = v
                block[0] = amax
                s[b, hv, 32 * vb:32 * vb + 32] = block.reshape(32, 128)
    q = gdnr.quantize_checkpoint(to_dev(s, torch.float32), quant_divisor=divisor)
    ref = O.quantize_vblock32(s, divisor=divisor)
    assert compare_payload(to_np(q.payload), ref.payload) == 0


def int8_edge_state(rng, B=3, HV=4):
    """Finite edge cases for the int8 codec (NaN codes are host-defined)."""
    s = (0.05 * rng.standard_normal((B, HV, 128, 128))).astype(np.float32)
    s[0, 0, 0:32] = 0.0  # amax 0 -> scale 1
    s[0, 1, 32:64] *= np.float32(1e-6)  # fp16 scale underflow -> x/0
    s[0, 2, 64:96] *= np.float32(1e9)  # fp16 scale overflow
    # exact ties of x / scale: amax = 127/8 -> scale 1/8, x = (k + 1/2)/8
    t = (rng.integers(-126, 126, (32, 128)).astype(np.float32) + np.float32(0.5)) * np.float32(0.125)
    t[0, 0] = np.float32(127.0 * 0.125)
    s[1, 0, 0:32] = t
    s[2, 3, 32:64, 7] = np.float32(1e30)  # one huge value: everything else rounds to 0
    return s


@pytest.mark.parametrize("divisor", ["oracle", "rounded"])
@pytest.mark.parametrize("scale_dtype", [torch.float16, torch.float32])
def test_quantize_int8_bit_exact(cuda_device, divisor, scale_dtype):
    """granularity 'vblock_int8' (ref.py:44-47, :96-97): int8 codes and scales
    bit-exact with the oracle, ties of x/scale rounded to even."""
    rng = np.random.default_rng(44)
    s = int8_edge_state(rng)
    q = gdnr.quantize_checkpoint(to_dev(s, torch.float32), "vblock_int8", scale_dtype=scale_dtype,
                                 quant_divisor=divisor)
    ref = O.quantize_vblock32(s, divisor=divisor, int8=True)
    assert q.payload.dtype == torch.int8 and q.granularity == "vblock_int8"
    assert np.array_equal(q.payload.cpu().numpy(), ref.payload)
    got_scale = q.scale.float().cpu().numpy()
    assert np.array_equal(np.nan_to_num(got_scale, posinf=7e7), np.nan_to_num(ref.scale.astype(np.float32), posinf=7e7))
    assert q.saturation_fraction == pytest.approx(ref.saturation_fraction, rel=1e-6, abs=1e-12)
    # the tie block really has ties, and they went to even
    y = (s[1, 0, 0:32] / np.float32(0.125)).ravel()[1:]  # [0, 0] is the amax element
    assert np.all(np.abs(y - np.floor(y)) == 0.5)


def test_dequantize_int8_exact(cuda_device):
    rng = np.random.default_rng(45)
    s = (0.05 * rng.standard_normal((2, 8, 128, 128))).astype(np.float32)
    ref = O.quantize_checkpoint(s, "vblock_int8", 32)
    ck = gdnr.QuantizedCheckpoint(to_dev(ref.payload, torch.int8), to_dev(ref.scale, torch.float16),
                                  "vblock_int8", 32, 0.0)
    d = gdnr.dequantize_checkpoint(ck)
    assert np.array_equal(to_np(d), O.dequantize_checkpoint(ref))
