"""The C ABI without a GPU: the library loads, exports every symbol that
include/gdnr.h declares, its structs have the layout the ctypes binding
assumes, and argument validation rejects bad calls before any launch."""

import ctypes
import pathlib
import re
import shutil
import subprocess

import pytest

from gdnr import _lib

ROOT = pathlib.Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "gdnr.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(gdnr_\w+)\s*\(", text, re.M)))


def test_header_declares_the_expected_surface():
    names = declared_functions()
    for must in ("gdnr_fused_step", "gdnr_replay", "gdnr_replay_split", "gdnr_prep_ring", "gdnr_bf16_step",
                 "gdnr_quantize_vblock32", "gdnr_dequantize_vblock32", "gdnr_last_error"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version_strings():
    lib = _lib.load()
    assert lib.gdnr_abi_version() == 2
    assert b"sm_100a" in lib.gdnr_version()


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_struct_layout_matches_c(tmp_path):
    src = tmp_path / "sz.c"
    structs = {
        "gdnr_tensor": _lib.Tensor,
        "gdnr_replay_args": _lib.ReplayArgs,
        "gdnr_replay_split_args": _lib.ReplaySplitArgs,
        "gdnr_replay_split_static_args": _lib.ReplaySplitStaticArgs,
        "gdnr_prep_args": _lib.PrepArgs,
        "gdnr_step_args": _lib.StepArgs,
        "gdnr_codec_args": _lib.CodecArgs,
        "gdnr_bf16_step_args": _lib.Bf16StepArgs,
    }
    body = "\n".join(f'  printf("{n} %zu\\n", sizeof({n}));' for n in structs)
    body += '\n  printf("off_error_flag %zu\\n", offsetof(gdnr_step_args, error_flag));'
    src.write_text(f'#include <stdio.h>\n#include <stddef.h>\n#include "gdnr.h"\nint main(void) {{\n{body}\n  return 0;\n}}\n')
    exe = tmp_path / "sz"
    subprocess.run(["gcc", "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], check=True, capture_output=True,
                                                       text=True).stdout.splitlines())
    for n, cls in structs.items():
        assert int(out[n]) == ctypes.sizeof(cls), n
    assert int(out["off_error_flag"]) == _lib.StepArgs.error_flag.offset


# ---------------------------------------------------------------- validation (no launch)

FAKE = 0x10000  # 16-byte aligned, never dereferenced: every call below fails validation or has B == 0


def desc(shape, dtype, stride=None, data=FAKE):
    d = _lib.Tensor()
    d.data = data
    d.dtype = dtype
    d.ndim = len(shape)
    if stride is None:
        stride, acc = [], 1
        for s in reversed(shape):
            stride.insert(0, acc)
            acc *= s
    for i, (s, st) in enumerate(zip(shape, stride)):
        d.shape[i] = s
        d.stride[i] = st
    return d


def replay_args(B=2, H=2, HV=4, L=4, K=128, V=128, **over):
    a = _lib.ReplayArgs()
    a.checkpoint = desc([B, HV, V, K], _lib.E4M3)
    a.scale = desc([B, HV, V // 32], _lib.F16)
    a.q = desc([B, H, K], _lib.BF16)
    a.k_ring = desc([B, L, H, K], _lib.BF16)
    a.v_ring = desc([B, L, HV, V], _lib.BF16)
    a.g_ring = desc([B, L, HV], _lib.F32)
    a.beta_ring = desc([B, L, HV], _lib.F32)
    a.valid_len = desc([B], _lib.I32)
    a.flush = desc([B], _lib.U8)
    a.out = desc([B, HV, V], _lib.BF16)
    a.error_flag = FAKE
    for k, v in over.items():
        setattr(a, k, v)
    return a


def call_replay(a):
    lib = _lib.load()
    rc = lib.gdnr_replay(ctypes.byref(a), None)
    return rc, lib.gdnr_last_error().decode()


def test_replay_empty_batch_is_a_noop():
    rc, _ = call_replay(replay_args(B=0))
    assert rc == _lib.OK


@pytest.mark.parametrize(
    "over,code,needle",
    [
        (dict(K=64, V=64), _lib.ERR_UNSUPPORTED, "K = V = 128"),
        (dict(L=65), _lib.ERR_UNSUPPORTED, "ring length"),
        (dict(HV=3), _lib.ERR_ARG, "multiple of H"),
        (dict(H=1, HV=8), _lib.ERR_UNSUPPORTED, "HV/H"),
    ],
)
def test_replay_geometry_errors(over, code, needle):
    rc, msg = call_replay(replay_args(**over))
    assert rc == code and needle in msg


def test_replay_dtype_error():
    a = replay_args(B=0)
    a.k_ring = desc([0, 4, 2, 128], _lib.F32)
    rc, msg = call_replay(a)
    assert rc == _lib.ERR_DTYPE and "k_ring" in msg


def test_replay_shape_mismatch():
    a = replay_args(B=0)
    a.out = desc([0, 4, 64], _lib.BF16)
    rc, msg = call_replay(a)
    assert rc == _lib.ERR_ARG and "out" in msg


def test_replay_layout_errors():
    a = replay_args(B=0)
    a.checkpoint = desc([0, 4, 128, 128], _lib.E4M3, stride=[65536, 16384, 128, 2])
    rc, msg = call_replay(a)
    assert rc == _lib.ERR_LAYOUT and "innermost" in msg
    a = replay_args(B=0)
    a.k_ring = desc([0, 4, 2, 128], _lib.BF16, data=FAKE + 8)
    rc, msg = call_replay(a)
    assert rc == _lib.ERR_LAYOUT and "16-byte" in msg
    a = replay_args(B=2)
    a.v_ring = desc([2, 4, 4, 128], _lib.BF16, stride=[4 * 4 * 132, 4 * 132, 132, 1])
    rc, msg = call_replay(a)
    assert rc == _lib.ERR_LAYOUT and "v_ring" in msg


def test_replay_block_v_error():
    a = replay_args(B=0, block_v=48)
    rc, msg = call_replay(a)
    assert rc == _lib.ERR_ARG and "block_v" in msg


def test_replay_null_args():
    lib = _lib.load()
    assert lib.gdnr_replay(None, None) == _lib.ERR_ARG


def step_args(B=2, H=2, HV=4, L=4, **over):
    a = _lib.StepArgs()
    a.mixed_qkv = desc([B, 2 * H * 128 + HV * 128], _lib.BF16)
    a.a = desc([B, HV], _lib.BF16)
    a.b = desc([B, HV], _lib.BF16)
    a.a_log = desc([HV], _lib.F32)
    a.dt_bias = desc([HV], _lib.F32)
    a.pos = desc([B], _lib.I32)
    a.checkpoint = desc([B, HV, 128, 128], _lib.E4M3)
    a.scale = desc([B, HV, 4], _lib.F32)
    a.k_ring = desc([B, L, H, 128], _lib.BF16)
    a.v_ring = desc([B, L, HV, 128], _lib.BF16)
    a.g_ring = desc([B, L, HV], _lib.F32)
    a.beta_ring = desc([B, L, HV], _lib.F32)
    a.out = desc([B, HV, 128], _lib.BF16)
    a.error_flag = FAKE
    for k, v in over.items():
        setattr(a, k, v)
    return a


def test_fused_step_pos_alias_rejected():
    a = step_args(B=2)
    a.pos_out = desc([2], _lib.I32)  # same FAKE address as pos
    lib = _lib.load()
    assert lib.gdnr_fused_step(ctypes.byref(a), None) == _lib.ERR_ALIAS


def test_fused_step_mixed_width_checked():
    a = step_args(B=2)
    a.mixed_qkv = desc([2, 1000], _lib.BF16)
    lib = _lib.load()
    assert lib.gdnr_fused_step(ctypes.byref(a), None) == _lib.ERR_ARG
    assert "mixed_qkv" in lib.gdnr_last_error().decode()


def test_fused_step_empty_batch_is_a_noop():
    lib = _lib.load()
    assert lib.gdnr_fused_step(ctypes.byref(step_args(B=0)), None) == _lib.OK


def test_f32_checkpoint_rejects_scale():
    a = replay_args(B=0)
    a.checkpoint = desc([0, 4, 128, 128], _lib.F32)
    rc, msg = call_replay(a)
    assert rc == _lib.ERR_ARG and "scale" in msg


def test_codec_alias_rejected():
    a = _lib.CodecArgs()
    a.state = desc([1, 2, 128, 128], _lib.F32)
    a.payload = desc([1, 2, 128, 128], _lib.E4M3)  # same address
    a.scale = desc([1, 2, 4], _lib.F16, data=FAKE * 4)
    lib = _lib.load()
    assert lib.gdnr_quantize_vblock32(ctypes.byref(a), None) == _lib.ERR_ALIAS


def test_python_wrapper_rejects_host_tensors():
    import torch

    import gdnr

    state = torch.zeros(1, 2, 128, 128)
    with pytest.raises(ValueError, match="CUDA"):
        gdnr.quantize_checkpoint(state)
