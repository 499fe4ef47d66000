"""ctypes binding of libgdnr.so (the C ABI declared in include/gdnr.h).

The library is loaded from this directory.  There is no fallback: if the
shared object is missing, every operator raises.
"""

from __future__ import annotations

import ctypes
import pathlib
import threading

import torch

LIB_PATH = pathlib.Path(__file__).resolve().parent / "libgdnr.so"

# gdnr_dtype
DT_NONE, F32, F16, BF16, E4M3, I32, U8, I8 = range(8)

_TORCH_DT = {
    torch.float32: F32,
    torch.float16: F16,
    torch.bfloat16: BF16,
    torch.float8_e4m3fn: E4M3,
    torch.int32: I32,
    torch.bool: U8,
    torch.uint8: U8,
    torch.int8: I8,
}

# gdnr_status
OK, ERR_ARG, ERR_DTYPE, ERR_LAYOUT, ERR_ALIAS, ERR_UNSUPPORTED, ERR_CUDA = 0, -1, -2, -3, -4, -5, -6
STATUS_NAMES = {
    ERR_ARG: "GDNR_ERR_ARG",
    ERR_DTYPE: "GDNR_ERR_DTYPE",
    ERR_LAYOUT: "GDNR_ERR_LAYOUT",
    ERR_ALIAS: "GDNR_ERR_ALIAS",
    ERR_UNSUPPORTED: "GDNR_ERR_UNSUPPORTED",
    ERR_CUDA: "GDNR_ERR_CUDA",
}

DEVERR_WAIT_TIMEOUT = 0x1
DEVERR_BAD_POS = 0x2
DEVERR_BAD_HINT = 0x4
DEVERR_BAD_SLOT = 0x8
DEVERR_LAYOUT = 0x10


class Tensor(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("ndim", ctypes.c_int32),
        ("shape", ctypes.c_int64 * 4),
        ("stride", ctypes.c_int64 * 4),
    ]


_U32P = ctypes.POINTER(ctypes.c_uint32)


class ReplayArgs(ctypes.Structure):
    _fields_ = [(n, Tensor) for n in ("checkpoint", "scale", "q", "k_ring", "v_ring", "g_ring", "beta_ring",
                                      "valid_len", "flush", "out")] + [
        ("block_v", ctypes.c_int32),
        ("quant_divisor", ctypes.c_int32),
        ("error_flag", ctypes.c_void_p),
        ("flush_hint", ctypes.c_int32),
        ("launch_flags", ctypes.c_int32),
    ]


class ReplaySplitArgs(ctypes.Structure):
    _fields_ = [(n, Tensor) for n in ("checkpoint", "scale", "q", "k_ring", "v_ring", "g_ring", "beta_ring",
                                      "valid_len", "tq", "coef", "out")] + [
        ("block_v", ctypes.c_int32),
        ("error_flag", ctypes.c_void_p),
    ]


class ReplaySplitStaticArgs(ctypes.Structure):
    _fields_ = [(n, Tensor) for n in ("checkpoint", "scale", "q", "k_ring", "v_ring", "g_ring", "beta_ring",
                                      "valid_len", "out")] + [
        ("block_v", ctypes.c_int32),
        ("error_flag", ctypes.c_void_p),
    ]


class PrepArgs(ctypes.Structure):
    _fields_ = [(n, Tensor) for n in ("mixed_qkv", "a", "b", "a_log", "dt_bias", "pos", "q_out", "k_ring",
                                      "v_ring", "g_ring", "beta_ring")] + [
        ("error_flag", ctypes.c_void_p),
    ]


class StepArgs(ctypes.Structure):
    _fields_ = [(n, Tensor) for n in ("mixed_qkv", "a", "b", "a_log", "dt_bias", "pos", "pos_out", "checkpoint",
                                      "scale", "k_ring", "v_ring", "g_ring", "beta_ring", "out", "q_out")] + [
        ("quant_divisor", ctypes.c_int32),
        ("error_flag", ctypes.c_void_p),
        ("flush_hint", ctypes.c_int32),
        ("launch_flags", ctypes.c_int32),
    ]


class PackedDecodeArgs(ctypes.Structure):
    _fields_ = [(n, Tensor) for n in ("mixed_qkv", "a", "b", "a_log", "dt_bias", "state_indices", "pos", "pos_out",
                                      "checkpoint", "scale", "k_ring", "v_ring", "g_ring", "beta_ring", "out")] + [
        ("qk_scale", ctypes.c_float),
        ("use_qk_l2norm", ctypes.c_int32),
        ("quant_divisor", ctypes.c_int32),
        ("error_flag", ctypes.c_void_p),
        ("flush_hint", ctypes.c_int32),
        ("launch_flags", ctypes.c_int32),
    ]


class CodecArgs(ctypes.Structure):
    _fields_ = [(n, Tensor) for n in ("state", "payload", "scale")] + [
        ("quant_divisor", ctypes.c_int32),
        ("saturation_count", ctypes.c_void_p),
    ]


class Bf16StepArgs(ctypes.Structure):
    _fields_ = [(n, Tensor) for n in ("state", "q", "k", "v", "g", "beta", "out")]


# symbol -> (argtypes, restype); every symbol include/gdnr.h declares
SIGNATURES = {
    "gdnr_replay": ([ctypes.POINTER(ReplayArgs), ctypes.c_void_p], ctypes.c_int),
    "gdnr_replay_split": ([ctypes.POINTER(ReplaySplitArgs), ctypes.c_void_p], ctypes.c_int),
    "gdnr_replay_split_static": ([ctypes.POINTER(ReplaySplitStaticArgs), ctypes.c_void_p], ctypes.c_int),
    "gdnr_prep_ring": ([ctypes.POINTER(PrepArgs), ctypes.c_void_p], ctypes.c_int),
    "gdnr_fused_step": ([ctypes.POINTER(StepArgs), ctypes.c_void_p], ctypes.c_int),
    "gdnr_packed_decode": ([ctypes.POINTER(PackedDecodeArgs), ctypes.c_void_p], ctypes.c_int),
    "gdnr_quantize_vblock32": ([ctypes.POINTER(CodecArgs), ctypes.c_void_p], ctypes.c_int),
    "gdnr_dequantize_vblock32": ([ctypes.POINTER(CodecArgs), ctypes.c_void_p], ctypes.c_int),
    "gdnr_bf16_step": ([ctypes.POINTER(Bf16StepArgs), ctypes.c_void_p], ctypes.c_int),
    "gdnr_last_error": ([], ctypes.c_char_p),
    "gdnr_version": ([], ctypes.c_char_p),
    "gdnr_abi_version": ([], ctypes.c_int),
    "gdnr_read_device_error": ([_U32P, ctypes.c_int], ctypes.c_int),
    "gdnr_selftest_wait_timeout": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p], ctypes.c_int),
}

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load libgdnr.so once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python fp8-replayssm-gdn-kernel_b200/csrc/build.py` "
                    "(there is no CPU fallback)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (argtypes, restype) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = argtypes
                fn.restype = restype
            _lib = lib
    return _lib


class GdnrError(RuntimeError):
    """A libgdnr call failed; ``status`` is the gdnr_status code."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class GdnrValueError(GdnrError, ValueError):
    """Invalid arguments (shape/dtype/layout/alias/unsupported geometry)."""


def check(rc: int) -> None:
    if rc == OK:
        return
    msg = load().gdnr_last_error().decode(errors="replace")
    if rc == ERR_CUDA:
        raise GdnrError(rc, msg)
    raise GdnrValueError(rc, msg)


def tensor_desc(t: torch.Tensor | None, require_cuda: bool = True) -> Tensor:
    """Describe a torch tensor for the C ABI (None -> absent argument)."""
    d = Tensor()
    if t is None:
        return d
    if t.dtype not in _TORCH_DT:
        raise ValueError(f"dtype {t.dtype} is not supported by libgdnr")
    if require_cuda and t.device.type != "cuda":
        raise ValueError(f"libgdnr operates on CUDA tensors; got a tensor on {t.device}")
    if t.dim() > 4:
        raise ValueError("libgdnr tensors have at most 4 dimensions")
    d.data = t.data_ptr() if t.numel() > 0 else (t.data_ptr() or 16)
    d.dtype = _TORCH_DT[t.dtype]
    d.ndim = t.dim()
    for i, (s, st) in enumerate(zip(t.shape, t.stride())):
        d.shape[i] = s
        d.stride[i] = st
    return d


def stream_handle(device: torch.device | None = None) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def call(name: str, args: ctypes.Structure, device: torch.device) -> None:
    """Run entry point ``name`` on ``device``'s current stream with that device
    current (the library configures and launches on the current device)."""
    fn = getattr(load(), name)
    if device.index is None or device.index == torch.cuda.current_device():
        check(fn(ctypes.byref(args), stream_handle(device)))
        return
    with torch.cuda.device(device):
        check(fn(ctypes.byref(args), stream_handle(device)))
