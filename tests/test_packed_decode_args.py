"""Host-side rules of the packed-decode adapter (no GPU): the production call's
use_qk_l2norm_in_kernel and scale arguments are checked before anything is
launched, as the C entry point also does."""

import pytest
import torch

import gdnr


class _NoState:
    """Stands in for the slot pool: the checks fire before the state is touched."""


def _call(**kw):
    z = torch.zeros(1)
    args = dict(mixed_qkv=z, a=z, b=z, A_log=z, dt_bias=z, scale=128 ** -0.5, initial_state=_NoState(), out=z,
                ssm_state_indices=z, use_qk_l2norm_in_kernel=True)
    args.update(kw)
    return gdnr.fused_recurrent_gated_delta_rule_packed_decode(**args)


def test_rejects_unnormalised_qk():
    with pytest.raises(gdnr.GdnrValueError, match="use_qk_l2norm_in_kernel"):
        _call(use_qk_l2norm_in_kernel=False)


@pytest.mark.parametrize("scale", [1.0, 0.0884, 64 ** -0.5])
def test_rejects_other_scales(scale):
    with pytest.raises(gdnr.GdnrValueError, match="scale"):
        _call(scale=scale)


def test_abi_declares_packed_decode():
    text = (pytest.importorskip("pathlib").Path(__file__).resolve().parent.parent / "include" / "gdnr.h").read_text()
    assert "int gdnr_packed_decode(const gdnr_packed_decode_args* args, void* stream);" in text
    assert "gdnr_packed_decode" in gdnr._lib.SIGNATURES
