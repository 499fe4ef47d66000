"""Persistent decode state of the replay scheme, resident in HBM.

Per sequence and GDN layer the state is the tuple the reference passes to
its kernels (prototype/gdn_replayssm_fp8_kernel.py:344-405 and
prototype/bench_gdn_full_contract.py:113-135):

* ``checkpoint`` [B,HV,V,K] float8_e4m3fn -- the FP8 snapshot at the start
  of the current window (int8 codes for the "vblock_int8" option, float32 for
  the full-precision variant);
* ``scale`` [B,HV,V/32] -- one scale per 32 value rows (float16 as the
  reference stores it, or float32 holding the float16-rounded value);
* the ring of the last L tokens: ``k`` [B,L,H,K] bf16, ``v`` [B,L,HV,V] bf16,
  ``g``/``beta`` [B,L,HV] float32 (or bf16);
* ``pos`` [B] int32 -- the ring slot the next token goes to.

HBM per sequence and layer at H=16, HV=32, K=V=128, L=16: 512 KiB checkpoint,
512 B scales (f32), 12.25 KiB per ring slot (196 KiB for L=16).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops


@dataclass
class ReplayState:
    checkpoint: torch.Tensor
    scale: torch.Tensor | None
    k_ring: torch.Tensor
    v_ring: torch.Tensor
    g_ring: torch.Tensor
    beta_ring: torch.Tensor
    pos: torch.Tensor

    @property
    def batch(self) -> int:
        return self.k_ring.shape[0]

    @property
    def ring_len(self) -> int:
        return self.k_ring.shape[1]

    @classmethod
    def allocate(cls, batch: int, heads: int = 16, value_heads: int = 32, ring_len: int = 16,
                 key_dim: int = 128, value_dim: int = 128, device: torch.device | str = "cuda",
                 scale_dtype: torch.dtype = torch.float32, gate_dtype: torch.dtype = torch.float32,
                 checkpoint_dtype: torch.dtype = torch.float8_e4m3fn) -> "ReplayState":
        dev = torch.device(device)
        ck = torch.zeros(batch, value_heads, value_dim, key_dim, dtype=checkpoint_dtype, device=dev)
        sc = (torch.ones(batch, value_heads, value_dim // 32, dtype=scale_dtype, device=dev)
              if checkpoint_dtype != torch.float32 else None)
        return cls(
            checkpoint=ck,
            scale=sc,
            k_ring=torch.zeros(batch, ring_len, heads, key_dim, dtype=torch.bfloat16, device=dev),
            v_ring=torch.zeros(batch, ring_len, value_heads, value_dim, dtype=torch.bfloat16, device=dev),
            g_ring=torch.zeros(batch, ring_len, value_heads, dtype=gate_dtype, device=dev),
            beta_ring=torch.zeros(batch, ring_len, value_heads, dtype=gate_dtype, device=dev),
            pos=torch.zeros(batch, dtype=torch.int32, device=dev),
        )

    def load_state(self, state: torch.Tensor, quant_divisor: str = "oracle") -> None:
        """Set the checkpoint from a float32 state [B,HV,V,K] (quantised on the GPU)."""
        if self.checkpoint.dtype == torch.float32:
            self.checkpoint.copy_(state)
            return
        gran = "vblock_int8" if self.checkpoint.dtype == torch.int8 else "vblock"
        ops.quantize_checkpoint(state.float().contiguous(), gran, payload=self.checkpoint, scale=self.scale,
                                scale_dtype=self.scale.dtype, quant_divisor=quant_divisor,
                                compute_saturation=False)

    def snapshot(self) -> "ReplayState":
        """Deep copy (checkpoint/resume of the persistent decode state)."""
        return ReplayState(*(None if t is None else t.clone() for t in (
            self.checkpoint, self.scale, self.k_ring, self.v_ring, self.g_ring, self.beta_ring, self.pos)))

    def restore(self, snap: "ReplayState") -> None:
        for dst, src in zip((self.checkpoint, self.scale, self.k_ring, self.v_ring, self.g_ring, self.beta_ring,
                             self.pos), (snap.checkpoint, snap.scale, snap.k_ring, snap.v_ring, snap.g_ring,
                                         snap.beta_ring, snap.pos)):
            if dst is not None:
                dst.copy_(src)

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (
            self.checkpoint, self.scale, self.k_ring, self.v_ring, self.g_ring, self.beta_ring, self.pos)
            if t is not None)

    def step(self, mixed_qkv, a, b, a_log, dt_bias, out=None, pos_out=None, q_out=None,
             quant_divisor: str = "oracle", error_flag=None, flush_hint: str = "auto",
             pdl: bool = False) -> torch.Tensor:
        """One fused decode step on this state (see :func:`gdnr.ops.gdn_fused_step`)."""
        return ops.gdn_fused_step(mixed_qkv, a, b, a_log, dt_bias, self.pos, self.checkpoint, self.scale,
                                  self.k_ring, self.v_ring, self.g_ring, self.beta_ring, out=out, q_out=q_out,
                                  pos_out=pos_out, quant_divisor=quant_divisor, error_flag=error_flag,
                                  flush_hint=flush_hint, pdl=pdl)
