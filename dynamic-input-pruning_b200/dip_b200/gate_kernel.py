"""gate_gemv() — the reference's gate_kernel.py API over the sm_100a kernel.

The reference loads kernels/int4_gemv/*.so with ctypes and falls back when it
is absent (gate_kernel.py:12-26).  Here the kernel is always present (import
fails otherwise), so _use_gate is True.
"""
import torch

from ._lib import load_ops

load_ops()
_use_gate = True


def gate_gemv(qweight: torch.Tensor, scales: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """gate_kernel.py:29-34: gate_proj(x) for one token x [in] -> bf16 [out]."""
    return torch.ops.int4_ops.int4_gemv(qweight, scales, x.to(torch.bfloat16).contiguous())


def gate_silu(qweight: torch.Tensor, scales: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """bf16(silu(gate_proj(x))) in one launch (the SiLU of
    dip_stream_predispatch.py:182 fused into the GEMV epilogue)."""
    return torch.ops.dip_b200.gate_silu(qweight, scales, x.to(torch.bfloat16).contiguous())
