"""INT4 (g128, symmetric) linear layer — the reference's qlinear.py API on B200.

Format (qlinear.py:1-15 of the reference): qweight int8 [out, in/2], two signed
nibbles per byte, low nibble = even column; scales bf16 [out, in/128].

QuantLinear.forward runs the sm_100a int4 GEMV for a single token and, for
several tokens, the dequantise kernel followed by a dense GEMM.  All tensors
live on the GPU; there is no CPU path.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from ._lib import load_ops

load_ops()

GROUP_SIZE = 128


def _require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("dip_b200 runs on CUDA tensors only (got a tensor on "
                               f"{t.device}); move the weights to the GPU first")


def _unpack_int4(qweight: torch.Tensor) -> torch.Tensor:
    """qlinear.py:28-49: int8 [out, in/2] -> int8 [out, in] with values in [-8, 7]."""
    q = qweight.view(torch.uint8)
    lo = (q & 0x0F).to(torch.int8)
    hi = ((q >> 4) & 0x0F).to(torch.int8)
    lo = torch.where(lo >= 8, lo - 16, lo)
    hi = torch.where(hi >= 8, hi - 16, hi)
    return torch.stack([lo, hi], dim=-1).reshape(q.shape[0], q.shape[1] * 2)


def dequantize(qweight: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """qlinear.py:52-64: bf16 [out, in] = bf16(q * s), bit exact (CUDA kernel)."""
    _require_cuda(qweight, scales)
    return torch.ops.dip_b200.dequantize_int4(qweight.contiguous(), scales.contiguous())


class QuantLinear(nn.Module):
    """INT4 g128 symmetric linear (qlinear.py:67-88), same buffers."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        assert in_features % GROUP_SIZE == 0
        self.register_buffer("qweight",
                             torch.empty(out_features, in_features // 2, dtype=torch.int8))
        self.register_buffer("scales", torch.empty(out_features, in_features // GROUP_SIZE,
                                                   dtype=torch.bfloat16))
        self.bias = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        _require_cuda(x, self.qweight)
        if x.numel() == self.in_features:  # one token: int4 GEMV kernel
            y = torch.ops.int4_ops.int4_gemv(self.qweight, self.scales,
                                             x.reshape(-1).to(torch.bfloat16))
            return y.to(x.dtype).reshape(*x.shape[:-1], self.out_features)
        from .fastpath import tc_linear, tc_linear_ok
        if tc_linear_ok(self.in_features, x):  # tokens x rows GEMM on the tensor cores
            y = tc_linear(self.qweight, self.scales, x.reshape(-1, self.in_features))
            return y.reshape(*x.shape[:-1], self.out_features)
        w = dequantize(self.qweight, self.scales)
        return F.linear(x, w.to(x.dtype))


def _replace_linears_with_quant(model: nn.Module) -> list[str]:
    """qlinear.py:91-106: swap the seven projection nn.Linear modules per layer
    for QuantLinear (empty buffers; weights are loaded separately)."""
    names = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
    replaced = []
    for name, module in model.named_modules():
        for child_name, child in list(module.named_children()):
            full = f"{name}.{child_name}" if name else child_name
            if isinstance(child, nn.Linear) and any(s in full for s in names):
                setattr(module, child_name, QuantLinear(child.in_features, child.out_features))
                replaced.append(full)
    return replaced
