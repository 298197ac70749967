"""Selective DIP MLP — the reference's dip_stream_predispatch.py API on B200.

On the reference's T4 the up/down rows of the selected channels were gathered
on the CPU and streamed over PCIe each token.  On a B200 the whole int4 model
is resident in HBM, so StreamingDIPMlp keeps every weight on the GPU and a
decode token is one persistent kernel (gate GEMV + SiLU, exact top-k,
gathered up GEMV with h = g*u, gathered down; layer_fused_kernel) where the
shape allows it, else four kernels with no host synchronisation (reference
forward: dip_stream_predispatch.py:176-204).  Prefill (_dense) runs the
dense GEMMs on the tcgen05 tensor cores.  Constructor signatures, attribute
names and the _dense path are kept.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from ._lib import load_ops
from .qlinear import GROUP_SIZE, _require_cuda, dequantize
from .fastpath import dense_mlp, fused_layer_supported
from .gate_kernel import gate_gemv, _use_gate  # noqa: F401
from .topk_kernel import select_topk, _use_topk  # noqa: F401

load_ops()
_use_gather = True
_use_down = True


def _unpack_int4_rows(qweight: torch.Tensor) -> torch.Tensor:
    """dip_stream_predispatch.py:77-89: int8 [R, C/2] -> int8 [R, C]."""
    q = qweight.view(torch.uint8)
    lo = (q & 0x0F).to(torch.int8)
    hi = ((q >> 4) & 0x0F).to(torch.int8)
    lo = torch.where(lo >= 8, lo - 16, lo)
    hi = torch.where(hi >= 8, hi - 16, hi)
    return torch.stack([lo, hi], dim=-1).reshape(q.shape[0], q.shape[1] * 2)


def _pack_int4_rows(q: torch.Tensor) -> torch.Tensor:
    """dip_stream_predispatch.py:92-97: int8 [R, C] in [-8, 7] -> packed [R, C/2]."""
    lo = (q[:, 0::2] & 0x0F).to(torch.uint8)
    hi = (q[:, 1::2] & 0x0F).to(torch.uint8)
    return (lo | (hi << 4)).to(torch.int8)


def _transpose_down_to_int4(down_qw: torch.Tensor, down_sc: torch.Tensor):
    """dip_stream_predispatch.py:100-120: [out, inter] int4 -> transposed
    [inter, out] int4 with scales [inter, out/128] (dequantise, transpose,
    requantise g128 along out), bit exact, on the GPU.  CPU inputs are moved
    to the current CUDA device and the result returned on their device."""
    dev = down_qw.device
    if not down_qw.is_cuda:
        cur = torch.device("cuda", torch.cuda.current_device())
        tq, ts = torch.ops.dip_b200.transpose_down_int4(down_qw.to(cur).contiguous(),
                                                        down_sc.to(cur).contiguous())
        return tq.to(dev), ts.to(dev)
    return torch.ops.dip_b200.transpose_down_int4(down_qw.contiguous(), down_sc.contiguous())


class SharedBuffers:
    """dip_stream_predispatch.py:123-142.  The reference's per-model staging
    buffers for streamed rows.  With HBM-resident weights nothing is staged:
    the gpu_*/pin_* attributes are kept as empty tensors for code that reads
    them, and `local_idx` is kept as in the reference."""

    def __init__(self, k, up_in_packed, up_ngroups, down_out, down_ngroups, device):
        self.k = k
        self.device = torch.device(device)
        e8 = torch.empty(0, up_in_packed, dtype=torch.int8, device=device)
        ebf = torch.empty(0, up_ngroups, dtype=torch.bfloat16, device=device)
        self.gpu_up_qw, self.gpu_up_sc = e8, ebf
        self.gpu_dn_qw = torch.empty(0, down_out // 2, dtype=torch.int8, device=device)
        self.gpu_dn_sc = torch.empty(0, down_ngroups, dtype=torch.bfloat16, device=device)
        self.pin_up_qw = self.pin_up_sc = self.pin_dn_qw = self.pin_dn_sc = None
        self.local_idx = torch.arange(k, dtype=torch.int32, device=device)
        self.copy_stream = None


class StreamingDIPMlp(nn.Module):
    """dip_stream_predispatch.py:145-215, with every weight resident in HBM."""

    def __init__(self, gate_qw, gate_sc, up_qw, up_sc, down_qw, down_sc,
                 shared, keep_ratio=0.6, device="cuda:0"):
        super().__init__()
        self.keep_ratio = keep_ratio
        self.device = torch.device(device)
        self.buf = shared
        self.gate_qw = gate_qw.to(device).contiguous()
        self.gate_sc = gate_sc.to(device).contiguous()
        self.up_qw = up_qw.to(device).contiguous()
        self.up_sc = up_sc.to(device).contiguous()
        self.inter = up_qw.shape[0]
        dn_t_qw, dn_t_sc = _transpose_down_to_int4(down_qw.to(device), down_sc.to(device))
        self.down_t_qw = dn_t_qw.contiguous()   # [inter, out/2]
        self.down_t_sc = dn_t_sc.contiguous()   # [inter, out/128]
        self.out_features = dn_t_qw.shape[1] * 2
        self.k = shared.k
        # Intermediates of the last decode call (device tensors, no sync).
        self.last_g = None
        self.last_idx = None
        self._fused = fused_layer_supported(self.out_features, self.inter, self.device)
        self._ws = None  # decode workspace, zeroed once, left reusable by every call

    def _gate(self, x):
        """dip_stream_predispatch.py:166-174."""
        if x.dim() == 3 and x.shape[1] == 1 and x.shape[0] == 1:
            out = gate_gemv(self.gate_qw, self.gate_sc, x.reshape(-1))
            return out.reshape(x.shape[0], 1, -1)
        w = dequantize(self.gate_qw, self.gate_sc).to(x.dtype)
        return F.linear(x, w)

    def _workspace(self):
        if self._ws is None:
            op = (torch.ops.dip_b200.mlp_fused_workspace_bytes if self._fused
                  else torch.ops.dip_b200.mlp_workspace_bytes)
            nb = op(self.out_features, self.inter, self.k)
            self._ws = torch.zeros(nb, dtype=torch.uint8, device=self.device)
        return self._ws

    def reset_workspace(self):
        """Zero the decode workspace again (after the device error word
        reported a bounded wait that ran out)."""
        if self._ws is not None:
            self._ws.zero_()

    def decode_token(self, xf: torch.Tensor):
        """One token [hidden] -> (y [hidden] bf16, g [inter] bf16, idx [k] int32)."""
        xf = xf.reshape(-1).to(torch.bfloat16)
        args = (self.gate_qw, self.gate_sc, self.up_qw, self.up_sc, self.down_t_qw,
                self.down_t_sc)
        if self._fused:
            return torch.ops.dip_b200.mlp_decode_fused(*args, xf, None, 1e-6, self.k,
                                                       self._workspace())
        return torch.ops.dip_b200.mlp_decode(*args, xf, self.k, self._workspace())

    def forward(self, x):
        if x.dim() != 3 or x.shape[1] != 1 or self.keep_ratio >= 0.999:
            return self._dense(x)
        _require_cuda(x)
        xdt = x.dtype
        ys = []
        # The reference decode path handles one token; each row of a batch is
        # an independent DIP token with its own selection.
        for b in range(x.shape[0]):
            y, g, idx = self.decode_token(x[b, 0])
            ys.append(y)
        self.last_g, self.last_idx = g, idx
        return torch.stack(ys).to(xdt).reshape(x.shape[0], 1, -1)

    def _dense(self, x):
        """dip_stream_predispatch.py:206-215 (prefill / keep_ratio ~ 1): the
        three GEMMs on the tensor cores (dequantize + F.linear for shapes the
        tcgen05 GEMMs do not take)."""
        y = dense_mlp(self.gate_qw, self.gate_sc, self.up_qw, self.up_sc, self.down_t_qw,
                      self.down_t_sc, x)
        if y is not None:
            return y
        g = F.silu(self._gate(x))
        up_w = dequantize(self.up_qw, self.up_sc).to(x.dtype)
        u = F.linear(x, up_w)
        del up_w
        h = g * u
        dn_t = dequantize(self.down_t_qw, self.down_t_sc).to(x.dtype)
        return h @ dn_t
