"""Batched DIP decode (config 3): B independent tokens per step.

The reference's decode path is batch-1 (dip_stream_predispatch.py:170 and
:182 flatten x and g), so a batch is B independent batch-1 DIP decodes: each
token gets its own top-k over its own gate activations.

path "tc" (default): the tokens share every weight stream.  The gate is a dense
int4 x bf16 GEMM on the tcgen05 tensor cores with the SiLU epilogue; each
token's top-k (`topk_select_batched`) becomes per-channel counts
(`select_count`); the up GEMM's epilogue keeps h = bf16(g * bf16(u)) for the
token's selected channels and 0 elsewhere; the down projection is a dense GEMM
over h (zeros contribute nothing), split over the channels.  With 8 or more
tokens practically every channel is selected by some token, so every row is
read anyway and a dense pass reads each weight once for the whole batch.

path "gather": the per-token form, `gemv_batched` for the gate (up to 8 tokens
per pass over the gate weights, bit identical to the per-token GEMV) and each
token's own gathered up and down over its index list.
"""
from __future__ import annotations

import torch

from ._lib import load_ops
from .stack import RMS_EPS, StackConfig, make_layer

load_ops()


def batched_dip_layer(L: dict, x: torch.Tensor, k: int, path: str = "tc"):
    """x [B, hidden] bf16 -> (y [B, hidden], g [B, inter], idx [B, k])."""
    if path == "tc":
        g = torch.ops.dip_b200.gemm_tc(L["gate_qw"], L["gate_sc"], x, 1)
        idx = torch.ops.dip_b200.topk_select_batched(g, k)
        cnt = torch.ops.dip_b200.select_count(idx, L["gate_qw"].shape[0])
        h = torch.ops.dip_b200.gemm_tc(L["up_qw"], L["up_sc"], x, 2, g, cnt)
        y = torch.ops.dip_b200.down_tc(L["down_t_qw"], L["down_t_sc"], h)
        return y, g, idx
    if path != "gather":
        raise ValueError(f"unknown path {path!r}")
    g = torch.ops.dip_b200.gemv_batched(L["gate_qw"], L["gate_sc"], x, True)
    idx = torch.ops.dip_b200.topk_select_batched(g, k)
    ys = []
    for b in range(x.shape[0]):
        h = torch.ops.dip_b200.gather_up_h(L["up_qw"], L["up_sc"], x[b], g[b], idx[b])
        ys.append(torch.ops.dip_b200.gather_down_idx(L["down_t_qw"], L["down_t_sc"], h, idx[b]))
    return torch.stack(ys), g, idx


class BatchedDipStack:
    """The config-1 stack decoding B tokens per step; per layer the input of
    token b is RMSNorm(y_b + r_b) (unit weight), r an N(0,1) residual."""

    def __init__(self, cfg: StackConfig, batch: int, device="cuda:0", layers=None,
                 path: str = "auto"):
        self.cfg = cfg
        self.batch = batch
        # measured on B200: the dense tensor-core pass wins from 16 tokens on
        self.path = path if path != "auto" else ("tc" if batch >= 16 else "gather")
        self.device = torch.device(device)
        self.layers = layers if layers is not None else [
            make_layer(cfg, l, self.device) for l in range(cfg.n_layers)]
        self._graph = None
        self._static_in = None
        self._static_out = None
        self.last_idx = None

    def step(self, x0: torch.Tensor, resid: torch.Tensor, record: bool = False):
        """x0 [B, H], resid [L, B, H] -> last layer's y [B, H]."""
        y, idxs = None, []
        for l, L in enumerate(self.layers):
            x = x0 if l == 0 else torch.ops.dip_b200.residual_rmsnorm(y, resid[l], RMS_EPS)
            y, g, idx = batched_dip_layer(L, x, self.cfg.k, self.path)
            if record:
                idxs.append(idx)
        if record:
            self.last_idx = idxs
        return y

    def capture(self) -> None:
        B, H, n = self.batch, self.cfg.hidden, self.cfg.n_layers
        self._static_in = (torch.zeros(B, H, dtype=torch.bfloat16, device=self.device),
                           torch.zeros(n, B, H, dtype=torch.bfloat16, device=self.device))
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):
                self.step(*self._static_in)
        torch.cuda.current_stream(self.device).wait_stream(s)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            self._static_out = self.step(*self._static_in)
        self._graph = gr

    def replay(self):
        self._graph.replay()
        return self._static_out
