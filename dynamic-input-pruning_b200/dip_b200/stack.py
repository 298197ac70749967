"""Synthetic Qwen3-32B-shaped DIP decode stack (configs 1 and 2 of the benchmark).

Per layer the input is RMSNorm(prev_y + r) with unit weight, r an N(0,1) bf16
residual; the first layer's input is an N(0,1) token.  Weights are bf16
N(0, 0.02) generated on the GPU from per-layer seeds, quantised int4 g128
with the sm_100a quantiser (bit exact with scripts/quantize.py) and down is
transposed with _transpose_down_to_int4's rule.  The whole stack (64 x ~203
MB) stays resident in HBM.

`DipStack.decode(x0, resid)` is the public call: one token through every
layer, replayed from a CUDA graph captured on first use for the given
buffers' shapes.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ._lib import load_ops

load_ops()

RMS_EPS = 1e-6


@dataclass
class StackConfig:
    n_layers: int = 64
    hidden: int = 5120
    inter: int = 25600
    keep_ratio: float = 0.6
    cache_frac: float = 0.3
    seed: int = 0
    std: float = 0.02
    gate_lognormal: bool = False  # config 2: per-channel LogNormal(0,1) gate row scale

    @property
    def k(self) -> int:
        return max(1, int(round(self.inter * self.keep_ratio)))

    @property
    def cache_n(self) -> int:
        return int(round(self.inter * self.cache_frac))


def make_layer(cfg: StackConfig, layer: int, device) -> dict:
    """One layer's packed weights, generated and quantised on `device`."""
    gen = torch.Generator(device=device).manual_seed(cfg.seed * 100003 + layer)
    H, I = cfg.hidden, cfg.inter
    q = torch.ops.dip_b200.quantize_int4
    wg = torch.randn(I, H, generator=gen, device=device) * cfg.std
    if cfg.gate_lognormal:
        scale = torch.exp(torch.randn(I, 1, generator=gen, device=device))
        wg = wg * scale
    gq, gs = q(wg.to(torch.bfloat16))
    del wg
    wu = (torch.randn(I, H, generator=gen, device=device) * cfg.std).to(torch.bfloat16)
    uq, us = q(wu)
    del wu
    wd = (torch.randn(H, I, generator=gen, device=device) * cfg.std).to(torch.bfloat16)
    dq, ds = q(wd)
    del wd
    tq, ts = torch.ops.dip_b200.transpose_down_int4(dq, ds)
    return {"gate_qw": gq, "gate_sc": gs, "up_qw": uq, "up_sc": us, "down_t_qw": tq,
            "down_t_sc": ts}


def layer_weight_bytes(cfg: StackConfig) -> dict:
    """Algorithmic HBM bytes one decode step of one layer must read."""
    row = cfg.hidden // 2 + 2 * (cfg.hidden // 128)
    return {"gate": cfg.inter * row, "up": cfg.k * row, "down": cfg.k * row,
            "total": (cfg.inter + 2 * cfg.k) * row}


class DipStack:
    """A stack of resident DIP MLP layers with the synthetic inter-layer step.

    mode "fused": one persistent kernel per layer (dip_mlp_decode_fused,
    RMSNorm folded in); "chain": the separate-launch chain (dip_mlp_decode);
    "ca": cache-aware DIP (dip_ca.py:127-188) in one launch per layer
    (dip_mlp_decode_fused_ca: hits read the layer's resident hot rows, misses
    the full matrices); "ca_chain": the same as separate launches (gate, top-k,
    hit/miss split, dual-source up and down).  The CA modes need calibrate_ca()
    first; recording steps also return each layer's split."""

    def __init__(self, cfg: StackConfig, device="cuda:0", layers: list | None = None,
                 fused: bool = True, mode: str | None = None):
        self.cfg = cfg
        self.mode = mode if mode is not None else ("fused" if fused else "chain")
        if self.mode not in ("fused", "chain", "ca", "ca_chain"):
            raise ValueError(f"unknown mode {self.mode!r}")
        self.fused = self.mode == "fused"
        self.device = torch.device(device)
        self.layers = layers if layers is not None else [
            make_layer(cfg, l, self.device) for l in range(cfg.n_layers)]
        self._graph = None
        self._static_in = None
        self._static_out = None
        # Last token's per-layer selections and CA splits (filled when recording).
        self.last_idx = None
        self.last_split = None
        self.ca = None  # per layer: id2slot, cache_ids and resident rows

    @classmethod
    def from_checkpoint(cls, ckpt_dir, device="cuda:0", n_layers: int | None = None,
                        keep_ratio: float = 0.6, mode: str = "fused") -> "DipStack":
        """A stack on the MLP weights of an int4 checkpoint written by the
        reference's scripts/quantize.py (model_int4.safetensors +
        quant_config.json), layers 0 .. n_layers-1."""
        from .checkpoint import load_mlp_layers
        layers = load_mlp_layers(ckpt_dir, device, n_layers)
        I, H = layers[0]["gate_qw"].shape[0], layers[0]["gate_qw"].shape[1] * 2
        cfg = StackConfig(n_layers=len(layers), hidden=H, inter=I, keep_ratio=keep_ratio)
        return cls(cfg, device, layers=layers, mode=mode)

    # -- cache-aware DIP ---------------------------------------------------
    def calibrate_ca(self, x0s: torch.Tensor, resids: torch.Tensor) -> list:
        """Runs the tokens x0s [T, H] (residuals [T, L, H]) through the DIP
        stack, counts every layer's selected channels (as the reference's hook
        does, dip_ca.py:272-300) and loads each layer's hot set: the top
        cache_n channels by (count desc, id asc), kept sorted ascending, with
        id2slot[id] = rank and resident copies of their up / down rows
        (dip_ca.py:107-117).  Returns the per-layer counts."""
        from .dip_ca import _hot_order
        saved = self.mode
        self.mode, self.fused = "fused", True
        cnt = [torch.zeros(self.cfg.inter, dtype=torch.long, device=self.device)
               for _ in self.layers]
        try:
            for t in range(x0s.shape[0]):
                self.step(x0s[t].to(self.device), resids[t].to(self.device), record=True)
                for l, idx in enumerate(self.last_idx):
                    i = idx.long()
                    cnt[l].index_add_(0, i, torch.ones_like(i))
        finally:
            self.mode, self.fused = saved, saved == "fused"
        self.ca = []
        for l, L in enumerate(self.layers):
            hot = _hot_order(cnt[l], self.cfg.inter)[: self.cfg.cache_n].sort().values
            id2 = torch.full((self.cfg.inter,), -1, dtype=torch.long, device=self.device)
            id2[hot] = torch.arange(len(hot), device=self.device)
            self.ca.append({"cache_ids": hot, "id2slot": id2,
                            "res_up_qw": L["up_qw"][hot].contiguous(),
                            "res_up_sc": L["up_sc"][hot].contiguous(),
                            "res_dn_qw": L["down_t_qw"][hot].contiguous(),
                            "res_dn_sc": L["down_t_sc"][hot].contiguous()})
        self._graph = None
        return cnt

    # -- one token, eager -------------------------------------------------
    def step(self, x0: torch.Tensor, resid: torch.Tensor, record: bool = False) -> torch.Tensor:
        """x0 [hidden] bf16, resid [n_layers, hidden] bf16 -> last layer's y."""
        k = self.cfg.k
        fused_ws = self.mode in ("fused", "ca")
        if self.mode != "ca_chain" and (getattr(self, "_ws", None) is None
                                        or self._ws.device != x0.device
                                        or getattr(self, "_ws_fused", None) != fused_ws):
            op = (torch.ops.dip_b200.mlp_fused_workspace_bytes if fused_ws
                  else torch.ops.dip_b200.mlp_workspace_bytes)
            nb = op(self.cfg.hidden, self.cfg.inter, k)
            # zeroed once; every decode call leaves it reusable
            self._ws = torch.zeros(nb, dtype=torch.uint8, device=x0.device)
            self._ws_fused = fused_ws
        if self.mode in ("ca", "ca_chain") and self.ca is None:
            raise RuntimeError("cache-aware mode needs calibrate_ca() first")
        idxs, splits, ys = [], [], []
        y = None
        for l, L in enumerate(self.layers):
            # the next layer's gate rows (layer 0's after the last layer: the
            # next token) are moved into L2 during this layer's tail
            nxt = self.layers[(l + 1) % len(self.layers)]
            if self.mode == "fused":
                xin, r = (x0, None) if l == 0 else (y, resid[l])
                y, g, idx = torch.ops.dip_b200.mlp_decode_fused(
                    L["gate_qw"], L["gate_sc"], L["up_qw"], L["up_sc"], L["down_t_qw"],
                    L["down_t_sc"], xin, r, RMS_EPS, k, self._ws, None, nxt["gate_qw"],
                    nxt["gate_sc"])
            elif self.mode == "ca":
                C = self.ca[l]
                xin, r = (x0, None) if l == 0 else (y, resid[l])
                y, g, idx = torch.ops.dip_b200.mlp_decode_fused_ca(
                    L["gate_qw"], L["gate_sc"], L["up_qw"], L["up_sc"], L["down_t_qw"],
                    L["down_t_sc"], C["id2slot"], C["res_up_qw"], C["res_up_sc"],
                    C["res_dn_qw"], C["res_dn_sc"], xin, r, RMS_EPS, k, self._ws, nxt["gate_qw"],
                    nxt["gate_sc"])
                if record:
                    splits.append(torch.ops.dip_b200.ca_split(idx, C["id2slot"]))
            else:
                x = x0 if l == 0 else torch.ops.dip_b200.residual_rmsnorm(y, resid[l], RMS_EPS)
                if self.mode == "chain":
                    y, g, idx = torch.ops.dip_b200.mlp_decode(L["gate_qw"], L["gate_sc"],
                                                              L["up_qw"], L["up_sc"],
                                                              L["down_t_qw"], L["down_t_sc"],
                                                              x, k, self._ws)
                else:
                    C = self.ca[l]
                    g = torch.ops.dip_b200.gate_silu(L["gate_qw"], L["gate_sc"], x)
                    idx = torch.ops.topk_ops.topk_select(g, k)
                    comb, src, row, n_hit = torch.ops.dip_b200.ca_split(idx, C["id2slot"])
                    h = torch.ops.dip_b200.srcrow_up_h(C["res_up_qw"], C["res_up_sc"],
                                                       L["up_qw"], L["up_sc"], x, g, comb, src,
                                                       row)
                    y = torch.ops.dip_b200.srcrow_down(C["res_dn_qw"], C["res_dn_sc"],
                                                       L["down_t_qw"], L["down_t_sc"], h, src,
                                                       row)
                    if record:
                        splits.append((comb, src, row, n_hit))
            if record:
                idxs.append(idx)
                ys.append(y)
        if record:
            self.last_idx = idxs
            self.last_y = ys
            self.last_split = splits if self.mode in ("ca", "ca_chain") else None
        return y

    def take_device_error(self) -> int:
        """Reads and clears the library's device error word.  A nonzero value
        means a bounded wait ran out: that call's outputs are invalid and the
        workspace's selection state (histograms, counters) may be stale, so
        the workspace is zeroed here before the next call."""
        err = int(torch.ops.dip_b200.take_device_error())
        if err and getattr(self, "_ws", None) is not None:
            self._ws.zero_()
        return err

    # -- one token, CUDA graph --------------------------------------------
    def capture(self) -> None:
        H, n = self.cfg.hidden, self.cfg.n_layers
        self._static_in = (torch.zeros(H, dtype=torch.bfloat16, device=self.device),
                           torch.zeros(n, H, dtype=torch.bfloat16, device=self.device))
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):  # warm the allocator and kernels before capture
                self.step(*self._static_in)
        torch.cuda.current_stream(self.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._static_out = self.step(*self._static_in)
        self._graph = g

    def replay(self) -> torch.Tensor:
        self._graph.replay()
        return self._static_out

    def decode(self, x0: torch.Tensor, resid: torch.Tensor) -> torch.Tensor:
        """Public call: one decode token through every layer.  Inputs may live
        on the host (copied in) or the device; returns y on the inputs' device."""
        if self._graph is None:
            self.capture()
        xi, ri = self._static_in
        xi.copy_(x0, non_blocking=True)
        ri.copy_(resid, non_blocking=True)
        out = self.replay()
        if x0.device.type == "cpu":
            res = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
            res.copy_(out, non_blocking=True)
            torch.cuda.current_stream(self.device).synchronize()
            return res
        return out


def make_stack(cfg: StackConfig, device="cuda:0") -> DipStack:
    return DipStack(cfg, device)


def token_inputs(cfg: StackConfig, n_tokens: int, seed: int, device="cpu"):
    """Seeded N(0,1) bf16 first-layer inputs [T, H] and residuals [T, L, H]."""
    gen = torch.Generator().manual_seed(seed)
    x0 = torch.randn(n_tokens, cfg.hidden, generator=gen).to(torch.bfloat16)
    r = torch.randn(n_tokens, cfg.n_layers, cfg.hidden, generator=gen).to(torch.bfloat16)
    if device != "cpu":
        x0, r = x0.to(device), r.to(device)
    return x0, r
