"""Cache-aware DIP — the reference's dip_ca.py API on B200.

The reference keeps the most frequently selected channels' up/down rows
resident on the GPU and streams the misses over PCIe (dip_ca.py:1-13).  On a
B200 both the resident cache and the full weights sit in HBM; a decode token
is one persistent kernel (layer_fused_kernel with the cache: each selected
channel's up and down rows come from its cache slot when id2slot has one,
else from the full rows) where the shape allows it, else the separate
launches

    gate GEMV + SiLU -> top-k -> hit/miss split (id2slot) ->
    dual-source up GEMV (h = g*u) -> dual-source down

with the split computed on the device (no `.to("cpu")`, no host sync) in the
reference's order: hits in idx order, then misses in idx order
(dip_ca.py:137-142, 164-171); `last_split` gives that split for the last
token either way.  Hits read the resident cache rows, misses the
full resident rows.  Calibration and the deterministic hot-set key
(count*I - id, dip_ca.py:306-308) are unchanged.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from ._lib import load_ops
from .qlinear import _require_cuda, dequantize
from .gate_kernel import gate_gemv, gate_silu
from .topk_kernel import select_topk
from .dip_stream_predispatch import _transpose_down_to_int4
from .fastpath import dense_mlp, fused_layer_supported

load_ops()
_use_ca_fused = True


class CABuffers:
    """dip_ca.py:58-73.  Staging for streamed misses; unused with resident
    weights (attributes kept as empty tensors)."""

    def __init__(self, k, up_in_packed, up_ngroups, down_out, down_ngroups, device):
        self.device = torch.device(device)
        self.gpu_up_qw = torch.empty(0, up_in_packed, dtype=torch.int8, device=device)
        self.gpu_up_sc = torch.empty(0, up_ngroups, dtype=torch.bfloat16, device=device)
        self.gpu_dn_qw = torch.empty(0, down_out // 2, dtype=torch.int8, device=device)
        self.gpu_dn_sc = torch.empty(0, down_ngroups, dtype=torch.bfloat16, device=device)
        self.pin_up_qw = self.pin_up_sc = self.pin_dn_qw = self.pin_dn_sc = None
        self.copy_stream = None


class CADIPMlp(nn.Module):
    """dip_ca.py:76-196 with HBM-resident cache and full weights."""

    def __init__(self, gate_qw, gate_sc, up_qw, up_sc, down_qw, down_sc,
                 buf, keep_ratio=0.6, cache_frac=0.3, device="cuda:0"):
        super().__init__()
        self.device = torch.device(device)
        self.keep_ratio = keep_ratio
        self.buf = buf
        self.gate_qw = gate_qw.to(device).contiguous()
        self.gate_sc = gate_sc.to(device).contiguous()
        self.up_qw = up_qw.to(device).contiguous()
        self.up_sc = up_sc.to(device).contiguous()
        self.inter = up_qw.shape[0]
        dn_t_qw, dn_t_sc = _transpose_down_to_int4(down_qw.to(device), down_sc.to(device))
        self.down_t_qw = dn_t_qw.contiguous()
        self.down_t_sc = dn_t_sc.contiguous()
        self.out_features = dn_t_qw.shape[1] * 2
        self.k = int(round(self.inter * keep_ratio))
        self.cache_n = int(round(self.inter * cache_frac))
        self.register_buffer("cache_ids", torch.empty(0, dtype=torch.long, device=device),
                             persistent=False)
        self.register_buffer("id2slot", torch.full((self.inter,), -1, dtype=torch.long,
                                                   device=device), persistent=False)
        self._res_up_qw = None
        self._res_up_sc = None
        self._res_dn_qw = None
        self._res_dn_sc = None
        self.last_g = None
        self.last_idx = None
        self._last_split = None
        self._fused = fused_layer_supported(self.out_features, self.inter, self.device)
        self._ws = None  # fused decode workspace, zeroed once, left reusable

    @property
    def last_split(self):
        """(combined_ids, src, row, n_hit) of the last decode token: hits then
        misses, each in idx order (dip_ca.py:137-142, 164-171)."""
        if self._last_split is None and self.last_idx is not None:
            self._last_split = torch.ops.dip_b200.ca_split(self.last_idx, self.id2slot)
        return self._last_split

    @last_split.setter
    def last_split(self, v):
        self._last_split = v

    def reset_workspace(self):
        """Zero the decode workspace again (after the device error word
        reported a bounded wait that ran out)."""
        if self._ws is not None:
            self._ws.zero_()

    def set_cache(self, hot_ids):
        """dip_ca.py:107-117: keep hot_ids[:cache_n] sorted ascending; id2slot[id]
        = its rank; copy those channels' up/down rows into the resident cache."""
        hot_ids = hot_ids.to(self.device)[: self.cache_n].sort().values
        self.cache_ids = hot_ids
        id2 = torch.full((self.inter,), -1, dtype=torch.long, device=self.device)
        id2[hot_ids] = torch.arange(len(hot_ids), device=self.device)
        self.id2slot = id2
        self._res_up_qw = self.up_qw[hot_ids].contiguous()
        self._res_up_sc = self.up_sc[hot_ids].contiguous()
        self._res_dn_qw = self.down_t_qw[hot_ids].contiguous()
        self._res_dn_sc = self.down_t_sc[hot_ids].contiguous()

    def _gate(self, x):
        """dip_ca.py:119-125."""
        if x.dim() == 3 and x.shape[1] == 1 and x.shape[0] == 1:
            out = gate_gemv(self.gate_qw, self.gate_sc, x.reshape(-1))
            return out.reshape(x.shape[0], 1, -1)
        w = dequantize(self.gate_qw, self.gate_sc).to(x.dtype)
        return F.linear(x, w)

    def decode_token(self, xf: torch.Tensor):
        """One token: returns (y, g, idx, (combined_ids, src, row, n_hit)); the
        split is None on the one-launch path (computed on demand)."""
        xf = xf.reshape(-1).to(torch.bfloat16)
        if self._fused:
            if self._ws is None:
                nb = torch.ops.dip_b200.mlp_fused_workspace_bytes(self.out_features, self.inter,
                                                                  self.k)
                self._ws = torch.zeros(nb, dtype=torch.uint8, device=self.device)
            y, g, idx = torch.ops.dip_b200.mlp_decode_fused_ca(
                self.gate_qw, self.gate_sc, self.up_qw, self.up_sc, self.down_t_qw,
                self.down_t_sc, self.id2slot, self._res_up_qw, self._res_up_sc, self._res_dn_qw,
                self._res_dn_sc, xf, None, 1e-6, self.k, self._ws)
            return y, g, idx, None
        g = gate_silu(self.gate_qw, self.gate_sc, xf)
        idx = torch.ops.topk_ops.topk_select(g, self.k)
        comb, src, row, n_hit = torch.ops.dip_b200.ca_split(idx, self.id2slot)
        h = torch.ops.dip_b200.srcrow_up_h(self._res_up_qw, self._res_up_sc, self.up_qw,
                                           self.up_sc, xf, g, comb, src, row)
        y = torch.ops.dip_b200.srcrow_down(self._res_dn_qw, self._res_dn_sc, self.down_t_qw,
                                           self.down_t_sc, h, src, row)
        return y, g, idx, (comb, src, row, n_hit)

    def forward(self, x):
        if (x.dim() != 3 or x.shape[1] != 1 or self.keep_ratio >= 0.999
                or self._res_up_qw is None):
            return self._dense(x)
        _require_cuda(x)
        ys = []
        for b in range(x.shape[0]):
            y, g, idx, split = self.decode_token(x[b, 0])
            ys.append(y)
        self.last_g, self.last_idx, self.last_split = g, idx, split
        return torch.stack(ys).to(x.dtype).reshape(x.shape[0], 1, -1)

    def _dense(self, x):
        """dip_ca.py:190-196, the GEMMs on the tensor cores where the shapes
        allow (dequantize + F.linear otherwise)."""
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


def _hot_order(cnt: torch.Tensor, inter: int) -> torch.Tensor:
    """dip_ca.py:302-308: total order by (frequency desc, channel id asc)."""
    key = cnt.to(torch.long) * inter - torch.arange(inter, dtype=torch.long, device=cnt.device)
    return key.argsort(descending=True)


def calibrate_cache(model, tok, cas, prompt, calib_tokens=30):
    """dip_ca.py:272-309: count each layer's selected channels over a short
    greedy generation (forward hooks on the CA modules, which run _dense
    while no cache is set), then load each layer's hot set."""
    counts = [torch.zeros(c.inter, dtype=torch.long, device=c.device) for c in cas]
    handles = []

    def mk(lid, c):
        def hook(module, inp, out):
            x = inp[0]
            if x.dim() == 3 and x.shape[1] == 1:
                for b in range(x.shape[0]):
                    g = gate_silu(c.gate_qw, c.gate_sc, x[b, 0])
                    idx = select_topk(g, c.k)
                    counts[lid].index_add_(0, idx, torch.ones_like(idx))
        return hook

    for lid, c in enumerate(cas):
        handles.append(c.register_forward_hook(mk(lid, c)))
    ids = tok.apply_chat_template([{"role": "user", "content": prompt}],
                                  add_generation_prompt=True, return_tensors="pt")
    if not torch.is_tensor(ids):
        ids = ids["input_ids"]
    ids = ids.to(cas[0].device)
    with torch.no_grad():
        model.generate(ids, max_new_tokens=calib_tokens, do_sample=False, use_cache=True,
                       pad_token_id=tok.eos_token_id)
    for h in handles:
        h.remove()
    for lid, c in enumerate(cas):
        c.set_cache(_hot_order(counts[lid], c.inter))
    return counts


def calibrate_cache_inputs(cas, inputs):
    """Calibration without a language model: `inputs[lid]` is a [T, hidden]
    tensor of decode inputs for layer lid.  Counts each token's selection
    (gate + SiLU + top-k, as the reference hook does) and loads the hot set.
    Returns the per-layer counts."""
    counts = []
    for lid, c in enumerate(cas):
        cnt = torch.zeros(c.inter, dtype=torch.long, device=c.device)
        xs = inputs[lid].to(c.device)
        for t in range(xs.shape[0]):
            g = gate_silu(c.gate_qw, c.gate_sc, xs[t])
            idx = select_topk(g, c.k)
            cnt.index_add_(0, idx, torch.ones_like(idx))
        c.set_cache(_hot_order(cnt, c.inter))
        counts.append(cnt)
    return counts
