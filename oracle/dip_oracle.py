"""CPU oracle for the decode-time DIP SwiGLU MLP path — TEST INFRASTRUCTURE ONLY.

This module restates, on the CPU, the reference's algorithm for the path
(rohitpotluri/dynamic-input-pruning).  It is the checker for the CUDA kernels
and the timed CPU baseline; nothing in the product imports it.  Each function
names the reference file:line it follows.

Parity pins: the weight-format functions are checked bit for bit against
golden vectors produced by the reference's own Python code
(tests/golden/make_golden.py); the top-k restatement is checked against the
reference CUDA kernel compiled from its own source (oracle/Makefile,
tests/test_ref_kernels_gpu.py) and against committed vectors produced by it.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

GROUP_SIZE = 128  # qlinear.py:23, scripts/quantize.py:25
QMAX = 7          # scripts/quantize.py:26


# --------------------------------------------------------------------------
# Weight format
# --------------------------------------------------------------------------
def quantize_int4_g128(w: torch.Tensor):
    """scripts/quantize.py:32-64: symmetric int4, group 128 along columns,
    s = max|w_g| / 7 clamped >= 1e-8, q = clamp(round(w/s), -8, 7), two
    nibbles per byte with the even column in the low nibble, bf16 scales."""
    out_f, in_f = w.shape
    assert in_f % GROUP_SIZE == 0
    wg = w.float().reshape(out_f, in_f // GROUP_SIZE, GROUP_SIZE)
    s = (wg.abs().amax(dim=2, keepdim=True) / QMAX).clamp(min=1e-8)
    q = torch.round(wg / s).clamp(-8, 7).to(torch.int8).reshape(out_f, in_f)
    return pack_int4(q), s.squeeze(-1).to(torch.bfloat16)


def pack_int4(q: torch.Tensor) -> torch.Tensor:
    """dip_stream_predispatch.py:92-97 (_pack_int4_rows)."""
    lo = (q[:, 0::2] & 0x0F).to(torch.uint8)
    hi = (q[:, 1::2] & 0x0F).to(torch.uint8)
    return (lo | (hi << 4)).to(torch.int8)


def unpack_int4(qweight: torch.Tensor) -> torch.Tensor:
    """qlinear.py:28-49: int8 [R, C/2] -> int8 [R, C], values in [-8, 7]."""
    q = qweight.to(torch.uint8)
    lo = (q & 0x0F).to(torch.int16)
    hi = ((q >> 4) & 0x0F).to(torch.int16)
    lo = torch.where(lo >= 8, lo - 16, lo)
    hi = torch.where(hi >= 8, hi - 16, hi)
    out = torch.empty(q.shape[0], q.shape[1] * 2, dtype=torch.int8)
    out[:, 0::2] = lo.to(torch.int8)
    out[:, 1::2] = hi.to(torch.int8)
    return out


def dequantize(qweight: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """qlinear.py:52-64: bf16(q * s) with the product in fp32."""
    q = unpack_int4(qweight)
    r, c = q.shape
    w = q.float().reshape(r, c // GROUP_SIZE, GROUP_SIZE) * scales.float().reshape(r, -1, 1)
    return w.reshape(r, c).to(torch.bfloat16)


def transpose_down_to_int4(down_qw: torch.Tensor, down_sc: torch.Tensor):
    """dip_stream_predispatch.py:100-120: dequantize -> transpose -> requantise
    g128 along the new last dimension (hidden)."""
    wt = dequantize(down_qw, down_sc).t().contiguous()
    return quantize_int4_g128(wt)


# --------------------------------------------------------------------------
# Kernel semantics
# --------------------------------------------------------------------------
def int4_gemv_f32(qweight: torch.Tensor, scales: torch.Tensor, x: torch.Tensor,
                  rows=None) -> torch.Tensor:
    """kernels/int4_gemv/int4_gemv.cu:39-87 (and the gather variants,
    int4_gather_gemv.cu:39-85, ca_fused_gemv.cu:44-85): sum_c (q*s)*x with an
    fp32-or-better accumulation, returned in fp32 before the bf16 rounding.
    `rows` selects (gathers) rows first.  Computed in float64 in chunks."""
    if rows is not None:
        rows = torch.as_tensor(rows, dtype=torch.long)
        qweight, scales = qweight[rows], scales[rows]
    xd = x.reshape(-1).double()
    out = torch.empty(qweight.shape[0], dtype=torch.float64)
    step = 2048
    for r0 in range(0, qweight.shape[0], step):
        q = unpack_int4(qweight[r0:r0 + step]).double()
        n = q.shape[0]
        s = scales[r0:r0 + step].double().repeat_interleave(GROUP_SIZE, dim=1)
        out[r0:r0 + n] = (q * s) @ xd
    return out.float()


def int4_gemv(qweight, scales, x, rows=None) -> torch.Tensor:
    """Kernel output: bf16 round-to-nearest of the fp32 sum (int4_gemv.cu:85)."""
    return int4_gemv_f32(qweight, scales, x, rows).to(torch.bfloat16)


def silu_bf16(v: torch.Tensor) -> torch.Tensor:
    """dip_stream_predispatch.py:182: F.silu on the bf16 gate output."""
    return F.silu(v.to(torch.bfloat16))


def topk_select(s: torch.Tensor, k: int) -> torch.Tensor:
    """kernels/topk_select/topk_select.cu:134-164, literally: fp32 max of |s|,
    25 bisection steps `cnt > k -> lo = t else hi = t` (each count taken over
    every element, :46-57 / :148-156), then tier A = |s| > hi in ascending
    index (:74-98) and tier B = lo < |s| <= hi in ascending index (:101-131),
    truncated to k, remaining slots 0 (:160).  Returns int32 [k]."""
    a = np.abs(s.float().numpy().astype(np.float32)).reshape(-1)
    valid = ~np.isnan(a)
    hi = np.float32(a[valid].max()) if valid.any() else np.float32(0.0)
    hi = max(np.float32(0.0), hi)
    lo = np.float32(0.0)
    half = np.float32(0.5)
    t = np.float32(half * np.float32(lo + hi))
    for _ in range(25):
        cnt = int(np.count_nonzero(a > t))
        if cnt > k:
            lo = t
        else:
            hi = t
        t = np.float32(half * np.float32(lo + hi))
    tier_a = np.nonzero(a > hi)[0]
    tier_b = np.nonzero((a > lo) & (a <= hi))[0]
    sel = np.concatenate([tier_a, tier_b])[:k]
    out = np.zeros(k, dtype=np.int32)
    out[: len(sel)] = sel
    return torch.from_numpy(out)


def topk_lexicographic(s: torch.Tensor, k: int) -> torch.Tensor:
    """The set the bisection selects in the non-degenerate case: the k largest
    |s| with ties broken by lowest index, emitted strict tier then tie tier,
    each ascending.  Used to state the semantics in tests."""
    a = s.float().abs().reshape(-1).numpy()
    order = np.lexsort((np.arange(a.size), -a))[:k]
    kth = a[order[-1]]
    strict = np.sort(order[a[order] > kth])
    ties = np.sort(order[a[order] == kth])
    return torch.from_numpy(np.concatenate([strict, ties]).astype(np.int32))


def gather_down_f32(down_t_qw, down_t_sc, h: torch.Tensor, rows=None) -> torch.Tensor:
    """kernels/int4_down/int4_gather_down.cu:41-75: y[o] = sum_j h[j] *
    q(down_t[r_j, o]) * s(down_t[r_j, o/128]); float64 accumulation here."""
    if rows is not None:
        rows = torch.as_tensor(rows, dtype=torch.long)
        down_t_qw, down_t_sc = down_t_qw[rows], down_t_sc[rows]
    hd = h.reshape(-1).double()
    y = torch.zeros(down_t_qw.shape[1] * 2, dtype=torch.float64)
    step = 2048
    for r0 in range(0, down_t_qw.shape[0], step):
        q = unpack_int4(down_t_qw[r0:r0 + step]).double()
        s = down_t_sc[r0:r0 + step].double().repeat_interleave(GROUP_SIZE, dim=1)
        y += hd[r0:r0 + q.shape[0]] @ (q * s)
    return y.float()


# --------------------------------------------------------------------------
# Module forwards
# --------------------------------------------------------------------------
def dip_mlp_decode(x, gate_qw, gate_sc, up_qw, up_sc, down_t_qw, down_t_sc, k):
    """StreamingDIPMlp.forward (dip_stream_predispatch.py:176-204) for one
    decode token, with the kernels' rounding points:
      g = bf16(silu(bf16(gate x)))                         :182
      idx = topk_select(g, k)                              :184
      u = bf16(W_up[idx] x)                                :199-200
      h = bf16(g[idx] * u)                                 :201
      y = bf16(sum_j h_j W_down_t[idx_j])                  :202-203
    Returns a dict of all intermediates (CPU tensors)."""
    g = silu_bf16(int4_gemv(gate_qw, gate_sc, x))
    idx = topk_select(g, k)
    u = int4_gemv(up_qw, up_sc, x, rows=idx.long())
    h = (g[idx.long()].float() * u.float()).to(torch.bfloat16)
    y_f32 = gather_down_f32(down_t_qw, down_t_sc, h, rows=idx.long())
    return {"g": g, "idx": idx, "u": u, "h": h, "y_f32": y_f32, "y": y_f32.to(torch.bfloat16)}


def ca_split(idx: torch.Tensor, id2slot: torch.Tensor):
    """dip_ca.py:137-142 and :164-171: hits (slot >= 0) in idx order, then
    misses in idx order.  Returns (combined_ids, src, row, n_hit) with
    src 0 = resident cache (row = slot), 1 = full weights (row = channel)."""
    idx = idx.long()
    slots = id2slot[idx]
    hit = slots >= 0
    hit_ids, miss_ids = idx[hit], idx[~hit]
    combined = torch.cat([hit_ids, miss_ids])
    src = torch.cat([torch.zeros(hit_ids.numel(), dtype=torch.int32),
                     torch.ones(miss_ids.numel(), dtype=torch.int32)])
    row = torch.cat([slots[hit].to(torch.int32), miss_ids.to(torch.int32)])
    return combined.to(torch.int32), src, row, int(hit_ids.numel())


def cache_hot_order(counts: torch.Tensor) -> torch.Tensor:
    """dip_ca.py:306-308: order channels by key = count*I - id, descending
    (frequency descending, then channel id ascending)."""
    inter = counts.numel()
    key = counts.to(torch.long) * inter - torch.arange(inter, dtype=torch.long)
    return key.argsort(descending=True)


def set_cache_ids(hot_ids: torch.Tensor, cache_n: int, inter: int):
    """dip_ca.py:107-117: keep hot_ids[:cache_n], sorted ascending; id2slot
    maps a cached id to its rank, -1 elsewhere."""
    ids = hot_ids[:cache_n].sort().values
    id2slot = torch.full((inter,), -1, dtype=torch.long)
    id2slot[ids] = torch.arange(len(ids))
    return ids, id2slot


def ca_mlp_decode(x, gate_qw, gate_sc, up_qw, up_sc, down_t_qw, down_t_sc, k, id2slot):
    """CADIPMlp.forward (dip_ca.py:127-188): same g and idx as the streaming
    path; up and down run over combined = [hits, misses]."""
    g = silu_bf16(int4_gemv(gate_qw, gate_sc, x))
    idx = topk_select(g, k)
    combined, src, row, n_hit = ca_split(idx, id2slot)
    cl = combined.long()
    u = int4_gemv(up_qw, up_sc, x, rows=cl)
    h = (g[cl].float() * u.float()).to(torch.bfloat16)
    y_f32 = gather_down_f32(down_t_qw, down_t_sc, h, rows=cl)
    return {"g": g, "idx": idx, "combined": combined, "src": src, "row": row, "n_hit": n_hit,
            "h": h, "y_f32": y_f32, "y": y_f32.to(torch.bfloat16)}


# --------------------------------------------------------------------------
# The reference's own CPU math, as it runs (timed CPU baseline)
# --------------------------------------------------------------------------
def reference_cpu_layer(x, gate_qw, gate_sc, up_qw, up_sc, down_t_qw, down_t_sc, k):
    """One DIP layer the way the reference computes it with torch on the CPU:
    dequantize per call (qlinear.py:86-88), F.linear in bf16, F.silu, the
    top-k of topk_select.cu, index_select of the selected up / down_t rows,
    dequantize, then the products (dip_stream_predispatch.py:176-215)."""
    xb = x.reshape(1, -1).to(torch.bfloat16)
    g = F.silu(F.linear(xb, dequantize(gate_qw, gate_sc))).reshape(-1)
    idx = topk_select(g, k).long()
    up_w = dequantize(torch.index_select(up_qw, 0, idx), torch.index_select(up_sc, 0, idx))
    u = F.linear(xb, up_w).reshape(-1)
    h = (g[idx] * u).to(torch.bfloat16)
    dn = dequantize(torch.index_select(down_t_qw, 0, idx), torch.index_select(down_t_sc, 0, idx))
    return (h.reshape(1, -1) @ dn).reshape(-1)


# --------------------------------------------------------------------------
# Synthetic inputs
# --------------------------------------------------------------------------
def make_layer_cpu(hidden: int, inter: int, seed: int, std: float = 0.02,
                   gate_row_scale: torch.Tensor | None = None):
    """A config-0-style layer on the CPU: bf16 N(0, std) weights quantised as
    in scripts/quantize.py, down transposed as in _transpose_down_to_int4."""
    gen = torch.Generator().manual_seed(seed)
    wg = (torch.randn(inter, hidden, generator=gen) * std)
    if gate_row_scale is not None:
        wg = wg * gate_row_scale.reshape(-1, 1)
    wg = wg.to(torch.bfloat16)
    wu = (torch.randn(inter, hidden, generator=gen) * std).to(torch.bfloat16)
    wd = (torch.randn(hidden, inter, generator=gen) * std).to(torch.bfloat16)
    gq, gs = quantize_int4_g128(wg)
    uq, us = quantize_int4_g128(wu)
    dq, ds = quantize_int4_g128(wd)
    dtq, dts = transpose_down_to_int4(dq, ds)
    return {"gate_qw": gq, "gate_sc": gs, "up_qw": uq, "up_sc": us, "down_qw": dq,
            "down_sc": ds, "down_t_qw": dtq, "down_t_sc": dts}
