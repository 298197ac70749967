"""Tensor-parallel DIP MLP along the intermediate dimension.

The reference is single-GPU only.  Here rank r of P owns the contiguous
channel range [r*I/P, (r+1)*I/P) of gate, up and the transposed down.  Per
decode token:

  1. local gate GEMV + SiLU on the owned rows            -> g_local [I/P]
  2. all-gather of g (bf16, I*2 bytes in total)         -> g [I] on every rank
  3. the same exact top-k on every rank                  -> idx [k] (identical
     to the single-GPU selection, bit for bit: every row of g is computed by
     the same kernel with the same reduction order whatever the sharding)
  4. keep the selected channels this rank owns (device-side count, no sync)
  5. gathered up (h = g*u) and down over those rows      -> fp32 partial [H]
  6. all-reduce (sum) of the fp32 partials, bf16 cast    -> y [H]

Communication per token and layer: one all-gather of I bf16 values and one
all-reduce of H fp32 values.  Exchanging g itself (2 bytes per channel)
instead of (|g|, id) candidates is cheaper and, because k > I/P for every
P <= 8 at keep_ratio 0.6, a local pre-selection would prune nothing.

The compute backend is pluggable so the orchestration (sharding, collectives,
merge) can be exercised by CPU tests with a `gloo` group; the default backend
is the sm_100a kernels.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(inter: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous, equal shards; inter must divide by world."""
    if inter % world:
        raise ValueError(f"intermediate size {inter} is not divisible by {world} ranks")
    per = inter // world
    return rank * per, (rank + 1) * per


def shard_layer(layer: dict, rank: int, world: int) -> dict:
    """Rows [lo, hi) of gate, up and down_t of a full layer dict."""
    inter = layer["gate_qw"].shape[0]
    lo, hi = shard_range(inter, rank, world)
    out = {n: layer[n][lo:hi].contiguous() for n in
           ("gate_qw", "gate_sc", "up_qw", "up_sc", "down_t_qw", "down_t_sc")}
    out["lo"], out["hi"], out["inter"] = lo, hi, inter
    return out


class CudaOps:
    """The sm_100a kernels (default backend)."""

    def gate_silu(self, qw, sc, x):
        return torch.ops.dip_b200.gate_silu(qw, sc, x)

    def topk(self, g, k):
        return torch.ops.topk_ops.topk_select(g, k)

    def shard_select(self, idx, lo, hi):
        return torch.ops.dip_b200.shard_select(idx, lo, hi)

    def up_h(self, qw, sc, x, g_local, local_idx, count):
        return torch.ops.dip_b200.gather_up_h_count(qw, sc, x, g_local, local_idx, count)

    def down_partial(self, qw, sc, h, local_idx, count):
        return torch.ops.dip_b200.gather_down_partial(qw, sc, h, local_idx, count)


class TPDipMlp:
    """One DIP MLP layer sharded along I over a process group."""

    def __init__(self, shard: dict, k: int, group=None, ops=None):
        self.s = shard
        self.k = k
        self.group = group
        self.ops = ops if ops is not None else CudaOps()
        self.world = dist.get_world_size(group)
        self.last_idx = None

    def decode_token(self, x: torch.Tensor) -> torch.Tensor:
        s, ops = self.s, self.ops
        g_local = ops.gate_silu(s["gate_qw"], s["gate_sc"], x)
        g = torch.empty(s["inter"], dtype=g_local.dtype, device=g_local.device)
        dist.all_gather_into_tensor(g, g_local, group=self.group)
        idx = ops.topk(g, self.k)
        local, count = ops.shard_select(idx, s["lo"], s["hi"])
        h = ops.up_h(s["up_qw"], s["up_sc"], x, g_local, local, count)
        y = ops.down_partial(s["down_t_qw"], s["down_t_sc"], h, local, count)
        dist.all_reduce(y, op=dist.ReduceOp.SUM, group=self.group)
        self.last_idx = idx
        return y.to(torch.bfloat16)


class TPDipStack:
    """Config 4: the synthetic 64-layer stack (dip_b200.stack) with every layer
    sharded along I over the process group.  Each rank generates a layer's full
    weights from the same seed, keeps its shard and frees the rest.  The
    inter-layer step (RMSNorm(y + r)) runs replicated on every rank on the
    all-reduced y, so all ranks see identical inputs."""

    def __init__(self, cfg, device, group=None):
        from .stack import make_layer
        self.cfg = cfg
        self.device = torch.device(device)
        self.group = group
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        self.mlps = []
        for l in range(cfg.n_layers):
            full = make_layer(cfg, l, self.device)
            self.mlps.append(TPDipMlp(shard_layer(full, rank, world), cfg.k, group))
            del full
        torch.cuda.empty_cache()
        self._graph = None
        self._static_in = None
        self._static_out = None
        self.last_idx = None

    def step(self, x0, resid, record=False):
        from .stack import RMS_EPS
        y, idxs = None, []
        for l, m in enumerate(self.mlps):
            x = x0 if l == 0 else torch.ops.dip_b200.residual_rmsnorm(y, resid[l], RMS_EPS)
            y = m.decode_token(x)
            if record:
                idxs.append(m.last_idx)
        if record:
            self.last_idx = idxs
        return y

    def capture(self):
        H, n = self.cfg.hidden, self.cfg.n_layers
        self._static_in = (torch.zeros(H, dtype=torch.bfloat16, device=self.device),
                           torch.zeros(n, H, dtype=torch.bfloat16, device=self.device))
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):  # collectives and kernels initialised before capture
                self.step(*self._static_in)
        torch.cuda.current_stream(self.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._static_out = self.step(*self._static_in)
        self._graph = g

    def replay(self):
        self._graph.replay()
        return self._static_out
