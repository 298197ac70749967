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
all-reduce of H fp32 values, either through NCCL (comm="nccl") or through
this library's peer-memory exchange (comm="p2p", `P2PExchange`: every rank
stores its slice into every rank's mailbox over NVLink and publishes a flag;
the partials are summed in rank order, identically on every rank).  Exchanging g itself (2 bytes per channel)
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


class _DeviceView:
    """Raw device memory owned elsewhere, seen by torch through
    __cuda_array_interface__."""

    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class P2PExchange:
    """The layer's two exchanges over peer memory (csrc/p2p.cu): one mailbox
    per rank (full g buffer + P partial slots + flags), mapped by every peer
    through CUDA IPC.  Built once per process group and shared by all layers
    (every rank makes the same sequence of calls)."""

    def __init__(self, inter: int, hidden: int, device, group=None):
        import ctypes
        from ._lib import core
        self.lib = lib = core()
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.inter, self.hidden = inter, hidden
        self.device = torch.device(device)
        vp, i64 = ctypes.c_void_p, ctypes.c_int64
        lib.dip_p2p_mailbox_bytes.restype = ctypes.c_size_t
        lib.dip_p2p_mailbox_bytes.argtypes = [i64, i64, i64]
        lib.dip_p2p_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(vp)]
        lib.dip_ipc_handle.argtypes = [vp, ctypes.c_char_p]
        lib.dip_ipc_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(vp)]
        lib.dip_p2p_gather.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.POINTER(vp), vp, i64,
                                       i64, vp]
        lib.dip_p2p_reduce.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.POINTER(vp), vp, i64,
                                       i64, vp, vp]
        with torch.cuda.device(self.device):
            mine = vp()
            nbytes = lib.dip_p2p_mailbox_bytes(inter, hidden, self.world)
            self._check(lib.dip_p2p_alloc(nbytes, ctypes.byref(mine)), "dip_p2p_alloc")
            handle = ctypes.create_string_buffer(64)
            self._check(lib.dip_ipc_handle(mine, handle), "dip_ipc_handle")
            handles = [None] * self.world
            dist.all_gather_object(handles, handle.raw, group=group)
            ptrs = []
            for q, hq in enumerate(handles):
                if q == self.rank:
                    ptrs.append(mine.value)
                    continue
                pq = vp()
                self._check(lib.dip_ipc_open(ctypes.create_string_buffer(hq, 64), ctypes.byref(pq)),
                            "dip_ipc_open")
                ptrs.append(pq.value)
        self.mailboxes = (vp * self.world)(*ptrs)
        # the gathered g lives in this rank's mailbox at byte offset 512
        self.g_all = torch.as_tensor(_DeviceView(mine.value + 512, inter, "<i2"),
                                     device=self.device).view(torch.bfloat16)
        dist.barrier(group=group)

    @staticmethod
    def _check(st, what):
        if st != 0:
            raise RuntimeError(f"{what} failed with status {st}")

    def gather(self, g_local: torch.Tensor) -> torch.Tensor:
        st = torch.cuda.current_stream(self.device).cuda_stream
        self._check(self.lib.dip_p2p_gather(self.rank, self.world, self.mailboxes, g_local.data_ptr(),
                                            g_local.numel(), self.hidden, st), "dip_p2p_gather")
        return self.g_all

    def reduce(self, partial: torch.Tensor) -> torch.Tensor:
        y = torch.empty(self.hidden, dtype=torch.bfloat16, device=self.device)
        st = torch.cuda.current_stream(self.device).cuda_stream
        self._check(self.lib.dip_p2p_reduce(self.rank, self.world, self.mailboxes, partial.data_ptr(),
                                            self.inter, self.hidden, y.data_ptr(), st),
                    "dip_p2p_reduce")
        return y


class TPDipMlp:
    """One DIP MLP layer sharded along I over a process group; the exchanges
    through NCCL, or through `P2PExchange` when one is given."""

    def __init__(self, shard: dict, k: int, group=None, ops=None, p2p: "P2PExchange | None" = None):
        self.s = shard
        self.k = k
        self.group = group
        self.ops = ops if ops is not None else CudaOps()
        self.world = dist.get_world_size(group)
        self.p2p = p2p
        self.last_idx = None

    def decode_token(self, x: torch.Tensor) -> torch.Tensor:
        s, ops = self.s, self.ops
        g_local = ops.gate_silu(s["gate_qw"], s["gate_sc"], x)
        if self.p2p is not None:
            g = self.p2p.gather(g_local)
        else:
            g = torch.empty(s["inter"], dtype=g_local.dtype, device=g_local.device)
            dist.all_gather_into_tensor(g, g_local, group=self.group)
        idx = ops.topk(g, self.k)
        local, count = ops.shard_select(idx, s["lo"], s["hi"])
        h = ops.up_h(s["up_qw"], s["up_sc"], x, g_local, local, count)
        y = ops.down_partial(s["down_t_qw"], s["down_t_sc"], h, local, count)
        self.last_idx = idx
        if self.p2p is not None:
            return self.p2p.reduce(y)
        dist.all_reduce(y, op=dist.ReduceOp.SUM, group=self.group)
        return y.to(torch.bfloat16)


class TPDipStack:
    """Config 4: the synthetic 64-layer stack (dip_b200.stack) with every layer
    sharded along I over the process group.  Each rank generates a layer's full
    weights from the same seed, keeps its shard and frees the rest.  The
    inter-layer step (RMSNorm(y + r)) runs replicated on every rank on the
    all-reduced y, so all ranks see identical inputs."""

    def __init__(self, cfg, device, group=None, comm: str = "p2p"):
        from .stack import make_layer
        self.cfg = cfg
        self.device = torch.device(device)
        self.group = group
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        self.p2p = P2PExchange(cfg.inter, cfg.hidden, self.device, group) if comm == "p2p" else None
        self.mlps = []
        for l in range(cfg.n_layers):
            full = make_layer(cfg, l, self.device)
            self.mlps.append(TPDipMlp(shard_layer(full, rank, world), cfg.k, group, p2p=self.p2p))
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
