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

`TPFusedStack` is the fast form of the same sharded layer: ONE cooperative
kernel per layer and rank (dip_mlp_decode_fused_tp) in which the exchange is
part of the kernel.  Each rank's gate CTAs add their |g| keys to every rank's
selection histograms over NVLink, so every rank finds the same selection
without moving g; after the gathered down projection each CTA stores its
quads of the fp32 partial y into every rank's y slots and sums the slots in
rank order.  No all-gather of g and no separate all-reduce launch.
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


def _sm_count(device) -> int:
    return torch.cuda.get_device_properties(device).multi_processor_count


class TPFusedWorkspace:
    """The per-rank workspace of the tensor-parallel fused layer: allocated
    zeroed by the library (dip_p2p_alloc), its CUDA IPC handle shared through
    the process group and the peers' workspaces mapped over NVLink
    (dip_ipc_open).  `ptrs[q]` is rank q's workspace as this process maps it.
    One workspace serves every layer (the layers run one after another)."""

    def __init__(self, hidden: int, inter_total: int, k: int, device, group=None):
        import ctypes
        from ._lib import core
        self.lib = lib = core()
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.device = torch.device(device)
        vp = ctypes.c_void_p
        lib.dip_p2p_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(vp)]
        lib.dip_ipc_handle.argtypes = [vp, ctypes.c_char_p]
        lib.dip_ipc_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(vp)]
        lib.dip_ipc_close.argtypes = [vp]
        lib.dip_p2p_free.argtypes = [vp]
        self.nbytes = int(torch.ops.dip_b200.mlp_fused_tp_workspace_bytes(hidden, inter_total, k))
        with torch.cuda.device(self.device):
            mine = vp()
            P2PExchange._check(lib.dip_p2p_alloc(self.nbytes, ctypes.byref(mine)), "dip_p2p_alloc")
            handle = ctypes.create_string_buffer(64)
            P2PExchange._check(lib.dip_ipc_handle(mine, handle), "dip_ipc_handle")
            info = [None] * self.world
            dist.all_gather_object(info, (handle.raw, _sm_count(self.device), self.nbytes),
                                   group=group)
            if len({(n, b) for _, n, b in info}) != 1:
                raise RuntimeError(f"tensor-parallel ranks disagree on SM count / workspace size: "
                                   f"{[(n, b) for _, n, b in info]}")
            ptrs, self._opened = [], []
            for q, (hq, _, _) in enumerate(info):
                if q == self.rank:
                    ptrs.append(mine.value)
                    continue
                pq = vp()
                P2PExchange._check(lib.dip_ipc_open(ctypes.create_string_buffer(hq, 64),
                                                    ctypes.byref(pq)), "dip_ipc_open")
                ptrs.append(pq.value)
                self._opened.append(pq.value)
        self.ptrs = ptrs
        self._mine = mine.value
        self.view = torch.as_tensor(_DeviceView(mine.value, self.nbytes, "|u1"), device=self.device)
        dist.barrier(group=group)

    def zero_(self) -> None:
        """Clears this rank's workspace (needed after a device-side timeout;
        every rank must clear its own before the next call)."""
        self.view.zero_()


class TPFusedStack:
    """Config 4 on the one-launch TP layer: the synthetic 64-layer stack with
    every layer sharded along I over the process group (rank r keeps rows
    [r I/P, (r+1) I/P) of gate, up and down_t), one dip_mlp_decode_fused_tp
    launch per layer and rank.  The inter-layer step RMSNorm(y + r) is folded
    into the next layer's kernel, as in DipStack's fused mode; y is identical
    on every rank.  keep_full keeps each layer's unsharded weights too (the
    in-run check against one GPU)."""

    def __init__(self, cfg, device, group=None, keep_full: bool = False):
        from .stack import make_layer
        self.cfg = cfg
        self.device = torch.device(device)
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if cfg.inter % self.world:
            raise ValueError(f"intermediate size {cfg.inter} is not divisible by {self.world} ranks")
        self.ws = TPFusedWorkspace(cfg.hidden, cfg.inter, cfg.k, self.device, group)
        self.shards, self.full = [], [] if keep_full else None
        for l in range(cfg.n_layers):
            full = make_layer(cfg, l, self.device)
            self.shards.append(shard_layer(full, self.rank, self.world))
            if keep_full:
                self.full.append(full)
            del full
        torch.cuda.empty_cache()
        self._graph = None
        self._static_in = None
        self._static_out = None
        self.last_idx = None
        self.last_x = None

    def step(self, x0, resid, record=False):
        """x0 [H], resid [L, H] -> last y [H].  With record, also the per-layer
        inputs (as the kernels normalised them) and the full index lists
        (every rank's entries, summed over the group)."""
        from .stack import RMS_EPS
        cfg, ws = self.cfg, self.ws
        y = None
        idxs, xs = [], []
        for l, s in enumerate(self.shards):
            xin, r = (x0, None) if l == 0 else (y, resid[l])
            idx = xu = None
            if record:
                idx = torch.zeros(cfg.k, dtype=torch.int32, device=self.device)
                xu = torch.empty(cfg.hidden, dtype=torch.bfloat16, device=self.device)
            nxt = self.shards[(l + 1) % len(self.shards)]
            y, _ = torch.ops.dip_b200.mlp_decode_fused_tp(
                s["gate_qw"], s["gate_sc"], s["up_qw"], s["up_sc"], s["down_t_qw"],
                s["down_t_sc"], xin, r, RMS_EPS, cfg.k, cfg.inter, self.rank, self.world,
                ws.ptrs, ws.nbytes, idx, xu, None, nxt["gate_qw"], nxt["gate_sc"])
            if record:
                idxs.append(idx)
                xs.append(xu)
        if record:
            allidx = torch.stack(idxs)
            dist.all_reduce(allidx, op=dist.ReduceOp.SUM, group=self.group)
            self.last_idx = list(allidx)
            self.last_x = xs
        return y

    def capture(self):
        H, n = self.cfg.hidden, self.cfg.n_layers
        self._static_in = (torch.zeros(H, dtype=torch.bfloat16, device=self.device),
                           torch.zeros(n, H, dtype=torch.bfloat16, device=self.device))
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):
                self.step(*self._static_in)
        torch.cuda.current_stream(self.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._static_out = self.step(*self._static_in)
        self._graph = g

    def replay(self):
        self._graph.replay()
        return self._static_out

    def decode(self, x0: torch.Tensor, resid: torch.Tensor) -> torch.Tensor:
        """Public call (every rank): one token through every layer; host
        inputs are copied in, the result comes back to the host."""
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


class TPBatchedDipStack:
    """Config 4 at batch B: the batched stack (dip_b200.batch, tcgen05 path)
    with every layer sharded along I.  Per layer and rank:

      g_loc = GEMM(gate shard, x) with the full layer's K split   [B, I/P]
      g     = all-gather of g_loc (NCCL)                          [B, I]
      idx   = per-token top-k of |g| (the same on every rank)     [B, k]
      h_loc = GEMM(up shard, x), epilogue h * count of the rank's channels
      y_loc = fp32 down projection of h_loc                       [B, H]
      y     = bf16(all-reduce sum of y_loc) (NCCL)

    Every gate row is computed with the same K ranges as the unsharded GEMM,
    so g and the indices are bit-identical to one GPU's; y agrees up to the
    order of the fp32 sums.  keep_full keeps the unsharded weights (the
    in-run check)."""

    def __init__(self, cfg, batch: int, device, group=None, keep_full: bool = False):
        from .stack import make_layer
        self.cfg, self.batch = cfg, batch
        self.device = torch.device(device)
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.lo, self.hi = shard_range(cfg.inter, self.rank, self.world)
        self.ksplit = int(torch.ops.dip_b200.gemm_tc_auto_split(cfg.inter, cfg.hidden))
        self.shards, self.full = [], [] if keep_full else None
        for l in range(cfg.n_layers):
            full = make_layer(cfg, l, self.device)
            self.shards.append(shard_layer(full, self.rank, self.world))
            if keep_full:
                self.full.append(full)
            del full
        torch.cuda.empty_cache()
        self._graph = self._static_in = self._static_out = None
        self.last_idx = self.last_x = None

    def layer(self, s, x):
        B, I, P = x.shape[0], self.cfg.inter, self.world
        g_loc = torch.ops.dip_b200.gemm_tc(s["gate_qw"], s["gate_sc"], x, 1, None, None,
                                           self.ksplit)
        parts = torch.empty(P, B, I // P, dtype=g_loc.dtype, device=x.device)
        dist.all_gather_into_tensor(parts, g_loc.contiguous(), group=self.group)
        g = parts.permute(1, 0, 2).reshape(B, I)
        idx = torch.ops.dip_b200.topk_select_batched(g, self.cfg.k)
        cnt = torch.ops.dip_b200.select_count(idx, I)[:, self.lo:self.hi].contiguous()
        h = torch.ops.dip_b200.gemm_tc(s["up_qw"], s["up_sc"], x, 2, g_loc, cnt, self.ksplit)
        y = torch.ops.dip_b200.down_tc_f32(s["down_t_qw"], s["down_t_sc"], h)
        dist.all_reduce(y, op=dist.ReduceOp.SUM, group=self.group)
        return y.to(torch.bfloat16), idx

    def step(self, x0, resid, record=False):
        from .stack import RMS_EPS
        y, idxs, xs = None, [], []
        for l, s in enumerate(self.shards):
            x = x0 if l == 0 else torch.ops.dip_b200.residual_rmsnorm(y, resid[l], RMS_EPS)
            y, idx = self.layer(s, x)
            if record:
                idxs.append(idx)
                xs.append(x)
        if record:
            self.last_idx, self.last_x = idxs, xs
        return y

    def capture(self):
        B, H, n = self.batch, self.cfg.hidden, self.cfg.n_layers
        self._static_in = (torch.zeros(B, H, dtype=torch.bfloat16, device=self.device),
                           torch.zeros(n, B, H, dtype=torch.bfloat16, device=self.device))
        st = torch.cuda.Stream(device=self.device)
        st.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(st):
            for _ in range(2):
                self.step(*self._static_in)
        torch.cuda.current_stream(self.device).wait_stream(st)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            self._static_out = self.step(*self._static_in)
        self._graph = gr

    def replay(self):
        self._graph.replay()
        return self._static_out
