"""Tensor-parallel orchestration on the CPU (gloo, world sizes 2 and 4).

The sm_100a kernels are replaced by the CPU oracle through TPDipMlp's
pluggable backend, so sharding, the all-gather of g, the replicated top-k,
the owned-channel selection and the partial all-reduce are exercised without
a GPU.  The selection must equal the single-device one bit for bit; y within
the path tolerance (summation order differs)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


class OracleOps:
    def __init__(self, O):
        self.O = O

    def gate_silu(self, qw, sc, x):
        return self.O.silu_bf16(self.O.int4_gemv(qw, sc, x))

    def topk(self, g, k):
        return self.O.topk_select(g, k)

    def shard_select(self, idx, lo, hi):
        own = idx[(idx >= lo) & (idx < hi)] - lo
        return own.to(torch.int32), torch.tensor([own.numel()], dtype=torch.int32)

    def up_h(self, qw, sc, x, g_local, local, count):
        n = int(count[0])
        rows = local[:n].long()
        u = self.O.int4_gemv(qw, sc, x, rows=rows)
        return (g_local[rows].float() * u.float()).to(torch.bfloat16)

    def down_partial(self, qw, sc, h, local, count):
        n = int(count[0])
        if n == 0:
            return torch.zeros(qw.shape[1] * 2)
        return self.O.gather_down_f32(qw, sc, h[:n], rows=local[:n].long())


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(repo), str(repo / "dynamic-input-pruning_b200")]
    from oracle import dip_oracle as O
    from dip_b200.tp import TPDipMlp, shard_layer
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        L = O.make_layer_cpu(512, 1024, seed=31)
        x = torch.randn(512, generator=torch.Generator().manual_seed(32)).to(torch.bfloat16)
        k = int(round(1024 * 0.6))
        tp = TPDipMlp(shard_layer(L, rank, world), k, ops=OracleOps(O))
        y = tp.decode_token(x)
        q.put((rank, y, tp.last_idx))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tp_matches_single_device(oracle, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    L = oracle.make_layer_cpu(512, 1024, seed=31)
    x = torch.randn(512, generator=torch.Generator().manual_seed(32)).to(torch.bfloat16)
    ref = oracle.dip_mlp_decode(x, L["gate_qw"], L["gate_sc"], L["up_qw"], L["up_sc"],
                                L["down_t_qw"], L["down_t_sc"], int(round(1024 * 0.6)))
    for _, y, idx in res:
        assert torch.equal(idx, ref["idx"])
        err = (y.float() - ref["y_f32"]).abs()
        assert bool((err <= 2e-3 + 1e-2 * ref["y_f32"].abs()).all())


def _dead_worker(rank, world, port, q):
    """Rank 1 leaves before the collective; rank 0 must get an error from the
    process-group timeout instead of hanging."""
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    # the timeout also bounds the rendezvous: generous enough for a loaded host
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=15))
    except Exception as e:
        q.put((rank, "init failed:" + type(e).__name__))
        return
    if rank == 1:
        q.put((rank, "left"))
        return  # exits without joining the all-gather
    try:
        t = torch.zeros(4)
        out = torch.empty(8)
        dist.all_gather_into_tensor(out, t)
        q.put((rank, "no error"))
    except Exception as e:  # timeout / connection closed
        q.put((rank, "error:" + type(e).__name__))


def test_tp_rank_failure_is_reported_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dead_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert res[1] == "left"
    assert res[0].startswith("error:")
