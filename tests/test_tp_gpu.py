"""Tensor parallelism on 2 GPUs (config 4 at one layer), with the exchanges
through NCCL and through the library's peer-memory exchange: the sharded
layer selects exactly the single-GPU channels and its y agrees with the
single-GPU y up to summation order; three tokens in a row, so the p2p
mailboxes are reused.  Skipped on boxes with fewer than 2 GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, comm):
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(repo / "dynamic-input-pruning_b200")]
    import torch.distributed as dist
    import dip_b200  # noqa: F401
    from dip_b200.stack import StackConfig, make_layer
    from dip_b200.tp import P2PExchange, TPDipMlp, shard_layer
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        cfg = StackConfig(n_layers=1, seed=3)
        L = make_layer(cfg, 0, dev)
        p2p = P2PExchange(cfg.inter, cfg.hidden, dev) if comm == "p2p" else None
        m = TPDipMlp(shard_layer(L, rank, world), cfg.k, p2p=p2p)
        res = []
        for t in range(3):
            x = torch.randn(cfg.hidden, generator=torch.Generator().manual_seed(4 + t))
            x = x.to(torch.bfloat16).to(dev)
            y = m.decode_token(x)
            y2, g2, idx2 = torch.ops.dip_b200.mlp_decode(L["gate_qw"], L["gate_sc"], L["up_qw"],
                                                         L["up_sc"], L["down_t_qw"],
                                                         L["down_t_sc"], x, cfg.k)
            torch.cuda.synchronize()
            same_idx = torch.equal(m.last_idx, idx2)
            err = (y.float() - y2.float()).abs().max().item()
            tol = 1e-2 * y2.float().abs().max().item() + 2e-3
            res.append((same_idx, err, tol))
        q.put((rank, res, torch.ops.dip_b200.take_device_error()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("comm", ["nccl", "p2p"])
def test_tp_two_gpus_matches_single(comm):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q, comm)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in ps]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, tokens, dev_err in res:
        assert dev_err == 0, f"rank {rank}: device error word {dev_err}"
        for t, (same_idx, err, tol) in enumerate(tokens):
            assert same_idx, f"rank {rank}, token {t}: indices differ from one GPU"
            assert err <= tol, f"rank {rank}, token {t}: max err {err:.3e} > {tol:.3e}"
