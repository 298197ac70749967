"""Batch tensor parallelism on 2 GPUs (config 4 at batch B, TPBatchedDipStack):
per-token indices bit-identical to the single-GPU batched layer on the full
weights (the gate shard uses the full layer's K split), y within the path
tolerance and identical on both ranks.  Skipped with fewer than 2 GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 2e-3


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import sys
    from pathlib import Path
    sys.path[:0] = [str(Path(__file__).resolve().parents[1] / "dynamic-input-pruning_b200")]
    import torch.distributed as dist
    import dip_b200  # noqa: F401
    from dip_b200.stack import StackConfig
    from dip_b200.batch import batched_dip_layer
    from dip_b200.tp import TPBatchedDipStack
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        cfg = StackConfig(n_layers=2, seed=4)
        B = 24
        st = TPBatchedDipStack(cfg, B, dev, keep_full=True)
        gen = torch.Generator().manual_seed(5)
        x0 = torch.randn(B, cfg.hidden, generator=gen).to(torch.bfloat16).to(dev)
        r = torch.randn(2, B, cfg.hidden, generator=gen).to(torch.bfloat16).to(dev)
        y = st.step(x0, r, record=True)
        res = []
        for l in range(2):
            y1, _, idx1 = batched_dip_layer(st.full[l], st.last_x[l], cfg.k, "tc")
            res.append(bool(torch.equal(idx1, st.last_idx[l])))
        # last layer's y against the single-GPU layer on the same input
        err = (y.float() - y1.float()).abs()
        ok = bool((err <= ATOL + RTOL * y1.float().abs()).all())
        y_all = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(y_all, y)
        same = all(torch.equal(v, y) for v in y_all)
        torch.cuda.synchronize()
        q.put((rank, res, ok, same, float(err.max()), torch.ops.dip_b200.take_device_error()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_batch_two_gpus_matches_single():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=600) for _ in ps]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, idx_ok, y_ok, same, err, dev_err in res:
        assert dev_err == 0
        assert all(idx_ok), f"rank {rank}: per-token indices differ from one GPU ({idx_ok})"
        assert y_ok, f"rank {rank}: y max err {err:.3e}"
        assert same, f"rank {rank}: y differs between ranks"
