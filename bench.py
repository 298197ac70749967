"""Benchmark: Qwen3-32B-shaped DIP decode MLP stack (BASELINE configs 1 and 4).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one decode token through the 64-layer int4 DIP MLP stack at batch 1
(hidden 5120, intermediate 25600, keep_ratio 0.6 -> k = 15360), inputs
resident in HBM, replayed from a CUDA graph.  Every step reads ~9.5 GB of
weights, far more than the 126 MB L2, so no L2 flush is needed.  Prints one
JSON line (rank 0).

One GPU: config 1, one layer_fused_kernel launch per layer.  Under torchrun
with N > 1 ranks: config 4, the same token stream with every layer sharded
along I over the N GPUs (one dip_mlp_decode_fused_tp launch per layer and
rank; strong scaling), checked in the run against one GPU's indices.
`--replicas` instead runs N independent single-GPU stacks.

--impl reference times the reference's own CPU math for the same layer
(dequantise per call, F.linear, SiLU, the topk_select.cu selection, row
gather, matmul) on the host cores; it never touches the GPU.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "dynamic-input-pruning_b200"))
sys.path.insert(0, str(REPO))

RMS_EPS_BENCH = 1e-6
METRIC = "dip_mlp_decode_tok_s"
UNIT = "tok/s"


def _peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _traffic():
    p = REPO / "profiles" / "ncu_traffic.json"
    if p.exists():
        return json.loads(p.read_text())
    return {}


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML during the timed region."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, index: int):
        self.samples, self.reasons, self.max_mhz = [], 0, None
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML unavailable: report nothing rather than guess
            self._nv = None
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self._nv.nvmlDeviceGetClockInfo(self._h,
                                                                    self._nv.NVML_CLOCK_SM))
                self.reasons |= self._nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            except Exception:
                pass
            time.sleep(0.005)

    def __enter__(self):
        if self._nv:
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._nv:
            self._t.join()

    def summary(self):
        if not self._nv:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml_unavailable"]}
        names = [n for b, n in self.REASONS.items() if self.reasons & b and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples)}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def cpu_reference_layer_time(n_layers_sample: int, seed: int = 0, layer=None):
    """Seconds per layer of the reference's CPU math (oracle port), using all
    host threads.  `layer` (CPU packed weights) may be given; else generated."""
    from oracle import dip_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    if layer is None:
        layer = O.make_layer_cpu(5120, 25600, seed=seed)
    gen = torch.Generator().manual_seed(seed + 1)
    xs = torch.randn(n_layers_sample + 1, 5120, generator=gen).to(torch.bfloat16)
    args = (layer["gate_qw"], layer["gate_sc"], layer["up_qw"], layer["up_sc"],
            layer["down_t_qw"], layer["down_t_sc"], 15360)
    O.reference_cpu_layer(xs[0], *args)  # warm-up
    t0 = time.perf_counter()
    for i in range(n_layers_sample):
        O.reference_cpu_layer(xs[i + 1], *args)
    return (time.perf_counter() - t0) / n_layers_sample, torch.get_num_threads()


def run_reference(args):
    """The reference's own math for this path (dequantise per call, F.linear,
    SiLU, the topk_select.cu selection, row gather, matmul) on the host cores,
    through the CPU port in oracle/ (the reference's CUDA kernels are sm_75
    code with host round trips; its CPU path is plain torch).  A step here is
    a bounded sample of 2 layers of the 64-layer token; the token rate is
    extrapolated as 1 / (64 x seconds per layer).  Under torchrun only rank 0
    runs; the CPU math does not shard over GPUs, so the same sample stands for
    every N."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    per_step_layers = 2
    from oracle import dip_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    layer = O.make_layer_cpu(5120, 25600, seed=0)
    for _ in range(max(0, min(args.warmup, 1))):
        cpu_reference_layer_time(1, layer=layer)
    n_layers = per_step_layers * args.steps
    sec, cores = cpu_reference_layer_time(n_layers, layer=layer)
    tok_s = 1.0 / (64 * sec)
    sample = (f"{n_layers} config-1 layers (hidden 5120, inter 25600, k 15360) of the "
              f"reference CPU math on {cores} threads; tok/s = 1/(64 x s/layer)")
    cfg = {"workload": ("config1: 64-layer Qwen3-32B-shape DIP decode MLP stack, batch 1"
                        if world == 1 else
                        f"config4: the config-1 stack sharded along I over {world} GPUs, batch 1"),
           "hidden": 5120, "inter": 25600, "k": 15360, "layers": 64, "keep_ratio": 0.6,
           "parallelism": "single" if world == 1 else f"tp{world}",
           "l2": "no flush: each step reads ~9.5 GB of weights (> 126 MB L2)"}
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": tok_s, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 64 * sec * 1e3,
        "higher_is_better": True, "scaling": "weak" if world == 1 else "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": cfg,
        "us_per_layer": sec * 1e6,
        "layers_timed": n_layers, "step_definition": f"{per_step_layers} layers per step",
        "extrapolated_to": "64 x s/layer per token (ms_per_step is that extrapolation)",
        "cpu_baseline": {"value": tok_s, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": tok_s, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_single_layer(n):
    """n launches of the fused kernel on one config-1 layer (a small, fixed case
    for ncu captures: ~0.2 GB on the device, one kernel per launch)."""
    import dip_b200  # noqa: F401
    from dip_b200.stack import StackConfig, make_layer
    dev = torch.device("cuda", 0)
    cfg = StackConfig(n_layers=1, seed=0)
    L = make_layer(cfg, 0, dev)
    ws = torch.zeros(torch.ops.dip_b200.mlp_fused_workspace_bytes(cfg.hidden, cfg.inter, cfg.k),
                     dtype=torch.uint8, device=dev)
    x = torch.randn(cfg.hidden, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    x = x.to(dev)
    for _ in range(n):
        y, _, _ = torch.ops.dip_b200.mlp_decode_fused(L["gate_qw"], L["gate_sc"], L["up_qw"],
                                                      L["up_sc"], L["down_t_qw"], L["down_t_sc"],
                                                      x, None, RMS_EPS_BENCH, cfg.k, ws)
    torch.cuda.synchronize()
    assert torch.ops.dip_b200.take_device_error() == 0
    print(json.dumps({"single_layer_launches": n, "y_abs_sum": float(y.float().abs().sum())}))


def run_gemm_tc(n):
    """n launches of the batch-64 gate GEMM (tcgen05, SiLU epilogue) on one
    config-1 layer: the small fixed case for ncu captures of gemm_tc_kernel."""
    import dip_b200  # noqa: F401
    from dip_b200.stack import StackConfig, make_layer
    dev = torch.device("cuda", 0)
    cfg = StackConfig(n_layers=1, seed=0)
    L = make_layer(cfg, 0, dev)
    x = torch.randn(64, cfg.hidden, generator=torch.Generator().manual_seed(1))
    x = x.to(torch.bfloat16).to(dev)
    for _ in range(n):
        g = torch.ops.dip_b200.gemm_tc(L["gate_qw"], L["gate_sc"], x, 1)
    torch.cuda.synchronize()
    assert torch.ops.dip_b200.take_device_error() == 0
    print(json.dumps({"gemm_tc_launches": n, "g_abs_sum": float(g.float().abs().sum())}))


def _module_forward_us(dev, reps=20):
    """Config 0 through the drop-in module: StreamingDIPMlp(...)(x) with x
    [1, 1, 5120], eager calls (Python, output allocation and the one fused
    launch each), CUDA events around `reps` calls after warm-up."""
    import dip_b200
    from dip_b200.stack import StackConfig, make_layer
    cfg = StackConfig(n_layers=1, seed=0)
    L = make_layer(cfg, 0, dev)
    # the module takes the untransposed down projection, as the reference does
    gen = torch.Generator(device=dev).manual_seed(7)
    wd = (torch.randn(cfg.hidden, cfg.inter, generator=gen, device=dev) * cfg.std)
    dq, ds = torch.ops.dip_b200.quantize_int4(wd.to(torch.bfloat16))
    del wd
    shared = dip_b200.SharedBuffers(cfg.k, cfg.hidden // 2, cfg.hidden // 128, cfg.hidden,
                                    cfg.hidden // 128, dev)
    m = dip_b200.StreamingDIPMlp(L["gate_qw"], L["gate_sc"], L["up_qw"], L["up_sc"], dq, ds,
                                 shared, cfg.keep_ratio, dev)
    x = torch.randn(1, 1, cfg.hidden, generator=torch.Generator().manual_seed(3))
    x = x.to(torch.bfloat16).to(dev)
    for _ in range(5):
        m(x)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        m(x)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / reps, bool(m._fused)


def _time_stack(stack, x0, resid, warmup, steps, dev):
    """Graph-replayed decode steps: warm-up, then `steps` timed with CUDA events."""
    stack.capture()
    xi, ri = stack._static_in
    for t in range(warmup):
        xi.copy_(x0[t]); ri.copy_(resid[t]); stack.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clk:
        e0.record()
        for t in range(warmup, warmup + steps):
            xi.copy_(x0[t]); ri.copy_(resid[t]); stack.replay()
        e1.record()
        torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps, clk.summary()


def run_config2(args, emit=True):
    """Config 2: cache-aware DIP on the 64-layer stack with LogNormal(0,1)
    gate-row scales; calibration on 32 N(0,1) tokens run through the DIP
    stack, cache_n = 0.3 I hot channels per layer.  Reports us/layer and
    tok/s of the one-launch CA layer (and of the separate-launch CA chain and
    the streaming fused layer on the same weights), the hit rate, and whether
    every recorded hit/miss split equals its definition (hits then misses,
    each in top-k order) recomputed with torch ops from the same indices."""
    import dip_b200  # noqa: F401
    from dip_b200.stack import StackConfig, DipStack, token_inputs
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = StackConfig(n_layers=args.layers, seed=0, gate_lognormal=True)
    stack = DipStack(cfg, dev, mode="ca")
    xc, rc = token_inputs(cfg, 32, seed=2000, device=dev)
    stack.calibrate_ca(xc, rc)
    T = args.warmup + args.steps
    x0, resid = token_inputs(cfg, T, seed=1000, device=dev)
    ms_ca, clk = _time_stack(stack, x0, resid, args.warmup, args.steps, dev)
    # hit rate and split exactness over recorded eager tokens
    hits, exact, n_tok = 0, True, min(8, args.steps)
    for t in range(n_tok):
        stack.step(x0[t], resid[t], record=True)
        for l, (idx, (comb, src, row, n_hit)) in enumerate(zip(stack.last_idx, stack.last_split)):
            id2 = stack.ca[l]["id2slot"]
            il = idx.long()
            hitm = id2[il] >= 0
            ref = torch.cat([il[hitm], il[~hitm]])
            nh = int(hitm.sum())
            ok = (torch.equal(comb.long(), ref) and int(n_hit) == nh and
                  torch.equal(src.long(), torch.cat([torch.zeros(nh, dtype=torch.long, device=dev),
                                                     torch.ones(il.numel() - nh, dtype=torch.long,
                                                                device=dev)])) and
                  torch.equal(row.long(), torch.cat([id2[il[hitm]], il[~hitm]])))
            exact = exact and ok
            hits += nh
    hit_rate = hits / (n_tok * cfg.n_layers * cfg.k)
    stack.mode, stack.fused, stack._graph = "ca_chain", False, None
    ms_chain, _ = _time_stack(stack, x0, resid, args.warmup, args.steps, dev)
    stack.mode, stack.fused, stack._graph = "fused", True, None
    ms_fused, _ = _time_stack(stack, x0, resid, args.warmup, args.steps, dev)
    us_ca = ms_ca * 1e3 / cfg.n_layers
    del stack
    rec = {
        "metric": "dip_ca_mlp_decode_tok_s", "value": 1e3 / ms_ca, "unit": "tok/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_ca,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) int4 g128 weights, gate rows x LogNormal(0,1), "
                "N(0,1) tokens)",
        "config": {"workload": "config2: cache-aware DIP, 64-layer stack, batch 1",
                   "layers": cfg.n_layers, "k": cfg.k, "cache_n": cfg.cache_n,
                   "calibration": "32 N(0,1) tokens through the DIP stack"},
        "us_per_layer": us_ca, "hit_rate": hit_rate, "split_exact": bool(exact),
        "split_checked_tokens": n_tok,
        "ca_separate_launches_us_per_layer": ms_chain * 1e3 / cfg.n_layers,
        "streaming_fused_us_per_layer_same_weights": ms_fused * 1e3 / cfg.n_layers,
        "gpu_launches": args.steps * cfg.n_layers,
        "clocks": clk}
    if emit:
        print(json.dumps(rec), flush=True)
    return rec


def run_tp(args):
    """Config 4: the stack sharded along I over the N ranks of torchrun: per
    layer one all-gather of g (bf16, I values) and one all-reduce of the fp32
    [H] partials, through the library's peer-memory exchange (`--comm p2p`,
    default) or NCCL (`--comm nccl`).  All N GPUs work on the same token:
    `value` is the token rate of that one stream (strong scaling).
    `comm_us_per_layer` times the same two exchanges alone (graph-replayed,
    64 per step); they run on the compute stream, so all of it is exposed."""
    rank, world, local = dist_env()
    import torch.distributed as dist
    import dip_b200  # noqa: F401
    from dip_b200.stack import StackConfig, token_inputs
    from dip_b200.tp import TPDipStack
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world == 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(_free_port()))
        os.environ.setdefault("RANK", "0")
        os.environ.setdefault("WORLD_SIZE", "1")
    dist.init_process_group("nccl", device_id=dev)
    cfg = StackConfig(n_layers=args.layers, seed=0)
    stack = TPDipStack(cfg, dev, comm=args.comm)
    T = args.warmup + args.steps
    x0, resid = token_inputs(cfg, T, seed=1000, device=dev)
    ms, clk = _time_stack(stack, x0, resid, args.warmup, args.steps, dev)
    tt = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms = tt.item()
    if _device_error_all(world, dev):
        raise SystemExit("a bounded device wait ran out during the timed steps: run invalid")
    # the collectives alone
    g_loc = torch.zeros(cfg.inter // world, dtype=torch.bfloat16, device=dev)
    g_all = torch.zeros(cfg.inter, dtype=torch.bfloat16, device=dev)
    part = torch.zeros(cfg.hidden, dtype=torch.float32, device=dev)

    def comm():
        for _ in range(cfg.n_layers):
            if world > 1 and stack.p2p is not None:
                stack.p2p.gather(g_loc)
                stack.p2p.reduce(part)
            elif world > 1:
                dist.all_gather_into_tensor(g_all, g_loc)
                dist.all_reduce(part)
    comm_us = 0.0
    if world > 1:
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            comm(); comm()
        torch.cuda.current_stream(dev).wait_stream(s)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            comm()
        for _ in range(3):
            gr.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            gr.replay()
        e1.record()
        torch.cuda.synchronize()
        ct = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev)
        dist.all_reduce(ct, op=dist.ReduceOp.MAX)
        comm_us = ct.item() * 1e3 / cfg.n_layers
        if _device_error_all(world, dev):
            raise SystemExit("a bounded device wait ran out in the exchange timing: run invalid")
    layer_us = ms * 1e3 / cfg.n_layers
    if rank == 0:
        print(json.dumps({
            "metric": "dip_mlp_decode_tok_s", "value": 1e3 / ms, "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,0.02) int4 g128 weights, N(0,1) tokens)",
            "config": {"workload": "config4: 64-layer stack sharded along I, batch 1",
                       "layers": cfg.n_layers, "k": cfg.k, "parallelism": f"tp{world}",
                       "comm": args.comm},
            "us_per_layer": layer_us, "comm_us_per_layer": comm_us,
            "comm_frac_of_layer": comm_us / layer_us if layer_us else None,
            "gpu_launches": args.steps * (cfg.n_layers * 5 + cfg.n_layers - 1),
            "clocks": clk}), flush=True)
    # Tearing the process group down after NCCL work was captured into CUDA
    # graphs can block; every rank is done, so leave directly.
    dist.barrier()
    torch.cuda.synchronize()
    sys.stdout.flush()
    os._exit(0)


def _free_port():
    import socket
    so = socket.socket()
    so.bind(("127.0.0.1", 0))
    port = so.getsockname()[1]
    so.close()
    return port


def run_config3(args, emit=True):
    """Config 3: B independent tokens per step through the 64-layer stack
    (per-token DIP selection; `--path tc` (default) streams every weight once
    for the batch through the tcgen05 GEMMs, `--path gather` gathers each
    token's rows).  `value` is tokens per second of the whole batch.  Under
    torchrun with N > 1 ranks: config 4 at batch B (run_tp_batch)."""
    if dist_env()[1] > 1:
        return run_tp_batch(args)
    import dip_b200  # noqa: F401
    from dip_b200.stack import StackConfig, layer_weight_bytes
    from dip_b200.batch import BatchedDipStack
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B = args.batch
    cfg = StackConfig(n_layers=args.layers, seed=0)
    stack = BatchedDipStack(cfg, B, dev, path=args.path if args.path in ("tc", "gather") else "auto")
    path = stack.path
    T = args.warmup + args.steps
    gen = torch.Generator().manual_seed(3000)
    x0 = torch.randn(T, B, cfg.hidden, generator=gen).to(torch.bfloat16).to(dev)
    resid = torch.randn(T, cfg.n_layers, B, cfg.hidden, generator=gen).to(torch.bfloat16).to(dev)
    stack.capture()
    xi, ri = stack._static_in
    for t in range(args.warmup):
        xi.copy_(x0[t]); ri.copy_(resid[t]); stack.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        e0.record()
        for t in range(args.warmup, T):
            xi.copy_(x0[t]); ri.copy_(resid[t]); stack.replay()
        e1.record()
        torch.cuda.synchronize()
    clk = clk.summary()
    ms = e0.elapsed_time(e1) / args.steps
    nb = layer_weight_bytes(cfg)
    passes = (B + 7) // 8
    if path == "tc":  # every row of the three matrices once per step
        layer_bytes = nb["gate"] * 3
        # permute + gate, top-k, counts, permute + up, down + reduce, RMSNorm
        launches = 9
    else:
        layer_bytes = passes * nb["gate"] + B * (nb["up"] + nb["down"])
        launches = passes + 1 + 2 * B + 1
    layer_us = ms * 1e3 / cfg.n_layers
    peak, peak_kind = _peaks()
    del stack
    rec = {
        "metric": "dip_mlp_decode_tok_s", "value": B * 1e3 / ms, "unit": "tok/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) int4 g128 weights, N(0,1) tokens)",
        "config": {"workload": f"config3: 64-layer stack, batch {B} independent tokens",
                   "batch": B, "layers": cfg.n_layers, "k": cfg.k, "path": path},
        "us_per_layer": layer_us, "us_per_token_layer": layer_us / B,
        "layer_bytes": layer_bytes, "layer_hbm_gbs": layer_bytes / (layer_us * 1e-6) / 1e9,
        "layer_hbm_frac": layer_bytes / (layer_us * 1e-6) / 1e9 / peak, "peak_kind": peak_kind,
        "gpu_launches": args.steps * cfg.n_layers * launches,
        "clocks": clk}
    if emit:
        print(json.dumps(rec), flush=True)
    return rec


def run_tp_batch(args):
    """Config 4 at batch B (`--config 3 --batch B` under torchrun): the
    batched stack sharded along I (TPBatchedDipStack: tcgen05 GEMMs on each
    rank's rows, NCCL all-gather of g and all-reduce of the fp32 partials).
    After the timed steps rank 0 checks one step's per-token indices at every
    layer against the single-GPU batched layer on the full weights and the
    same inputs (tp_idx_exact)."""
    rank, world, local = dist_env()
    import torch.distributed as dist
    import dip_b200  # noqa: F401
    from dip_b200.stack import StackConfig, layer_weight_bytes
    from dip_b200.batch import batched_dip_layer
    from dip_b200.tp import TPBatchedDipStack
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev)
    B = args.batch
    cfg = StackConfig(n_layers=args.layers, seed=0)
    stack = TPBatchedDipStack(cfg, B, dev, keep_full=(rank == 0))
    T = args.warmup + args.steps
    gen = torch.Generator().manual_seed(3000)
    x0 = torch.randn(T, B, cfg.hidden, generator=gen).to(torch.bfloat16).to(dev)
    resid = torch.randn(T, cfg.n_layers, B, cfg.hidden, generator=gen).to(torch.bfloat16).to(dev)
    ms, clk = _timed_replays(stack, x0, resid, args.warmup, args.steps, dev, world)
    if _device_error_all(world, dev):
        raise SystemExit("a bounded device wait ran out during the timed steps: run invalid")
    stack.step(x0[args.warmup], resid[args.warmup], record=True)
    torch.cuda.synchronize()
    n_bad = 0
    if rank == 0:
        for l in range(cfg.n_layers):
            _, _, idx1 = batched_dip_layer(stack.full[l], stack.last_x[l], cfg.k, "tc")
            n_bad += int(not torch.equal(idx1, stack.last_idx[l]))
    flag = torch.tensor([n_bad], device=dev)
    dist.broadcast(flag, 0)
    n_bad = int(flag.item())
    nb = layer_weight_bytes(cfg)
    layer_us = ms * 1e3 / cfg.n_layers
    per_gpu = nb["gate"] * 3 // world
    peak, peak_kind = _peaks()
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": B * 1e3 / ms, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,0.02) int4 g128 weights, N(0,1) tokens)",
            "config": {"workload": f"config4: the batch-{B} stack sharded along I over "
                                   f"{world} GPUs", "batch": B, "layers": cfg.n_layers,
                       "k": cfg.k, "parallelism": f"tp{world}", "path": "tc"},
            "us_per_layer": layer_us, "us_per_token_layer": layer_us / B,
            "per_gpu_hbm_gbs": per_gpu / (layer_us * 1e-6) / 1e9,
            "per_gpu_hbm_frac_of_measured": per_gpu / (layer_us * 1e-6) / 1e9 / peak,
            "peak_kind": peak_kind,
            "tp_idx_exact": n_bad == 0, "tp_idx_layers_checked": cfg.n_layers,
            "tp_idx_layers_differing": n_bad,
            "gpu_launches": args.steps * cfg.n_layers * 9,
            "clocks": clk}), flush=True)
    _barrier(world)
    torch.cuda.synchronize()
    sys.stdout.flush()
    os._exit(0 if n_bad == 0 else 3)


def _barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def _max_over_ranks(v: float, world: int, dev) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _timed_replays(stack, x0, resid, warmup, steps, dev, world):
    """Graph replays: `warmup` untimed, then `steps` between a barrier +
    synchronize on both sides, timed with CUDA events on the replay stream;
    returns (ms per step, max over ranks; clock summary)."""
    stack.capture()
    xi, ri = stack._static_in
    for t in range(warmup):
        xi.copy_(x0[t]); ri.copy_(resid[t]); stack.replay()
    torch.cuda.synchronize()
    _barrier(world); torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clk:
        e0.record()
        for t in range(warmup, warmup + steps):
            xi.copy_(x0[t]); ri.copy_(resid[t]); stack.replay()
        e1.record()
        torch.cuda.synchronize()
    _barrier(world); torch.cuda.synchronize()
    ms = _max_over_ranks(e0.elapsed_time(e1), world, dev)
    return ms / steps, clk.summary()


def _e2e(stack, x0, resid, warmup, steps, dev, world, n_layers, hidden):
    """The public call (stack.decode) with pinned host inputs and a host
    result every step: H2D of the token and its 64 residuals, D2H of y."""
    x0h = x0.cpu().pin_memory()
    rh = resid.cpu().pin_memory()
    for t in range(min(3, warmup)):
        stack.decode(x0h[t], rh[t])
    _barrier(world); torch.cuda.synchronize()
    t0 = time.perf_counter()
    for t in range(warmup, warmup + steps):
        stack.decode(x0h[t], rh[t])
    torch.cuda.synchronize()
    e2e_s = _max_over_ranks(time.perf_counter() - t0, world, dev)
    return {"value": steps / e2e_s, "unit": UNIT,
            "h2d_bytes_per_step": (x0[0].numel() + resid[0].numel()) * 2,
            "d2h_bytes_per_step": hidden * 2}


def _device_error_all(world, dev) -> int:
    """The library's device error word, OR-ed over the ranks (a bounded wait
    that ran out anywhere makes the run invalid)."""
    err = int(torch.ops.dip_b200.take_device_error())
    return int(_max_over_ranks(float(err), world, dev))


def _config1(cfg, world, parallelism):
    return {"workload": ("config1: 64-layer Qwen3-32B-shape DIP decode MLP stack, batch 1"
                         if world == 1 else
                         f"config4: the config-1 stack sharded along I over {world} GPUs, batch 1"),
            "hidden": cfg.hidden, "inter": cfg.inter, "k": cfg.k, "layers": cfg.n_layers,
            "keep_ratio": cfg.keep_ratio, "parallelism": parallelism,
            "l2": "no flush: each step reads ~9.5 GB of weights (> 126 MB L2)"}


def _roofline(kern, alg_bytes, layer_us, traffic, peak, peak_kind):
    """The dominant kernel is the whole layer (one launch per layer), so its
    duration per launch is the graph-replayed step time / layers: the launch
    plus the gap to the next one (an upper bound on the kernel time)."""
    achieved = alg_bytes / (layer_us * 1e-6) / 1e9
    return {"kernel": kern, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak, "peak_kind": f"{peak_kind} (burst copy)",
            "traffic": traffic, "algorithmic_bytes": alg_bytes, "avg_launch_us": layer_us,
            "launch_time_from": "graph-replayed timed region: ms_per_step / layers"}


def run_ours(args):
    rank, world, local = dist_env()
    if world > 1 and not args.replicas:
        return run_tp_fused(args)
    import dip_b200  # noqa: F401  (loads the kernels; raises if unbuilt)
    from dip_b200.stack import StackConfig, DipStack, token_inputs, layer_weight_bytes

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)
    cfg = StackConfig(n_layers=args.layers, seed=rank)
    stack = DipStack(cfg, dev, fused=(args.path == "fused"))
    T = args.warmup + args.steps
    x0, resid = token_inputs(cfg, T, seed=1000 + rank, device=dev)
    ms_per_step, clk = _timed_replays(stack, x0, resid, args.warmup, args.steps, dev, world)
    if _device_error_all(world, dev):
        raise SystemExit("a bounded device wait ran out during the timed steps: run invalid")
    value = world * 1e3 / ms_per_step
    e2e = _e2e(stack, x0, resid, args.warmup, args.steps, dev, world, cfg.n_layers, cfg.hidden)
    e2e["value"] *= world

    nb = layer_weight_bytes(cfg)
    peak, peak_kind = _peaks()
    layer_us = ms_per_step * 1e3 / cfg.n_layers
    layer_gbs = nb["total"] / (layer_us / 1e6) / 1e9
    if stack.fused:
        kern = "layer_fused_kernel (one decode layer: gate, exact top-k, gathered up/down)"
        roof = _roofline(kern, nb["total"], layer_us, _traffic().get("layer_fused_kernel"), peak,
                         peak_kind)
    else:
        roof = None
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) int4 g128 weights, N(0,1) tokens)",
        "config": _config1(cfg, 1, "single" if world == 1 else f"replicas{world}"),
        "us_per_layer": layer_us,
        "layer_hbm_gbs": layer_gbs,
        "layer_hbm_frac_of_measured": layer_gbs / peak,
        "layer_hbm_frac_of_8tbs": layer_gbs / 8000.0,
        "roofline": roof,
        "e2e": e2e,
        "gpu_launches": args.steps * (cfg.n_layers if stack.fused else cfg.n_layers * 6 - 1),
        "path": args.path,
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # bounded CPU sample on layer 0's own weights
        L0 = {k: v.cpu() for k, v in stack.layers[0].items()}
        sec, cores = cpu_reference_layer_time(args.cpu_layers, layer=L0)
        line["cpu_baseline"] = {
            "value": 1.0 / (64 * sec), "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{args.cpu_layers} layers of the reference CPU math on layer 0's "
                      f"weights; tok/s = 1/(64 x {sec:.3f} s/layer)"}
    if rank == 0 and world == 1 and args.subresults:
        del stack
        torch.cuda.empty_cache()
        line["subresults"] = _subresults(args, dev)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_tp_fused(args):
    """Config 4: one token stream, every layer sharded along I over the N
    ranks, one dip_mlp_decode_fused_tp launch per layer and rank.  After the
    timed steps: one recorded token whose per-layer indices (all ranks'
    entries) rank 0 compares with the single-GPU fused layer on the full
    weights and the same layer inputs (tp_idx_exact), and the same shards
    timed with no exchange at all (each rank alone on its rows, k / N) to
    give the exposed cost of the cross-GPU steps."""
    rank, world, local = dist_env()
    import torch.distributed as dist
    import dip_b200  # noqa: F401
    from dip_b200.stack import StackConfig, DipStack, token_inputs, layer_weight_bytes, RMS_EPS
    from dip_b200.tp import TPFusedStack
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev)
    cfg = StackConfig(n_layers=args.layers, seed=0)
    stack = TPFusedStack(cfg, dev, keep_full=(rank == 0))
    T = args.warmup + args.steps
    x0, resid = token_inputs(cfg, T, seed=1000, device=dev)
    ms_per_step, clk = _timed_replays(stack, x0, resid, args.warmup, args.steps, dev, world)
    if _device_error_all(world, dev):
        raise SystemExit("a bounded device wait ran out during the timed steps: run invalid")
    e2e = _e2e(stack, x0, resid, args.warmup, args.steps, dev, world, cfg.n_layers, cfg.hidden)
    if _device_error_all(world, dev):
        raise SystemExit("a bounded device wait ran out during the e2e steps: run invalid")

    # in-run parity against one GPU: the first timed token, recorded
    stack.step(x0[args.warmup], resid[args.warmup], record=True)
    torch.cuda.synchronize()
    exact, y_ok, n_bad = True, True, 0
    if rank == 0:
        ws1 = torch.zeros(torch.ops.dip_b200.mlp_fused_workspace_bytes(cfg.hidden, cfg.inter, cfg.k),
                          dtype=torch.uint8, device=dev)
        for l in range(cfg.n_layers):
            L = stack.full[l]
            y1, _, idx1 = torch.ops.dip_b200.mlp_decode_fused(
                L["gate_qw"], L["gate_sc"], L["up_qw"], L["up_sc"], L["down_t_qw"],
                L["down_t_sc"], stack.last_x[l], None, RMS_EPS, cfg.k, ws1)
            if not torch.equal(idx1, stack.last_idx[l]):
                exact = False
                n_bad += 1
        del ws1
    flag = torch.tensor([0 if exact else 1], device=dev)
    dist.broadcast(flag, 0)
    exact = flag.item() == 0

    # the same shards with no cross-GPU step: each rank alone on its rows
    stack.full = None
    torch.cuda.empty_cache()
    cfg_loc = StackConfig(n_layers=cfg.n_layers, inter=cfg.inter // world, seed=0)
    local_stack = DipStack(cfg_loc, dev, layers=stack.shards)
    ms_loc, _ = _timed_replays(local_stack, x0, resid, args.warmup, args.steps, dev, world)
    if _device_error_all(world, dev):
        raise SystemExit("a bounded device wait ran out in the local-only timing: run invalid")

    nb = layer_weight_bytes(cfg)
    peak, peak_kind = _peaks()
    layer_us = ms_per_step * 1e3 / cfg.n_layers
    loc_us = ms_loc * 1e3 / cfg.n_layers
    per_gpu_bytes = nb["total"] // world
    line = {
        "metric": METRIC, "value": 1e3 / ms_per_step, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) int4 g128 weights, N(0,1) tokens)",
        "config": _config1(cfg, world, f"tp{world}"),
        "us_per_layer": layer_us,
        "per_gpu_hbm_gbs": per_gpu_bytes / (layer_us * 1e-6) / 1e9,
        "per_gpu_hbm_frac_of_measured": per_gpu_bytes / (layer_us * 1e-6) / 1e9 / peak,
        "tp_idx_exact": exact, "tp_idx_layers_checked": cfg.n_layers,
        "tp_idx_layers_differing": n_bad,
        "local_only_us_per_layer": loc_us,
        "comm_us_per_layer": layer_us - loc_us,
        "comm_frac_of_layer": (layer_us - loc_us) / layer_us,
        "comm_note": ("exposed cost of the cross-GPU steps inside the fused TP kernel (remote "
                      "histogram increments, count words, y-slot exchange, waiting for the "
                      "slowest rank) = TP layer time - the same shards run alone with k/N"),
        "roofline": _roofline("layer_fused_kernel<TP> (one sharded decode layer per rank)",
                              per_gpu_bytes, layer_us, None, peak, peak_kind),
        "e2e": e2e,
        "gpu_launches": args.steps * cfg.n_layers,
        "clocks": clk,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    _barrier(world)
    torch.cuda.synchronize()
    sys.stdout.flush()
    code = 0 if exact else 3
    if rank == 0 and not exact:
        print(f"tensor-parallel indices differ from one GPU's on {n_bad} layers", file=sys.stderr)
    os._exit(code)


def _subresults(args, dev):
    """Short sub-runs recorded in the headline line: config 2 (cache-aware
    DIP, hit rate and split exactness) and config 3 (batch 64 through the
    tcgen05 GEMMs)."""
    import argparse as _ap
    out = {}
    sub = _ap.Namespace(**vars(args))
    sub.steps, sub.warmup = args.sub_steps, 3
    out["config2"] = run_config2(sub, emit=False)
    torch.cuda.empty_cache()
    sub.batch, sub.path = 64, "tc"
    out["config3_b64"] = run_config3(sub, emit=False)
    torch.cuda.empty_cache()
    us, fused = _module_forward_us(dev)
    out["config0_module_forward"] = {
        "us_per_call": us, "fused_layer": fused,
        "what": "StreamingDIPMlp.forward on one config-0 layer, eager (no CUDA graph), "
                "cold weights only on the first call"}
    torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=64)
    ap.add_argument("--cpu-layers", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", type=int, default=1, choices=[1, 2, 3],
                    help="1: DIP stack (the headline line); 2: cache-aware DIP stack; "
                         "3: batched decode (--batch)")
    ap.add_argument("--batch", type=int, default=8, help="config 3: tokens per step")
    ap.add_argument("--comm", default="p2p", choices=["p2p", "nccl"],
                    help="config 4: exchanges over peer memory (p2p) or NCCL")
    ap.add_argument("--tp", action="store_true",
                    help="config 4 as separate launches (gate, top-k, up, down, exchange "
                         "kernels or NCCL, --comm) over the torchrun ranks")
    ap.add_argument("--replicas", action="store_true",
                    help="under torchrun: N independent single-GPU stacks instead of config 4")
    ap.add_argument("--no-subresults", dest="subresults", action="store_false",
                    help="skip the config-2 and config-3 sub-runs of the one-GPU line")
    ap.add_argument("--sub-steps", type=int, default=8)
    ap.add_argument("--gemm-tc", type=int, default=0, metavar="N",
                    help="profiling aid: N launches of the batch-64 tcgen05 gate GEMM, then exit")
    ap.add_argument("--single-layer", type=int, default=0, metavar="N",
                    help="profiling aid: N launches of one config-1 fused layer, then exit")
    ap.add_argument("--path", default="fused", choices=["fused", "chain", "tc", "gather"],
                    help="config 1: fused (one persistent kernel per layer) or chain (separate "
                         "launches); config 3: tc (default, dense tcgen05 GEMMs) or gather")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.single_layer:
        run_single_layer(args.single_layer)
    elif args.gemm_tc:
        run_gemm_tc(args.gemm_tc)
    elif args.config == 2:
        run_config2(args)
    elif args.config == 3:
        run_config3(args)
    elif args.tp:
        run_tp(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
