"""Parity with the reference's OWN kernels (GPU).

The reference's five .cu files are compiled from its sources for sm_100a into
oracle/_ref (oracle/Makefile) and run in a subprocess on the same inputs.
Top-k indices must be identical; float outputs within the path tolerance.
Also writes tests/golden/topk_ref_golden.pt when DIP_WRITE_GOLDEN is set (the
committed top-k vectors the CPU oracle test pins against)."""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]
REF_LIB = REPO / "oracle" / "_ref"
RTOL, ATOL = 1e-2, 2e-3


def _topk_inputs():
    g = torch.Generator().manual_seed(123)
    cases = {}
    for n, k in [(25600, 15360), (4096, 2458), (1000, 1), (777, 777)]:
        cases[f"topk_normal_{n}_{k}"] = torch.randn(n, generator=g)
    cases["topk_ties"] = torch.randint(-6, 7, (25600,), generator=g).float() / 4
    z = torch.randn(4096, generator=g)
    z[torch.rand(4096, generator=g) < 0.6] = 0
    cases["topk_zeros"] = z
    w = torch.randn(4096, generator=g) * 1e-9
    w[:50] = 1e4
    cases["topk_wide"] = w
    cases["topk_silu"] = torch.nn.functional.silu(torch.randn(25600, generator=g) * 1.4)
    ks = {"topk_ties": 15360, "topk_zeros": 2458, "topk_wide": 2458, "topk_silu": 15360}
    out = {}
    for name, s in cases.items():
        k = ks.get(name) or int(name.split("_")[-1])
        out[name] = {"op": "topk", "args": [s.to(torch.bfloat16), k]}
    return out


def _float_inputs(oracle):
    g = torch.Generator().manual_seed(0)
    q = torch.randint(-8, 8, (4096, 5120), dtype=torch.int8, generator=g)
    sc = (torch.rand(4096, 40, generator=g) * 0.01 + 0.001).to(torch.bfloat16)
    qw = oracle.pack_int4(q)
    x = torch.randn(5120, generator=g).to(torch.bfloat16)
    idx = torch.randperm(4096, generator=g)[:2457].sort().values.to(torch.int32)
    h = torch.randn(4096, generator=g).to(torch.bfloat16)
    src = (torch.rand(2457, generator=g) < 0.4).to(torch.int32)
    row = torch.randint(0, 2048, (2457,), generator=g).to(torch.int32)
    return {
        "gemv": {"op": "gemv", "args": [qw, sc, x]},
        "gather": {"op": "gather", "args": [qw, sc, x, idx]},
        "down": {"op": "down", "args": [qw, sc, h]},
        "ca": {"op": "ca", "args": [qw[:2048], sc[:2048], qw[2048:], sc[2048:], x, src, row]},
    }


@pytest.fixture(scope="module")
def ref_outputs(tmp_path_factory, oracle):
    if not any(REF_LIB.glob("*.so")):
        pytest.fail("oracle/_ref is empty: build it with `make -C oracle` (needs the "
                    "reference checkout)")
    cases = {**_topk_inputs(), **_float_inputs(oracle)}
    d = tmp_path_factory.mktemp("ref")
    torch.save(cases, d / "in.pt")
    subprocess.run([sys.executable, str(REPO / "tests" / "ref_kernel_runner.py"),
                    str(d / "in.pt"), str(d / "out.pt")], check=True)
    return cases, torch.load(d / "out.pt")


def test_topk_identical_to_reference_kernel(dip, oracle, ref_outputs):
    cases, ref = ref_outputs
    golden = {}
    for name, c in cases.items():
        if c["op"] != "topk":
            continue
        s, k = c["args"]
        mine = torch.ops.topk_ops.topk_select(s.cuda(), k).cpu()
        assert torch.equal(mine, ref[name]), name
        assert torch.equal(oracle.topk_select(s, k), ref[name]), name
        golden[name] = {"s": s, "k": k, "idx": ref[name]}
    if os.environ.get("DIP_WRITE_GOLDEN"):
        out = Path(os.environ["DIP_WRITE_GOLDEN"])
        out.parent.mkdir(parents=True, exist_ok=True)
        torch.save(golden, out)


@pytest.mark.parametrize("name", ["gemv", "gather", "down", "ca"])
def test_float_ops_match_reference_kernels(dip, ref_outputs, name):
    cases, ref = ref_outputs
    c = cases[name]
    a = [t.cuda() if torch.is_tensor(t) else t for t in c["args"]]
    op = {"gemv": torch.ops.int4_ops.int4_gemv,
          "gather": torch.ops.int4_gather_ops.int4_gather_gemv,
          "down": torch.ops.int4_down_ops.int4_gather_down,
          "ca": torch.ops.ca_fused_ops.ca_fused_gemv}[name]
    mine = op(*a).cpu().float()
    r = ref[name].float()
    err = (mine - r).abs()
    assert bool((err <= ATOL + RTOL * r.abs()).all()), f"{name}: max err {err.max():.3e}"
