"""Runs the REFERENCE's own CUDA kernels (compiled from its sources into
oracle/_ref by oracle/Makefile) on inputs from a .pt file and saves their
outputs.  Used by tests/test_ref_kernels_gpu.py in a separate process,
because the reference registers the same operator namespaces as dip_b200.

    python tests/ref_kernel_runner.py in.pt out.pt
"""
import sys
from pathlib import Path

import torch

REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref"


def main(inp: str, out: str) -> None:
    for so in sorted(REF_LIB.glob("*.so")):
        torch.ops.load_library(str(so))
    cases = torch.load(inp)
    dev = torch.device("cuda", 0)
    res = {}
    for name, c in cases.items():
        op = c["op"]
        a = [t.to(dev) if torch.is_tensor(t) else t for t in c["args"]]
        if op == "topk":
            r = torch.ops.topk_ops.topk_select(*a)
        elif op == "gemv":
            r = torch.ops.int4_ops.int4_gemv(*a)
        elif op == "gather":
            r = torch.ops.int4_gather_ops.int4_gather_gemv(*a)
        elif op == "down":
            r = torch.ops.int4_down_ops.int4_gather_down(*a)
        elif op == "ca":
            r = torch.ops.ca_fused_ops.ca_fused_gemv(*a)
        else:
            raise ValueError(op)
        res[name] = r.cpu()
    torch.cuda.synchronize()
    torch.save(res, out)


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2])
