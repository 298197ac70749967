"""Generate the weight-format golden vectors from the reference's OWN code.

Imports the reference's Python functions (scripts/quantize.py:32-64,
qlinear.py:28-64, dip_stream_predispatch.py:77-120) from a checkout of
rohitpotluri/dynamic-input-pruning and records their outputs on small seeded
inputs, including edge cases (an all-zero group -> scale clamp, exact .5
quotients -> round-half-even, +-max values, large magnitudes).

    python tests/golden/make_golden.py /path/to/reference

Writes tests/golden/format_golden.pt.  Only this script needs the reference;
the tests read the committed file.
"""
import importlib.util
import sys
from pathlib import Path

import torch


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main(ref_root: str) -> None:
    ref = Path(ref_root)
    sys.path.insert(0, str(ref))  # dip_stream_predispatch imports qlinear by name
    quant = _load("ref_quantize", ref / "scripts" / "quantize.py")
    qlin = _load("qlinear", ref / "qlinear.py")
    dsp = _load("ref_dip_stream_predispatch", ref / "dip_stream_predispatch.py")

    gen = torch.Generator().manual_seed(20261201)
    cases = {}
    # gate/up-like matrix with edge rows
    w = (torch.randn(64, 512, generator=gen) * 0.02)
    w[1, :128] = 0.0                                   # all-zero group -> s clamp 1e-8
    w[2, :128] = torch.linspace(-7, 7, 128) * 0.01     # exact multiples of s -> .5 ties
    w[3, 128:256] = torch.tensor([3.5, -3.5] * 64) * 1e-3
    w[4] = torch.randn(512, generator=gen) * 50.0      # large magnitudes
    w = w.to(torch.bfloat16)
    qw, sc = quant.quantize_tensor_int4_groupwise(w)
    deq = qlin.dequantize(qw, sc)
    unpacked = qlin._unpack_int4(qw)
    cases["gate"] = {"w": w, "qweight": qw, "scales": sc, "dequant": deq, "unpacked": unpacked}
    # down-like matrix [hidden, inter] and its transposed requantisation
    wd = (torch.randn(256, 384, generator=gen) * 0.02).to(torch.bfloat16)
    dq, ds = quant.quantize_tensor_int4_groupwise(wd)
    tq, ts = dsp._transpose_down_to_int4(dq, ds)
    cases["down"] = {"w": wd, "qweight": dq, "scales": ds, "down_t_qw": tq, "down_t_sc": ts}
    out = Path(__file__).with_name("format_golden.pt")
    torch.save(cases, out)
    print("wrote", out)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
