"""Loader for the in-tree sm_100a libraries (built by ../build.py).

  libdip_core.so    C ABI of include/dip_b200.h, loaded with ctypes
  dip_torch_ops.so  torch operator registrations (the reference's five schemas
                    plus namespace dip_b200), loaded with torch.ops.load_library

There is deliberately no fallback: if a library is missing, importing the
package raises, because the decode path has no CPU or pure-torch substitute.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import torch

LIBDIR = Path(__file__).resolve().parent / "_lib"
CORE_SO = LIBDIR / "libdip_core.so"
OPS_SO = LIBDIR / "dip_torch_ops.so"

_core: ctypes.CDLL | None = None
_ops_loaded = False


def _missing(p: Path) -> ImportError:
    return ImportError(
        f"{p.name} not found in {p.parent}. Build the sm_100a kernels first: "
        "python dynamic-input-pruning_b200/build.py (or __graft_entry__.build())")


def core() -> ctypes.CDLL:
    """The C ABI library (ctypes handle)."""
    global _core
    if _core is None:
        if not CORE_SO.exists():
            raise _missing(CORE_SO)
        _core = ctypes.CDLL(str(CORE_SO))
    return _core


def load_ops() -> None:
    """Register the torch operators (idempotent)."""
    global _ops_loaded
    if _ops_loaded:
        return
    if not OPS_SO.exists():
        raise _missing(OPS_SO)
    core()  # resolve libdip_core first (rpath also finds it)
    torch.ops.load_library(str(OPS_SO))
    _register_fakes()
    _register_fakes_fused()
    _ops_loaded = True


def _register_fakes() -> None:
    """Meta implementations, as the reference registers them
    (gate_kernel.py:21-23, topk_kernel.py:21-23,
    dip_stream_predispatch.py:59-71, dip_ca.py:50-52)."""
    rf = torch.library.register_fake

    @rf("int4_ops::int4_gemv")
    def _(qweight, scales, x):
        return torch.empty(qweight.shape[0], dtype=torch.bfloat16, device=x.device)

    @rf("topk_ops::topk_select")
    def _(s, k):
        return torch.empty(k, dtype=torch.int32, device=s.device)

    @rf("int4_gather_ops::int4_gather_gemv")
    def _(qweight, scales, x, indices):
        return torch.empty(indices.shape[0], dtype=torch.bfloat16, device=x.device)

    @rf("int4_down_ops::int4_gather_down")
    def _(down_t_sel, scales, h_sel):
        return torch.empty(down_t_sel.shape[1] * 2, dtype=torch.bfloat16, device=h_sel.device)

    @rf("ca_fused_ops::ca_fused_gemv")
    def _(res_qw, res_sc, str_qw, str_sc, x, src, row):
        return torch.empty(src.shape[0], dtype=torch.bfloat16, device=x.device)

    @rf("dip_b200::gate_silu")
    def _(qweight, scales, x):
        return torch.empty(qweight.shape[0], dtype=torch.bfloat16, device=x.device)

    @rf("dip_b200::topk_select_batched")
    def _(s, k):
        return torch.empty(s.shape[0], k, dtype=torch.int32, device=s.device)

    @rf("dip_b200::gather_up_h")
    def _(up_qw, up_sc, x, g, idx):
        return torch.empty(idx.shape[0], dtype=torch.bfloat16, device=x.device)

    @rf("dip_b200::gather_down_idx")
    def _(dt_qw, dt_sc, h, idx):
        return torch.empty(dt_qw.shape[1] * 2, dtype=torch.bfloat16, device=h.device)

    @rf("dip_b200::mlp_decode")
    def _(gq, gs, uq, us, dq, ds, x, k, workspace=None):
        return (torch.empty(gq.shape[1] * 2, dtype=torch.bfloat16, device=x.device),
                torch.empty(gq.shape[0], dtype=torch.bfloat16, device=x.device),
                torch.empty(k, dtype=torch.int32, device=x.device))


def _register_fakes_fused():
    @torch.library.register_fake("dip_b200::mlp_decode_fused")
    def _(gq, gs, uq, us, dq, ds, x, resid, eps, k, workspace=None, h_out=None,
          next_gate_qw=None, next_gate_sc=None):
        return (torch.empty(gq.shape[1] * 2, dtype=torch.bfloat16, device=x.device),
                torch.empty(gq.shape[0], dtype=torch.bfloat16, device=x.device),
                torch.empty(k, dtype=torch.int32, device=x.device))


    @torch.library.register_fake("dip_b200::mlp_decode_fused_ca")
    def _(gq, gs, uq, us, dq, ds, id2slot, ruq, rus, rdq, rds, x, resid, eps, k, workspace=None,
          next_gate_qw=None, next_gate_sc=None):
        return (torch.empty(gq.shape[1] * 2, dtype=torch.bfloat16, device=x.device),
                torch.empty(gq.shape[0], dtype=torch.bfloat16, device=x.device),
                torch.empty(k, dtype=torch.int32, device=x.device))

    @torch.library.register_fake("dip_b200::mlp_decode_fused_tp")
    def _(gq, gs, uq, us, dq, ds, x, resid, eps, k, inter_total, rank, world, workspaces,
          workspace_bytes, idx_out=None, x_used=None, h_out=None, next_gate_qw=None,
          next_gate_sc=None):
        return (torch.empty(gq.shape[1] * 2, dtype=torch.bfloat16, device=x.device),
                torch.empty(gq.shape[0], dtype=torch.bfloat16, device=x.device))

    @torch.library.register_fake("dip_b200::gemv_batched")
    def _(qweight, scales, x, silu):
        return torch.empty(x.shape[0], qweight.shape[0], dtype=torch.bfloat16, device=x.device)

    @torch.library.register_fake("dip_b200::down_tc_f32")
    def _(dt_qw, dt_sc, h):
        return torch.empty(h.shape[0], dt_qw.shape[1] * 2, dtype=torch.float32, device=h.device)

    @torch.library.register_fake("dip_b200::gemm_tc")
    def _(qweight, scales, x, epilogue, g=None, cnt=None, ksplit=0):
        return torch.empty(x.shape[0], qweight.shape[0], dtype=torch.bfloat16, device=x.device)

    @torch.library.register_fake("dip_b200::down_tc")
    def _(dt_qw, dt_sc, h):
        return torch.empty(h.shape[0], dt_qw.shape[1] * 2, dtype=torch.bfloat16, device=h.device)

    @torch.library.register_fake("dip_b200::select_count")
    def _(idx, inter):
        return torch.empty(idx.shape[0], inter, dtype=torch.int32, device=idx.device)


def header_symbols() -> list[str]:
    """Every function the public header declares (DIP_API ...)."""
    import re
    hdr = Path(__file__).resolve().parents[2] / "include" / "dip_b200.h"
    return re.findall(r"^DIP_API [^(]*?\b(dip_\w+)\(", hdr.read_text(), flags=re.M)
