"""The allocation-free down projection, called through the C ABI (GPU).

dip_int4_gather_down_noalloc serves callers that cannot allocate device
memory at call time (a host framework owns the memory pool, a fixed memory
budget, or an FFI caller without a CUDA allocator): it keeps its partial sums
in a static device array of the library instead of a caller workspace.  Its
output must equal dip_int4_gather_down's bit for bit, on two calls in a row
(the second call reuses the array the first one left behind), and the CPU
oracle's within the path tolerance.
This file is collected last so that a stop-at-first-failure run has already
run every other test when it gets here.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 2e-3


def _core():
    import sys
    from pathlib import Path
    pkg = Path(__file__).resolve().parents[1] / "dynamic-input-pruning_b200"
    if str(pkg) not in sys.path:
        sys.path.insert(0, str(pkg))
    from dip_b200 import _lib
    core = _lib.core()
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    core.dip_int4_gather_down_noalloc.argtypes = [vp, vp, i64, vp, vp, i64, i64, vp, vp]
    core.dip_int4_gather_down.argtypes = [vp, vp, i64, vp, vp, i64, i64, vp, ctypes.c_size_t,
                                          vp, vp]
    core.dip_gather_down_workspace_bytes.restype = ctypes.c_size_t
    core.dip_gather_down_workspace_bytes.argtypes = [i64]
    return core


def _case(seed, n_rows, out_f, k, dev):
    g = torch.Generator().manual_seed(seed)
    q = torch.randint(0, 256, (n_rows, out_f // 2), dtype=torch.uint8, generator=g)
    sc = (torch.rand(n_rows, out_f // 128, generator=g) * 0.01 + 0.001).to(torch.bfloat16)
    h = torch.randn(k, generator=g).to(torch.bfloat16)
    idx = torch.randperm(n_rows, generator=g)[:k].to(torch.int32)
    return [t.to(dev) for t in (q.view(torch.int8), sc, h, idx)]


def test_noalloc_down_matches_workspace_version():
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    core = _core()
    stream = torch.cuda.current_stream().cuda_stream
    out_f, n_rows, k = 5120, 25600, 15360
    for call, seed in enumerate((101, 202)):  # two calls in a row
        q, sc, h, idx = _case(seed, n_rows, out_f, k, dev)
        y_na = torch.empty(out_f, dtype=torch.bfloat16, device=dev)
        st = core.dip_int4_gather_down_noalloc(q.data_ptr(), sc.data_ptr(), n_rows, h.data_ptr(),
                                               idx.data_ptr(), k, out_f, y_na.data_ptr(), stream)
        assert st == 0, f"call {call}: status {st}"
        nws = core.dip_gather_down_workspace_bytes(out_f)
        ws = torch.empty(nws, dtype=torch.uint8, device=dev)
        y_ws = torch.empty(out_f, dtype=torch.bfloat16, device=dev)
        st = core.dip_int4_gather_down(q.data_ptr(), sc.data_ptr(), n_rows, h.data_ptr(),
                                       idx.data_ptr(), k, out_f, ws.data_ptr(), nws,
                                       y_ws.data_ptr(), stream)
        assert st == 0
        torch.cuda.synchronize()
        # the same launch sequence with the same fixed-order reduction, only
        # the scratch lives elsewhere: the outputs must be bit-identical
        assert torch.equal(y_na, y_ws), f"call {call}: differs from the workspace version"
        if call == 0:  # and both agree with the CPU oracle within the path tolerance
            from oracle import dip_oracle as O
            ref = O.gather_down_f32(q.cpu(), sc.cpu(), h.cpu(), rows=idx.cpu().long())
            err = (y_na.float().cpu() - ref).abs()
            assert bool((err <= ATOL + RTOL * ref.abs()).all()), f"max err {err.max():.3e}"


def test_noalloc_down_rejects_oversize():
    core = _core()
    st = core.dip_int4_gather_down_noalloc(None, None, 1, None, None, 1, 16384, None, None)
    assert st == 4  # DIP_ERR_UNSUPPORTED: out_features above the static array's limit
