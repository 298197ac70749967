"""The drop-in boundary without a GPU: the C-ABI library loads and exports
every symbol include/dip_b200.h declares, host-side argument checks reject
bad calls before any launch, and the torch extension registers the
reference's operator schemas verbatim."""
import ctypes

import pytest
import torch


@pytest.fixture(scope="module")
def core():
    from dip_b200 import _lib
    return _lib.core()


def test_every_header_symbol_is_exported(core):
    from dip_b200 import _lib
    syms = _lib.header_symbols()
    assert len(syms) >= 20
    for name in syms:
        assert hasattr(core, name), name


def test_version_and_status_strings(core):
    assert core.dip_version() >= 100
    core.dip_status_string.restype = ctypes.c_char_p
    assert core.dip_status_string(0) == b"ok"
    assert b"invalid" in core.dip_status_string(1)
    assert core.dip_status_string(99) == b"unknown status"


def test_workspace_helpers(core):
    core.dip_gather_down_workspace_bytes.restype = ctypes.c_size_t
    core.dip_gather_down_workspace_bytes.argtypes = [ctypes.c_int64]
    assert core.dip_gather_down_workspace_bytes(5120) == 148 * 5120 * 4
    core.dip_mlp_workspace_bytes.restype = ctypes.c_size_t
    core.dip_mlp_workspace_bytes.argtypes = [ctypes.c_int64] * 3
    n = core.dip_mlp_workspace_bytes(5120, 25600, 15360)
    assert n >= 25600 * 2 + 15360 * 6 + 148 * 5120 * 4
    assert core.dip_mlp_workspace_bytes(0, 25600, 15360) == 0


def test_pdl_switch(core):
    prev = core.dip_set_pdl(0)
    assert core.dip_set_pdl(prev) == 0


def test_argument_checks_need_no_gpu(core):
    vp = ctypes.c_void_p
    core.dip_int4_gemv.argtypes = [vp, vp, vp, vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, vp]
    # null pointers / bad in_features are rejected before any CUDA call
    assert core.dip_int4_gemv(None, None, None, None, 16, 5120, 1, None) == 1
    assert core.dip_int4_gemv(None, None, None, None, 16, 100, 1, None) == 1
    assert core.dip_int4_gemv(None, None, None, None, 0, 5120, 1, None) == 0  # empty: no-op
    core.dip_topk_select.argtypes = [vp, ctypes.c_int64, ctypes.c_int64, vp, vp]
    assert core.dip_topk_select(None, 25600, 15360, None, None) == 1
    assert core.dip_topk_select(None, 1 << 20, 5, None, None) == 1
    core.dip_int4_gather_down.argtypes = [vp, vp, ctypes.c_int64, vp, vp, ctypes.c_int64,
                                          ctypes.c_int64, vp, ctypes.c_size_t, vp, vp]
    assert core.dip_int4_gather_down(None, None, 10, None, None, 5, 5120, None, 0, None,
                                     None) == 1
    # misaligned weight pointer
    assert core.dip_int4_gemv(vp(8), vp(16), vp(16), vp(16), 16, 5120, 0, None) == 1


REFERENCE_SCHEMAS = {
    ("int4_ops", "int4_gemv"): "int4_gemv(Tensor qweight, Tensor scales, Tensor x) -> Tensor",
    ("topk_ops", "topk_select"): "topk_select(Tensor s, int k) -> Tensor",
    ("int4_gather_ops", "int4_gather_gemv"):
        "int4_gather_gemv(Tensor qweight, Tensor scales, Tensor x, Tensor indices) -> Tensor",
    ("int4_down_ops", "int4_gather_down"):
        "int4_gather_down(Tensor down_t_sel, Tensor scales, Tensor h_sel) -> Tensor",
    ("ca_fused_ops", "ca_fused_gemv"):
        "ca_fused_gemv(Tensor res_qw, Tensor res_sc, Tensor str_qw, Tensor str_sc, Tensor x, "
        "Tensor src, Tensor row) -> Tensor",
}


@pytest.mark.parametrize("ns,op", list(REFERENCE_SCHEMAS))
def test_reference_schemas(dip, ns, op):
    schema = str(getattr(getattr(torch.ops, ns), op).default._schema)
    assert schema == f"{ns}::{REFERENCE_SCHEMAS[(ns, op)]}"


def test_no_cpu_kernel(dip):
    """The decode ops have no CPU implementation: calling one on CPU tensors
    raises instead of silently falling back."""
    qw = torch.zeros(16, 64, dtype=torch.int8)
    sc = torch.zeros(16, 1, dtype=torch.bfloat16)
    x = torch.zeros(128, dtype=torch.bfloat16)
    with pytest.raises(Exception):
        torch.ops.int4_ops.int4_gemv(qw, sc, x)


def test_fake_tensor_shapes(dip):
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        qw = torch.empty(256, 64, dtype=torch.int8, device="cuda")
        sc = torch.empty(256, 1, dtype=torch.bfloat16, device="cuda")
        x = torch.empty(128, dtype=torch.bfloat16, device="cuda")
        assert torch.ops.int4_ops.int4_gemv(qw, sc, x).shape == (256,)
        assert torch.ops.topk_ops.topk_select(x, 7).shape == (7,)
        y, g, idx = torch.ops.dip_b200.mlp_decode(qw, sc, qw, sc, qw[:, :], sc, x, 9)
        assert idx.shape == (9,) and g.shape == (256,)


def test_modules_importable(dip):
    assert dip.StreamingDIPMlp and dip.CADIPMlp and dip.QuantLinear
    from dip_b200 import dip_stream_predispatch as dsp
    assert dsp._use_gather and dsp._use_down


def test_python_modules_import():
    """Every module of the package imports on a host without a GPU (the
    kernels load; nothing runs)."""
    import importlib
    for m in ("dip_b200.stack", "dip_b200.batch", "dip_b200.tp", "dip_b200.dip_ca",
              "dip_b200.dip_stream_predispatch", "dip_b200.qlinear"):
        importlib.import_module(m)
