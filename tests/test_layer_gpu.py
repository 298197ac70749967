"""Whole-layer parity (GPU): the fused decode chain, the drop-in modules and
the C ABI against the oracle.  Selected indices and cache splits are compared
bit for bit given the same g; g, h and y within the path's tolerance."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 2e-3


def close(out, ref):
    out, ref = out.float().cpu(), ref.float().cpu()
    err = (out - ref).abs()
    bad = err > ATOL + RTOL * ref.abs()
    assert not bad.any(), f"{int(bad.sum())} out of tolerance, max err {err.max():.3e}"


@pytest.fixture(scope="module")
def layer_c0(dip, oracle):
    """hidden 5120, inter 25600, N(0, 0.02) weights,
    quantised on the GPU (bit exactness of that step is tested separately)."""
    dev = torch.device("cuda", 0)
    gen = torch.Generator().manual_seed(0)
    H, I = 5120, 25600
    wg = (torch.randn(I, H, generator=gen) * 0.02).to(torch.bfloat16)
    wu = (torch.randn(I, H, generator=gen) * 0.02).to(torch.bfloat16)
    wd = (torch.randn(H, I, generator=gen) * 0.02).to(torch.bfloat16)
    q = torch.ops.dip_b200.quantize_int4
    gq, gs = q(wg.to(dev))
    uq, us = q(wu.to(dev))
    dq, ds = q(wd.to(dev))
    tq, ts = torch.ops.dip_b200.transpose_down_int4(dq, ds)
    x = torch.randn(H, generator=gen).to(torch.bfloat16)
    return {"gate_qw": gq, "gate_sc": gs, "up_qw": uq, "up_sc": us, "down_qw": dq,
            "down_sc": ds, "down_t_qw": tq, "down_t_sc": ts, "x": x.to(dev), "k": 15360}


def _check_chain(oracle, L, y, g, idx):
    cpu = {k: v.cpu() for k, v in L.items() if torch.is_tensor(v)}
    x = cpu["x"]
    # g vs the oracle's g (bf16 rounding points identical; order of sums differs)
    g_ref = oracle.silu_bf16(oracle.int4_gemv(cpu["gate_qw"], cpu["gate_sc"], x))
    close(g, g_ref)
    # indices: bit exact given the same g
    g_cpu = g.cpu()
    assert torch.equal(idx.cpu(), oracle.topk_select(g_cpu, L["k"]))
    # y vs the oracle chain run from the kernel's g and idx
    il = idx.cpu().long()
    u = oracle.int4_gemv(cpu["up_qw"], cpu["up_sc"], x, rows=il)
    h = (g_cpu[il].float() * u.float()).to(torch.bfloat16)
    y_ref = oracle.gather_down_f32(cpu["down_t_qw"], cpu["down_t_sc"], h, rows=il)
    close(y, y_ref)


def test_mlp_decode_config0(dip, oracle, layer_c0):
    L = layer_c0
    y, g, idx = torch.ops.dip_b200.mlp_decode(L["gate_qw"], L["gate_sc"], L["up_qw"],
                                              L["up_sc"], L["down_t_qw"], L["down_t_sc"],
                                              L["x"], L["k"])
    torch.cuda.synchronize()
    _check_chain(oracle, L, y, g, idx)


def test_mlp_decode_deterministic(dip, layer_c0):
    L = layer_c0
    args = (L["gate_qw"], L["gate_sc"], L["up_qw"], L["up_sc"], L["down_t_qw"], L["down_t_sc"],
            L["x"], L["k"])
    a = torch.ops.dip_b200.mlp_decode(*args)
    b = torch.ops.dip_b200.mlp_decode(*args)
    for u, v in zip(a, b):
        assert torch.equal(u, v)


def test_mlp_decode_pdl_off_equal(dip, layer_c0):
    L = layer_c0
    args = (L["gate_qw"], L["gate_sc"], L["up_qw"], L["up_sc"], L["down_t_qw"], L["down_t_sc"],
            L["x"], L["k"])
    a = torch.ops.dip_b200.mlp_decode(*args)
    prev = torch.ops.dip_b200.set_pdl(0)
    try:
        b = torch.ops.dip_b200.mlp_decode(*args)
    finally:
        torch.ops.dip_b200.set_pdl(prev)
    for u, v in zip(a, b):
        assert torch.equal(u, v)


def test_c_abi_mlp_decode(dip, layer_c0):
    """The whole layer through the C entry point with raw device pointers."""
    from dip_b200 import _lib
    core = _lib.core()
    L = layer_c0
    H, I, k = 5120, 25600, L["k"]

    class Layer(ctypes.Structure):
        _fields_ = [("gate_qw", ctypes.c_void_p), ("gate_sc", ctypes.c_void_p),
                    ("up_qw", ctypes.c_void_p), ("up_sc", ctypes.c_void_p),
                    ("down_t_qw", ctypes.c_void_p), ("down_t_sc", ctypes.c_void_p),
                    ("hidden", ctypes.c_int64), ("inter", ctypes.c_int64)]

    lay = Layer(L["gate_qw"].data_ptr(), L["gate_sc"].data_ptr(), L["up_qw"].data_ptr(),
                L["up_sc"].data_ptr(), L["down_t_qw"].data_ptr(), L["down_t_sc"].data_ptr(),
                H, I)
    core.dip_mlp_workspace_bytes.restype = ctypes.c_size_t
    core.dip_mlp_workspace_bytes.argtypes = [ctypes.c_int64] * 3
    nws = core.dip_mlp_workspace_bytes(H, I, k)
    ws = torch.empty(nws, dtype=torch.uint8, device="cuda")
    y = torch.empty(H, dtype=torch.bfloat16, device="cuda")
    idx = torch.empty(k, dtype=torch.int32, device="cuda")
    vp = ctypes.c_void_p
    core.dip_mlp_decode.argtypes = [ctypes.POINTER(Layer), vp, ctypes.c_int64, vp,
                                    ctypes.c_size_t, vp, vp, vp, vp]
    stream = torch.cuda.current_stream().cuda_stream
    st = core.dip_mlp_decode(ctypes.byref(lay), L["x"].data_ptr(), k, ws.data_ptr(), nws,
                             y.data_ptr(), None, idx.data_ptr(), stream)
    assert st == 0
    assert core.dip_mlp_decode(ctypes.byref(lay), L["x"].data_ptr(), k, ws.data_ptr(), nws - 1,
                               y.data_ptr(), None, idx.data_ptr(), stream) == 3
    y2, g2, idx2 = torch.ops.dip_b200.mlp_decode(L["gate_qw"], L["gate_sc"], L["up_qw"],
                                                 L["up_sc"], L["down_t_qw"], L["down_t_sc"],
                                                 L["x"], k)
    assert torch.equal(idx, idx2) and torch.equal(y, y2)


# ---------------------------------------------------------------- modules
@pytest.fixture(scope="module")
def small_layer(oracle):
    return oracle.make_layer_cpu(1024, 3072, seed=9)


def test_streaming_dip_module(dip, oracle, small_layer, dev):
    L = small_layer
    k = int(round(3072 * 0.6))
    shared = dip.SharedBuffers(k, 512, 8, 1024, 8, dev)
    m = dip.StreamingDIPMlp(L["gate_qw"], L["gate_sc"], L["up_qw"], L["up_sc"], L["down_qw"],
                            L["down_sc"], shared, 0.6, dev)
    # the module's own transpose equals the reference's
    assert torch.equal(m.down_t_qw.cpu(), L["down_t_qw"])
    x = torch.randn(1, 1, 1024, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    y = m(x.to(dev))
    assert y.shape == (1, 1, 1024) and y.dtype == torch.bfloat16
    r = oracle.dip_mlp_decode(x.reshape(-1), L["gate_qw"], L["gate_sc"], L["up_qw"],
                              L["up_sc"], L["down_t_qw"], L["down_t_sc"], k)
    close(m.last_g, r["g"])
    assert torch.equal(m.last_idx.cpu(), oracle.topk_select(m.last_g.cpu(), k))
    il = m.last_idx.cpu().long()
    u = oracle.int4_gemv(L["up_qw"], L["up_sc"], x.reshape(-1), rows=il)
    h = (m.last_g.cpu()[il].float() * u.float()).to(torch.bfloat16)
    close(y.reshape(-1), oracle.gather_down_f32(L["down_t_qw"], L["down_t_sc"], h, rows=il))
    # prefill path (seq > 1) runs the dense MLP
    xp = torch.randn(1, 3, 1024, device=dev, dtype=torch.bfloat16)
    assert m(xp).shape == (1, 3, 1024)


def test_streaming_dip_batch_rows_independent(dip, small_layer, dev):
    L = small_layer
    k = int(round(3072 * 0.6))
    shared = dip.SharedBuffers(k, 512, 8, 1024, 8, dev)
    m = dip.StreamingDIPMlp(L["gate_qw"], L["gate_sc"], L["up_qw"], L["up_sc"], L["down_qw"],
                            L["down_sc"], shared, 0.6, dev)
    x = torch.randn(3, 1, 1024, device=dev, dtype=torch.bfloat16)
    yb = m(x)
    for b in range(3):
        assert torch.equal(yb[b], m(x[b:b + 1])[0])


def test_ca_dip_module(dip, oracle, small_layer, dev):
    L = small_layer
    inter = 3072
    buf = dip.CABuffers(int(round(inter * 0.6)), 512, 8, 1024, 8, dev)
    m = dip.CADIPMlp(L["gate_qw"], L["gate_sc"], L["up_qw"], L["up_sc"], L["down_qw"],
                     L["down_sc"], buf, 0.6, 0.3, dev)
    gen = torch.Generator().manual_seed(2)
    calib = torch.randn(1, 32, 1024, generator=gen).to(torch.bfloat16)
    counts = dip.calibrate_cache_inputs([m], calib.to(dev))
    # hot set = oracle ordering of the same counts
    hot = oracle.cache_hot_order(counts[0].cpu())
    ids, id2slot = oracle.set_cache_ids(hot, m.cache_n, inter)
    assert torch.equal(m.cache_ids.cpu(), ids) and torch.equal(m.id2slot.cpu(), id2slot)
    x = torch.randn(1, 1, 1024, generator=gen).to(torch.bfloat16)
    y = m(x.to(dev))
    comb, src, row, n_hit = m.last_split
    rc, rs, rr, rn = oracle.ca_split(m.last_idx.cpu(), id2slot)
    assert torch.equal(comb.cpu(), rc) and torch.equal(src.cpu(), rs)
    assert torch.equal(row.cpu(), rr) and n_hit.item() == rn
    assert 0 < rn < m.k
    # g within tolerance, idx exact given the module's g, y against the
    # oracle chain run from the module's own g over the combined order
    g = m.last_g.cpu()
    close(g, oracle.silu_bf16(oracle.int4_gemv(L["gate_qw"], L["gate_sc"], x.reshape(-1))))
    assert torch.equal(m.last_idx.cpu(), oracle.topk_select(g, m.k))
    cl = comb.cpu().long()
    u = oracle.int4_gemv(L["up_qw"], L["up_sc"], x.reshape(-1), rows=cl)
    h = (g[cl].float() * u.float()).to(torch.bfloat16)
    close(y.reshape(-1), oracle.gather_down_f32(L["down_t_qw"], L["down_t_sc"], h, rows=cl))
    # CA output equals the streaming module's up to summation order
    shared = dip.SharedBuffers(m.k, 512, 8, 1024, 8, dev)
    s = dip.StreamingDIPMlp(L["gate_qw"], L["gate_sc"], L["up_qw"], L["up_sc"], L["down_qw"],
                            L["down_sc"], shared, 0.6, dev)
    close(y, s(x.to(dev)))


def test_quantlinear(dip, oracle, dev):
    gen = torch.Generator().manual_seed(4)
    w = (torch.randn(256, 512, generator=gen) * 0.02).to(torch.bfloat16)
    qw, sc = oracle.quantize_int4_g128(w)
    ql = dip.QuantLinear(512, 256).to(dev)
    ql.qweight.copy_(qw)
    ql.scales.copy_(sc)
    x = torch.randn(1, 1, 512, generator=gen).to(torch.bfloat16)
    close(ql(x.to(dev)).reshape(-1), oracle.int4_gemv_f32(qw, sc, x))
    xs = torch.randn(4, 512, generator=gen).to(torch.bfloat16)
    ref = xs.float() @ oracle.dequantize(qw, sc).float().t()
    close(ql(xs.to(dev)), ref)


# ------------------------------------------- drop-in modules on the fast paths
@pytest.fixture(scope="module")
def fused_shape_layer(oracle):
    """hidden 2560, inter 8192: a shape the one-launch fused layer takes."""
    return oracle.make_layer_cpu(2560, 8192, seed=21)


def test_modules_decode_on_fused_layer(dip, oracle, fused_shape_layer, dev):
    L = fused_shape_layer
    k = int(round(8192 * 0.6))
    shared = dip.SharedBuffers(k, 1280, 20, 2560, 20, dev)
    m = dip.StreamingDIPMlp(L["gate_qw"], L["gate_sc"], L["up_qw"], L["up_sc"], L["down_qw"],
                            L["down_sc"], shared, 0.6, dev)
    assert m._fused
    gen = torch.Generator().manual_seed(3)
    for t in range(2):  # the module-owned workspace is reused
        x = torch.randn(1, 1, 2560, generator=gen).to(torch.bfloat16)
        y = m(x.to(dev))
        g = m.last_g.cpu()
        close(g, oracle.silu_bf16(oracle.int4_gemv(L["gate_qw"], L["gate_sc"], x.reshape(-1))))
        assert torch.equal(m.last_idx.cpu(), oracle.topk_select(g, k))
        il = m.last_idx.cpu().long()
        u = oracle.int4_gemv(L["up_qw"], L["up_sc"], x.reshape(-1), rows=il)
        h = (g[il].float() * u.float()).to(torch.bfloat16)
        close(y.reshape(-1), oracle.gather_down_f32(L["down_t_qw"], L["down_t_sc"], h, rows=il))
    # cache-aware module on the same weights: same g / idx, split exact
    buf = dip.CABuffers(k, 1280, 20, 2560, 20, dev)
    c = dip.CADIPMlp(L["gate_qw"], L["gate_sc"], L["up_qw"], L["up_sc"], L["down_qw"],
                     L["down_sc"], buf, 0.6, 0.3, dev)
    calib = torch.randn(1, 16, 2560, generator=gen).to(torch.bfloat16)
    dip.calibrate_cache_inputs([c], calib.to(dev))
    assert c._fused
    yc = c(x.to(dev))
    assert torch.equal(c.last_idx, m.last_idx) and torch.equal(c.last_g, m.last_g)
    comb, src, row, n_hit = c.last_split
    rc, rs, rr, rn = oracle.ca_split(c.last_idx.cpu(), c.id2slot.cpu())
    assert torch.equal(comb.cpu(), rc) and torch.equal(src.cpu(), rs)
    assert torch.equal(row.cpu(), rr) and int(n_hit) == rn and 0 < rn < k
    close(yc, y)


def test_dense_prefill_on_tensor_cores(dip, oracle, fused_shape_layer, dev):
    """_dense (dip_stream_predispatch.py:206-215) for a 5-token prefill: the
    tcgen05 GEMMs against the reference's dequantize + F.linear math in fp32."""
    L = fused_shape_layer
    k = int(round(8192 * 0.6))
    shared = dip.SharedBuffers(k, 1280, 20, 2560, 20, dev)
    m = dip.StreamingDIPMlp(L["gate_qw"], L["gate_sc"], L["up_qw"], L["up_sc"], L["down_qw"],
                            L["down_sc"], shared, 0.6, dev)
    x = torch.randn(1, 5, 2560, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    y = m(x.to(dev))
    assert y.shape == (1, 5, 2560)
    xf = x.reshape(5, 2560).float()
    g = torch.nn.functional.silu(
        (xf @ oracle.dequantize(L["gate_qw"], L["gate_sc"]).float().t()).to(torch.bfloat16))
    u = (xf @ oracle.dequantize(L["up_qw"], L["up_sc"]).float().t()).to(torch.bfloat16)
    h = (g * u).to(torch.bfloat16)
    ref = h.float() @ oracle.dequantize(L["down_t_qw"], L["down_t_sc"]).float()
    close(y.reshape(5, 2560), ref)
