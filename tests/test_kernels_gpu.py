"""Parity of the sm_100a kernels with the CPU oracle (GPU).

Tolerances: integer / index / byte outputs are compared bit for bit.  Float
outputs follow the path's contract — within 1e-2 relative + 2e-3 absolute of
the fp32-accumulated value, elementwise — and additionally the reference's own
kernel-test criterion max|err| / max|ref| < 2 % (kernels/*/test_*.py).
The shapes and seeds of the reference's kernel tests are reproduced.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 2e-3


def close(out, ref):
    out = out.float().cpu()
    ref = ref.float().cpu()
    err = (out - ref).abs()
    bad = err > ATOL + RTOL * ref.abs()
    rel = err.max().item() / (ref.abs().max().item() + 1e-6)
    assert not bad.any(), f"{int(bad.sum())} elements out of tolerance, max err {err.max():.3e}"
    assert rel < 0.02


def rand_packed(rows, cols, gen, oracle):
    q = torch.randint(-8, 8, (rows, cols), dtype=torch.int8, generator=gen)
    sc = (torch.rand(rows, cols // 128, generator=gen) * 0.01 + 0.001).to(torch.bfloat16)
    return oracle.pack_int4(q), sc


# ---------------------------------------------------------------- format
def test_quantize_bit_exact(dip, oracle, dev):
    gen = torch.Generator().manual_seed(11)
    w = (torch.randn(1024, 5120, generator=gen) * 0.02).to(torch.bfloat16)
    w[3, :128] = 0
    w[5] *= 1000
    qw, sc = torch.ops.dip_b200.quantize_int4(w.to(dev))
    rq, rs = oracle.quantize_int4_g128(w)
    assert torch.equal(qw.cpu(), rq)
    assert torch.equal(sc.cpu().view(torch.int16), rs.view(torch.int16))


def test_dequantize_bit_exact(dip, oracle, dev):
    gen = torch.Generator().manual_seed(12)
    qw, sc = rand_packed(512, 1024, gen, oracle)
    d = torch.ops.dip_b200.dequantize_int4(qw.to(dev), sc.to(dev))
    assert torch.equal(d.cpu().view(torch.int16), oracle.dequantize(qw, sc).view(torch.int16))


@pytest.mark.parametrize("out_f,inter", [(256, 384), (5120, 1024)])
def test_transpose_down_bit_exact(dip, oracle, dev, out_f, inter):
    gen = torch.Generator().manual_seed(13)
    w = (torch.randn(out_f, inter, generator=gen) * 0.02).to(torch.bfloat16)
    dq, ds = oracle.quantize_int4_g128(w)
    tq, ts = torch.ops.dip_b200.transpose_down_int4(dq.to(dev), ds.to(dev))
    rq, rs = oracle.transpose_down_to_int4(dq, ds)
    assert torch.equal(tq.cpu(), rq)
    assert torch.equal(ts.cpu().view(torch.int16), rs.view(torch.int16))


def test_format_golden_on_gpu(dip, dev):
    from pathlib import Path
    g = torch.load(Path(__file__).with_name("golden") / "format_golden.pt")
    qw, sc = torch.ops.dip_b200.quantize_int4(g["gate"]["w"].to(dev))
    assert torch.equal(qw.cpu(), g["gate"]["qweight"])
    assert torch.equal(sc.cpu().view(torch.int16), g["gate"]["scales"].view(torch.int16))
    d = torch.ops.dip_b200.dequantize_int4(qw, sc)
    assert torch.equal(d.cpu().view(torch.int16), g["gate"]["dequant"].view(torch.int16))
    tq, ts = torch.ops.dip_b200.transpose_down_int4(g["down"]["qweight"].to(dev),
                                                     g["down"]["scales"].to(dev))
    assert torch.equal(tq.cpu(), g["down"]["down_t_qw"])
    assert torch.equal(ts.cpu().view(torch.int16), g["down"]["down_t_sc"].view(torch.int16))


# ---------------------------------------------------------------- GEMV family
def test_int4_gemv_reference_test_shape(dip, oracle, dev):
    """kernels/int4_gemv/test_int4_gemv.py:32-55: seed 0, out=4096, in=5120."""
    gen = torch.Generator().manual_seed(0)
    qw, sc = rand_packed(4096, 5120, gen, oracle)
    x = torch.randn(5120, generator=gen).to(torch.bfloat16)
    y = torch.ops.int4_ops.int4_gemv(qw.to(dev), sc.to(dev), x.to(dev))
    close(y, oracle.int4_gemv_f32(qw, sc, x))


@pytest.mark.parametrize("rows,cols", [(1, 128), (17, 256), (100, 640), (25600, 5120)])
def test_gate_silu(dip, oracle, dev, rows, cols):
    gen = torch.Generator().manual_seed(rows)
    w = (torch.randn(rows, cols, generator=gen) * 0.02).to(torch.bfloat16)
    qw, sc = oracle.quantize_int4_g128(w)
    x = torch.randn(cols, generator=gen).to(torch.bfloat16)
    g = torch.ops.dip_b200.gate_silu(qw.to(dev), sc.to(dev), x.to(dev)).cpu()
    pre = oracle.int4_gemv_f32(qw, sc, x)
    close(g, oracle.silu_bf16(pre.to(torch.bfloat16)))
    plain = torch.ops.int4_ops.int4_gemv(qw.to(dev), sc.to(dev), x.to(dev)).cpu()
    close(plain, pre)


def test_int4_gather_gemv_reference_test_shape(dip, oracle, dev):
    """kernels/int4_gather/test_gather.py:28-55: k = 0.6*4096 sorted rows."""
    gen = torch.Generator().manual_seed(0)
    qw, sc = rand_packed(4096, 5120, gen, oracle)
    x = torch.randn(5120, generator=gen).to(torch.bfloat16)
    idx = torch.randperm(4096, generator=gen)[: int(0.6 * 4096)].sort().values.to(torch.int32)
    y = torch.ops.int4_gather_ops.int4_gather_gemv(qw.to(dev), sc.to(dev), x.to(dev),
                                                   idx.to(dev))
    close(y, oracle.int4_gemv_f32(qw, sc, x, rows=idx.long()))


def test_gather_up_h(dip, oracle, dev):
    gen = torch.Generator().manual_seed(21)
    qw, sc = rand_packed(2048, 1024, gen, oracle)
    x = torch.randn(1024, generator=gen).to(torch.bfloat16)
    g = torch.randn(2048, generator=gen).to(torch.bfloat16)
    idx = torch.randperm(2048, generator=gen)[:1229].to(torch.int32)
    h = torch.ops.dip_b200.gather_up_h(qw.to(dev), sc.to(dev), x.to(dev), g.to(dev),
                                       idx.to(dev)).cpu()
    u = torch.ops.int4_gather_ops.int4_gather_gemv(qw.to(dev), sc.to(dev), x.to(dev),
                                                   idx.to(dev)).cpu()
    # h is exactly bf16(g[idx] * u) of the kernel's own u
    ref_h = (g[idx.long()].float() * u.float()).to(torch.bfloat16)
    assert torch.equal(h.view(torch.int16), ref_h.view(torch.int16))
    close(u, oracle.int4_gemv_f32(qw, sc, x, rows=idx.long()))


def test_ca_fused_gemv_reference_test_shape(dip, oracle, dev):
    """kernels/ca_fused/test_ca_fused.py:26-79: in=5120, k=15360, cache_n=7680,
    n_hit=5855; hits at cache slots 0..n_hit-1, misses at staging rows."""
    gen = torch.Generator().manual_seed(0)
    in_f, k, cache_n, n_hit = 5120, 15360, 7680, 5855
    q_full = torch.randint(-8, 8, (k, in_f), dtype=torch.int8, generator=gen)
    sc_full = (torch.rand(k, in_f // 128, generator=gen) * 0.01 + 0.001).to(torch.bfloat16)
    x = torch.randn(in_f, generator=gen).to(torch.bfloat16)
    packed = oracle.pack_int4(q_full)
    res_q = torch.zeros(cache_n, in_f // 2, dtype=torch.int8)
    res_s = torch.zeros(cache_n, in_f // 128, dtype=torch.bfloat16)
    res_q[:n_hit], res_s[:n_hit] = packed[:n_hit], sc_full[:n_hit]
    str_q = torch.zeros(k, in_f // 2, dtype=torch.int8)
    str_s = torch.zeros(k, in_f // 128, dtype=torch.bfloat16)
    str_q[: k - n_hit], str_s[: k - n_hit] = packed[n_hit:], sc_full[n_hit:]
    src = torch.cat([torch.zeros(n_hit), torch.ones(k - n_hit)]).to(torch.int32)
    row = torch.cat([torch.arange(n_hit), torch.arange(k - n_hit)]).to(torch.int32)
    y = torch.ops.ca_fused_ops.ca_fused_gemv(res_q.to(dev), res_s.to(dev), str_q.to(dev),
                                             str_s.to(dev), x.to(dev), src.to(dev), row.to(dev))
    close(y, oracle.int4_gemv_f32(packed, sc_full, x))


# ---------------------------------------------------------------- down
def test_int4_gather_down_reference_test_shape(dip, oracle, dev):
    """kernels/int4_down/test_down.py:30-54: k=15360, out=5120, staged rows."""
    gen = torch.Generator().manual_seed(0)
    dtw, sc = rand_packed(15360, 5120, gen, oracle)
    h = torch.randn(15360, generator=gen).to(torch.bfloat16)
    y = torch.ops.int4_down_ops.int4_gather_down(dtw.to(dev), sc.to(dev), h.to(dev))
    close(y, oracle.gather_down_f32(dtw, sc, h))


@pytest.mark.parametrize("k", [1, 5, 147, 149, 1000])
def test_gather_down_idx(dip, oracle, dev, k):
    gen = torch.Generator().manual_seed(k)
    dtw, sc = rand_packed(2000, 1024, gen, oracle)
    h = torch.randn(k, generator=gen).to(torch.bfloat16)
    idx = torch.randperm(2000, generator=gen)[:k].to(torch.int32)
    y = torch.ops.dip_b200.gather_down_idx(dtw.to(dev), sc.to(dev), h.to(dev), idx.to(dev))
    close(y, oracle.gather_down_f32(dtw, sc, h, rows=idx.long()))


# ---------------------------------------------------------------- top-k
def _topk_case(name, gen):
    n, k = 25600, 15360
    if name == "normal":
        s = torch.randn(n, generator=gen)
    elif name == "ties":      # few distinct values -> large tie bands
        s = torch.randint(-6, 7, (n,), generator=gen).float() / 4
    elif name == "zeros":     # fewer non-zeros than k -> zero padding
        s = torch.randn(n, generator=gen)
        s[torch.rand(n, generator=gen) < 0.6] = 0
    elif name == "all_equal":
        s = torch.full((n,), -0.75)
    elif name == "nan_inf":
        s = torch.randn(n, generator=gen)
        s[::97] = float("nan")
        s[5] = float("inf")
        s[6] = float("-inf")
    elif name == "wide_range":  # k-th value far below max * 2^-25
        s = torch.randn(n, generator=gen) * 1e-9
        s[:100] = 1e4
    elif name == "silu_like":
        s = torch.nn.functional.silu(torch.randn(n, generator=gen) * 1.4)
    else:
        raise ValueError(name)
    return s.to(torch.bfloat16), k


@pytest.mark.parametrize("name", ["normal", "ties", "zeros", "all_equal", "nan_inf",
                                  "wide_range", "silu_like"])
def test_topk_exact(dip, oracle, dev, name):
    s, k = _topk_case(name, torch.Generator().manual_seed(7))
    idx = torch.ops.topk_ops.topk_select(s.to(dev), k).cpu()
    assert torch.equal(idx, oracle.topk_select(s, k))


@pytest.mark.parametrize("n,k", [(1, 1), (2, 1), (7, 3), (1000, 1), (1000, 999),
                                 (1000, 1000), (1000, 1500), (4097, 2458), (98304, 40000)])
def test_topk_sizes(dip, oracle, dev, n, k):
    s = torch.randn(n, generator=torch.Generator().manual_seed(n + k)).to(torch.bfloat16)
    idx = torch.ops.topk_ops.topk_select(s.to(dev), k).cpu()
    assert torch.equal(idx, oracle.topk_select(s, k))


def test_topk_reference_test_overlap(dip, dev):
    """kernels/topk_select/test_topk.py:21-38 criterion: > 98 % set overlap
    with torch.topk at I=25600, k=15360, s ~ N(0,1) bf16."""
    torch.manual_seed(0)
    s = torch.randn(25600, dtype=torch.bfloat16, device=dev)
    a = set(torch.ops.topk_ops.topk_select(s, 15360).tolist())
    b = set(s.abs().topk(15360).indices.tolist())
    assert len(a & b) / 15360 > 0.98


def test_topk_batched(dip, oracle, dev):
    gen = torch.Generator().manual_seed(3)
    s = torch.randn(8, 25600, generator=gen).to(torch.bfloat16)
    idx = torch.ops.dip_b200.topk_select_batched(s.to(dev), 15360).cpu()
    for b in range(8):
        assert torch.equal(idx[b], oracle.topk_select(s[b], 15360))


# ---------------------------------------------------------------- cache split
def test_ca_split_exact(dip, oracle, dev):
    gen = torch.Generator().manual_seed(5)
    inter, k, cache_n = 25600, 15360, 7680
    idx = torch.randperm(inter, generator=gen)[:k].sort().values.to(torch.int32)
    hot = torch.randperm(inter, generator=gen)
    _, id2slot = oracle.set_cache_ids(hot, cache_n, inter)
    comb, src, row, nh = torch.ops.dip_b200.ca_split(idx.to(dev), id2slot.to(dev))
    rc, rs, rr, rn = oracle.ca_split(idx, id2slot)
    assert torch.equal(comb.cpu(), rc) and torch.equal(src.cpu(), rs)
    assert torch.equal(row.cpu(), rr) and nh.item() == rn


# ---------------------------------------------------------------- GEMV variants
@pytest.mark.parametrize("in_f", [1024, 2048, 5120])
@pytest.mark.parametrize("rows", [7, 16, 300, 4097])
def test_ring_and_simple_gemv_agree(dip, oracle, dev, in_f, rows):
    """The persistent bulk-copy ring kernel and the simple kernel give the same
    values (up to fp32 summation order) in every row mode and epilogue, and
    both match the oracle."""
    gen = torch.Generator().manual_seed(rows + in_f)
    qw, sc = rand_packed(rows, in_f, gen, oracle)
    x = torch.randn(in_f, generator=gen).to(torch.bfloat16)
    g = torch.randn(rows, generator=gen).to(torch.bfloat16)
    k = max(1, rows // 2)
    idx = torch.randperm(rows, generator=gen)[:k].to(torch.int32)
    d = [t.to(dev) for t in (qw, sc, x, g, idx)]
    outs = []
    for simple in (0, 1):
        prev = torch.ops.dip_b200.set_gemv_variant(simple)
        try:
            outs.append((torch.ops.dip_b200.gate_silu(d[0], d[1], d[2]).cpu(),
                         torch.ops.int4_gather_ops.int4_gather_gemv(d[0], d[1], d[2], d[4]).cpu(),
                         torch.ops.dip_b200.gather_up_h(d[0], d[1], d[2], d[3], d[4]).cpu()))
        finally:
            torch.ops.dip_b200.set_gemv_variant(prev)
    torch.cuda.synchronize()
    assert torch.ops.dip_b200.take_device_error() == 0
    ref_full = oracle.int4_gemv_f32(qw, sc, x)
    for a, b in zip(*outs):
        close(a, b)
    close(outs[0][0], oracle.silu_bf16(ref_full.to(torch.bfloat16)))
    close(outs[0][1], ref_full[idx.long()])


@pytest.mark.parametrize("out_f", [1024, 5120])
@pytest.mark.parametrize("k", [1, 15, 16, 17, 300, 15360])
def test_down_variants_agree(dip, oracle, dev, out_f, k):
    """Tensor-core (ring) and CUDA-core down projections agree and match the
    oracle, with idx gather, the staged (identity) layout and odd k."""
    gen = torch.Generator().manual_seed(out_f + k)
    n = max(k, 64)
    dtw, sc = rand_packed(n, out_f, gen, oracle)
    h = torch.randn(k, generator=gen).to(torch.bfloat16)
    idx = torch.randperm(n, generator=gen)[:k].to(torch.int32)
    ys = []
    for simple in (0, 1):
        prev = torch.ops.dip_b200.set_gemv_variant(simple)
        try:
            ys.append(torch.ops.dip_b200.gather_down_idx(dtw.to(dev), sc.to(dev), h.to(dev),
                                                         idx.to(dev)).cpu())
        finally:
            torch.ops.dip_b200.set_gemv_variant(prev)
    assert torch.ops.dip_b200.take_device_error() == 0
    ref = oracle.gather_down_f32(dtw, sc, h, rows=idx.long())
    close(ys[0], ref)
    close(ys[1], ref)
