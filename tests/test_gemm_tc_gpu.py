"""tcgen05 int4 GEMMs (GPU) against the reference's pure-PyTorch math: every
weight dequantised to bf16(q * s) (qlinear.py:52-64), products accumulated in
fp32, outputs rounded to bf16 where the reference's tensors are bf16.  Paths
are checked elementwise within 1e-2 relative + 2e-3 absolute (plus 4e-4 of the
largest value for the long down sums, whose fp32 summation order differs)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 2e-3


def close(out, ref, scale_tol=0.0):
    out, ref = out.float().cpu(), ref.float().cpu()
    err = (out - ref).abs()
    tol = ATOL + RTOL * ref.abs() + scale_tol * ref.abs().max()
    bad = err > tol
    if bad.any():
        i = int((err - tol).argmax())
        raise AssertionError(f"{int(bad.sum())} of {out.numel()} out of tolerance, max err "
                             f"{err.max():.3e}; worst at {i}: got {float(out.flatten()[i]):.6f}, "
                             f"want {float(ref.flatten()[i]):.6f}")


def _packed(rows, cols, seed, std=0.02):
    gen = torch.Generator().manual_seed(seed)
    w = (torch.randn(rows, cols, generator=gen) * std).to(torch.bfloat16).cuda()
    return torch.ops.dip_b200.quantize_int4(w)


@pytest.mark.parametrize("rows,K,B", [(256, 256, 16), (384, 512, 5), (256, 1024, 33),
                                      (512, 5120, 64), (640, 2560, 100), (25600, 5120, 64)])
def test_gemm_tc_plain_and_silu(dip, oracle, rows, K, B):
    qw, sc = _packed(rows, K, rows + K + B)
    x = torch.randn(B, K, generator=torch.Generator().manual_seed(B)).to(torch.bfloat16).cuda()
    ref = (x.float().cpu() @ oracle.dequantize(qw.cpu(), sc.cpu()).float().T).to(torch.bfloat16)
    out = torch.ops.dip_b200.gemm_tc(qw, sc, x, 0)
    torch.cuda.synchronize()
    assert torch.ops.dip_b200.take_device_error() == 0
    close(out, ref)
    # SiLU of the same accumulator: compared against SiLU of the plain output, since
    # a one-ulp difference in bf16(x W) (fp32 summation order) can move the
    # rounded SiLU by two ulps
    out1 = torch.ops.dip_b200.gemm_tc(qw, sc, x, 1)
    close(out1, oracle.silu_bf16(out.cpu()))


def test_gemm_tc_up_product(dip, oracle):
    rows, K, B = 384, 1024, 20
    qw, sc = _packed(rows, K, 5)
    gen = torch.Generator().manual_seed(6)
    x = torch.randn(B, K, generator=gen).to(torch.bfloat16).cuda()
    g = torch.randn(B, rows, generator=gen).to(torch.bfloat16).cuda()
    cnt = torch.randint(0, 3, (B, rows), generator=gen, dtype=torch.int32).cuda()
    u = (x.float().cpu() @ oracle.dequantize(qw.cpu(), sc.cpu()).float().T).to(torch.bfloat16)
    ref = (g.cpu().float() * u.float()).to(torch.bfloat16).float() * cnt.cpu().float()
    out = torch.ops.dip_b200.gemm_tc(qw, sc, x, 2, g, cnt)
    close(out, ref.to(torch.bfloat16))
    assert bool((out.cpu()[cnt.cpu() == 0] == 0).all())


@pytest.mark.parametrize("inter,H,B", [(1024, 512, 16), (4096, 1024, 7), (25600, 5120, 64)])
def test_down_tc(dip, oracle, inter, H, B):
    dq, ds = _packed(H, inter, inter + B)
    tq, ts = torch.ops.dip_b200.transpose_down_int4(dq, ds)
    gen = torch.Generator().manual_seed(B)
    h = torch.randn(B, inter, generator=gen) * 0.5
    h[torch.rand(B, inter, generator=gen) < 0.4] = 0.0
    h = h.to(torch.bfloat16).cuda()
    y = torch.ops.dip_b200.down_tc(tq, ts, h)
    torch.cuda.synchronize()
    assert torch.ops.dip_b200.take_device_error() == 0
    ref = h.float().cpu() @ oracle.dequantize(tq.cpu(), ts.cpu()).float()
    close(y, ref)
    assert torch.equal(y, torch.ops.dip_b200.down_tc(tq, ts, h))  # deterministic


def test_select_count(dip):
    idx = torch.tensor([[3, 1, 0, 0, 0], [4, 2, 1, 3, 0]], dtype=torch.int32).cuda()
    cnt = torch.ops.dip_b200.select_count(idx, 6).cpu()
    assert cnt.tolist() == [[3, 1, 0, 1, 0, 0], [1, 1, 1, 1, 1, 0]]
