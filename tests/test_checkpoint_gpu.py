"""The int4 checkpoint loader on the GPU: a 2-layer checkpoint in the
reference's format (model_int4.safetensors + quant_config.json, written by
tests/ckpt_util.py, whose output equals scripts/quantize.py's byte for byte,
tests/test_checkpoint_cpu.py) loads into a DipStack; the down projection is
transposed on the GPU exactly as _transpose_down_to_int4 does
(dip_stream_predispatch.py:100-120), and a decode token through the loaded
layers matches the oracle stage by stage."""
import pytest
import torch

from ckpt_util import bf16_state, write_int4_checkpoint

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 2e-3


def close(out, ref):
    out, ref = out.float().cpu(), ref.float().cpu()
    err = (out - ref).abs()
    bad = err > ATOL + RTOL * ref.abs()
    assert not bad.any(), f"{int(bad.sum())} out of tolerance, max err {err.max():.3e}"


def test_checkpoint_loads_and_decodes(dip, oracle, tmp_path):
    from dip_b200.stack import DipStack
    H, I = 2560, 8192
    sd = bf16_state(n_layers=2, hidden=H, inter=I, seed=7)
    write_int4_checkpoint(tmp_path, sd)
    dev = torch.device("cuda", 0)
    st = DipStack.from_checkpoint(tmp_path, dev)
    assert st.cfg.n_layers == 2 and st.cfg.hidden == H and st.cfg.inter == I
    k = st.cfg.k
    x = torch.randn(H, generator=torch.Generator().manual_seed(8)).to(torch.bfloat16)
    for l, L in enumerate(st.layers):
        b = f"model.layers.{l}.mlp"
        gq, gs = oracle.quantize_int4_g128(sd[f"{b}.gate_proj.weight"])
        uq, us = oracle.quantize_int4_g128(sd[f"{b}.up_proj.weight"])
        dq, ds = oracle.quantize_int4_g128(sd[f"{b}.down_proj.weight"])
        tq, ts = oracle.transpose_down_to_int4(dq, ds)
        assert torch.equal(L["gate_qw"].cpu(), gq) and torch.equal(L["gate_sc"].cpu(), gs)
        assert torch.equal(L["up_qw"].cpu(), uq) and torch.equal(L["up_sc"].cpu(), us)
        assert torch.equal(L["down_t_qw"].cpu(), tq) and torch.equal(L["down_t_sc"].cpu(), ts)
    # one decode token through layer 0 of the loaded stack, stage by stage
    L = st.layers[0]
    ws = torch.zeros(torch.ops.dip_b200.mlp_fused_workspace_bytes(H, I, k), dtype=torch.uint8,
                     device=dev)
    h = torch.zeros(I, dtype=torch.bfloat16, device=dev)
    y, g, idx = torch.ops.dip_b200.mlp_decode_fused(L["gate_qw"], L["gate_sc"], L["up_qw"],
                                                    L["up_sc"], L["down_t_qw"], L["down_t_sc"],
                                                    x.to(dev), None, 1e-6, k, ws, h)
    torch.cuda.synchronize()
    c = {n: t.cpu() for n, t in L.items()}
    close(g, oracle.silu_bf16(oracle.int4_gemv(c["gate_qw"], c["gate_sc"], x)))
    gc = g.cpu()
    assert torch.equal(idx.cpu(), oracle.topk_select(gc, k))
    il = idx.cpu().long()
    u = oracle.int4_gemv(c["up_qw"], c["up_sc"], x, rows=il)
    close(h.cpu()[il], (gc[il].float() * u.float()).to(torch.bfloat16))
    close(y, oracle.gather_down_f32(c["down_t_qw"], c["down_t_sc"], h.cpu()[il], rows=il))
    # and the whole 2-layer stack decodes a token
    r = torch.randn(2, H, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16)
    out = st.decode(x, r)
    assert out.shape == (H,) and bool(torch.isfinite(out.float()).all())
    assert st.take_device_error() == 0
