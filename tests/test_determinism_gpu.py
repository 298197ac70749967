"""Run-to-run determinism of the whole 64-layer stack (GPU), the synthetic
stand-in for the reference's two-greedy-runs text check
(tests/test_ca_determinism.py:32-48, which needs the Qwen3 checkpoint): two
separate runs of the same tokens through freshly built stacks give bitwise
equal indices and outputs at every layer, on the one-launch streaming layer
and on the cache-aware layer (calibrated on the same tokens both times)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _run(mode, lognormal):
    from dip_b200.stack import StackConfig, DipStack, token_inputs
    dev = torch.device("cuda", 0)
    cfg = StackConfig(n_layers=64, seed=5, gate_lognormal=lognormal)
    st = DipStack(cfg, dev, mode=mode)
    if mode == "ca":
        xc, rc = token_inputs(cfg, 8, seed=77, device=dev)
        st.calibrate_ca(xc, rc)
    x0, r = token_inputs(cfg, 3, seed=78, device=dev)
    out = []
    for t in range(3):
        st.step(x0[t], r[t], record=True)
        out.append(([i.clone() for i in st.last_idx], [y.clone() for y in st.last_y]))
    torch.cuda.synchronize()
    assert st.take_device_error() == 0
    hot = [c["cache_ids"].clone() for c in st.ca] if st.ca else None
    del st
    torch.cuda.empty_cache()
    return out, hot


@pytest.mark.parametrize("mode,lognormal", [("fused", False), ("ca", True)])
def test_stack_two_runs_bitwise_equal(dip, mode, lognormal):
    a, hot_a = _run(mode, lognormal)
    b, hot_b = _run(mode, lognormal)
    if hot_a is not None:
        assert all(torch.equal(p, q) for p, q in zip(hot_a, hot_b)), "hot sets differ"
    for t, ((ia, ya), (ib, yb)) in enumerate(zip(a, b)):
        for l in range(len(ia)):
            assert torch.equal(ia[l], ib[l]), f"token {t} layer {l}: indices differ"
            assert torch.equal(ya[l], yb[l]), f"token {t} layer {l}: y differs"
