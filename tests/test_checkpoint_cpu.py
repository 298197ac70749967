"""The int4 checkpoint loader (dip_b200.checkpoint) on the CPU.

The reference's own converter, scripts/quantize.py, is run on a tiny
synthetic bf16 model when the reference checkout is present (test
infrastructure only): the loader must return its MLP tensors byte for byte,
and the test-side writer (tests/ckpt_util.py, used by the GPU test) must
produce the same tensors.  quant_config.json is validated field by field.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from ckpt_util import bf16_state, make_bf16_model, write_int4_checkpoint

REF = Path(os.environ.get("DIP_REFERENCE", "/root/reference"))


def _ckpt():
    from dip_b200 import checkpoint
    return checkpoint


@pytest.mark.skipif(not (REF / "scripts" / "quantize.py").exists(),
                    reason="reference checkout not present")
def test_loader_reads_reference_converter_output(tmp_path):
    ck = _ckpt()
    sd = bf16_state(n_layers=2, hidden=256, inter=512, seed=1)
    make_bf16_model(tmp_path / "bf16", sd)
    r = subprocess.run([sys.executable, str(REF / "scripts" / "quantize.py"), "--model_dir",
                        str(tmp_path / "bf16"), "--out_dir", str(tmp_path / "int4")],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    ck.read_quant_config(tmp_path / "int4")
    assert ck.count_mlp_layers(tmp_path / "int4") == 2
    write_int4_checkpoint(tmp_path / "ours", sd)
    from safetensors.torch import load_file
    ref_all = load_file(str(tmp_path / "int4" / "model_int4.safetensors"))
    ours_all = load_file(str(tmp_path / "ours" / "model_int4.safetensors"))
    assert set(ref_all) == set(ours_all)
    for k in ref_all:  # the test-side writer equals the reference converter
        assert torch.equal(ref_all[k].view(torch.uint8) if ref_all[k].dtype == torch.int8
                           else ref_all[k],
                           ours_all[k].view(torch.uint8) if ours_all[k].dtype == torch.int8
                           else ours_all[k]), k
    for l in range(2):
        t = ck.read_mlp_layer(tmp_path / "int4", l)
        for short, proj in (("gate", "gate_proj"), ("up", "up_proj"), ("down", "down_proj")):
            base = f"model.layers.{l}.mlp.{proj}"
            assert torch.equal(t[f"{short}_qw"].view(torch.uint8),
                               ref_all[base + ".qweight"].view(torch.uint8))
            assert torch.equal(t[f"{short}_sc"], ref_all[base + ".scales"])
        assert tuple(t["gate_qw"].shape) == (512, 128) and tuple(t["down_qw"].shape) == (256, 256)


def test_quant_config_is_validated(tmp_path):
    ck = _ckpt()
    sd = bf16_state(n_layers=1, hidden=256, inter=512, seed=2)
    write_int4_checkpoint(tmp_path, sd)
    ck.read_quant_config(tmp_path)
    for key, bad in (("group_size", 64), ("bits", 8), ("symmetric", False),
                     ("packing", "two_int4_per_int8_low_odd_high_even"), ("qmax", 8)):
        cfg = json.loads((tmp_path / "quant_config.json").read_text())
        cfg[key] = bad
        (tmp_path / "quant_config.json").write_text(json.dumps(cfg))
        with pytest.raises(ValueError, match=key):
            ck.read_quant_config(tmp_path)
        write_int4_checkpoint(tmp_path, sd)  # restore


def test_missing_or_inconsistent_tensors_are_rejected(tmp_path):
    ck = _ckpt()
    from safetensors.torch import load_file, save_file
    sd = bf16_state(n_layers=1, hidden=256, inter=512, seed=3)
    write_int4_checkpoint(tmp_path / "good", sd)
    full = {k: v.clone() for k, v in
            load_file(str(tmp_path / "good" / "model_int4.safetensors")).items()}

    def broken_dir(name, state):
        d = tmp_path / name
        d.mkdir()
        save_file(state, str(d / "model_int4.safetensors"))
        return d

    b = dict(full)
    del b["model.layers.0.mlp.up_proj.scales"]
    with pytest.raises(ValueError, match="up_proj.scales"):
        ck.read_mlp_layer(broken_dir("missing", b), 0)
    b = dict(full)
    b["model.layers.0.mlp.down_proj.scales"] = \
        full["model.layers.0.mlp.down_proj.scales"][:, :2].contiguous()
    with pytest.raises(ValueError, match="down_proj"):
        ck.read_mlp_layer(broken_dir("shape", b), 0)
