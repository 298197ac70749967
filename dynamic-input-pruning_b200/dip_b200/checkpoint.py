"""Loading the reference's int4 checkpoint into the B200 decode path.

The reference writes one file `model_int4.safetensors` in which every
quantised projection `<name>.weight` is replaced by `<name>.qweight` (int8
[out, in/2], two int4 per byte, low nibble = even column) and `<name>.scales`
(bf16 [out, in/128]), plus `quant_config.json` describing the format
(scripts/quantize.py:114-151).  Its loader checks the group size
(qlinear.py:119-122) and places the tensors into QuantLinear buffers
(qlinear.py:148-162).

Here the MLP projections of each decoder layer,
`model.layers.{i}.mlp.{gate,up,down}_proj.{qweight,scales}`, are read
tensor by tensor (safetensors' lazy reader, so a 64-layer checkpoint is never
held in host memory at once) and put on the GPU in the layout the kernels
read: gate and up as stored, down transposed once with the rule of
_transpose_down_to_int4 (dip_stream_predispatch.py:100-120) by the sm_100a
transpose kernel.  `DipStack.from_checkpoint` builds a decode stack on them.
"""
from __future__ import annotations

import json
from pathlib import Path

import torch

GROUP_SIZE = 128
QMAX = 7
# the format fields scripts/quantize.py:140-148 writes, with the values this
# path reads
EXPECTED_QUANT_CONFIG = {
    "quant_method": "self_int4_symmetric_groupwise",
    "group_size": GROUP_SIZE,
    "bits": 4,
    "symmetric": True,
    "packing": "two_int4_per_int8_low_even_high_odd",
    "qmax": QMAX,
}
CHECKPOINT_FILE = "model_int4.safetensors"
PROJ = ("gate_proj", "up_proj", "down_proj")


def read_quant_config(ckpt_dir) -> dict:
    """quant_config.json, checked field by field against the only format the
    kernels read (the reference asserts the group size, qlinear.py:121; a
    different bit width, packing or asymmetric scheme would be misread just
    as silently, so those are checked too).  Raises ValueError."""
    p = Path(ckpt_dir) / "quant_config.json"
    if not p.exists():
        raise ValueError(f"{p} not found: not an int4 checkpoint of scripts/quantize.py")
    cfg = json.loads(p.read_text())
    for key, want in EXPECTED_QUANT_CONFIG.items():
        if cfg.get(key) != want:
            raise ValueError(f"quant_config.json: {key} = {cfg.get(key)!r}, expected {want!r}")
    return cfg


def mlp_tensor_names(layer: int) -> dict:
    """Checkpoint key of each MLP tensor of decoder layer `layer`."""
    base = f"model.layers.{layer}.mlp"
    out = {}
    for proj, short in zip(PROJ, ("gate", "up", "down")):
        out[f"{short}_qw"] = f"{base}.{proj}.qweight"
        out[f"{short}_sc"] = f"{base}.{proj}.scales"
    return out


def count_mlp_layers(ckpt_dir) -> int:
    """Number of consecutive decoder layers 0, 1, ... with all six MLP tensors."""
    from safetensors import safe_open
    with safe_open(str(Path(ckpt_dir) / CHECKPOINT_FILE), framework="pt", device="cpu") as f:
        keys = set(f.keys())
    n = 0
    while all(k in keys for k in mlp_tensor_names(n).values()):
        n += 1
    return n


def _check_pair(name: str, qw: torch.Tensor, sc: torch.Tensor) -> None:
    if qw.dtype not in (torch.int8, torch.uint8) or qw.dim() != 2:
        raise ValueError(f"{name}.qweight: expected a 2-D int8 tensor, got {qw.dtype} {tuple(qw.shape)}")
    if sc.dtype != torch.bfloat16 or sc.dim() != 2:
        raise ValueError(f"{name}.scales: expected a 2-D bf16 tensor, got {sc.dtype} {tuple(sc.shape)}")
    if qw.shape[0] != sc.shape[0] or qw.shape[1] * 2 != sc.shape[1] * GROUP_SIZE:
        raise ValueError(f"{name}: qweight {tuple(qw.shape)} and scales {tuple(sc.shape)} "
                         f"disagree for group size {GROUP_SIZE}")


def read_mlp_layer(ckpt_dir, layer: int) -> dict:
    """The six MLP tensors of one layer exactly as stored (CPU tensors):
    gate_qw [I, H/2], gate_sc [I, H/128], up_* likewise, down_qw [H, I/2],
    down_sc [H, I/128].  Shapes are checked against each other."""
    from safetensors import safe_open
    names = mlp_tensor_names(layer)
    out = {}
    with safe_open(str(Path(ckpt_dir) / CHECKPOINT_FILE), framework="pt", device="cpu") as f:
        keys = set(f.keys())
        for k, n in names.items():
            if n not in keys:
                raise ValueError(f"{n} missing from {CHECKPOINT_FILE}")
            out[k] = f.get_tensor(n)
    for short, proj in zip(("gate", "up", "down"), PROJ):
        _check_pair(f"model.layers.{layer}.mlp.{proj}", out[f"{short}_qw"], out[f"{short}_sc"])
    I, H = out["gate_qw"].shape[0], out["gate_qw"].shape[1] * 2
    if out["up_qw"].shape != out["gate_qw"].shape or tuple(out["down_qw"].shape) != (H, I // 2):
        raise ValueError(f"layer {layer}: gate {tuple(out['gate_qw'].shape)}, up "
                         f"{tuple(out['up_qw'].shape)}, down {tuple(out['down_qw'].shape)} do "
                         f"not form a SwiGLU MLP")
    for k in ("gate_qw", "up_qw", "down_qw"):
        out[k] = out[k].view(torch.int8)
    return out


def load_mlp_layer(ckpt_dir, layer: int, device) -> dict:
    """One layer on `device` in the kernels' layout: gate / up as stored, the
    down projection transposed to down_t_qw [I, H/2], down_t_sc [I, H/128]
    (dip_stream_predispatch.py:100-120, on the GPU)."""
    t = read_mlp_layer(ckpt_dir, layer)
    dev = torch.device(device)
    out = {k: t[k].to(dev).contiguous() for k in ("gate_qw", "gate_sc", "up_qw", "up_sc")}
    out["down_t_qw"], out["down_t_sc"] = torch.ops.dip_b200.transpose_down_int4(
        t["down_qw"].to(dev).contiguous(), t["down_sc"].to(dev).contiguous())
    return out


def load_mlp_layers(ckpt_dir, device, n_layers: int | None = None) -> list:
    """Layers 0 .. n_layers-1 (all of them by default), after validating
    quant_config.json."""
    read_quant_config(ckpt_dir)
    n = count_mlp_layers(ckpt_dir) if n_layers is None else n_layers
    if n < 1:
        raise ValueError(f"no decoder-layer MLP tensors in {Path(ckpt_dir) / CHECKPOINT_FILE}")
    return [load_mlp_layer(ckpt_dir, l, device) for l in range(n)]
