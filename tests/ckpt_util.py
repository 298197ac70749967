"""Test helper: tiny synthetic checkpoints in the reference's int4 format.

`make_bf16_model` writes a bf16 Qwen3-like `model.safetensors` (embeddings,
norms, attention and MLP projections, lm_head) of the given size.
`write_int4_checkpoint` converts such a state dict the way
scripts/quantize.py:114-151 does (projections -> .qweight / .scales with the
oracle's quantiser, everything else kept, quant_config.json); the CPU test
checks that its output equals the reference script's byte for byte, so GPU
tests (where the reference is absent) can use it.
"""
from __future__ import annotations

import json
from pathlib import Path

import torch

QUANT_CONFIG = {
    "quant_method": "self_int4_symmetric_groupwise",
    "group_size": 128,
    "bits": 4,
    "symmetric": True,
    "packing": "two_int4_per_int8_low_even_high_odd",
    "qmax": 7,
}
PROJS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def bf16_state(n_layers: int, hidden: int, inter: int, seed: int = 0, vocab: int = 64) -> dict:
    gen = torch.Generator().manual_seed(seed)

    def w(*s):
        return (torch.randn(*s, generator=gen) * 0.02).to(torch.bfloat16)

    sd = {"model.embed_tokens.weight": w(vocab, hidden), "lm_head.weight": w(vocab, hidden),
          "model.norm.weight": torch.ones(hidden, dtype=torch.bfloat16)}
    for l in range(n_layers):
        b = f"model.layers.{l}"
        sd[f"{b}.input_layernorm.weight"] = torch.ones(hidden, dtype=torch.bfloat16)
        sd[f"{b}.post_attention_layernorm.weight"] = torch.ones(hidden, dtype=torch.bfloat16)
        for p in ("q_proj", "k_proj", "v_proj", "o_proj"):
            sd[f"{b}.self_attn.{p}.weight"] = w(hidden, hidden)
        sd[f"{b}.mlp.gate_proj.weight"] = w(inter, hidden)
        sd[f"{b}.mlp.up_proj.weight"] = w(inter, hidden)
        sd[f"{b}.mlp.down_proj.weight"] = w(hidden, inter)
    return sd


def make_bf16_model(model_dir, sd: dict) -> None:
    from safetensors.torch import save_file
    d = Path(model_dir)
    d.mkdir(parents=True, exist_ok=True)
    save_file(sd, str(d / "model.safetensors"))


def _quantize(name: str) -> bool:
    ln = name.lower()
    return (name.endswith(".weight") and "embed_tokens" not in ln and "lm_head" not in ln
            and "norm" not in ln and any(p in ln for p in PROJS))


def write_int4_checkpoint(out_dir, sd: dict) -> None:
    from safetensors.torch import save_file
    from oracle import dip_oracle as O
    d = Path(out_dir)
    d.mkdir(parents=True, exist_ok=True)
    out = {}
    for name, t in sd.items():
        if _quantize(name):
            qw, sc = O.quantize_int4_g128(t)
            out[name[:-len(".weight")] + ".qweight"] = qw
            out[name[:-len(".weight")] + ".scales"] = sc
        else:
            out[name] = t
    save_file(out, str(d / "model_int4.safetensors"))
    (d / "quant_config.json").write_text(json.dumps(QUANT_CONFIG, indent=2))
