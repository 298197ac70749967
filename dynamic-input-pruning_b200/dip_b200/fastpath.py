"""Which sm_100a kernel serves a drop-in call, decided from the shapes.

* Decode, one token: the one-launch fused layer (layer_fused_kernel via
  dip_b200::mlp_decode_fused / mlp_decode_fused_ca) wherever its shape
  limits allow (hidden = 2560 or 5120, intermediate a multiple of 8 with at
  most 191 rows per worker SM).  Other shapes use the separate-launch chain
  (gate, top-k, up, down kernels).  Both compute the reference's
  StreamingDIPMlp.forward (dip_stream_predispatch.py:176-204).
* Prefill and other multi-token calls: the dense int4 x bf16 GEMMs on the
  tcgen05 tensor cores (dip_int4_gemm_tc / dip_int4_down_tc) for
  QuantLinear.forward (qlinear.py:86-88) and the modules' _dense
  (dip_stream_predispatch.py:206-215, dip_ca.py:190-196), in bf16 with fp32
  accumulation like the reference's F.linear.  Shapes the GEMMs do not take
  (in_features not a multiple of 256, non-bf16 activations) run
  dequantize + F.linear, still on the GPU.
"""
from __future__ import annotations

import torch

from ._lib import load_ops

load_ops()

_TC_MAX_ROWS = 128  # activation rows per tcgen05 GEMM call


def fused_layer_supported(hidden: int, inter: int, device) -> bool:
    """The fused layer's shape limits (dip_mlp_decode_fused_ca's checks)."""
    if hidden % 128 or (hidden // 128) not in (20, 40) or inter % 8:
        return False
    nb = torch.cuda.get_device_properties(torch.device(device)).multi_processor_count
    if nb < 2 or nb > 160:
        return False
    return (inter + nb - 2) // (nb - 1) <= 16 * 12 - 1 and inter * nb < 2 ** 31


def tc_linear_ok(in_features: int, x: torch.Tensor) -> bool:
    return x.dtype == torch.bfloat16 and in_features % 256 == 0


def tc_linear(qweight: torch.Tensor, scales: torch.Tensor, x2d: torch.Tensor,
              epilogue: int = 0) -> torch.Tensor:
    """out [T, rows] = epi(x2d [T, in] @ dequant(W)^T) on the tensor cores,
    in chunks of at most 128 activation rows.  epilogue 0: bf16(acc);
    1: bf16(silu(bf16(acc)))."""
    x2d = x2d.contiguous()
    outs = [torch.ops.dip_b200.gemm_tc(qweight, scales, x2d[i:i + _TC_MAX_ROWS], epilogue)
            for i in range(0, x2d.shape[0], _TC_MAX_ROWS)]
    return outs[0] if len(outs) == 1 else torch.cat(outs)


def tc_down_ok(inter: int, out_features: int, x: torch.Tensor) -> bool:
    return x.dtype == torch.bfloat16 and inter % 64 == 0 and out_features % 256 == 0


def tc_down(down_t_qw: torch.Tensor, down_t_sc: torch.Tensor, h2d: torch.Tensor) -> torch.Tensor:
    """y [T, out] = h2d [T, inter] @ dequant(W_down_t) on the tensor cores."""
    h2d = h2d.contiguous()
    outs = [torch.ops.dip_b200.down_tc(down_t_qw, down_t_sc, h2d[i:i + _TC_MAX_ROWS])
            for i in range(0, h2d.shape[0], _TC_MAX_ROWS)]
    return outs[0] if len(outs) == 1 else torch.cat(outs)


def dense_mlp(gate_qw, gate_sc, up_qw, up_sc, down_t_qw, down_t_sc, x: torch.Tensor):
    """The dense SwiGLU MLP of _dense (dip_stream_predispatch.py:206-215):
    g = silu(x W_gate^T), u = x W_up^T, y = (g * u) W_down_t, each GEMM on
    the tensor cores.  Returns None when a shape is not supported (the caller
    then runs its dequantize + F.linear form)."""
    hidden = gate_qw.shape[1] * 2
    inter = gate_qw.shape[0]
    out_f = down_t_qw.shape[1] * 2
    if not (tc_linear_ok(hidden, x) and tc_down_ok(inter, out_f, x)):
        return None
    x2d = x.reshape(-1, hidden)
    g = tc_linear(gate_qw, gate_sc, x2d, epilogue=1)
    u = tc_linear(up_qw, up_sc, x2d, epilogue=0)
    y = tc_down(down_t_qw, down_t_sc, g * u)
    return y.reshape(*x.shape[:-1], out_f)
