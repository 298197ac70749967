"""dip_b200 — B200-native (sm_100a) decode-time Dynamic Input Pruning MLP.

A drop-in for the reference's DIP path (rohitpotluri/dynamic-input-pruning):
the same module classes and torch.ops schemas, backed by hand-written CUDA.
Importing the package loads the kernels; it raises if they were not built.
"""
from ._lib import load_ops as _load_ops

_load_ops()

from .qlinear import GROUP_SIZE, QuantLinear, dequantize  # noqa: E402
from .gate_kernel import gate_gemv  # noqa: E402
from .topk_kernel import select_topk  # noqa: E402
from .dip_stream_predispatch import SharedBuffers, StreamingDIPMlp  # noqa: E402
from .dip_ca import CABuffers, CADIPMlp, calibrate_cache, calibrate_cache_inputs  # noqa: E402

__all__ = ["GROUP_SIZE", "QuantLinear", "dequantize", "gate_gemv", "select_topk",
           "SharedBuffers", "StreamingDIPMlp", "CABuffers", "CADIPMlp", "calibrate_cache",
           "calibrate_cache_inputs"]
