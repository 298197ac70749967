"""select_topk() — the reference's topk_kernel.py API over the sm_100a kernel.

The selection is exactly that of kernels/topk_select/topk_select.cu (k
indices: |s| above the bisection threshold in ascending order, then the tie
band in ascending order) but computed in one launch without host syncs.
"""
import torch

from ._lib import load_ops

load_ops()
_use_topk = True


def select_topk(s: torch.Tensor, k: int) -> torch.Tensor:
    """topk_kernel.py:29-40: k channel ids of the largest |s|, int64 [k]."""
    return torch.ops.topk_ops.topk_select(s.contiguous(), k).to(torch.long)
