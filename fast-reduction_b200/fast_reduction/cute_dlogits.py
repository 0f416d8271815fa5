"""Drop-in for `fast_reduction.cute_dlogits` (reference file of the same name).

    dz_j = p_j * (g_ce - g_ent * (log p_j + H)) - g_ce * 1{j == target},  p_j = exp(z_j - lse)

over fp32 logits [M, V], written as fp32 [M, V] (reference cute_dlogits.py:1-17, 87-100). Like
the reference, no target value is treated as ignored here: a target outside [0, V) simply
matches no column. The training path of gemm_kernel.py calls the same libfrx kernel with
bf16 output and ignore_index = -100 instead.
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import ops


def _prep_target(target: Tensor) -> Tensor:
    if target.dtype not in (torch.int32, torch.int64):
        raise KeyError(target.dtype)  # the reference looks the dtype up in an int32/int64 map
    return target.to(torch.int64).contiguous()


def compute_dlogits_out(logits: Tensor, target: Tensor, lse: Tensor, entropy: Tensor, g_ce: Tensor,
                        g_ent: Tensor, dlogits: Tensor) -> None:
    """Fused dlogits into a pre-allocated fp32 output (reference custom op, :121-159)."""
    if logits.dim() != 2:
        raise ValueError("logits must be 2-D [M, V]")
    if not logits.is_cuda:
        raise ValueError("logits must be a CUDA tensor")
    M, V = logits.shape
    ops.dlogits(
        logits, _prep_target(target), lse.float().contiguous(), entropy.float().contiguous(), dlogits,
        rows=M, vocab_shard=V, g_ce=g_ce.float().contiguous(), g_ent=g_ent.float().contiguous(),
    )


def compute_dlogits(logits: Tensor, target: Tensor, lse: Tensor, entropy: Tensor, g_ce: Tensor,
                    g_ent: Tensor) -> Tensor:
    """Returns dlogits (M, V) fp32 (reference :162-183)."""
    dlogits = torch.empty_like(logits)
    compute_dlogits_out(logits, target, lse, entropy, g_ce, g_ent, dlogits)
    return dlogits
