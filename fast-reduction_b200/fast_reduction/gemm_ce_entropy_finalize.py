"""Drop-in for `fast_reduction.gemm_ce_entropy_finalize` (reference file of the same name).

The reference's partials contract is kept verbatim here: ``partials`` is [N_tiles, M, 4] fp32 with
(max, sum exp(x - max), sum x * exp(x - max), target logit or 0) per (tile, row)
(reference gemm_ce_entropy_finalize.py:1-12, epilogue gemm_ce_entropy_epilogue.py:263-271).
The merge runs in libfrx (`frx_finalize` with FRX_PARTIALS_REF_LAYOUT).
"""

from __future__ import annotations

from typing import Tuple

import torch
from torch import Tensor

from . import ops


def _check(partials: Tensor, n_tiles: int) -> int:
    if partials.dim() != 3 or partials.size(2) != 4:
        raise ValueError(f"partials must be [N_tiles, M, 4], got {tuple(partials.shape)}")
    if partials.dtype != torch.float32:
        raise TypeError("partials must be float32")
    if not (0 <= n_tiles <= partials.size(0)):
        raise ValueError(f"n_tiles={n_tiles} outside [0, {partials.size(0)}]")
    return partials.size(1)


def _run(partials: Tensor, n_tiles: int, loss: Tensor, entropy: Tensor, lse: Tensor | None) -> None:
    M = partials.size(1)
    p = partials if partials.is_contiguous() else partials.contiguous()
    ops.finalize(p, n_tiles, M, M, ref_layout=True, ce=loss, entropy=entropy, lse=lse)


def finalize_ce_entropy_out(partials: Tensor, loss: Tensor, entropy: Tensor, n_tiles: int) -> None:
    """Merge partial reductions -> loss + entropy, written into the given tensors
    (reference custom op fast_reduction::finalize_ce_entropy, :123-133)."""
    _check(partials, n_tiles)
    _run(partials, n_tiles, loss, entropy, None)


def finalize_ce_entropy_lse_out(partials: Tensor, loss: Tensor, entropy: Tensor, lse: Tensor, n_tiles: int) -> None:
    """Merge partial reductions -> loss + entropy + lse (reference :136-148)."""
    _check(partials, n_tiles)
    _run(partials, n_tiles, loss, entropy, lse)


def finalize_ce_entropy(partials: Tensor, n_tiles: int) -> Tuple[Tensor, Tensor]:
    """partials [N_tiles, M, 4] fp32 -> (loss [M], entropy [M]) fp32 (reference :182-195)."""
    M = _check(partials, n_tiles)
    loss = torch.empty(M, device=partials.device, dtype=torch.float32)
    entropy = torch.empty(M, device=partials.device, dtype=torch.float32)
    _run(partials, n_tiles, loss, entropy, None)
    return loss, entropy


def finalize_ce_entropy_with_lse(partials: Tensor, n_tiles: int) -> Tuple[Tensor, Tensor, Tensor]:
    """partials [N_tiles, M, 4] fp32 -> (loss, entropy, lse), each [M] fp32 (reference :198-212)."""
    M = _check(partials, n_tiles)
    loss = torch.empty(M, device=partials.device, dtype=torch.float32)
    entropy = torch.empty(M, device=partials.device, dtype=torch.float32)
    lse = torch.empty(M, device=partials.device, dtype=torch.float32)
    _run(partials, n_tiles, loss, entropy, lse)
    return loss, entropy, lse
