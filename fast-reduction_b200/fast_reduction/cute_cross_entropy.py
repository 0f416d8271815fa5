"""Drop-in for the standalone reductions of `fast_reduction.cute_cross_entropy` (reference file
of the same name, :583-735): cross-entropy / entropy / logsumexp of a materialised logits matrix.

    ce_fwd(x, target) -> loss [M]                    (target < 0 -> loss 0)
    entropy_fwd(x) -> entropy [M]
    ce_entropy_fwd(x, target) -> (loss, entropy)
    ce_entropy_fwd_with_lse(x, target) -> (loss, entropy, lse)
    ..._out(...) variants write into given fp32 tensors.

x is [M, N] bf16, fp16 or fp32; results are fp32. On B200 the rows are cut into column tiles so
that even a handful of long rows spread over every SM: libfrx's frx_logits_partials reduces each
(row, tile) to a softmax partial and frx_finalize merges them.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import Tensor

from . import ops

_TILE_COLS_MIN = 2048


def _tile_cols(M: int, N: int) -> int:
    # one warp per (row, tile): enough of them to fill every SM (64 warps each) about twice over;
    # tiles a multiple of 8 columns
    try:
        sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    except Exception:
        sms = 148
    want_units = 2 * 64 * sms
    want_tiles = max(1, (want_units + max(M, 1) - 1) // max(M, 1))
    tile = max(_TILE_COLS_MIN, (N + want_tiles - 1) // want_tiles)
    return (tile + 7) // 8 * 8


def _prep(x: Tensor, target: Optional[Tensor]):
    if x.dim() != 2:
        raise ValueError(f"x must be 2-D [M, N], got shape {tuple(x.shape)}")
    if not x.is_cuda:
        raise ValueError("x must be a CUDA tensor")
    if x.stride(1) != 1:
        x = x.contiguous()
    t = None
    if target is not None:
        if target.dim() != 1:
            raise ValueError("target must be 1-D")
        if target.dtype not in (torch.int32, torch.int64):
            raise KeyError(target.dtype)  # the reference maps only int32 / int64 targets
        t = target.to(torch.int64).contiguous()
    return x, t


def _run(x: Tensor, target: Optional[Tensor], loss: Optional[Tensor], entropy: Optional[Tensor],
         lse: Optional[Tensor]) -> None:
    x, t = _prep(x, target)
    M, N = x.shape
    if M == 0:
        return
    tile = _tile_cols(M, N)
    n_tiles = (N + tile - 1) // tile
    partials = torch.empty(n_tiles, M, 4, device=x.device, dtype=torch.float32)
    ops.logits_partials(x, t, partials, tile, M)
    ops.finalize(partials, n_tiles, M, M, ignore_negative=True, target=t, vocab_size=N, ce=loss, entropy=entropy,
                 lse=lse)


def ce_fwd_out(x: Tensor, target: Tensor, loss: Tensor) -> None:
    """Cross-entropy forward into a pre-allocated fp32 loss (reference :588-610)."""
    _run(x, target, loss, None, None)


def ce_fwd(x: Tensor, target: Tensor) -> Tensor:
    """Cross-entropy loss from logits. Returns loss [M] fp32 (reference :613-618)."""
    loss = torch.empty(x.size(0), device=x.device, dtype=torch.float32)
    ce_fwd_out(x, target, loss)
    return loss


def entropy_fwd_out(x: Tensor, entropy: Tensor) -> None:
    """Entropy forward into a pre-allocated fp32 tensor (reference :621-642)."""
    _run(x, None, None, entropy, None)


def entropy_fwd(x: Tensor) -> Tensor:
    """Entropy from logits. Returns entropy [M] fp32 (reference :645-650)."""
    entropy = torch.empty(x.size(0), device=x.device, dtype=torch.float32)
    entropy_fwd_out(x, entropy)
    return entropy


def ce_entropy_fwd_out(x: Tensor, target: Tensor, loss: Tensor, entropy: Tensor) -> None:
    """Cross-entropy + entropy into pre-allocated outputs (reference :653-663)."""
    _run(x, target, loss, entropy, None)


def ce_entropy_fwd_lse_out(x: Tensor, target: Tensor, loss: Tensor, entropy: Tensor, lse: Tensor) -> None:
    """Cross-entropy + entropy + LSE into pre-allocated outputs (reference :666-677)."""
    _run(x, target, loss, entropy, lse)


def ce_entropy_fwd(x: Tensor, target: Tensor) -> Tuple[Tensor, Tensor]:
    """Cross-entropy loss and entropy from logits in one pass (reference :707-716)."""
    M = x.size(0)
    loss = torch.empty(M, device=x.device, dtype=torch.float32)
    entropy = torch.empty(M, device=x.device, dtype=torch.float32)
    ce_entropy_fwd_out(x, target, loss, entropy)
    return loss, entropy


def ce_entropy_fwd_with_lse(x: Tensor, target: Tensor) -> Tuple[Tensor, Tensor, Tensor]:
    """Cross-entropy loss, entropy and LSE from logits in one pass (reference :719-735)."""
    M = x.size(0)
    loss = torch.empty(M, device=x.device, dtype=torch.float32)
    entropy = torch.empty(M, device=x.device, dtype=torch.float32)
    lse = torch.empty(M, device=x.device, dtype=torch.float32)
    ce_entropy_fwd_lse_out(x, target, loss, entropy, lse)
    return loss, entropy, lse
