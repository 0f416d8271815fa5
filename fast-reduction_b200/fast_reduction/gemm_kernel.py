"""Drop-in for `fast_reduction.gemm_kernel` (reference: fast_reduction/gemm_kernel.py), B200 engine.

Public functions keep the reference's names, signatures and return conventions:

  gemm_fused_ce_entropy(hidden_states, weight, target, bias=None, chunk_size=4096, tile_M=128, tile_N=256)
      -> (ce_loss, entropy, log_probs), fp32, shaped like hidden_states.shape[:-1]
      (reference gemm_kernel.py:276-356)
  gemm_megakernel_fast(hidden_states, weight, target, bias=None, chunk_size=4096, ce_weight=1.0, ent_weight=-1.0)
      -> (loss, ce_loss, entropy); loss is a 0-d tensor that requires grad, loss.backward() fills
      hidden.grad / weight.grad (reference gemm_kernel.py:883-934)

Engine (all device work is libfrx, sm_100a):
  forward   frx_fwd_partials: tcgen05 GEMM whose epilogue reduces each 128x256 fp32 TMEM tile to
            per-row softmax partials; logits never reach HBM.  frx_finalize: partials -> ce/H/lse.
  training  the same GEMM also streams fp32 logits of one row chunk to HBM; frx_dlogits turns
            them into bf16 (fp16) dlogits for all rows; frx_gemm_dhidden / frx_gemm_dweight run once
            over the full batch (d_weight accumulates over every row in TMEM: no fp32 d_weight
            read-modify-write per chunk, no transposed weight copy).

Semantics chosen where the reference is inconsistent:
  * ignore_index (default -100): ce = 0, log_probs = 0 and no CE gradient for such rows; the
    entropy and its gradient are kept (torch nll_loss semantics, reference baseline.py:80).
  * bias: the reference accepts it but never adds it to the logits in its GEMM path
    (gemm_kernel.py:280) while its fp32 baseline does (baseline.py:76); here a bias [V] (dtype of
    the weight) is added to every logit in the GEMM epilogue, and its gradient is the column sum
    of dlogits (the reference's `d_bias.add_(dlogits.sum(dim=0))`, gemm_kernel.py:867-869).
  * loss = ce_weight * sum(ce) + ent_weight * sum(entropy) (a sum, gemm_kernel.py:897).
  * tile_M / tile_N are accepted for signature compatibility and ignored (tiles are fixed at
    128 x 256 by the sm_100a kernel; the partials use 256-column vocabulary tiles).
"""

from __future__ import annotations

import os
from typing import Optional, Tuple

import torch
from torch import Tensor

from . import ops

IGNORE_INDEX = -100

# Run each chunk's dlogits (HBM-bound) on a side stream so it overlaps the next chunk's forward
# GEMM (tensor-bound). FRX_OVERLAP_DLOGITS=0 serialises them (for measurement).
_OVERLAP_DLOGITS = os.environ.get("FRX_OVERLAP_DLOGITS", "1") != "0"
# The training forward hands its logits to the dlogits pass as fp16 z - m (m = the maximum of the
# logit's 256-column tile, already in the partials): 2 bytes per logit written and read back
# instead of 4. FRX_TRAIN_LOGITS=f32 keeps the reference's fp32 logits (for A/B measurement);
# fp32 operands always use fp32 logits.
_TILEREL_LOGITS = os.environ.get("FRX_TRAIN_LOGITS", "f16rel") != "f32"
# The training pass's chunk_size bounds the logits memory, as the reference's per-chunk fp32 logits
# buffer does (chunk_size x V x 4 bytes): rows go in launches as large as fit that budget, so a
# vocabulary shard runs fewer forward launches and cross-rank statistics exchanges.
# FRX_TRAIN_MERGE=0 keeps launches of chunk_size rows (for A/B measurement).
_TRAIN_MERGE = os.environ.get("FRX_TRAIN_MERGE", "1") != "0"
_side_streams: dict = {}


def _side_stream(dev: torch.device) -> torch.cuda.Stream:
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    st = _side_streams.get(idx)
    if st is None:
        st = torch.cuda.Stream(device=torch.device("cuda", idx))
        _side_streams[idx] = st
    return st


def _input_device(*tensors: Optional[Tensor]) -> Optional[torch.device]:
    """None when every given tensor is on a GPU; otherwise (some are host tensors) the device the
    host-streamed path runs on: the CUDA device of the GPU-resident ones, else the current one."""
    cuda = [t.device for t in tensors if t is not None and t.is_cuda]
    host = [t for t in tensors if t is not None and t.device.type == "cpu"]
    if not host:
        return None
    for t in tensors:
        if t is not None and not t.is_cuda and t.device.type != "cpu":
            raise ValueError(f"inputs must be CUDA or CPU tensors, got one on {t.device}")
    if any(d != cuda[0] for d in cuda):
        raise ValueError(f"CUDA inputs must share one device, got {sorted(set(map(str, cuda)))}")
    if cuda:
        return cuda[0]
    if not torch.cuda.is_available():
        raise RuntimeError("fast_reduction (B200 engine) needs a CUDA device; none is visible")
    return torch.device("cuda", torch.cuda.current_device())


def _prepare(hidden_states: Tensor, weight: Tensor, target: Tensor, bias: Optional[Tensor], allow_host: bool = False):
    if hidden_states.dtype != weight.dtype or hidden_states.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        raise NotImplementedError(
            "the B200 engine computes in bf16, fp16 or fp32 (hidden and weight of the same type); got hidden "
            f"{hidden_states.dtype}, weight {weight.dtype}"
        )
    if weight.dim() != 2:
        raise ValueError(f"weight must be [V, H], got shape {tuple(weight.shape)}")
    H = hidden_states.shape[-1]
    if weight.shape[1] != H:
        raise ValueError(f"hidden size mismatch: hidden [..., {H}] vs weight {tuple(weight.shape)}")
    if H % 8 != 0 and hidden_states.dtype != torch.float32:
        raise NotImplementedError(f"hidden size must be a multiple of 8 (TMA row alignment), got {H}")
    batch_shape = hidden_states.shape[:-1]
    hidden_2d = hidden_states.reshape(-1, H)
    if hidden_2d.stride(1) != 1 or hidden_2d.stride(0) % 8 != 0 or hidden_2d.data_ptr() % 16 != 0:
        hidden_2d = hidden_2d.contiguous()
    if weight.stride(1) != 1 or weight.stride(0) % 8 != 0 or weight.data_ptr() % 16 != 0:
        weight = weight.contiguous()
    target_1d = target.reshape(-1)
    if target_1d.numel() != hidden_2d.shape[0]:
        raise ValueError(f"target has {target_1d.numel()} elements, expected {hidden_2d.shape[0]}")
    if target_1d.dtype != torch.int64:
        if target_1d.dtype.is_floating_point or target_1d.dtype == torch.bool:
            raise TypeError(f"target must be an integer tensor, got {target_1d.dtype}")
        target_1d = target_1d.to(torch.int64)
    target_1d = target_1d.contiguous()
    if bias is not None:
        if bias.dim() != 1 or bias.numel() != weight.shape[0]:
            raise ValueError(f"bias must be [V={weight.shape[0]}], got shape {tuple(bias.shape)}")
        if bias.dtype != weight.dtype:
            raise NotImplementedError(f"bias must have the weight's dtype {weight.dtype}, got {bias.dtype}")
        bias = bias.contiguous()
    if not (allow_host and _input_device(hidden_2d, weight, target_1d, bias) is not None):
        ops._require_cuda(hidden_2d, weight, target_1d, bias)
    return batch_shape, hidden_2d, weight, target_1d, bias


def _chunk_rows(chunk_size: int, B: int) -> int:
    if chunk_size is None or chunk_size <= 0:
        raise ValueError(f"chunk_size must be positive, got {chunk_size}")
    return max(1, min(int(chunk_size), B))


def _fp32_k_operands(hidden_2d: Tensor, weight: Tensor, bias: Optional[Tensor]) -> Tuple[Tensor, Tensor]:
    """bf16 operands whose product is the fp32 product hidden @ weight.T (+ bias), for the forward GEMM.

    bf16x6 (Henry, Tang, Heinecke, ARITH 2019): each fp32 matrix is split into bf16 hi / mid / lo parts
    (frx_split_f32) and six parts of each are concatenated along K, so one bf16 GEMM with K = 6 H sums
    hi.hi + hi.mid + mid.hi + hi.lo + lo.hi + mid.mid in fp32 TMEM. A bias rides along as three more
    K columns (ones against its own hi / mid / lo). K is zero-padded to a multiple of 8."""
    B, H = hidden_2d.shape
    V = weight.shape[0]
    dev = hidden_2d.device
    n = len(ops.SPLIT_LEFT)
    extra = 3 if bias is not None else 0
    K = ops.round_up(n * H + extra, 8)
    x6 = torch.empty(B, K, device=dev, dtype=torch.bfloat16)
    w6 = torch.empty(V, K, device=dev, dtype=torch.bfloat16)
    x6[:, n * H:].zero_()
    w6[:, n * H:].zero_()
    if B:
        ops.split_f32(hidden_2d, x6, ops.SPLIT_LEFT, part_stride=H)
    ops.split_f32(weight, w6, ops.SPLIT_RIGHT, part_stride=H)
    if bias is not None:
        x6[:, n * H:n * H + 3] = 1.0
        ops.split_f32(bias.view(V, 1), w6[:, n * H:], (_HI, _MID, _LO), part_stride=1)
    return x6, w6


_HI, _MID, _LO = 0, 1, 2


def _fp32_parts(x: Tensor) -> Tensor:
    """[3, rows, cols] bf16 views (row stride a multiple of 8 elements, as TMA wants): the hi / mid /
    lo parts of the fp32 matrix x [rows, cols]."""
    rows, cols = x.shape
    ld = ops.round_up(max(cols, 1), 8)
    out = torch.empty(3, rows, ld, device=x.device, dtype=torch.bfloat16)
    if rows and cols:
        ops.split_f32(x, out[0], (_HI, _MID, _LO), part_stride=rows * ld)
    return out[:, :, :cols]


# The forward launches chunk_size rows at a time, or a multiple of it while the partials of one
# launch ([tiles, rows, 4] fp32) stay within this many bytes. Small vocabulary shards then run as
# one launch over many rows: one pipeline fill and one tail instead of several, and fewer partial
# waves. Measured on one B200 over 32768 rows (4096-row bands): shard 16032 (8 GPUs) 2.74-2.79 ms
# in 4096-row launches vs 2.64 ms in one launch; shard 32064 5.77 vs 5.66 ms; shard 64128 and the
# full 128256 vocabulary unchanged within noise (the full vocabulary keeps 4096-row launches).
_FWD_LAUNCH_PARTIALS_BYTES = 48 << 20


def _launch_rows(chunk: int, B: int, n_tiles: int) -> int:
    k = max(1, _FWD_LAUNCH_PARTIALS_BYTES // (16 * max(1, n_tiles) * chunk))
    return min(B, chunk * k)


def forward_stats(
    hidden_2d: Tensor,
    weight: Tensor,
    target_1d: Tensor,
    chunk_size: int,
    *,
    vocab_offset: int = 0,
    ce: Optional[Tensor] = None,
    entropy: Optional[Tensor] = None,
    lse: Optional[Tensor] = None,
    log_probs: Optional[Tensor] = None,
    merged: Optional[Tensor] = None,
    vocab_size: Optional[int] = None,
    ignore_index: int = IGNORE_INDEX,
    bias: Optional[Tensor] = None,
) -> None:
    """Forward over one vocabulary shard, chunked over rows: GEMM-epilogue partials + finalize.

    Writes whichever of ce / entropy / lse / log_probs / merged ([B, 4] (M, S, U, ZT) per row,
    for a later cross-shard merge) are given. Rows go in launches of chunk_size rows or a multiple
    of it (_launch_rows); a row's results do not depend on how rows are grouped.
    """
    B = hidden_2d.shape[0]
    V = weight.shape[0]
    if B == 0:
        return
    T = ops.n_vocab_tiles(V)
    chunk = _launch_rows(_chunk_rows(chunk_size, B), B, T)
    partials = torch.empty(T, chunk, 4, device=hidden_2d.device, dtype=torch.float32)
    vocab_size = V if vocab_size is None else vocab_size
    for start in range(0, B, chunk):
        end = min(start + chunk, B)
        rows = end - start
        with ops.phase("frx.forward.chunk"):
            ops.fwd_partials(hidden_2d[start:end], weight, target_1d[start:end], partials, chunk, vocab_offset,
                             bias=bias)
        ops.finalize(
            partials, T, rows, chunk,
            target=target_1d[start:end], vocab_size=vocab_size, ignore_index=ignore_index,
            ce=None if ce is None else ce[start:end],
            entropy=None if entropy is None else entropy[start:end],
            lse=None if lse is None else lse[start:end],
            log_probs=None if log_probs is None else log_probs[start:end],
            merged=None if merged is None else merged[start:end],
        )


# Host-resident inputs (forward_stats_from_host): the weight is uploaded in slices of this many
# 256-row vocabulary tiles, so the GEMM over one slice runs while the next is in flight. The first
# slices are smaller (_HOST_FIRST_SLICE_TILES, doubling up to _HOST_SLICE_TILES) so the first GEMM
# after the hidden is resident waits for less weight.
_HOST_SLICE_TILES = 32
_HOST_FIRST_SLICE_TILES = 4
# Bound on the [tiles, rows, 4] fp32 partials buffer of the host-streamed path.
_HOST_PARTIALS_BYTES = 1 << 30
# When hidden and weight are both on the host, this many weight rows (the "head") go up first and
# the hidden follows in chunks of _HOST_HIDDEN_CHUNK rows; each chunk's GEMM against the head runs
# while the next chunk is in flight. The head is sized so that those GEMMs last about as long as the
# chunk uploads: rows*head*H*2 FLOP at the tensor rate F equals rows*H*2 bytes at the PCIe rate P
# when head = F / P, about 1.5e15 / 57e9 = 26,000 rows for 16-bit operands on a B200 (independent of
# rows and H). Without a head the tensor cores wait for the whole hidden before the first GEMM.
_HOST_HEAD_VOCAB = 96 * 256
_HOST_HIDDEN_CHUNK = 2048
_copy_streams: dict = {}


def _copy_stream(dev: torch.device) -> torch.cuda.Stream:
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    st = _copy_streams.get(idx)
    if st is None:
        st = torch.cuda.Stream(device=torch.device("cuda", idx))
        _copy_streams[idx] = st
    return st


def _to_device(t: Optional[Tensor], dev: torch.device, stream: torch.cuda.Stream) -> Optional[Tensor]:
    """`t` itself when it already lives on `dev`, else an upload of it enqueued on `stream`."""
    if t is None or t.device == dev:
        return t
    out = torch.empty(t.shape, dtype=t.dtype, device=dev)
    with torch.cuda.stream(stream):
        out.copy_(t, non_blocking=True)
    return out


def _host_upload_plan(B: int, V: int, *, w_host: bool, h_host: bool, shared_hidden: bool, one_group: bool):
    """Upload schedule of forward_stats_from_host: (head, hidden chunks, weight slices).

    head: weight rows [0, head) uploaded before the hidden (0: none); hidden chunks: row ranges
    uploaded one by one after the head, each followed by its GEMM against the head (empty: the
    hidden goes up whole); weight slices: row ranges [head, V) uploaded after the hidden, each
    followed by its GEMM over all rows. A head needs both operands on the host, a hidden that is not
    split across ranks, and the partials of all rows in one buffer."""
    tile = ops.VOCAB_TILE
    head = 0
    if w_host and h_host and not shared_hidden and one_group:
        head = min(V, max(tile, _HOST_HEAD_VOCAB // tile * tile))
    if w_host:
        slices, a, tiles = [], head, max(1, min(_HOST_FIRST_SLICE_TILES, _HOST_SLICE_TILES))
        while a < V:
            slices.append((a, min(a + tiles * tile, V)))
            a, tiles = slices[-1][1], min(2 * tiles, _HOST_SLICE_TILES)
    else:
        slices = [(0, V)] if V > 0 else []
    chunk = max(1, _HOST_HIDDEN_CHUNK)
    chunks = [(a, min(a + chunk, B)) for a in range(0, B, chunk)] if head else []
    return head, chunks, slices


def _upload_rows(src: Tensor, dst: Optional[Tensor], dev: torch.device, bounds, stream: torch.cuda.Stream):
    """Enqueues on `stream` the copy of src[a:b] into a device buffer for each (a, b) in `bounds`
    (none when `src` is already on `dev`); returns (buffer, [(a, b, event after that copy)])."""
    if src.device == dev:
        buf, out = src, []
        with torch.cuda.stream(stream):
            for a, b in bounds:
                ev = torch.cuda.Event()
                ev.record(stream)
                out.append((a, b, ev))
        return buf, out
    buf = torch.empty(src.shape, dtype=src.dtype, device=dev) if dst is None else dst
    out = []
    with torch.cuda.stream(stream):
        for a, b in bounds:
            buf[a:b].copy_(src[a:b], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(stream)
            out.append((a, b, ev))
    return buf, out


def forward_stats_from_host(
    hidden_2d: Tensor,
    weight: Tensor,
    target_1d: Tensor,
    dev: torch.device,
    *,
    bias: Optional[Tensor] = None,
    vocab_offset: int = 0,
    vocab_size: Optional[int] = None,
    ignore_index: int = IGNORE_INDEX,
    ce: Optional[Tensor] = None,
    entropy: Optional[Tensor] = None,
    lse: Optional[Tensor] = None,
    log_probs: Optional[Tensor] = None,
    merged: Optional[Tensor] = None,
    hidden_share=None,
) -> None:
    """forward_stats when some inputs are host (CPU) tensors: the uploads overlap the GEMMs.

    On a copy stream: target and bias (whichever are on the host), then hidden and weight. The
    weight goes up in slices of up to _HOST_SLICE_TILES vocabulary tiles; when hidden and weight are both
    on the host (and the partials of all rows fit in one buffer) the first _HOST_HEAD_VOCAB weight
    rows go first and the hidden follows in _HOST_HIDDEN_CHUNK-row chunks. The current stream
    launches one GEMM-epilogue per (hidden chunk, head) as each chunk lands, then one per remaining
    weight slice over all rows of a row group. Each launch writes the partials of its own rows and
    vocabulary tiles, and a row's partials over a tile do not depend on how rows are grouped, so the
    result equals the device-resident path bit for bit (the same tiles, each reduced in the same
    order). Outputs are device tensors given by the caller. Host inputs should be pinned for the
    copies to overlap; pageable memory is correct but serialises.

    ``hidden_share = (rank, world, gather)`` splits the upload of a host ``hidden_2d`` over ranks that
    all hold the same rows: this rank uploads only rows [rank*c, (rank+1)*c) of c = ceil(B/world) into
    a [c, H] buffer, and ``gather(share)`` (enqueued on the current stream, e.g. an NCCL all-gather)
    returns the [world*c, H] device tensor whose first B rows are hidden.
    """
    B, H = hidden_2d.shape
    V = weight.shape[0]
    if B == 0:
        return
    cur = torch.cuda.current_stream(dev)
    cp = _copy_stream(dev)
    # Device buffers come from the current stream's pool: copies into them start after its prior work.
    cp.wait_stream(cur)
    T = ops.n_vocab_tiles(V)
    group = max(ops.VOCAB_TILE, _HOST_PARTIALS_BYTES // (16 * T) // ops.VOCAB_TILE * ops.VOCAB_TILE)
    group = min(group, B)
    vocab_size = V if vocab_size is None else vocab_size
    t_d = _to_device(target_1d, dev, cp)
    b_d = _to_device(bias, dev, cp)
    w_host = weight.device != dev
    h_host = hidden_2d.device != dev
    head, chunk_bounds, bounds = _host_upload_plan(B, V, w_host=w_host, h_host=h_host,
                                                   shared_hidden=hidden_share is not None, one_group=group == B)
    w_d, _ = _upload_rows(weight, None, dev, [(0, head)] if head else [], cp)
    share_ev, h_chunks = None, []
    if hidden_share is not None and h_host:
        rank, world, gather = hidden_share
        c = (B + world - 1) // world
        lo, hi = min(B, rank * c), min(B, (rank + 1) * c)
        share = torch.empty(c, H, dtype=hidden_2d.dtype, device=dev)
        with torch.cuda.stream(cp):
            if hi > lo:
                share[: hi - lo].copy_(hidden_2d[lo:hi], non_blocking=True)
            share_ev = torch.cuda.Event()
            share_ev.record(cp)
        h_d = None
    elif head:
        h_d, h_chunks = _upload_rows(hidden_2d, None, dev, chunk_bounds, cp)
    else:
        h_d = _to_device(hidden_2d, dev, cp)
    # rest: (first row, end row, event after which the slice and every earlier upload are resident)
    w_d, rest = _upload_rows(weight, w_d if w_host else None, dev, bounds, cp)
    if share_ev is not None:
        cur.wait_event(share_ev)
        h_d = gather(share)[:B]
    partials = torch.empty(T, group, 4, device=dev, dtype=torch.float32)
    flat = partials.view(-1)
    for r0, r1, ev in h_chunks:
        # the head was enqueued before every hidden chunk, so this event covers it too
        cur.wait_event(ev)
        ops.fwd_partials(h_d[r0:r1], w_d[:head], t_d[r0:r1], flat[4 * r0:], group, vocab_offset,
                         bias=None if b_d is None else b_d[:head])
    for start in range(0, B, group):
        end = min(start + group, B)
        for a, b, ev in rest:
            if start == 0:
                cur.wait_event(ev)
            ops.fwd_partials(h_d[start:end], w_d[a:b], t_d[start:end], partials[a // ops.VOCAB_TILE:], group,
                             vocab_offset + a, bias=None if b_d is None else b_d[a:b])
        ops.finalize(
            partials, T, end - start, group,
            target=t_d[start:end], vocab_size=vocab_size, ignore_index=ignore_index,
            ce=None if ce is None else ce[start:end],
            entropy=None if entropy is None else entropy[start:end],
            lse=None if lse is None else lse[start:end],
            log_probs=None if log_probs is None else log_probs[start:end],
            merged=None if merged is None else merged[start:end],
        )


def gemm_fused_ce_entropy(
    hidden_states: Tensor,
    weight: Tensor,
    target: Tensor,
    bias: Optional[Tensor] = None,
    chunk_size: int = 4096,
    tile_M: int = 128,
    tile_N: int = 256,
    ignore_index: int = IGNORE_INDEX,
) -> Tuple[Tensor, Tensor, Tensor]:
    """Fused linear + CE + entropy forward. Returns (ce_loss, entropy, log_probs), each fp32
    and shaped like ``hidden_states.shape[:-1]``. The [chunk, V] logits never reach HBM.

    Inputs may also be host (CPU) tensors, ideally pinned: they are uploaded to the GPU of the
    CUDA inputs (else the current device) with the weight streamed in slices under the GEMMs, and
    the results are returned on ``hidden_states``' device (the call waits for them when that is
    the host)."""
    batch_shape, hidden_2d, weight, target_1d, bias = _prepare(hidden_states, weight, target, bias,
                                                               allow_host=True)
    dev = _input_device(hidden_2d, weight, target_1d, bias)
    if dev is not None and hidden_2d.dtype == torch.float32:
        # fp32 operands are split on the device before the GEMM: upload them whole, then run there
        moved = [None if t is None else t.to(dev, non_blocking=True) for t in (hidden_2d, weight, target_1d, bias)]
        res = gemm_fused_ce_entropy(*moved, chunk_size=chunk_size, ignore_index=ignore_index)
        return _results_to(hidden_states.device, batch_shape, *res)
    if dev is not None:
        B = hidden_2d.shape[0]
        ce, ent, logp = (torch.empty(B, device=dev, dtype=torch.float32) for _ in range(3))
        forward_stats_from_host(hidden_2d, weight, target_1d, dev, bias=bias, ce=ce, entropy=ent, log_probs=logp,
                                ignore_index=ignore_index)
        return _results_to(hidden_states.device, batch_shape, ce, ent, logp)
    B = hidden_2d.shape[0]
    dev = hidden_2d.device
    ce = torch.empty(B, device=dev, dtype=torch.float32)
    ent = torch.empty(B, device=dev, dtype=torch.float32)
    logp = torch.empty(B, device=dev, dtype=torch.float32)
    if hidden_2d.dtype == torch.float32:
        hidden_2d, weight = _fp32_k_operands(hidden_2d, weight, bias)
        bias = None
    forward_stats(hidden_2d, weight, target_1d, chunk_size, ce=ce, entropy=ent, log_probs=logp,
                  ignore_index=ignore_index, bias=bias)
    return ce.view(batch_shape), ent.view(batch_shape), logp.view(batch_shape)


def _results_to(out_dev: torch.device, batch_shape, *results: Tensor) -> Tuple[Tensor, ...]:
    """Per-row results shaped like ``batch_shape`` on ``out_dev``; for the host, copied into pinned
    buffers on the current stream and waited for."""
    if out_dev.type != "cpu":
        return tuple(r.to(out_dev).view(batch_shape) for r in results)
    outs = tuple(torch.empty(r.shape, dtype=r.dtype, pin_memory=True) for r in results)
    for o, r in zip(outs, results):
        o.copy_(r, non_blocking=True)
    done = torch.cuda.Event()
    done.record(torch.cuda.current_stream(results[0].device))
    done.synchronize()
    return tuple(o.view(batch_shape) for o in outs)


class GemmFusedCEEntropy(torch.autograd.Function):
    """Differentiable forward (reference GemmFusedCEEntropy, gemm_kernel.py:541-568).

    Forward: the GEMM-epilogue path (no logits in HBM); saves the per-row lse and entropy.
    Backward(g_ce, g_ent, g_lp): arbitrary per-row upstream gradients; since log_probs = -ce,
    the CE weight is g_ce - g_lp (reference :559-562). The logits are recomputed chunk by chunk by
    the same deterministic GEMM (bitwise equal to the forward's), turned into 16-bit dlogits with
    the per-row weights, and fed to the d_hidden / d_weight GEMMs.
    """

    @staticmethod
    def forward(ctx, hidden_states, weight, target, bias, chunk_size):
        batch_shape, hidden_2d, weight_c, target_1d, bias_c = _prepare(hidden_states, weight, target, bias)
        B = hidden_2d.shape[0]
        dev = hidden_2d.device
        ce = torch.empty(B, device=dev, dtype=torch.float32)
        ent = torch.empty(B, device=dev, dtype=torch.float32)
        lse = torch.empty(B, device=dev, dtype=torch.float32)
        logp = torch.empty(B, device=dev, dtype=torch.float32)
        if hidden_2d.dtype == torch.float32:
            x_fwd, w_fwd = _fp32_k_operands(hidden_2d, weight_c, bias_c)
            forward_stats(x_fwd, w_fwd, target_1d, chunk_size, ce=ce, entropy=ent, lse=lse, log_probs=logp)
            del x_fwd, w_fwd
        else:
            forward_stats(hidden_2d, weight_c, target_1d, chunk_size, ce=ce, entropy=ent, lse=lse, log_probs=logp,
                          bias=bias_c)
        ctx.save_for_backward(hidden_2d, weight_c, target_1d, lse, ent, bias_c)
        ctx.chunk_size = chunk_size
        ctx.hidden_shape = hidden_states.shape
        return ce.view(batch_shape), ent.view(batch_shape), logp.view(batch_shape)

    @staticmethod
    def backward(ctx, g_ce, g_ent, g_lp):
        hidden_2d, weight, target_1d, lse, ent, bias = ctx.saved_tensors
        B = hidden_2d.shape[0]
        dev = hidden_2d.device
        zeros = None

        def per_row(g):
            nonlocal zeros
            if g is None:
                if zeros is None:
                    zeros = torch.zeros(B, device=dev, dtype=torch.float32)
                return zeros
            return g.reshape(-1).to(torch.float32).contiguous()

        gce = per_row(g_ce)
        if g_lp is not None:
            gce = gce - per_row(g_lp)
        gent = per_row(g_ent)
        if B == 0:
            return (torch.zeros(ctx.hidden_shape, device=dev, dtype=hidden_2d.dtype), torch.zeros_like(weight), None,
                    None if bias is None else torch.zeros_like(bias), None)
        d_hidden, d_weight, d_bias, _ = fwd_bwd_shard(
            hidden_2d, weight, target_1d, ctx.chunk_size, 0.0, 0.0, lse=lse, entropy=ent,
            ignore_index=IGNORE_INDEX, stats_fn=lambda *args: None, g_ce=gce, g_ent=gent, bias=bias,
        )
        return d_hidden.view(ctx.hidden_shape), d_weight, None, d_bias, None


def gemm_fused_ce_entropy_differentiable(
    hidden_states: Tensor,
    weight: Tensor,
    target: Tensor,
    bias: Optional[Tensor] = None,
    chunk_size: int = 4096,
) -> Tuple[Tensor, Tensor, Tensor]:
    """Differentiable gemm_fused_ce_entropy: (ce_loss, entropy, log_probs) that support
    .backward() with any per-row upstream gradients (reference gemm_kernel.py:571-582)."""
    return GemmFusedCEEntropy.apply(hidden_states, weight, target, bias, chunk_size)


# The reference's two-pass epilogue variant (Level 5.2, gemm_kernel.py:363-534) exists for
# precision: no online merge inside a CTA tile. The sm_100a epilogue already reduces each
# 256-column tile in two passes against the exact tile max, so both names run the same engine.
gemm_fused_ce_entropy_v2 = gemm_fused_ce_entropy


def _train_launch_rows(chunk: int, B: int, ld_logits: int, logit_bytes: int, vocab_size: int) -> int:
    """Rows per forward launch of the training pass. The budget is the reference's per-chunk fp32
    logits buffer, chunk x vocab_size x 4 bytes (vocab_size = the whole vocabulary, also on a
    shard). All rows go in one launch when their logits fit it; otherwise two launch buffers
    (overlapped dlogits) share it, in multiples of chunk rows, and never fewer than chunk rows."""
    if not _TRAIN_MERGE:
        return chunk
    budget = chunk * max(vocab_size, 1) * 4
    if B * ld_logits * logit_bytes <= budget:
        return B
    rows = budget // (2 * ld_logits * logit_bytes) // chunk * chunk
    return min(B, max(chunk, rows))


def fwd_bwd_shard(
    hidden_2d: Tensor,
    weight: Tensor,
    target_1d: Tensor,
    chunk_size: int,
    ce_weight: float,
    ent_weight: float,
    *,
    lse: Tensor,
    entropy: Tensor,
    vocab_offset: int = 0,
    ignore_index: int = IGNORE_INDEX,
    stats_fn=None,
    g_ce: Optional[Tensor] = None,
    g_ent: Optional[Tensor] = None,
    dhidden_fn=None,
    bias: Optional[Tensor] = None,
    vocab_size: Optional[int] = None,
    dweight_max_sms: int = 0,
):
    """Training pass over one vocabulary shard; returns (d_hidden, d_weight [V_shard, H],
    d_bias [V_shard] or None, pending).

    By default d_hidden is this shard's [B, H] contribution in the hidden dtype and pending is None.
    A ``dhidden_fn(pairs)`` replaces that step (it runs between the dlogits pass and the d_weight GEMM,
    so a cross-shard reduction it starts overlaps the d_weight GEMM) and its (d_hidden, pending) pair
    is returned instead; ``pairs`` lists the (dlogits, weight) operand pairs whose frx_gemm_dhidden
    products sum to the contribution (one pair, or six bf16x6 pairs for fp32 operands).

    Rows go in forward launches of _train_launch_rows rows (chunk_size rows, or more while their
    logits fit the reference's per-chunk logits budget; ``vocab_size`` is the whole vocabulary,
    default V_shard). For each launch: the GEMM epilogue writes the launch's logits (fp16 z - m of
    the logit's tile by default, fp32 for fp32 operands or FRX_TRAIN_LOGITS=f32) and partials; the
    per-row lse / entropy are produced by ``stats_fn(start, end, partials, T, rows_per_launch)``
    (single GPU: a local finalize; vocabulary-parallel: local merge + cross-rank exchange), which
    runs on the side stream with the launch's dlogits when there are several launches; the
    dlogits kernel writes the launch's dlogits (in the operands' 16-bit type) into a [B, V_shard]
    buffer. Then one d_hidden GEMM and one d_weight GEMM over all rows (on at most ``dweight_max_sms``
    SMs when it is positive, so a collective started by ``dhidden_fn`` can run beside it).
    """
    B, H = hidden_2d.shape
    V = weight.shape[0]
    dev = hidden_2d.device
    f32 = hidden_2d.dtype == torch.float32
    rel = _TILEREL_LOGITS and not f32
    ld_logits = ops.round_up(V, 8 if rel else 4)
    chunk = _train_launch_rows(_chunk_rows(chunk_size, B), B, ld_logits, 2 if rel else 4,
                               V if vocab_size is None else vocab_size)
    T = ops.n_vocab_tiles(V)
    n_chunks = (B + chunk - 1) // chunk
    overlap = _OVERLAP_DLOGITS and n_chunks > 1
    # Two logits (and partials) buffers when the statistics and dlogits of launch c run on a side
    # stream under the forward GEMM of launch c+1 (tensor-bound); the GEMM of launch c+2 waits for
    # them. The main stream then never waits on a cross-rank statistics exchange.
    n_buf = 2 if overlap else 1
    logits_bufs = [torch.empty(chunk, ld_logits, device=dev, dtype=torch.float16 if rel else torch.float32)
                   for _ in range(n_buf)]
    partials_bufs = [torch.empty(T, chunk, 4, device=dev, dtype=torch.float32) for _ in range(n_buf)]
    ldz = ops.round_up(V, 8)
    if f32:
        # fp32 operands (the reference's fp32 matmul): the forward GEMM runs on bf16x6 K-concatenated
        # operands (bias folded in), the fp32 dlogits are split into hi / mid / lo parts, and each
        # backward product is the sum of six bf16 GEMMs accumulated in an fp32 output.
        x_fwd, w_fwd = _fp32_k_operands(hidden_2d, weight, bias)
        fwd_bias = None
        dz_parts = torch.empty(3, B, ldz, device=dev, dtype=torch.bfloat16)
        dz32 = torch.empty(chunk, ops.round_up(V, 4), device=dev, dtype=torch.float32)
        dz = None
    else:
        x_fwd, w_fwd, fwd_bias = hidden_2d, weight, bias
        dz = torch.empty(B, ldz, device=dev, dtype=hidden_2d.dtype)
    main = torch.cuda.current_stream(dev)
    side = _side_stream(dev) if overlap else None
    if side is not None:
        side.wait_stream(main)
    done = [None, None]
    for c, start in enumerate(range(0, B, chunk)):
        end = min(start + chunk, B)
        rows = end - start
        buf = c % n_buf
        logits, partials = logits_bufs[buf], partials_bufs[buf]
        if done[buf] is not None:
            main.wait_event(done[buf])
        with ops.phase("frx.train.forward_chunk"):
            if rel:
                ops.fwd_partials(x_fwd[start:end], w_fwd, target_1d[start:end], partials, chunk, vocab_offset,
                                 logits_rel=logits, bias=fwd_bias)
            else:
                ops.fwd_partials(x_fwd[start:end], w_fwd, target_1d[start:end], partials, chunk, vocab_offset,
                                 logits=logits, bias=fwd_bias)

        def run_dlogits(logits=logits, partials=partials, start=start, end=end, rows=rows):
            with ops.phase("frx.train.stats"):
                stats_fn(start, end, partials, T, chunk)
            common = dict(rows=rows, vocab_shard=V, ce_weight=ce_weight, ent_weight=ent_weight,
                          g_ce=None if g_ce is None else g_ce[start:end],
                          g_ent=None if g_ent is None else g_ent[start:end],
                          vocab_offset=vocab_offset, ignore_index=ignore_index)
            if rel:
                ops.dlogits_tilerel(logits, partials, chunk, target_1d[start:end], lse[start:end],
                                    entropy[start:end], dz[start:end], **common)
            else:
                ops.dlogits(logits, target_1d[start:end], lse[start:end], entropy[start:end],
                            dz32 if f32 else dz[start:end], **common)
            if f32:
                ops.split_f32(dz32[:rows, :V], dz_parts[0, start:end], (_HI, _MID, _LO), part_stride=B * ldz)

        if side is None:
            run_dlogits()
        else:
            ready = torch.cuda.Event()
            ready.record(main)
            side.wait_event(ready)
            with torch.cuda.stream(side):
                run_dlogits()
                ev = torch.cuda.Event()
                ev.record(side)
            done[buf] = ev
    if side is not None:
        main.wait_stream(side)
        for t_ in logits_bufs + partials_bufs + [dz, lse, entropy, target_1d, g_ce, g_ent] + (
                [dz32, dz_parts] if f32 else []):
            if t_ is not None:
                t_.record_stream(side)
    del logits_bufs, partials_bufs, partials
    if f32:
        del x_fwd, w_fwd, dz32
        w_parts = _fp32_parts(weight)
        dh_pairs = [(dz_parts[i], w_parts[j]) for i, j in zip(ops.SPLIT_LEFT, ops.SPLIT_RIGHT)]
    else:
        dh_pairs = [(dz, weight)]
    with ops.phase("frx.train.dhidden"):
        if dhidden_fn is not None:
            d_hidden, pending = dhidden_fn(dh_pairs)
        else:
            d_hidden = torch.empty(B, H, device=dev, dtype=hidden_2d.dtype)
            for i, (a_op, b_op) in enumerate(dh_pairs):
                ops.gemm_dhidden(a_op, b_op, d_hidden, rows=B, vocab_shard=V, accumulate=i > 0)
            pending = None
    d_weight = torch.empty(V, H, device=dev, dtype=weight.dtype)
    with ops.phase("frx.train.dweight"):
        if f32:
            del w_parts, dh_pairs
            x_parts = _fp32_parts(hidden_2d)
            for n_, (i, j) in enumerate(zip(ops.SPLIT_LEFT, ops.SPLIT_RIGHT)):
                ops.gemm_dweight(dz_parts[i], x_parts[j], d_weight, rows=B, vocab_shard=V, accumulate=n_ > 0,
                                 max_sms=dweight_max_sms)
        else:
            ops.gemm_dweight(dz, hidden_2d, d_weight, rows=B, vocab_shard=V, max_sms=dweight_max_sms)
    d_bias = None
    if bias is not None:
        d_bias32 = torch.empty(V, device=dev, dtype=torch.float32)
        if f32:
            # the parts' column sums, added in a fixed order (hi + mid + lo = the fp32 dlogits)
            sums = torch.empty(3, V, device=dev, dtype=torch.float32)
            for i in range(3):
                ops.column_sums(dz_parts[i], sums[i], rows=B, cols=V)
            torch.add(sums[0], sums[1], out=d_bias32)
            d_bias32.add_(sums[2])
        else:
            ops.column_sums(dz, d_bias32, rows=B, cols=V)
        d_bias = d_bias32.to(bias.dtype)
    return d_hidden, d_weight, d_bias, pending


def _megakernel_fwd_bwd(hidden_2d, weight, target_1d, chunk_size, ce_weight, ent_weight, ignore_index, bias=None):
    B = hidden_2d.shape[0]
    V = weight.shape[0]
    dev = hidden_2d.device
    ce = torch.empty(B, device=dev, dtype=torch.float32)
    ent = torch.empty(B, device=dev, dtype=torch.float32)
    lse = torch.empty(B, device=dev, dtype=torch.float32)
    if B == 0:
        return ce, ent, torch.zeros_like(hidden_2d), torch.zeros_like(weight), \
            None if bias is None else torch.zeros_like(bias)

    def local_stats(start, end, partials, T, chunk):
        ops.finalize(
            partials, T, end - start, chunk, target=target_1d[start:end], vocab_size=V, ignore_index=ignore_index,
            ce=ce[start:end], entropy=ent[start:end], lse=lse[start:end],
        )

    d_hidden, d_weight, d_bias, _ = fwd_bwd_shard(
        hidden_2d, weight, target_1d, chunk_size, ce_weight, ent_weight, lse=lse, entropy=ent,
        ignore_index=ignore_index, stats_fn=local_stats, bias=bias,
    )
    return ce, ent, d_hidden, d_weight, d_bias


def _weighted_loss(ce: Tensor, ent: Tensor, ce_weight: float, ent_weight: float) -> Tensor:
    """0-d fp32 loss = ce_weight * sum(ce) + ent_weight * sum(ent) (reference gemm_kernel.py:897), reduced
    by one deterministic libfrx kernel."""
    loss = torch.empty((), device=ce.device, dtype=torch.float32)
    ops.loss_sum(ce, ent, loss, rows=ce.numel(), ce_weight=ce_weight, ent_weight=ent_weight)
    return loss


def _keep_grads(ctx, *grads) -> None:
    """Stores the precomputed gradients on the autograd node for _hand_over_grads (not through
    save_for_backward, whose extra reference would make autograd copy them into .grad)."""
    ctx.frx_grads = list(grads)


def _hand_over_grads(ctx, dloss: Tensor):
    """The gradients the forward precomputed, scaled by dloss (the reference's `d_hidden * dloss`,
    gemm_kernel.py:905-913) and handed to autograd.

    The scaling runs in place on the device (frx_scale_inplace, a no-op kernel when dloss is exactly
    1), so the host never waits for dloss; the node keeps no reference afterwards, so autograd
    stores the tensors as .grad without copying them. A second backward through the same graph
    (retain_graph=True) therefore has nothing left to hand over and raises."""
    grads = getattr(ctx, "frx_grads", None)
    if grads is None:
        raise RuntimeError("the gradients of this gemm_megakernel_fast call were already handed to autograd by an "
                           "earlier backward; a second backward through the same graph is not supported (call the "
                           "op again instead of using retain_graph=True)")
    ctx.frx_grads = None
    scale = dloss.detach().reshape(1)
    if scale.dtype != torch.float32:
        scale = scale.to(torch.float32)
    for g in grads:
        if g is not None:
            ops.scale_inplace(g, scale)
    return grads


class GemmMegakernel(torch.autograd.Function):
    """Training op: all gradient work runs in forward; backward only scales by dloss
    (reference GemmMegakernel, gemm_kernel.py:883-913)."""

    @staticmethod
    def forward(ctx, hidden_states, weight, target, bias, chunk_size, ce_weight, ent_weight):
        batch_shape, hidden_2d, weight_c, target_1d, bias_c = _prepare(hidden_states, weight, target, bias)
        ce, ent, d_hidden, d_weight, d_bias = _megakernel_fwd_bwd(
            hidden_2d, weight_c, target_1d, chunk_size, float(ce_weight), float(ent_weight), IGNORE_INDEX, bias_c,
        )
        loss = _weighted_loss(ce, ent, float(ce_weight), float(ent_weight))
        _keep_grads(ctx, d_hidden.view(hidden_states.shape), d_weight, d_bias)
        ce = ce.view(batch_shape)
        ent = ent.view(batch_shape)
        ctx.mark_non_differentiable(ce, ent)
        return loss, ce, ent

    @staticmethod
    def backward(ctx, dloss, _g_ce, _g_ent):
        d_hidden, d_weight, d_bias = _hand_over_grads(ctx, dloss)
        return d_hidden, d_weight, None, d_bias, None, None, None


def gemm_megakernel_fast(
    hidden_states: Tensor,
    weight: Tensor,
    target: Tensor,
    bias: Optional[Tensor] = None,
    chunk_size: int = 4096,
    ce_weight: float = 1.0,
    ent_weight: float = -1.0,
) -> Tuple[Tensor, Tensor, Tensor]:
    """Training megakernel. Returns (loss, ce_loss, entropy): loss is a scalar that requires
    grad; ce_loss and entropy are per-row and detached."""
    return GemmMegakernel.apply(hidden_states, weight, target, bias, chunk_size, ce_weight, ent_weight)


# The reference's Level-5 "fast" variant (gemm_kernel.py:713-764) has the same contract as the
# megakernel (gradients precomputed in forward, backward scales by dloss); here both names run
# the same sm_100a training path.
gemm_fused_ce_entropy_fast = gemm_megakernel_fast
GemmFusedCEEntropyFast = GemmMegakernel
