"""Vocabulary-parallel fused linear + CE + entropy over the GPUs of one node.

Each rank owns a contiguous slice [vocab_start, vocab_start + V_r) of the vocabulary (its rows
of the weight) and the full hidden states and targets. The forward exchanges only per-row
merged softmax statistics: every rank reduces its slice to (M, S, U, ZT) per row with the
fused GEMM epilogue + a local merge, all-gathers the [B, 4] fp32 rows (16 bytes per row per
rank) and merges them with the same associative rule as the per-tile merge
(reference merge: fast_reduction/gemm_ce_entropy_finalize.py:78-92). Every rank then holds the
full ce / entropy / lse.

Training: dlogits and d_weight of a slice are local; d_hidden is a sum over slices. Each rank
computes its partial d_hidden in fp32; on a side stream, overlapped with the d_weight GEMM, an NCCL
reduce-scatter sums every rank's share of the rows, the share is cast to the hidden dtype, and an
all-gather assembles d_hidden on every rank (FRX_DH_COLLECTIVE=allreduce: one fp32 all-reduce and a
full-size cast instead). An alternative (FRX_NVLS=1) fuses the sum into the d_hidden GEMM: its
epilogue adds every finished fp32 tile into all ranks' copies of a symmetric-memory buffer through
the NVSwitch (`frx_gemm_dhidden_multicast`, multimem.red). It is correct but slower on B200 at this
volume (512 MiB of reductions per rank: the fused GEMM took 13.5 ms vs 11.5 ms + overlapped NCCL at
2 GPUs, 6.8 ms vs 2.8 ms at 8 GPUs), so NCCL is the default.

The reference is single-GPU; this module adds the sharded path around the same libfrx kernels.
"""

from __future__ import annotations

import os
from typing import Optional, Tuple

import torch
import torch.distributed as dist
from torch import Tensor

from . import gemm_kernel as gk
from . import ops


# FRX_NVLS=1 selects the multicast-fused d_hidden reduction (when the GPUs support NVLS).
_USE_NVLS = os.environ.get("FRX_NVLS", "0") == "1"
_DH_COLLECTIVE = os.environ.get("FRX_DH_COLLECTIVE", "rs_ag")
# The persistent d_weight GEMM holds every SM, so the d_hidden reduce-scatter / all-gather queued beside
# it runs after it. With k SMs left free (frx_gemm_dweight_sms) and the collective on a communicator of
# its own limited to k NCCL CTAs on a high-priority stream, it runs beside the GEMM instead, at the
# price of the GEMM's extra waves on fewer SMs. Measured at 8 GPUs (headline shape): k = 32 gives a
# 10.01 ms training step against 10.32 ms with no SMs left free; k = 20 gave 10.95 ms and k = 4 15.4 ms
# (too few NCCL CTAs: the collective outlasts the GEMM). FRX_DH_OVERLAP_SMS=k forces k (0: never);
# by default _dh_overlap_sms decides per shape.
_DH_OVERLAP_ENV = os.environ.get("FRX_DH_OVERLAP_SMS", "auto")
_DH_OVERLAP_CTAS = 32
# Rates of the estimate in _dh_overlap_sms, measured at 8 GPUs on the headline shape: the d_weight
# GEMM's bf16 rate at the clocks short per-rank steps reach, and the NCCL reduce-scatter + all-gather
# rate per rank (bytes sent or received per second).
_DW_FLOPS = 1.6e15
_DH_COLLECTIVE_BYTES_PER_S = 0.78e12
_dh_groups: dict = {}


def _dh_overlap_sms(world: int, rows: int, hidden: int, vocab_shard: int, sms: int, elem_bytes: int) -> int:
    """SMs to leave free of the d_weight GEMM for the d_hidden collective: _DH_OVERLAP_CTAS when the
    GEMM's extra time on the remaining SMs (whole waves of 256 x 512 tiles over CTA pairs) is smaller
    than the collective it hides (fp32 reduce-scatter + 16-bit all-gather of the [rows, hidden] sum),
    else 0. This enables it at 8 GPUs for the headline shape and configs[4], and not at 2 or 4 GPUs
    where the d_weight GEMM is long and its extra waves cost more."""
    if _DH_OVERLAP_ENV != "auto":
        return max(0, int(_DH_OVERLAP_ENV or 0))
    if world < 2:
        return 0
    k = _DH_OVERLAP_CTAS
    tiles = -(-vocab_shard // 256) * -(-hidden // 512)
    pairs_all, pairs_left = sms // 2, (sms - k) // 2
    if pairs_left < 1:
        return 0
    waves_all, waves_left = -(-tiles // pairs_all), -(-tiles // pairs_left)
    t_gemm = 2.0 * rows * hidden * vocab_shard / _DW_FLOPS
    extra = t_gemm * (waves_left - waves_all) / waves_all
    t_coll = rows * hidden * (4 + elem_bytes) * (world - 1) / world / _DH_COLLECTIVE_BYTES_PER_S
    return k if extra < t_coll else 0


def _dh_group(group, ctas: int):
    """A communicator over `group`'s ranks for the d_hidden collective, limited to `ctas` NCCL CTAs on
    a high-priority stream; created on first use (collective: every rank of `group` calls it)."""
    ranks = dist.get_process_group_ranks(group) if group is not None else list(range(dist.get_world_size()))
    # keyed by the members and the current default group, so a process group torn down and created
    # again (a new default group) never reuses a communicator of the old one
    key = (tuple(ranks), ctas, id(dist.group.WORLD))
    g = _dh_groups.get(key)
    if g is None:
        opts = dist.ProcessGroupNCCL.Options(is_high_priority_stream=True)
        opts.config.min_ctas = ctas
        opts.config.max_ctas = ctas
        g = dist.new_group(ranks=ranks, pg_options=opts, backend="nccl")
        _dh_groups[key] = g
    return g
# The d_hidden sum over ranks: "rs_ag" (default) reduce-scatters the fp32 contributions, casts this
# rank's rows to the hidden dtype and all-gathers them into d_hidden (25% fewer bytes over NVLink
# than an fp32 all-reduce, and no full-size cast afterwards); "allreduce" sums the whole fp32 matrix
# on every rank and casts it (for A/B measurement).
_nvls_buffers: dict = {}


def _nvls_dhidden_buffer(rows: int, hidden: int, device: torch.device, group):
    """Symmetric-memory fp32 [rows, hidden] buffer bound to an NVLS multicast object, cached per
    (group, shape, device), or (None, None) when multicast is unavailable. Collective: every rank
    of the group calls it with the same shape."""
    pg = group if group is not None else dist.group.WORLD
    key = (id(pg), rows, hidden, device.index)
    hit = _nvls_buffers.get(key)
    if hit is None:
        hit = (None, None)
        try:
            import torch.distributed._symmetric_memory as symm

            buf = symm.empty(rows, hidden, dtype=torch.float32, device=device)
            hdl = symm.rendezvous(buf, pg)
            if hdl.multicast_ptr:
                hit = (buf, hdl)
        except Exception:
            hit = (None, None)
        _nvls_buffers[key] = hit
    return hit


def shard_bounds(vocab_size: int, world_size: int, rank: int) -> Tuple[int, int]:
    """[start, end) of `rank`'s vocabulary slice: an even split, the remainder spread over the
    first ranks (shards need not be multiples of the 256-column tile)."""
    if world_size < 1 or not (0 <= rank < world_size):
        raise ValueError(f"bad rank {rank} for world size {world_size}")
    base, rem = divmod(vocab_size, world_size)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def merge_rows(merged_all: Tensor, target_1d: Tensor, vocab_size: int, ignore_index: int,
               ce: Optional[Tensor] = None, entropy: Optional[Tensor] = None, lse: Optional[Tensor] = None,
               log_probs: Optional[Tensor] = None) -> None:
    """[world, B, 4] gathered per-shard statistics -> per-row outputs (frx_finalize over shards)."""
    world, B, _ = merged_all.shape
    ops.finalize(merged_all, world, B, B, target=target_1d, vocab_size=vocab_size, ignore_index=ignore_index,
                 ce=ce, entropy=entropy, lse=lse, log_probs=log_probs)


def _gather_stats(local: Tensor, group) -> Tensor:
    """All-gathers the [rows, 4] per-row statistics of every rank into [world, rows, 4]."""
    world = dist.get_world_size(group)
    out = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), device=local.device, dtype=local.dtype)
    dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    return out.view((world,) + tuple(local.shape))


def vocab_parallel_ce_entropy(
    hidden_states: Tensor,
    weight_shard: Tensor,
    target: Tensor,
    vocab_start: int,
    vocab_size: int,
    group=None,
    chunk_size: int = 4096,
    ignore_index: int = gk.IGNORE_INDEX,
    bias_shard: Optional[Tensor] = None,
) -> Tuple[Tensor, Tensor, Tensor]:
    """Forward over this rank's vocabulary slice; returns the full (ce_loss, entropy, log_probs)
    (identical on every rank), shaped like hidden_states.shape[:-1]. ``bias_shard`` is the bias of
    this rank's vocabulary rows, if any."""
    if weight_shard.dim() == 2 and weight_shard.shape[0] == 0:
        raise ValueError("every rank needs a non-empty vocabulary slice (vocab_size >= world size)")
    batch_shape, hidden_2d, weight_shard, target_1d, bias_shard = gk._prepare(hidden_states, weight_shard, target,
                                                                              bias_shard, allow_host=True)
    B = hidden_2d.shape[0]
    host_dev = gk._input_device(hidden_2d, weight_shard, target_1d, bias_shard)
    dev = hidden_2d.device if host_dev is None else host_dev
    local = torch.empty(B, 4, device=dev, dtype=torch.float32)
    if host_dev is not None and hidden_2d.dtype == torch.float32:
        # fp32 operands are split on the device before the GEMM: upload them whole first
        hidden_2d, weight_shard, target_1d, bias_shard = (
            None if t is None else t.to(host_dev, non_blocking=True)
            for t in (hidden_2d, weight_shard, target_1d, bias_shard))
        host_dev = None
    if host_dev is None:
        if hidden_2d.dtype == torch.float32:
            hidden_2d, weight_shard = gk._fp32_k_operands(hidden_2d, weight_shard, bias_shard)
            bias_shard = None
        gk.forward_stats(hidden_2d, weight_shard, target_1d, chunk_size, vocab_offset=vocab_start, merged=local,
                         vocab_size=vocab_size, ignore_index=ignore_index, bias=bias_shard)
        t_d = target_1d
    else:
        # Host inputs: each rank uploads 1/world of the hidden rows over its own PCIe link and the
        # rows are all-gathered over NVLink, while the weight slice streams in under the GEMMs.
        world = dist.get_world_size(group)
        share = (dist.get_rank(group), world, lambda part: _gather_stats(part, group).view(-1, part.shape[1]))
        t_d = target_1d.to(dev, non_blocking=True)
        gk.forward_stats_from_host(hidden_2d, weight_shard, t_d, dev, bias=bias_shard, vocab_offset=vocab_start,
                                   vocab_size=vocab_size, ignore_index=ignore_index, merged=local,
                                   hidden_share=share if world > 1 else None)
    gathered = _gather_stats(local, group)
    ce = torch.empty(B, device=dev, dtype=torch.float32)
    ent = torch.empty(B, device=dev, dtype=torch.float32)
    logp = torch.empty(B, device=dev, dtype=torch.float32)
    merge_rows(gathered, t_d, vocab_size, ignore_index, ce=ce, entropy=ent, log_probs=logp)
    return gk._results_to(hidden_states.device, batch_shape, ce, ent, logp)


def _fwd_bwd_vocab_parallel(hidden_2d, weight_shard, target_1d, vocab_start, vocab_size, group, chunk_size,
                            ce_weight, ent_weight, ignore_index, bias_shard=None):
    B, H = hidden_2d.shape
    dev = hidden_2d.device
    ce = torch.empty(B, device=dev, dtype=torch.float32)
    ent = torch.empty(B, device=dev, dtype=torch.float32)
    lse = torch.empty(B, device=dev, dtype=torch.float32)
    local = torch.empty(B, 4, device=dev, dtype=torch.float32)
    Vr = weight_shard.shape[0]

    def exchange_stats(start, end, partials, T, chunk):
        rows = end - start
        ops.finalize(partials, T, rows, chunk, merged=local[start:end])
        with ops.phase("frx.vp.stats_allgather"):
            gathered = _gather_stats(local[start:end], group)
        merge_rows(gathered, target_1d[start:end], vocab_size, ignore_index, ce=ce[start:end],
                   entropy=ent[start:end], lse=lse[start:end])

    if Vr == 0:
        raise ValueError("every rank needs a non-empty vocabulary slice")
    buf, hdl = (None, None)
    dweight_sms = 0
    if _USE_NVLS and dist.get_world_size(group) > 1:
        buf, hdl = _nvls_dhidden_buffer(B, H, dev, group)
    if buf is not None:
        # Zeroed before the forward chunks: their all-gathers order every rank's zeroing before any
        # rank's d_hidden GEMM starts adding into the buffers.
        buf.zero_()

        def dhidden_fn(pairs):
            for a_op, b_op in pairs:  # multimem.red adds every product into every rank's copy
                ops.gemm_dhidden_multicast(a_op, b_op, hdl.multicast_ptr, H, rows=B, vocab_shard=Vr, device=dev)
            return None, None
    elif _DH_COLLECTIVE == "allreduce":
        def dhidden_fn(pairs):
            dh = torch.empty(B, H, device=dev, dtype=torch.float32)
            for i, (a_op, b_op) in enumerate(pairs):
                ops.gemm_dhidden(a_op, b_op, dh, rows=B, vocab_shard=Vr, accumulate=i > 0)
            return dh, _allreduce_async(dh, group)
    else:
        world = dist.get_world_size(group)
        share = (B + world - 1) // world
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        free = _dh_overlap_sms(world, B, H, Vr, sms, hidden_2d.element_size())
        if free > 0 and world > 1:
            dweight_sms = max(2, sms - free)
            dh_group = _dh_group(group, free)
        else:
            dweight_sms, dh_group = 0, group

        def dhidden_fn(pairs):
            # [world * share, H] so that reduce-scatter hands every rank `share` rows; the padded rows
            # past B are never written and only ever reach the padded rows of the result
            dh = torch.empty(world * share, H, device=dev, dtype=torch.float32)
            for i, (a_op, b_op) in enumerate(pairs):
                ops.gemm_dhidden(a_op, b_op, dh, rows=B, vocab_shard=Vr, accumulate=i > 0)
            return None, _reduce_scatter_gather_async(dh, share, hidden_2d.dtype, dh_group)

    d_hidden_f32, d_weight, d_bias, pending = gk.fwd_bwd_shard(
        hidden_2d, weight_shard, target_1d, chunk_size, ce_weight, ent_weight, lse=lse, entropy=ent,
        vocab_offset=vocab_start, ignore_index=ignore_index, stats_fn=exchange_stats, dhidden_fn=dhidden_fn,
        bias=bias_shard, vocab_size=vocab_size, dweight_max_sms=dweight_sms,
    )
    if buf is not None:
        hdl.barrier()  # every rank's reductions have landed in every copy
        return ce, ent, buf.to(hidden_2d.dtype), d_weight, d_bias
    pending.wait_into_current()
    if d_hidden_f32 is None:  # reduce-scatter + all-gather: already summed and in the hidden dtype
        return ce, ent, pending.result[:B], d_weight, d_bias
    return ce, ent, d_hidden_f32.to(hidden_2d.dtype), d_weight, d_bias


class _PendingAllReduce:
    def __init__(self, event: torch.cuda.Event, result: Optional[Tensor] = None):
        self.event = event
        self.result = result

    def wait_into_current(self):
        torch.cuda.current_stream().wait_event(self.event)


_side_streams: dict[int, torch.cuda.Stream] = {}


def _allreduce_async(t: Tensor, group) -> _PendingAllReduce:
    """All-reduce `t` (SUM) on a side stream, so the caller's next kernel (the d_weight GEMM)
    overlaps the NVLink transfer; returns a handle whose wait orders the caller's stream after it."""
    dev = t.device.index
    side = _side_streams.get(dev)
    if side is None:
        side = torch.cuda.Stream(device=t.device)
        _side_streams[dev] = side
    main = torch.cuda.current_stream()
    side.wait_stream(main)
    with torch.cuda.stream(side), ops.phase("frx.vp.dhidden_allreduce"):
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
        done = torch.cuda.Event()
        done.record(side)
    t.record_stream(side)
    return _PendingAllReduce(done)


def _reduce_scatter_gather_async(dh32: Tensor, share: int, dtype: torch.dtype, group) -> _PendingAllReduce:
    """Sum of every rank's fp32 [world * share, H] contribution, in `dtype`, on a side stream (so it
    overlaps the caller's next kernel, the d_weight GEMM): reduce-scatter in fp32 (this rank gets
    rows [rank * share, (rank + 1) * share) summed), cast of those rows (bf16: libfrx's round to
    nearest, the hi part of frx_split_f32), all-gather of the casts. Returns a handle whose wait
    orders the caller's stream after it and whose `result` is the [world * share, H] sum."""
    dev = dh32.device.index
    side = _side_streams.get(dev)
    if side is None:
        side = torch.cuda.Stream(device=dh32.device)
        _side_streams[dev] = side
    H = dh32.shape[1]
    world = dh32.shape[0] // share
    main = torch.cuda.current_stream()
    side.wait_stream(main)
    with torch.cuda.stream(side), ops.phase("frx.vp.dhidden_reduce_scatter_gather"):
        part32 = torch.empty(share, H, device=dh32.device, dtype=torch.float32)
        dist.reduce_scatter_tensor(part32, dh32, op=dist.ReduceOp.SUM, group=group)
        if dtype == torch.float32:
            part = part32
        elif dtype == torch.bfloat16:
            part = torch.empty(share, H, device=dh32.device, dtype=torch.bfloat16)
            ops.split_f32(part32, part, (ops.nat.FRX_PART_HI,), part_stride=0)
        else:
            part = part32.to(dtype)
        out = torch.empty(world * share, H, device=dh32.device, dtype=dtype)
        dist.all_gather_into_tensor(out, part, group=group)
        done = torch.cuda.Event()
        done.record(side)
    for t in (dh32, part32, part, out):
        t.record_stream(side)
    return _PendingAllReduce(done, out)


class VocabParallelMegakernel(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden_states, weight_shard, target, vocab_start, vocab_size, group, chunk_size, ce_weight,
                ent_weight, bias_shard):
        batch_shape, hidden_2d, weight_c, target_1d, bias_c = gk._prepare(hidden_states, weight_shard, target,
                                                                          bias_shard)
        ce, ent, d_hidden, d_weight, d_bias = _fwd_bwd_vocab_parallel(
            hidden_2d, weight_c, target_1d, vocab_start, vocab_size, group, chunk_size, float(ce_weight),
            float(ent_weight), gk.IGNORE_INDEX, bias_c,
        )
        loss = gk._weighted_loss(ce, ent, float(ce_weight), float(ent_weight))
        gk._keep_grads(ctx, d_hidden.view(hidden_states.shape), d_weight, d_bias)
        ce = ce.view(batch_shape)
        ent = ent.view(batch_shape)
        ctx.mark_non_differentiable(ce, ent)
        return loss, ce, ent

    @staticmethod
    def backward(ctx, dloss, _g_ce, _g_ent):
        d_hidden, d_weight, d_bias = gk._hand_over_grads(ctx, dloss)
        return d_hidden, d_weight, None, None, None, None, None, None, None, d_bias


def vocab_parallel_megakernel(
    hidden_states: Tensor,
    weight_shard: Tensor,
    target: Tensor,
    vocab_start: int,
    vocab_size: int,
    group=None,
    chunk_size: int = 4096,
    ce_weight: float = 1.0,
    ent_weight: float = -1.0,
    bias_shard: Optional[Tensor] = None,
) -> Tuple[Tensor, Tensor, Tensor]:
    """Vocabulary-parallel gemm_megakernel_fast. Returns (loss, ce_loss, entropy), identical on
    every rank; loss.backward() gives every rank the full d_hidden and its own weight-slice (and
    bias-slice) gradient."""
    return VocabParallelMegakernel.apply(hidden_states, weight_shard, target, vocab_start, vocab_size, group,
                                         chunk_size, ce_weight, ent_weight, bias_shard)
