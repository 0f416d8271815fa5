"""Tensor-level wrappers over the libfrx C ABI (one function per entry point).

These functions take torch tensors, validate them, and pass raw device pointers plus sizes
to libfrx on the tensors' current CUDA stream. Outputs are written into caller-provided
tensors, as in the reference's custom ops (`mutates_args`, e.g.
fast_reduction/gemm_ce_entropy_finalize.py:123-148, cute_dlogits.py:121-159).
"""

from __future__ import annotations

import contextlib
import os

import torch

from . import _native as nat

VOCAB_TILE = nat.FRX_VOCAB_TILE
# Never equal to a real target id: disables the ignore_index rule.
NO_IGNORE = -(2**63)

# Optional launch observer (used by bench.py to time each libfrx kernel with CUDA events on the
# launching stream): an object with before(name, device) / after(name, device), or None.
_observer = None


def set_launch_observer(observer):
    """Installs `observer` (or None) and returns the previous one."""
    global _observer
    prev, _observer = _observer, observer
    return prev


# NVTX ranges (visible in Nsight Systems / Nsight Compute timelines): one per libfrx launch, named
# "frx.<entry point>", inside the phase ranges of the Python layer. FRX_NVTX=0 turns them off.
_NVTX = os.environ.get("FRX_NVTX", "1") != "0"


def _nvtx_push(name: str) -> bool:
    if not _NVTX:
        return False
    try:
        torch.cuda.nvtx.range_push(name)
        return True
    except Exception:  # a torch build without NVTX
        return False


@contextlib.contextmanager
def phase(name: str):
    """NVTX range around one phase of the path (e.g. "frx.train.dhidden")."""
    pushed = _nvtx_push(name)
    try:
        yield
    finally:
        if pushed:
            torch.cuda.nvtx.range_pop()


def _launch(name: str, dev: torch.device, call) -> int:
    pushed = _nvtx_push("frx." + name)
    try:
        obs = _observer
        if obs is None:
            return call()
        obs.before(name, dev)
        rc = call()
        obs.after(name, dev)
        return rc
    finally:
        if pushed:
            torch.cuda.nvtx.range_pop()


def n_vocab_tiles(vocab_shard: int) -> int:
    return (vocab_shard + VOCAB_TILE - 1) // VOCAB_TILE


def round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


# Operand types of the tcgen05 GEMMs (kind::f16: both operands bf16, or both fp16).
_GEMM_DTYPES = {torch.bfloat16: nat.FRX_DTYPE_BF16, torch.float16: nat.FRX_DTYPE_F16}
_OUT_DTYPES = {**_GEMM_DTYPES, torch.float32: nat.FRX_DTYPE_F32}


def _gemm_dtype(*tensors: torch.Tensor) -> int:
    """FRX dtype code shared by the GEMM operands; raises unless all are bf16 or all fp16."""
    dts = {t.dtype for t in tensors}
    if len(dts) != 1 or next(iter(dts)) not in _GEMM_DTYPES:
        raise TypeError(f"GEMM operands must all be bfloat16 or all float16, got {sorted(map(str, dts))}")
    return _GEMM_DTYPES[next(iter(dts))]


def _require_cuda(*tensors: torch.Tensor | None) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("fast_reduction (B200 engine) requires CUDA tensors; got a tensor on " + str(t.device))
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"all tensors must be on one device, got {dev} and {t.device}")
    return dev


def _row_major(t: torch.Tensor, name: str) -> int:
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be a 2-D tensor with unit column stride, got shape {tuple(t.shape)} "
                         f"stride {t.stride()}")
    return t.stride(0)


def fwd_partials(
    hidden: torch.Tensor,
    weight: torch.Tensor,
    target: torch.Tensor | None,
    partials: torch.Tensor,
    tile_stride: int,
    vocab_offset: int = 0,
    logits: torch.Tensor | None = None,
    bias: torch.Tensor | None = None,
    logits_rel: torch.Tensor | None = None,
) -> None:
    """partials[t, r] <- (m, s, u, zt) of z = hidden @ weight.T (+ bias) over vocab tile t (see include/frx.h).

    Optionally also writes every logit: fp32 ``logits`` (frx_fwd_partials), or fp16 ``logits_rel`` =
    z - m of the logit's tile (frx_fwd_partials_tilerel, half the bytes)."""
    dev = _require_cuda(hidden, weight, target, partials, logits, bias, logits_rel)
    ldh = _row_major(hidden, "hidden")
    ldw = _row_major(weight, "weight")
    rows, hdim = hidden.shape
    vshard = weight.shape[0]
    if weight.shape[1] != hdim:
        raise ValueError(f"hidden dim mismatch: hidden {tuple(hidden.shape)} vs weight {tuple(weight.shape)}")
    dt = _gemm_dtype(hidden, weight)
    if target is not None and (target.dtype != torch.int64 or not target.is_contiguous() or target.numel() < rows):
        raise ValueError("target must be a contiguous int64 tensor with one id per row")
    if partials.dtype != torch.float32 or not partials.is_contiguous():
        raise ValueError("partials must be contiguous float32")
    if tile_stride < rows or partials.numel() < 4 * ((n_vocab_tiles(vshard) - 1) * tile_stride + rows):
        raise ValueError("partials buffer too small")
    if bias is not None and (bias.dtype != hidden.dtype or not bias.is_contiguous() or bias.numel() != vshard):
        raise ValueError("bias must be a contiguous tensor of the weight's dtype with one value per vocabulary row "
                         "of the shard")
    ldl = 0
    if logits is not None:
        ldl = _row_major(logits, "logits")
        if logits.dtype != torch.float32 or logits.shape[0] < rows or logits.shape[1] < vshard:
            raise ValueError("logits must be float32 [rows, >= vocab_shard]")
    lib = nat.load()
    if logits_rel is not None:
        if logits is not None:
            raise ValueError("pass at most one of logits and logits_rel")
        ldr = _row_major(logits_rel, "logits_rel")
        if logits_rel.dtype != torch.float16 or logits_rel.shape[0] < rows or logits_rel.shape[1] < vshard:
            raise ValueError("logits_rel must be float16 [rows, >= vocab_shard]")
        rc = _launch("fwd_partials", dev, lambda: lib.frx_fwd_partials_tilerel(
            hidden.data_ptr(), ldh, weight.data_ptr(), ldw, dt, nat.ptr(bias), nat.ptr(target), rows, vshard, hdim,
            vocab_offset, partials.data_ptr(), tile_stride, logits_rel.data_ptr(), ldr,
            nat.status_word(dev).data_ptr(), nat.stream_of(dev),
        ))
        nat.check(rc, "frx_fwd_partials_tilerel")
        return
    rc = _launch("fwd_partials", dev, lambda: lib.frx_fwd_partials(
        hidden.data_ptr(), ldh, weight.data_ptr(), ldw, dt, nat.ptr(bias), nat.ptr(target), rows, vshard, hdim,
        vocab_offset,
        partials.data_ptr(), tile_stride, nat.ptr(logits), ldl, nat.status_word(dev).data_ptr(), nat.stream_of(dev),
    ))
    nat.check(rc, "frx_fwd_partials")


def finalize(
    partials: torch.Tensor,
    n_tiles: int,
    rows: int,
    tile_stride: int,
    *,
    ref_layout: bool = False,
    ignore_negative: bool = False,
    target: torch.Tensor | None = None,
    vocab_size: int = 0,
    ignore_index: int = NO_IGNORE,
    ce: torch.Tensor | None = None,
    entropy: torch.Tensor | None = None,
    lse: torch.Tensor | None = None,
    log_probs: torch.Tensor | None = None,
    merged: torch.Tensor | None = None,
) -> None:
    """Merges [n_tiles, tile_stride] float4 partials into per-row outputs (any may be None)."""
    dev = _require_cuda(partials, target, ce, entropy, lse, log_probs, merged)
    if partials.dtype != torch.float32 or not partials.is_contiguous():
        raise ValueError("partials must be contiguous float32")
    if partials.numel() < 4 * n_tiles * tile_stride or tile_stride < rows:
        raise ValueError("partials buffer smaller than n_tiles * tile_stride float4")
    for name, t in (("ce", ce), ("entropy", entropy), ("lse", lse), ("log_probs", log_probs)):
        if t is not None and (t.dtype != torch.float32 or not t.is_contiguous() or t.numel() < rows):
            raise ValueError(f"{name} must be contiguous float32 with >= rows elements")
    if merged is not None and (merged.dtype != torch.float32 or not merged.is_contiguous()
                               or merged.numel() < 4 * rows):
        raise ValueError("merged must be contiguous float32 [rows, 4]")
    if target is not None and (target.dtype != torch.int64 or not target.is_contiguous() or target.numel() < rows):
        raise ValueError("target must be a contiguous int64 tensor with one id per row")
    lib = nat.load()
    rc = _launch("finalize", dev, lambda: lib.frx_finalize(
        partials.data_ptr(), n_tiles, rows, tile_stride,
        (nat.FRX_PARTIALS_REF_LAYOUT if ref_layout else 0)
        | (nat.FRX_IGNORE_NEGATIVE_TARGETS if ignore_negative else 0),
        nat.ptr(target), vocab_size, ignore_index, nat.ptr(ce), nat.ptr(entropy), nat.ptr(lse), nat.ptr(log_probs),
        nat.ptr(merged), nat.status_word(dev).data_ptr(), nat.stream_of(dev),
    ))
    nat.check(rc, "frx_finalize")


def dlogits(
    logits: torch.Tensor,
    target: torch.Tensor | None,
    lse: torch.Tensor,
    entropy: torch.Tensor,
    out: torch.Tensor,
    *,
    rows: int,
    vocab_shard: int,
    g_ce: torch.Tensor | None = None,
    g_ent: torch.Tensor | None = None,
    ce_weight: float = 1.0,
    ent_weight: float = -1.0,
    vocab_offset: int = 0,
    ignore_index: int = NO_IGNORE,
) -> None:
    """out[r, j] <- d(sum g_ce*ce + g_ent*H)/dz[r, j] from fp32 logits (bf16, fp16 or fp32 out)."""
    dev = _require_cuda(logits, target, lse, entropy, out, g_ce, g_ent)
    ldl = _row_major(logits, "logits")
    ldo = _row_major(out, "dlogits")
    if logits.dtype != torch.float32:
        raise TypeError("logits must be float32")
    odt = _OUT_DTYPES.get(out.dtype)
    if odt is None:
        raise TypeError("dlogits output must be bfloat16, float16 or float32")
    if logits.shape[0] < rows or out.shape[0] < rows or logits.shape[1] < vocab_shard or out.shape[1] < vocab_shard:
        raise ValueError("logits/out smaller than [rows, vocab_shard]")
    for name, t in (("lse", lse), ("entropy", entropy), ("g_ce", g_ce), ("g_ent", g_ent)):
        if t is not None and (t.dtype != torch.float32 or not t.is_contiguous() or t.numel() < rows):
            raise ValueError(f"{name} must be contiguous float32 with >= rows elements")
    if target is not None and (target.dtype != torch.int64 or not target.is_contiguous() or target.numel() < rows):
        raise ValueError("target must be a contiguous int64 tensor with one id per row")
    lib = nat.load()
    rc = _launch("dlogits", dev, lambda: lib.frx_dlogits(
        logits.data_ptr(), ldl, nat.ptr(target), lse.data_ptr(), entropy.data_ptr(), nat.ptr(g_ce), nat.ptr(g_ent),
        float(ce_weight), float(ent_weight), out.data_ptr(), ldo, odt, rows, vocab_shard, vocab_offset, ignore_index,
        nat.stream_of(dev),
    ))
    nat.check(rc, "frx_dlogits")


def dlogits_tilerel(
    logits_rel: torch.Tensor,
    partials: torch.Tensor,
    tile_stride: int,
    target: torch.Tensor | None,
    lse: torch.Tensor,
    entropy: torch.Tensor,
    out: torch.Tensor,
    *,
    rows: int,
    vocab_shard: int,
    g_ce: torch.Tensor | None = None,
    g_ent: torch.Tensor | None = None,
    ce_weight: float = 1.0,
    ent_weight: float = -1.0,
    vocab_offset: int = 0,
    ignore_index: int = NO_IGNORE,
) -> None:
    """dlogits (as `dlogits`) from fp16 tile-relative logits z - m_t and the partials holding each tile's
    maximum m_t (the outputs of one fwd_partials launch with logits_rel)."""
    dev = _require_cuda(logits_rel, partials, target, lse, entropy, out, g_ce, g_ent)
    ldl = _row_major(logits_rel, "logits_rel")
    ldo = _row_major(out, "dlogits")
    if logits_rel.dtype != torch.float16:
        raise TypeError("logits_rel must be float16")
    odt = _OUT_DTYPES.get(out.dtype)
    if odt is None:
        raise TypeError("dlogits output must be bfloat16, float16 or float32")
    if (logits_rel.shape[0] < rows or out.shape[0] < rows or logits_rel.shape[1] < vocab_shard
            or out.shape[1] < vocab_shard):
        raise ValueError("logits_rel/out smaller than [rows, vocab_shard]")
    if partials.dtype != torch.float32 or not partials.is_contiguous() or tile_stride < rows or \
            partials.numel() < 4 * ((n_vocab_tiles(vocab_shard) - 1) * tile_stride + rows):
        raise ValueError("partials must be contiguous float32 covering every tile of the launch")
    for name, t in (("lse", lse), ("entropy", entropy), ("g_ce", g_ce), ("g_ent", g_ent)):
        if t is not None and (t.dtype != torch.float32 or not t.is_contiguous() or t.numel() < rows):
            raise ValueError(f"{name} must be contiguous float32 with >= rows elements")
    if target is not None and (target.dtype != torch.int64 or not target.is_contiguous() or target.numel() < rows):
        raise ValueError("target must be a contiguous int64 tensor with one id per row")
    lib = nat.load()
    rc = _launch("dlogits", dev, lambda: lib.frx_dlogits_tilerel(
        logits_rel.data_ptr(), ldl, partials.data_ptr(), tile_stride, nat.ptr(target), lse.data_ptr(),
        entropy.data_ptr(), nat.ptr(g_ce), nat.ptr(g_ent), float(ce_weight), float(ent_weight), out.data_ptr(), ldo,
        odt, rows, vocab_shard, vocab_offset, ignore_index, nat.stream_of(dev),
    ))
    nat.check(rc, "frx_dlogits_tilerel")


def _out_dtype(t: torch.Tensor, accumulate: bool = False) -> int:
    if t.dtype not in _OUT_DTYPES:
        raise TypeError("GEMM output must be bfloat16, float16 or float32")
    if accumulate:
        if t.dtype != torch.float32:
            raise TypeError("accumulating GEMM output must be float32")
        return _OUT_DTYPES[t.dtype] | nat.FRX_OUT_ACCUMULATE
    return _OUT_DTYPES[t.dtype]


# bf16x6 emulation of an fp32 product (Henry, Tang, Heinecke, ARITH 2019): the left operand's parts
# in this order times the right operand's parts in the other order sum to the product up to the
# mid*lo, lo*mid and lo*lo terms.
SPLIT_LEFT = (nat.FRX_PART_HI, nat.FRX_PART_HI, nat.FRX_PART_MID, nat.FRX_PART_HI, nat.FRX_PART_LO, nat.FRX_PART_MID)
SPLIT_RIGHT = (nat.FRX_PART_HI, nat.FRX_PART_MID, nat.FRX_PART_HI, nat.FRX_PART_LO, nat.FRX_PART_HI, nat.FRX_PART_MID)


def split_f32(x: torch.Tensor, out: torch.Tensor, parts, *, part_stride: int) -> None:
    """out (bf16, row stride out.stride(0)) + p * part_stride <- part parts[p] (hi / mid / lo) of the
    fp32 matrix x [rows, cols]: x = hi + mid + lo to ~24 bits (frx_split_f32)."""
    dev = _require_cuda(x, out)
    if x.dtype != torch.float32 or out.dtype != torch.bfloat16:
        raise TypeError("split_f32 takes a float32 matrix and writes bfloat16 parts")
    ldx = _row_major(x, "x")
    ldo = _row_major(out, "out")
    rows, cols = x.shape
    code = 0
    for p, sel in enumerate(parts):
        code |= int(sel) << (2 * p)
    lib = nat.load()
    rc = _launch("split_f32", dev, lambda: lib.frx_split_f32(
        x.data_ptr(), ldx, rows, cols, code, len(parts), out.data_ptr(), ldo, part_stride, nat.stream_of(dev)))
    nat.check(rc, "frx_split_f32")


def gemm_dhidden(dz: torch.Tensor, weight: torch.Tensor, out: torch.Tensor, *, rows: int, vocab_shard: int,
                 accumulate: bool = False) -> None:
    """out[rows, H] <- dz[rows, vocab_shard] @ weight[vocab_shard, H] (``accumulate``: fp32 out +=)."""
    dev = _require_cuda(dz, weight, out)
    dt = _gemm_dtype(dz, weight)
    ldz = _row_major(dz, "dz")
    ldw = _row_major(weight, "weight")
    ldo = _row_major(out, "d_hidden")
    hdim = weight.shape[1]
    if out.shape[0] < rows or out.shape[1] < hdim or weight.shape[0] < vocab_shard or dz.shape[1] < vocab_shard:
        raise ValueError("shape mismatch in gemm_dhidden")
    lib = nat.load()
    rc = _launch("gemm_dhidden", dev, lambda: lib.frx_gemm_dhidden(
        dz.data_ptr(), ldz, weight.data_ptr(), ldw, dt, out.data_ptr(), ldo, _out_dtype(out, accumulate), rows, hdim,
        vocab_shard,
        nat.status_word(dev).data_ptr(), nat.stream_of(dev),
    ))
    nat.check(rc, "frx_gemm_dhidden")


def gemm_dweight(dz: torch.Tensor, hidden: torch.Tensor, out: torch.Tensor, *, rows: int, vocab_shard: int,
                 accumulate: bool = False, max_sms: int = 0) -> None:
    """out[vocab_shard, H] <- dz[rows, vocab_shard]^T @ hidden[rows, H] (``accumulate``: fp32 out +=), on at
    most ``max_sms`` SMs when it is positive (frx_gemm_dweight_sms)."""
    dev = _require_cuda(dz, hidden, out)
    dt = _gemm_dtype(dz, hidden)
    ldz = _row_major(dz, "dz")
    ldh = _row_major(hidden, "hidden")
    ldo = _row_major(out, "d_weight")
    hdim = hidden.shape[1]
    if out.shape[0] < vocab_shard or out.shape[1] < hdim or hidden.shape[0] < rows or dz.shape[0] < rows:
        raise ValueError("shape mismatch in gemm_dweight")
    lib = nat.load()
    if max_sms > 0:
        rc = _launch("gemm_dweight", dev, lambda: lib.frx_gemm_dweight_sms(
            dz.data_ptr(), ldz, hidden.data_ptr(), ldh, dt, out.data_ptr(), ldo, _out_dtype(out, accumulate),
            vocab_shard, hdim, rows, int(max_sms), nat.status_word(dev).data_ptr(), nat.stream_of(dev),
        ))
        nat.check(rc, "frx_gemm_dweight_sms")
        return
    rc = _launch("gemm_dweight", dev, lambda: lib.frx_gemm_dweight(
        dz.data_ptr(), ldz, hidden.data_ptr(), ldh, dt, out.data_ptr(), ldo, _out_dtype(out, accumulate), vocab_shard,
        hdim, rows,
        nat.status_word(dev).data_ptr(), nat.stream_of(dev),
    ))
    nat.check(rc, "frx_gemm_dweight")


_LOGITS_DTYPES = {torch.bfloat16: nat.FRX_DTYPE_BF16, torch.float16: nat.FRX_DTYPE_F16,
                  torch.float32: nat.FRX_DTYPE_F32}


def logits_partials(logits: torch.Tensor, target: torch.Tensor | None, partials: torch.Tensor, tile_cols: int,
                    tile_stride: int) -> None:
    """partials[t, r] <- (m, s, u, zt) of logits[r, t*tile_cols : (t+1)*tile_cols] (any float dtype)."""
    dev = _require_cuda(logits, target, partials)
    ld = _row_major(logits, "logits")
    if logits.dtype not in _LOGITS_DTYPES:
        raise TypeError(f"logits must be bfloat16, float16 or float32, got {logits.dtype}")
    rows, cols = logits.shape
    if target is not None and (target.dtype != torch.int64 or not target.is_contiguous() or target.numel() < rows):
        raise ValueError("target must be a contiguous int64 tensor with one id per row")
    n_tiles = (cols + tile_cols - 1) // tile_cols
    if partials.dtype != torch.float32 or not partials.is_contiguous() or partials.numel() < 4 * n_tiles * tile_stride:
        raise ValueError("partials must be contiguous float32 with n_tiles * tile_stride float4")
    lib = nat.load()
    rc = _launch("logits_partials", dev, lambda: lib.frx_logits_partials(
        logits.data_ptr(), _LOGITS_DTYPES[logits.dtype], ld, rows, cols, nat.ptr(target), tile_cols,
        partials.data_ptr(), tile_stride, nat.stream_of(dev),
    ))
    nat.check(rc, "frx_logits_partials")


def column_sums(x: torch.Tensor, out: torch.Tensor, *, rows: int, cols: int) -> None:
    """out[c] <- sum_r x[r, c] for a bf16 / fp16 [rows, >= cols] matrix, fp32 out (deterministic order)."""
    dev = _require_cuda(x, out)
    ld = _row_major(x, "x")
    if x.dtype not in _GEMM_DTYPES:
        raise TypeError("column_sums input must be bfloat16 or float16")
    if out.dtype != torch.float32 or not out.is_contiguous() or out.numel() < cols:
        raise ValueError("out must be contiguous float32 with >= cols elements")
    lib = nat.load()
    rc = _launch("column_sums", dev, lambda: lib.frx_column_sums(
        x.data_ptr(), _GEMM_DTYPES[x.dtype], ld, rows, cols, out.data_ptr(), nat.stream_of(dev)))
    nat.check(rc, "frx_column_sums")


def gemm_dhidden_multicast(dz: torch.Tensor, weight: torch.Tensor, mc_ptr: int, ld_out: int, *, rows: int,
                           vocab_shard: int, device: torch.device) -> None:
    """Adds dz[rows, vocab_shard] @ weight[vocab_shard, H] into the fp32 matrix behind the NVLS
    multicast address `mc_ptr` (row stride ld_out): the cross-rank d_hidden sum inside the GEMM."""
    dev = _require_cuda(dz, weight)
    dt = _gemm_dtype(dz, weight)
    if not mc_ptr:
        raise ValueError("a multicast address is required")
    ldz = _row_major(dz, "dz")
    ldw = _row_major(weight, "weight")
    hdim = weight.shape[1]
    lib = nat.load()
    rc = _launch("gemm_dhidden", dev, lambda: lib.frx_gemm_dhidden_multicast(
        dz.data_ptr(), ldz, weight.data_ptr(), ldw, dt, mc_ptr, ld_out, rows, hdim, vocab_shard,
        nat.status_word(dev).data_ptr(), nat.stream_of(dev),
    ))
    nat.check(rc, "frx_gemm_dhidden_multicast")


def loss_sum(ce: torch.Tensor | None, entropy: torch.Tensor | None, loss: torch.Tensor, *, rows: int,
             ce_weight: float, ent_weight: float) -> None:
    """loss (0-d fp32) <- ce_weight * sum(ce[:rows]) + ent_weight * sum(entropy[:rows]) (deterministic)."""
    dev = _require_cuda(ce, entropy, loss)
    for name, t in (("ce", ce), ("entropy", entropy)):
        if t is not None and (t.dtype != torch.float32 or not t.is_contiguous() or t.numel() < rows):
            raise ValueError(f"{name} must be contiguous float32 with >= rows elements")
    if loss.dtype != torch.float32 or loss.numel() != 1:
        raise ValueError("loss must be a one-element float32 tensor")
    lib = nat.load()
    rc = _launch("loss_sum", dev, lambda: lib.frx_loss_sum(
        nat.ptr(ce), nat.ptr(entropy), rows, float(ce_weight), float(ent_weight), loss.data_ptr(), nat.stream_of(dev)))
    nat.check(rc, "frx_loss_sum")


def scale_inplace(x: torch.Tensor, scale: torch.Tensor) -> None:
    """x *= scale[0] on the device (a no-op kernel when the scale is exactly 1; no host synchronisation)."""
    dev = _require_cuda(x, scale)
    if not x.is_contiguous() or x.dtype not in _OUT_DTYPES:
        raise ValueError("x must be a contiguous bfloat16, float16 or float32 tensor")
    if scale.dtype != torch.float32 or scale.numel() != 1:
        raise ValueError("scale must be a one-element float32 tensor")
    lib = nat.load()
    rc = _launch("scale_inplace", dev, lambda: lib.frx_scale_inplace(
        x.data_ptr(), _OUT_DTYPES[x.dtype], x.numel(), scale.data_ptr(), nat.stream_of(dev)))
    nat.check(rc, "frx_scale_inplace")
