"""CPU oracle: a restatement of the reference's algorithm for the fused linear + CE + entropy path.

TEST INFRASTRUCTURE ONLY. This module is the checker: only tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / --impl reference legs may import it. The product (fast_reduction,
libfrx.so) never imports or calls it and has no CPU fallback.

Every function cites the reference code (justinchiu/fast-reduction) whose behaviour it restates.
Pinning: tests/test_oracle.py checks these functions against golden vectors produced by
running the reference's own fast_reduction/baseline.py in the build container
(tests/golden/make_golden.py), and against the reference's finalize known-answer construction
(tests/test_ce_impls.py:101-138). The reference's quack/CuTe WGMMA epilogue cannot run here
(sm_90a only, and its gemm_kernel.py does not import against the installed quack), so
bit-parity with that kernel is unpinned; its arithmetic is restated from source in
tile_partials() / finalize_partials() below.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import numpy as np
import torch
import torch.nn.functional as F

IGNORE_INDEX = -100
VOCAB_TILE = 256


# ---------------------------------------------------------------------------------------------
# fp32 ground truth
# ---------------------------------------------------------------------------------------------
def fp32_reference(hidden: torch.Tensor, weight: torch.Tensor, target: torch.Tensor,
                   ignore_index: int = IGNORE_INDEX, bias: Optional[torch.Tensor] = None):
    """fp32 matmul + fp32 reductions -> (ce, entropy, log_probs, lse), per row.

    Restates tests/test_ce_impls.py:17-25 (`_fp32_reference`) plus the row logsumexp. Rows whose
    target equals ignore_index get ce = 0 and log_probs = 0 (nll_loss, baseline.py:80).
    """
    h = hidden.detach().float().reshape(-1, hidden.shape[-1])
    w = weight.detach().float()
    t = target.reshape(-1)
    logits = F.linear(h, w, None if bias is None else bias.detach().float())
    lse = torch.logsumexp(logits, dim=-1)
    log_sm = logits - lse[:, None]
    sm = log_sm.exp()
    ce = F.nll_loss(log_sm, t, reduction="none", ignore_index=ignore_index)
    ent = -(sm * log_sm).sum(dim=-1)
    valid = t != ignore_index
    lp = torch.zeros_like(ce)
    rows = torch.arange(len(t), device=t.device)
    lp[valid] = log_sm[rows[valid], t[valid]]
    return ce, ent, lp, lse


def fp32_reference_grads(hidden: torch.Tensor, weight: torch.Tensor, target: torch.Tensor,
                         g_ce: Optional[torch.Tensor] = None, g_ent: Optional[torch.Tensor] = None,
                         ignore_index: int = IGNORE_INDEX):
    """fp32 autograd of loss = sum(g_ce * ce) + sum(g_ent * entropy) -> (ce, ent, d_hidden, d_weight).

    Restates baseline_linear_xent_entropy_backward (baseline.py:91-150); g_ce defaults to 1 and
    g_ent to -1 (baseline.py:127-134). Gradients are returned in fp32.
    """
    h = hidden.detach().float().reshape(-1, hidden.shape[-1]).requires_grad_(True)
    w = weight.detach().float().requires_grad_(True)
    t = target.reshape(-1)
    logits = F.linear(h, w)
    log_sm = F.log_softmax(logits, dim=-1)
    sm = log_sm.exp()
    ce = F.nll_loss(log_sm, t, reduction="none", ignore_index=ignore_index)
    ent = -(sm * log_sm).sum(dim=-1)
    gc = torch.ones_like(ce) if g_ce is None else g_ce.reshape(-1).float().to(ce.device)
    ge = -torch.ones_like(ent) if g_ent is None else g_ent.reshape(-1).float().to(ent.device)
    (gc * ce + ge * ent).sum().backward()
    return ce.detach(), ent.detach(), h.grad.detach(), w.grad.detach()


def fp32_reference_grads_with_bias(hidden: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
                                   target: torch.Tensor, g_ce: Optional[torch.Tensor] = None,
                                   g_ent: Optional[torch.Tensor] = None, ignore_index: int = IGNORE_INDEX):
    """fp32 autograd with a bias (baseline.py:115-142: logits = F.linear(h, w, b)) ->
    (ce, ent, d_hidden, d_weight, d_bias)."""
    h = hidden.detach().float().reshape(-1, hidden.shape[-1]).requires_grad_(True)
    w = weight.detach().float().requires_grad_(True)
    b = bias.detach().float().requires_grad_(True)
    t = target.reshape(-1)
    log_sm = F.log_softmax(F.linear(h, w, b), dim=-1)
    sm = log_sm.exp()
    ce = F.nll_loss(log_sm, t, reduction="none", ignore_index=ignore_index)
    ent = -(sm * log_sm).sum(dim=-1)
    gc = torch.ones_like(ce) if g_ce is None else g_ce.reshape(-1).float().to(ce.device)
    ge = -torch.ones_like(ent) if g_ent is None else g_ent.reshape(-1).float().to(ent.device)
    (gc * ce + ge * ent).sum().backward()
    return ce.detach(), ent.detach(), h.grad.detach(), w.grad.detach(), b.grad.detach()


def fp32_reference_grads_chunked(hidden, weight, target, ce_weight=1.0, ent_weight=-1.0, chunk=2048,
                                 ignore_index: int = IGNORE_INDEX):
    """Same as fp32_reference_grads with scalar weights, over row chunks (bounded memory); d_weight
    is accumulated across chunks in fp32 (the benchmarks' chunked ground truth,
    benchmarks/bench_fwd_bwd.py:108-131)."""
    B = hidden.shape[0]
    ces, ents, dhs = [], [], []
    dw = torch.zeros(weight.shape, dtype=torch.float32, device=weight.device)
    for s in range(0, B, chunk):
        e = min(s + chunk, B)
        n = e - s
        ce, ent, dh, dwc = fp32_reference_grads(
            hidden[s:e], weight, target[s:e], torch.full((n,), float(ce_weight), device=weight.device),
            torch.full((n,), float(ent_weight), device=weight.device), ignore_index=ignore_index,
        )
        ces.append(ce)
        ents.append(ent)
        dhs.append(dh)
        dw += dwc
    return torch.cat(ces), torch.cat(ents), torch.cat(dhs), dw


# ---------------------------------------------------------------------------------------------
# The reference's chunked torch path (the CPU baseline)
# ---------------------------------------------------------------------------------------------
def chunked_linear_xent_entropy(hidden: torch.Tensor, weight: torch.Tensor, target: torch.Tensor,
                                chunk_size: int = 4096) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Restates baseline.chunked_linear_xent_entropy (baseline.py:207-241): per row chunk,
    logits = F.linear in the input dtype, log_softmax in fp32, nll_loss, entropy, log_probs."""
    batch_shape = hidden.shape[:-1]
    h2 = hidden.reshape(-1, hidden.shape[-1])
    t1 = target.reshape(-1)
    B = h2.shape[0]
    ce = torch.empty(B, dtype=torch.float32)
    ent = torch.empty(B, dtype=torch.float32)
    lp = torch.empty(B, dtype=torch.float32)
    for s in range(0, B, chunk_size):
        e = min(s + chunk_size, B)
        logits = F.linear(h2[s:e], weight)
        log_sm = F.log_softmax(logits.float(), dim=-1)
        sm = log_sm.exp()
        t = t1[s:e]
        ce[s:e] = F.nll_loss(log_sm, t, reduction="none")
        ent[s:e] = -(sm * log_sm).sum(dim=-1)
        lp[s:e] = log_sm[torch.arange(e - s), t]
    return ce.view(batch_shape), ent.view(batch_shape), lp.view(batch_shape)


def chunked_fwd_bwd(hidden: torch.Tensor, weight: torch.Tensor, target: torch.Tensor, chunk_size: int = 4096):
    """Restates the chunked autograd training loop of benchmarks/bench_fwd_bwd.py:177-195:
    loss = sum(ce) - sum(entropy) over bf16 logits chunks, then backward. Returns (loss, dH, dW)."""
    h = hidden.detach().requires_grad_(True)
    w = weight.detach().requires_grad_(True)
    B = h.shape[0]
    ces, ents = [], []
    for s in range(0, B, chunk_size):
        e = min(s + chunk_size, B)
        logits = F.linear(h[s:e], w)
        log_sm = F.log_softmax(logits.float(), dim=-1)
        sm = log_sm.exp()
        ces.append(F.nll_loss(log_sm, target[s:e], reduction="none"))
        ents.append(-(sm * log_sm).sum(dim=-1))
    loss = torch.cat(ces).sum() - torch.cat(ents).sum()
    loss.backward()
    return loss.detach(), h.grad, w.grad


# ---------------------------------------------------------------------------------------------
# Epilogue / finalize / dlogits arithmetic (numpy, float64 unless noted)
# ---------------------------------------------------------------------------------------------
def tile_partials(logits: np.ndarray, target: np.ndarray, tile: int = VOCAB_TILE, vocab_offset: int = 0,
                  layout: str = "u") -> np.ndarray:
    """Per-(tile, row) partials of one vocabulary shard -> array [T, M, 4].

    Restates the reference epilogue (gemm_ce_entropy_epilogue.py:209-271): per row and per
    256-column vocabulary tile, m = max z (columns >= V skipped, :221-224), s = sum exp(z - m),
    zt = z[target] if the target lies in the tile else 0 (:225-226, :258). Third slot:
    layout "ref" -> sx = sum z exp(z - m) (:240); layout "u" -> u = sum (z - m) exp(z - m).
    """
    logits = np.asarray(logits, dtype=np.float64)
    M, V = logits.shape
    T = (V + tile - 1) // tile
    out = np.zeros((T, M, 4), dtype=np.float64)
    lt = np.asarray(target, dtype=np.int64) - vocab_offset
    for t in range(T):
        z = logits[:, t * tile:min((t + 1) * tile, V)]
        m = z.max(axis=1)
        e = np.exp(z - m[:, None])
        out[t, :, 0] = m
        out[t, :, 1] = e.sum(axis=1)
        out[t, :, 2] = (z * e).sum(axis=1) if layout == "ref" else ((z - m[:, None]) * e).sum(axis=1)
        inside = (lt >= t * tile) & (lt < min((t + 1) * tile, V))
        rows = np.nonzero(inside)[0]
        out[t, rows, 3] = logits[rows, lt[rows]]
    return out


def merge_partials(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Associative merge of two (m, s, u, zt) rows-arrays [M, 4] (u layout).

    Restates the online-softmax merge of gemm_ce_entropy_finalize.py:84-92 (max, rescaled sums,
    target logits added) for the centred third slot: u' = u + (m - M) s before rescaling.
    """
    out = np.empty_like(a)
    M_ = np.maximum(a[:, 0], b[:, 0])
    with np.errstate(invalid="ignore"):
        da = np.where(np.isneginf(a[:, 0]), 0.0, a[:, 0] - M_)
        db = np.where(np.isneginf(b[:, 0]), 0.0, b[:, 0] - M_)
    ea = np.where(np.isneginf(a[:, 0]), 0.0, np.exp(da))
    eb = np.where(np.isneginf(b[:, 0]), 0.0, np.exp(db))
    out[:, 0] = M_
    out[:, 1] = a[:, 1] * ea + b[:, 1] * eb
    out[:, 2] = (a[:, 2] + da * a[:, 1]) * ea + (b[:, 2] + db * b[:, 1]) * eb
    out[:, 3] = a[:, 3] + b[:, 3]
    return out


def finalize_partials(partials: np.ndarray, layout: str = "u", target: Optional[np.ndarray] = None,
                      vocab_size: Optional[int] = None, ignore_index: int = IGNORE_INDEX):
    """partials [T, M, 4] -> (ce, entropy, lse, log_probs, merged[M, 4]).

    Restates Finalize (gemm_ce_entropy_finalize.py:78-97): lse = M + log S, ce = lse - ZT,
    entropy = lse - SX / S (== log S - U / S in the centred layout). With a target array,
    ignore_index rows get ce = 0 (nll_loss semantics) and out-of-range ids give NaN.
    """
    p = np.asarray(partials, dtype=np.float64).copy()
    if layout == "ref":
        p[:, :, 2] = p[:, :, 2] - p[:, :, 0] * p[:, :, 1]
    acc = np.stack([np.full(p.shape[1], -np.inf), np.zeros(p.shape[1]), np.zeros(p.shape[1]),
                    np.zeros(p.shape[1])], axis=1)
    for t in range(p.shape[0]):
        acc = merge_partials(acc, p[t])
    log_s = np.log(acc[:, 1])
    lse = acc[:, 0] + log_s
    ent = log_s - acc[:, 2] / acc[:, 1]
    ce = lse - acc[:, 3]
    if target is not None:
        target = np.asarray(target, dtype=np.int64)
        ce = np.where(target == ignore_index, 0.0, ce)
        if vocab_size is not None:
            bad = (target != ignore_index) & ((target < 0) | (target >= vocab_size))
            ce = np.where(bad, np.nan, ce)
    return ce, ent, lse, -ce, acc


def dlogits(logits: np.ndarray, target: np.ndarray, lse: np.ndarray, ent: np.ndarray, g_ce, g_ent,
            vocab_offset: int = 0, ignore_index: Optional[int] = IGNORE_INDEX) -> np.ndarray:
    """dz_j = p_j (g_ce - g_ent (log p_j + H)) - g_ce [j == t], p = exp(z - lse).

    Restates ComputeDlogits (cute_dlogits.py:87-100). With ignore_index set, rows whose target
    equals it drop the CE term (g_ce -> 0), keeping the entropy term; ignore_index=None
    reproduces the reference kernel, which has no ignore rule.
    """
    z = np.asarray(logits, dtype=np.float64)
    M, V = z.shape
    t = np.asarray(target, dtype=np.int64)
    gc = np.broadcast_to(np.asarray(g_ce, dtype=np.float64), (M,)).copy()
    ge = np.broadcast_to(np.asarray(g_ent, dtype=np.float64), (M,)).copy()
    if ignore_index is not None:
        gc = np.where(t == ignore_index, 0.0, gc)
    lp = z - np.asarray(lse, dtype=np.float64)[:, None]
    p = np.exp(lp)
    dz = p * ((gc - ge * np.asarray(ent, dtype=np.float64))[:, None] - ge[:, None] * lp)
    lt = t - vocab_offset
    rows = np.nonzero((lt >= 0) & (lt < V))[0]
    dz[rows, lt[rows]] -= gc[rows]
    return dz


def tile_relative_logits(logits32: torch.Tensor, tile: int = VOCAB_TILE) -> Tuple[torch.Tensor, torch.Tensor]:
    """(fp16 d = z - m_t, fp32 m [T, M]) of fp32 logits [M, V]: m_t is the maximum of the row over
    the logit's `tile`-column tile, d the fp32 difference rounded to nearest fp16.

    Not a reference format: the reference stores the fp32 logits themselves
    (gemm_ce_entropy_bwd_epilogue.py:218) for its dlogits kernel (cute_dlogits.py:87-100). This
    restates the engine's 2-byte hand-over of the same logits so the tests can check it bit for
    bit; dlogits() of (d + m_t) then gives the gradient the engine forms from it, since
    log p = d - (lse - m_t) = (d + m_t) - lse.
    """
    z = logits32.float()
    M, V = z.shape
    T = (V + tile - 1) // tile
    m = torch.empty(T, M, dtype=torch.float32, device=z.device)
    d = torch.empty(M, V, dtype=torch.float16, device=z.device)
    for t in range(T):
        blk = z[:, t * tile:min((t + 1) * tile, V)]
        m[t] = blk.max(dim=1).values
        d[:, t * tile:min((t + 1) * tile, V)] = (blk - m[t][:, None]).to(torch.float16)
    return d, m


def expand_tile_max(m: torch.Tensor, V: int, tile: int = VOCAB_TILE) -> torch.Tensor:
    """[T, M] per-tile maxima -> [M, V] (each column gets its tile's maximum)."""
    return m.t().repeat_interleave(tile, dim=1)[:, :V]


# ---------------------------------------------------------------------------------------------
# Seeded inputs with the BASELINE.json distributions
# ---------------------------------------------------------------------------------------------
def make_inputs(B: int, H: int, V: int, seed: int = 0, weight_std: Optional[float] = None,
                ignore_frac: float = 0.0, tail_frac: float = 0.0, tail_cols: int = VOCAB_TILE):
    """CPU-generated bf16 inputs: hidden ~ N(0, 1), weight ~ N(0, weight_std) (default 1/sqrt(H),
    configs[0]), targets uniform in [0, V). Draw order hidden, weight, target from a
    torch.Generator seeded with `seed`. Optionally a seeded fraction of targets is set to
    ignore_index or moved into the final partial vocabulary tile."""
    g = torch.Generator().manual_seed(seed)
    std = (1.0 / math.sqrt(H)) if weight_std is None else weight_std
    hidden = torch.randn(B, H, generator=g).to(torch.bfloat16)
    weight = (torch.randn(V, H, generator=g) * std).to(torch.bfloat16)
    target = torch.randint(0, V, (B,), generator=g, dtype=torch.int64)
    if tail_frac > 0:
        n = int(round(tail_frac * B))
        idx = torch.randperm(B, generator=g)[:n]
        last_start = (V - 1) // tail_cols * tail_cols
        target[idx] = torch.randint(last_start, V, (n,), generator=g, dtype=torch.int64)
    if ignore_frac > 0:
        n = int(round(ignore_frac * B))
        idx = torch.randperm(B, generator=g)[:n]
        target[idx] = IGNORE_INDEX
    return hidden, weight, target


def split_bf16x3(x: torch.Tensor):
    """(hi, mid, lo) bf16 parts of an fp32 tensor with x = hi + mid + lo to ~24 bits: the split of the
    bf16x6 emulation of fp32 products (Henry, Tang, Heinecke, "Leveraging the bfloat16 Artificial
    Intelligence Datatype For Higher-Precision Computations", ARITH 2019). Each residual is exact in
    fp32. Restates what frx_split_f32 computes, for the CPU checks of the method."""
    x = x.float()
    hi = x.to(torch.bfloat16)
    r1 = x - hi.float()
    mid = r1.to(torch.bfloat16)
    r2 = r1 - mid.float()
    lo = r2.to(torch.bfloat16)
    return hi, mid, lo


# Part pairs whose products the bf16x6 scheme keeps: (left part, right part), 0 = hi, 1 = mid, 2 = lo.
BF16X6_PAIRS = ((0, 0), (0, 1), (1, 0), (0, 2), (2, 0), (1, 1))


def bf16x6_matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """a @ b from the six bf16 part products (each exact in fp64 here), the arithmetic the GPU path
    performs with fp32 accumulation."""
    pa, pb = split_bf16x3(a), split_bf16x3(b)
    out = torch.zeros(a.shape[0], b.shape[1], dtype=torch.float64)
    for i, j in BF16X6_PAIRS:
        out += pa[i].double() @ pb[j].double()
    return out
