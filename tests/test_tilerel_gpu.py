"""GPU: the training pass's 2-byte logits hand-over and the small kernels around the training op.

* frx_fwd_partials_tilerel writes fp16 z - m_t (m_t = the tile maximum of the same launch's partials):
  bit-equal to rounding the fp32 logits of frx_fwd_partials minus m_t, and the partials are
  bit-equal to a launch without logits output.
* frx_dlogits_tilerel matches the oracle's dlogits of (d + m_t) in fp64, and stays within the
  fp16 rounding bound of the dlogits formed from fp32 logits.
* The training op with tile-relative logits (the default) and with fp32 logits (FRX_TRAIN_LOGITS=f32)
  both meet the fp32 autograd gate; merging row chunks into fewer launches changes no bit.
* frx_loss_sum, frx_scale_inplace and the gradient hand-over of the autograd op.
"""

import numpy as np
import pytest
import torch

from oracle import reference_math as rm

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(autouse=True)
def _status_clean():
    from fast_reduction import _native as nat

    yield
    torch.cuda.synchronize()
    nat.raise_on_status(torch.device(DEV))


def _launch_both(h, w, t, off=0, bias=None):
    """(partials plain, partials+fp32 logits, fp32 logits, partials+tile-relative, tile-relative)."""
    from fast_reduction import ops

    B = h.shape[0]
    V = w.shape[0]
    T = ops.n_vocab_tiles(V)
    p0 = torch.full((T, B, 4), float("nan"), device=DEV)
    p1 = torch.full((T, B, 4), float("nan"), device=DEV)
    p2 = torch.full((T, B, 4), float("nan"), device=DEV)
    # 16 spare columns past the 16-byte boundary of each row: the stores must not reach them
    z32 = torch.full((B, ops.round_up(V, 4) + 16), 7.0, device=DEV)
    rel = torch.full((B, ops.round_up(V, 8) + 16), 7.0, device=DEV, dtype=torch.float16)
    ops.fwd_partials(h, w, t, p0, B, off, bias=bias)
    ops.fwd_partials(h, w, t, p1, B, off, logits=z32, bias=bias)
    ops.fwd_partials(h, w, t, p2, B, off, logits_rel=rel, bias=bias)
    return p0, p1, z32, p2, rel


@pytest.mark.parametrize("B,H,V,dtype,with_bias", [
    (300, 256, 1003, torch.bfloat16, False),   # ragged rows, last tile 235 columns
    (257, 128, 788, torch.float16, True),      # last tile 20 columns (< 32), fp16 operands + bias
    (1024, 512, 16032, torch.bfloat16, False),  # an 8-GPU headline shard width
    (128, 64, 40, torch.bfloat16, True),       # a single partial tile
])
def test_tilerel_logits_bit_exact(B, H, V, dtype, with_bias):
    from fast_reduction import ops

    h, w, t = rm.make_inputs(B, H, V, seed=B + V, weight_std=0.3)
    h, w, t = h.to(DEV, dtype), w.to(DEV, dtype), t.to(DEV)
    off = 1000
    t = t + off
    bias = (torch.randn(V, generator=torch.Generator().manual_seed(1)) * 2).to(DEV, dtype) if with_bias else None
    p0, p1, z32, p2, rel = _launch_both(h, w, t, off, bias)
    torch.cuda.synchronize()
    # the logits outputs change no partial
    assert torch.equal(p0, p1) and torch.equal(p0, p2)
    m = p2[:, :, 0]
    exp = (z32[:, :V] - rm.expand_tile_max(m, V)).to(torch.float16)
    assert torch.equal(rel[:, :V], exp)
    # The TMA unit writes whole 16-byte chunks: the row's pad columns up to the next 16-byte
    # boundary may be written, nothing beyond it.
    assert bool((rel[:, ops.round_up(V, 8):] == 7.0).all())
    assert bool((z32[:, ops.round_up(V, 4):] == 7.0).all())
    torch.testing.assert_close(z32[:, :V], (h.float() @ w.float().T + (0 if bias is None else bias.float())),
                               atol=1e-2, rtol=1e-2)
    # the oracle's restatement of the format agrees bit for bit
    d_o, m_o = rm.tile_relative_logits(z32[:, :V])
    assert torch.equal(m_o, m) and torch.equal(d_o, rel[:, :V])


def _rand_case(M, V, seed, with_neg_inf=False):
    g = torch.Generator().manual_seed(seed)
    T = (V + 255) // 256
    m = (torch.randn(T, M, generator=g, dtype=torch.float64) * 3).float().double()  # what the kernel reads
    d = -(torch.rand(M, V, generator=g, dtype=torch.float64) * 25)
    d16 = d.to(torch.float16)
    if with_neg_inf:
        d16[::7, 3::11] = float("-inf")
    z = d16.double() + rm.expand_tile_max(m, V).double()  # the logits the stored pair stands for
    zf = torch.where(torch.isinf(z), torch.full_like(z, -1e30), z)
    lse = torch.logsumexp(zf, -1)
    p = torch.softmax(zf, -1)
    ent = -(p * torch.log_softmax(zf, -1)).sum(-1)
    return m.float(), d16, zf, lse, ent


@pytest.mark.parametrize("out_dtype,aligned", [(torch.float32, True), (torch.bfloat16, True), (torch.float16, True),
                                               (torch.bfloat16, False)])
def test_dlogits_tilerel_matches_oracle(out_dtype, aligned):
    from fast_reduction import ops

    M, V, off = 70, 1003, 500
    m, d16, z, lse, ent = _rand_case(M, V, 5, with_neg_inf=True)
    g = torch.Generator().manual_seed(6)
    t = torch.randint(off, off + V, (M,), generator=g)
    t[::9] = -100
    t[1::13] = off + V + 3  # target on another shard
    gce = torch.rand(M, generator=g)
    gent = torch.randn(M, generator=g)
    ld = 1008
    if aligned:
        rel = torch.zeros(M, ld, device=DEV, dtype=torch.float16)
    else:  # rows start 2 bytes past a 16-byte boundary: the element-wise load path
        rel = torch.zeros(M, ld + 1, device=DEV, dtype=torch.float16)[:, 1:]
    rel[:, :V] = d16.to(DEV)
    T = m.shape[0]
    part = torch.zeros(T, M, 4, device=DEV)
    part[:, :, 0] = m.to(DEV)
    out = torch.zeros(M, ld, device=DEV, dtype=out_dtype)
    ops.dlogits_tilerel(rel, part, M, t.to(DEV), lse.float().to(DEV), ent.float().to(DEV), out, rows=M, vocab_shard=V,
                        g_ce=gce.to(DEV), g_ent=gent.to(DEV), vocab_offset=off, ignore_index=-100)
    exp = rm.dlogits(z.numpy(), t.numpy(), lse.numpy(), ent.numpy(), gce.numpy(), gent.numpy(), vocab_offset=off)
    got = out[:, :V].float().cpu().numpy()
    assert np.isfinite(got).all()
    assert (got[d16.numpy() == -np.inf] == 0).all()
    if out_dtype == torch.float32:
        np.testing.assert_allclose(got, exp, atol=2e-6, rtol=1e-4)
    else:
        np.testing.assert_allclose(got, exp, atol=1e-5, rtol=8e-3)
    assert (out[:, V:] == 0).all()


@pytest.mark.parametrize("std", [0.05, 0.6])
def test_tilerel_dz_within_fp16_bound_of_fp32_path(std):
    """Same GEMM, same statistics: the dlogits from z - m_t in fp16 differ from those from fp32
    logits only by the fp16 rounding of z - m_t, |d| 2^-11 per logit, i.e.
    |dz_rel - dz_32| <= p |d| 2^-11 (|a + b lp| + |b|) (+ fp32 rounding)."""
    from fast_reduction import ops

    B, H, V = 512, 512, 5000
    h, w, t = rm.make_inputs(B, H, V, seed=11, weight_std=std)
    h, w, t = h.to(DEV), w.to(DEV), t.to(DEV)
    p0, p1, z32, p2, rel = _launch_both(h, w, t)
    T = p0.shape[0]
    ce, ent, lse = (torch.empty(B, device=DEV) for _ in range(3))
    ops.finalize(p2, T, B, B, target=t, vocab_size=V, ignore_index=-100, ce=ce, entropy=ent, lse=lse)
    out32 = torch.empty(B, ops.round_up(V, 4), device=DEV)
    outr = torch.empty(B, ops.round_up(V, 4), device=DEV)
    ops.dlogits(z32, t, lse, ent, out32, rows=B, vocab_shard=V, ignore_index=-100)
    ops.dlogits_tilerel(rel, p2, B, t, lse, ent, outr, rows=B, vocab_shard=V, ignore_index=-100)
    torch.cuda.synchronize()
    z = z32[:, :V].double()
    lp = z - lse.double()[:, None]
    p = lp.exp()
    a = (1.0 - (-1.0) * ent.double())[:, None]
    bnd = p * (rel[:, :V].double().abs() + 1e-3) * 2.0 ** -11 * ((a + lp).abs() + 1.0)
    diff = (outr[:, :V].double() - out32[:, :V].double()).abs()
    assert bool((diff <= 1.5 * bnd + 1e-5 * out32[:, :V].double().abs() + 1e-12).all())
    # and both are close to each other on the scale of a bf16 dlogit
    assert float(diff.max()) <= 2.0 ** -9 * float(out32[:, :V].abs().max())


@pytest.mark.parametrize("logits", ["f16rel", "f32"])
def test_megakernel_both_logits_formats_meet_gate(monkeypatch, logits):
    from fast_reduction import gemm_kernel as gk

    monkeypatch.setattr(gk, "_TILEREL_LOGITS", logits == "f16rel")
    B, H, V = 512, 256, 3000
    h, w, t = rm.make_inputs(B, H, V, seed=21, weight_std=0.1, ignore_frac=0.05)
    hd = h.to(DEV).requires_grad_(True)
    wd = w.to(DEV).requires_grad_(True)
    loss, ce, ent = gk.gemm_megakernel_fast(hd, wd, t.to(DEV), chunk_size=128)
    loss.backward()
    _, _, dh_ref, dw_ref = rm.fp32_reference_grads(h, w, t)
    assert float((hd.grad.float().cpu() - dh_ref).abs().mean()) < 2e-3
    assert float((wd.grad.float().cpu() - dw_ref).abs().mean()) < 2e-3


def test_launch_merge_changes_no_bit(monkeypatch):
    """chunk_size as a memory cap: rows merged into one forward launch give bit-identical results."""
    from fast_reduction import gemm_kernel as gk

    B, H, V = 512, 256, 2048
    h, w, t = rm.make_inputs(B, H, V, seed=3, weight_std=0.1)
    res = []
    for merge in (False, True):
        monkeypatch.setattr(gk, "_TRAIN_MERGE", merge)
        assert gk._train_launch_rows(256, B, V, 2, V) == (B if merge else 256)
        hd = h.to(DEV).requires_grad_(True)
        wd = w.to(DEV).requires_grad_(True)
        loss, ce, ent = gk.gemm_megakernel_fast(hd, wd, t.to(DEV), chunk_size=256)
        loss.backward()
        res.append((loss.detach(), ce, ent, hd.grad, wd.grad))
    for a, b in zip(*res):
        assert torch.equal(a, b)


def test_loss_sum_kernel():
    from fast_reduction import ops

    g = torch.Generator().manual_seed(2)
    for rows in (0, 1, 511, 32768, 100003):
        ce = (torch.rand(rows, generator=g) * 12).to(DEV)
        ent = (torch.rand(rows, generator=g) * 10).to(DEV)
        loss = torch.full((), float("nan"), device=DEV)
        ops.loss_sum(ce, ent, loss, rows=rows, ce_weight=0.7, ent_weight=-1.3)
        exp = 0.7 * ce.double().sum() - 1.3 * ent.double().sum()
        assert abs(float(loss) - float(exp)) <= 1e-6 * max(1.0, abs(float(exp)))
        loss2 = torch.full((), float("nan"), device=DEV)
        ops.loss_sum(ce, ent, loss2, rows=rows, ce_weight=0.7, ent_weight=-1.3)
        assert torch.equal(loss, loss2)  # deterministic


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_scale_inplace_kernel(dtype):
    from fast_reduction import ops

    g = torch.Generator().manual_seed(9)
    for n in (1, 7, 4096 + 3, 1 << 20):
        x = torch.randn(n, generator=g).to(DEV, dtype)
        x0 = x.clone()
        ops.scale_inplace(x, torch.ones(1, device=DEV))
        assert torch.equal(x, x0)
        s = torch.tensor([0.37], device=DEV)
        ops.scale_inplace(x, s)
        exp = (x0.float() * 0.37).to(dtype)
        assert torch.equal(x, exp)
        buf = x0.clone()
        y = buf[1:]  # unaligned start: the scalar path
        ops.scale_inplace(y, s)
        assert torch.equal(y, (x0[1:].float() * 0.37).to(dtype)) and torch.equal(buf[:1], x0[:1])


def test_backward_hands_gradients_over_without_copy_or_sync():
    """loss.backward() puts the op's own gradient buffers into .grad (no copy) and a retained second
    backward through the same graph is refused instead of silently double-scaling."""
    from fast_reduction.gemm_kernel import gemm_megakernel_fast

    h, w, t = rm.make_inputs(256, 128, 1000, seed=4, weight_std=0.2)
    hd = h.to(DEV).requires_grad_(True)
    wd = w.to(DEV).requires_grad_(True)
    loss, _, _ = gemm_megakernel_fast(hd, wd, t.to(DEV), chunk_size=128)
    loss.backward(retain_graph=True)
    g1 = hd.grad.clone()
    with pytest.raises(RuntimeError, match="already handed"):
        loss.backward()
    # a fresh call works, and its gradient equals the first one
    hd.grad = None
    loss, _, _ = gemm_megakernel_fast(hd, wd, t.to(DEV), chunk_size=128)
    loss.backward()
    assert torch.equal(hd.grad, g1)
