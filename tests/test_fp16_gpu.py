"""GPU: fp16 inputs (the reference's native fp16 path, fast_reduction/kernel.py:32-45 — matmul in
the input dtype when hidden and weight share it) through every kernel of the path: forward GEMM
epilogue (+ fp16 bias), dlogits with fp16 output, the two backward GEMMs on fp16 operands, column
sums, the megakernel and the differentiable op, against fp32 / fp64 ground truth and against the
reference's own fp16 golden outputs."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import reference_math as rm

pytestmark = pytest.mark.gpu

DEV = "cuda"
GOLDEN = np.load(Path(__file__).parent / "golden" / "reference_baseline.npz")


@pytest.fixture(autouse=True)
def _status_clean():
    from fast_reduction import _native as nat

    yield
    torch.cuda.synchronize()
    nat.raise_on_status(torch.device(DEV))


def _half_inputs(B, H, V, seed, **kw):
    h, w, t = rm.make_inputs(B, H, V, seed=seed, **kw)
    return h.half(), w.half(), t


@pytest.mark.parametrize("B,H,V", [(520, 256, 3001), (128, 64, 256), (77, 320, 1000)])
def test_forward_fp16_matches_fp32(B, H, V):
    from fast_reduction.gemm_kernel import gemm_fused_ce_entropy

    h, w, t = _half_inputs(B, H, V, seed=B, weight_std=0.2, ignore_frac=0.05, tail_frac=0.02)
    ce, ent, lp = gemm_fused_ce_entropy(h.to(DEV), w.to(DEV), t.to(DEV), chunk_size=200)
    ce_r, ent_r, lp_r, _ = rm.fp32_reference(h, w, t)
    # fp16 values are exact in fp32 and the GEMM accumulates in fp32: only the summation order and
    # the exp approximation differ from the fp32 reference.
    torch.testing.assert_close(ce.cpu(), ce_r, atol=1e-4, rtol=1e-5)
    torch.testing.assert_close(ent.cpu(), ent_r, atol=1e-4, rtol=1e-5)
    torch.testing.assert_close(lp.cpu(), lp_r, atol=1e-4, rtol=1e-5)


def test_forward_fp16_vs_reference_golden_chunked():
    """The reference's chunked fp16 path rounds its logits to fp16 before reducing; ours keeps them in
    fp32, so the two agree to the fp16 rounding of the logits."""
    from fast_reduction.gemm_kernel import gemm_fused_ce_entropy

    g = GOLDEN
    h = torch.from_numpy(g["chunked16_hidden"]).view(torch.float16)
    w = torch.from_numpy(g["chunked16_weight"]).view(torch.float16)
    t = torch.from_numpy(g["chunked16_target"])
    ce, ent, lp = gemm_fused_ce_entropy(h.to(DEV), w.to(DEV), t.to(DEV), chunk_size=int(g["chunked16_chunk"]))
    np.testing.assert_allclose(ce.cpu().numpy(), g["chunked16_ce"], atol=5e-3)
    np.testing.assert_allclose(ent.cpu().numpy(), g["chunked16_ent"], atol=5e-3)
    np.testing.assert_allclose(lp.cpu().numpy(), g["chunked16_lp"], atol=5e-3)


def test_forward_fp16_with_bias_and_partials_match_oracle():
    from fast_reduction import ops
    from fast_reduction.gemm_kernel import gemm_fused_ce_entropy

    B, H, V, off = 200, 128, 1000, 300
    h, w, t = _half_inputs(B, H, V, seed=21, weight_std=0.3)
    b = (torch.randn(V, generator=torch.Generator().manual_seed(5)) * 0.5).half()
    t = t + off
    T = ops.n_vocab_tiles(V)
    part = torch.full((T, B, 4), float("nan"), device=DEV)
    ops.fwd_partials(h.to(DEV), w.to(DEV), t.to(DEV), part, B, vocab_offset=off, bias=b.to(DEV))
    z = (h.double() @ w.double().T + b.double()).numpy()
    exp = rm.tile_partials(z, t.numpy(), vocab_offset=off)
    got = part.cpu().double().numpy()
    np.testing.assert_allclose(got[..., 0], exp[..., 0], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(got[..., 1], exp[..., 1], rtol=2e-5, atol=1e-5)
    np.testing.assert_allclose(got[..., 2], exp[..., 2], rtol=2e-4, atol=2e-4)
    np.testing.assert_allclose(got[..., 3], exp[..., 3], rtol=1e-5, atol=1e-5)
    ce, ent, _ = gemm_fused_ce_entropy(h.to(DEV), w.to(DEV), (t - off).to(DEV), bias=None)
    ce_b, _, _ = gemm_fused_ce_entropy(h.to(DEV), w.to(DEV), (t - off).to(DEV), bias=b.to(DEV))
    ce_r, _, _, _ = rm.fp32_reference(h, w, t - off, bias=b)
    torch.testing.assert_close(ce_b.cpu(), ce_r, atol=1e-4, rtol=1e-5)
    assert not torch.equal(ce, ce_b)


def test_dlogits_fp16_output():
    from fast_reduction import ops

    M, V = 64, 1003
    g = torch.Generator().manual_seed(6)
    z = torch.randn(M, V, generator=g) * 3
    t = torch.randint(0, V, (M,), generator=g)
    lse = torch.logsumexp(z.double(), -1)
    p = torch.softmax(z.double(), -1)
    ent = -(p * torch.log_softmax(z.double(), -1)).sum(-1)
    ld = 1008
    zd = torch.zeros(M, ld, device=DEV)
    zd[:, :V] = z.to(DEV)
    out = torch.zeros(M, ld, device=DEV, dtype=torch.float16)
    ops.dlogits(zd, t.to(DEV), lse.float().to(DEV), ent.float().to(DEV), out, rows=M, vocab_shard=V)
    exp = rm.dlogits(z.double().numpy(), t.numpy(), lse.numpy(), ent.numpy(), 1.0, -1.0)
    # fp16 keeps 11 significant bits; values below its normal range lose relative precision
    np.testing.assert_allclose(out[:, :V].float().cpu().numpy(), exp, atol=1e-6, rtol=1e-3)
    assert (out[:, V:] == 0).all()


@pytest.mark.parametrize("rows,V,H", [(300, 1000, 200), (129, 77, 64), (1000, 4096, 1024)])
def test_backward_gemms_fp16_match_fp64(rows, V, H):
    from fast_reduction import ops

    g = torch.Generator(device=DEV).manual_seed(rows + V + 1)
    ldz = ops.round_up(V, 8)
    dz = torch.zeros(rows, ldz, device=DEV, dtype=torch.float16)
    dz[:, :V] = (torch.randn(rows, V, device=DEV, generator=g) * 0.1).half()
    w = torch.randn(V, H, device=DEV, generator=g).half()
    h = torch.randn(rows, H, device=DEV, generator=g).half()
    dh = torch.empty(rows, H, device=DEV, dtype=torch.float32)
    dw = torch.empty(V, H, device=DEV, dtype=torch.float32)
    ops.gemm_dhidden(dz, w, dh, rows=rows, vocab_shard=V)
    ops.gemm_dweight(dz, h, dw, rows=rows, vocab_shard=V)
    dz64 = dz[:, :V].double()
    torch.testing.assert_close(dh.double(), dz64 @ w.double(), atol=1e-4 * max(1.0, V / 1000), rtol=1e-4)
    torch.testing.assert_close(dw.double(), dz64.T @ h.double(), atol=1e-4 * max(1.0, rows / 1000), rtol=1e-4)
    dh16 = torch.empty(rows, H, device=DEV, dtype=torch.float16)
    ops.gemm_dhidden(dz, w, dh16, rows=rows, vocab_shard=V)
    assert torch.equal(dh16, dh.half())
    dw16 = torch.empty(V, H, device=DEV, dtype=torch.float16)
    ops.gemm_dweight(dz, h, dw16, rows=rows, vocab_shard=V)
    assert torch.equal(dw16, dw.half())
    with pytest.raises(TypeError, match="all be bfloat16 or all float16"):
        ops.gemm_dhidden(dz, w.to(torch.bfloat16), dh, rows=rows, vocab_shard=V)


def test_column_sums_fp16():
    from fast_reduction import ops

    x = torch.randn(1000, 3001, device=DEV).half()
    out = torch.empty(3001, device=DEV)
    ops.column_sums(x, out, rows=1000, cols=3001)
    torch.testing.assert_close(out.double(), x.double().sum(0), atol=1e-3, rtol=1e-5)


def test_megakernel_fp16_matches_fp32_and_reference_golden():
    from fast_reduction.gemm_kernel import gemm_megakernel_fast

    g = GOLDEN
    h = torch.from_numpy(g["bwd16_hidden"]).view(torch.float16)
    w = torch.from_numpy(g["bwd16_weight"]).view(torch.float16)
    t = torch.from_numpy(g["bwd16_target"])
    hd = h.to(DEV).requires_grad_(True)
    wd = w.to(DEV).requires_grad_(True)
    loss, ce, ent = gemm_megakernel_fast(hd, wd, t.to(DEV), chunk_size=16)
    loss.backward()
    assert hd.grad.dtype == torch.float16 and wd.grad.dtype == torch.float16
    np.testing.assert_allclose(ce.detach().cpu().numpy(), g["bwd16_ce"], atol=1e-4, rtol=1e-5)
    np.testing.assert_allclose(ent.detach().cpu().numpy(), g["bwd16_ent"], atol=1e-4, rtol=1e-5)
    for got, key in ((hd.grad, "bwd16_dh"), (wd.grad, "bwd16_dw")):
        ref = torch.from_numpy(g[key]).view(torch.float16).float()
        rel = (got.float().cpu() - ref).norm() / ref.norm()
        assert rel < 3e-3, (key, float(rel))


def test_megakernel_and_differentiable_fp16_with_bias():
    from fast_reduction.gemm_kernel import gemm_fused_ce_entropy_differentiable, gemm_megakernel_fast

    B, H, V = 384, 128, 1500
    h, w, t = _half_inputs(B, H, V, seed=34, weight_std=0.2, ignore_frac=0.05)
    b = torch.randn(V, generator=torch.Generator().manual_seed(4)).half()
    ce_r, ent_r, dh_r, dw_r, db_r = rm.fp32_reference_grads_with_bias(h, w, b, t)
    for fn in ("mega", "diff"):
        hd = h.to(DEV).requires_grad_(True)
        wd = w.to(DEV).requires_grad_(True)
        bd = b.to(DEV).requires_grad_(True)
        if fn == "mega":
            loss, ce, ent = gemm_megakernel_fast(hd, wd, t.to(DEV), bias=bd, chunk_size=100)
            loss.backward()
        else:
            ce, ent, _ = gemm_fused_ce_entropy_differentiable(hd, wd, t.to(DEV), bias=bd, chunk_size=100)
            (ce.sum() - ent.sum()).backward()
        torch.testing.assert_close(ce.detach().cpu(), ce_r, atol=1e-4, rtol=1e-5)
        assert bd.grad.dtype == torch.float16
        for got, ref in ((hd.grad, dh_r), (wd.grad, dw_r), (bd.grad, db_r)):
            rel = (got.float().cpu() - ref).norm() / ref.norm()
            assert rel < 3e-3, (fn, float(rel))
