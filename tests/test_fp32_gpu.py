"""GPU: fp32 inputs — the reference's fp32 matmul path (fast_reduction/kernel.py:32-45; megakernel
dH/dW in fp32, gemm_kernel.py:859-871) — computed on the bf16 tensor cores by the bf16x6 split
(frx_split_f32: hi / mid / lo parts, six part products accumulated in fp32), against fp64 ground
truth and the reference's own fp32 golden outputs."""

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


def _f64_reference(h, w, t, b=None, ignore_index=-100):
    z = h.double() @ w.double().T + (0 if b is None else b.double())
    lse = torch.logsumexp(z, -1)
    ls = z - lse[:, None]
    ent = -(ls.exp() * ls).sum(-1)
    valid = t != ignore_index
    ce = torch.zeros_like(lse)
    ce[valid] = lse[valid] - z[valid, t[valid]]
    return ce, ent


def test_split_kernel_matches_oracle_bitwise():
    from fast_reduction import ops

    g = torch.Generator().manual_seed(3)
    x = torch.randn(37, 101, generator=g) * torch.logspace(-15, 15, 101).float()
    x[0, :5] = torch.tensor([0.0, -0.0, 1e-40, -3e38, 1.0])
    out = torch.empty(3, 37, 104, device=DEV, dtype=torch.bfloat16)
    ops.split_f32(x.to(DEV), out[0], (0, 1, 2), part_stride=37 * 104)
    for got, ref in zip(out[:, :, :101].cpu(), rm.split_bf16x3(x)):
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16))


@pytest.mark.parametrize("B,H,V,with_bias", [(300, 256, 3001, False), (129, 100, 1000, True), (64, 64, 128, False)])
def test_forward_fp32_matches_fp64(B, H, V, with_bias):
    from fast_reduction.gemm_kernel import gemm_fused_ce_entropy

    g = torch.Generator().manual_seed(B + V)
    h = torch.randn(B, H, generator=g)
    w = torch.randn(V, H, generator=g) * 0.2
    t = torch.randint(0, V, (B,), generator=g)
    t[::17] = -100
    b = torch.randn(V, generator=g) if with_bias else None
    ce, ent, lp = gemm_fused_ce_entropy(h.to(DEV), w.to(DEV), t.to(DEV), bias=None if b is None else b.to(DEV),
                                        chunk_size=128)
    ce_r, ent_r = _f64_reference(h, w, t, b)
    # fp32-level agreement: a few fp32 ulps of values up to ~20 (a bf16 product is off by ~1e-2 here)
    torch.testing.assert_close(ce.double().cpu(), ce_r, atol=2e-5, rtol=1e-5)
    torch.testing.assert_close(ent.double().cpu(), ent_r, atol=2e-5, rtol=1e-5)
    torch.testing.assert_close(lp.double().cpu(), -ce_r, atol=2e-5, rtol=1e-5)
    if H % 8 == 0:  # (bf16 operands need H to be a multiple of 8; fp32 ones do not)
        bf16 = gemm_fused_ce_entropy(h.to(DEV).bfloat16(), w.to(DEV).bfloat16(), t.to(DEV),
                                     bias=None if b is None else b.to(DEV).bfloat16(), chunk_size=128)[0]
        assert (bf16.double().cpu() - ce_r).abs().max() > 20 * (ce.double().cpu() - ce_r).abs().max()


def test_forward_fp32_vs_reference_unfused_golden():
    """The reference's fp32 unfused baseline (baseline.py:62-88) on its own test shape."""
    from fast_reduction.gemm_kernel import gemm_fused_ce_entropy

    g = GOLDEN
    h, w, t = (torch.from_numpy(g[k]) for k in ("unfused_hidden", "unfused_weight", "unfused_target"))
    ce, ent, lp = gemm_fused_ce_entropy(h.to(DEV), w.to(DEV), t.to(DEV))
    np.testing.assert_allclose(ce.cpu().numpy(), g["unfused_ce"], rtol=1e-5, atol=2e-5)
    np.testing.assert_allclose(ent.cpu().numpy(), g["unfused_ent"], rtol=1e-5, atol=2e-5)
    np.testing.assert_allclose(lp.cpu().numpy(), g["unfused_lp"], rtol=1e-5, atol=2e-5)


def test_accumulating_backward_gemms():
    from fast_reduction import ops

    rows, V, H = 300, 1000, 200
    g = torch.Generator(device=DEV).manual_seed(9)
    dz = (torch.randn(rows, 1000, device=DEV, generator=g) * 0.1).to(torch.bfloat16)
    w = torch.randn(V, H, device=DEV, generator=g).to(torch.bfloat16)
    h = torch.randn(rows, H, device=DEV, generator=g).to(torch.bfloat16)
    dh = torch.empty(rows, H, device=DEV)
    dw = torch.empty(V, H, device=DEV)
    ops.gemm_dhidden(dz, w, dh, rows=rows, vocab_shard=V)
    ops.gemm_dweight(dz, h, dw, rows=rows, vocab_shard=V)
    dh2, dw2 = dh.clone(), dw.clone()
    ops.gemm_dhidden(dz, w, dh2, rows=rows, vocab_shard=V, accumulate=True)
    ops.gemm_dweight(dz, h, dw2, rows=rows, vocab_shard=V, accumulate=True)
    assert torch.equal(dh2, 2 * dh) and torch.equal(dw2, 2 * dw)
    with pytest.raises(TypeError, match="float32"):
        ops.gemm_dhidden(dz, w, dh.to(torch.bfloat16), rows=rows, vocab_shard=V, accumulate=True)


def test_megakernel_fp32_matches_reference_golden_grads():
    """The reference's fp32 autograd backward (baseline.py:91-150) golden gradients."""
    from fast_reduction.gemm_kernel import gemm_megakernel_fast

    g = GOLDEN
    h, w, t = (torch.from_numpy(g[k]) for k in ("bwd_hidden", "bwd_weight", "bwd_target"))
    hd = h.to(DEV).requires_grad_(True)
    wd = w.to(DEV).requires_grad_(True)
    loss, ce, ent = gemm_megakernel_fast(hd, wd, t.to(DEV), chunk_size=8)
    loss.backward()
    assert hd.grad.dtype == torch.float32 and wd.grad.dtype == torch.float32
    np.testing.assert_allclose(ce.cpu().numpy(), g["bwd_ce"], rtol=1e-5, atol=2e-5)
    np.testing.assert_allclose(ent.cpu().numpy(), g["bwd_ent"], rtol=1e-5, atol=2e-5)
    np.testing.assert_allclose(hd.grad.cpu().numpy(), g["bwd_dh"], rtol=1e-4, atol=2e-6)
    np.testing.assert_allclose(wd.grad.cpu().numpy(), g["bwd_dw"], rtol=1e-4, atol=2e-6)


def test_fp32_training_with_bias_and_per_row_grads_vs_fp64():
    from fast_reduction.gemm_kernel import gemm_fused_ce_entropy_differentiable, gemm_megakernel_fast

    B, H, V = 256, 96, 1500
    g = torch.Generator().manual_seed(12)
    h = torch.randn(B, H, generator=g)
    w = torch.randn(V, H, generator=g) * 0.3
    b = torch.randn(V, generator=g)
    t = torch.randint(0, V, (B,), generator=g)
    t[::11] = -100
    gce = torch.rand(B, generator=g)
    gent = torch.randn(B, generator=g)
    h64 = h.double().requires_grad_(True)
    w64 = w.double().requires_grad_(True)
    b64 = b.double().requires_grad_(True)
    z = h64 @ w64.T + b64
    ls = torch.log_softmax(z, -1)
    ce64 = torch.nn.functional.nll_loss(ls, t, reduction="none", ignore_index=-100)
    ent64 = -(ls.exp() * ls).sum(-1)
    (gce.double() * ce64 + gent.double() * ent64).sum().backward()
    hd = h.to(DEV).requires_grad_(True)
    wd = w.to(DEV).requires_grad_(True)
    bd = b.to(DEV).requires_grad_(True)
    ce, ent, _ = gemm_fused_ce_entropy_differentiable(hd, wd, t.to(DEV), bias=bd, chunk_size=100)
    (gce.to(DEV) * ce + gent.to(DEV) * ent).sum().backward()
    for got, ref in ((hd.grad, h64.grad), (wd.grad, w64.grad), (bd.grad, b64.grad)):
        assert got.dtype == torch.float32
        rel = (got.double().cpu() - ref).norm() / ref.norm()
        assert rel < 1e-5, float(rel)
    hd2 = h.to(DEV).requires_grad_(True)
    wd2 = w.to(DEV).requires_grad_(True)
    loss, _, _ = gemm_megakernel_fast(hd2, wd2, t.to(DEV), chunk_size=64)
    loss.backward()
    h64.grad = None
    w64.grad = None
    z = h64 @ w64.T
    ls = torch.log_softmax(z, -1)
    ce64 = torch.nn.functional.nll_loss(ls, t, reduction="sum", ignore_index=-100)
    ent64 = -(ls.exp() * ls).sum()
    (ce64 - ent64).backward()
    for got, ref in ((hd2.grad, h64.grad), (wd2.grad, w64.grad)):
        rel = (got.double().cpu() - ref).norm() / ref.norm()
        assert rel < 1e-5, float(rel)


def test_fp32_host_inputs():
    from fast_reduction.gemm_kernel import gemm_fused_ce_entropy

    g = torch.Generator().manual_seed(2)
    h = torch.randn(100, 64, generator=g)
    w = torch.randn(700, 64, generator=g) * 0.2
    t = torch.randint(0, 700, (100,), generator=g)
    out = gemm_fused_ce_entropy(h, w, t)
    ref = gemm_fused_ce_entropy(h.to(DEV), w.to(DEV), t.to(DEV))
    for a, b_ in zip(out, ref):
        assert a.device.type == "cpu" and torch.equal(a, b_.cpu())
