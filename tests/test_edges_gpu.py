"""GPU: edge shapes through the public API — empty batches, a single row, a one-word vocabulary,
the smallest hidden size, every target ignored — in bf16, fp16 and fp32, against the fp32 oracle."""

import pytest
import torch

from oracle import reference_math as rm

pytestmark = pytest.mark.gpu

DEV = "cuda"
DTYPES = [torch.bfloat16, torch.float16, torch.float32]


@pytest.fixture(autouse=True)
def _status_clean():
    from fast_reduction import _native as nat

    yield
    torch.cuda.synchronize()
    nat.raise_on_status(torch.device(DEV))


@pytest.mark.parametrize("dtype", DTYPES)
def test_empty_batch(dtype):
    from fast_reduction.gemm_kernel import (gemm_fused_ce_entropy, gemm_fused_ce_entropy_differentiable,
                                            gemm_megakernel_fast)

    h = torch.empty(0, 64, device=DEV, dtype=dtype, requires_grad=True)
    w = torch.randn(100, 64, device=DEV).to(dtype).requires_grad_(True)
    t = torch.empty(0, dtype=torch.int64, device=DEV)
    ce, ent, lp = gemm_fused_ce_entropy(h, w, t)
    assert ce.shape == ent.shape == lp.shape == (0,)
    loss, ce, ent = gemm_megakernel_fast(h, w, t)
    loss.backward()
    assert float(loss.detach()) == 0.0 and h.grad.shape == (0, 64) and torch.count_nonzero(w.grad) == 0
    ce, ent, _ = gemm_fused_ce_entropy_differentiable(h, w, t)
    assert ce.shape == (0,)


def _check(h, w, t, dtype, chunk=64, atol=2e-3):
    from fast_reduction.gemm_kernel import gemm_fused_ce_entropy, gemm_megakernel_fast

    hd = h.to(DEV).to(dtype).requires_grad_(True)
    wd = w.to(DEV).to(dtype).requires_grad_(True)
    ce, ent, lp = gemm_fused_ce_entropy(hd, wd, t.to(DEV), chunk_size=chunk)
    ce_r, ent_r, lp_r, _ = rm.fp32_reference(hd.detach().cpu(), wd.detach().cpu(), t)
    torch.testing.assert_close(ce.cpu(), ce_r, atol=atol, rtol=1e-3)
    torch.testing.assert_close(ent.cpu(), ent_r, atol=atol, rtol=1e-3)
    torch.testing.assert_close(lp.cpu(), lp_r, atol=atol, rtol=1e-3)
    loss, _, _ = gemm_megakernel_fast(hd, wd, t.to(DEV), chunk_size=chunk)
    loss.backward()
    _, _, dh_r, dw_r = rm.fp32_reference_grads(hd.detach().cpu(), wd.detach().cpu(), t)
    torch.testing.assert_close(hd.grad.float().cpu(), dh_r, atol=atol, rtol=2e-2)
    torch.testing.assert_close(wd.grad.float().cpu(), dw_r, atol=atol, rtol=2e-2)
    return ce, ent


@pytest.mark.parametrize("dtype", DTYPES)
def test_single_row_and_smallest_hidden(dtype):
    g = torch.Generator().manual_seed(1)
    _check(torch.randn(1, 8, generator=g), torch.randn(300, 8, generator=g), torch.tensor([7]), dtype)


@pytest.mark.parametrize("dtype", DTYPES)
def test_one_word_vocabulary(dtype):
    """Softmax over one class: ce = 0, entropy = 0, zero gradients."""
    g = torch.Generator().manual_seed(2)
    ce, ent = _check(torch.randn(5, 16, generator=g), torch.randn(1, 16, generator=g),
                     torch.zeros(5, dtype=torch.int64), dtype)
    assert torch.equal(ce.cpu(), torch.zeros(5)) and (ent.cpu().abs() < 1e-6).all()


@pytest.mark.parametrize("dtype", DTYPES)
def test_every_target_ignored(dtype):
    g = torch.Generator().manual_seed(3)
    ce, _ = _check(torch.randn(70, 32, generator=g), torch.randn(500, 32, generator=g) * 0.3,
                   torch.full((70,), -100, dtype=torch.int64), dtype, chunk=32)
    assert torch.equal(ce.cpu(), torch.zeros(70))
