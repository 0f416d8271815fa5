"""GPU: the standalone CE / entropy / logsumexp reductions over given logits (reference
fast_reduction/cute_cross_entropy.py:583-735), for bf16 / fp16 / fp32 logits, against a float64
torch reference. Like the reference, any negative target gives loss 0."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ref(x, t):
    x64 = x.double()
    lse = torch.logsumexp(x64, -1)
    ls = x64 - lse[:, None]
    ent = -(ls.exp() * ls).sum(-1)
    valid = t >= 0
    ce = torch.zeros_like(lse)
    rows = torch.arange(x.shape[0], device=x.device)
    ce[valid] = lse[valid] - x64[rows[valid], t[valid]]
    return ce, ent, lse


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("M,N", [(64, 1000), (3, 128256), (517, 3001), (1024, 32768)])
def test_ce_entropy_lse_match_float64(dtype, M, N):
    from fast_reduction.cute_cross_entropy import ce_entropy_fwd_with_lse, ce_fwd, entropy_fwd

    g = torch.Generator(device=DEV).manual_seed(M + N)
    x = (torch.randn(M, N, device=DEV, generator=g) * 3).to(dtype)
    t = torch.randint(0, N, (M,), device=DEV, generator=g)
    t[::7] = -100
    t[1::11] = -1
    t[2::13] = N - 1
    ce, ent, lse = ce_entropy_fwd_with_lse(x, t)
    ce_r, ent_r, lse_r = _ref(x, t)
    tol = dict(atol=2e-4, rtol=2e-5)
    torch.testing.assert_close(ce.double(), ce_r, **tol)
    torch.testing.assert_close(ent.double(), ent_r, **tol)
    torch.testing.assert_close(lse.double(), lse_r, **tol)
    assert (ce[t < 0] == 0).all()
    assert torch.equal(ce_fwd(x, t.to(torch.int32)), ce)
    assert torch.equal(entropy_fwd(x), ent)


def test_unaligned_rows_take_the_scalar_path():
    from fast_reduction.cute_cross_entropy import ce_entropy_fwd

    x = (torch.randn(40, 1003, device=DEV) * 2).to(torch.bfloat16)[:, 1:1002]  # row stride 1003, offset 1
    t = torch.randint(0, 1001, (40,), device=DEV)
    ce, ent = ce_entropy_fwd(x, t)
    ce_r, ent_r, _ = _ref(x, t)
    torch.testing.assert_close(ce.double(), ce_r, atol=2e-4, rtol=2e-5)
    torch.testing.assert_close(ent.double(), ent_r, atol=2e-4, rtol=2e-5)


def test_uniform_logits_entropy_is_log_n():
    from fast_reduction.cute_cross_entropy import entropy_fwd

    x = torch.zeros(8, 50000, device=DEV, dtype=torch.bfloat16)
    ent = entropy_fwd(x)
    torch.testing.assert_close(ent.double(), torch.full((8,), math.log(50000), device=DEV, dtype=torch.float64),
                               atol=1e-5, rtol=1e-6)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_rising_and_wide_range_logits(dtype):
    """Rows whose running max rises at every vector (the online reference point is rescaled again and
    again), rows spanning +-1e4, and N = 65536 (the reference's large-vocabulary regression sizes)."""
    from fast_reduction.cute_cross_entropy import ce_entropy_fwd_with_lse

    N = 65536
    rising = torch.linspace(-60.0, 60.0, N, device=DEV)
    falling = rising.flip(0)
    g = torch.Generator(device=DEV).manual_seed(1)
    wide = torch.randn(N, device=DEV, generator=g) * 1e4
    spiky = torch.randn(N, device=DEV, generator=g)
    spiky[::4096] = 80.0
    x = torch.stack([rising, falling, wide, spiky, rising * 1e-3]).to(dtype)
    t = torch.tensor([N - 1, 0, 5, 4096, 17], device=DEV)
    ce, ent, lse = ce_entropy_fwd_with_lse(x, t)
    ce_r, ent_r, lse_r = _ref(x, t)
    torch.testing.assert_close(lse.double(), lse_r, atol=1e-3, rtol=2e-6)
    torch.testing.assert_close(ce.double(), ce_r, atol=1e-3, rtol=2e-5)
    torch.testing.assert_close(ent.double(), ent_r, atol=2e-4, rtol=2e-5)
