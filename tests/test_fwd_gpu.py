"""GPU parity tests of the forward path (libfrx through the C ABI) against the CPU oracle and an
fp32 ground truth. Shapes and seeds follow the reference's own tests (tests/test_ce_impls.py) plus
the ragged / ignore_index / sharding cases the reference lacks."""


import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import reference_math as rm

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(autouse=True)
def _status_clean():
    from fast_reduction import _native as nat

    yield
    torch.cuda.synchronize()
    nat.raise_on_status(torch.device(DEV))


def _exact_logits(h: torch.Tensor, w: torch.Tensor) -> np.ndarray:
    return h.double().cpu().numpy() @ w.double().cpu().numpy().T


def test_finalize_known_answer_reference_layout():
    """Reference KAT tests/test_ce_impls.py:101-138: hand-built partials [4, 128, 4] in the
    reference's layout merge to log_softmax's CE / entropy."""
    from fast_reduction.gemm_ce_entropy_finalize import finalize_ce_entropy, finalize_ce_entropy_with_lse

    torch.manual_seed(42)
    M, V, n_tiles = 128, 1024, 4
    logits = torch.randn(M, V, device=DEV, dtype=torch.float32)
    target = torch.randint(0, V, (M,), device=DEV)
    log_sm = F.log_softmax(logits, dim=-1)
    ce_ref = F.nll_loss(log_sm, target, reduction="none")
    ent_ref = -(log_sm.exp() * log_sm).sum(dim=-1)
    chunk_n = (V + n_tiles - 1) // n_tiles
    partials = torch.zeros(n_tiles, M, 4, device=DEV, dtype=torch.float32)
    for t in range(n_tiles):
        n_start, n_end = t * chunk_n, min((t + 1) * chunk_n, V)
        chunk = logits[:, n_start:n_end]
        partials[t, :, 0] = chunk.max(dim=-1).values
        partials[t, :, 1] = torch.exp(chunk - partials[t, :, 0:1]).sum(dim=-1)
        partials[t, :, 2] = (chunk * torch.exp(chunk - partials[t, :, 0:1])).sum(dim=-1)
        mask = (target >= n_start) & (target < n_end)
        local_idx = (target - n_start).clamp(0, n_end - n_start - 1)
        vals = chunk[torch.arange(M, device=DEV), local_idx]
        partials[t, :, 3] = torch.where(mask, vals, torch.zeros_like(vals))
    loss, entropy = finalize_ce_entropy(partials, n_tiles)
    torch.testing.assert_close(loss, ce_ref, atol=1e-3, rtol=1e-3)
    torch.testing.assert_close(entropy, ent_ref, atol=1e-3, rtol=1e-3)
    # tighter: against the oracle's float64 merge of the same partials
    ce_o, ent_o, lse_o, _, _ = rm.finalize_partials(partials.cpu().double().numpy(), layout="ref")
    np.testing.assert_allclose(loss.cpu().numpy(), ce_o, atol=2e-5, rtol=1e-5)
    np.testing.assert_allclose(entropy.cpu().numpy(), ent_o, atol=2e-5, rtol=1e-5)
    loss2, ent2, lse2 = finalize_ce_entropy_with_lse(partials, n_tiles)
    assert torch.equal(loss2, loss) and torch.equal(ent2, entropy)
    np.testing.assert_allclose(lse2.cpu().numpy(), lse_o, atol=2e-5, rtol=1e-6)


@pytest.mark.parametrize("B,H,V,offset", [(200, 128, 1000, 0), (128, 64, 256, 0), (77, 256, 3000, 1234),
                                          (300, 64, 100, 0)])
def test_fwd_partials_match_oracle(B, H, V, offset):
    """frx_fwd_partials vs the oracle's restated epilogue (ragged rows, ragged vocab tiles,
    vocabulary offset of a shard)."""
    from fast_reduction import ops

    h, w, t = rm.make_inputs(B, H, V, seed=B + V, weight_std=0.3)
    t = t + offset
    t[::7] = offset + V - 1  # targets in the final (partial) tile
    t[3::11] = offset - 1 if offset > 0 else V + 5  # targets outside this shard
    T = ops.n_vocab_tiles(V)
    part = torch.full((T, B, 4), float("nan"), device=DEV)
    ops.fwd_partials(h.to(DEV), w.to(DEV), t.to(DEV), part, B, vocab_offset=offset)
    got = part.cpu().double().numpy()
    exp = rm.tile_partials(_exact_logits(h, w), t.numpy(), vocab_offset=offset)
    np.testing.assert_allclose(got[..., 0], exp[..., 0], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(got[..., 1], exp[..., 1], rtol=2e-5, atol=1e-5)
    np.testing.assert_allclose(got[..., 2], exp[..., 2], rtol=2e-4, atol=2e-4)
    np.testing.assert_allclose(got[..., 3], exp[..., 3], rtol=1e-5, atol=1e-5)


def test_logits_output_matches_fp32_matmul():
    from fast_reduction import ops

    B, H, V = 150, 320, 700
    h, w, t = rm.make_inputs(B, H, V, seed=3)
    hd, wd, td = h.to(DEV), w.to(DEV), t.to(DEV)
    part = torch.empty(ops.n_vocab_tiles(V), B, 4, device=DEV)
    logits = torch.full((B, 704), float("nan"), device=DEV)
    ops.fwd_partials(hd, wd, td, part, B, logits=logits)
    exp = torch.from_numpy(_exact_logits(h, w)).float()
    torch.testing.assert_close(logits[:, :V].cpu(), exp, atol=1e-4, rtol=1e-5)
    assert torch.isnan(logits[:, V:]).all()  # padding columns untouched


def test_gemm_fused_matches_fp32_reference_test():
    """Reference tests/test_ce_impls.py:141-165 (B=256, H=128, V=1024, N(0,1) weights, seed 123)."""
    from fast_reduction.gemm_kernel import gemm_fused_ce_entropy

    torch.manual_seed(123)
    B, H, V = 256, 128, 1024
    hidden = torch.randn(B, H, device=DEV, dtype=torch.bfloat16)
    weight = torch.randn(V, H, device=DEV, dtype=torch.bfloat16)
    target = torch.randint(0, V, (B,), device=DEV)
    ce, ent, lp = gemm_fused_ce_entropy(hidden, weight, target, chunk_size=B)
    ce_ref, ent_ref, lp_ref, _ = rm.fp32_reference(hidden.cpu(), weight.cpu(), target.cpu())
    torch.testing.assert_close(ce.cpu(), ce_ref, atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(ent.cpu(), ent_ref, atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(lp.cpu(), lp_ref, atol=1e-2, rtol=1e-2)
    assert torch.equal(lp, -ce)


def test_config0_parity_vs_fp32_and_reference_chunked():
    """B=1024, H=1024, V=32000, chunk 512, seed 0. Gates from the north star:
    CE MAE <= 2e-3 and entropy MAE <= 1e-4 vs fp32 ground truth; the reference's own chunked
    bf16-logit outputs (golden, made by running its baseline.py) agree to their bf16 rounding."""
    from pathlib import Path

    from fast_reduction.gemm_kernel import gemm_fused_ce_entropy

    golden = np.load(Path(__file__).parent / "golden" / "reference_baseline.npz")
    h, w, t = rm.make_inputs(1024, 1024, 32000, seed=0)
    ce, ent, lp = gemm_fused_ce_entropy(h.to(DEV), w.to(DEV), t.to(DEV), chunk_size=512)
    ce, ent, lp = ce.cpu(), ent.cpu(), lp.cpu()
    ce32, ent32, lp32, _ = rm.fp32_reference(h, w, t)
    assert (ce - ce32).abs().mean() <= 2e-3
    assert (ent - ent32).abs().mean() <= 1e-4
    assert (lp - lp32).abs().mean() <= 2e-3
    ref_ce = torch.from_numpy(golden["cfg0_ce"])
    ref_ent = torch.from_numpy(golden["cfg0_ent"])
    assert (ce - ref_ce).abs().mean() <= 3e-3  # reference's own error vs fp32 is ~1.2e-3
    assert (ent - ref_ent).abs().mean() <= 2e-4


def test_chunking_is_bit_invariant_and_deterministic(monkeypatch):
    from fast_reduction import gemm_kernel as gk
    from fast_reduction.gemm_kernel import gemm_fused_ce_entropy

    h, w, t = rm.make_inputs(1000, 256, 5000, seed=11, weight_std=0.1)
    hd, wd, td = h.to(DEV), w.to(DEV), t.to(DEV)
    a = gemm_fused_ce_entropy(hd, wd, td, chunk_size=1000)
    # small shards merge chunks into one launch: a budget of 0 keeps one launch per 96-row chunk
    monkeypatch.setattr(gk, "_FWD_LAUNCH_PARTIALS_BYTES", 0)
    b = gemm_fused_ce_entropy(hd, wd, td, chunk_size=96)
    # 3 chunks per launch (the last launch ragged)
    monkeypatch.setattr(gk, "_FWD_LAUNCH_PARTIALS_BYTES", 16 * 20 * 96 * 3)
    c = gemm_fused_ce_entropy(hd, wd, td, chunk_size=96)
    monkeypatch.undo()
    d = gemm_fused_ce_entropy(hd, wd, td, chunk_size=1000)
    for x, y, z, u in zip(a, b, c, d):
        assert torch.equal(x, y)
        assert torch.equal(x, z)
        assert torch.equal(x, u)


def test_ignore_index_and_batch_shapes():
    from fast_reduction.gemm_kernel import gemm_fused_ce_entropy

    h, w, t = rm.make_inputs(4 * 37, 128, 2000, seed=5, weight_std=0.2, ignore_frac=0.1)
    ce, ent, lp = gemm_fused_ce_entropy(h.view(4, 37, 128).to(DEV), w.to(DEV), t.view(4, 37).to(DEV))
    assert ce.shape == (4, 37) and ent.shape == (4, 37) and lp.shape == (4, 37)
    ce32, ent32, lp32, _ = rm.fp32_reference(h, w, t)
    ign = (t == -100).view(4, 37)
    assert int(ign.sum()) > 0
    assert (ce.cpu()[ign] == 0).all() and (lp.cpu()[ign] == 0).all()
    torch.testing.assert_close(ce.cpu().view(-1), ce32, atol=2e-3, rtol=1e-3)
    torch.testing.assert_close(ent.cpu().view(-1), ent32, atol=2e-3, rtol=1e-3)


def test_bad_target_sets_status_and_nan():
    from fast_reduction import _native as nat
    from fast_reduction.gemm_kernel import gemm_fused_ce_entropy

    h, w, t = rm.make_inputs(64, 64, 500, seed=2)
    t[5] = 500  # out of range, not ignore_index
    ce, ent, lp = gemm_fused_ce_entropy(h.to(DEV), w.to(DEV), t.to(DEV))
    torch.cuda.synchronize()
    assert torch.isnan(ce[5]) and not torch.isnan(ce[:5]).any()
    assert nat.read_status(torch.device(DEV)) & nat.FRX_STATUS_BAD_TARGET


def test_vocab_shard_merge_equals_unsharded():
    """Single-GPU emulation of vocabulary sharding: per-shard partials merged per row, then merged
    across shards, equal the unsharded forward (ragged shard sizes, targets on every shard)."""
    from fast_reduction import gemm_kernel as gk
    from fast_reduction import ops

    B, H, V = 333, 128, 4100
    h, w, t = rm.make_inputs(B, H, V, seed=9, weight_std=0.2)
    hd, wd, td = h.to(DEV), w.to(DEV), t.to(DEV)
    ce, ent, lp = gk.gemm_fused_ce_entropy(hd, wd, td)
    bounds = [0, 1025, 2051, 3076, V]
    merged = torch.empty(len(bounds) - 1, B, 4, device=DEV)
    for r, (a, b) in enumerate(zip(bounds[:-1], bounds[1:])):
        gk.forward_stats(hd, wd[a:b], td, 128, vocab_offset=a, merged=merged[r], vocab_size=V)
    ce2 = torch.empty(B, device=DEV)
    ent2 = torch.empty(B, device=DEV)
    ops.finalize(merged, len(bounds) - 1, B, B, target=td, vocab_size=V, ignore_index=-100, ce=ce2, entropy=ent2)
    torch.testing.assert_close(ce2, ce, atol=2e-5, rtol=1e-5)
    torch.testing.assert_close(ent2, ent, atol=2e-5, rtol=1e-5)


def test_large_shape_mae_gates():
    """A larger case (B=2048, H=4096, V=32768, weight N(0, 0.02)) against fp32 torch on the GPU
    (TF32 off): north-star CE / entropy MAE gates."""
    from fast_reduction.gemm_kernel import gemm_fused_ce_entropy

    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator(device=DEV).manual_seed(1)
    B, H, V = 2048, 4096, 32768
    h = torch.randn(B, H, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(V, H, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    t = torch.randint(0, V, (B,), device=DEV, generator=g)
    ce, ent, lp = gemm_fused_ce_entropy(h, w, t)
    ce32, ent32, lp32, _ = rm.fp32_reference(h, w, t)
    assert (ce - ce32).abs().mean() <= 2e-3
    assert (ent - ent32).abs().mean() <= 1e-4


def test_forward_with_bias_matches_fp32():
    """Bias added to every logit (the reference's fp32 baseline semantics, baseline.py:76)."""
    from fast_reduction.gemm_kernel import gemm_fused_ce_entropy

    B, H, V = 300, 256, 2000
    h, w, t = rm.make_inputs(B, H, V, seed=31, weight_std=0.1, ignore_frac=0.05)
    b = (torch.randn(V, generator=torch.Generator().manual_seed(2)) * 2).to(torch.bfloat16)
    ce, ent, lp = gemm_fused_ce_entropy(h.to(DEV), w.to(DEV), t.to(DEV), bias=b.to(DEV), chunk_size=128)
    ce_r, ent_r, lp_r, _ = rm.fp32_reference(h, w, t, bias=b)
    torch.testing.assert_close(ce.cpu(), ce_r, atol=2e-3, rtol=1e-3)
    torch.testing.assert_close(ent.cpu(), ent_r, atol=2e-3, rtol=1e-3)
    # the bias really moved the result
    ce0, _, _ = gemm_fused_ce_entropy(h.to(DEV), w.to(DEV), t.to(DEV), chunk_size=128)
    assert (ce0.cpu() - ce_r).abs().mean() > 0.1
