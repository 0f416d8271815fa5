"""CPU: the oracle restatement pinned against the reference's own outputs (golden vectors made by
running the reference's fast_reduction/baseline.py, tests/golden/make_golden.py) and against the
reference's finalize known-answer construction (reference tests/test_ce_impls.py:101-138)."""

from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import reference_math as rm

GOLDEN = np.load(Path(__file__).parent / "golden" / "reference_baseline.npz")


def test_fp32_reference_matches_reference_unfused():
    g = GOLDEN
    ce, ent, lp, lse = rm.fp32_reference(torch.from_numpy(g["unfused_hidden"]), torch.from_numpy(g["unfused_weight"]),
                                         torch.from_numpy(g["unfused_target"]))
    np.testing.assert_allclose(ce.numpy(), g["unfused_ce"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(ent.numpy(), g["unfused_ent"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(lp.numpy(), g["unfused_lp"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(lp.numpy(), -ce.numpy(), atol=1e-6)


def test_chunked_restatement_matches_reference_bitwise():
    g = GOLDEN
    h = torch.from_numpy(g["chunked_hidden"]).view(torch.bfloat16)
    w = torch.from_numpy(g["chunked_weight"]).view(torch.bfloat16)
    t = torch.from_numpy(g["chunked_target"])
    ce, ent, lp = rm.chunked_linear_xent_entropy(h, w, t, chunk_size=int(g["chunked_chunk"]))
    assert torch.equal(ce, torch.from_numpy(g["chunked_ce"]))
    assert torch.equal(ent, torch.from_numpy(g["chunked_ent"]))
    assert torch.equal(lp, torch.from_numpy(g["chunked_lp"]))


def test_chunked_restatement_matches_reference_bitwise_fp16():
    g = GOLDEN
    h = torch.from_numpy(g["chunked16_hidden"]).view(torch.float16)
    w = torch.from_numpy(g["chunked16_weight"]).view(torch.float16)
    t = torch.from_numpy(g["chunked16_target"])
    ce, ent, lp = rm.chunked_linear_xent_entropy(h, w, t, chunk_size=int(g["chunked16_chunk"]))
    assert torch.equal(ce, torch.from_numpy(g["chunked16_ce"]))
    assert torch.equal(ent, torch.from_numpy(g["chunked16_ent"]))
    assert torch.equal(lp, torch.from_numpy(g["chunked16_lp"]))


def test_grads_restatement_matches_reference_autograd_fp16_inputs():
    """fp16 inputs: the reference differentiates in fp32 and casts the gradients to fp16."""
    g = GOLDEN
    h = torch.from_numpy(g["bwd16_hidden"]).view(torch.float16)
    w = torch.from_numpy(g["bwd16_weight"]).view(torch.float16)
    t = torch.from_numpy(g["bwd16_target"])
    ce, ent, dh, dw = rm.fp32_reference_grads(h, w, t)
    np.testing.assert_allclose(ce.numpy(), g["bwd16_ce"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(ent.numpy(), g["bwd16_ent"], rtol=1e-5, atol=1e-6)
    ref_dh = torch.from_numpy(g["bwd16_dh"]).view(torch.float16)
    ref_dw = torch.from_numpy(g["bwd16_dw"]).view(torch.float16)
    # one fp16 rounding apart at most
    assert (dh.half().float() - ref_dh.float()).abs().max() <= 1e-3 * ref_dh.float().abs().max()
    assert (dw.half().float() - ref_dw.float()).abs().max() <= 1e-3 * ref_dw.float().abs().max()


def test_grads_restatement_matches_reference_autograd():
    g = GOLDEN
    h, w, t = (torch.from_numpy(g[k]) for k in ("bwd_hidden", "bwd_weight", "bwd_target"))
    ce, ent, dh, dw = rm.fp32_reference_grads(h, w, t)
    np.testing.assert_allclose(ce.numpy(), g["bwd_ce"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(ent.numpy(), g["bwd_ent"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(dh.numpy(), g["bwd_dh"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(dw.numpy(), g["bwd_dw"], rtol=1e-5, atol=1e-6)
    _, _, dh2, dw2 = rm.fp32_reference_grads(h, w, t, torch.from_numpy(g["bwd_gce"]), torch.from_numpy(g["bwd_gent"]))
    np.testing.assert_allclose(dh2.numpy(), g["bwd_dh_g"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(dw2.numpy(), g["bwd_dw_g"], rtol=1e-5, atol=1e-6)


def test_analytic_dlogits_matches_reference_autograd():
    """dz from the restated ComputeDlogits formula, pushed through the linear layer, equals the
    reference's fp32 autograd gradients (per-row g_ce / g_ent)."""
    g = GOLDEN
    h, w, t = (torch.from_numpy(g[k]).double() for k in ("bwd_hidden", "bwd_weight", "bwd_target"))
    t = t.long()
    z = (h @ w.T).numpy()
    lse = np.log(np.exp(z - z.max(1, keepdims=True)).sum(1)) + z.max(1)
    p = np.exp(z - lse[:, None])
    ent = -(p * (z - lse[:, None])).sum(1)
    dz = rm.dlogits(z, t.numpy(), lse, ent, g["bwd_gce"], g["bwd_gent"])
    np.testing.assert_allclose(dz @ w.numpy(), g["bwd_dh_g"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(dz.T @ h.numpy(), g["bwd_dw_g"], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("layout", ["ref", "u"])
def test_partials_and_finalize_restatement_known_answer(layout):
    """The reference's finalize KAT (tests/test_ce_impls.py:101-138): partials built per tile from
    fp32 logits must merge to log_softmax's CE / entropy."""
    torch.manual_seed(42)
    M, V, n_tiles = 128, 1024, 4
    logits = torch.randn(M, V, dtype=torch.float32)
    target = torch.randint(0, V, (M,))
    log_sm = F.log_softmax(logits, dim=-1)
    ce_ref = F.nll_loss(log_sm, target, reduction="none")
    ent_ref = -(log_sm.exp() * log_sm).sum(-1)
    parts = rm.tile_partials(logits.numpy(), target.numpy(), tile=V // n_tiles, layout=layout)
    ce, ent, lse, lp, _ = rm.finalize_partials(parts, layout=layout)
    np.testing.assert_allclose(ce, ce_ref.numpy(), atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(ent, ent_ref.numpy(), atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(lse, torch.logsumexp(logits.double(), -1).numpy(), atol=1e-9)


def test_finalize_partials_shard_merge_associative():
    """Merging per-shard merged stats == merging all tiles at once (vocabulary sharding)."""
    rng = np.random.default_rng(3)
    z = rng.normal(size=(40, 1500)) * 3
    t = rng.integers(0, 1500, size=40)
    whole = rm.finalize_partials(rm.tile_partials(z, t))
    bounds = [0, 377, 800, 1500]
    merged = []
    for a, b in zip(bounds[:-1], bounds[1:]):
        merged.append(rm.finalize_partials(rm.tile_partials(z[:, a:b], t, vocab_offset=a))[4])
    shard = rm.finalize_partials(np.stack(merged))
    for x, y in zip(whole[:4], shard[:4]):
        np.testing.assert_allclose(x, y, rtol=1e-12, atol=1e-12)


def test_ignore_index_semantics():
    torch.manual_seed(5)
    h = torch.randn(16, 32)
    w = torch.randn(50, 32)
    t = torch.randint(0, 50, (16,))
    t[::3] = rm.IGNORE_INDEX
    ce, ent, lp, lse = rm.fp32_reference(h, w, t)
    assert (ce[t == -100] == 0).all() and (lp[t == -100] == 0).all()
    z = (h @ w.T).double().numpy()
    parts = rm.tile_partials(z, t.numpy(), tile=16)
    ce2, ent2, lse2, lp2, _ = rm.finalize_partials(parts, target=t.numpy(), vocab_size=50)
    np.testing.assert_allclose(ce2, ce.numpy(), atol=1e-4)
    np.testing.assert_allclose(ent2, ent.numpy(), atol=1e-4)
    # ignored rows keep only the entropy gradient
    _, _, dh, dw = rm.fp32_reference_grads(h, w, t)
    dz = rm.dlogits(z, t.numpy(), lse2, ent2, 1.0, -1.0)
    np.testing.assert_allclose(dz @ w.double().numpy(), dh.numpy(), atol=1e-4, rtol=1e-4)


def test_cfg0_inputs_regenerate_and_match_reference_outputs():
    """configs[0] (B=1024, H=1024, V=32000, chunk 512, seed 0): inputs regenerate bit-exactly
    from the seed, and the restated chunked path reproduces the reference's outputs."""
    import hashlib

    h, w, t = rm.make_inputs(1024, 1024, 32000, seed=0)
    hsh = hashlib.sha256()
    hsh.update(h.contiguous().view(torch.uint8).numpy().tobytes())
    hsh.update(w.contiguous().view(torch.uint8).numpy().tobytes())
    hsh.update(t.numpy().tobytes())
    assert hsh.hexdigest() == str(GOLDEN["cfg0_digest"])
    ce, ent, lp = rm.chunked_linear_xent_entropy(h, w, t, chunk_size=512)
    assert torch.equal(ce, torch.from_numpy(GOLDEN["cfg0_ce"]))
    assert torch.equal(ent, torch.from_numpy(GOLDEN["cfg0_ent"]))
    assert torch.equal(lp, torch.from_numpy(GOLDEN["cfg0_lp"]))
    # fp32 ground truth vs the reference's bf16-logit chunked path (about 1.2e-3 / 5e-5 at this shape)
    ce32, ent32, _, _ = rm.fp32_reference(h, w, t)
    assert (ce - ce32).abs().mean() < 2e-3
    assert (ent - ent32).abs().mean() < 1e-4


def test_make_inputs_distributions():
    h, w, t = rm.make_inputs(64, 256, 4096, seed=1, weight_std=0.05, ignore_frac=0.05, tail_frac=0.01)
    assert h.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and t.dtype == torch.int64
    assert abs(float(w.float().std()) - 0.05) < 0.005
    assert int((t == -100).sum()) == round(0.05 * 64)


def test_bias_restatement_matches_reference_autograd():
    g = GOLDEN
    h, w, b, t = (torch.from_numpy(g[k]) for k in ("bias_hidden", "bias_weight", "bias_bias", "bias_target"))
    ce, ent, dh, dw, db = rm.fp32_reference_grads_with_bias(h, w, b, t)
    for got, key in ((ce, "bias_ce"), (ent, "bias_ent"), (dh, "bias_dh"), (dw, "bias_dw"), (db, "bias_db")):
        np.testing.assert_allclose(got.numpy(), g[key], rtol=1e-5, atol=1e-6)
    ce2, ent2, _, _ = rm.fp32_reference(h, w, t, bias=b)
    np.testing.assert_allclose(ce2.numpy(), g["bias_ce"], rtol=1e-5, atol=1e-6)


def test_bf16x6_split_is_exact_and_product_is_fp32_accurate():
    """The fp32 input path's arithmetic (bf16x6, Henry et al. 2019) on the CPU: hi + mid + lo
    reproduces x, and the six kept part products give a @ b to fp32 accuracy."""
    g = torch.Generator().manual_seed(5)
    x = torch.randn(64, 96, generator=g) * torch.logspace(-20, 20, 96).float()
    hi, mid, lo = rm.split_bf16x3(x)
    rec = hi.double() + mid.double() + lo.double()
    rel = ((rec - x.double()).abs() / x.double().abs().clamp_min(1e-30)).max()
    assert rel < 2 ** -22, float(rel)
    a = torch.randn(50, 300, generator=g)
    b = torch.randn(300, 70, generator=g)
    exact = a.double() @ b.double()
    emu = rm.bf16x6_matmul(a, b)
    scale = (a.double().abs() @ b.double().abs())
    assert ((emu - exact).abs() / scale).max() < 2 ** -21
    one_pass = a.to(torch.bfloat16).double() @ b.to(torch.bfloat16).double()
    assert ((one_pass - exact).abs() / scale).max() > 2 ** -12  # what a plain bf16 product would lose
