"""GPU: the forward over host (CPU) inputs — weight uploaded in slices under the GEMMs, a head of the
weight ahead of a chunked hidden upload, rows in groups bounded by the partials buffer — returns
exactly what the device-resident forward returns."""

import pytest
import torch

from fast_reduction import gemm_kernel as gk
from oracle import reference_math as rm

pytestmark = pytest.mark.gpu


@pytest.fixture
def small_slices(monkeypatch):
    # 2 vocabulary tiles (512 weight rows) per upload slice and 256-row groups at V=3001, so a
    # small case crosses several slices and several row groups, both ragged.
    monkeypatch.setattr(gk, "_HOST_SLICE_TILES", 2)
    monkeypatch.setattr(gk, "_HOST_PARTIALS_BYTES", 16 * 12 * 256)


@pytest.mark.parametrize("pinned", [True, False], ids=["pinned", "pageable"])
@pytest.mark.parametrize("with_bias", [False, True], ids=["no-bias", "bias"])
def test_host_inputs_match_device_path(small_slices, pinned, with_bias):
    B, H, V = 700, 256, 3001
    h, w, t = rm.make_inputs(B, H, V, seed=11, weight_std=0.1, ignore_frac=0.05, tail_frac=0.02)
    bias = (torch.randn(V, generator=torch.Generator().manual_seed(3)) * 0.5).to(torch.bfloat16) if with_bias else None
    dev = torch.device("cuda", 0)
    ref = gk.gemm_fused_ce_entropy(h.to(dev), w.to(dev), t.to(dev), bias=None if bias is None else bias.to(dev),
                                   chunk_size=256)
    hh, wh, th = (x.pin_memory() if pinned else x for x in (h, w, t))
    bh = None if bias is None else (bias.pin_memory() if pinned else bias)
    out = gk.gemm_fused_ce_entropy(hh, wh, th, bias=bh)
    for a, b in zip(out, ref):
        assert a.device.type == "cpu" and a.shape == b.shape
        assert torch.equal(a, b.cpu())


@pytest.mark.parametrize("head_tiles", [3, 64], ids=["head-3-tiles", "head-covers-weight"])
@pytest.mark.parametrize("with_bias", [False, True], ids=["no-bias", "bias"])
def test_head_first_schedule_matches_device_path(monkeypatch, head_tiles, with_bias):
    """Hidden and weight both on the host: a head of the weight goes up first, the hidden follows in
    256-row chunks (the last one ragged) whose GEMMs against the head write partials at row offsets,
    then 2-tile slices over all rows. With 64 head tiles the head is the whole (12-tile) weight."""
    monkeypatch.setattr(gk, "_HOST_SLICE_TILES", 2)
    monkeypatch.setattr(gk, "_HOST_HEAD_VOCAB", head_tiles * 256)
    monkeypatch.setattr(gk, "_HOST_HIDDEN_CHUNK", 256)
    B, H, V = 700, 256, 3001
    h, w, t = rm.make_inputs(B, H, V, seed=14, weight_std=0.1, ignore_frac=0.05, tail_frac=0.02)
    bias = (torch.randn(V, generator=torch.Generator().manual_seed(4)) * 0.5).to(torch.bfloat16) if with_bias else None
    dev = torch.device("cuda", 0)
    ref = gk.gemm_fused_ce_entropy(h.to(dev), w.to(dev), t.to(dev), bias=None if bias is None else bias.to(dev))
    out = gk.gemm_fused_ce_entropy(h.pin_memory(), w.pin_memory(), t.pin_memory(),
                                   bias=None if bias is None else bias.pin_memory())
    for a, b in zip(out, ref):
        assert a.device.type == "cpu" and torch.equal(a, b.cpu())


def test_host_weight_device_hidden(small_slices):
    """Only the weight on the host (offloaded weight): results land on the hidden's GPU."""
    B, H, V = 300, 128, 1500
    h, w, t = rm.make_inputs(B, H, V, seed=12, weight_std=0.1)
    dev = torch.device("cuda", 0)
    ref = gk.gemm_fused_ce_entropy(h.to(dev), w.to(dev), t.to(dev))
    out = gk.gemm_fused_ce_entropy(h.to(dev), w.pin_memory(), t.to(dev))
    for a, b in zip(out, ref):
        assert a.device == dev
        assert torch.equal(a, b)


def test_host_inputs_batch_shape_and_empty():
    dev = torch.device("cuda", 0)
    h, w, t = rm.make_inputs(2 * 3, 64, 700, seed=13, weight_std=0.1)
    out = gk.gemm_fused_ce_entropy(h.view(2, 3, 64), w, t.view(2, 3))
    ref = gk.gemm_fused_ce_entropy(h.view(2, 3, 64).to(dev), w.to(dev), t.view(2, 3).to(dev))
    for a, b in zip(out, ref):
        assert a.shape == (2, 3) and torch.equal(a, b.cpu())
    empty = gk.gemm_fused_ce_entropy(h[:0], w, t[:0])
    assert all(x.shape == (0,) and x.device.type == "cpu" for x in empty)
