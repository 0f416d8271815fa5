"""CPU: host-side validation of the drop-in API raises before any device work, mirroring the
reference's Python-level error behaviour (asserts / KeyError / NotImplementedError)."""

import pytest
import torch

from fast_reduction import gemm_kernel as gk
from fast_reduction import ops
from fast_reduction.gemm_ce_entropy_finalize import finalize_ce_entropy
from fast_reduction.cute_dlogits import compute_dlogits


def _inputs(dtype=torch.bfloat16, B=8, H=16, V=40):
    return torch.randn(B, H).to(dtype), torch.randn(V, H).to(dtype), torch.randint(0, V, (B,))


def test_cpu_tensors_rejected_no_fallback():
    h, w, t = _inputs()
    with pytest.raises(ValueError, match="CUDA"):
        gk.gemm_megakernel_fast(h, w, t)
    if not torch.cuda.is_available():
        # host inputs are streamed to a GPU, never computed on the CPU
        with pytest.raises(RuntimeError, match="CUDA device"):
            gk.gemm_fused_ce_entropy(h, w, t)


def test_host_input_device_rules():
    h, w, t = _inputs()
    assert gk._input_device(None, None) is None
    meta = torch.empty(4, device="meta")
    with pytest.raises(ValueError, match="CUDA or CPU"):
        gk._input_device(h, meta)
    if not torch.cuda.is_available():
        with pytest.raises(RuntimeError, match="CUDA device"):
            gk._input_device(h, w, t)


def test_bias_checks():
    h, w, t = _inputs()
    with pytest.raises(ValueError, match="bias must be"):
        gk.gemm_fused_ce_entropy(h, w, t, bias=torch.zeros(39, dtype=torch.bfloat16))
    with pytest.raises(NotImplementedError, match="weight's dtype"):
        gk.gemm_fused_ce_entropy(h, w, t, bias=torch.zeros(40))


def test_unsupported_dtypes_rejected():
    h, w, t = _inputs(dtype=torch.float64)
    with pytest.raises(NotImplementedError, match="bf16, fp16 or fp32"):
        gk.gemm_fused_ce_entropy(h, w, t)
    h, w, t = _inputs()
    with pytest.raises(NotImplementedError, match="same type"):
        gk.gemm_fused_ce_entropy(h, w.to(torch.float16), t)
    with pytest.raises(TypeError, match="all be bfloat16 or all float16"):
        ops._gemm_dtype(h, w.to(torch.float16))
    assert ops._gemm_dtype(h.half(), w.half()) == ops.nat.FRX_DTYPE_F16


def test_shape_checks():
    h, w, t = _inputs()
    with pytest.raises(ValueError, match="hidden size mismatch"):
        gk.gemm_fused_ce_entropy(h, w[:, :8], t)
    with pytest.raises(ValueError, match="target has"):
        gk.gemm_fused_ce_entropy(h, w, t[:3])
    h2 = torch.randn(8, 12).to(torch.bfloat16)
    with pytest.raises(NotImplementedError, match="multiple of 8"):
        gk.gemm_fused_ce_entropy(h2, torch.randn(40, 12).to(torch.bfloat16), t)
    with pytest.raises(TypeError):
        gk.gemm_fused_ce_entropy(h, w, t.float())


def test_finalize_mirror_checks():
    with pytest.raises(ValueError, match=r"\[N_tiles, M, 4\]"):
        finalize_ce_entropy(torch.zeros(2, 3, 5), 2)
    with pytest.raises(ValueError, match="n_tiles"):
        finalize_ce_entropy(torch.zeros(2, 3, 4), 3)


def test_dlogits_mirror_checks():
    from fast_reduction import cute_dlogits

    with pytest.raises(ValueError, match="CUDA"):
        compute_dlogits(torch.zeros(2, 3), torch.zeros(2, dtype=torch.int64), torch.zeros(2), torch.zeros(2),
                        torch.zeros(2), torch.zeros(2))
    with pytest.raises(KeyError):  # the reference maps only int32 / int64 targets
        cute_dlogits._prep_target(torch.zeros(2, dtype=torch.int16))


def test_tile_helpers():
    assert ops.n_vocab_tiles(128256) == 501
    assert ops.n_vocab_tiles(256) == 1 and ops.n_vocab_tiles(257) == 2
    assert ops.round_up(1000, 8) == 1000 and ops.round_up(1001, 8) == 1008


def test_forward_launch_rows():
    """Rows per forward launch: chunk_size, or a multiple of it while one launch's partials stay
    within _FWD_LAUNCH_PARTIALS_BYTES (48 MiB)."""
    T = ops.n_vocab_tiles
    assert gk._launch_rows(4096, 32768, T(128256)) == 4096      # full vocabulary: as given
    assert gk._launch_rows(4096, 32768, T(64128)) == 12288      # 2 GPUs: 3 chunks per launch
    assert gk._launch_rows(4096, 32768, T(32064)) == 24576      # 4 GPUs: 6 chunks per launch
    assert gk._launch_rows(4096, 32768, T(16032)) == 32768      # 8 GPUs: one launch
    assert gk._launch_rows(512, 1024, T(32000)) == 1024
    assert gk._launch_rows(300, 200, T(1000)) == 200
    assert gk._launch_rows(4096, 65536, T(1 << 24)) == 4096     # partials of one chunk exceed the budget


def test_training_launch_rows():
    """chunk_size caps the training pass's logits memory at the reference's per-chunk fp32 logits
    buffer (chunk x V x 4 bytes): all rows in one launch when they fit, else two buffers of a
    multiple of chunk rows, never fewer than chunk rows."""
    V = 128256
    ld16, ld32 = ops.round_up(V, 8), ops.round_up(V, 4)
    # one GPU, headline: 2-byte logits give two 4096-row buffers (= one fp32 chunk buffer)
    assert gk._train_launch_rows(4096, 32768, ld16, 2, V) == 4096
    assert gk._train_launch_rows(4096, 32768, ld32, 4, V) == 4096
    # vocabulary shards of the headline over 2 / 4 / 8 GPUs
    assert gk._train_launch_rows(4096, 32768, ops.round_up(64128, 8), 2, V) == 8192
    assert gk._train_launch_rows(4096, 32768, ops.round_up(32064, 8), 2, V) == 32768
    assert gk._train_launch_rows(4096, 32768, ops.round_up(16032, 8), 2, V) == 32768
    # fewer rows than a chunk, and the opt-out
    assert gk._train_launch_rows(4096, 100, ld16, 2, V) == 100
    old = gk._TRAIN_MERGE
    try:
        gk._TRAIN_MERGE = False
        assert gk._train_launch_rows(4096, 32768, ops.round_up(16032, 8), 2, V) == 4096
    finally:
        gk._TRAIN_MERGE = old


def test_dhidden_overlap_rule():
    """SMs the d_weight GEMM leaves for the vocabulary-parallel d_hidden collective: only where its
    extra waves cost less than the collective hides (8 GPUs at the headline shape and configs[4])."""
    from fast_reduction import vocab_parallel as vp

    def free(B, H, V, N):
        a, b = vp.shard_bounds(V, N, 0)
        return vp._dh_overlap_sms(N, B, H, b - a, 148, 2)

    assert [free(32768, 4096, 128256, n) for n in (1, 2, 4, 8)] == [0, 0, 0, 32]
    assert [free(65536, 5120, 152064, n) for n in (2, 4, 8)] == [0, 0, 32]
    assert [free(16384, 4096, 256000, n) for n in (2, 4, 8)] == [0, 0, 0]


def test_host_upload_plan():
    """Upload schedule of the host-streamed forward (no GPU needed): a weight head before the hidden
    when both are on the host, hidden chunks only with a head, and weight slices that start small,
    double up to the slice size and tile [head, V) without gaps."""
    tile = ops.VOCAB_TILE

    def check_slices(slices, start, V):
        assert slices[0][0] == start and slices[-1][1] == V
        assert all(a < b for a, b in slices)
        assert all(x[1] == y[0] for x, y in zip(slices, slices[1:]))
        assert all(a % tile == 0 for a, _ in slices)

    head, chunks, slices = gk._host_upload_plan(32768, 128256, w_host=True, h_host=True, shared_hidden=False,
                                                one_group=True)
    assert head == gk._HOST_HEAD_VOCAB == 24576
    assert chunks == [(a, a + 2048) for a in range(0, 32768, 2048)]
    check_slices(slices, head, 128256)
    sizes = [(b - a) // tile for a, b in slices]
    assert sizes[:4] == [4, 8, 16, 32] and max(sizes) == gk._HOST_SLICE_TILES
    # no head: hidden split over ranks, hidden already on the device, or several partials groups
    for kw in (dict(h_host=True, shared_hidden=True, one_group=True), dict(h_host=False, shared_hidden=False,
               one_group=True), dict(h_host=True, shared_hidden=False, one_group=False)):
        head, chunks, slices = gk._host_upload_plan(32768, 64128, w_host=True, **kw)
        assert head == 0 and chunks == []
        check_slices(slices, 0, 64128)
    # weight resident: one "slice" covering it, no head
    assert gk._host_upload_plan(100, 5000, w_host=False, h_host=True, shared_hidden=False,
                                one_group=True) == (0, [], [(0, 5000)])
    # a vocabulary smaller than the head: the whole weight is the head, no slices after the hidden
    head, chunks, slices = gk._host_upload_plan(5000, 3001, w_host=True, h_host=True, shared_hidden=False,
                                                one_group=True)
    assert head == 3001 and slices == [] and chunks[-1] == (4096, 5000)


def test_lazy_exports():
    import fast_reduction

    assert gk.GemmFusedCEEntropyFast is gk.GemmMegakernel

    assert fast_reduction.gemm_fused_ce_entropy is gk.gemm_fused_ce_entropy
    assert fast_reduction.gemm_megakernel_fast is gk.gemm_megakernel_fast
    with pytest.raises(AttributeError):
        fast_reduction.does_not_exist


def test_nvtx_phase_is_harmless_without_a_profiler():
    with ops.phase("frx.test.phase"):
        pass
