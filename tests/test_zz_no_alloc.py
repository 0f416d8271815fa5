"""GPU: the allocation-free forward entry point (frx_fwd_ce_entropy_noalloc).

It exists for callers that cannot call cudaMalloc on their call path (a framework that owns all
device memory, a serving loop that must not synchronise on an allocation, a fixed memory budget):
the partials between the GEMM and the finalize live in a 32 MiB array inside the library image.
This file is collected last on purpose; it checks the entry point, through the C ABI, against the
existing two-call path (frx_fwd_partials + frx_finalize with a caller-allocated partials buffer)
on two calls in a row, and that oversized calls are refused.
"""

import pytest
import torch

from oracle import reference_math as rm

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _noalloc(lib, h, w, t, ignore_index=-100):
    B, H = h.shape
    V = w.shape[0]
    outs = [torch.full((B,), float("nan"), device=DEV) for _ in range(4)]
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = lib.frx_fwd_ce_entropy_noalloc(
        h.data_ptr(), h.stride(0), w.data_ptr(), w.stride(0), t.data_ptr(), B, V, H, ignore_index,
        outs[0].data_ptr(), outs[1].data_ptr(), outs[2].data_ptr(), outs[3].data_ptr(), status.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    return rc, outs, status


def _existing_path(h, w, t, ignore_index=-100):
    from fast_reduction import ops

    B = h.shape[0]
    V = w.shape[0]
    T = ops.n_vocab_tiles(V)
    partials = torch.empty(T, B, 4, device=DEV)
    ops.fwd_partials(h, w, t, partials, B)
    outs = [torch.empty(B, device=DEV) for _ in range(4)]
    ops.finalize(partials, T, B, B, target=t, vocab_size=V, ignore_index=ignore_index, ce=outs[0], entropy=outs[1],
                 lse=outs[2], log_probs=outs[3])
    return outs


def test_noalloc_matches_existing_path_two_calls_in_a_row():
    from fast_reduction import _native as nat

    lib = nat.load()
    # The first call fills 63 vocabulary tiles x 2048 rows of the scratch; the second (same rows,
    # 20 tiles) lands entirely on slots that still hold the first call's partials, so a slot it
    # failed to write would show up as a mismatch. The third changes the row count (new layout).
    cases = [(2048, 512, 128256 // 8, 2), (2048, 256, 5000, 1), (1000, 256, 5000, 3)]
    for B, H, V, seed in cases:
        h, w, t = rm.make_inputs(B, H, V, seed=seed, weight_std=0.1, ignore_frac=0.02)
        h, w, t = h.to(DEV), w.to(DEV), t.to(DEV)
        rc, got, status = _noalloc(lib, h, w, t)
        assert rc == nat.FRX_OK, lib.frx_last_error()
        exp = _existing_path(h, w, t)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        for g, e in zip(got, exp):
            torch.testing.assert_close(g, e, atol=1e-6, rtol=1e-6)
        ignored = t == -100
        assert int(ignored.sum()) > 0
        assert bool((got[0][ignored] == 0).all()) and bool((got[3][ignored] == 0).all())
        assert bool(torch.isfinite(got[1]).all()) and bool(torch.isfinite(got[2]).all())
        ce32, ent32, lp32, lse32 = rm.fp32_reference(h, w, t)
        assert (got[0] - ce32).abs().mean() <= 2e-3
        assert (got[1] - ent32).abs().mean() <= 1e-4


def test_noalloc_rejects_calls_beyond_the_scratch():
    from fast_reduction import _native as nat

    lib = nat.load()
    V, H = 128256, 64
    w = torch.zeros(V, H, device=DEV, dtype=torch.bfloat16)
    h = torch.zeros(4200, H, device=DEV, dtype=torch.bfloat16)  # 4200 * 501 * 16 B > 32 MiB
    t = torch.zeros(4200, device=DEV, dtype=torch.int64)
    rc, _, _ = _noalloc(lib, h, w, t)
    assert rc == nat.FRX_ERR_INVALID_ARG
    max_rows = (32 << 20) // 16 // 501  # 32 MiB of float4 slots over 501 vocabulary tiles
    assert f"at most {max_rows} rows".encode() in lib.frx_last_error()
