"""GPU: concurrent callers. ctypes releases the GIL inside every libfrx call, so Python threads call
the library concurrently: each thread, on its own CUDA stream, runs the forward and the training pass
over its own inputs while the others do the same, and every result equals the same calls made
alone, bit for bit (the kernels are deterministic and keep no state between calls)."""

import concurrent.futures as cf

import pytest
import torch

from oracle import reference_math as rm

pytestmark = pytest.mark.gpu


def _case(i):
    B, H, V = 520 + 64 * i, 256, 3001 + 500 * i
    h, w, t = rm.make_inputs(B, H, V, seed=40 + i, weight_std=0.1, ignore_frac=0.05)
    return h.cuda(), w.cuda(), t.cuda()


def _run(h, w, t):
    from fast_reduction.gemm_kernel import gemm_fused_ce_entropy, gemm_megakernel_fast

    ce, ent, lp = gemm_fused_ce_entropy(h, w, t, chunk_size=256)
    hd = h.detach().clone().requires_grad_(True)
    wd = w.detach().clone().requires_grad_(True)
    loss, _, _ = gemm_megakernel_fast(hd, wd, t, chunk_size=256)
    loss.backward()
    return [ce, ent, lp, loss.detach(), hd.grad, wd.grad]


def test_threads_on_own_streams_match_serial_calls():
    from fast_reduction import _native as nat

    cases = [_case(i) for i in range(4)]
    serial = [_run(*c) for c in cases]
    torch.cuda.synchronize()

    def work(i):
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.default_stream())
        with torch.cuda.stream(stream):
            outs = None
            for _ in range(3):
                outs = _run(*cases[i])
        stream.synchronize()
        return outs

    with cf.ThreadPoolExecutor(max_workers=4) as ex:
        parallel = list(ex.map(work, range(4)))
    torch.cuda.synchronize()
    nat.raise_on_status(torch.device("cuda", 0))
    for i, (got, want) in enumerate(zip(parallel, serial)):
        for name, a, b in zip(("ce", "entropy", "log_probs", "loss", "d_hidden", "d_weight"), got, want):
            assert torch.equal(a, b), (i, name)
