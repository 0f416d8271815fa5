"""GPU: failure detection without a fault. A test hook leaves one pipeline stage of the forward GEMM
unfilled on purpose (a barrier nothing will complete); the MMA warp's bounded wait runs out, the
kernel takes its abort path (roles leave their loops, in-flight copies and MMAs are waited for,
tensor memory is freed) and reports FRX_STATUS_TIMEOUT_* bits, and the context stays usable: the
next forward on the same stream is correct. Covers the CTA-pair kernel (default) and, in a child
process, the single-CTA kernel."""

import os
import subprocess
import sys
import time
from pathlib import Path

import pytest
import torch

from oracle import reference_math as rm

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
REPO = Path(__file__).resolve().parents[1]
TIMEOUT_BITS = 1 | 2 | 4 | 16  # producer / MMA / epilogue timeouts, drain timeout


def stall_once_and_recover() -> dict:
    from fast_reduction import _native as nat
    from fast_reduction import ops
    from fast_reduction.gemm_kernel import gemm_fused_ce_entropy

    lib = nat.load()
    B, H, V = 512, 512, 2048
    h, w, t = rm.make_inputs(B, H, V, seed=3, weight_std=0.1)
    hd, wd, td = h.to(DEV), w.to(DEV), t.to(DEV)
    T = ops.n_vocab_tiles(V)
    partials = torch.zeros(T, B, 4, device=DEV)
    torch.cuda.synchronize()
    nat.read_status(DEV)  # start from a clean status word
    t0 = time.perf_counter()
    rc = lib.frx_test_stalled_fwd(hd.data_ptr(), H, wd.data_ptr(), H, td.data_ptr(), B, V, H, partials.data_ptr(), B,
                                  1, 20000, nat.status_word(DEV).data_ptr(), nat.stream_of(DEV))
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    bits = nat.read_status(DEV)  # read and clear
    ce, ent, _ = gemm_fused_ce_entropy(hd, wd, td, chunk_size=256)
    ce_r, ent_r, _, _ = rm.fp32_reference(h, w, t)
    err = max(float((ce.cpu() - ce_r).abs().max()), float((ent.cpu() - ent_r).abs().max()))
    after = nat.read_status(DEV)
    return {"rc": rc, "bits": bits, "elapsed": elapsed, "err": err, "after": after}


def _check(r):
    assert r["rc"] == 0
    assert r["bits"] & 2, f"the MMA warp's wait should have run out, status 0x{r['bits']:x}"
    assert r["bits"] & ~TIMEOUT_BITS == 0, f"unexpected status bits 0x{r['bits']:x}"
    assert r["elapsed"] < 10.0  # bounded: 20 ms waits plus bounded drains
    assert r["err"] < 2e-3  # the context is usable and the next forward is right
    assert r["after"] == 0


def test_stalled_pair_pipeline_times_out_and_recovers():
    _check(stall_once_and_recover())


def test_stalled_single_cta_pipeline_times_out_and_recovers():
    code = ("import sys, json; sys.path[:0] = [%r, %r, %r];"
            "import test_failure_gpu as t; print('RESULT', json.dumps(t.stall_once_and_recover()))"
            % (str(REPO / "tests"), str(REPO / "fast-reduction_b200"), str(REPO)))
    env = dict(os.environ, FRX_GEMM_VARIANT="single")
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    import json

    line = [x for x in out.stdout.splitlines() if x.startswith("RESULT ")][-1]
    _check(json.loads(line[len("RESULT "):]))
