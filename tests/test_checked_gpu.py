"""GPU: the checked build (libfrx_checked.so, FRX_CHECKED=1) and the buffer range check behind it.

frx_check_range (exported by every build) accepts a range inside one device allocation and refuses
host memory and ranges that run past the allocation's end, without launching anything. The checked
build runs that check on every buffer before each launch plus device-side invariant checks; the
parity suites pass under it (a failed device check would surface as FRX_STATUS_CHECK_FAILED through
the suites' status-word fixtures)."""

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]


def test_check_range_accepts_inside_and_refuses_outside():
    from fast_reduction import _native as nat

    lib = nat.load()
    x = torch.empty(1000, device="cuda", dtype=torch.float32)
    assert lib.frx_check_range(x.data_ptr(), x.numel() * 4) == nat.FRX_OK
    assert lib.frx_check_range(x.data_ptr() + 40, 400) == nat.FRX_OK
    assert lib.frx_check_range(x.data_ptr(), 1 << 40) == nat.FRX_ERR_INVALID_ARG  # far past the allocation
    assert b"past the end" in lib.frx_last_error()
    host = torch.empty(1000, dtype=torch.float32)
    assert lib.frx_check_range(host.data_ptr(), 4000) == nat.FRX_ERR_INVALID_ARG  # not device memory
    assert lib.frx_check_range(None, 0) == nat.FRX_OK


def test_parity_suites_pass_under_the_checked_build():
    sys.path.insert(0, str(REPO / "fast-reduction_b200"))
    import build as frx_build

    frx_build.build(checked=True)
    env = dict(os.environ, FRX_LIB="checked")
    suites = ["tests/test_fwd_gpu.py", "tests/test_bwd_gpu.py", "tests/test_reductions_gpu.py",
              "tests/test_fp16_gpu.py", "tests/test_fp32_gpu.py", "tests/test_host_stream_gpu.py",
              "tests/test_zz_no_alloc.py"]
    code = ("import sys; from fast_reduction import _native as nat; "
            "assert nat.library_path().name == 'libfrx_checked.so', nat.library_path()")
    probe_env = dict(env, PYTHONPATH=str(REPO / "fast-reduction_b200"))
    probe = subprocess.run([sys.executable, "-c", code], cwd=REPO, env=probe_env, capture_output=True, text=True,
                           timeout=300)
    assert probe.returncode == 0, probe.stderr[-2000:]
    out = subprocess.run([sys.executable, "-m", "pytest", *suites, "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider"],
                         cwd=REPO, env=env, capture_output=True, text=True, timeout=1200)
    assert out.returncode == 0, (out.stdout[-3000:], out.stderr[-2000:])


def test_clock_probe_reads_a_plausible_sm_clock():
    """frx_clock_probe stamps every SM; two probes around GPU work give that work's SM clock."""
    from fast_reduction import _native as nat

    lib = nat.load()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    buf = torch.zeros(2, 2 * 256, dtype=torch.int64, device="cuda")
    stream = nat.stream_of(buf.device)
    assert lib.frx_clock_probe(buf[0].data_ptr(), 256, stream) == nat.FRX_OK
    a = torch.randn(4096, 4096, device="cuda")
    for _ in range(20):
        a = a @ a * 1e-3
    assert lib.frx_clock_probe(buf[1].data_ptr(), 256, stream) == nat.FRX_OK
    b = buf.cpu().view(2, 256, 2)
    stamped = [s for s in range(256) if b[0, s, 1] and b[1, s, 1]]
    assert len(stamped) >= sms // 2
    mhz = sorted(float(b[1, s, 0] - b[0, s, 0]) / float(b[1, s, 1] - b[0, s, 1]) * 1000 for s in stamped)
    assert 300 < mhz[len(mhz) // 2] < 2500
    assert lib.frx_clock_probe(buf[0].data_ptr(), 0, stream) == nat.FRX_ERR_INVALID_ARG
