"""The C ABI from a plain C program (tests/c_caller/frx_c_caller.c): no Python or torch in the
caller's process. CPU: it compiles and links against libfrx.so with only include/frx.h and the CUDA
runtime. GPU: it runs the training pass through the ABI and checks it in double precision."""

import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
SRC = ROOT / "tests" / "c_caller" / "frx_c_caller.c"
LIBDIR = ROOT / "fast-reduction_b200" / "fast_reduction" / "_native"
CUDA = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


def _compile(out: Path) -> None:
    gcc = shutil.which("gcc")
    if gcc is None or not (CUDA / "include" / "cuda_runtime.h").exists():
        pytest.skip("gcc or the CUDA runtime headers are not available")
    if not (LIBDIR / "libfrx.so").exists():
        pytest.skip("libfrx.so is not built")
    cmd = [gcc, "-std=c11", "-O2", "-Wall", "-Wextra", "-Werror", f"-I{ROOT / 'include'}", f"-I{CUDA / 'include'}",
           str(SRC), f"-L{LIBDIR}", "-lfrx", f"-L{CUDA / 'lib64'}", "-lcudart", "-lm", f"-Wl,-rpath,{LIBDIR}",
           "-o", str(out)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr


def test_c_caller_compiles_and_links(tmp_path):
    _compile(tmp_path / "frx_c_caller")
    assert (tmp_path / "frx_c_caller").exists()


@pytest.mark.gpu
def test_c_caller_training_pass_matches_double_precision(tmp_path):
    exe = tmp_path / "frx_c_caller"
    _compile(exe)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "frx C caller ok" in res.stdout
