"""CPU: libfrx.so loads, exports exactly what include/frx.h declares, and rejects bad arguments
with a status code and message (no abort, no GPU needed for argument checks)."""

import ctypes
import re
from pathlib import Path


REPO = Path(__file__).resolve().parents[1]
HEADER = REPO / "include" / "frx.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*FRX_API\s+(?:const\s+)?\w+\s*\*?\s*(frx_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = declared_functions()
    for must in ("frx_fwd_partials", "frx_finalize", "frx_dlogits", "frx_gemm_dhidden", "frx_gemm_dweight",
                 "frx_logits_partials", "frx_column_sums", "frx_last_error", "frx_abi_version"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from fast_reduction import _native as nat

    lib = nat.load()
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in frx.h but not exported"
        assert name in nat.SIGNATURES, f"{name} has no ctypes signature in _native.py"


def test_abi_version_and_error_string():
    from fast_reduction import _native as nat

    lib = nat.load()
    hdr = HEADER.read_text()
    ver = int(re.search(r"#define FRX_ABI_VERSION (\d+)", hdr).group(1))
    assert lib.frx_abi_version() == ver
    assert isinstance(lib.frx_last_error(), bytes)


def test_constants_match_header():
    from fast_reduction import _native as nat

    hdr = HEADER.read_text()
    for name in ("FRX_OK", "FRX_ERR_INVALID_ARG", "FRX_ERR_UNSUPPORTED", "FRX_ERR_CUDA", "FRX_DTYPE_BF16",
                 "FRX_DTYPE_F32", "FRX_DTYPE_F16", "FRX_VOCAB_TILE", "FRX_PARTIALS_REF_LAYOUT",
                 "FRX_IGNORE_NEGATIVE_TARGETS", "FRX_STATUS_BAD_TARGET",
                 "FRX_STATUS_TIMEOUT_PRODUCER", "FRX_STATUS_TIMEOUT_MMA", "FRX_STATUS_TIMEOUT_EPILOGUE",
                 "FRX_STATUS_DRAIN_TIMEOUT", "FRX_OUT_ACCUMULATE", "FRX_PART_HI", "FRX_PART_MID", "FRX_PART_LO"):
        val = int(re.search(rf"#define {name} (\d+)", hdr).group(1))
        assert getattr(nat, name) == val, name


def test_invalid_arguments_return_codes_without_gpu():
    from fast_reduction import _native as nat

    lib = nat.load()
    # negative sizes are rejected before any CUDA call
    rc = lib.frx_fwd_partials(None, 0, None, 0, 0, None, None, -1, 10, 64, 0, None, 0, None, 0, None, None)
    assert rc == nat.FRX_ERR_INVALID_ARG
    assert b"bad sizes" in lib.frx_last_error()
    rc = lib.frx_fwd_partials(1 << 20, 64, 1 << 21, 64, 0, None, None, 8, 10, 60, 0, 1 << 22, 8, None, 0, None, None)
    assert rc == nat.FRX_ERR_UNSUPPORTED  # hidden_dim not a multiple of 8
    rc = lib.frx_fwd_partials(1 << 20, 64, 1 << 21, 64, nat.FRX_DTYPE_F32, None, None, 8, 10, 64, 0, 1 << 22, 8,
                              None, 0, None, None)
    assert rc == nat.FRX_ERR_UNSUPPORTED  # fp32 operands: the GEMM core takes bf16 or fp16
    assert b"dtype" in lib.frx_last_error()
    rc = lib.frx_finalize(None, 3, 10, 5, 0, None, 0, 0, None, None, None, None, None, None, None)
    assert rc == nat.FRX_ERR_INVALID_ARG  # tile_stride < rows
    rc = lib.frx_finalize(None, 1, 10, 10, 0x40, None, 0, 0, None, None, None, None, None, None, None)
    assert rc == nat.FRX_ERR_INVALID_ARG  # unknown flag
    rc = lib.frx_dlogits(None, 0, None, None, None, None, None, 1.0, -1.0, None, 0, 7, 4, 4, 0, 0, None)
    assert rc == nat.FRX_ERR_INVALID_ARG
    rc = lib.frx_gemm_dhidden(None, 0, None, 0, 0, None, 0, 0, -5, 64, 64, None, None)
    assert rc == nat.FRX_ERR_INVALID_ARG
    rc = lib.frx_gemm_dweight(None, 0, None, 0, 0, None, 0, 0, 64, 64, 0, None, None)
    assert rc == nat.FRX_ERR_INVALID_ARG
    rc = lib.frx_column_sums(1 << 20, nat.FRX_DTYPE_F32, 8, 4, 8, 1 << 21, None)
    assert rc == nat.FRX_ERR_INVALID_ARG  # column sums read 16-bit matrices only
    rc = lib.frx_dlogits(1 << 20, 8, None, 1 << 21, 1 << 21, None, None, 1.0, -1.0, 1 << 22, 8, 9, 4, 4, 0, 0, None)
    assert rc == nat.FRX_ERR_INVALID_ARG  # unknown out_dtype
    rc = lib.frx_gemm_dhidden(1 << 20, 64, 1 << 21, 64, 0, 1 << 22, 64, nat.FRX_DTYPE_BF16 | nat.FRX_OUT_ACCUMULATE,
                              64, 64, 64, None, None)
    assert rc == nat.FRX_ERR_INVALID_ARG  # accumulation needs an fp32 output
    assert b"FRX_OUT_ACCUMULATE" in lib.frx_last_error()
    rc = lib.frx_split_f32(1 << 20, 8, 4, 8, 3, 1, 1 << 21, 8, 32, None)
    assert rc == nat.FRX_ERR_INVALID_ARG  # part selector 3 does not exist
    assert lib.frx_split_f32(None, 8, 0, 8, 0, 1, None, 8, 0, None) == nat.FRX_OK  # empty
    rc = lib.frx_test_stalled_fwd(1 << 20, 64, 1 << 21, 64, None, 8, 256, 64, 1 << 22, 8, 5, 1000, None, None)
    assert rc == nat.FRX_ERR_INVALID_ARG  # stall past the last k-block
    rc = lib.frx_test_stalled_fwd(1 << 20, 64, 1 << 21, 64, None, 8, 256, 64, 1 << 22, 8, 0, 0, None, None)
    assert rc == nat.FRX_ERR_INVALID_ARG  # wait limit must be positive
    rc = lib.frx_gemm_dweight_sms(1 << 20, 64, 1 << 21, 64, 0, 1 << 22, 64, 0, 8, 64, 8, -1, None, None)
    assert rc == nat.FRX_ERR_INVALID_ARG and b"max_sms" in lib.frx_last_error()


def _stub_module():
    import importlib.util

    spec = importlib.util.spec_from_file_location("frx_ctypes_stub", REPO / "include" / "frx_ctypes.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_reference_side_stub_matches_the_bindings():
    """include/frx_ctypes.py (the binding a maintainer adds to the reference package) declares, for
    every entry point of include/frx.h, the same argument types as the package's own binding."""
    from fast_reduction import _native as nat

    stub = _stub_module()
    for name in declared_functions():
        if name == "frx_last_error":
            continue
        assert name in stub.ARGTYPES, f"{name} missing from include/frx_ctypes.py"
        assert list(stub.ARGTYPES[name]) == list(nat.SIGNATURES[name][1]), name
    lib = stub.load(str(nat._LIB_PATH))
    assert lib.frx_abi_version() == nat.load().frx_abi_version()


def test_reference_side_stub_calls_pass_every_argument():
    """Every `_lib.frx_*(...)` call in include/frx_ctypes.py passes as many arguments as the entry
    point takes."""
    import ast

    from fast_reduction import _native as nat

    tree = ast.parse((REPO / "include" / "frx_ctypes.py").read_text())
    seen = 0
    for node in ast.walk(tree):
        if (isinstance(node, ast.Call) and isinstance(node.func, ast.Attribute)
                and isinstance(node.func.value, ast.Name) and node.func.value.id == "_lib"
                and node.func.attr.startswith("frx_") and node.func.attr != "frx_last_error"):
            assert len(node.args) == len(nat.SIGNATURES[node.func.attr][1]), node.func.attr
            seen += 1
    assert seen >= 13


def test_last_error_is_per_thread():
    """frx_last_error() reports the last failure of the calling thread only (ctypes releases the
    GIL around each call, so the two threads' calls interleave for real)."""
    import threading

    from fast_reduction import _native as nat

    lib = nat.load()
    step = threading.Barrier(2, timeout=30)
    seen = {}

    def a():
        lib.frx_fwd_partials(None, 0, None, 0, 0, None, None, -1, 10, 64, 0, None, 0, None, 0, None, None)
        step.wait()  # 1: A has failed
        step.wait()  # 2: B has failed
        seen["a"] = lib.frx_last_error()

    def b():
        step.wait()
        seen["b_before"] = lib.frx_last_error()
        lib.frx_fwd_partials(1 << 20, 64, 1 << 21, 64, nat.FRX_DTYPE_F32, None, None, 8, 10, 64, 0, 1 << 22, 8,
                             None, 0, None, None)
        seen["b"] = lib.frx_last_error()
        step.wait()

    threads = [threading.Thread(target=a), threading.Thread(target=b)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(60)
    assert b"bad sizes" in seen["a"] and b"dtype" not in seen["a"]
    assert seen["b_before"] == b""
    assert b"dtype" in seen["b"] and b"bad sizes" not in seen["b"]


def test_empty_problems_are_noops():
    from fast_reduction import _native as nat

    lib = nat.load()
    assert lib.frx_fwd_partials(None, 0, None, 0, 0, None, None, 0, 10, 64, 0, None, 0, None, 0, None,
                                None) == nat.FRX_OK
    assert lib.frx_finalize(None, 0, 0, 0, 0, None, 0, 0, None, None, None, None, None, None, None) == nat.FRX_OK


def test_checked_build_exports_the_same_symbols():
    """libfrx_checked.so (FRX_CHECKED=1) is a drop-in for libfrx.so: same exported entry points."""
    import sys

    sys.path.insert(0, str(REPO / "fast-reduction_b200"))
    import build as frx_build

    path = frx_build.build(checked=True)
    lib = ctypes.CDLL(str(path))
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} missing from the checked build"
    lib.frx_check_range.argtypes = [ctypes.c_void_p, ctypes.c_int64]
    assert lib.frx_check_range(None, 0) == 0
