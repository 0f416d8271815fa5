"""ctypes binding of libfrx.so as the reference package would add it (as fast_reduction/_frx.py).

The reference's Level-5 path launches CuTe-DSL kernels from fast_reduction/gemm_kernel.py; each
function below replaces one of those launches with one C call on torch's current stream, with the
arguments include/frx.h documents. ARGTYPES declares every entry point of the C ABI.
The package in this repository binds the same ABI itself (fast_reduction/_native.py, ops.py);
tests/test_abi.py checks that both declare the same signatures and that every call below passes
every argument.
"""

import ctypes

import torch

P, I64, I32, F32, U32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_uint32

ARGTYPES = {
    "frx_fwd_partials": [P, I64, P, I64, I32, P, P, I64, I64, I64, I64, P, I64, P, I64, P, P],
    "frx_fwd_partials_tilerel": [P, I64, P, I64, I32, P, P, I64, I64, I64, I64, P, I64, P, I64, P, P],
    "frx_finalize": [P, I64, I64, I64, I32, P, I64, I64, P, P, P, P, P, P, P],
    "frx_dlogits": [P, I64, P, P, P, P, P, F32, F32, P, I64, I32, I64, I64, I64, I64, P],
    "frx_dlogits_tilerel": [P, I64, P, I64, P, P, P, P, P, F32, F32, P, I64, I32, I64, I64, I64, I64, P],
    "frx_gemm_dhidden": [P, I64, P, I64, I32, P, I64, I32, I64, I64, I64, P, P],
    "frx_gemm_dweight": [P, I64, P, I64, I32, P, I64, I32, I64, I64, I64, P, P],
    "frx_gemm_dweight_sms": [P, I64, P, I64, I32, P, I64, I32, I64, I64, I64, I32, P, P],
    "frx_column_sums": [P, I32, I64, I64, I64, P, P],
    "frx_split_f32": [P, I64, I64, I64, U32, I32, P, I64, I64, P],
    "frx_logits_partials": [P, I32, I64, I64, I64, P, I64, P, I64, P],
    "frx_loss_sum": [P, P, I64, F32, F32, P, P],
    "frx_scale_inplace": [P, I32, I64, P, P],
    "frx_fwd_ce_entropy_noalloc": [P, I64, P, I64, P, I64, I64, I64, I64, P, P, P, P, P, P],
    "frx_gemm_dhidden_multicast": [P, I64, P, I64, I32, P, I64, I64, I64, I64, P, P],
    "frx_test_stalled_fwd": [P, I64, P, I64, P, I64, I64, I64, P, I64, I32, I64, P, P],
    "frx_check_range": [P, I64],
    "frx_clock_probe": [P, I32, P],
    "frx_abi_version": [],
}

FRX_DTYPE = {torch.bfloat16: 0, torch.float32: 1, torch.float16: 2}
NO_IGNORE = -(2**63)  # an ignore_index no target equals (the reference kernels have no ignore rule)

_lib = None


def load(path: str = "libfrx.so"):
    """Opens libfrx.so and declares every entry point (restype int, argtypes above)."""
    global _lib
    lib = ctypes.CDLL(path)
    for name, args in ARGTYPES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = I32
    lib.frx_last_error.argtypes = []
    lib.frx_last_error.restype = ctypes.c_char_p
    _lib = lib
    return lib


def _check(rc: int) -> None:
    if rc:
        raise RuntimeError(_lib.frx_last_error().decode())


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


def fwd_partials(A, W, target, partials, *, bias=None, logits=None, vocab_offset=0):
    """Replaces `_gemm_ce_entropy_kernel` (gemm_kernel.py:58-165) and, with fp32 `logits`,
    `_gemm_ce_entropy_bwd_kernel` (:168-273). partials: fp32 [ceil(V / 256), M, 4]."""
    M, K = A.shape
    V = W.shape[0]
    _check(_lib.frx_fwd_partials(A.data_ptr(), A.stride(0), W.data_ptr(), W.stride(0), FRX_DTYPE[A.dtype],
                                 _ptr(bias), _ptr(target), M, V, K, vocab_offset, partials.data_ptr(), M,
                                 _ptr(logits), 0 if logits is None else logits.stride(0), None, _stream(A)))


def fwd_partials_tilerel(A, W, target, partials, logits_rel, *, bias=None, vocab_offset=0):
    """The training forward's 2-byte logits: fp16 z - m_tile into `logits_rel` [M, >= round_up(V, 8)]."""
    M, K = A.shape
    V = W.shape[0]
    _check(_lib.frx_fwd_partials_tilerel(A.data_ptr(), A.stride(0), W.data_ptr(), W.stride(0), FRX_DTYPE[A.dtype],
                                         _ptr(bias), _ptr(target), M, V, K, vocab_offset, partials.data_ptr(), M,
                                         logits_rel.data_ptr(), logits_rel.stride(0), None, _stream(A)))


def finalize(partials, n_tiles, M, *, loss, entropy, lse=None, reference_layout=True):
    """Replaces the `finalize_ce_entropy[_with_lse]` custom ops (gemm_ce_entropy_finalize.py:123-212);
    flag 1 reads the reference's (max, sum exp, sum x exp, target) layout."""
    _check(_lib.frx_finalize(partials.data_ptr(), n_tiles, M, M, 1 if reference_layout else 0, None, 0, 0,
                             loss.data_ptr(), entropy.data_ptr(), _ptr(lse), None, None, None, _stream(partials)))


def compute_dlogits(logits, target, lse, entropy, g_ce, g_ent, out):
    """Replaces the `compute_dlogits` custom op (cute_dlogits.py:121-183): fp32 out, no ignore rule."""
    M, V = logits.shape
    _check(_lib.frx_dlogits(logits.data_ptr(), logits.stride(0), target.to(torch.int64).data_ptr(), lse.data_ptr(),
                            entropy.data_ptr(), g_ce.data_ptr(), g_ent.data_ptr(), 0.0, 0.0, out.data_ptr(),
                            out.stride(0), FRX_DTYPE[out.dtype], M, V, 0, NO_IGNORE, _stream(logits)))


def dlogits_tilerel(logits_rel, partials, target, lse, entropy, out, *, ce_weight=1.0, ent_weight=-1.0,
                    ignore_index=-100):
    """dlogits from the 2-byte logits of fwd_partials_tilerel and the same launch's partials."""
    M = lse.shape[0]
    V = out.shape[1]
    _check(_lib.frx_dlogits_tilerel(logits_rel.data_ptr(), logits_rel.stride(0), partials.data_ptr(), M,
                                    target.data_ptr(), lse.data_ptr(), entropy.data_ptr(), None, None, ce_weight,
                                    ent_weight, out.data_ptr(), out.stride(0), FRX_DTYPE[out.dtype], M, V, 0,
                                    ignore_index, _stream(out)))


def gemm_dhidden(dz, W, dh):
    """Replaces `torch.mm(dlogits_mm, weight)` (gemm_kernel.py:859-862); dz in the weight's 16-bit type."""
    B, V = dz.shape
    H = W.shape[1]
    _check(_lib.frx_gemm_dhidden(dz.data_ptr(), dz.stride(0), W.data_ptr(), W.stride(0), FRX_DTYPE[W.dtype],
                                 dh.data_ptr(), dh.stride(0), FRX_DTYPE[dh.dtype], B, H, V, None, _stream(dz)))


def gemm_dweight(dz, X, dw):
    """Replaces the per-chunk `d_weight.add_(torch.mm(dlogits_mm.t(), h_chunk).float())` and the final
    cast (gemm_kernel.py:864-871): one call over all rows."""
    B, V = dz.shape
    H = X.shape[1]
    _check(_lib.frx_gemm_dweight(dz.data_ptr(), dz.stride(0), X.data_ptr(), X.stride(0), FRX_DTYPE[X.dtype],
                                 dw.data_ptr(), dw.stride(0), FRX_DTYPE[dw.dtype], V, H, B, None, _stream(dz)))


def column_sums(dz, db32):
    """Replaces `d_bias.add_(dlogits.sum(dim=0))` (gemm_kernel.py:867-869), fp32 out."""
    B, V = dz.shape
    _check(_lib.frx_column_sums(dz.data_ptr(), FRX_DTYPE[dz.dtype], dz.stride(0), B, V, db32.data_ptr(),
                                _stream(dz)))


def logits_partials(L, target, partials, tile_cols):
    """Replaces the CrossEntropyOnly / EntropyOnly / CrossEntropyEntropy launches
    (cute_cross_entropy.py:171-578); then finalize with flag 2 (negative targets ignored)."""
    M, N = L.shape
    _check(_lib.frx_logits_partials(L.data_ptr(), FRX_DTYPE[L.dtype], L.stride(0), M, N, _ptr(target), tile_cols,
                                    partials.data_ptr(), M, _stream(L)))


def split_f32(X, out, parts, n_parts, part_stride):
    """bf16 hi / mid / lo parts of an fp32 matrix for the bf16x6 product that replaces the fp32
    `torch.mm` calls of the reference's fp32 inputs (kernel.py:32-45, gemm_kernel.py:859-866)."""
    M, K = X.shape
    _check(_lib.frx_split_f32(X.data_ptr(), X.stride(0), M, K, parts, n_parts, out.data_ptr(), out.stride(0),
                              part_stride, _stream(X)))


def loss_sum(ce, entropy, loss, ce_weight, ent_weight):
    """Replaces `ce_weight * ce.sum() + ent_weight * ent.sum()` (gemm_kernel.py:897)."""
    _check(_lib.frx_loss_sum(ce.data_ptr(), entropy.data_ptr(), ce.numel(), ce_weight, ent_weight, loss.data_ptr(),
                             _stream(ce)))


def scale_inplace(g, dloss):
    """Replaces `d_hidden * dloss` (gemm_kernel.py:905-913), in place, with no host synchronisation."""
    _check(_lib.frx_scale_inplace(g.data_ptr(), FRX_DTYPE[g.dtype], g.numel(), dloss.data_ptr(), _stream(g)))


def fwd_ce_entropy_noalloc(A, W, target, ce, entropy, lse, log_probs, ignore_index=-100):
    """The forward in one call that allocates nothing (bf16 operands; at most
    floor(2097152 / ceil(V / 256)) rows per call)."""
    M, K = A.shape
    V = W.shape[0]
    _check(_lib.frx_fwd_ce_entropy_noalloc(A.data_ptr(), A.stride(0), W.data_ptr(), W.stride(0), target.data_ptr(),
                                           M, V, K, ignore_index, ce.data_ptr(), entropy.data_ptr(), _ptr(lse),
                                           _ptr(log_probs), None, _stream(A)))
