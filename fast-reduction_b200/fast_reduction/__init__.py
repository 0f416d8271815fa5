"""fast_reduction (B200 engine): fused linear + cross-entropy + entropy on sm_100a.

Drop-in for the hot path of justinchiu/fast-reduction: the GEMM-epilogue forward and the
training megakernel of `fast_reduction.gemm_kernel`, exported lazily as in the reference
(fast_reduction/__init__.py:37-53). All device work runs in libfrx.so (hand-written CUDA for
sm_100a behind a C ABI, include/frx.h); there is no CPU or library fallback.
"""

__all__ = [
    "gemm_fused_ce_entropy",
    "gemm_fused_ce_entropy_v2",
    "gemm_fused_ce_entropy_differentiable",
    "gemm_fused_ce_entropy_fast",
    "gemm_megakernel_fast",
    "vocab_parallel_ce_entropy",
    "vocab_parallel_megakernel",
]

_GEMM_KERNEL_NAMES = {
    "gemm_fused_ce_entropy",
    "gemm_fused_ce_entropy_v2",
    "gemm_fused_ce_entropy_differentiable",
    "gemm_fused_ce_entropy_fast",
    "gemm_megakernel_fast",
}
_VOCAB_PARALLEL_NAMES = {"vocab_parallel_ce_entropy", "vocab_parallel_megakernel"}


def __getattr__(name):
    if name in _GEMM_KERNEL_NAMES:
        from fast_reduction import gemm_kernel

        return getattr(gemm_kernel, name)
    if name in _VOCAB_PARALLEL_NAMES:
        from fast_reduction import vocab_parallel

        return getattr(vocab_parallel, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
