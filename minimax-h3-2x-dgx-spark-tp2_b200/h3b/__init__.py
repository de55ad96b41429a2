"""h3b -- B200-native (sm_100a) DiT attention-block hot path: Ulysses sequence-parallel attention wrapped in
online-FP8 projections, with the h3_tp2 plugin's Python surface.

Modules mirror the reference plugin's hot-path modules (knapcio/MiniMax-H3-2x-DGX-Spark-TP2, package ``h3_tp2``):
``ulysses_exact``, ``ulysses_outq``, ``ulysses_overlap``, ``ulysses_nocopy``, ``fp8_gemm``, ``fp8_cutlass``,
``fp8_quant_fuse``, ``fp8_swiglu``, ``fp8_consumers``, ``a2a_timing`` and ``plugin``, with ``sources`` the
reviewed-upstream-source gate of their model wiring; ``ops`` holds the tensor-level kernel entry points and ``block``
the DiT attention block built from them.  All compute runs in the CUDA library ``libh3b.so`` (C ABI
``include/h3b.h``); nothing falls back to the CPU.
"""
from . import _lib, ops  # noqa: F401

__all__ = ["ops", "load_library"]


def load_library():
    """Load ``libh3b.so`` (raises if it was not built)."""
    return _lib.load()
