"""Mirror of ``h3_tp2/fp8_cutlass.py``: the fused FP8 GEMM for the DiT block's qkv / out / fc1 sites.

The reference compiles a CuTe-DSL sm_120 kernel (``DslGemm``) and routes the running block's GEMMs to it, returning
None whenever the kernel cannot take a call (fp16 output, bias, misalignment, M = 0) so the dispatcher falls through.
Here the same entry points run the library's tcgen05 kernel, which also takes a (bf16) bias and fp16 output; None is
returned only where the kernel's own guards refuse (M = 0, K or N not a multiple of 16, unaligned operands, a bias
that is not bf16).
"""
from __future__ import annotations

import logging
import threading

import torch

from . import fp8_gemm, ops

logger = logging.getLogger("h3b.fp8_cutlass")

SITES = ("qkv", "out", "fc1")
_tls = threading.local()
_state = {"ok": True}
_stats = {"taken": 0, "fallthrough": 0}


class DslGemm:
    """The kernel object of the reference (compiled once, run per call); here a thin handle on the tcgen05 GEMM."""

    def run(self, a: torch.Tensor, w: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        return ops.fp8_gemm(a, w, sa, sb, None, y.dtype, out=y)


_gemm = DslGemm()


def _aligned(*ts: torch.Tensor) -> bool:
    return all(t.data_ptr() % 16 == 0 for t in ts)


def scaled_mm(a: torch.Tensor, b: torch.Tensor, scale_a: torch.Tensor, scale_b: torch.Tensor, out_dtype: torch.dtype,
              bias: torch.Tensor | None = None) -> torch.Tensor | None:
    """[M, N] for a dispatcher-eligible call (``b`` [K, N] with ``b.t()`` contiguous), or None when not taken."""
    if a.shape[0] == 0 or not a.is_cuda or not _state["ok"]:
        return None
    if not fp8_gemm.eligible(a, b, scale_a, scale_b, out_dtype, bias) or not _aligned(a, b):
        return None
    return fp8_gemm.scaled_mm(a, b, scale_a, scale_b, out_dtype, bias)


def route(a, b, scale_a, scale_b, out_dtype, bias):  # noqa: ANN001,ANN201
    """fp8_gemm router: the kernel for the running block's registered sites (``block_want``), else None."""
    want = getattr(_tls, "want", None)
    if not want or want.get((b.data_ptr(), tuple(b.shape))) is None:
        return None
    try:
        y = scaled_mm(a, b, scale_a, scale_b, out_dtype, bias)
    except Exception as exc:  # noqa: BLE001  (never take the rank down: later calls fall through)
        logger.warning("h3b fp8 cutlass: launch failed (%s); falling through for the rest of this process", exc)
        _state["ok"] = False
        y = None
    _stats["taken" if y is not None else "fallthrough"] += 1
    return y


def block_want(block, sites=SITES) -> dict:  # noqa: ANN001
    """{(weight data_ptr, weight.t() shape): site} for the block's quantised linears (h3_tp2/fp8_cutlass.py:252);
    ``block`` exposes ``to_qkv`` / ``to_out`` / ``fc1`` style linears with a ``weight`` of shape [N, K]."""
    names = {"qkv": ("to_qkv", "qkv"), "out": ("to_out", "out_proj", "o_proj"), "fc1": ("fc1", "w13", "gate_up_proj")}
    want = {}
    for site in sites:
        for n in names[site]:
            lin = getattr(block, n, None)
            w = getattr(lin, "weight", None)
            if w is not None:
                want[(w.data_ptr(), tuple(w.t().shape))] = site
                break
    return want


def selfcheck(gemm: DslGemm | None = None, device="cuda") -> list[str]:  # noqa: ANN001
    """Failed checks (empty = pass): integer-input GEMMs on partial tiles, exact in any summation order."""
    dev = torch.device(device)
    fails = []
    for M, N, K in ((1, 128, 64), (200, 400, 512), (333, 272, 1024)):
        g = torch.Generator(device=dev).manual_seed(M + N + K)
        a = torch.randint(-4, 5, (M, K), device=dev, generator=g).to(torch.float8_e4m3fn)
        w = torch.randint(-2, 3, (N, K), device=dev, generator=g).to(torch.float8_e4m3fn)
        sa = torch.full((M,), 2.0 ** -6, device=dev)
        sb = torch.full((N,), 2.0 ** -4, device=dev)
        y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        (gemm or _gemm).run(a, w, sa, sb, y)
        ref = ((a.float() @ w.float().t()) * 2.0 ** -4 * 2.0 ** -6).to(torch.bfloat16)
        if not torch.equal(y.view(torch.int16), ref.view(torch.int16)):
            fails.append(f"M={M} N={N} K={K}")
    return fails


def probe(device="cuda") -> bool:  # noqa: ANN001
    """True when the kernel serves on ``device`` and passes ``selfcheck``."""
    if not fp8_gemm.probe_fused(device):
        return False
    fails = selfcheck(_gemm, device)
    if fails:
        logger.warning("h3b fp8 cutlass: selfcheck failed (%s)", ", ".join(fails))
    return not fails


def stats() -> dict[str, int]:
    return dict(_stats)
