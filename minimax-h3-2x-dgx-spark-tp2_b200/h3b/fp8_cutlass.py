"""Mirror of ``h3_tp2/fp8_cutlass.py``: the fused FP8 GEMM for the DiT block's qkv / out / fc1 sites.

The reference compiles a CuTe-DSL sm_120 kernel (``DslGemm``) and routes the running block's GEMMs to it, returning
None whenever the kernel cannot take a call (fp16 output, bias, misalignment, M = 0) so the dispatcher falls through.
Here the same entry points run the library's tcgen05 kernel, which also takes a (bf16) bias and fp16 output; None is
returned only where the kernel's own guards refuse (M = 0, K or N not a multiple of 16, unaligned operands, a bias
that is not bf16).
"""
from __future__ import annotations

import functools
import logging
import os
import threading

import torch

from . import fp8_gemm, ops

logger = logging.getLogger("h3b.fp8_cutlass")

SITES = ("qkv", "out", "fc1")
_tls = threading.local()
_state = {"ok": True, "verify": os.environ.get("H3_TP2_FP8_CUTLASS_VERIFY", "0").strip() == "1"}
_stats = {"dsl": 0, "fallthrough": 0}
_warned: set = set()


class DslGemm:
    """The kernel object of the reference (compiled once, run per call); here a thin handle on the tcgen05 GEMM."""

    def run(self, a: torch.Tensor, w: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        torch.ops.h3b.fp8_gemm_out(a, w, sa, sb, None, y)
        return y


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
    """fp8_gemm router (h3_tp2/fp8_cutlass.py:134; runs before the stash hooks): the kernel for the running block's
    registered sites (``block_want``), else None.  A launch that raises turns the router off for the process."""
    want = getattr(_tls, "want", None)
    if not want:
        return None
    site = want.get((b.data_ptr(), tuple(b.shape)))
    if site is None:
        return None
    try:
        y = scaled_mm(a, b, scale_a, scale_b, out_dtype, bias)
    except Exception as exc:  # noqa: BLE001  (never take the rank down: later calls fall through)
        logger.warning("h3b fp8 cutlass: launch failed (%s: %s); falling through for the rest of this process",
                       type(exc).__name__, exc)
        _state["ok"] = False
        y = None
    if y is None:
        _stats["fallthrough"] += 1
        if "ft-" + site not in _warned:
            _warned.add("ft-" + site)
            logger.warning("h3b fp8 cutlass: %s GEMM M=%d N=%d not taken (guards); the dispatcher's path", site,
                           a.shape[0], b.shape[1])
        return None
    _stats["dsl"] += 1
    if _state["verify"]:
        _verify(site, a, b, scale_a, scale_b, out_dtype, bias, y)
    return y


def _two_pass(a, b, scale_a, scale_b, out_dtype, bias):  # noqa: ANN001,ANN202
    """The reference's two-pass arithmetic: the fp32 product (cuBLASLt on the GPU, a matmul on the CPU), then the
    scale pass."""
    M, N = a.shape[0], b.shape[1]
    sa, sb = ops.vec_scales(scale_a, scale_b, M, N)
    if a.is_cuda:
        one = fp8_gemm.unit_scale(a.device)
        x32 = torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.float32)
        return ops.scale_bias_cast(x32, sa, sb, bias, out_dtype)
    return fp8_gemm.epilogue_torch(a.float() @ b.float(), sa, sb, bias, out_dtype)


def _verify(site, a, b, scale_a, scale_b, out_dtype, bias, y) -> None:  # noqa: ANN001
    """``H3_TP2_FP8_CUTLASS_VERIFY=1`` (diagnosis only, slow): each routed output against the two-pass arithmetic on the
    same operands; mismatches are counted and logged (the routed output is still returned) (h3_tp2/fp8_cutlass.py:166)."""
    ref = _two_pass(a, b, scale_a, scale_b, out_dtype, bias)
    diff = y.view(torch.int16) != ref.view(torch.int16)
    nd = int(diff.sum())
    _stats["verify_calls"] = _stats.get("verify_calls", 0) + 1
    if nd:
        _stats["verify_mismatch"] = _stats.get("verify_mismatch", 0) + 1
        if _stats["verify_mismatch"] <= 20:
            rows = diff.any(1).nonzero().flatten()
            logger.warning("h3b fp8 cutlass VERIFY: %s M=%d N=%d K=%d call %d: %d elements differ from two-pass "
                           "(rows %d..%d)", site, a.shape[0], b.shape[1], a.shape[1], _stats["dsl"], nd,
                           int(rows.min()), int(rows.max()))


def block_want(block, sites=SITES) -> dict:  # noqa: ANN001
    """{(weight data_ptr, weight shape): site} for the DiT block's FP8 qkv / out / fc1 weights (h3_tp2/fp8_cutlass.py:252):
    ``block.attn.qkv_proj``, ``block.attn.out_proj``, ``block.mlp.fc1``, whose e4m3 weight is stored [K, N] (the
    dispatcher's ``b``)."""
    attn, mlp = getattr(block, "attn", None), getattr(block, "mlp", None)
    layers = {"qkv": getattr(attn, "qkv_proj", None), "out": getattr(attn, "out_proj", None),
              "fc1": getattr(mlp, "fc1", None)}
    want = {}
    for site in sites:
        w = getattr(layers.get(site), "weight", None)
        if isinstance(w, torch.Tensor) and w.dtype == torch.float8_e4m3fn and w.dim() == 2:
            want[(w.data_ptr(), tuple(w.shape))] = site
    return want


def make_block_forward(orig_forward, sites=SITES):  # noqa: ANN001,ANN201
    """The DiT block's forward with the router told the block's weights for its duration (h3_tp2/fp8_cutlass.py:266)."""
    @functools.wraps(orig_forward)
    def forward(self, *args, **kwargs):  # noqa: ANN001,ANN202
        compiling = getattr(getattr(torch, "compiler", None), "is_compiling", None)
        if compiling is not None and compiling():
            return orig_forward(self, *args, **kwargs)
        prev = getattr(_tls, "want", None)
        _tls.want = block_want(self, sites)
        try:
            return orig_forward(self, *args, **kwargs)
        finally:
            _tls.want = prev

    forward._h3b_cutlass = True
    return forward


def install_sites(tr=None, sites=SITES) -> bool:  # noqa: ANN001
    """Wrap ``MiniMaxH3DiTBlock.forward`` of the transformer module ``tr`` (default: vLLM-Omni's MiniMax H3) and register
    the router with the FP8 dispatcher (h3_tp2/fp8_cutlass.py:285)."""
    if tr is None:
        from vllm_omni.diffusion.models.minimax_h3 import minimax_h3_transformer as tr  # noqa: PLC0415
    cls = tr.MiniMaxH3DiTBlock
    if not getattr(cls.forward, "_h3b_cutlass", False):
        cls.forward = make_block_forward(cls.forward, sites)
    fp8_gemm.set_router(route)
    return True


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
