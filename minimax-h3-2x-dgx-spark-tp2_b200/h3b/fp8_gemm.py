"""Drop-in for ``ops.cutlass_scaled_mm`` on per-token x per-channel scaled FP8 linears.

Mirrors ``h3_tp2/fp8_gemm.py``: ``scaled_mm_tensor32(a, b, scale_a, scale_b, out_dtype, bias)`` (a [M, K] e4m3
row-major, b [K, N] e4m3 with ``b.t()`` contiguous, scale_a [M, 1] or scalar fp32, scale_b [N] or scalar fp32) ->
[M, N] in bf16/fp16, with the epilogue ``y = out(sa[m] * (sb[n] * acc))`` (bias by fma).  On B200 every level runs
the one tcgen05 kernel with the epilogue fused (no fp32 product, no second pass); routers and stash hooks keep the
reference's dispatch order (``route``).
"""
from __future__ import annotations

import logging

import torch

from . import ops

logger = logging.getLogger("h3b.fp8_gemm")

_state = {"level": "tcgen05", "installed": False}
_stash_hooks: list = []
_routers: list = []


def eligible(a: torch.Tensor, b: torch.Tensor, scale_a: torch.Tensor, scale_b: torch.Tensor, out_dtype,  # noqa: ANN001
             bias: torch.Tensor | None) -> bool:
    """The dispatcher's guards (h3_tp2/fp8_gemm.py:364-372), plus: a bias must be bf16 (the kernels read it as bf16;
    any other bias falls through to the stock dispatch)."""
    M, N = a.shape[0], b.shape[-1]
    return not (a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[0]
                or (scale_a.numel() == 1 and scale_b.numel() == 1)
                or scale_a.numel() not in (1, M) or scale_b.numel() not in (1, N)
                or scale_a.dtype != torch.float32 or scale_b.dtype != torch.float32
                or a.dtype != torch.float8_e4m3fn or b.dtype != torch.float8_e4m3fn
                or a.device != b.device or out_dtype not in (torch.bfloat16, torch.float16)
                or (bias is not None and (bias.dim() != 1 or bias.numel() != N or bias.dtype != torch.bfloat16))
                or not a.is_contiguous() or not b.t().is_contiguous() or a.shape[1] % 16 or N % 16)


def scaled_mm(a: torch.Tensor, b: torch.Tensor, scale_a: torch.Tensor, scale_b: torch.Tensor, out_dtype: torch.dtype,
              bias: torch.Tensor | None = None) -> torch.Tensor:
    """One tcgen05 FP8 GEMM with the scaled epilogue (the reference's ``scaled_mm_tensor32`` / ``scaled_mm_fused`` /
    ``fp8_cutlass.scaled_mm`` arithmetic)."""
    return torch.ops.h3b.fp8_gemm(a, b.t(), scale_a, scale_b, bias, out_dtype)


scaled_mm_tensor32 = scaled_mm     # h3_tp2/fp8_gemm.py:149
scaled_mm_fused = scaled_mm        # h3_tp2/fp8_gemm.py:240


def launch_fused(a: torch.Tensor, b: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, bias: torch.Tensor | None,
                 y: torch.Tensor, cfg=None) -> torch.Tensor:  # noqa: ANN001
    """One fused launch into ``y`` (h3_tp2/fp8_gemm.py:213): sa [M], sb [N] fp32 vectors, b [K, N], y bf16 or f16.
    ``cfg`` (the Triton kernel's tile choice) is accepted and has no effect: the tcgen05 kernel has one tile shape.
    The Triton kernel's raw-accumulator form (fp32 ``y``) is not provided: the epilogue always writes the scaled
    output."""
    del cfg
    if y.dtype == torch.float32:
        raise NotImplementedError("launch_fused: fp32 y (the raw accumulator) is not provided by the fused tcgen05 "
                                  "kernel; it writes the scaled bf16 / f16 output")
    torch.ops.h3b.fp8_gemm_out(a, b.t(), sa, sb, bias, y)
    return y


def fused_config() -> tuple[int, int, int, int, int]:
    """(BLOCK_M, BLOCK_N, BLOCK_K, warps, stages) of the tcgen05 kernel, in the order of h3_tp2/fp8_gemm.py:202 (which
    returns the Triton kernel's): a 256 x 256 tile per CTA pair (128 rows per CTA), 6 warps and 6 stages per CTA."""
    return 256, 256, 128, 6, 6


def tile_coords(pid: int, M: int, N: int, block_m: int = 256, block_n: int = 256, group_m: int = 16) -> tuple[int, int]:
    """Grouped raster of the persistent kernel: pair tile ``pid`` -> (row block, column block); GROUP_M row blocks
    share each column block's W tile in L2 (h3_tp2/fp8_gemm.py:188 is the same raster; the defaults are this
    kernel's: 256 x 256 pair tiles in groups of 16 row blocks)."""
    num_mb, num_nb = -(-M // block_m), -(-N // block_n)
    in_group = group_m * num_nb
    group = pid // in_group
    first = group * group_m
    gsize = min(num_mb - first, group_m)
    r = pid - group * in_group
    return first + r % gsize, r // gsize


def unit_scale(device) -> torch.Tensor:  # noqa: ANN001
    """A cached fp32 scalar 1 (h3_tp2/fp8_gemm.py:132)."""
    key = str(device)
    t = _unit.get(key)
    if t is None:
        t = _unit[key] = torch.ones((), dtype=torch.float32, device=device)
    return t


_unit: dict = {}


def probe_fused(device) -> bool:  # noqa: ANN001
    """True when the tcgen05 kernel can serve on ``device``: an sm_100 GPU and the library loads; a small GEMM
    against integer inputs (exact in any summation order) confirms it (h3_tp2/fp8_gemm.py:251)."""
    dev = torch.device(device)
    if dev.type != "cuda" or not torch.cuda.is_available() or torch.cuda.get_device_capability(dev) != (10, 0):
        return False
    g = torch.Generator(device=dev).manual_seed(0)
    a = torch.randint(-3, 4, (130, 64), device=dev, generator=g).to(torch.float8_e4m3fn)
    w = torch.randint(-3, 4, (272, 64), device=dev, generator=g).to(torch.float8_e4m3fn)
    sa = torch.full((130,), 0.5, device=dev)
    sb = torch.full((272,), 0.25, device=dev)
    y = torch.ops.h3b.fp8_gemm(a, w, sa, sb, None, torch.bfloat16)
    ref = ((a.float() @ w.float().t()) * 0.25 * 0.5).to(torch.bfloat16)
    return bool(torch.equal(y.view(torch.int16), ref.view(torch.int16)))


def _rows(v: torch.Tensor) -> torch.Tensor:
    return v.reshape(-1, 1).float()


def _cols(v: torch.Tensor) -> torch.Tensor:
    return v.reshape(1, -1).float()


def epilogue_torch(acc: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, bias: torch.Tensor | None,
                   out_dtype: torch.dtype) -> torch.Tensor:
    """The kernel's epilogue in eager torch on an fp32 product (h3_tp2/fp8_gemm.py:174): the column scale first, then
    the row scale, in fp32; with a bias, row scale x that product + bias as one fma, carried out in float64 (where the
    fp32 product is exact) and rounded to fp32; then one rounding to ``out_dtype``.  A CPU function by design (the
    reference's eager mirror), not a fallback of the GPU path."""
    t = _cols(sb) * acc.float()
    if bias is None:
        y = _rows(sa) * t
    else:
        y = (_rows(sa).double() * t.double() + _cols(bias).double()).float()
    return y.to(out_dtype)


def scale_bias_cast_torch(x32: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, bias: torch.Tensor | None,
                          out_dtype: torch.dtype) -> torch.Tensor:
    """The two-pass scale pass in eager torch (h3_tp2/fp8_gemm.py:120): column scale, row scale, then the bias as a
    separate fp32 add (not an fma), one rounding to ``out_dtype``."""
    y = (_cols(sb) * x32.float()) * _rows(sa)
    if bias is not None:
        y = y + _cols(bias)
    return y.to(out_dtype)


def epilogue_reference_order() -> str:
    return "t = scale_b * acc; y = scale_a * t (bias: fma(scale_a, t, bias)); one rounding"


def set_stash_hook(fn) -> None:  # noqa: ANN001
    if fn not in _stash_hooks:
        _stash_hooks.append(fn)


def set_router(fn) -> None:  # noqa: ANN001
    if fn not in _routers:
        _routers.append(fn)


def route(a, b, scale_a, scale_b, out_dtype, bias=None, two_pass=None):  # noqa: ANN001,ANN201
    """Routers, then stash hooks, then the GEMM (h3_tp2/fp8_gemm.py:328)."""
    for router in _routers:
        y = router(a, b, scale_a, scale_b, out_dtype, bias)
        if y is not None:
            return y
    for hook in _stash_hooks:
        ph = hook(a, b, scale_a, scale_b, out_dtype, bias)
        if ph is not None:
            return ph
    return (two_pass or scaled_mm)(a, b, scale_a, scale_b, out_dtype, bias)


def _route_summary() -> str:
    """At the cutlass level, how many of the taken calls the block router served (h3_tp2/fp8_gemm.py:304)."""
    if _state["level"] != "cutlass":
        return ""
    from . import fp8_cutlass  # noqa: PLC0415
    st = fp8_cutlass.stats()
    return f" (block router: taken {st['dsl']}, fell through {st['fallthrough']})"


def _install_into(vops, level: str, probe=None, cutlass_probe=None) -> None:  # noqa: ANN001
    """``install`` on the module ``vops`` that holds ``cutlass_scaled_mm``; ``probe(device)`` / ``cutlass_probe(device)``
    default to ``probe_fused`` and ``fp8_cutlass.probe``."""
    if level not in ("tensor32", "fused", "cutlass"):
        raise ValueError(f"unknown FP8 GEMM level {level!r}")
    orig = vops.cutlass_scaled_mm
    if getattr(orig, "_h3b", False):
        return
    probe = probe or probe_fused
    if not probe("cuda"):
        _state.update(level="stock", installed=False)
        logger.warning("h3b: the tcgen05 FP8 GEMM does not serve on this device (needs sm_100 and the library's "
                       "self-check); vLLM's stock kernel stays")
        return
    stats = {"two_pass": 0, "stock": 0}   # the reference's names: calls this dispatch took / left to the stock kernel
    seen: set = set()

    def _mm(a, b, scale_a, scale_b, out_dtype, bias=None):  # noqa: ANN001
        if not (a.is_cuda and eligible(a, b, scale_a, scale_b, out_dtype, bias)):
            stats["stock"] += 1
            return orig(a, b, scale_a, scale_b, out_dtype, bias)
        stats["two_pass"] += 1
        shape = (a.shape[0], b.shape[1], a.shape[1])
        if len(seen) < 64 and shape not in seen:          # each distinct shape once (h3_tp2/fp8_gemm.py:375-381)
            seen.add(shape)
            logger.info("h3b: FP8 GEMM shape M=%d N=%d K=%d", *shape)
        n = stats["two_pass"] + stats["stock"]
        if n == 2000 or n % 20000 == 0:
            logger.info("h3b: FP8 GEMM dispatch so far: taken %d, stock %d%s", stats["two_pass"], stats["stock"],
                        _route_summary())
        return route(a, b, scale_a, scale_b, out_dtype, bias)

    _mm._h3b = True
    _mm.stats = stats
    vops.cutlass_scaled_mm = _mm
    _state.update(level=level, installed=True)
    if level == "cutlass":
        if cutlass_probe is None:
            from . import fp8_cutlass  # noqa: PLC0415
            cutlass_probe = fp8_cutlass.probe
        if cutlass_probe("cuda"):
            from . import fp8_cutlass  # noqa: PLC0415
            set_router(fp8_cutlass.route)
        else:
            _state["level"] = "tensor32"
            logger.warning("h3b: FP8 GEMM cutlass level unavailable (block routing failed its self-check); tensor32")
    logger.info("h3b: FP8 GEMM (tcgen05, fused scaled epilogue) installed for level %s", _state["level"])


def install(level: str = "tensor32") -> None:
    """Replace vLLM's ``_custom_ops.cutlass_scaled_mm`` for eligible calls (h3_tp2/fp8_gemm.py:344).  ``level`` is
    accepted for compatibility ("tensor32", "fused", "cutlass"): all run the same fused tcgen05 kernel; "cutlass" also
    routes the running DiT block's qkv / out / fc1 weights (``fp8_cutlass``), falling back to "tensor32" when that
    check fails.  When the kernel does not serve on the device the stock kernel stays (``_state["level"]`` "stock");
    ``_state["level"]`` is the level actually running."""
    from vllm import _custom_ops as vops  # noqa: PLC0415
    _install_into(vops, level)
