"""The FP8 GEMM's scaled epilogue and the SwiGLU epilogue, as the reference's eager mirrors compute them.

Reference: ``h3_tp2/fp8_gemm.py:174-185`` (``epilogue_torch``: t = sb * acc, y = sa * t in fp32, or
fma(sa, t, bias) emulated in float64, one rounding to the output dtype), ``h3_tp2/fp8_gemm.py:149-164``
(``scaled_mm_tensor32``: acc = A @ W^T in fp32), ``h3_tp2/fp8_swiglu.py:203-212`` (``swiglu_epilogue_torch``: bf16
gate/up, -0 up -> +0, silu in fp32 rounded to bf16, product rounded to bf16) and the weight quant of the GPU tests
(``tests/test_fp8_cutlass_gpu.py:30-34``: per-output-channel absmax scale).
"""
from __future__ import annotations

import torch

from .quant import E4M3, FP8_MAX, MIN_SCALE


def epilogue(acc: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, bias: torch.Tensor | None,
             out_dtype: torch.dtype) -> torch.Tensor:
    t = sb.reshape(1, -1).float() * acc.float()
    sa2 = sa.reshape(-1, 1).float()
    if bias is None:
        y = sa2 * t
    else:
        y = (sa2.double() * t.double() + bias.reshape(1, -1).double()).float()
    return y.to(out_dtype)


def accumulate(a8: torch.Tensor, w8: torch.Tensor) -> torch.Tensor:
    """fp32 A @ W^T of e4m3 operands (exact whenever the fp32 partial sums are, e.g. for integer-valued inputs)."""
    return a8.float() @ w8.float().t()


def scaled_mm(a8, w8, sa, sb, bias=None, out_dtype=torch.bfloat16):
    return epilogue(accumulate(a8, w8), sa, sb, bias, out_dtype)


def quant_weight(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-output-channel e4m3 weight quant: sb[n] = max(absmax_n / 448, 1/(448*512)), w8 = e4m3(clamp(w / sb))."""
    wf = w.float()
    sb = torch.clamp(wf.abs().amax(dim=1) / FP8_MAX, min=MIN_SCALE)
    w8 = torch.clamp(wf / sb[:, None], -FP8_MAX, FP8_MAX).to(E4M3)
    return w8, sb


def silu_mul_bf16(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """vLLM act_and_mul arithmetic on bf16-valued fp32 gate/up: up -0 -> +0, silu(g) = g / (1 + exp(-g)) rounded to
    bf16, the product rounded to bf16 (h3_tp2/fp8_swiglu.py:62-67, :203-212)."""
    u = torch.where(u == 0, u.abs(), u)
    s = (g / (1.0 + torch.exp(-g))).to(torch.bfloat16).float()
    return (s * u).to(torch.bfloat16)


def swiglu_epilogue(acc: torch.Tensor, sa, sb, bias) -> torch.Tensor:
    h = epilogue(acc, sa, sb, bias, torch.bfloat16).float()
    half = h.shape[1] // 2
    return silu_mul_bf16(h[:, :half], h[:, half:])


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    """silu_and_mul on bf16 [M, 2d] (h3_tp2/fp8_quant_fuse.py:263-278 arithmetic)."""
    d = x.shape[-1] // 2
    return silu_mul_bf16(x[..., :d].float(), x[..., d:].float())


def indexed_gate(x: torch.Tensor, gate: torch.Tensor, other: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
    """x + gate[indices] * other in fp32 (product and sum rounded separately), to x's dtype: the eager mirror
    ``_gate_torch`` of ``_scale_indexed_gate_kernel`` (h3_tp2/fp8_consumers.py:367-371); ``other`` is the bf16 fc2
    output (the GEMM epilogue rounded to bf16)."""
    return (x.float() + gate.index_select(0, indices).float() * other.float()).to(x.dtype)
