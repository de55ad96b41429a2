"""Fused FP8 fc1 epilogue + SwiGLU (mirrors ``h3_tp2/fp8_swiglu.py``).

``gemm_swiglu`` is the fc1 GEMM whose CTA tile holds gate columns n and up columns F + n in two halves of one TMEM
accumulator; the epilogue applies the scaled epilogue to both, rounds each to bf16, sets up = -0 to +0, computes
silu(g) = g / (1 + exp(-g)) in fp32 (CUDA's ``expf``, IEEE division) rounded to bf16, and writes bf16(silu * up).
``scale_swiglu`` / ``scale_swiglu_quant`` are the same arithmetic over an fp32 product (the two-pass form).
"""
from __future__ import annotations

import torch

from . import ops


def scale_swiglu(x32: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    """h3_tp2/fp8_swiglu.py:180."""
    return ops.scale_swiglu(x32, sa, sb, bias)


def scale_swiglu_quant(x32: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, bias: torch.Tensor | None):
    """h3_tp2/fp8_swiglu.py:191: (fp8 [M, F], scale [M, 1])."""
    return ops.scale_swiglu_quant(x32, sa, sb, bias)


def gemm_swiglu(a: torch.Tensor, b: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, bias: torch.Tensor | None,
                cfg=None) -> torch.Tensor:  # noqa: ANN001
    """h3_tp2/fp8_swiglu.py:230: fc1 + epilogue + SwiGLU in one kernel; b [K, 2F] with b.t() contiguous."""
    del cfg
    return ops.fp8_gemm_swiglu(a, b.t(), sa, sb, bias)


def ffn(x: torch.Tensor, norm_weight: torch.Tensor, w1: torch.Tensor, s1: torch.Tensor, w2: torch.Tensor,
        s2: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """BASELINE config 4's FFN: RMSNorm + per-token quant -> fc1 (gate/up, SwiGLU epilogue) -> per-token quant ->
    fc2.  x [M, C] bf16, w1 [2F, C] e4m3 with per-channel s1, w2 [C, F] e4m3 with s2 -> [M, C] bf16."""
    q, sq = ops.rms_quant(x, norm_weight, eps=eps)
    h = ops.fp8_gemm_swiglu(q, w1, sq, s1)
    hq, sh = ops.quant(h)
    return ops.fp8_gemm(hq, w2, sh, s2)
