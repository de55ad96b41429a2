"""Fused FP8 fc1 epilogue + SwiGLU (mirrors ``h3_tp2/fp8_swiglu.py``).

``gemm_swiglu`` is the fc1 GEMM whose CTA tile holds gate columns n and up columns F + n in two halves of one TMEM
accumulator; the epilogue applies the scaled epilogue to both, rounds each to bf16, sets up = -0 to +0, computes
silu(g) = g / (1 + exp(-g)) in fp32 (CUDA's ``expf``, IEEE division) rounded to bf16, and writes bf16(silu * up).
``scale_swiglu`` / ``scale_swiglu_quant`` are the same arithmetic over an fp32 product (the two-pass form).
"""
from __future__ import annotations

import torch

from . import fp8_gemm, ops


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


def swiglu_epilogue_torch(acc: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    """The SwiGLU epilogue in eager torch on an fp32 fc1 product [M, 2*half] (h3_tp2/fp8_swiglu.py:203): the scaled
    epilogue rounded to bf16 for the gate and up halves, up -0 -> +0, silu(g) = g / (1 + exp(-g)) in fp32 rounded to
    bf16, the product rounded to bf16.  torch's exp here, CUDA's expf in the kernel (within 1 bf16 ulp)."""
    h = fp8_gemm.epilogue_torch(acc, sa, sb, bias, torch.bfloat16).float()
    gate, up = h.chunk(2, dim=1)
    up = torch.where(up == 0, torch.zeros_like(up), up)
    silu = (gate / (1.0 + torch.exp(-gate))).to(torch.bfloat16).float()
    return (silu * up).to(torch.bfloat16)


def swiglu_config() -> tuple[int, int, int, int, int]:
    """(BLOCK_M, BLOCK_N, BLOCK_K, warps, stages) of the fc1 + SwiGLU kernel (h3_tp2/fp8_swiglu.py:247 returns the
    Triton kernel's): the FP8 GEMM's CTA-pair tile, whose 256 accumulator columns hold 128 gate and 128 up columns."""
    return fp8_gemm.fused_config()


def probe_gemm_swiglu(device) -> bool:  # noqa: ANN001
    """True when the fused fc1 + SwiGLU kernel serves on ``device`` and equals the eager epilogue on integer inputs
    (exact accumulators in any summation order) within 1 bf16 ulp (torch's exp against CUDA's expf)
    (h3_tp2/fp8_swiglu.py:258)."""
    dev = torch.device(device)
    if dev.type != "cuda" or torch.cuda.get_device_capability(dev) != (10, 0):
        return False
    g = torch.Generator(device=dev).manual_seed(0)
    a = torch.randint(-3, 4, (130, 64), device=dev, generator=g).to(torch.float8_e4m3fn)
    w = torch.randint(-3, 4, (512, 64), device=dev, generator=g).to(torch.float8_e4m3fn)
    sa = torch.full((130,), 0.5, device=dev)
    sb = torch.full((512,), 0.03125, device=dev)
    y = ops.fp8_gemm_swiglu(a, w, sa, sb)
    ref = swiglu_epilogue_torch(a.float().cpu() @ w.float().cpu().t(), sa.cpu(), sb.cpu(), None)
    diff = (y.cpu().view(torch.int16).int() - ref.view(torch.int16).int()).abs()
    return bool(diff.max().item() <= 1)
