"""RMSNorm + AdaLN modulation producers of the qkv / fc1 inputs, restated in eager fp32.

Reference: the eager mirrors of the upstream Triton kernels used by the reference's CPU tests,
``tests/fake_h3_consumers.py:66-84`` (``indexed_gate_rms_norm_scale_shift``, ``rms_norm_indexed_scale_shift``), which
``h3_tp2/fp8_quant_fuse.py:330-376`` (``rms_quant`` / ``gate_rms_quant``) follow with the per-token quant.
"""
from __future__ import annotations

import torch

from .quant import quant


def _rows(t: torch.Tensor | None, indices: torch.Tensor | None, n: int) -> torch.Tensor | None:
    if t is None:
        return None
    if indices is None:
        return t[:1].expand(n, -1)
    return t.index_select(0, indices)


def rms_norm_scale_shift(x, weight, shift=None, scale=None, indices=None, eps=1e-6) -> torch.Tensor:
    """bf16 [M, H] -> bf16: x * rsqrt(mean(x^2) + eps) * weight [* (1 + scale) + shift]."""
    n, h = x.shape
    xf = x.float()
    var = (xf * xf).sum(dim=1, keepdim=True) / h
    out = xf * torch.rsqrt(var + eps) * weight.float()
    if shift is not None:
        out = out * (1.0 + _rows(scale, indices, n).float()) + _rows(shift, indices, n).float()
    return out.to(torch.bfloat16)


def gate_rms_norm_scale_shift(residual, gate, branch, weight, shift, scale, indices, eps):
    """(residual_out bf16 = bf16(residual + gate[idx] * branch), modulated RMSNorm of it as bf16)."""
    n, h = residual.shape
    upd = (residual.float() + _rows(gate, indices, n).float() * branch.float()).to(torch.bfloat16).float()
    var = (upd * upd).sum(dim=1, keepdim=True) / h
    out = upd * torch.rsqrt(var + eps) * weight.float()
    if shift is not None:
        out = out * (1.0 + _rows(scale, indices, n).float()) + _rows(shift, indices, n).float()
    return upd.to(torch.bfloat16), out.to(torch.bfloat16)


def rms_quant(x, weight, shift=None, scale=None, indices=None, eps=1e-6):
    return quant(rms_norm_scale_shift(x, weight, shift, scale, indices, eps))
