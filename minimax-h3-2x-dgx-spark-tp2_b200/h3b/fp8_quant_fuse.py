"""Per-token FP8 quant fused into the producers of each GEMM input (mirrors ``h3_tp2/fp8_quant_fuse.py``).

Sites: qkv (RMSNorm + AdaLN modulation), out (the Ulysses reverse unpack), fc1 (gated residual + RMSNorm +
modulation), fc2 (SiLU-mul).  Each entry point runs one CUDA row kernel that produces the bf16 value the stock
producer would store, keeps it in registers and writes the e4m3 row and its fp32 scale.  ``stock`` arguments of the
reference signatures are accepted and ignored (the GPU path never runs the stock producer).
"""
from __future__ import annotations

import torch

from . import ops

SITES = ("qkv", "out", "fc1", "fc2")
FP8_MAX = 448.0
MIN_SCALE = 1.0 / (FP8_MAX * 512.0)


def quant(h: torch.Tensor, div_mode: int = ops.DIV_IEEE):
    """h3_tp2/fp8_quant_fuse.py:318."""
    return ops.quant(h, div_mode=div_mode)


def rms_quant(x, weight, shift, scale, indices, eps, stock=None, ph=None, div_mode: int = ops.DIV_IEEE):  # noqa: ANN001,ANN201
    """h3_tp2/fp8_quant_fuse.py:330: (fp8 [M, H], scale [M, 1]); ``ph`` also receives the bf16 row."""
    del stock
    return ops.rms_quant(x, weight, shift, scale, indices, eps, ph, div_mode=div_mode)


def gate_rms_quant(residual, gate, branch, weight, shift, scale, indices, eps, stock=None, ph=None,  # noqa: ANN001,ANN201
                   div_mode: int = ops.DIV_IEEE):
    """h3_tp2/fp8_quant_fuse.py:350: (residual_out bf16, fp8, scale)."""
    del stock
    if ph is not None:
        raise NotImplementedError("gate_rms_quant: the bf16 copy (ph) is not produced on this path")
    return ops.gate_rms_quant(residual, gate, branch, weight, shift, scale, indices, eps, div_mode=div_mode)


def unpack_quant(recv: torch.Tensor, div_mode: int = ops.DIV_IEEE):
    """h3_tp2/fp8_quant_fuse.py:379: the reverse unpack + per-token quant of [M, P*hl*d]."""
    return ops.quant_from_recv(recv.contiguous(), div_mode=div_mode)


def silu_mul_quant(x: torch.Tensor, stock=None, div_mode: int = ops.DIV_IEEE):  # noqa: ANN001
    """h3_tp2/fp8_quant_fuse.py:392: silu_and_mul on bf16 [M, 2d] + per-token quant."""
    del stock
    return ops.silu_mul_quant(x, div_mode=div_mode)


def quant_torch(h: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token dynamic e4m3 quant in eager torch (vLLM ``QuantFP8.forward_native``, h3_tp2/fp8_quant_fuse.py:302):
    scale = max(amax / 448, 1/229376) per row (NaN propagates), q = e4m3(clamp(h * (1 / scale), +-448)).  Returns
    (q [M, K] e4m3, scale [M, 1] fp32).  A CPU function by design, not a fallback of ``quant``."""
    amax = h.abs().amax(dim=-1, keepdim=True).float()
    amax = torch.where(torch.isnan(h).any(dim=-1, keepdim=True), torch.full_like(amax, float("nan")), amax)
    scale = torch.clamp(amax / FP8_MAX, min=MIN_SCALE)
    q = torch.clamp(h.float() * torch.reciprocal(scale), -FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q, scale


def unpack_stock(recv: torch.Tensor, heads: int) -> torch.Tensor:
    """Stock's reverse unpack (h3_tp2/fp8_quant_fuse.py:371): receive [P, M, hl, d] -> [1, M, H, d] contiguous."""
    p, m, hl, d = recv.shape
    if p * hl != heads:
        raise ValueError(f"unpack_stock: {p} x {hl} heads received, {heads} expected")
    return recv.permute(1, 0, 2, 3).reshape(1, m, heads, d).contiguous()


_ON = ("1", "all", "on", "true")
_OFF = ("", "0", "off", "false")


def parse_sites(value: str | None) -> tuple[str, ...]:
    """``H3_TP2_FP8_QUANT_FUSE`` (h3_tp2/fp8_quant_fuse.py:836): "1"/"all"/"on"/"true" = every site, a comma list
    selects sites (in SITES order), anything else or empty = none."""
    v = (value or "").strip().lower()
    if v in _ON:
        return SITES
    if v in _OFF:
        return ()
    chosen = {part.strip() for part in v.split(",")}
    return tuple(site for site in SITES if site in chosen)


def is_explicit(value: str | None) -> bool:
    """True when the switch names its sites rather than turning all on or off (h3_tp2/fp8_quant_fuse.py:847)."""
    return (value or "").strip().lower() not in _ON + _OFF
