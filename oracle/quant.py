"""Per-token dynamic FP8-e4m3 quant, as the reference's eager path computes it.

Reference: ``h3_tp2/fp8_quant_fuse.py:302-307`` (``quant_torch``) = ``h3_tp2/ulysses_outq.py:126-135``
(``quant_reference_eager``) = vLLM ``QuantFP8.forward_native`` (dynamic, per token), and the segmented addressing of
``ulysses_outq.quant_rows`` (``h3_tp2/ulysses_outq.py:109-123``).  Per row of bf16 x:
    amax = max |x| (in fp32; NaN propagates), scale = max(amax / 448, 1/(448*512)) (IEEE fp32 division),
    q = e4m3_rn(clamp(x * (1 / scale), -448, 448)).
"""
from __future__ import annotations

import torch

FP8_MAX = 448.0
MIN_SCALE = 1.0 / (FP8_MAX * 512.0)
E4M3 = torch.float8_e4m3fn


def quant(h: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """h [M, K] (bf16) -> (q [M, K] e4m3, scale [M, 1] fp32)."""
    x = h.to(torch.float32)
    amax = x.abs().amax(dim=-1, keepdim=True)
    # amax propagates NaN on CPU torch; keep that explicit for clarity
    amax = torch.where(torch.isnan(x).any(dim=-1, keepdim=True), torch.full_like(amax, float("nan")), amax)
    scale = torch.clamp(amax / torch.tensor(FP8_MAX, dtype=torch.float32), min=MIN_SCALE)
    inv = torch.tensor(1.0, dtype=torch.float32) / scale
    q = torch.clamp(x * inv, -FP8_MAX, FP8_MAX).to(E4M3)
    return q, scale


def rows_view(base: torch.Tensor, m: int, p: int, seg: int, stride_p: int, stride_m: int) -> torch.Tensor:
    """The [m, p*seg] matrix whose row r is concat_s base_flat[s*stride_p + r*stride_m :][:seg]
    (``ulysses_outq.quant_rows`` addressing, h3_tp2/ulysses_outq.py:109-123)."""
    flat = base.reshape(-1)
    return flat.as_strided((m, p, seg), (stride_m, stride_p, 1)).reshape(m, p * seg)


def quant_rows(base: torch.Tensor, m: int, p: int, seg: int, stride_p: int, stride_m: int):
    return quant(rows_view(base, m, p, seg, stride_p, stride_m))


def quant_from_recv(recv: torch.Tensor):
    """recv [P, M, hl, d] -> quant of the unpacked [M, P*hl*d] rows (h3_tp2/ulysses_outq.py:138-143)."""
    p, m, hl, d = recv.shape
    seg = hl * d
    return quant_rows(recv.contiguous(), m, p, seg, m * seg, seg)


def dequant(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return q.to(torch.float32) * scale.reshape(-1, 1)
