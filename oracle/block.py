"""The DiT attention block of BASELINE's configs on the CPU: per-token quant -> FP8 qkv projection -> Ulysses
seq->head exchange -> non-causal SDPA -> head->seq exchange -> per-token quant -> FP8 out projection.

It composes the oracle pieces (``quant``, ``gemm``, ``ulysses``, ``attention``) in the order of the reference's block
(``h3_tp2/ulysses_exact.py:187-220`` ``exact_forward`` for the exchange and the attention, the FP8 linear path of
``h3_tp2/fp8_gemm.py:149-164`` for the projections).  Config 0 of BASELINE runs it in fp32 without quantisation
(plain fp32 projections), which ``fp32_block`` does with ``exact_forward``'s layout and a real collective.
"""
from __future__ import annotations

import torch

from . import attention, gemm, quant, ulysses


def make_weights(hidden: int, heads: int, seed: int = 1, head_dim: int = 128):
    """Wqkv [3*H*d, C] and Wo [C, H*d] ~ N(0, 0.02), quantised per output channel to e4m3."""
    g = torch.Generator().manual_seed(seed)
    wqkv = torch.randn(3 * heads * head_dim, hidden, generator=g) * 0.02
    wo = torch.randn(hidden, heads * head_dim, generator=g) * 0.02
    wqkv8, sqkv = gemm.quant_weight(wqkv)
    wo8, so = gemm.quant_weight(wo)
    return wqkv8, sqkv, wo8, so


def fp8_block_local(x: torch.Tensor, wqkv8, sqkv, wo8, so, heads: int, head_dim: int = 128):
    """One rank, P = 1: x [N, C] bf16 -> y [N, C] bf16 through the FP8 projections and fp32 SDPA (bf16 q/k/v)."""
    n = x.shape[0]
    q8, sx = quant.quant(x)
    qkv = gemm.scaled_mm(q8, wqkv8, sx, sqkv)                      # [N, 3*H*d] bf16
    q, k, v = (t.reshape(n, heads, head_dim) for t in qkv.split(heads * head_dim, dim=1))
    o = attention.sdpa(q, k, v).to(torch.bfloat16)                  # [N, H, d]
    o8, so_ = quant.quant(o.reshape(n, heads * head_dim))
    return gemm.scaled_mm(o8, wo8, so_, so)


def fp32_block(x_local: torch.Tensor, wqkv: torch.Tensor, wo: torch.Tensor, heads: int, ws: int, a2a,
               head_dim: int = 128):
    """BASELINE config 0 on one rank: fp32 projections, Ulysses exchange with the collective ``a2a(out, inp)``,
    fp32 SDPA over the full sequence for H/P heads, reverse exchange, out projection."""
    m = x_local.shape[0]
    qkv = x_local @ wqkv.t()
    q, k, v = (t.reshape(m, heads, head_dim) for t in qkv.split(heads * head_dim, dim=1))
    recv = []
    for t in (q, k, v):
        send = ulysses.pack(t, ws)
        r = torch.empty_like(send)
        a2a(r, send)
        recv.append(r.reshape(ws * m, heads // ws, head_dim))
    o = attention.sdpa(*recv)                                       # [P*M, H/P, d] fp32
    back = torch.empty((ws, m, heads // ws, head_dim), dtype=o.dtype)
    a2a(back, o.contiguous().view(ws, m, heads // ws, head_dim))
    out = ulysses.unpack(back).reshape(m, heads * head_dim)
    return out @ wo.t()
