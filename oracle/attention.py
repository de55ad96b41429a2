"""Non-causal scaled-dot-product attention in fp32 (the numerical oracle for the attention kernel).

The reference runs cuDNN SDPA (upstream vLLM-Omni, not vendored), whose results are not reproducible here, so the
attention parity contract is against an fp32 SDPA on the same bf16 inputs: rel-L2 <= 2e-3 and max-abs <= 2e-2
(the reference's CPU tests use ``SDPBackend.MATH`` with scale d^-1/2, ``tests/test_ulysses_exact.py:101-105``).
Computed in query chunks so the score matrix never exceeds ``chunk * S_kv`` floats.
"""
from __future__ import annotations

import torch


def sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float | None = None, valid_kv: int | None = None,
         chunk: int = 2048) -> torch.Tensor:
    """q [S_q, H, d], k/v [S_kv, H, d] (any float dtype) -> fp32 [S_q, H, d]."""
    s_q, h, d = q.shape
    if valid_kv is not None:
        k, v = k[:valid_kv], v[:valid_kv]
    sc = d ** -0.5 if scale is None else scale
    kf = k.float().permute(1, 2, 0)        # [H, d, S_kv]
    vf = v.float().permute(1, 0, 2)        # [H, S_kv, d]
    out = torch.empty((s_q, h, d), dtype=torch.float32)
    for c0 in range(0, s_q, chunk):
        qf = q[c0:c0 + chunk].float().permute(1, 0, 2)   # [H, c, d]
        s = torch.bmm(qf, kf) * sc
        s = s - s.amax(dim=-1, keepdim=True)
        p = torch.exp(s)
        o = torch.bmm(p, vf) / p.sum(dim=-1, keepdim=True)
        out[c0:c0 + chunk] = o.permute(1, 0, 2)
    return out


def rel_l2(x: torch.Tensor, ref: torch.Tensor) -> float:
    x, ref = x.double(), ref.double()
    return float((x - ref).norm() / ref.norm().clamp_min(1e-300))
