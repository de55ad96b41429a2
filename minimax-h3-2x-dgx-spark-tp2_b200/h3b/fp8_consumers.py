"""Consumers of an FP8 GEMM's output fused with the GEMM (mirror of ``h3_tp2/fp8_consumers.py``).

The reference keeps the fp32 product of the qkv / out / fc2 GEMMs (a "stash", ``Stash`` :388) and replaces the kernel
that consumes each bf16 output with a copy that applies the scale pass's arithmetic itself, so the bf16 [M, N]
intermediate is never written.  On B200 the consumer's arithmetic runs in the GEMM's own epilogue instead, so not even
the fp32 product reaches HBM: a ``Stash`` here holds the GEMM's operands, and each consumer launches one kernel.

* ``qk_norm_rope_fused`` (:406): q and k RMSNorm + partial RoPE and the v scale pass — the qkv GEMM with the
  norm + RoPE epilogue (``h3b_fp8_gemm`` with ``H3B_EPI_QKV_SEND`` and norm weights, P = 1 layout = [M, H, d]).
* ``gate_fused`` (:468): ``x + gate[indices] * fc2`` — the fc2 GEMM with the indexed-gate epilogue
  (``h3b_fp8_gemm_gate``).
* ``gate_rms_fused`` (:445) has no one-kernel form (the RMS needs whole rows of the out projection, the GEMM works
  on 256-column tiles): it materialises the out projection, runs the gated residual + RMSNorm + modulation row kernel
  for ``residual_out`` and the RMSNorm + modulation row kernel on that for the bf16 modulated rows.
"""
from __future__ import annotations

import torch

from . import ops

SITES = ("qkv", "out", "fc2")


class Stash:
    """The operands of one FP8 GEMM whose output a fused consumer reads (reference ``Stash``: the fp32 product)."""
    __slots__ = ("a", "w", "sa", "sb", "bias", "ph")

    def __init__(self, a: torch.Tensor, w: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor,
                 bias: torch.Tensor | None, ph: torch.Tensor | None = None):
        self.a, self.w, self.sa, self.sb, self.bias, self.ph = a, w, sa, sb, bias, ph

    def materialize(self) -> torch.Tensor:
        """The ordinary bf16 output (into the placeholder when one was given)."""
        return ops.fp8_gemm(self.a, self.w, self.sa, self.sb, self.bias, out=self.ph)

    def rows(self, r: int) -> "Stash":
        return Stash(self.a[:r], self.w, self.sa[:r], self.sb, self.bias, None)


def qk_norm_rope_fused(st: Stash, num_heads: int, num_kv_heads: int, head_dim: int, q_weight: torch.Tensor,
                       k_weight: torch.Tensor, rope_table: torch.Tensor, eps: float):
    """(q, k, v) [T, H, d] bf16: per-head RMSNorm + partial RoPE (rotary dims = rope_table's width, cos | sin) on q
    and k, v scale-passed, all in the qkv GEMM's epilogue."""
    if num_kv_heads != num_heads or head_dim != 128:
        raise ValueError("qk_norm_rope_fused: equal q/kv heads of 128 dims only")
    if st.bias is not None:
        raise ValueError("qk_norm_rope_fused: the norm epilogue takes no bias")
    q, k, v = ops.fp8_gemm_qkv_send(st.a, st.w, st.sa, st.sb, num_heads, 1,
                                    qk_norm=(q_weight, k_weight, rope_table.float(), eps))
    T = st.a.shape[0]
    return tuple(t.view(T, num_heads, head_dim) for t in (q, k, v))


def qkv_into_send(st: Stash, num_heads: int, ws: int, q_weight: torch.Tensor, k_weight: torch.Tensor,
                  rope_table: torch.Tensor, eps: float, sends=None):  # noqa: ANN001
    """The qkv GEMM of ``st`` with the norm + RoPE epilogue writing per destination (the producer ``ulysses_exact``'s
    redirection uses; h3_tp2/ulysses_exact.py:278 ``fused_into_send``): (send_q, send_k, send_v) [P, M, H/P, 128] bf16,
    q and k normalised and rotated, v the plain scale pass; into ``sends`` when given."""
    return ops.fp8_gemm_qkv_send(st.a, st.w, st.sa, st.sb, num_heads, ws, sends=sends,
                                 qk_norm=(q_weight, k_weight, rope_table.float(), eps))


def gate_fused(st: Stash, x: torch.Tensor, gate: torch.Tensor, indices: torch.Tensor,
               reuse_placeholder: bool = True) -> torch.Tensor:
    """``indexed_gate(x, gate, fc2_output, indices)`` with the fc2 GEMM: written into the placeholder when ``x`` is
    contiguous (stock: ``empty_like(x)``)."""
    out = st.ph if (reuse_placeholder and st.ph is not None and x.is_contiguous()) else None
    if x.shape[0] == 0:
        return out if out is not None else torch.empty_like(x)
    return ops.fp8_gemm_gate(st.a, st.w, st.sa, st.sb, x, gate, indices, st.bias, out=out)


def gate_rms_fused(st: Stash, residual: torch.Tensor, gate: torch.Tensor, weight: torch.Tensor, shift: torch.Tensor,
                   scale: torch.Tensor, indices: torch.Tensor, eps: float, reuse_placeholder: bool = True):
    """``indexed_gate_rms_norm_scale_shift(residual, gate, branch, ...)`` with branch = the out projection of ``st``
    (h3_tp2/fp8_consumers.py:445): returns (residual_out = bf16(residual + gate[indices] * branch), modulated_out =
    bf16 RMSNorm(residual_out) * weight * (1 + scale[indices]) + shift[indices]); ``residual_out`` goes into the
    placeholder when ``reuse_placeholder`` and the stash has one."""
    rows = residual.shape[0]
    residual_out = st.ph if (reuse_placeholder and st.ph is not None) else torch.empty_like(residual)
    modulated_out = torch.empty_like(residual)
    if rows == 0:
        return residual_out, modulated_out
    branch = ops.fp8_gemm(st.a, st.w, st.sa, st.sb, st.bias)
    r_out, _, _ = ops.gate_rms_quant(residual, gate, branch, weight, shift, scale, indices, eps)
    ops.rms_quant(r_out, weight, shift, scale, indices, eps, modulated_out)
    if residual_out is not r_out:
        residual_out.copy_(r_out)
    return residual_out, modulated_out


def epilogue_bf16_torch(acc: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    """The bf16 epilogue in eager torch on broadcastable fp32 tensors (h3_tp2/fp8_consumers.py:305): column scale,
    row scale (bias by an fma carried out in float64), rounded to bf16 and returned as fp32."""
    t = sb * acc
    y = sa * t if bias is None else (sa.double() * t.double() + bias.double()).float()
    return y.to(torch.bfloat16).float()


def scale_pass_into(x32: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, bias: torch.Tensor | None,
                    y: torch.Tensor) -> torch.Tensor:
    """The ordinary two-pass scale pass into ``y`` (h3_tp2/fp8_consumers.py:373): the scale-pass kernel on the GPU.
    CPU tensors raise (the reference's eager CPU branch is ``fp8_gemm.epilogue_torch``, called explicitly)."""
    y.copy_(ops.scale_bias_cast(x32, sa, sb, bias, y.dtype))
    return y


def parse_sites(value: str | None) -> tuple[str, ...]:
    """``H3_TP2_FP8_CONSUMER_FUSE`` (h3_tp2/fp8_consumers.py:813): "1"/"all"/"on"/"true" = every site, a comma list of
    qkv,out,fc2 selects sites, anything else or empty = none."""
    v = (value or "").strip().lower()
    if v in ("1", "all", "on", "true"):
        return SITES
    if v in ("", "0", "off", "false"):
        return ()
    chosen = {part.strip() for part in v.split(",")}
    return tuple(site for site in SITES if site in chosen)
