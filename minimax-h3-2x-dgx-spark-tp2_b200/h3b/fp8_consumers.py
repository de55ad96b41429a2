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
  on 256-column tiles): ``materialize`` the out projection and use ``h3b.fp8_quant_fuse.gate_rms_quant``, which also
  quantises the modulated output for fc1.
"""
from __future__ import annotations

import torch

from . import ops


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


def gate_fused(st: Stash, x: torch.Tensor, gate: torch.Tensor, indices: torch.Tensor,
               reuse_placeholder: bool = True) -> torch.Tensor:
    """``indexed_gate(x, gate, fc2_output, indices)`` with the fc2 GEMM: written into the placeholder when ``x`` is
    contiguous (stock: ``empty_like(x)``)."""
    out = st.ph if (reuse_placeholder and st.ph is not None and x.is_contiguous()) else None
    if x.shape[0] == 0:
        return out if out is not None else torch.empty_like(x)
    return ops.fp8_gemm_gate(st.a, st.w, st.sa, st.sb, x, gate, indices, st.bias, out=out)
