"""The out-projection's per-token FP8 quant read straight from the reverse all-to-all's receive buffer.

Mirrors ``h3_tp2/ulysses_outq.py``: row m of the out-projection input is concat_p recv[p, m] (P segments of H/P*d
bf16), quantised per token into the [M, H*d] e4m3 input plus the [M, 1] fp32 scale, so stock's unpack copy (copy 5)
and its [1, M, H, d] tensor are never made.  ``defer`` returns a ``Deferred`` holding the receive buffer; the
out-projection calls ``quantize()`` (or ``materialize()`` for a consumer that needs the bf16 tensor).
"""
from __future__ import annotations

import torch

from . import ops

FP8_MAX = 448.0
FP8_MIN = -448.0
MIN_SCALE = 1.0 / (FP8_MAX * 512.0)


def quant_rows(base: torch.Tensor, m: int, p: int, seg: int, stride_p: int, stride_m: int, warps: int = 8,
               div_mode: int = ops.DIV_IEEE):
    """h3_tp2/ulysses_outq.py:109 (``warps`` is accepted for signature compatibility; the CUDA kernel picks its own
    launch shape).  Returns (q [M, P*seg] e4m3, scale [M, 1] fp32)."""
    del warps
    return ops.quant_rows(base, m, p, seg, stride_p, stride_m, div_mode=div_mode)


def quant_reference_eager(x: torch.Tensor, out=None):  # noqa: ANN001,ANN201
    """Per-token dynamic e4m3 quant in eager torch (h3_tp2/ulysses_outq.py:126; ``fp8_quant_fuse.quant_torch``): (q,
    scale [.., 1]), or copied into ``out = (q, scale)`` and returned.  A CPU function by design."""
    from .fp8_quant_fuse import quant_torch  # noqa: PLC0415
    q, scale = quant_torch(x)
    if out is None:
        return q, scale
    out[0].copy_(q)
    out[1].copy_(scale)
    return out


def quant_from_recv(recv: torch.Tensor, warps: int = 8, div_mode: int = ops.DIV_IEEE):
    """h3_tp2/ulysses_outq.py:138: recv [P, M, hl, d] -> the quant of stock's unpacked [M, P*hl*d] rows."""
    del warps
    return ops.quant_from_recv(recv, div_mode=div_mode)


def unpack_rows(recv: torch.Tensor) -> torch.Tensor:
    """Stock's copy 5 (h3_tp2/ulysses_outq.py:146): [P, M, hl, d] -> contiguous [M, P*hl*d]."""
    p, m, hl, d = recv.shape
    return ops.unpack_recv(recv).view(m, p * hl * d)


class Deferred:
    """A reverse exchange whose unpack is left to the out-projection quant (h3_tp2/ulysses_outq.py:208)."""

    __slots__ = ("recv", "heads", "_done")

    def __init__(self, recv: torch.Tensor, heads: int):
        self.recv, self.heads, self._done = recv, heads, False

    @property
    def shape(self):  # noqa: ANN201
        p, m, hl, d = self.recv.shape
        return (1, m, p * hl, d)

    def quantize(self, div_mode: int = ops.DIV_IEEE):
        if self._done:
            raise RuntimeError("h3b ulysses_outq: deferred receive quantised twice")
        self._done = True
        return quant_from_recv(self.recv, div_mode=div_mode)

    def materialize(self) -> torch.Tensor:
        """The bf16 [1, M, H, d] tensor stock's unpack makes (for consumers other than the FP8 out-projection)."""
        p, m, hl, d = self.recv.shape
        return unpack_rows(self.recv).view(1, m, p * hl, d)


def defer(recv: torch.Tensor, heads: int) -> Deferred:
    """h3_tp2/ulysses_outq.py:407."""
    p, m, hl, d = recv.shape
    if p * hl != heads:
        raise ValueError(f"ulysses_outq.defer: {p} x {hl} heads received, {heads} expected")
    return Deferred(recv, heads)
