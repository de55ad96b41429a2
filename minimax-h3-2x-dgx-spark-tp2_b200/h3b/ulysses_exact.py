"""Ulysses exact exchange (strict Ulysses at batch 1) with the reference's layouts and signatures.

Mirrors ``h3_tp2/ulysses_exact.py``: the send buffer is stock's ``input_t`` [P, M, H/P, d] (head h = p*(H/P) + j goes
to rank p), the forward all-to-all receives [P, M, H/P, d] viewed [1, P*M, H/P, d] (= stock's q/k/v), the attention
output [P*M, H/P, d] is sent back as is and the receive [P, M, H/P, d] is unpacked into [1, M, H, d] (or left to the
out-projection quant, ``back="defer"``).  On B200 the producers that fill the send buffers are the qkv GEMM's
epilogue (``ops.fp8_gemm_qkv_send``) or the ``pack`` kernel; the collective is NCCL ``all_to_all_single`` over
NVLink (or any injected ``a2a(out, inp, group=)``).

``pack`` / ``unpack_fn`` default to the CUDA layout kernels; host-logic tests inject CPU implementations.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops

MODES = ("1", "2", "fwd", "verify")


def _a2a(out: torch.Tensor, inp: torch.Tensor, group=None) -> None:  # noqa: ANN001
    dist.all_to_all_single(out, inp, group=group)


def send_shape(m: int, heads: int, d: int, ws: int) -> tuple[int, int, int, int]:
    """Stock's ``input_t`` for batch 1 without the unit dim (h3_tp2/ulysses_exact.py:108)."""
    return (ws, m, heads // ws, d)


def by_dest(x: torch.Tensor, ws: int) -> torch.Tensor:
    """[M, H, d] -> view [P, M, H/P, d] (h3_tp2/ulysses_exact.py:113)."""
    m, h, d = x.shape
    return x.unflatten(1, (ws, h // ws)).transpose(0, 1)


def pack_into(send: torch.Tensor, x: torch.Tensor, ws: int) -> None:
    """Stock's pack copy into ``send`` (h3_tp2/ulysses_exact.py:119), as one CUDA kernel."""
    ops.pack_by_dest(x, ws, out=send, to_f16=send.dtype == torch.float16 and x.dtype == torch.bfloat16)


def unpack(send: torch.Tensor) -> torch.Tensor:
    """[P, M, hl, d] -> [M, H, d] contiguous (h3_tp2/ulysses_exact.py:124)."""
    return ops.unpack_recv(send.contiguous())


def rope_into_send(send_q, send_k, q, k, q_weight, k_weight, rope_table, eps, launch=None) -> None:  # noqa: ANN001
    """The norm+RoPE producer writing straight into the send buffers (h3_tp2/ulysses_exact.py:264): q/k [M, H, d]
    views of the qkv output -> send_q / send_k [P, M, H/P, d].  ``launch`` (the reference's per-destination launcher
    argument) is accepted for signature compatibility; one CUDA kernel covers all destinations."""
    del launch
    ws = send_q.shape[0]
    ops.norm_rope_send(q, q_weight, rope_table, eps, ws, out=send_q)
    ops.norm_rope_send(k, k_weight, rope_table, eps, ws, out=send_k)


def exchange_fwd(send: torch.Tensor, a2a, pg=None) -> torch.Tensor:  # noqa: ANN001
    """One forward all-to-all; the receive buffer viewed [1, P*M, hl, d] (h3_tp2/ulysses_exact.py:130)."""
    recv = torch.empty_like(send)
    a2a(recv, send, group=pg)
    p, m, hl, d = recv.shape
    return recv.view(1, p * m, hl, d)


def exchange_back(o: torch.Tensor, heads: int, ws: int, a2a, pg=None, defer: bool = False,  # noqa: ANN001
                  unpack_fn=None):
    """Attention output [1, P*M, hl, d] -> [1, M, H, d]: one all-to-all of ``o`` itself, then the unpack
    (h3_tp2/ulysses_exact.py:156).  With ``defer`` the receive buffer is handed to ``ulysses_outq.defer`` and its
    ``Deferred`` (whose ``quantize()`` reads the receive buffer) is returned instead of the unpacked tensor."""
    o3 = o[0]
    if not o3.is_contiguous():
        o3 = o3.contiguous()
    s, hl, d = o3.shape
    m = s // ws
    recv = torch.empty((ws, m, hl, d), dtype=o3.dtype, device=o3.device)
    a2a(recv, o3, group=pg)
    if defer:
        from . import ulysses_outq
        return ulysses_outq.defer(recv, heads)
    res = (unpack_fn or unpack)(recv)
    return res.reshape(1, m, heads, d)


def exact_forward(query, key, value, run_attn, *, ws, pg=None, a2a=None, sends=None, back="exact",  # noqa: ANN001,ANN201
                  stock_back=None, pack=None, unpack_fn=None):
    """Strict Ulysses at batch 1 (h3_tp2/ulysses_exact.py:187).  ``sends``: [send_q, send_k(, send_v)] already filled
    by a redirected producer (consumed here), else q/k/v are packed.  ``back``: "exact", "defer" or "stock"."""
    a2a = a2a or _a2a
    _, m, heads, d = value.shape
    shape = send_shape(m, heads, d, ws)
    dt, dev = value.dtype, value.device

    def do_pack(x):
        if pack is not None:
            return pack(x, ws)
        buf = torch.empty(shape, dtype=dt, device=dev)
        pack_into(buf, x, ws)
        return buf

    if sends:
        send_q, send_k = sends[0], sends[1]
        send_v = sends[2] if len(sends) > 2 else None
        sends.clear()
    else:
        send_q, send_k, send_v = do_pack(query[0]), do_pack(key[0]), None
    q = exchange_fwd(send_q, a2a, pg)
    del send_q
    k = exchange_fwd(send_k, a2a, pg)
    del send_k
    if send_v is None:
        send_v = do_pack(value[0])
    v = exchange_fwd(send_v, a2a, pg)
    del send_v
    o = run_attn(q, k, v)
    del q, k, v
    if back == "stock":
        if stock_back is None:
            raise ValueError("exact_forward: back='stock' needs stock_back")
        return stock_back(o)
    return exchange_back(o, heads, ws, a2a, pg, defer=back == "defer", unpack_fn=unpack_fn)


def eligible_shape(query, key, value, ws: int) -> bool:  # noqa: ANN001
    """Strict Ulysses eligibility (h3_tp2/ulysses_exact.py:367-373)."""
    if query.ndim != 4 or key.shape != query.shape or value.shape != query.shape:
        return False
    if query.shape[0] != 1 or ws < 2 or query.shape[2] % ws != 0:
        return False
    return key.dtype == query.dtype == value.dtype and key.device == query.device == value.device


def local_attention(q, k, v, attn_metadata=None):  # noqa: ANN001,ANN201
    """The B200 local attention (replaces cuDNN SDPA): q/k/v [1, S, hl, d] -> [1, S, hl, d] bf16."""
    valid = None
    if attn_metadata is not None:
        valid = getattr(attn_metadata, "valid_kv_length", None)
    return ops.flash_attn(q, k, v, valid_kv=valid)


def make_forward_impl(orig, mode: str, strategy_info, *, a2a=None):  # noqa: ANN001,ANN201
    """Wrap ``Attention._forward_impl(self, query, key, value, attn_metadata=None)`` (h3_tp2/ulysses_exact.py:472):
    eligible strict-Ulysses calls run ``exact_forward`` with the B200 attention; anything else runs ``orig``."""
    if mode not in MODES:
        raise ValueError(f"H3_TP2_ULYSSES_EXACT must be one of {MODES}, got {mode!r}")

    def _forward_impl(self, query, key, value, attn_metadata=None):  # noqa: ANN001
        info = strategy_info(self, attn_metadata)
        if info is None or not eligible_shape(query, key, value, info[1]):
            return orig(self, query, key, value, attn_metadata)
        pg, ws = info
        back = {"2": "defer", "fwd": "exact"}.get(mode, "exact")
        res = exact_forward(query, key, value, lambda q, k, v: local_attention(q, k, v, attn_metadata), ws=ws, pg=pg,
                            a2a=a2a, back=back)
        if back == "defer":
            return res.materialize()
        return res

    return _forward_impl


def install(mode: str = "1") -> None:
    """Wrap vLLM-Omni's ``Attention._forward_impl`` (h3_tp2/ulysses_exact.py:552); needs vLLM-Omni."""
    try:
        from vllm_omni.diffusion.attention import layer as layer_mod  # noqa: PLC0415
    except ImportError as exc:  # pragma: no cover - vLLM-Omni is not part of this image
        raise RuntimeError("h3b.ulysses_exact.install needs vLLM-Omni (not installed)") from exc
    from .plugin import vllm_strategy_info  # noqa: PLC0415
    mode = mode.strip().lower()
    cls = layer_mod.Attention
    prev = getattr(cls, "_h3b_exact", None)
    if prev:
        if prev != mode:
            raise RuntimeError(f"h3b ulysses exact already installed with mode {prev}, cannot change to {mode}")
        return
    cls._forward_impl = make_forward_impl(cls._forward_impl, mode, vllm_strategy_info)
    cls._h3b_exact = mode
