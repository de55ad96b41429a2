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

# call counters (h3_tp2/ulysses_exact.py:88 ``stats``) and the two producer hooks (:144, :151)
_stats = {k: 0 for k in ("pack", "redirect", "fallback", "out_copy", "unpack_hook", "verify_equal", "verify_differs")}
_hooks = {"key": None, "unpack": None}


def stats() -> dict[str, int]:
    return dict(_stats)


def set_key_hook(fn) -> None:  # noqa: ANN001
    """``fn(send_k)`` runs on this rank's packed keys [P, M, hl, d] right before their exchange; None: nothing runs
    (h3_tp2/ulysses_exact.py:144)."""
    _hooks["key"] = fn


def set_unpack_hook(fn) -> None:  # noqa: ANN001
    """``fn(recv [P, M, hl, d], heads)`` may replace the reverse unpack: it returns stock's [1, M, H, d] result, or None
    for the ordinary unpack (h3_tp2/ulysses_exact.py:151)."""
    _hooks["unpack"] = fn


def _a2a(out: torch.Tensor, inp: torch.Tensor, group=None) -> None:  # noqa: ANN001
    dist.all_to_all_single(out, inp, group=group)


def _stock_a2a_4d(x: torch.Tensor, scatter_idx: int, gather_idx: int, pg) -> torch.Tensor:  # noqa: ANN001
    """vLLM-Omni's stock all-to-all (the comparison side of ``verify``); needs vLLM-Omni."""
    try:
        from vllm_omni.diffusion.distributed.comm import all_to_all_4D  # noqa: PLC0415
    except ImportError as exc:  # pragma: no cover - vLLM-Omni is not part of this image
        raise RuntimeError("the stock all-to-all needs vLLM-Omni (not installed): pass stock_fwd / stock_back") from exc
    return all_to_all_4D(x, scatter_idx, gather_idx, group=pg)


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
    (h3_tp2/ulysses_exact.py:156).  With ``defer`` the receive buffer is offered to ``ulysses_outq.defer``: when this
    forward was armed for it, its stride-0 placeholder is returned instead of the unpacked tensor (the out-projection
    quant then reads the receive buffer); otherwise the unpack runs as without."""
    o3 = o[0]
    if not o3.is_contiguous():
        _stats["out_copy"] += 1
        o3 = o3.contiguous()
    s, hl, d = o3.shape
    m = s // ws
    recv = torch.empty((ws, m, hl, d), dtype=o3.dtype, device=o3.device)
    a2a(recv, o3, group=pg)
    if defer:  # the armed forward's out-projection quant reads the receive buffer (a placeholder stands for copy 5)
        from . import ulysses_outq
        ph = ulysses_outq.defer(recv, heads)
        if ph is not None:
            return ph
    else:
        hook = _hooks["unpack"]
        if hook is not None:
            res = hook(recv, heads)
            if res is not None:
                _stats["unpack_hook"] += 1
                return res
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
        _stats["redirect"] += 1
        send_q, send_k = sends[0], sends[1]
        send_v = sends[2] if len(sends) > 2 else None
        sends.clear()
    else:
        _stats["pack"] += 1
        send_q, send_k, send_v = do_pack(query[0]), do_pack(key[0]), None
    q = exchange_fwd(send_q, a2a, pg)
    del send_q
    if _hooks["key"] is not None:
        _hooks["key"](send_k)
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


def _same(a: torch.Tensor, b: torch.Tensor) -> bool:
    """Bitwise equality (NaN payloads included) of same-shape, same-dtype tensors."""
    if a.shape != b.shape or a.dtype != b.dtype:
        return False
    if a.element_size() == 2:
        return torch.equal(a.contiguous().view(torch.int16), b.contiguous().view(torch.int16))
    return torch.equal(a, b)


def _same_layout(a: torch.Tensor, b: torch.Tensor) -> bool:
    """Same shape and the same strides in every dimension longer than 1 (a stride of a size-1 dimension is
    arbitrary)."""
    return a.shape == b.shape and all(sa == sb for n, sa, sb in zip(a.shape, a.stride(), b.stride()) if n > 1)


def verify_forward(query, key, value, run_attn, *, ws, pg=None, a2a=None, stock_fwd=None, stock_back=None,  # noqa: ANN001,ANN201
                   pack=None, unpack_fn=None):
    """Runs the stock exchange (``stock_fwd`` seq->head and ``stock_back`` head->seq, default vLLM-Omni's
    ``all_to_all_4D``) and the exact one on the same q/k/v [1, M, H, d]; returns (stock result, {"q", "k", "v",
    "attn", "result": bitwise equal}) (h3_tp2/ulysses_exact.py:232).  ``pack`` / ``unpack_fn`` as in
    ``exact_forward``."""
    a2a = a2a or _a2a
    stock_fwd = stock_fwd or (lambda t: _stock_a2a_4d(t, 2, 1, pg))
    stock_back = stock_back or (lambda t: _stock_a2a_4d(t, 1, 2, pg))
    _, m, heads, d = value.shape
    sq, sk, sv = stock_fwd(query), stock_fwd(key), stock_fwd(value)
    so = run_attn(sq, sk, sv)
    sres = stock_back(so)
    eq = {}
    received = []
    for name, x, ref in (("q", query, sq), ("k", key, sk), ("v", value, sv)):
        if pack is not None:
            send = pack(x[0], ws)
        else:
            send = torch.empty(send_shape(m, heads, d, ws), dtype=x.dtype, device=x.device)
            pack_into(send, x[0], ws)
        r = exchange_fwd(send, a2a, pg)
        eq[name] = _same_layout(r, ref) and _same(r, ref)
        received.append(r)
    del sq, sk, sv
    o = run_attn(*received)
    eq["attn"] = _same(o, so)
    res = exchange_back(o, heads, ws, a2a, pg, unpack_fn=unpack_fn)
    eq["result"] = res.is_contiguous() and _same(res, sres)
    _stats["verify_equal" if all(eq.values()) else "verify_differs"] += 1
    return sres, eq


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
            _stats["fallback"] += 1
            return orig(self, query, key, value, attn_metadata)
        pg, ws = info
        attn = lambda q, k, v: local_attention(q, k, v, attn_metadata)  # noqa: E731
        if mode == "verify":   # both exchanges on the same tensors; the stock result is returned
            res, _ = verify_forward(query, key, value, attn, ws=ws, pg=pg, a2a=a2a)
            return res
        back = {"2": "defer", "fwd": "exact"}.get(mode, "exact")
        return exact_forward(query, key, value, attn, ws=ws, pg=pg, a2a=a2a, back=back)

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
