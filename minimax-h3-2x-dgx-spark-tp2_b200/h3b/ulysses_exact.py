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

import logging
import threading
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import ops

logger = logging.getLogger("h3b.ulysses_exact")

MODES = ("1", "2", "fwd", "verify")

# call counters (h3_tp2/ulysses_exact.py:88 ``stats``) and the two producer hooks (:144, :151)
_stats = {k: 0 for k in ("pack", "redirect", "materialize", "fallback", "out_copy", "unpack_hook", "verify_equal",
                         "verify_differs")}
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
    views of the qkv output -> send_q / send_k [P, M, H/P, d].  Without ``launch`` one CUDA kernel covers all
    destinations; with it (the reference's launcher ``launch(x_block, weight, rope_table, eps, out)``) it is called
    once per destination and tensor on that destination's heads."""
    ws, _, hl, _ = send_q.shape
    if launch is None:
        ops.norm_rope_send(q, q_weight, rope_table, eps, ws, out=send_q)
        ops.norm_rope_send(k, k_weight, rope_table, eps, ws, out=send_k)
        return
    for p in range(ws):
        heads = slice(p * hl, (p + 1) * hl)
        launch(q[:, heads], q_weight, rope_table, eps, send_q[p])
        launch(k[:, heads], k_weight, rope_table, eps, send_k[p])


def fused_into_send(fc, st, heads: int, head_dim: int, q_weight, k_weight, rope_table, eps, sends) -> None:  # noqa: ANN001
    """Consumer-fused producer (:278): the qkv projection of stash ``st`` written per destination into send_q / send_k
    / send_v [P, T, H/P, d], q and k normalised and rotated.  The reference runs three scale passes over the stashed
    fp32 product; here the qkv GEMM's epilogue does all three (``fc.qkv_into_send``), so the stash holds the FP8
    operands and the norm epilogue takes no bias."""
    if head_dim != 128:
        raise ValueError(f"fused_into_send: head_dim {head_dim} (the epilogue covers 128)")
    if getattr(st, "bias", None) is not None:
        raise ValueError("fused_into_send: the norm + RoPE epilogue takes no bias")
    fc.qkv_into_send(st, heads, sends[0].shape[0], q_weight, k_weight, rope_table, eps, sends=sends)


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


# ---------------------------------------------------------------------------------------------------------------
# producer redirection: placeholders, pending send buffers, the armed attention forward
# ---------------------------------------------------------------------------------------------------------------

_SELFCHECK_ROWS = 64   # producer calls of this many rows or fewer (a consumer's self-check) are never redirected
_tls = threading.local()  # armed: (attention, rows) of the running forward; pending: Pending


def _placeholder(like: torch.Tensor) -> torch.Tensor:
    """A tensor of ``like``'s shape owning one element (every stride 0): nothing may read it."""
    return like.new_empty(1).as_strided(tuple(like.shape), (0,) * like.ndim)


def _is_placeholder(t: torch.Tensor) -> bool:
    return t.numel() > 1 and all(st == 0 for st in t.stride())


@dataclass
class Pending:
    """Send buffers a redirected producer filled for the attention that follows (h3_tp2/ulysses_exact.py:320): q and k
    (and v) [P, M, hl, d] each, the placeholders the model holds for q and k, and the model's v view when the
    producer wrote v into send_v instead."""
    sends: list
    q_ph: torch.Tensor
    k_ph: torch.Tensor
    ws: int
    v_view: torch.Tensor | None = None
    unpack_fn: object = None   # [P, M, hl, d] -> [M, H, d]; default: the unpack kernel

    def matches(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor) -> bool:
        ok = (query.ndim == 4 and query.data_ptr() == self.q_ph.data_ptr() and key.data_ptr() == self.k_ph.data_ptr()
              and tuple(query.shape[1:]) == tuple(self.q_ph.shape))
        if ok and self.v_view is not None:
            ok = (value.ndim == 4 and value.data_ptr() == self.v_view.data_ptr()
                  and tuple(value.shape[1:]) == tuple(self.v_view.shape) and value[0].stride() == self.v_view.stride())
        return ok

    def materialize(self):  # noqa: ANN201
        """The real q, k [1, M, H, d] (and v written into the model's view) for a stock fallback."""
        _stats["materialize"] += 1
        un = self.unpack_fn or unpack
        q, k = un(self.sends[0]).unsqueeze(0), un(self.sends[1]).unsqueeze(0)
        if self.v_view is not None:
            self.v_view.copy_(un(self.sends[2]))
        self.sends = []
        return q, k


def take_pending(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor) -> Pending | None:
    """This thread's pending send buffers if q/k are their placeholders (consumed), else None; placeholder q/k without
    their buffers raise (h3_tp2/ulysses_exact.py:348)."""
    pend = getattr(_tls, "pending", None)
    if pend is not None and pend.matches(query, key, value):
        _tls.pending = None
        return pend
    if _is_placeholder(query) or _is_placeholder(key):
        raise RuntimeError("h3b ulysses exact: placeholder q/k reached attention without their send buffers")
    return None


def _take_arm(rows: int):  # noqa: ANN202
    """The attention whose forward is running, once, if ``rows`` is its row count (not a self-check sub-call) and it
    has no VSA gate (h3_tp2/ulysses_exact.py:358)."""
    arm = getattr(_tls, "armed", None)
    if arm is None or rows != arm[1] or rows <= _SELFCHECK_ROWS:
        return None
    _tls.armed = None
    owner = arm[0]
    return owner if getattr(owner, "to_gate_compress", None) is None else None


def make_armed_forward(orig_fwd, outq: bool = False):  # noqa: ANN001,ANN201
    """Wrap the model attention's ``forward(self, x, ...)`` so the producers know which attention their q/k feed and,
    with ``outq``, so its reverse exchange may leave copy 5 to its out-projection quant (h3_tp2/ulysses_exact.py:376)."""

    def forward(self, x, *a, **kw):  # noqa: ANN001,ANN202
        prev = getattr(_tls, "armed", None)
        rows = int(x.shape[0]) if hasattr(x, "shape") and x.ndim >= 1 else -1
        _tls.armed = (self, rows)
        if outq:
            from . import ulysses_outq  # noqa: PLC0415
            oprev = ulysses_outq.arm(self, rows)
        done = False
        try:
            out = orig_fwd(self, x, *a, **kw)
            done = True
            return out
        finally:
            _tls.armed = prev
            _tls.pending = None    # send buffers never outlive the forward that made them
            if outq:
                ulysses_outq.disarm(oprev, check=done)

    forward._h3b_exact_armed = True
    return forward


def rope_supported(q: torch.Tensor, k: torch.Tensor, rope_table: torch.Tensor, interleaved: bool) -> bool:
    """What the norm+RoPE send kernel takes: bf16 q/k [M, H, 128] with unit head-dim stride, half-split (not
    interleaved) rotation over a width that is a multiple of 8 and at most 128, on the GPU."""
    return (not interleaved and q.is_cuda and q.dtype == k.dtype == torch.bfloat16 and q.shape[-1] == 128
            and q.stride(-1) == 1 and k.stride(-1) == 1 and rope_table.shape[-1] % 8 == 0
            and rope_table.shape[-1] <= 128)


def make_rope(orig, strategy_info, launch=None, supported=None, *, unpack_fn=None):  # noqa: ANN001,ANN201
    """Wrap the transformer's ``fused_qk_norm_rope(q, k, q_weight, k_weight, rope_table, eps, *, head_dim,
    rotary_dim, interleaved)`` (h3_tp2/ulysses_exact.py:403): inside an armed attention forward whose attention will run
    strict Ulysses, q and k are normalised, rotated and written per destination into fresh send buffers and
    placeholders are returned; any other call runs ``orig``.  ``launch`` / ``supported``: a per-destination launcher and
    its guard (default: the send kernel and ``rope_supported``); ``unpack_fn`` for a fallback's materialisation."""
    supported = supported or rope_supported

    def fused_qk_norm_rope(q, k, q_weight, k_weight, rope_table, eps, *, head_dim=None, rotary_dim=None,  # noqa: ANN001,ANN202
                           interleaved=False):
        owner = _take_arm(int(q.shape[0])) if q.ndim == 3 else None
        info = strategy_info(owner.attention, None) if owner is not None else None
        if (info is None or q.shape != k.shape or head_dim not in (None, q.shape[-1])
                or rotary_dim not in (None, rope_table.shape[-1])
                or rope_table.shape != (q.shape[0], rope_table.shape[-1])
                or not eligible_shape(q.unsqueeze(0), k.unsqueeze(0), k.unsqueeze(0), info[1])
                or not supported(q, k, rope_table, interleaved)):
            return orig(q, k, q_weight, k_weight, rope_table, eps, head_dim=head_dim, rotary_dim=rotary_dim,
                        interleaved=interleaved)
        ws = info[1]
        m, heads, d = q.shape
        sends = [torch.empty(send_shape(m, heads, d, ws), dtype=q.dtype, device=q.device) for _ in range(2)]
        rope_into_send(sends[0], sends[1], q, k, q_weight.contiguous(), k_weight.contiguous(),
                       rope_table.contiguous(), eps, launch)
        _tls.pending = Pending(sends=sends, q_ph=_placeholder(q), k_ph=_placeholder(k), ws=ws, unpack_fn=unpack_fn)
        _stats["redirect"] += 1
        return _tls.pending.q_ph, _tls.pending.k_ph

    fused_qk_norm_rope._h3b_exact = True
    return fused_qk_norm_rope


def make_fused_producer(orig, fc, strategy_info, *, unpack_fn=None):  # noqa: ANN001,ANN201
    """Wrap ``fp8_consumers.qk_norm_rope_fused(st, num_heads, num_kv_heads, head_dim, q_weight, k_weight, rope_table,
    eps)`` (h3_tp2/ulysses_exact.py:433): inside an armed forward the qkv GEMM with the norm + RoPE epilogue writes q, k
    and v per destination (``fc.qkv_into_send``), placeholders stand for q and k and the model's v view of the stash's
    placeholder is returned unwritten; any other call runs ``orig``."""

    def qk_norm_rope_fused(st, num_heads, num_kv_heads, head_dim, q_weight, k_weight, rope_table, eps):  # noqa: ANN001,ANN202
        t = int(st.a.shape[0])
        owner = _take_arm(t)
        info = strategy_info(owner.attention, None) if owner is not None else None
        hd = num_heads * head_dim
        if (info is None or num_kv_heads != num_heads or num_heads % info[1] != 0 or head_dim != 128
                or st.bias is not None or st.ph is None or st.ph.dim() != 2 or st.ph.shape != (t, 3 * hd)
                or not st.ph.is_contiguous()):
            return orig(st, num_heads, num_kv_heads, head_dim, q_weight, k_weight, rope_table, eps)
        ws = info[1]
        sends = list(fc.qkv_into_send(st, num_heads, ws, q_weight.contiguous(), k_weight.contiguous(),
                                      rope_table.contiguous(), eps))
        like = st.ph[:, :hd].view(t, num_heads, head_dim)
        v_view = st.ph[:, 2 * hd:].view(t, num_kv_heads, head_dim)   # the model's v view (left unwritten)
        pend = Pending(sends=sends, q_ph=_placeholder(like), k_ph=_placeholder(like), ws=ws, v_view=v_view,
                       unpack_fn=unpack_fn)
        _tls.pending = pend
        _stats["redirect"] += 1
        return pend.q_ph, pend.k_ph, v_view

    qk_norm_rope_fused._h3b_exact = True
    return qk_norm_rope_fused


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
    return torch.ops.h3b.flash_attn(q, k, v, None, valid)


def make_forward_impl(orig, mode: str, strategy_info, *, a2a=None, stock_fwd=None, stock_back=None, on_first=None,  # noqa: ANN001,ANN201
                      attn=None, pack=None, unpack_fn=None):
    """Wrap ``Attention._forward_impl(self, query, key, value, attn_metadata=None)`` (h3_tp2/ulysses_exact.py:472):
    eligible strict-Ulysses calls run ``exact_forward`` (on the send buffers a redirected producer filled, when q/k are
    its placeholders) with the B200 attention; a placeholder call that is not eligible is materialised and, like
    anything else, runs ``orig``.  ``on_first()`` runs once, on the first call (attaches the producer hooks).
    ``attn(q, k, v, attn_metadata)`` (default ``local_attention``), ``pack`` / ``unpack_fn``: as in
    ``exact_forward``."""
    if mode not in MODES:
        raise ValueError(f"H3_TP2_ULYSSES_EXACT must be one of {MODES}, got {mode!r}")
    attn = attn or local_attention
    hooked = {"done": False}

    def _forward_impl(self, query, key, value, attn_metadata=None):  # noqa: ANN001
        if on_first is not None and not hooked["done"]:
            hooked["done"] = True
            on_first()
        pend = take_pending(query, key, value)
        info = strategy_info(self, attn_metadata)
        ok = info is not None and eligible_shape(query, key, value, info[1])  # placeholders carry the real shape
        if pend is not None and (not ok or pend.ws != info[1]):
            query, key = pend.materialize()
            pend = None
        if not ok:
            _stats["fallback"] += 1
            return orig(self, query, key, value, attn_metadata)
        pg, ws = info

        def run(q, k, v):  # noqa: ANN001,ANN202
            return attn(q, k, v, attn_metadata)

        if mode == "verify":   # both exchanges on the same tensors; the stock result is returned
            res, eq = verify_forward(query, key, value, run, ws=ws, pg=pg, a2a=a2a, stock_fwd=stock_fwd,
                                     stock_back=stock_back, pack=pack, unpack_fn=unpack_fn)
            differs = not all(eq.values())
            if differs or _stats["verify_equal"] % 500 == 0:
                logger.warning("h3b ulysses exact verify: %s (%d equal, %d differ so far)",
                               " ".join(f"{n}={'eq' if e else 'DIFF'}" for n, e in eq.items()),
                               _stats["verify_equal"], _stats["verify_differs"])
            return res
        sends = None
        if pend is not None:
            sends, pend.sends = pend.sends, []
        back = {"fwd": "stock", "2": "defer"}.get(mode, "exact")
        sb = stock_back or (lambda t: _stock_a2a_4d(t, 1, 2, pg))
        return exact_forward(query, key, value, run, ws=ws, pg=pg, a2a=a2a, sends=sends, back=back, stock_back=sb,
                             pack=pack, unpack_fn=unpack_fn)

    return _forward_impl


def _hook_producers(strategy_info, mode: str = "1") -> None:  # noqa: ANN001
    """Attach the arming wrapper and the producer hook to vLLM-Omni's MiniMax H3 model (the first wrapped attention
    call does this; h3_tp2/ulysses_exact.py:521)."""
    from vllm_omni.diffusion.models.minimax_h3 import minimax_h3_transformer as tr  # noqa: PLC0415
    _hook_producers_on(tr, strategy_info, mode)


def _hook_producers_on(tr, strategy_info, mode: str = "1") -> None:  # noqa: ANN001
    """``_hook_producers`` on the transformer module ``tr``: in mode 2 the deferral's upstream path is checked first,
    on the attention forward as upstream wrote it (a changed path keeps the reverse unpack, ``ulysses_outq.prepare``
    refuses every attention)."""
    att_cls = tr.MiniMaxH3Attention
    if not getattr(att_cls.forward, "_h3b_exact_armed", False):
        outq = mode == "2"
        if outq:
            from . import ulysses_outq  # noqa: PLC0415
            reason = ulysses_outq.check_sources(att_cls.forward)
            logger.warning("h3b ulysses exact: the reverse unpack %s", "left to the out-projection quant (self-check "
                           "on the first call)" if reason is None else f"kept ({reason})")
        att_cls.forward = make_armed_forward(att_cls.forward, outq=outq)
    if getattr(tr.fused_qk_norm_rope, "_h3b_consumer_fuse", False):
        from . import fp8_consumers as fc  # noqa: PLC0415
        if not getattr(fc.qk_norm_rope_fused, "_h3b_exact", False):
            fc.qk_norm_rope_fused = make_fused_producer(fc.qk_norm_rope_fused, fc, strategy_info)
    elif not getattr(tr.fused_qk_norm_rope, "_h3b_exact", False):
        tr.fused_qk_norm_rope = make_rope(tr.fused_qk_norm_rope, strategy_info)


def install(mode: str = "1") -> None:
    """Wrap vLLM-Omni's ``Attention._forward_impl`` (h3_tp2/ulysses_exact.py:552); needs vLLM-Omni."""
    try:
        from vllm_omni.diffusion.attention import layer as layer_mod  # noqa: PLC0415
    except ImportError as exc:  # pragma: no cover - vLLM-Omni is not part of this image
        raise RuntimeError("h3b.ulysses_exact.install needs vLLM-Omni (not installed)") from exc
    from .plugin import vllm_strategy_info  # noqa: PLC0415
    mode = mode.strip().lower()
    cls = layer_mod.Attention
    if getattr(cls, "_h3b_overlap", 0) or getattr(cls, "_h3b_nocopy", 0):
        raise RuntimeError("h3b: a grouped Ulysses exchange (overlap or nocopy) is installed; exact replaces it")
    prev = getattr(cls, "_h3b_exact", None)
    if prev:
        if prev != mode:
            raise RuntimeError(f"h3b ulysses exact already installed with mode {prev}, cannot change to {mode}")
        return
    hook = None if mode == "verify" else (lambda: _hook_producers(vllm_strategy_info, mode))  # verify: stock producers
    cls._forward_impl = make_forward_impl(cls._forward_impl, mode, vllm_strategy_info, on_first=hook)
    cls._h3b_exact = mode
