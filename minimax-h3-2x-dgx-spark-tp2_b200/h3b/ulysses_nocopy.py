"""The combined q/k/v Ulysses exchange (mirror of ``h3_tp2/ulysses_nocopy.py``).

Stock strict Ulysses runs three forward all-to-alls (q, k, v) per block.  This layout puts q, k and v of a token side
by side in ONE send buffer ``send[group, dest, M, 3, hl, d]`` (``send_shape``, :74), so each head group needs one
exchange; the receive buffer ``recv[dest, M, 3, hl, d]`` viewed as [P*M, 3, hl, d] gives q, k and v as strided views
(row stride 3*hl*d, ``qkv_views`` :105) that the attention kernel reads through its 3-D TMA descriptors with no copy.
On B200 the producer is the qkv GEMM itself (``ops.fp8_gemm_qkv_send(..., interleaved=True)`` writes the layout in its
epilogue); ``pack_qkv`` is the reference's fallback producer for q/k/v that come from elsewhere.  The reverse exchange
sends the dense attention output of each group and unpacks it into the [1, M, H, d] result (``back_into`` :112).
"""
from __future__ import annotations

import threading
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import ops

_tls = threading.local()   # armed: the model attention whose forward is running; pending: Pending
_stats = {k: 0 for k in ("pack", "redirect", "materialize", "fallback")}


def stats() -> dict[str, int]:
    return dict(_stats)


def _a2a(out: torch.Tensor, inp: torch.Tensor, group=None) -> None:  # noqa: ANN001
    """The collective, looked up at call time (the a2a timing wrapper patches ``dist.all_to_all_single``)."""
    dist.all_to_all_single(out, inp, group=group)


def send_shape(s_loc: int, heads: int, d: int, ws: int, groups: int) -> tuple[int, ...]:
    """[G, P, M, 3, hl, d]: per head group and destination rank, each token's q, k and v side by side (:74)."""
    return (groups, ws, s_loc, 3, heads // (groups * ws), d)


def dest_view(x: torch.Tensor, ws: int, groups: int) -> torch.Tensor:
    """[M, H, d] (any strides) seen as [G, P, M, hl, d]: head h = (g * P + p) * hl + j goes to rank p in group g."""
    return x.unflatten(1, (groups, ws, x.shape[1] // (groups * ws))).movedim(0, 2)


def fill_slot(send: torch.Tensor, x: torch.Tensor, slot: int, ws: int, groups: int) -> None:
    """Slot ``slot`` (0 q, 1 k, 2 v) of the combined send buffer from x [M, H, d]."""
    ops._need_cuda(send, x)
    send.select(3, slot).copy_(dest_view(x, ws, groups))


def pack_qkv(send: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, ws: int, groups: int) -> None:
    """The producer for q, k, v that come from elsewhere: all three slots of send [G, P, M, 3, hl, d] (:84)."""
    for slot, x in enumerate((q, k, v)):
        fill_slot(send, x, slot, ws, groups)


def _kernel_launch(x_block, weight, rope_table, eps, out) -> None:  # noqa: ANN001
    """One destination's heads [M, hl, d] normalised and rotated by the send kernel into ``out`` (a strided slot view)."""
    out.copy_(ops.norm_rope_send(x_block, weight, rope_table, eps, 1)[0])


def rope_into_send(send, q, k, q_weight, k_weight, rope_table, eps, ws, groups, launch=None) -> None:  # noqa: ANN001
    """Redirected producer (:93): norm + RoPE of the heads that go to each destination, written into slots 0 (q) and 1
    (k) of the combined send buffer [G, P, M, 3, hl, d]; ``launch(x_block, weight, rope_table, eps, out_view)`` per
    destination (default: the send kernel)."""
    launch = launch or _kernel_launch
    hl = send.shape[4]
    hg = hl * ws
    for g in range(groups):
        for p in range(ws):
            h0 = g * hg + p * hl
            launch(q[:, h0:h0 + hl], q_weight, rope_table, eps, send[g, p, :, 0])
            launch(k[:, h0:h0 + hl], k_weight, rope_table, eps, send[g, p, :, 1])


def qkv_views(recv_g: torch.Tensor, v_f16: bool = False):
    """recv [P, M, 3, hl, d] (contiguous) -> q, k, v strided views [1, P*M, hl, d] (row stride 3*hl*d); with
    ``v_f16`` the v slots hold f16 bits (the qkv epilogue's exact f16 copy of v) and v is viewed as f16."""
    p, m, _, hl, d = recv_g.shape
    flat = recv_g.view(p * m, 3, hl, d)
    v = flat[:, 2].view(torch.float16) if v_f16 else flat[:, 2]
    return flat[:, 0].unsqueeze(0), flat[:, 1].unsqueeze(0), v.unsqueeze(0)


def back_into(o: torch.Tensor, recv_b: torch.Tensor, result: torch.Tensor, g: int, ws: int, a2a, pg) -> None:  # noqa: ANN001
    """Attention output o [1, S, hl, d] of head group g -> result[0, :, g*hg:(g+1)*hg] with one a2a and one copy."""
    o3 = o[0] if o[0].is_contiguous() else o[0].contiguous()
    (a2a or _a2a)(recv_b, o3, group=pg)  # dim 0 of o3 is S: chunk p = the rows of rank p's sequence shard
    _, s_loc, hl, d = recv_b.shape
    hg = hl * ws
    if g == 0 and hg == result.shape[2]:
        ops.unpack_recv(recv_b, out=result[0])
    else:
        result[0, :, g * hg:(g + 1) * hg].unflatten(1, (ws, hl)).copy_(recv_b.permute(1, 0, 2, 3))


def local_attention(q, k, v, attn_metadata=None):  # noqa: ANN001,ANN201
    valid = None
    if attn_metadata is not None:
        valid = getattr(attn_metadata, "valid_kv_length", None)
    return torch.ops.h3b.flash_attn(q, k, v, None, valid)


class _GroupExchange:
    """The buffers of one combined-exchange forward and its three steps per head group g: ``arrive(g)`` (the forward
    exchange of send[g]), ``attend(g)`` (the local attention on the strided q/k/v views of recv[g]) and ``depart(g, o)``
    (the reverse exchange of its output into the result's head columns)."""

    def __init__(self, send: torch.Tensor, result_shape: tuple, run_attn, ws: int, pg, a2a, v_f16: bool):  # noqa: ANN001
        self.send, self.ws, self.pg, self.a2a, self.v_f16, self.run_attn = send, ws, pg, a2a, v_f16, run_attn
        groups, _, s_loc, _, hl, d = send.shape
        self.recv = torch.empty_like(send)
        self.recv_b = torch.empty((groups, ws, s_loc, hl, d), dtype=send.dtype, device=send.device)
        self.result = torch.empty(result_shape, dtype=send.dtype, device=send.device)

    def arrive(self, g: int) -> None:
        self.a2a(self.recv[g], self.send[g], group=self.pg)

    def attend(self, g: int) -> torch.Tensor:
        return self.run_attn(*qkv_views(self.recv[g], self.v_f16))

    def depart(self, g: int, o: torch.Tensor) -> None:
        back_into(o, self.recv_b[g], self.result, g, self.ws, self.a2a, self.pg)


def _event_after(stream, work, after=None) -> torch.cuda.Event:  # noqa: ANN001
    """Enqueue ``work()`` on ``stream`` (behind the event ``after`` when given); the event marks its end."""
    with torch.cuda.stream(stream):
        if after is not None:
            stream.wait_event(after)
        work()
        done = torch.cuda.Event()
        done.record(stream)
    return done


def nocopy_forward(query, key, value, run_attn, *, ws, groups, pg=None, a2a=None, send_box=None, comm=None,  # noqa: ANN001,ANN201
                   v_f16=False, v_in_box=False):
    """Strict Ulysses for batch 1 with one combined exchange per head group (:124).  ``send_box`` may hold a send
    buffer a producer already filled with q and k (v is then written here from ``value``), or with all three
    (``v_in_box``: the qkv GEMM's interleaved epilogue, ``fp8_gemm_qkv_send(..., interleaved=True)``, whose v slots
    hold f16 bits with ``v_f16``).  Without ``comm`` every step runs on the current stream, group after group, and the
    send buffer is released once the forward exchanges are enqueued.  With a ``comm`` stream all forward exchanges are
    queued there at once, group g's attention starts when its exchange has landed, and its reverse exchange goes back
    on ``comm`` while the next group's attention runs; every buffer was allocated on the current stream and stays
    referenced until the current stream has waited for the last reverse exchange.  Returns [1, M, H, d] contiguous."""
    _, s_loc, heads, d = query.shape
    if send_box:
        send = send_box.pop()
        if not v_in_box:
            fill_slot(send, value[0], 2, ws, groups)
    else:
        send = torch.empty(send_shape(s_loc, heads, d, ws, groups), dtype=query.dtype, device=query.device)
        pack_qkv(send, query[0], key[0], value[0], ws, groups)
    xch = _GroupExchange(send, (1, s_loc, heads, d), run_attn, ws, pg, a2a or _a2a, v_f16)
    del send
    if comm is None:
        for g in range(groups):
            xch.arrive(g)
        xch.send = None
        for g in range(groups):
            xch.depart(g, xch.attend(g))
        return xch.result
    cur = torch.cuda.current_stream()
    comm.wait_stream(cur)
    try:
        landed = [_event_after(comm, lambda g=g: xch.arrive(g)) for g in range(groups)]
        outs, returned = [], []
        for g in range(groups):
            cur.wait_event(landed[g])
            outs.append(xch.attend(g))          # read on comm below: referenced until the join
            computed = torch.cuda.Event()
            computed.record(cur)
            returned.append(_event_after(comm, lambda g=g: xch.depart(g, outs[g]), after=computed))
        for ev in returned:
            cur.wait_event(ev)
        return xch.result
    except Exception:
        cur.wait_stream(comm)
        raise


def eligible_shape(query, key, value, ws: int, groups: int) -> bool:  # noqa: ANN001
    """(:237)"""
    if query.ndim != 4 or key.shape != query.shape or value.shape != query.shape:
        return False
    if query.shape[0] != 1 or ws < 2 or groups < 1:
        return False
    if query.shape[2] % (groups * ws) != 0:
        return False
    return key.dtype == query.dtype == value.dtype and key.device == query.device == value.device


@dataclass
class Pending:
    """The combined send buffer a redirected producer filled with q and k (:190), and the placeholders the model
    holds in their place."""
    send: torch.Tensor   # [G, P, M, 3, hl, d], q in slot 0, k in slot 1, slot 2 filled by the exchange
    q_ph: torch.Tensor
    k_ph: torch.Tensor
    ws: int
    groups: int

    def matches(self, query: torch.Tensor, key: torch.Tensor) -> bool:
        return (query.ndim == 4 and query.data_ptr() == self.q_ph.data_ptr()
                and key.data_ptr() == self.k_ph.data_ptr() and tuple(query.shape[1:]) == tuple(self.q_ph.shape))

    def materialize(self):  # noqa: ANN201
        """Real q, k [1, M, H, d] from the send buffer (only when the consumer falls back to stock)."""
        _stats["materialize"] += 1
        out = []
        for slot in (0, 1):
            x = self.send[:, :, :, slot]                      # [G, P, M, hl, d]
            g, p, m, hl, d = x.shape
            out.append(x.permute(2, 0, 1, 3, 4).reshape(m, g * p * hl, d).unsqueeze(0))
        return out[0], out[1]


def _placeholder(like: torch.Tensor) -> torch.Tensor:
    return like.new_empty(1).as_strided(tuple(like.shape), (0,) * like.ndim)


def _is_placeholder(t: torch.Tensor) -> bool:
    return t.numel() > 1 and all(st == 0 for st in t.stride())


def take_pending(query: torch.Tensor, key: torch.Tensor) -> Pending | None:
    """This thread's pending send buffer if q/k are its placeholders (consumed), else None; placeholders without
    their buffer raise (:227)."""
    pend = getattr(_tls, "pending", None)
    if pend is not None and pend.matches(query, key):
        _tls.pending = None
        return pend
    if _is_placeholder(query) or _is_placeholder(key):
        raise RuntimeError("h3b nocopy: placeholder q/k reached attention without their send buffer")
    return None


def make_forward_impl(orig, groups: int, strategy_info, comm_stream=None, a2a=None, *, attn=None):  # noqa: ANN001,ANN201
    """Wrap ``Attention._forward_impl`` (:248): eligible strict-Ulysses calls run ``nocopy_forward`` with the B200
    attention (on the send buffer a redirected producer filled, when q/k are its placeholders); a placeholder call that
    is not eligible is materialised and, like anything else, runs ``orig``.  ``attn(q, k, v, attn_metadata)``
    defaults to ``local_attention``."""
    attn = attn or local_attention

    def _forward_impl(self, query, key, value, attn_metadata=None):  # noqa: ANN001
        pend = take_pending(query, key)
        info = strategy_info(self, attn_metadata)
        ok = info is not None and eligible_shape(query, key, value, info[1], groups)
        if pend is not None and (not ok or pend.ws != info[1] or pend.groups != groups):
            query, key = pend.materialize()
            pend = None
        if not ok:
            _stats["fallback"] += 1
            return orig(self, query, key, value, attn_metadata)
        pg, ws = info
        box = None
        if pend is not None:
            box, pend.send = [pend.send], None
            _stats["redirect"] += 1
        else:
            _stats["pack"] += 1
        comm = comm_stream(query.device) if (groups > 1 and comm_stream is not None and query.is_cuda) else None
        return nocopy_forward(query, key, value, lambda q, k, v: attn(q, k, v, attn_metadata), ws=ws, groups=groups,
                              pg=pg, a2a=a2a, send_box=box, comm=comm)

    return _forward_impl


def make_rope(orig, groups: int, strategy_info, launch=None, supported=None):  # noqa: ANN001,ANN201
    """Wrap the transformer's ``fused_qk_norm_rope`` (:282): while a model attention forward is armed and its attention
    would take the combined exchange, q/k go normalised and rotated into a fresh send buffer and placeholders come
    back; anything else runs the stock function.  ``launch`` / ``supported``: the per-destination launcher and its
    guard (default: the send kernel and ``ulysses_exact.rope_supported``)."""
    from .ulysses_exact import rope_supported  # noqa: PLC0415
    supported = supported or rope_supported

    def fused_qk_norm_rope(q, k, q_weight, k_weight, rope_table, eps, *, head_dim=None, rotary_dim=None,  # noqa: ANN001,ANN202
                           interleaved=False):
        owner = getattr(_tls, "armed", None)
        _tls.armed = None                        # one redirect per armed forward
        info = None
        if owner is not None and getattr(owner, "to_gate_compress", None) is None:
            info = strategy_info(owner.attention, None)
        if (info is None or q.ndim != 3 or q.shape != k.shape or q.shape[0] == 0
                or head_dim not in (None, q.shape[-1]) or rotary_dim not in (None, rope_table.shape[-1])
                or rope_table.shape != (q.shape[0], rope_table.shape[-1])
                or not eligible_shape(q.unsqueeze(0), k.unsqueeze(0), k.unsqueeze(0), info[1], groups)
                or not supported(q, k, rope_table, interleaved)):
            return orig(q, k, q_weight, k_weight, rope_table, eps, head_dim=head_dim, rotary_dim=rotary_dim,
                        interleaved=interleaved)
        ws = info[1]
        m, heads, d = q.shape
        send = torch.empty(send_shape(m, heads, d, ws, groups), dtype=q.dtype, device=q.device)
        rope_into_send(send, q, k, q_weight.contiguous(), k_weight.contiguous(), rope_table.contiguous(), eps, ws,
                       groups, launch)
        _tls.pending = Pending(send=send, q_ph=_placeholder(q), k_ph=_placeholder(k), ws=ws, groups=groups)
        return _tls.pending.q_ph, _tls.pending.k_ph

    fused_qk_norm_rope._h3b_nocopy = True
    return fused_qk_norm_rope


class _Armed:
    """While a model attention's forward runs, the rope wrapper redirects q/k for that attention (``_tls.armed``).  On
    leaving, the previous owner comes back and a send buffer the forward made but did not use is dropped."""

    def __init__(self, owner):  # noqa: ANN001
        self.owner, self.prev = owner, None

    def __enter__(self) -> None:
        self.prev, _tls.armed = getattr(_tls, "armed", None), self.owner

    def __exit__(self, *exc) -> None:  # noqa: ANN002
        _tls.armed, _tls.pending = self.prev, None


def make_armed_forward(orig_fwd):  # noqa: ANN001,ANN201
    """The model attention's ``forward`` with its redirect armed (:316)."""
    def forward(self, *a, **kw):  # noqa: ANN001,ANN202
        with _Armed(self):
            return orig_fwd(self, *a, **kw)

    forward._h3b_nocopy_armed = True
    return forward


def _install_on(cls, tr, groups: int, strategy_info, comm_stream=None, *, launch=None, supported=None) -> None:  # noqa: ANN001
    """Wrap ``cls._forward_impl`` and redirect ``tr``'s producer (:415): ``tr.fused_qk_norm_rope`` writes into the send
    buffer while ``tr.MiniMaxH3Attention.forward`` is armed.  Refuses beside the grouped overlap (nocopy replaces it)
    and a second install with other ``groups``."""
    if getattr(cls, "_h3b_overlap", 0):
        raise RuntimeError("h3b: the Ulysses overlap is installed; nocopy replaces it (install only one)")
    prev = getattr(cls, "_h3b_nocopy", 0)
    if prev:
        if prev != groups:
            raise RuntimeError(f"h3b nocopy already installed with groups={prev}, cannot change to {groups}")
        return
    cls._forward_impl = make_forward_impl(cls._forward_impl, groups, strategy_info, comm_stream)
    cls._h3b_nocopy = groups
    if tr is None:
        return
    if not getattr(tr.fused_qk_norm_rope, "_h3b_nocopy", False):
        tr.fused_qk_norm_rope = make_rope(tr.fused_qk_norm_rope, groups, strategy_info, launch, supported)
    att_cls = tr.MiniMaxH3Attention
    if not getattr(att_cls.forward, "_h3b_nocopy_armed", False):
        att_cls.forward = make_armed_forward(att_cls.forward)


def install(groups: int = 1) -> None:
    """Wrap vLLM-Omni's ``Attention._forward_impl`` and the MiniMax H3 producer (:415); needs vLLM-Omni."""
    try:
        from vllm_omni.diffusion.attention import layer as layer_mod  # noqa: PLC0415
        from vllm_omni.diffusion.models.minimax_h3 import minimax_h3_transformer as tr  # noqa: PLC0415
    except ImportError as exc:  # pragma: no cover - vLLM-Omni is not part of this image
        raise RuntimeError("h3b.ulysses_nocopy.install needs vLLM-Omni (not installed)") from exc
    from .plugin import vllm_strategy_info  # noqa: PLC0415
    from .ulysses_overlap import comm_stream  # noqa: PLC0415
    _install_on(layer_mod.Attention, tr, groups, vllm_strategy_info, comm_stream if groups > 1 else None)
