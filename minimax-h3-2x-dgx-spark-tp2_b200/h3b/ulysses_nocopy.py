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

import torch
import torch.distributed as dist

from . import ops


def _a2a(out: torch.Tensor, inp: torch.Tensor, group=None) -> None:  # noqa: ANN001
    dist.all_to_all_single(out, inp, group=group)


def send_shape(s_loc: int, heads: int, d: int, ws: int, groups: int) -> tuple[int, ...]:
    return (groups, ws, s_loc, 3, heads // (groups * ws), d)


def _by_dest(x: torch.Tensor, ws: int, groups: int) -> torch.Tensor:
    """[M, H, d] (any strides) -> view [G, P, M, hl, d]; head h = g*hg + p*hl + j."""
    m, h, d = x.shape
    return x.unflatten(1, (groups, ws, h // (groups * ws))).permute(1, 2, 0, 3, 4)


def pack_qkv(send: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, ws: int, groups: int) -> None:
    """Fallback producer: q, k, v [M, H, d] -> send [G, P, M, 3, hl, d] in one stack (:84)."""
    ops._need_cuda(send, q, k, v)
    torch.stack((_by_dest(q, ws, groups), _by_dest(k, ws, groups), _by_dest(v, ws, groups)), dim=3, out=send)


def fill_slot(send: torch.Tensor, x: torch.Tensor, slot: int, ws: int, groups: int) -> None:
    ops._need_cuda(send, x)
    send[:, :, :, slot].copy_(_by_dest(x, ws, groups))


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
    return ops.flash_attn(q, k, v, valid_kv=valid)


def nocopy_forward(query, key, value, run_attn, *, ws, groups, pg=None, a2a=None, send_box=None, comm=None,  # noqa: ANN001,ANN201
                   v_f16=False):
    """Strict Ulysses for batch 1 with one combined exchange per head group (:124).  ``send_box`` may hold a send
    buffer a producer already filled (``fp8_gemm_qkv_send(..., interleaved=True)``); ``comm``: a stream on which the
    exchanges overlap the attention of earlier groups.  Returns [1, M, H, d] contiguous."""
    a2a = a2a or _a2a
    _, s_loc, heads, d = query.shape
    dt, dev = query.dtype, query.device
    if send_box:
        send = send_box.pop()
    else:
        send = torch.empty(send_shape(s_loc, heads, d, ws, groups), dtype=dt, device=dev)
        pack_qkv(send, query[0], key[0], value[0], ws, groups)
    hl = send.shape[4]
    recv = torch.empty_like(send)
    recv_b = torch.empty((groups, ws, s_loc, hl, d), dtype=dt, device=dev)
    result = torch.empty((1, s_loc, heads, d), dtype=dt, device=dev)
    if comm is None:
        for g in range(groups):
            a2a(recv[g], send[g], group=pg)
        del send
        for g in range(groups):
            o = run_attn(*qkv_views(recv[g], v_f16))
            back_into(o, recv_b[g], result, g, ws, a2a, pg)
        return result
    cur = torch.cuda.current_stream()
    comm.wait_stream(cur)
    try:
        ready = []
        with torch.cuda.stream(comm):
            for g in range(groups):
                a2a(recv[g], send[g], group=pg)
                ev = torch.cuda.Event()
                ev.record(comm)
                ready.append(ev)
        outs, back_ev = [], []
        for g in range(groups):
            cur.wait_event(ready[g])
            o = run_attn(*qkv_views(recv[g], v_f16))
            outs.append(o)
            done = torch.cuda.Event()
            done.record(cur)
            with torch.cuda.stream(comm):
                comm.wait_event(done)
                back_into(o, recv_b[g], result, g, ws, a2a, pg)
                ev = torch.cuda.Event()
                ev.record(comm)
            back_ev.append(ev)
        for ev in back_ev:
            cur.wait_event(ev)
        return result
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


def make_forward_impl(orig, groups: int, strategy_info, comm_stream=None, a2a=None):  # noqa: ANN001,ANN201
    """Wrap ``Attention._forward_impl`` (:248): eligible strict-Ulysses calls run ``nocopy_forward`` with the B200
    attention, anything else ``orig``."""

    def _forward_impl(self, query, key, value, attn_metadata=None):  # noqa: ANN001
        info = strategy_info(self, attn_metadata)
        if info is None or not eligible_shape(query, key, value, info[1], groups):
            return orig(self, query, key, value, attn_metadata)
        pg, ws = info
        return nocopy_forward(query, key, value, lambda q, k, v: local_attention(q, k, v, attn_metadata), ws=ws,
                              groups=groups, pg=pg, a2a=a2a, comm=comm_stream(query.device) if comm_stream else None)

    return _forward_impl


def install(groups: int = 1) -> None:
    """Wrap vLLM-Omni's ``Attention._forward_impl`` (:415); needs vLLM-Omni."""
    try:
        from vllm_omni.diffusion.attention import layer as layer_mod  # noqa: PLC0415
    except ImportError as exc:  # pragma: no cover - vLLM-Omni is not part of this image
        raise RuntimeError("h3b.ulysses_nocopy.install needs vLLM-Omni (not installed)") from exc
    from .plugin import vllm_strategy_info  # noqa: PLC0415
    from .ulysses_overlap import comm_stream  # noqa: PLC0415
    cls = layer_mod.Attention
    if getattr(cls, "_h3b_nocopy", None):
        return
    cls._forward_impl = make_forward_impl(cls._forward_impl, groups, vllm_strategy_info,
                                          comm_stream if groups > 1 else None)
    cls._h3b_nocopy = groups
