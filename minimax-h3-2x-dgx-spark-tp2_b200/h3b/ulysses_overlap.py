"""Ulysses all-to-alls overlapped with attention by head group (mirrors ``h3_tp2/ulysses_overlap.py``).

The local heads are split into G groups.  Every group's three forward all-to-alls go to a communication stream
(high priority, so NCCL's kernels are scheduled ahead of the attention's next CTAs), attention of group g runs on the
compute stream as soon as its receives land, and its reverse all-to-all is issued on the communication stream right
after.  Every byte still moves and every head is computed by the same kernel on the same keys in the same order, so
the result is bit-identical to the ungrouped exchange (tested).

Memory rule (as the reference's, ``h3_tp2/ulysses_overlap.py:101-108``): every buffer one stream writes and the other
reads is allocated on the compute stream and never ``record_stream``-ed; the compute stream waits for every
communication event before the function returns.

With the fused producer (``ops.fp8_gemm_qkv_send(..., groups=G)``) the send buffers are already group-major
[G, P, M, hgl, d] and the reverse receive buffer [G, P, M, hgl, d] is quantised by the out-projection directly
(``ops.quant_rows`` over G*P segments), so no pack or unpack copy exists.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from . import ops

_comm_streams: dict = {}


def comm_stream(device: torch.device) -> torch.cuda.Stream:
    """The communication stream of ``device`` (priority from ``H3_TP2_A2A_STREAM_PRIORITY``, default -1 = high)."""
    key = device.index if device.index is not None else torch.cuda.current_device()
    s = _comm_streams.get(key)
    if s is None:
        prio = int(os.environ.get("H3_TP2_A2A_STREAM_PRIORITY", "-1").strip() or -1)
        s = torch.cuda.Stream(device=device, priority=prio)
        _comm_streams[key] = s
    return s


def _a2a(out: torch.Tensor, inp: torch.Tensor, group=None) -> None:  # noqa: ANN001
    dist.all_to_all_single(out, inp, group=group)


def default_groups(heads: int, ws: int) -> int:
    """1: measured on B200 at SP=2 (cfg2), the ungrouped exchange is faster (150.1 ms per block, 3.1 % exposed
    all-to-all) than 2 or 4 head groups (153.1 ms: the per-group attention launches add wave tails and NCCL's kernels
    take SMs from the attention).  Grouping stays available through ``groups=`` / ``H3_TP2_A2A_OVERLAP``."""
    del heads, ws
    return 1


def grouped_attention(sends, ws: int, groups: int, attn, pg=None, a2a=None, marks=None) -> torch.Tensor:  # noqa: ANN001
    """sends: q, k, v send buffers [G, P, M, hgl, d] (q/k bf16, v bf16 or f16).  Runs the grouped forward exchange,
    ``attn(q, k, v)`` per group on [P*M, hgl, d] receive views, and the grouped reverse exchange; returns the reverse
    receive buffer [G, P, M, hgl, d] (row m of the out-projection input = concat over (g, p) of buf[g, p, m])."""
    a2a = a2a or _a2a
    G, P, M, hgl, d = sends[0].shape
    cur = torch.cuda.current_stream()
    comm = comm_stream(sends[0].device)
    recvs = [torch.empty_like(s) for s in sends]                      # compute-stream allocations
    back = torch.empty((G, P, M, hgl, d), dtype=torch.bfloat16, device=sends[0].device)
    outs = []
    comm.wait_stream(cur)
    ready = []
    with torch.cuda.stream(comm):
        for g in range(G):
            for t in range(3):
                a2a(recvs[t][g], sends[t][g], group=pg)
            ev = torch.cuda.Event()
            ev.record(comm)
            ready.append(ev)
    back_ev = []
    for g in range(G):
        cur.wait_event(ready[g])
        o = attn(*(r[g].view(P * M, hgl, d) for r in recvs))
        outs.append(o)                                               # alive until the comm stream is done with it
        done = torch.cuda.Event()
        done.record(cur)
        with torch.cuda.stream(comm):
            comm.wait_event(done)
            a2a(back[g], o.view(P, M, hgl, d), group=pg)
            ev = torch.cuda.Event()
            ev.record(comm)
        back_ev.append(ev)
    for ev in back_ev:
        cur.wait_event(ev)
    return back


def quant_grouped_back(back: torch.Tensor, div_mode: int = ops.DIV_IEEE):
    """The out-projection quant straight from the grouped reverse receive buffer [G, P, M, hgl, d]."""
    G, P, M, hgl, d = back.shape
    seg = hgl * d
    return torch.ops.h3b.quant_rows(back, M, G * P, seg, M * seg, seg, div_mode)


def _a2a_seq_to_heads(x: torch.Tensor, ws: int, pg, recv: torch.Tensor, a2a=None) -> torch.Tensor:  # noqa: ANN001
    """(1, S/P, hg, D) view -> (1, S, hg/P, D): the bytes all_to_all_4D(scatter 2, gather 1) moves
    (h3_tp2/ulysses_overlap.py:27); the pack is the CUDA layout kernel."""
    send = ops.pack_by_dest(x[0], ws)
    (a2a or _a2a)(recv, send, group=pg)
    p, m, hl, d = recv.shape
    return recv.view(1, p * m, hl, d)


def grouped_forward(query, key, value, run_attn, *, ws: int, groups: int, pg=None, a2a=None):  # noqa: ANN001,ANN201
    """Stock-layout entry (q/k/v [1, M, H, d] as the attention layer receives them): head group g's q/k/v are packed
    and exchanged on the communication stream, attention and reverse exchange overlap as above.  Returns
    [1, M, H, d] bf16 (h3_tp2/ulysses_overlap.py:116-159)."""
    _, m, heads, d = query.shape
    hg = heads // groups
    cur = torch.cuda.current_stream()
    comm = comm_stream(query.device)
    comm.wait_stream(cur)
    sends = []
    with torch.cuda.stream(comm):
        for t in (query, key, value):
            s = torch.empty((groups, ws, m, hg // ws, d), dtype=t.dtype, device=t.device)
            for g in range(groups):
                ops.pack_by_dest(t[0, :, g * hg:(g + 1) * hg], ws, out=s[g])
            sends.append(s)
    cur.wait_stream(comm)
    back = grouped_attention(sends, ws, groups, lambda q, k, v: run_attn(q.unsqueeze(0), k.unsqueeze(0),
                                                                         v.unsqueeze(0))[0], pg=pg, a2a=a2a)
    G, P, M, hgl, dd = back.shape
    # [G, P, M, hgl, d] -> [1, M, G*P*hgl, d]: head order g, p, j = the original head order
    return back.permute(2, 0, 1, 3, 4).reshape(1, M, G * P * hgl, dd).contiguous()


def install(groups: int) -> None:
    """Wrap vLLM-Omni's ``Attention._forward_impl`` with the grouped forward (h3_tp2/ulysses_overlap.py:50); needs
    vLLM-Omni (not part of this image)."""
    try:
        from vllm_omni.diffusion.attention import layer as layer_mod  # noqa: PLC0415
    except ImportError as exc:  # pragma: no cover
        raise RuntimeError("h3b.ulysses_overlap.install needs vLLM-Omni (not installed)") from exc
    from .plugin import vllm_strategy_info  # noqa: PLC0415
    from .ulysses_exact import local_attention  # noqa: PLC0415

    cls = layer_mod.Attention
    prev = getattr(cls, "_h3b_overlap", 0)
    if prev:
        if prev != groups:
            raise RuntimeError(f"h3b overlap already installed with groups={prev}, cannot change to {groups}")
        return
    orig = cls._forward_impl

    def _forward_impl(self, query, key, value, attn_metadata=None):  # noqa: ANN001
        info = vllm_strategy_info(self, attn_metadata)
        if (info is None or query.ndim != 4 or query.shape[0] != 1 or not (query.is_cuda and key.is_cuda and value.is_cuda)
                or key.shape != query.shape or value.shape != query.shape or query.shape[2] % (groups * info[1])):
            return orig(self, query, key, value, attn_metadata)
        pg, ws = info
        return grouped_forward(query, key, value, lambda q, k, v: local_attention(q, k, v, attn_metadata), ws=ws,
                               groups=groups, pg=pg)

    cls._forward_impl = _forward_impl
    cls._h3b_overlap = groups
