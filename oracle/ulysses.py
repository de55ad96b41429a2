"""Ulysses sequence<->head exchange layouts, restated from the reference's stock oracle and exact path.

Reference: the stock ``all_to_all_4D`` (vLLM-Omni ``comm.py:36-98``) as the reference reproduces it in
``tests/test_ulysses_exact.py:74-99`` (``stock_all_to_all_4d``), the exact path's send layout
``h3_tp2/ulysses_exact.py:108-127`` (``send_shape`` / ``by_dest`` / ``pack_into`` / ``unpack``), the forward
exchange ``:130-135`` and the reverse exchange + unpack ``:156-184``.  ``FakeA2A`` emulates
``all_to_all_single`` over threads with equal dim-0 splits, as ``tests/test_ulysses_exact.py:25-50`` does.
"""
from __future__ import annotations

import threading

import torch


def send_shape(m: int, heads: int, d: int, ws: int) -> tuple[int, int, int, int]:
    return (ws, m, heads // ws, d)


def pack(x: torch.Tensor, ws: int) -> torch.Tensor:
    """[M, H, d] -> contiguous [P, M, H/P, d]; head h = p*(H/P) + j goes to rank p."""
    m, h, d = x.shape
    return x.reshape(m, ws, h // ws, d).permute(1, 0, 2, 3).contiguous()


def unpack(send: torch.Tensor) -> torch.Tensor:
    """[P, M, hl, d] -> contiguous [M, P*hl, d]."""
    p, m, hl, d = send.shape
    return send.permute(1, 0, 2, 3).reshape(m, p * hl, d).contiguous()


def a2a_reference(sends: list[torch.Tensor]) -> list[torch.Tensor]:
    """all_to_all_single with equal dim-0 splits over ranks given all ranks' send buffers: rank r receives the r-th
    dim-0 chunk of every source, in source order."""
    ws = len(sends)
    return [torch.cat([sends[s].reshape(-1).chunk(ws)[r] for s in range(ws)]).view(sends[r].shape) for r in range(ws)]


def stock_all_to_all_4d(x: torch.Tensor, scatter_idx: int, gather_idx: int, ws: int, a2a) -> torch.Tensor:
    """Stock strict Ulysses exchange at any batch; ``a2a(out, inp)`` is the collective."""
    if scatter_idx == 2 and gather_idx == 1:
        bs, s_loc, hc, hs = x.shape
        inp = x.reshape(bs, s_loc, ws, hc // ws, hs).permute(2, 1, 0, 3, 4).contiguous()   # [P, S/P, B, hc/P, hs]
        out = torch.empty_like(inp)
        a2a(out, inp)
        return out.reshape(s_loc * ws, bs, hc // ws, hs).permute(1, 0, 2, 3).contiguous()
    bs, seq, shc, hs = x.shape
    s_loc = seq // ws
    inp = x.reshape(bs, ws, s_loc, shc, hs).permute(1, 3, 2, 0, 4).contiguous()           # [P, shc, S/P, B, hs]
    out = torch.empty_like(inp)
    a2a(out, inp)
    return out.reshape(shc * ws, s_loc, bs, hs).permute(2, 1, 0, 3).contiguous()


class FakeA2A:
    """``all_to_all_single`` over ``ws`` threads (one per rank), equal dim-0 splits, contiguous buffers."""

    def __init__(self, ws: int):
        self.ws = ws
        self.barrier = threading.Barrier(ws, timeout=60)
        self.slots: list = [None] * ws

    def bind(self, rank: int):
        def a2a(out, inp, group=None):  # noqa: ARG001
            assert out.is_contiguous() and inp.is_contiguous() and out.numel() == inp.numel()
            assert inp.shape[0] % self.ws == 0
            self.slots[rank] = inp
            self.barrier.wait()
            out.view(-1).copy_(torch.cat([self.slots[s].reshape(-1).chunk(self.ws)[rank] for s in range(self.ws)]))
            self.barrier.wait()
        return a2a


def run_ranks(fn, ws: int):
    """Run ``fn(rank, a2a)`` on ``ws`` threads sharing one FakeA2A; returns the per-rank results."""
    fake = FakeA2A(ws)
    res, err = [None] * ws, [None] * ws

    def body(r):
        try:
            res[r] = fn(r, fake.bind(r))
        except BaseException as e:  # noqa: BLE001
            err[r] = e
            fake.barrier.abort()

    ts = [threading.Thread(target=body, args=(r,)) for r in range(ws)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    for e in err:
        if e is not None and not isinstance(e, threading.BrokenBarrierError):
            raise e
    for e in err:
        if e is not None:
            raise e
    return res


def norm_rope(x: torch.Tensor, w: torch.Tensor, table: torch.Tensor, eps: float) -> torch.Tensor:
    """Per-(token, head) RMSNorm over head_dim then partial RoPE, as the reference's eager stand-in for the upstream
    ``_rms_norm_rope_kernel`` (``tests/test_ulysses_exact.py:107-116``): x [M, H, d] bf16, w [d], table [M, R] fp32
    holding cos[:R/2] | sin[R/2:]; n = bf16(x * rsqrt(mean(x^2) + eps) * w); the first R dims rotate in half-split
    pairs (a, b) = (n[i], n[i + R/2]) -> (a cos - b sin, b cos + a sin); the rest pass; result bf16."""
    xf = x.float()
    inv = torch.rsqrt((xf * xf).sum(-1, keepdim=True) / x.shape[-1] + eps)
    n = (xf * inv * w.float()).to(torch.bfloat16).float()
    half = table.shape[-1] // 2
    cos, sin = table[:, None, :half].float(), table[:, None, half:].float()
    a, b = n[..., :half], n[..., half:2 * half]
    return torch.cat((a * cos - b * sin, b * cos + a * sin, n[..., 2 * half:]), dim=-1).to(x.dtype)


def norm_rope_into_send(x: torch.Tensor, w: torch.Tensor, table: torch.Tensor, eps: float, ws: int) -> torch.Tensor:
    """``ulysses_exact.rope_into_send`` (h3_tp2/ulysses_exact.py:264-271) with the eager producer: the normed and
    rotated q (or k) of each destination's heads written into send [P, M, H/P, d]."""
    return pack(norm_rope(x, w, table, eps), ws)


# ---- the combined q/k/v exchange (h3_tp2/ulysses_nocopy.py:74-189) -------------------------------------------------

def nocopy_send_shape(m: int, heads: int, d: int, ws: int, groups: int) -> tuple[int, ...]:
    """[G, P, M, 3, H/(G*P), d] (h3_tp2/ulysses_nocopy.py:74)."""
    return (groups, ws, m, 3, heads // (groups * ws), d)


def pack_qkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, ws: int, groups: int) -> torch.Tensor:
    """q, k, v [M, H, d] -> contiguous [G, P, M, 3, hl, d]; head h = g*(H/G) + p*hl + j (:78-87)."""
    m, h, d = q.shape
    hl = h // (groups * ws)

    def by_dest(x):
        return x.reshape(m, groups, ws, hl, d).permute(1, 2, 0, 3, 4)
    return torch.stack((by_dest(q), by_dest(k), by_dest(v)), dim=3).contiguous()


def qkv_views(recv_g: torch.Tensor):
    """recv [P, M, 3, hl, d] of one group -> q, k, v views [1, P*M, hl, d] with row stride 3*hl*d (:105-109)."""
    p, m, _, hl, d = recv_g.shape
    flat = recv_g.reshape(p * m, 3, hl, d)
    return flat[:, 0].unsqueeze(0), flat[:, 1].unsqueeze(0), flat[:, 2].unsqueeze(0)


def nocopy_forward(q, k, v, attn, *, ws: int, groups: int, a2a) -> torch.Tensor:
    """One rank of the combined exchange (:124-160, same stream): pack, one a2a per group, attention on the strided
    views, the output's rows back with one a2a per group, unpacked into [1, M, H, d]."""
    _, m, heads, d = q.shape
    send = pack_qkv(q[0], k[0], v[0], ws, groups)
    hl = send.shape[4]
    hg = hl * ws
    recv = torch.empty_like(send)
    for g in range(groups):
        a2a(recv[g], send[g])
    result = torch.empty((1, m, heads, d), dtype=q.dtype)
    for g in range(groups):
        o = attn(*qkv_views(recv[g]))[0].contiguous()
        recv_b = torch.empty((ws, m, hl, d), dtype=q.dtype)
        a2a(recv_b, o)
        result[0, :, g * hg:(g + 1) * hg] = recv_b.permute(1, 0, 2, 3).reshape(m, hg, d)
    return result
