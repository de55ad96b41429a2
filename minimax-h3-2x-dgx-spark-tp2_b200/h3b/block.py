"""The DiT attention block of the hot path, built from the h3b kernels (one rank of a Ulysses group).

    x [M, C] bf16 (this rank's sequence rows)
      -> per-token e4m3 quant                                  (ops.quant; fp8_quant_fuse qkv site)
      -> qkv FP8 GEMM, epilogue writes q, k, v straight into the send buffers [P, M, H/P, d]
         (v as f16, exactly converted from its bf16 value, for the f16 P.V product)
      -> seq->head all-to-all x3 (NCCL over NVLink; skipped at P = 1)
      -> flash attention over all P*M tokens for H/P heads     (tcgen05, non-causal, d = 128)
      -> head->seq all-to-all of the output as is (skipped at P = 1)
      -> per-token quant straight from the receive buffer      (ulysses_outq: no unpack copy)
      -> out FP8 GEMM -> y [M, C] bf16
This is the reference's ``ULYSSES_EXACT=2`` + ``FP8_GEMM`` + quant-fuse data flow (h3_tp2/ulysses_exact.py:187-220,
h3_tp2/ulysses_outq.py:138, h3_tp2/fp8_gemm.py:149) with the pack copies moved into the GEMM epilogue.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from . import ops

FP8_MAX = 448.0
MIN_SCALE = 1.0 / (FP8_MAX * 512.0)


def quant_weight(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Online per-output-channel e4m3 weight quant (load time, not the hot path): sb = max(absmax/448, 1/229376)."""
    wf = w.float()
    sb = torch.clamp(wf.abs().amax(dim=1) / FP8_MAX, min=MIN_SCALE)
    w8 = torch.clamp(wf / sb[:, None], -FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return w8.contiguous(), sb.contiguous()


def block_flops(tokens: int, hidden: int, heads: int, head_dim: int = 128) -> dict:
    hd = heads * head_dim
    return {"attention": 4.0 * tokens * tokens * head_dim * heads,
            "qkv": 2.0 * tokens * hidden * 3 * hd,
            "out": 2.0 * tokens * hd * hidden}


class AttentionBlock:
    def __init__(self, hidden: int, heads: int, *, device, head_dim: int = 128, seed: int = 1, ws: int = 1, pg=None,
                 weights: tuple | None = None, init_device=None, a2a=None, groups: int | None = None,
                 exchange: str = "nccl", rank: int | None = None, range_check: bool = False):
        if head_dim != 128:
            raise ValueError("head_dim 128 only")
        if heads % ws:
            raise ValueError(f"heads {heads} not divisible by the Ulysses degree {ws}")
        self.hidden, self.heads, self.head_dim, self.ws, self.pg = hidden, heads, head_dim, ws, pg
        self.device = torch.device(device)
        if weights is None:
            gdev = torch.device(init_device) if init_device is not None else torch.device("cpu")
            g = torch.Generator(device=gdev).manual_seed(seed)
            wqkv = torch.randn(3 * heads * head_dim, hidden, generator=g, device=gdev) * 0.02
            wo = torch.randn(hidden, heads * head_dim, generator=g, device=gdev) * 0.02
            weights = (*quant_weight(wqkv), *quant_weight(wo))
        self.wqkv8, self.sqkv, self.wo8, self.so = (t.to(self.device) for t in weights)
        self.range_flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.a2a = a2a   # injected collective a2a(out, inp, group=None); default: NCCL all_to_all_single
        from .ulysses_overlap import default_groups
        self.groups = default_groups(heads, ws) if groups is None else int(groups)
        if heads % (self.groups * ws):
            raise ValueError(f"heads {heads} not divisible by groups {self.groups} x ws {ws}")
        # "nccl": the all-to-alls as collectives (stock's exchange); "nocopy": one combined q/k/v collective per head
        # group on the interleaved layout (h3b.ulysses_nocopy); "p2p": stored by the kernels into the peers' receive
        # buffers (h3b.ulysses_p2p), no collective on the data path
        if exchange not in ("nccl", "nocopy", "p2p"):
            raise ValueError(f"exchange {exchange!r}: 'nccl', 'nocopy' or 'p2p'")
        if exchange == "p2p" and self.groups != 1:
            raise ValueError("exchange 'p2p' has no head groups")
        self.exchange_kind = exchange
        self.rank = rank if rank is not None else (dist.get_rank(pg) if exchange == "p2p" and ws > 1 else 0)
        self._peers = None
        # v travels as f16 for the f16 P.V product.  With ``range_check`` a v outside f16's range (|v| > 65504) is
        # caught after the qkv projection (one host read of the group-wide flag per forward), and the block then
        # switches to bf16 v and bf16 P.V for good and recomputes the projection.  The read waits for the copy
        # engine, so a large device-to-host copy in flight on another stream delays the rest of the forward (11 ms
        # per block measured with the bench's overlapped output copies): it is off by default, and without it the
        # attention refuses f16 P.V on such a v (H3B_ERANGE in the device status word, output unwritten).
        self.range_check = range_check
        self.v_f16 = True

    def _peer_exchange(self, m: int):
        from .ulysses_p2p import PeerExchange
        if self._peers is None or self._peers.m != m or self._peers.v_f16 != self.v_f16:
            if self._peers is not None:
                self.close()
            self._peers = PeerExchange(m, self.heads, self.ws, self.rank, self.device, pg=self.pg,
                                       v_f16=self.v_f16)
        return self._peers

    def _v_overflowed(self, flag: torch.Tensor) -> bool:
        """True when the qkv projection just written left f16's range in some v (``flag``: the group-wide flag).  The
        block then switches to bf16 v for good; the caller recomputes the projection."""
        if not (self.v_f16 and self.range_check) or not bool(flag.item()):
            return False
        self.v_f16 = False
        flag.zero_()
        return True

    def close(self) -> None:
        """Releases the peer buffers of the p2p exchange (collective over the group)."""
        if self._peers is not None:
            pg = self.pg
            self._peers.close(host_barrier=lambda: dist.barrier(group=pg))
            self._peers = None

    def share_range_flag(self) -> None:
        """Max of the v-overflow flags of all ranks (a rank's flag covers only the v slabs it sent, while its attention
        reads the slabs every rank sent), through the same all-to-all the exchange uses."""
        if self.ws == 1:
            return
        recv = self.exchange(self.range_flag.repeat(self.ws))
        torch.amax(recv, dim=0, keepdim=True, out=self.range_flag)

    def exchange(self, send: torch.Tensor) -> torch.Tensor:
        if self.ws == 1:
            return send
        recv = torch.empty_like(send)
        self.exchange_into(recv, send)
        return recv

    def exchange_into(self, recv: torch.Tensor, send: torch.Tensor) -> None:
        if self.a2a is not None:
            self.a2a(recv, send, group=self.pg)
        else:
            dist.all_to_all_single(recv, send, group=self.pg)

    STAGES = ("quant_x", "qkv_gemm", "a2a_fwd", "attention", "a2a_back", "quant_out", "out_gemm")

    def forward(self, x: torch.Tensor, marks: list | None = None) -> torch.Tensor:
        """x [M, C] bf16 -> y [M, C] bf16.  ``marks``: if a list, a CUDA event is recorded on the current stream
        after each stage (``STAGES``), preceded by one at the start, for per-stage device timing."""
        def mark():
            if marks is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                marks.append(ev)

        m = x.shape[0]
        hl, d = self.heads // self.ws, self.head_dim
        mark()
        q8, sx = ops.quant(x)
        mark()
        if self.ws > 1 and self.exchange_kind == "p2p":
            px = self._peer_exchange(m)
            px.forward_qkv(q8, self.wqkv8, sx, self.sqkv)
            mark()
            px.barrier()
            if self._v_overflowed(px.range_flag):  # every rank saw the same flag (raised on all ranks)
                px = self._peer_exchange(m)         # rebuilt with bf16 v (collective)
                px.forward_qkv(q8, self.wqkv8, sx, self.sqkv)
                px.barrier()
            mark()
            px.attention(1.0 / math.sqrt(d))
            mark()
            px.barrier()
            mark()
            o8, so = ops.quant_from_recv(px.back)
        elif self.ws > 1 and self.exchange_kind == "nocopy":
            from .ulysses_nocopy import qkv_views
            from .ulysses_overlap import quant_grouped_back
            G = self.groups
            send = ops.fp8_gemm_qkv_send(q8, self.wqkv8, sx, self.sqkv, self.heads, self.ws, v_f16=self.v_f16,
                                         range_flag=self.range_flag, groups=G, interleaved=True)
            self.share_range_flag()
            if self._v_overflowed(self.range_flag):
                send = ops.fp8_gemm_qkv_send(q8, self.wqkv8, sx, self.sqkv, self.heads, self.ws, v_f16=False,
                                             groups=G, interleaved=True)
            mark()
            recv = torch.empty_like(send)
            for g in range(G):
                self.exchange_into(recv[g], send[g])
            mark()
            hgl = self.heads // (G * self.ws)
            outs = [ops.flash_attn(*qkv_views(recv[g], v_f16=self.v_f16), scale=1.0 / math.sqrt(d),
                                   range_flag=self.range_flag, pv_f16=self.v_f16) for g in range(G)]
            mark()
            back = torch.empty((G, self.ws, m, hgl, d), dtype=torch.bfloat16, device=self.device)
            for g in range(G):
                self.exchange_into(back[g], outs[g].view(self.ws, m, hgl, d))
            mark()
            o8, so = ops.quant_from_recv(back[0]) if G == 1 else quant_grouped_back(back)
        elif self.ws > 1 and self.groups > 1:
            from .ulysses_overlap import grouped_attention, quant_grouped_back
            sends = ops.fp8_gemm_qkv_send(q8, self.wqkv8, sx, self.sqkv, self.heads, self.ws, v_f16=self.v_f16,
                                          range_flag=self.range_flag, groups=self.groups)
            self.share_range_flag()
            if self._v_overflowed(self.range_flag):
                sends = ops.fp8_gemm_qkv_send(q8, self.wqkv8, sx, self.sqkv, self.heads, self.ws, v_f16=False,
                                              groups=self.groups)
            mark()
            mark()      # with head groups the exchanges overlap the attention: the attention stage holds all three
            pv_f16 = self.v_f16
            back = grouped_attention(sends, self.ws, self.groups,
                                     lambda q, k, v: ops.flash_attn(q, k, v, scale=1.0 / math.sqrt(d),
                                                                    range_flag=self.range_flag, pv_f16=pv_f16),
                                     pg=self.pg, a2a=self.a2a)
            mark()
            mark()
            o8, so = quant_grouped_back(back)
        else:
            sends = ops.fp8_gemm_qkv_send(q8, self.wqkv8, sx, self.sqkv, self.heads, self.ws, v_f16=self.v_f16,
                                          range_flag=self.range_flag)
            self.share_range_flag()
            if self._v_overflowed(self.range_flag):
                sends = ops.fp8_gemm_qkv_send(q8, self.wqkv8, sx, self.sqkv, self.heads, self.ws, v_f16=False)
            mark()
            q, k, v = (self.exchange(s).view(self.ws * m, hl, d) for s in sends)
            mark()
            o = ops.flash_attn(q, k, v, scale=1.0 / math.sqrt(d), range_flag=self.range_flag, pv_f16=self.v_f16)
            mark()
            back = self.exchange(o.view(self.ws, m, hl, d))
            mark()
            o8, so = ops.quant_from_recv(back)
        mark()
        y = ops.fp8_gemm(o8, self.wo8, so, self.so)
        mark()
        return y

    KERNELS_PER_FORWARD = 5   # h3b launches per forward: quant, qkv GEMM, attention, quant, out GEMM
    P2P_BARRIERS = 2          # extra h3b launches per forward with exchange "p2p" (the two epoch barriers)

    __call__ = forward
