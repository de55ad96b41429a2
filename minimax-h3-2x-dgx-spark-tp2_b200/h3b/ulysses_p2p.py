"""Ulysses exchange through peer memory over NVLink: the all-to-alls folded into the producing kernels.

Stock strict Ulysses moves q, k, v seq->heads and the attention output heads->seq with two
``dist.all_to_all_single`` exchanges (h3_tp2/ulysses_exact.py:94; the head-group overlap variant issues one per
group, h3_tp2/ulysses_overlap.py:34,45).  Here every rank registers one device buffer once (plain ``cudaMalloc`` +
CUDA IPC; no multicast object, so a dead rank leaves no NVLink multicast binding) holding

    [flags 256 B | q recv | k recv | v recv (f16) | back recv]      q/k/v/back each [P, M, H/P, 128]

and the kernels store across NVLink while they compute: the qkv GEMM epilogue writes destination rank p's slab into
rank p's q/k/v receive buffers (slot = source rank), the attention epilogue writes output row t into rank t // M's
back buffer (slot = this rank).  No send buffer and no collective remains; two epoch barriers per block
(``h3b_p2p_signal_wait``, one tiny kernel each) order the stores before the readers.

Ordering, one forward on every rank (all on the rank's current stream):

    quant -> qkv GEMM (peer stores) -> barrier e -> attention (peer stores) -> barrier e+1 -> quant(back) -> out GEMM

* rank p's receive buffers are complete once p passes barrier e: every rank signals e after its GEMM;
* rank r's next GEMM overwrites p's q/k/v only after r passed barrier e+1, which p signals after its attention;
* rank r's next attention overwrites p's back buffer only after barrier e+2, which p signals after its next GEMM,
  i.e. after its quant of the previous back buffer.

So two barriers per forward suffice and no buffer is double-buffered.  A rank that stops signalling makes the
others' barrier kernels give up after the library's wait bound (``h3b_set_wait_timeout_ns``) with H3B_ETIMEOUT in
the device status word; the context stays usable.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib, ops

_FLAGS_BYTES = 256
_RF_OFFSET = 64          # int32 v-overflow flag inside the flag block (epoch flags: int32[8] at 0)


def _round(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


class _CudaArray:
    """__cuda_array_interface__ over a raw device address (torch.as_tensor keeps this object alive)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None}


def _view(ptr: int, shape: tuple, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    typestr = {torch.float16: "<f2", torch.int32: "<i4", torch.bfloat16: "<i2"}[dtype]
    t = torch.as_tensor(_CudaArray(ptr, shape, typestr), device=device)
    return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t


def _default_allgather(pg):
    def allgather(blob: bytes) -> list[bytes]:
        out = [None] * dist.get_world_size(pg)
        dist.all_gather_object(out, blob, group=pg)
        return out
    return allgather


def probe(pg, device) -> tuple[bool, str]:
    """Collective check that every rank of ``pg`` can map every other rank's memory (CUDA IPC over NVLink): a 4 KiB
    exchange buffer per rank, all-gathered handles, every peer opened; the verdict is agreed by all ranks
    (all-reduce MIN), so they all take the same exchange path.  Returns (ok, reason of this rank's failure)."""
    ws, rank = dist.get_world_size(pg), dist.get_rank(pg)
    dev = torch.device(device)
    reason = ""
    px = None
    try:
        px = PeerExchange(1, ws, ws, rank, dev, pg=pg)
    except Exception as exc:  # noqa: BLE001  (the verdict is collective below)
        reason = f"{type(exc).__name__}: {exc}"
    flag = torch.tensor([0 if reason else 1], dtype=torch.int32, device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=pg)
    if px is not None:
        px.close(host_barrier=lambda: dist.barrier(group=pg))
    else:  # keep the two host barriers of the others' close() matched
        dist.barrier(group=pg)
        dist.barrier(group=pg)
    ok = bool(flag.item())
    if not ok and not reason:
        reason = "another rank could not map peer memory"
    return ok, reason


class PeerExchange:
    """Receive buffers of one Ulysses group for a fixed per-rank sequence length ``m`` (tokens per rank).

    Collective: every rank of the group constructs it with the same (m, heads, ws) and calls ``barrier`` and
    ``close`` in the same order.  ``allgather(bytes) -> list[bytes]`` exchanges the IPC handles (default: the
    process group's ``all_gather_object``)."""

    def __init__(self, m: int, heads: int, ws: int, rank: int, device, *, pg=None, allgather=None,
                 v_f16: bool = False):
        if ws < 1 or ws > _lib.MAX_RANKS or heads % ws or not 0 <= rank < ws:
            raise ValueError(f"PeerExchange: ws {ws} (1..{_lib.MAX_RANKS}), heads {heads}, rank {rank}")
        self.m, self.heads, self.ws, self.rank = m, heads, ws, rank
        self.device = torch.device(device)
        self.hl = heads // ws
        self.v_f16 = v_f16
        self.epoch = 0
        self._v16 = None   # f16 copy of the received v (bf16 v only), allocated by the first attention
        shape = (ws, m, self.hl, 128)
        slab = _round(ws * m * self.hl * 128 * 2)
        self._off = {"q": _FLAGS_BYTES, "k": _FLAGS_BYTES + slab, "v": _FLAGS_BYTES + 2 * slab,
                     "back": _FLAGS_BYTES + 3 * slab}
        self.nbytes = _FLAGS_BYTES + 4 * slab
        lib = _lib.load()
        with torch.cuda.device(self.device):
            own, handle = ctypes.c_void_p(), _lib.IpcHandle()
            _lib.check(lib.h3b_p2p_alloc(self.nbytes, ctypes.byref(own), ctypes.byref(handle)), "h3b_p2p_alloc")
            self._own = own.value
            self._opened: list[int] = []
            try:
                gather = allgather if allgather is not None else _default_allgather(pg)
                blobs = gather(bytes(handle.bytes))
                self.base = []
                for r in range(ws):
                    if r == rank:
                        self.base.append(self._own)
                        continue
                    h = _lib.IpcHandle()
                    ctypes.memmove(h.bytes, blobs[r], 64)
                    ptr = ctypes.c_void_p()
                    _lib.check(lib.h3b_p2p_open(ctypes.byref(h), ctypes.byref(ptr)), "h3b_p2p_open")
                    self._opened.append(ptr.value)
                    self.base.append(ptr.value)
            except BaseException:
                self._release()
                raise
        dev = self.device
        b = self._own
        self.q = _view(b + self._off["q"], shape, torch.bfloat16, dev)
        self.k = _view(b + self._off["k"], shape, torch.bfloat16, dev)
        self.v = _view(b + self._off["v"], shape, torch.float16 if v_f16 else torch.bfloat16, dev)
        self.back = _view(b + self._off["back"], shape, torch.bfloat16, dev)
        self.range_flag = _view(b + _RF_OFFSET, (1,), torch.int32, dev)
        self._flags = _view(b, (_lib.MAX_RANKS,), torch.int32, dev)

    # ---- what the kernels are given ----
    def qkv_targets(self):
        """``p2p`` argument of ``ops.fp8_gemm_qkv_send``: (rank, per-rank (q, k, v) addresses, range flags)."""
        o = self._off
        return (self.rank, [(b + o["q"], b + o["k"], b + o["v"]) for b in self.base],
                [b + _RF_OFFSET for b in self.base])

    def back_targets(self) -> list[int]:
        return [b + self._off["back"] for b in self.base]

    def barrier(self) -> None:
        """Epoch barrier on the current stream: work enqueued before it on every rank is visible after it."""
        self.epoch += 1
        ops.p2p_signal_wait(list(self.base), self._own, self.rank, self.epoch,
                            torch.cuda.current_stream(self.device).cuda_stream)

    # ---- one Ulysses attention through peer memory ----
    def forward_qkv(self, q8, wqkv8, sx, sqkv, *, bias=None) -> None:
        """qkv projection of this rank's m tokens, each destination's slab stored into its receive buffers."""
        if q8.shape[0] != self.m:
            raise ValueError(f"PeerExchange: {q8.shape[0]} rows, buffers hold {self.m}")
        ops.fp8_gemm_qkv_send(q8, wqkv8, sx, sqkv, self.heads, self.ws, bias=bias, v_f16=self.v_f16,
                              p2p=self.qkv_targets())

    def attention(self, scale: float, ctl: torch.Tensor | None = None) -> None:
        """This rank's heads over the whole sequence, each output row stored into its owner's back buffer.  With bf16
        v (the default) the received v is converted to f16 here and the device runs the f16 P.V product on it, or on
        a copy scaled per (head, column) when some value does not fit f16 (``ctl``: ``ops.attn_ctl`` control words,
        word 0 then says which pass ran); an f16 v buffer (``v_f16=True``: the peers' epilogues converted it and
        raised the buffer's range flag on an overflow) is used as is and refused on an overflow."""
        n = self.ws * self.m
        if self.v_f16:
            ops.flash_attn_p2p(self.q.view(n, self.hl, 128), self.k.view(n, self.hl, 128),
                               self.v.view(n, self.hl, 128), self.back_targets(), self.rank, scale=scale,
                               range_flag=self.range_flag)
            return
        if self._v16 is None:
            self._v16 = torch.empty((n, self.hl, 128), dtype=torch.float16, device=self.device)
        ops.flash_attn_p2p(self.q.view(n, self.hl, 128), self.k.view(n, self.hl, 128), self.v.view(n, self.hl, 128),
                           self.back_targets(), self.rank, scale=scale, v16=self._v16, ctl=ctl)

    # ---- teardown (collective; the q/k/v/back/range_flag views dangle afterwards) ----
    def close(self, host_barrier=None) -> None:
        """Waits for this device, then (after ``host_barrier()``, so no peer still writes here) unmaps the peers'
        buffers and frees this rank's one."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        if host_barrier is not None:
            host_barrier()
        with torch.cuda.device(self.device):
            for p in self._opened:
                _lib.check(_lib.load().h3b_p2p_close(ctypes.c_void_p(p)), "h3b_p2p_close")
            self._opened = []
            if host_barrier is not None:
                host_barrier()
            self._release()

    def _release(self) -> None:
        lib = _lib.load()
        for p in self._opened:
            lib.h3b_p2p_close(ctypes.c_void_p(p))
        self._opened = []
        if self._own is not None:
            lib.h3b_p2p_free(ctypes.c_void_p(self._own))
            self._own = None
