"""The out-projection's per-token FP8 quant read straight from the reverse all-to-all's receive buffer.

Mirrors ``h3_tp2/ulysses_outq.py``: row m of the out-projection input is concat_p recv[p, m] (P segments of H/P*d
bf16), quantised per token into the [M, H*d] e4m3 input plus the [M, 1] fp32 scale, so stock's unpack copy (copy 5)
and its [1, M, H, d] tensor are never made.

The deferral protocol is the reference's: an attention forward armed by ``arm(owner, rows)`` (its out-projection
``prepare``-d, i.e. that layer's ``quant_fp8`` wrapped in ``OutQuant``) gets from ``defer`` a stride-0 placeholder of
stock's [1, M, H, d] shape instead of the unpacked tensor; when the placeholder reaches the wrapped quant, the quant
runs on the receive buffer (the first time in a process after a bitwise self-check against copy 5 + the layer's own
quant).  A placeholder that reaches anything else, or a deferral the forward never consumed, raises.
"""
from __future__ import annotations

import logging
import threading

import torch

from . import ops

logger = logging.getLogger("h3b.ulysses_outq")
_warned: set = set()


def _warn_once(key: str, msg: str, *args) -> None:  # noqa: ANN002
    if key not in _warned:
        _warned.add(key)
        logger.warning("h3b ulysses_outq: " + msg, *args)

FP8_MAX = 448.0
FP8_MIN = -448.0
MIN_SCALE = 1.0 / (FP8_MAX * 512.0)


def quant_rows(base: torch.Tensor, m: int, p: int, seg: int, stride_p: int, stride_m: int, warps: int = 8,
               div_mode: int = ops.DIV_IEEE):
    """h3_tp2/ulysses_outq.py:109 (``warps`` is accepted for signature compatibility; the CUDA kernel picks its own
    launch shape).  Returns (q [M, P*seg] e4m3, scale [M, 1] fp32)."""
    del warps
    return torch.ops.h3b.quant_rows(base, m, p, seg, stride_p, stride_m, div_mode)


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
    return torch.ops.h3b.quant_from_recv(recv, div_mode)


def unpack_rows(recv: torch.Tensor) -> torch.Tensor:
    """Stock's copy 5 (h3_tp2/ulysses_outq.py:146): [P, M, hl, d] -> contiguous [M, P*hl*d]."""
    p, m, hl, d = recv.shape
    return ops.unpack_recv(recv).view(m, p * hl * d)


# ---------------------------------------------------------------------------------------------------------------
# deferral: a placeholder out of the reverse exchange, the quant from the receive buffer in the out-projection
# ---------------------------------------------------------------------------------------------------------------

_tls = threading.local()    # owner: (attention, rows) armed for one deferral; pending: Deferred
_state: dict = {"disabled": None, "checked": False, "sources": None}   # sources: why the upstream path is not reviewed
_stats = {k: 0 for k in ("deferred", "quant_recv", "selfcheck_pass", "selfcheck_fail", "not_prepared")}
# the two kernels the deferral runs (module-level so host-logic tests can substitute CPU implementations)
_kernels = {"quant_from_recv": lambda recv: quant_from_recv(recv), "unpack_rows": lambda recv: unpack_rows(recv)}


def stats() -> dict[str, int]:
    return dict(_stats)


def _placeholder(shape, like: torch.Tensor) -> torch.Tensor:  # noqa: ANN001
    """A tensor of ``shape`` owning one element of ``like``'s dtype and device (every stride 0): nothing may read it."""
    return like.new_empty(1).as_strided(tuple(shape), (0,) * len(shape))


def _is_placeholder(t: torch.Tensor) -> bool:
    return t.numel() > 1 and all(st == 0 for st in t.stride())


def is_placeholder(t: torch.Tensor) -> bool:
    """True for a placeholder made by ``defer`` or a view of it (h3_tp2/ulysses_outq.py:191): stride 0 everywhere and
    either the pending deferral's pointer or a one-element storage."""
    if not _is_placeholder(t):
        return False
    pend = getattr(_tls, "pending", None)
    if pend is not None and t.data_ptr() == pend.ph.data_ptr():
        return True
    return t.untyped_storage().nbytes() <= t.element_size()


def _bits(t: torch.Tensor) -> torch.Tensor:
    t = t.contiguous()
    return t.view(torch.uint8) if t.element_size() == 1 else t.view(torch.int32)


class Deferred:
    """A reverse exchange whose unpack is left to the out-projection quant (h3_tp2/ulysses_outq.py:208): the receive
    buffer [P, M, hl, d] and the placeholder that stands for its unpack."""

    __slots__ = ("recv", "heads", "ph", "m", "k", "_done")

    def __init__(self, recv: torch.Tensor, heads: int, ph: torch.Tensor | None = None):
        p, m, hl, d = recv.shape
        self.recv, self.heads, self._done = recv, heads, False
        self.m, self.k = m, p * hl * d
        self.ph = ph if ph is not None else _placeholder((1, m, p * hl, d), recv)

    @property
    def shape(self):  # noqa: ANN201
        p, m, hl, d = self.recv.shape
        return (1, m, p * hl, d)

    def matches(self, x: torch.Tensor) -> bool:
        """``x`` is this deferral's placeholder as the out-projection flattens it ([M, H*d])."""
        return x.data_ptr() == self.ph.data_ptr() and tuple(x.shape) == (self.m, self.k) and _is_placeholder(x)

    def quantize(self, orig=None, div_mode: int = ops.DIV_IEEE):  # noqa: ANN001,ANN201
        """(q [M, H*d] e4m3, scale [M, 1]) of stock's unpacked rows, read from the receive buffer.  ``orig`` (the
        layer's own quant, called as ``orig(x, None, None)``): the first deferral of the process is checked bit for bit
        against ``orig`` on copy 5 and the path is disabled for the process on any difference (the stock result is
        returned then, and by every later call)."""
        if self._done:
            raise RuntimeError("h3b ulysses_outq: deferred receive quantised twice")
        self._done = True
        if orig is None:
            _stats["quant_recv"] += 1
            return quant_from_recv(self.recv, div_mode=div_mode)
        if _state["disabled"] is None and not _state["checked"]:
            return _selfcheck(self, orig)
        if _state["disabled"] is not None:
            return orig(_kernels["unpack_rows"](self.recv), None, None)
        _stats["quant_recv"] += 1
        return _kernels["quant_from_recv"](self.recv)

    def materialize(self) -> torch.Tensor:
        """The bf16 [1, M, H, d] tensor stock's unpack makes (for consumers other than the FP8 out-projection)."""
        p, m, hl, d = self.recv.shape
        return _kernels["unpack_rows"](self.recv).view(1, m, p * hl, d)


def _selfcheck(pend: Deferred, orig):  # noqa: ANN001,ANN202
    """The first deferral of the process: copy 5 + the layer's own quant against the receive-buffer quant on the real
    tensor, bit for bit (values, scales, shapes, strides).  Returns the stock result."""
    _state["checked"] = True
    stock = orig(_kernels["unpack_rows"](pend.recv), None, None)
    try:
        got = _kernels["quant_from_recv"](pend.recv)
        ok = all(a.shape == b.shape and a.stride() == b.stride() and a.dtype == b.dtype and torch.equal(_bits(a), _bits(b))
                 for a, b in zip(stock, got))
        why = "" if ok else "FP8 values or scales differ"
    except Exception as exc:  # noqa: BLE001  (any failure disables the path for the process)
        ok, why = False, f"raised {exc!r}"
    if ok:
        _stats["selfcheck_pass"] += 1
    else:
        _stats["selfcheck_fail"] += 1
        _state["disabled"] = "self-check: " + why
        logger.warning("h3b ulysses_outq: %s; the reverse unpack stays for this process", _state["disabled"])
    return stock


def take(x: torch.Tensor) -> Deferred | None:
    """This thread's pending deferral if ``x`` is its placeholder (consumed), None for an ordinary tensor; a
    placeholder without its receive buffer (or in another shape) raises (h3_tp2/ulysses_outq.py:258)."""
    pend = getattr(_tls, "pending", None)
    if pend is not None and pend.matches(x):
        _tls.pending = None
        return pend
    if (pend is not None and x.data_ptr() == pend.ph.data_ptr()) or (pend is None and _is_placeholder(x)):
        raise RuntimeError("h3b ulysses_outq: a placeholder reached an out-projection quant without its receive buffer "
                           "(or in another shape)")
    return None


class OutQuant:
    """Stands in for one out-projection's ``quant_fp8`` (h3_tp2/ulysses_outq.py:233): the deferred placeholder is
    quantised from the receive buffer, every other input goes to the original quant unchanged."""

    _h3b_outq = True

    def __init__(self, orig):  # noqa: ANN001
        self._orig = orig

    def __getattr__(self, name: str):  # noqa: ANN204
        if name == "_orig":
            raise AttributeError(name)
        return getattr(self._orig, name)

    def __call__(self, x, scale=None, scale_ub=None, *args, **kwargs):  # noqa: ANN001,ANN204
        pend = take(x) if isinstance(x, torch.Tensor) else None
        if pend is None:
            return self._orig(x, scale, scale_ub, *args, **kwargs)
        if scale is not None or scale_ub is not None or args or kwargs:
            raise RuntimeError("h3b ulysses_outq: unexpected static scale / bound for a deferred quant")
        return pend.quantize(self._orig)


def layer_mismatch(owner) -> str | None:  # noqa: ANN001
    """None when ``owner.out_proj`` reaches a dynamic per-token quant as ``quant_method.fp8_linear.quant_fp8`` on the
    whole [M, H*d] input (a single-rank row-parallel linear), else the reason (h3_tp2/ulysses_outq.py:330; the upstream
    sources on the path are checked once by ``check_sources``)."""
    layer = getattr(owner, "out_proj", None)
    if layer is None:
        return "no out_proj"
    if getattr(layer, "tp_size", 1) != 1:
        return "out_proj tp_size != 1"
    k = getattr(owner, "num_heads", None), getattr(owner, "head_dim", None)
    width = getattr(layer, "input_size_per_partition", None)
    if None not in k and width is not None and int(width) != int(k[0]) * int(k[1]):
        return "out_proj input width != heads * head_dim"
    kernel = getattr(getattr(layer, "quant_method", None), "fp8_linear", None)
    quant = getattr(kernel, "quant_fp8", None)
    if not callable(quant):
        return "no fp8_linear.quant_fp8 on the out-projection"
    base = quant._orig if isinstance(quant, OutQuant) else quant
    if getattr(base, "static", False) or getattr(base, "is_group_quant", False) or \
            not getattr(base, "use_per_token_if_dynamic", True) or getattr(base, "num_token_padding", None) is not None:
        return "activation quant is not dynamic per-token without padding"
    return None


def source_fingerprints(attn_forward) -> dict[str, str | None]:  # noqa: ANN001
    """The fingerprints of every upstream function between the attention output and the quant (:300);
    ``attn_forward`` = the attention's forward as upstream wrote it, before wrapping."""
    from . import sources  # noqa: PLC0415
    return sources.outq_fingerprints(attn_forward)


def check_sources(attn_forward) -> str | None:  # noqa: ANN001
    """None when every function on the path has the reviewed source, else the reason, kept for ``prepare`` (:319)."""
    from . import sources  # noqa: PLC0415
    bad = sources.changed(sources.OUTQ_REVIEWED, source_fingerprints(attn_forward), sources.OUTQ_REVIEWED)
    _state["sources"] = ("upstream source changed: " + ", ".join(bad)) if bad else None
    if bad:
        _warn_once("sources", "%s; the reverse unpack stays", _state["sources"])
    return _state["sources"]


def prepare(owner) -> bool:  # noqa: ANN001
    """Once per attention: True when its out-projection's quant can take a deferred receive buffer, and then that
    layer's ``quant_fp8`` is wrapped in ``OutQuant`` (h3_tp2/ulysses_outq.py:370); never while ``check_sources``
    found the upstream path changed."""
    layer = getattr(owner, "out_proj", None)
    if layer is None:
        return False
    ok = getattr(layer, "_h3b_outq", None)
    if ok is None:
        reason = _state["sources"] or layer_mismatch(owner)
        ok = reason is None
        if ok:
            kernel = layer.quant_method.fp8_linear
            if not isinstance(kernel.quant_fp8, OutQuant):
                kernel.quant_fp8 = OutQuant(kernel.quant_fp8)
        else:
            _warn_once("layer-" + reason, "out-projection not eligible (%s); the reverse unpack stays there", reason)
        layer._h3b_outq = ok
    return bool(ok)


def arm(owner, rows: int) -> tuple:  # noqa: ANN001
    """Start of an armed attention forward: its reverse exchange may defer the unpack (h3_tp2/ulysses_outq.py:390).
    Returns the previous state for ``disarm``."""
    prev = (getattr(_tls, "owner", None), getattr(_tls, "pending", None))
    _tls.owner = (owner, rows) if _state["disabled"] is None and prepare(owner) else None
    _tls.pending = None
    return prev


def disarm(prev: tuple, check: bool) -> None:
    """End of the armed forward; with ``check`` (it returned normally) a deferral it made must have been consumed."""
    pend = getattr(_tls, "pending", None)
    _tls.owner, _tls.pending = prev
    if check and pend is not None:
        raise RuntimeError("h3b ulysses_outq: the attention returned without its out-projection quantising the deferred "
                           "receive buffer")


def defer(recv: torch.Tensor, heads: int) -> torch.Tensor | None:
    """From the reverse exchange (h3_tp2/ulysses_outq.py:407): a stride-0 placeholder [1, M, H, d] standing for the
    unpack of ``recv`` when this forward was armed for it (rows match, path enabled), else None (the caller makes
    copy 5)."""
    owner = getattr(_tls, "owner", None)
    p, m, hl, d = recv.shape
    if owner is None or owner[1] != m or p * hl != heads or _state["disabled"] is not None or \
            not recv.is_contiguous() or recv.dtype is not torch.bfloat16:
        if owner is not None:
            _stats["not_prepared"] += 1
        return None
    _tls.owner = None
    pend = Deferred(recv, heads)
    _tls.pending = pend
    _stats["deferred"] += 1
    return pend.ph
