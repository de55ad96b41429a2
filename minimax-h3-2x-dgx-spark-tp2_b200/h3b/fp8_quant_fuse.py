"""Per-token FP8 quant fused into the producers of each GEMM input (mirrors ``h3_tp2/fp8_quant_fuse.py``).

Sites: qkv (RMSNorm + AdaLN modulation), out (the Ulysses reverse unpack), fc1 (gated residual + RMSNorm +
modulation), fc2 (SiLU-mul).  Each entry point runs one CUDA row kernel that produces the bf16 value the stock
producer would store, keeps it in registers and writes the e4m3 row and its fp32 scale.  ``stock`` arguments of the
reference signatures are accepted and ignored (the GPU path never runs the stock producer).

The wiring into the model is the reference's protocol: inside a planned DiT block (``make_block_forward`` /
``block_plan``) a wrapped producer runs the fused kernel, stashes (fp8, scale) as ``Pending`` and returns an
uninitialised bf16 placeholder of the stock output's shape; the layer's wrapped ``QuantFP8.forward``
(``make_quant_forward``) recognises the placeholder (same quant instance, pointer, shape, strides) and returns the
stash instead of quantising.  A stash any other call meets first is materialised (the stock producer run into the
placeholder), a layer that returned without consuming its stash is run again, and the first call per site and width
is compared bit for bit with the stock producer + the layer's own quant on its first rows (a mismatch disables the
site for the process).
"""
from __future__ import annotations

import logging
from typing import Any, Callable

import torch

from . import _fusewire as _fw
from . import ops

logger = logging.getLogger("h3b.fp8_quant_fuse")
SITES = ("qkv", "out", "fc1", "fc2")
FP8_MAX = 448.0
MIN_SCALE = 1.0 / (FP8_MAX * 512.0)


def quant(h: torch.Tensor, div_mode: int = ops.DIV_IEEE):
    """h3_tp2/fp8_quant_fuse.py:318."""
    return torch.ops.h3b.quant(h, div_mode)


def rms_quant(x, weight, shift, scale, indices, eps, stock=None, ph=None, div_mode: int = ops.DIV_IEEE):  # noqa: ANN001,ANN201
    """h3_tp2/fp8_quant_fuse.py:330: (fp8 [M, H], scale [M, 1]); ``ph`` also receives the bf16 row."""
    del stock
    return torch.ops.h3b.rms_quant(x, weight, shift, scale, indices, float(eps), ph, div_mode)


def gate_rms_quant(residual, gate, branch, weight, shift, scale, indices, eps, stock=None, ph=None,  # noqa: ANN001,ANN201
                   div_mode: int = ops.DIV_IEEE):
    """h3_tp2/fp8_quant_fuse.py:350: (residual_out bf16, fp8, scale)."""
    del stock
    if ph is not None:
        raise NotImplementedError("gate_rms_quant: the bf16 copy (ph) is not produced on this path")
    return torch.ops.h3b.gate_rms_quant(residual, gate, branch, weight, shift, scale, indices, float(eps), div_mode)


def unpack_quant(recv: torch.Tensor, div_mode: int = ops.DIV_IEEE):
    """h3_tp2/fp8_quant_fuse.py:379: the reverse unpack + per-token quant of [M, P*hl*d]."""
    return torch.ops.h3b.quant_from_recv(recv.contiguous(), div_mode)


def silu_mul_quant(x: torch.Tensor, stock=None, div_mode: int = ops.DIV_IEEE):  # noqa: ANN001
    """h3_tp2/fp8_quant_fuse.py:392: silu_and_mul on bf16 [M, 2d] + per-token quant."""
    del stock
    return torch.ops.h3b.silu_mul_quant(x, div_mode)


def quant_torch(h: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token dynamic e4m3 quant in eager torch (vLLM ``QuantFP8.forward_native``, h3_tp2/fp8_quant_fuse.py:302):
    scale = max(amax / 448, 1/229376) per row (NaN propagates), q = e4m3(clamp(h * (1 / scale), +-448)).  Returns
    (q [M, K] e4m3, scale [M, 1] fp32).  A CPU function by design, not a fallback of ``quant``."""
    amax = h.abs().amax(dim=-1, keepdim=True).float()
    amax = torch.where(torch.isnan(h).any(dim=-1, keepdim=True), torch.full_like(amax, float("nan")), amax)
    scale = torch.clamp(amax / FP8_MAX, min=MIN_SCALE)
    q = torch.clamp(h.float() * torch.reciprocal(scale), -FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q, scale


def unpack_stock(recv: torch.Tensor, heads: int) -> torch.Tensor:
    """Stock's reverse unpack (h3_tp2/fp8_quant_fuse.py:371): receive [P, M, hl, d] -> [1, M, H, d] contiguous."""
    p, m, hl, d = recv.shape
    if p * hl != heads:
        raise ValueError(f"unpack_stock: {p} x {hl} heads received, {heads} expected")
    return recv.permute(1, 0, 2, 3).reshape(1, m, heads, d).contiguous()


_ON = ("1", "all", "on", "true")
_OFF = ("", "0", "off", "false")


def parse_sites(value: str | None) -> tuple[str, ...]:
    """``H3_TP2_FP8_QUANT_FUSE`` (h3_tp2/fp8_quant_fuse.py:836): "1"/"all"/"on"/"true" = every site, a comma list
    selects sites (in SITES order), anything else or empty = none."""
    v = (value or "").strip().lower()
    if v in _ON:
        return SITES
    if v in _OFF:
        return ()
    chosen = {part.strip() for part in v.split(",")}
    return tuple(site for site in SITES if site in chosen)


def is_explicit(value: str | None) -> bool:
    """True when the switch names its sites rather than turning all on or off (h3_tp2/fp8_quant_fuse.py:847)."""
    return (value or "").strip().lower() not in _ON + _OFF



# --------------------------------------------------------------------------------------------------------------------
# the wiring (the reference's protocol, h3_tp2/fp8_quant_fuse.py:404-921, on the shared machinery of h3b._fusewire)
# --------------------------------------------------------------------------------------------------------------------

_state: dict[str, Any] = {"sites": (), "checked": {}, "disabled": set(), "orig_quant": None, "quant_cls": None,
                          "act_cls": None, "verify": False, "modes": (0, 1), "device_types": ("cuda",)}
_stats: dict[str, int] = {k: 0 for k in ("fused_qkv", "fused_out", "fused_fc1", "fused_fc2", "consumed", "materialize",
                                         "rerun", "selfcheck_pass", "selfcheck_fail", "verify_calls", "verify_mismatch")}


def stats() -> dict[str, int]:
    return dict(_stats)


class Pending:
    """A producer's quantised output (fp8 ``q``, ``scale``) handed to the quant call of ``layer``.  The model holds
    ``ph``, an uninitialised bf16 placeholder of the stock producer's output; the linear layer reshapes it to
    [numel / k, k] (k: the GEMM input width) before its quant, so the claim compares that exact view, made once here.
    ``fill(ph)`` writes the stock producer's output into the placeholder when the handoff has to become real."""

    __slots__ = ("site", "ph", "k", "q", "scale", "quant", "layer", "fill", "_view")

    def __init__(self, site: str, ph: torch.Tensor, k: int, q: torch.Tensor, scale: torch.Tensor, quant, layer,  # noqa: ANN001
                 fill: Callable[[torch.Tensor], None]):
        self.site, self.ph, self.k, self.q, self.scale = site, ph, k, q, scale
        self.quant, self.layer, self.fill = quant, layer, fill
        # the quant input that is this placeholder: (data pointer, shape, strides, dtype, device), or None when the
        # placeholder is not dense (then nothing can claim it)
        self._view = (ph.data_ptr(), (ph.numel() // k, k), (k, 1), ph.dtype, ph.device) if ph.is_contiguous() else None

    def matches(self, quant_obj, x: torch.Tensor) -> bool:  # noqa: ANN001
        """True when ``quant_obj(x)`` is the planned quant of this placeholder."""
        return (self._view is not None and quant_obj is self.quant and x.dim() == 2
                and (x.data_ptr(), tuple(x.shape), x.stride(), x.dtype, x.device) == self._view)

    def materialize(self) -> torch.Tensor:
        self.fill(self.ph)
        return self.ph


def _realized(handoff: Pending) -> None:
    handoff.materialize()
    _stats["materialize"] += 1


_scopes = _fw.ScopeRegistry(_realized, lambda site, why: None)
_tls = _scopes.local      # ``_tls.ctx``: the running block's scope (plan: site -> (layer, its quant instance))
_verdicts = _fw.Verdicts(lambda: _state, lambda: _stats, logger, "fp8 quant fuse")


def scope(block, plan: dict) -> _fw.BlockScope:  # noqa: ANN001
    """The context in which a planned block's forward runs (``with scope(block, plan): ...``)."""
    return _fw.BlockScope(_scopes, block, plan)


def _outstanding(sc: _fw.BlockScope | None) -> Pending | None:
    return None if sc is None or not sc.handoffs else next(iter(sc.handoffs.values()))


def _realize_outstanding(sc: _fw.BlockScope) -> None:
    if sc.handoffs:
        _scopes.realize_all(sc, "")


def _stock_quant(quant_obj, h: torch.Tensor):  # noqa: ANN001,ANN202
    """The layer's own per-token quant (the unwrapped ``QuantFP8.forward``), called as the linear kernel calls it."""
    return _state["orig_quant"](quant_obj, h, None, None)


def _verify(p: Pending) -> None:
    """``H3_TP2_FP8_QUANT_FUSE_VERIFY=1``: every handoff is also made real and quantised by the stock quant; the two
    (fp8, scale) pairs must agree bit for bit (mismatches are counted)."""
    q_ref, s_ref = _stock_quant(p.quant, p.materialize().view(-1, p.k))
    _stats["verify_calls"] += 1
    if not _fw.same_bits((p.q, p.scale), (q_ref, s_ref)):
        _stats["verify_mismatch"] += 1


def pending_placeholder(x: torch.Tensor) -> bool:
    """True when ``x`` is the placeholder of this thread's outstanding handoff (h3_tp2/fp8_quant_fuse.py:545)."""
    p = _outstanding(_scopes.current())
    return p is not None and x.data_ptr() == p.ph.data_ptr()


def make_quant_forward(orig):  # noqa: ANN001,ANN201
    """``QuantFP8.forward`` (h3_tp2/fp8_quant_fuse.py:553).  A dynamic call (no static scale, no upper bound) on exactly
    the outstanding handoff's placeholder, by exactly its planned quant instance, returns the handoff's (fp8, scale).
    Any other call first makes an outstanding handoff real, then runs the stock quant with its arguments untouched.
    A deferred-unpack placeholder of ``ulysses_outq`` must never get here (it holds no data): that raises."""
    def forward(self, x, *args, **kwargs):  # noqa: ANN001,ANN202
        is_tensor = isinstance(x, torch.Tensor)
        if is_tensor:
            from . import ulysses_outq  # noqa: PLC0415
            if ulysses_outq.is_placeholder(x):
                raise RuntimeError("h3b fp8 quant fuse: a deferred-unpack placeholder reached a quant outside the "
                                   "out-projection's")
        sc = _scopes.current()
        p = _outstanding(sc)
        if p is not None:
            static = (args[0] if args else kwargs.get("scale"), args[1] if len(args) > 1 else kwargs.get("scale_ub"))
            if static == (None, None) and is_tensor and p.matches(self, x):
                sc.handoffs.pop(p.site)
                if _state["verify"]:
                    _verify(p)
                _stats["consumed"] += 1
                return p.q, p.scale
            _realize_outstanding(sc)
        return orig(self, x, *args, **kwargs)

    forward._h3b_quant_fuse = True
    forward.__wrapped__ = orig
    return forward


def _layer_post_hook(module, args, output):  # noqa: ANN001,ANN202
    """After a planned layer's forward: if its handoff is still outstanding the layer ran on the uninitialised
    placeholder, so the placeholder is made real and the layer runs again (h3_tp2/fp8_quant_fuse.py:575)."""
    sc = _scopes.current()
    p = _outstanding(sc)
    if p is None or p.layer is not module:
        return None
    _realize_outstanding(sc)
    _stats["rerun"] += 1
    return module.forward(*args)


# where each site's linear layer sits in a DiT block
_SITE_LAYER = {"qkv": ("attn", "qkv_proj"), "out": ("attn", "out_proj"), "fc1": ("mlp", "fc1"), "fc2": ("mlp", "fc2")}


def _quant_of(layer):  # noqa: ANN001,ANN202
    """The layer's quant instance if it is a dynamic per-token FP8 quant without static or group scales (what the fused
    kernels compute), else None."""
    qobj = getattr(getattr(getattr(layer, "quant_method", None), "fp8_linear", None), "quant_fp8", None)
    cls = _state["quant_cls"]
    if cls is None or not isinstance(qobj, cls):
        return None
    dynamic_per_token = (not getattr(qobj, "static", True) and getattr(qobj, "use_per_token_if_dynamic", False)
                         and not getattr(qobj, "is_group_quant", True)
                         and getattr(qobj, "num_token_padding", 0) is None)
    scaled_input = getattr(layer, "input_scale", None) is not None or getattr(layer, "input_scale_ub", None) is not None
    return qobj if dynamic_per_token and not scaled_input else None


def _blocker(site: str, layer, lora) -> str | None:  # noqa: ANN001
    """Why ``layer`` stops the whole block from being fused at ``site`` (None: it does not)."""
    if layer is None or (lora and isinstance(layer, lora)):
        return f"{site}: missing or LoRA-wrapped layer"
    if getattr(layer, "tp_size", 1) != 1:
        return f"{site}: tp_size != 1"
    if _quant_of(layer) is None:
        return f"{site}: not a dynamic per-token FP8 linear"
    return None


def _passed_over(site: str, block) -> bool:  # noqa: ANN001
    """Sites left to the stock path in a block that is otherwise fused: qkv when a VSA gate reads the qkv input a
    second time, fc2 when the MLP's activation is not the SiLU-and-mul this wiring wraps."""
    if site == "qkv":
        return getattr(getattr(block, "attn", None), "to_gate_compress", None) is not None
    if site == "fc2":
        act = _state["act_cls"]
        return act is not None and not isinstance(getattr(getattr(block, "mlp", None), "act_fn", None), act)
    return False


def block_plan(block, sites, lora_types=()) -> tuple[dict | None, str]:  # noqa: ANN001
    """{site: (layer, quant instance)} for this block, or (None, reason) (h3_tp2/fp8_quant_fuse.py:614)."""
    if _fw.compiling():
        return None, "torch.compile tracing"
    live = [s for s in sites if s not in _state["disabled"]]
    layers = {s: getattr(getattr(block, _SITE_LAYER[s][0], None), _SITE_LAYER[s][1], None) for s in live}
    for site in live:
        why = _blocker(site, layers[site], lora_types)
        if why is not None:
            return None, why
    plan = {s: (layers[s], _quant_of(layers[s])) for s in live if not _passed_over(s, block)}
    for layer, _ in plan.values():
        if not getattr(layer, "_h3b_quant_fuse_hook", False) and hasattr(layer, "register_forward_hook"):
            layer.register_forward_hook(_layer_post_hook)
            layer._h3b_quant_fuse_hook = True
    return (plan or None), "no site left"


def make_block_forward(orig_forward, sites, lora_types=()):  # noqa: ANN001,ANN201
    """The DiT block's forward, run in a scope with this block's plan (h3_tp2/fp8_quant_fuse.py:646)."""
    return _fw.wrap_block_forward(orig_forward, _scopes, lambda blk, *a, **kw: block_plan(blk, sites, lora_types),
                                  lambda why: None, "_h3b_quant_fuse")


# ---- the four producer sites ---------------------------------------------------------------------------------------


def _rows_ok(x: torch.Tensor, k: int, *others: torch.Tensor) -> bool:
    return (x.dim() == 2 and x.dtype == torch.bfloat16 and x.is_contiguous() and x.shape[0] > 0 and x.shape[1] == k
            and all(o.dim() == 2 and o.stride(1) == 1 for o in others))


def _k_of(layer) -> int:  # noqa: ANN001
    """The layer's input width (vLLM stores the weight [K, N])."""
    w = getattr(layer, "weight", None)
    return int(w.shape[0]) if isinstance(w, torch.Tensor) and w.dim() == 2 else -1


class _Site:
    """One producer site.  ``call`` is the wrapped function's argument tuple.  ``keep_row``: the fused kernel also
    stores the bf16 row (the RMS sites try without first; the other sites always produce it by other means)."""
    name = ""
    keep_row_modes: tuple | None = None      # None: one form only

    def accepts(self, sc, layer, call) -> bool:  # noqa: ANN001
        raise NotImplementedError

    def rows(self, call) -> int:  # noqa: ANN001
        raise NotImplementedError

    def key(self, call) -> tuple:  # noqa: ANN001
        raise NotImplementedError

    def fused(self, call, r: int, keep_row) -> tuple:  # noqa: ANN001
        raise NotImplementedError

    def stock(self, call, r: int, keep_row, qobj) -> tuple:  # noqa: ANN001
        raise NotImplementedError

    def produce(self, call, keep_row, qobj, layer) -> tuple:  # noqa: ANN001
        """(what the wrapped call returns, its Pending)."""
        raise NotImplementedError


def _serve(site: _Site, call: tuple):  # noqa: ANN202
    """The wrapped producer's result when ``site`` is planned in the running block, accepts the call and passes (or has
    passed) its first-call comparison; None sends the caller to the stock producer."""
    sc = _scopes.current()
    planned = None if sc is None else sc.plan.get(site.name)
    if planned is None or _verdicts.off(site.name):
        return None
    _realize_outstanding(sc)           # a handoff nobody claimed before the next producer ran
    layer, qobj = planned
    if not site.accepts(sc, layer, call):
        return None
    r = min(_fw.CHECK_ROWS, site.rows(call))
    if site.keep_row_modes is None:
        if not _verdicts.judge(site.key(call), lambda: site.fused(call, r, None),
                               lambda: site.stock(call, r, None, qobj)):
            return None
        mode = None
    else:
        mode = _verdicts.first_passing(site.key(call), _state["modes"], lambda m: site.fused(call, r, m),
                                       lambda m: site.stock(call, r, m, qobj))
        if mode is None:
            return None
    result, handoff = site.produce(call, mode, qobj, layer)
    sc.handoffs[site.name] = handoff
    _stats["fused_" + site.name] += 1
    return result


class _NormSite(_Site):
    """qkv: ``rms_norm_indexed_scale_shift(x, weight, shift, scale, indices, eps)`` of norm1 (the qkv GEMM's input)."""
    name, keep_row_modes = "qkv", (0, 1)

    def __init__(self, orig):  # noqa: ANN001
        self.orig = orig

    def accepts(self, sc, layer, call) -> bool:  # noqa: ANN001
        x, weight, shift, scale, indices, _ = call
        return (weight is getattr(getattr(sc.block, "norm1", None), "weight", None)
                and _rows_ok(x, _k_of(layer), shift, scale) and indices.dim() == 1 and indices.shape[0] == x.shape[0]
                and _fw.same_device(_state["device_types"], x, weight, shift, scale, indices))

    def rows(self, call) -> int:  # noqa: ANN001
        return call[0].shape[0]

    def key(self, call) -> tuple:  # noqa: ANN001
        return ("qkv", call[0].shape[1], call[2].dtype, call[1].dtype)

    def fused(self, call, r, keep_row) -> tuple:  # noqa: ANN001
        x, weight, shift, scale, indices, eps = call
        row = torch.empty_like(x[:r]) if keep_row else None
        q, s = rms_quant(x[:r], weight, shift, scale, indices[:r], eps, self.orig, row)
        return (q, s, row) if keep_row else (q, s)

    def stock(self, call, r, keep_row, qobj) -> tuple:  # noqa: ANN001
        x, weight, shift, scale, indices, eps = call
        h = self.orig(x[:r], weight, shift, scale, indices[:r], eps)
        return (*_stock_quant(qobj, h), h) if keep_row else _stock_quant(qobj, h)

    def produce(self, call, keep_row, qobj, layer) -> tuple:  # noqa: ANN001
        x = call[0]
        ph = torch.empty_like(x)
        q, s = rms_quant(*call, self.orig, ph if keep_row else None)
        fill = (lambda t: None) if keep_row else (lambda t, c=call: t.copy_(self.orig(*c)))
        return ph, Pending("qkv", ph, x.shape[1], q, s, qobj, layer, fill)


class _GateNormSite(_Site):
    """fc1: ``indexed_gate_rms_norm_scale_shift(residual, gate, branch, weight, shift, scale, indices, eps)`` of norm2,
    whose modulated output feeds fc1 (the residual output is returned as stock's)."""
    name, keep_row_modes = "fc1", (0, 1)

    def __init__(self, orig):  # noqa: ANN001
        self.orig = orig

    def accepts(self, sc, layer, call) -> bool:  # noqa: ANN001
        residual, gate, branch, weight, shift, scale, indices, _ = call
        return (weight is getattr(getattr(sc.block, "norm2", None), "weight", None)
                and _rows_ok(residual, _k_of(layer), gate, branch, shift, scale)
                and branch.shape == residual.shape and branch.dtype == residual.dtype
                and indices.dim() == 1 and indices.shape[0] == residual.shape[0]
                and _fw.same_device(_state["device_types"], residual, gate, branch, weight, shift, scale, indices))

    def rows(self, call) -> int:  # noqa: ANN001
        return call[0].shape[0]

    def key(self, call) -> tuple:  # noqa: ANN001
        return ("fc1", call[0].shape[1], call[1].dtype, call[3].dtype)

    def _first(self, call, r) -> tuple:  # noqa: ANN001
        residual, gate, branch, weight, shift, scale, indices, eps = call
        return residual[:r], gate, branch[:r], weight, shift, scale, indices[:r], eps

    def fused(self, call, r, keep_row) -> tuple:  # noqa: ANN001
        sub = self._first(call, r)
        row = torch.empty_like(sub[0]) if keep_row else None
        return tuple(gate_rms_quant(*sub, self.orig, row)) + ((row,) if keep_row else ())

    def stock(self, call, r, keep_row, qobj) -> tuple:  # noqa: ANN001
        res, mod = self.orig(*self._first(call, r))
        return (res, *_stock_quant(qobj, mod)) + ((mod,) if keep_row else ())

    def produce(self, call, keep_row, qobj, layer) -> tuple:  # noqa: ANN001
        residual = call[0]
        ph = torch.empty_like(residual)
        res, q, s = gate_rms_quant(*call, self.orig, ph if keep_row else None)
        fill = (lambda t: None) if keep_row else (lambda t, c=call: t.copy_(self.orig(*c)[1]))
        return (res, ph), Pending("fc1", ph, residual.shape[1], q, s, qobj, layer, fill)


class _UnpackSite(_Site):
    """out: the reverse unpack of ``ulysses_exact.exchange_back`` (receive [P, M, hl, d] -> [1, M, H, d]): the quant
    reads the receive buffer, the model gets a placeholder of the unpacked shape."""
    name = "out"

    def accepts(self, sc, layer, call) -> bool:  # noqa: ANN001
        recv, heads = call
        ws, m, hl, d = recv.shape
        return (recv.dtype == torch.bfloat16 and recv.is_contiguous() and m > 0 and ws * hl == heads
                and ws & (ws - 1) == 0 and heads * d == _k_of(layer) and _fw.same_device(_state["device_types"], recv))

    def rows(self, call) -> int:  # noqa: ANN001
        return call[0].shape[1]

    def key(self, call) -> tuple:  # noqa: ANN001
        ws, _, hl, d = call[0].shape
        return ("out", ws, hl * d)

    def fused(self, call, r, keep_row) -> tuple:  # noqa: ANN001
        return unpack_quant(call[0][:, :r].contiguous())

    def stock(self, call, r, keep_row, qobj) -> tuple:  # noqa: ANN001
        recv, heads = call
        return _stock_quant(qobj, unpack_stock(recv[:, :r], heads)[0].reshape(r, heads * recv.shape[3]))

    def produce(self, call, keep_row, qobj, layer) -> tuple:  # noqa: ANN001
        recv, heads = call
        ws, m, hl, d = recv.shape
        q, s = unpack_quant(recv)
        ph = torch.empty((1, m, heads, d), dtype=recv.dtype, device=recv.device)
        return ph, Pending("out", ph, heads * d, q, s, qobj, layer,
                           lambda t: t[0].view(m, ws, hl, d).copy_(recv.transpose(0, 1)))


class _ActSite(_Site):
    """fc2: ``SiluAndMul.forward(self, x)`` of the MLP's activation on fc1's bf16 output."""
    name = "fc2"

    def __init__(self, orig):  # noqa: ANN001
        self.orig = orig

    def accepts(self, sc, layer, call) -> bool:  # noqa: ANN001
        act, x = call
        return (act is getattr(getattr(sc.block, "mlp", None), "act_fn", None) and isinstance(x, torch.Tensor)
                and _rows_ok(x, 2 * _k_of(layer)) and _fw.same_device(_state["device_types"], x))

    def rows(self, call) -> int:  # noqa: ANN001
        return call[1].shape[0]

    def key(self, call) -> tuple:  # noqa: ANN001
        return ("fc2", call[1].shape[1])

    def fused(self, call, r, keep_row) -> tuple:  # noqa: ANN001
        return silu_mul_quant(call[1][:r])

    def stock(self, call, r, keep_row, qobj) -> tuple:  # noqa: ANN001
        return _stock_quant(qobj, self.orig(call[0], call[1][:r]))

    def produce(self, call, keep_row, qobj, layer) -> tuple:  # noqa: ANN001
        act, x = call
        q, s = silu_mul_quant(x)
        ph = torch.empty((x.shape[0], x.shape[1] // 2), dtype=x.dtype, device=x.device)
        return ph, Pending("fc2", ph, x.shape[1] // 2, q, s, qobj, layer, lambda t: t.copy_(self.orig(act, x)))


def make_rms_wrapper(orig):  # noqa: ANN001,ANN201
    """``rms_norm_indexed_scale_shift`` with the qkv site (h3_tp2/fp8_quant_fuse.py:704)."""
    site = _NormSite(orig)

    def rms_norm_indexed_scale_shift(x, weight, shift, scale, indices, eps):  # noqa: ANN001,ANN202
        out = _serve(site, (x, weight, shift, scale, indices, eps))
        return orig(x, weight, shift, scale, indices, eps) if out is None else out

    rms_norm_indexed_scale_shift._h3b_quant_fuse = True
    return rms_norm_indexed_scale_shift


def make_gate_rms_wrapper(orig):  # noqa: ANN001,ANN201
    """``indexed_gate_rms_norm_scale_shift`` with the fc1 site (h3_tp2/fp8_quant_fuse.py:744)."""
    site = _GateNormSite(orig)

    def indexed_gate_rms_norm_scale_shift(residual, gate, branch, weight, shift, scale, indices, eps):  # noqa: ANN001,ANN202
        call = (residual, gate, branch, weight, shift, scale, indices, eps)
        out = _serve(site, call)
        return orig(*call) if out is None else out

    indexed_gate_rms_norm_scale_shift._h3b_quant_fuse = True
    return indexed_gate_rms_norm_scale_shift


_UNPACK = _UnpackSite()


def unpack_hook(recv: torch.Tensor, heads: int) -> torch.Tensor | None:
    """``ulysses_exact.exchange_back``'s reverse unpack with the out site (h3_tp2/fp8_quant_fuse.py:785): the
    placeholder [1, M, H, d], or None for the stock unpack."""
    return _serve(_UNPACK, (recv, heads))


def make_act_forward(orig):  # noqa: ANN001,ANN201
    """``SiluAndMul.forward`` with the fc2 site (h3_tp2/fp8_quant_fuse.py:810)."""
    site = _ActSite(orig)

    def forward(self, x):  # noqa: ANN001,ANN202
        out = _serve(site, (self, x))
        return orig(self, x) if out is None else out

    forward._h3b_quant_fuse = True
    return forward


_lora_types = _fw.lora_types


def install(sites: tuple[str, ...] = SITES, tr=None, *, quant_cls=None, act_cls=None, check_source: bool = True,  # noqa: ANN001
            lora_types=None, ulysses_mode: str | None = None, explicit: bool = False, level: str | None = None,
            env=None) -> list[str]:  # noqa: ANN001
    """Patch the transformer module ``tr`` (default: vLLM-Omni's MiniMax H3), ``QuantFP8.forward`` and
    ``SiluAndMul.forward`` for the given sites (h3_tp2/fp8_quant_fuse.py:923); returns the installed sites.  Skipped,
    with a warning, as the reference skips them: everything under ``VLLM_BATCH_INVARIANT``; out unless the exact
    exchange runs in mode 1 (mode 2 leaves the unpack to ``ulysses_outq``); fc1 when the consumer fuse owns
    ``indexed_gate_rms_norm_scale_shift``; fc2 below the ``cutlass`` GEMM level (fc1's output reaches ``SiluAndMul``
    only there); with ``check_source`` a site whose upstream code (``sources.QUANT_SITE_SOURCES``) is not the
    reviewed source.  ``explicit``: the sites were named, which only changes the wording of the out site's mode-2
    line.  ``level`` / ``env`` default to the installed GEMM level and the process environment."""
    import os  # noqa: PLC0415
    from . import fp8_consumers, fp8_gemm, sources  # noqa: PLC0415
    env = os.environ if env is None else env
    sites = tuple(site for site in SITES if site in sites)
    if not sites:
        return []
    if env.get("VLLM_BATCH_INVARIANT", "0").strip() not in ("", "0"):
        logger.warning("h3b fp8 quant fuse: VLLM_BATCH_INVARIANT changes the FP8 linear path; skipped")
        return []
    if tr is None:
        from vllm_omni.diffusion.models.minimax_h3 import minimax_h3_transformer as tr  # noqa: PLC0415
    if quant_cls is None:
        from vllm.model_executor.layers.quantization.input_quant_fp8 import QuantFP8 as quant_cls  # noqa: PLC0415
    if act_cls is None and "fc2" in sites:
        from vllm_omni.diffusion.layers.activation import SiluAndMul as act_cls  # noqa: PLC0415
    block_cls = tr.MiniMaxH3DiTBlock
    if getattr(block_cls.forward, "_h3b_quant_fuse", False):
        return list(_state["sites"])
    skip: dict[str, str] = {}
    if "out" in sites:
        mode = ulysses_mode
        if mode is None:
            try:
                from vllm_omni.diffusion.attention import layer as layer_mod  # noqa: PLC0415
                mode = getattr(layer_mod.Attention, "_h3b_exact", None)
            except ImportError:
                mode = None
        if mode == "2":
            logger.warning("h3b fp8 quant fuse: site out %s: the exact exchange's mode 2 makes no reverse unpack copy "
                           "to fuse into (the out-projection quant reads the receive buffer)",
                           "requested but ignored" if explicit else "skipped automatically")
            sites = tuple(site for site in sites if site != "out")
            if not sites:
                return []
        elif mode != "1":
            skip["out"] = f"needs the exact exchange in mode 1 (installed: {mode})"
    if "fc1" in sites and ("out" in fp8_consumers._state.get("sites", ()) or
                           getattr(tr.indexed_gate_rms_norm_scale_shift, "_h3b_consumer_fuse", False)):
        skip["fc1"] = "the consumer fuse's out site owns indexed_gate_rms_norm_scale_shift"
    level = fp8_gemm._state.get("level") if level is None else level
    if "fc2" in sites and level != "cutlass":
        skip["fc2"] = "fc1's output reaches SiluAndMul only at the cutlass GEMM level"
    if check_source:
        fps = sources.quant_fingerprints(tr)
        for site in sites:
            bad = [f"{n} {fps.get(n)} (reviewed {sources.quant_expected(n)})" for n in sources.QUANT_SITE_SOURCES[site]
                   if fps.get(n) != sources.quant_expected(n)]
            if bad and site not in skip:
                skip[site] = "upstream source changed: " + ", ".join(bad)
    for site, why in skip.items():
        logger.warning("h3b fp8 quant fuse: site %s skipped (%s)", site, why)
    sites = tuple(site for site in sites if site not in skip)
    if not sites:
        return []
    _state["quant_cls"] = quant_cls
    _state["act_cls"] = act_cls if "fc2" in sites else None
    if not getattr(quant_cls.forward, "_h3b_quant_fuse", False):
        _state["orig_quant"] = quant_cls.forward
        quant_cls.forward = make_quant_forward(quant_cls.forward)
    # the transformer-module producers of the qkv and fc1 sites, the activation class of fc2; the out site is a hook
    # of the exact exchange's reverse unpack
    for site, name, wrap in (("qkv", "rms_norm_indexed_scale_shift", make_rms_wrapper),
                             ("fc1", "indexed_gate_rms_norm_scale_shift", make_gate_rms_wrapper)):
        if site in sites:
            setattr(tr, name, wrap(getattr(tr, name)))
    if "fc2" in sites and not getattr(act_cls.forward, "_h3b_quant_fuse", False):
        act_cls.forward = make_act_forward(act_cls.forward)
    if "out" in sites:
        from . import ulysses_exact  # noqa: PLC0415
        ulysses_exact.set_unpack_hook(unpack_hook)
    block_cls.forward = make_block_forward(block_cls.forward, sites, _lora_types() if lora_types is None else lora_types)
    _state["sites"] = sites
    _state["verify"] = env.get("H3_TP2_FP8_QUANT_FUSE_VERIFY", "0").strip() == "1"
    mode = env.get("H3_TP2_FP8_QUANT_FUSE_MODE", "auto").strip().lower()
    _state["modes"] = {"0": (0,), "1": (1,)}.get(mode, (0, 1))
    return list(sites)
