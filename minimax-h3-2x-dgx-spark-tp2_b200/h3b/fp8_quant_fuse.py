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

import functools
import logging
import threading
from typing import Any, Callable

import torch

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
# the stash, the block context, the quant hook (h3_tp2/fp8_quant_fuse.py:404-860)
# --------------------------------------------------------------------------------------------------------------------

_SELFCHECK_ROWS = 64
_tls = threading.local()   # ctx: the _Ctx of the DiT block whose forward is running in this thread
_state: dict[str, Any] = {"sites": (), "checked": {}, "disabled": set(), "orig_quant": None, "quant_cls": None,
                          "act_cls": None, "verify": False, "modes": (0, 1), "device_types": ("cuda",)}
_stats: dict[str, int] = {k: 0 for k in ("fused_qkv", "fused_out", "fused_fc1", "fused_fc2", "consumed", "materialize",
                                         "rerun", "selfcheck_pass", "selfcheck_fail", "verify_calls", "verify_mismatch")}


def stats() -> dict[str, int]:
    return dict(_stats)


class Pending:
    """A producer's (fp8, scale) waiting for the quant of ``layer`` (h3_tp2/fp8_quant_fuse.py:432): ``ph`` is the bf16
    placeholder the model holds, ``k`` the GEMM input width (the quant sees ``ph`` as a contiguous [numel / k, k]
    view), ``fill(ph)`` runs the stock producer into the placeholder."""

    __slots__ = ("site", "ph", "k", "q", "scale", "quant", "layer", "fill")

    def __init__(self, site: str, ph: torch.Tensor, k: int, q: torch.Tensor, scale: torch.Tensor, quant, layer,  # noqa: ANN001
                 fill: Callable[[torch.Tensor], None]):
        self.site, self.ph, self.k, self.q, self.scale = site, ph, k, q, scale
        self.quant, self.layer, self.fill = quant, layer, fill

    def matches(self, quant_obj, x: torch.Tensor) -> bool:  # noqa: ANN001
        ph, k = self.ph, self.k
        return (quant_obj is self.quant and x.dim() == 2 and x.dtype == ph.dtype and x.device == ph.device
                and x.data_ptr() == ph.data_ptr() and tuple(x.shape) == (ph.numel() // k, k)
                and x.stride() == (k, 1) and ph.is_contiguous())

    def materialize(self) -> torch.Tensor:
        self.fill(self.ph)
        return self.ph


class _Ctx:
    __slots__ = ("block", "plan", "pending")

    def __init__(self, block, plan: dict):  # noqa: ANN001
        self.block, self.plan, self.pending = block, plan, None   # plan: site -> (layer, its quant instance)


def _materialize(ctx: _Ctx) -> None:
    p, ctx.pending = ctx.pending, None
    if p is not None:
        p.materialize()
        _stats["materialize"] += 1


def _bits(t: torch.Tensor) -> torch.Tensor:
    t = t.contiguous()
    return t.view({1: torch.uint8, 2: torch.int16, 4: torch.int32}[t.element_size()])


def _selfcheck(key, fused_fn, stock_fn, *, last: bool = True) -> bool:  # noqa: ANN001
    """Once per key: the fused outputs against the stock ones on the first rows, bit for bit; a failure of the ``last``
    candidate disables the site (key[0]) for the process."""
    ok = _state["checked"].get(key)
    if ok is not None:
        return ok
    try:
        fused, stock = fused_fn(), stock_fn()
        ok = len(fused) == len(stock) and all(f.shape == t.shape and f.dtype == t.dtype and torch.equal(_bits(f), _bits(t))
                                              for f, t in zip(fused, stock))
    except Exception:  # noqa: BLE001  (a failing fused kernel counts as a mismatch)
        ok = False
    _state["checked"][key] = ok
    _stats["selfcheck_pass" if ok else "selfcheck_fail"] += 1
    if not ok and last:
        _state["disabled"].add(key[0])
    return ok


def _pick_mode(key, fused_for, stock_fn):  # noqa: ANN001,ANN202
    """The RMS sites: mode 0 (the bf16 row only in registers) if it passes, else mode 1 (the bf16 row stored too);
    None when neither is bit-identical.  ``stock_fn()`` returns the stock outputs with the bf16 row last."""
    modes = _state["modes"]
    for m in modes:
        if _selfcheck(key + (m,), lambda: fused_for(m), lambda: stock_fn()[:None if m else -1], last=m == modes[-1]):
            return m
    return None


def _stock_quant(quant_obj, h: torch.Tensor):  # noqa: ANN001,ANN202
    """The layer's own per-token quant (the unwrapped ``QuantFP8.forward``), called as the linear kernel calls it."""
    return _state["orig_quant"](quant_obj, h, None, None)


def _verify(p: Pending) -> None:
    """``H3_TP2_FP8_QUANT_FUSE_VERIFY=1``: the stock pair on the whole tensor against the stash (counted)."""
    h = p.materialize()
    q_ref, s_ref = _stock_quant(p.quant, h.view(-1, p.k))
    _stats["verify_calls"] += 1
    if not (torch.equal(_bits(p.q), _bits(q_ref)) and torch.equal(_bits(p.scale), _bits(s_ref))):
        _stats["verify_mismatch"] += 1


def pending_placeholder(x: torch.Tensor) -> bool:
    """True when ``x`` is this thread's pending stash placeholder (h3_tp2/fp8_quant_fuse.py:545)."""
    ctx = getattr(_tls, "ctx", None)
    p = ctx.pending if ctx is not None else None
    return p is not None and x.data_ptr() == p.ph.data_ptr()


def make_quant_forward(orig):  # noqa: ANN001,ANN201
    """Wrap ``QuantFP8.forward`` (h3_tp2/fp8_quant_fuse.py:553): the pending stash's (fp8, scale) for exactly its planned
    instance and placeholder; every other call goes to ``orig`` untouched (after materialising a pending stash)."""
    def forward(self, x, *args, **kwargs):  # noqa: ANN001,ANN202
        if isinstance(x, torch.Tensor):
            from . import ulysses_outq  # noqa: PLC0415
            if ulysses_outq.is_placeholder(x):
                raise RuntimeError("h3b fp8 quant fuse: a deferred-unpack placeholder reached a quant outside the "
                                   "out-projection's")
        ctx = getattr(_tls, "ctx", None)
        p = ctx.pending if ctx is not None else None
        if p is not None:
            scale = args[0] if args else kwargs.get("scale")
            scale_ub = args[1] if len(args) > 1 else kwargs.get("scale_ub")
            if scale is None and scale_ub is None and isinstance(x, torch.Tensor) and p.matches(self, x):
                ctx.pending = None
                if _state["verify"]:
                    _verify(p)
                _stats["consumed"] += 1
                return p.q, p.scale
            _materialize(ctx)
        return orig(self, x, *args, **kwargs)

    forward._h3b_quant_fuse = True
    forward.__wrapped__ = orig
    return forward


def _layer_post_hook(module, args, output):  # noqa: ANN001,ANN202
    """A planned layer that returned without its quant consuming the stash ran on the placeholder: materialise it and
    run the layer again (h3_tp2/fp8_quant_fuse.py:575)."""
    ctx = getattr(_tls, "ctx", None)
    p = ctx.pending if ctx is not None else None
    if p is None or p.layer is not module:
        return None
    _materialize(ctx)
    _stats["rerun"] += 1
    return module.forward(*args)


def _quant_of(layer):  # noqa: ANN001,ANN202
    """The layer's dynamic per-token quant instance (``quant_method.fp8_linear.quant_fp8``), or None."""
    q = getattr(getattr(getattr(layer, "quant_method", None), "fp8_linear", None), "quant_fp8", None)
    cls = _state["quant_cls"]
    if cls is None or not isinstance(q, cls):
        return None
    if getattr(q, "static", True) or not getattr(q, "use_per_token_if_dynamic", False) \
            or getattr(q, "is_group_quant", True) or getattr(q, "num_token_padding", 0) is not None:
        return None
    if getattr(layer, "input_scale", None) is not None or getattr(layer, "input_scale_ub", None) is not None:
        return None
    return q


def block_plan(block, sites, lora_types=()) -> tuple[dict | None, str]:  # noqa: ANN001
    """{site: (layer, quant instance)} for this block, or (None, reason) (h3_tp2/fp8_quant_fuse.py:614)."""
    compiling = getattr(getattr(torch, "compiler", None), "is_compiling", None)
    if compiling is not None and compiling():
        return None, "torch.compile tracing"
    attn, mlp = getattr(block, "attn", None), getattr(block, "mlp", None)
    layers = {"qkv": getattr(attn, "qkv_proj", None), "out": getattr(attn, "out_proj", None),
              "fc1": getattr(mlp, "fc1", None), "fc2": getattr(mlp, "fc2", None)}
    plan: dict = {}
    for site in sites:
        if site in _state["disabled"]:
            continue
        layer = layers[site]
        if layer is None or (lora_types and isinstance(layer, lora_types)):
            return None, f"{site}: missing or LoRA-wrapped layer"
        if getattr(layer, "tp_size", 1) != 1:
            return None, f"{site}: tp_size != 1"
        q = _quant_of(layer)
        if q is None:
            return None, f"{site}: not a dynamic per-token FP8 linear"
        if site == "qkv" and getattr(attn, "to_gate_compress", None) is not None:
            continue                      # a VSA gate reads the qkv input a second time
        if site == "fc2" and _state["act_cls"] is not None and not isinstance(getattr(mlp, "act_fn", None),
                                                                              _state["act_cls"]):
            continue
        plan[site] = (layer, q)
        if not getattr(layer, "_h3b_quant_fuse_hook", False) and hasattr(layer, "register_forward_hook"):
            layer.register_forward_hook(_layer_post_hook)
            layer._h3b_quant_fuse_hook = True
    return (plan or None), "no site left"


def make_block_forward(orig_forward, sites, lora_types=()):  # noqa: ANN001,ANN201
    """Wrap the DiT block's forward: plan the sites, run the block with the context set, materialise a stash left at
    its end (h3_tp2/fp8_quant_fuse.py:646)."""
    @functools.wraps(orig_forward)
    def forward(self, *args, **kwargs):  # noqa: ANN001,ANN202
        plan, _ = block_plan(self, sites, lora_types)
        if plan is None:
            return orig_forward(self, *args, **kwargs)
        prev = getattr(_tls, "ctx", None)
        ctx = _Ctx(self, plan)
        _tls.ctx = ctx
        ok = False
        try:
            out = orig_forward(self, *args, **kwargs)
            ok = True
            return out
        finally:
            _tls.ctx = prev
            if ctx.pending is not None:
                if ok:
                    _materialize(ctx)
                ctx.pending = None

    forward._h3b_quant_fuse = True
    return forward


def _take_site(site: str):  # noqa: ANN202
    """The running block's context when ``site`` is planned there (a stash pending in front of it is materialised)."""
    ctx = getattr(_tls, "ctx", None)
    if ctx is None or site not in ctx.plan or site in _state["disabled"]:
        return None
    if ctx.pending is not None:
        _materialize(ctx)
    return ctx


def _device_ok(*ts: torch.Tensor) -> bool:
    dev = ts[0].device
    return all(t.device == dev for t in ts) and dev.type in _state["device_types"]


def _rows_ok(x: torch.Tensor, k: int, *others: torch.Tensor) -> bool:
    return (x.dim() == 2 and x.dtype == torch.bfloat16 and x.is_contiguous() and x.shape[0] > 0 and x.shape[1] == k
            and all(o.dim() == 2 and o.stride(1) == 1 for o in others))


def _k_of(layer) -> int:  # noqa: ANN001
    """The layer's input width (vLLM stores the weight [K, N])."""
    w = getattr(layer, "weight", None)
    return int(w.shape[0]) if isinstance(w, torch.Tensor) and w.dim() == 2 else -1


def make_rms_wrapper(orig):  # noqa: ANN001,ANN201
    """``rms_norm_indexed_scale_shift(x, weight, shift, scale, indices, eps)`` of the block's norm1: the qkv site
    (h3_tp2/fp8_quant_fuse.py:704)."""
    def rms_norm_indexed_scale_shift(x, weight, shift, scale, indices, eps):  # noqa: ANN001,ANN202
        ctx = _take_site("qkv")
        if ctx is not None:
            layer, qobj = ctx.plan["qkv"]
            if (weight is getattr(getattr(ctx.block, "norm1", None), "weight", None)
                    and _rows_ok(x, _k_of(layer), shift, scale) and indices.dim() == 1
                    and indices.shape[0] == x.shape[0] and _device_ok(x, weight, shift, scale, indices)):
                r = min(_SELFCHECK_ROWS, x.shape[0])

                def fused_rows(mode):  # noqa: ANN001,ANN202
                    ph_r = torch.empty_like(x[:r]) if mode else None
                    q_r, s_r = rms_quant(x[:r], weight, shift, scale, indices[:r], eps, orig, ph_r)
                    return (q_r, s_r) + ((ph_r,) if mode else ())

                def stock_rows():  # noqa: ANN202
                    h = orig(x[:r], weight, shift, scale, indices[:r], eps)
                    return (*_stock_quant(qobj, h), h)

                mode = _pick_mode(("qkv", x.shape[1], shift.dtype, weight.dtype), fused_rows, stock_rows)
                if mode is not None:
                    ph = torch.empty_like(x)
                    q, sc = rms_quant(x, weight, shift, scale, indices, eps, orig, ph if mode else None)

                    def fill(t, _a=(x, weight, shift, scale, indices, eps)):  # noqa: ANN001,ANN202
                        t.copy_(orig(*_a))
                    ctx.pending = Pending("qkv", ph, x.shape[1], q, sc, qobj, layer, (lambda t: None) if mode else fill)
                    _stats["fused_qkv"] += 1
                    return ph
        return orig(x, weight, shift, scale, indices, eps)

    rms_norm_indexed_scale_shift._h3b_quant_fuse = True
    return rms_norm_indexed_scale_shift


def make_gate_rms_wrapper(orig):  # noqa: ANN001,ANN201
    """``indexed_gate_rms_norm_scale_shift(residual, gate, branch, weight, shift, scale, indices, eps)`` of the block's
    norm2: the fc1 site (its modulated output feeds fc1; h3_tp2/fp8_quant_fuse.py:744)."""
    def indexed_gate_rms_norm_scale_shift(residual, gate, branch, weight, shift, scale, indices, eps):  # noqa: ANN001,ANN202
        ctx = _take_site("fc1")
        if ctx is not None:
            layer, qobj = ctx.plan["fc1"]
            if (weight is getattr(getattr(ctx.block, "norm2", None), "weight", None)
                    and _rows_ok(residual, _k_of(layer), gate, branch, shift, scale)
                    and branch.shape == residual.shape and branch.dtype == residual.dtype
                    and indices.dim() == 1 and indices.shape[0] == residual.shape[0]
                    and _device_ok(residual, gate, branch, weight, shift, scale, indices)):
                r = min(_SELFCHECK_ROWS, residual.shape[0])

                def fused_rows(mode):  # noqa: ANN001,ANN202
                    ph_r = torch.empty_like(residual[:r]) if mode else None
                    out = gate_rms_quant(residual[:r], gate, branch[:r], weight, shift, scale, indices[:r], eps, orig,
                                         ph_r)
                    return tuple(out) + ((ph_r,) if mode else ())

                def stock_rows():  # noqa: ANN202
                    res, mod = orig(residual[:r], gate, branch[:r], weight, shift, scale, indices[:r], eps)
                    return (res, *_stock_quant(qobj, mod), mod)

                mode = _pick_mode(("fc1", residual.shape[1], gate.dtype, weight.dtype), fused_rows, stock_rows)
                if mode is not None:
                    ph = torch.empty_like(residual)
                    res, q, sc = gate_rms_quant(residual, gate, branch, weight, shift, scale, indices, eps, orig,
                                                ph if mode else None)

                    def fill(t, _a=(residual, gate, branch, weight, shift, scale, indices, eps)):  # noqa: ANN001,ANN202
                        t.copy_(orig(*_a)[1])
                    ctx.pending = Pending("fc1", ph, residual.shape[1], q, sc, qobj, layer,
                                          (lambda t: None) if mode else fill)
                    _stats["fused_fc1"] += 1
                    return res, ph
        return orig(residual, gate, branch, weight, shift, scale, indices, eps)

    indexed_gate_rms_norm_scale_shift._h3b_quant_fuse = True
    return indexed_gate_rms_norm_scale_shift


def unpack_hook(recv: torch.Tensor, heads: int) -> torch.Tensor | None:
    """The reverse unpack of ``ulysses_exact.exchange_back`` (the out site, h3_tp2/fp8_quant_fuse.py:785): a placeholder
    [1, M, H, d] with the quant of the unpacked rows stashed, or None for the stock unpack."""
    ctx = _take_site("out")
    if ctx is None:
        return None
    layer, qobj = ctx.plan["out"]
    ws, m, hl, d = recv.shape
    if (recv.dtype != torch.bfloat16 or not recv.is_contiguous() or m == 0 or ws * hl != heads or ws & (ws - 1)
            or heads * d != _k_of(layer) or not _device_ok(recv)):
        return None
    r = min(_SELFCHECK_ROWS, m)
    if not _selfcheck(("out", ws, hl * d), lambda: unpack_quant(recv[:, :r].contiguous()),
                      lambda: _stock_quant(qobj, unpack_stock(recv[:, :r], heads)[0].reshape(r, heads * d))):
        return None
    q, sc = unpack_quant(recv)
    ph = torch.empty((1, m, heads, d), dtype=recv.dtype, device=recv.device)

    def fill(t, _recv=recv):  # noqa: ANN001,ANN202
        t[0].view(m, ws, hl, d).copy_(_recv.transpose(0, 1))
    ctx.pending = Pending("out", ph, heads * d, q, sc, qobj, layer, fill)
    _stats["fused_out"] += 1
    return ph


def make_act_forward(orig):  # noqa: ANN001,ANN201
    """``SiluAndMul.forward`` (the MLP's act_fn on fc1's bf16 output): the fc2 site (h3_tp2/fp8_quant_fuse.py:810)."""
    def forward(self, x):  # noqa: ANN001,ANN202
        ctx = _take_site("fc2")
        if ctx is not None and self is getattr(getattr(ctx.block, "mlp", None), "act_fn", None):
            layer, qobj = ctx.plan["fc2"]
            if isinstance(x, torch.Tensor) and _rows_ok(x, 2 * _k_of(layer)) and _device_ok(x):
                r = min(_SELFCHECK_ROWS, x.shape[0])
                if _selfcheck(("fc2", x.shape[1]), lambda: silu_mul_quant(x[:r]),
                              lambda: _stock_quant(qobj, orig(self, x[:r]))):
                    q, sc = silu_mul_quant(x)
                    ph = torch.empty((x.shape[0], x.shape[1] // 2), dtype=x.dtype, device=x.device)

                    def fill(t, _x=x, _m=self):  # noqa: ANN001,ANN202
                        t.copy_(orig(_m, _x))
                    ctx.pending = Pending("fc2", ph, x.shape[1] // 2, q, sc, qobj, layer, fill)
                    _stats["fused_fc2"] += 1
                    return ph
        return orig(self, x)

    forward._h3b_quant_fuse = True
    return forward


def _lora_types() -> tuple:
    try:
        from vllm.lora.layers import BaseLayerWithLoRA  # noqa: PLC0415
        return (BaseLayerWithLoRA,)
    except ImportError:
        return ()


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
    if "qkv" in sites:
        tr.rms_norm_indexed_scale_shift = make_rms_wrapper(tr.rms_norm_indexed_scale_shift)
    if "fc1" in sites:
        tr.indexed_gate_rms_norm_scale_shift = make_gate_rms_wrapper(tr.indexed_gate_rms_norm_scale_shift)
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
