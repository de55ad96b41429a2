"""Consumers of an FP8 GEMM's output fused with the GEMM (mirror of ``h3_tp2/fp8_consumers.py``).

The reference keeps the fp32 product of the qkv / out / fc2 GEMMs (a "stash", ``Stash`` :388) and replaces the kernel
that consumes each bf16 output with a copy that applies the scale pass's arithmetic itself, so the bf16 [M, N]
intermediate is never written.  On B200 the consumer's arithmetic runs in the GEMM's own epilogue instead, so not even
the fp32 product reaches HBM: a ``Stash`` here holds the GEMM's operands, and each consumer launches one kernel.

* ``qk_norm_rope_fused`` (:406): q and k RMSNorm + partial RoPE and the v scale pass — the qkv GEMM with the
  norm + RoPE epilogue (``h3b_fp8_gemm`` with ``H3B_EPI_QKV_SEND`` and norm weights, P = 1 layout = [M, H, d]).
* ``gate_fused`` (:468): ``x + gate[indices] * fc2`` — the fc2 GEMM with the indexed-gate epilogue
  (``h3b_fp8_gemm_gate``).
* ``gate_rms_fused`` (:445) has no one-kernel form (the RMS needs whole rows of the out projection, the GEMM works
  on 256-column tiles): it materialises the out projection, runs the gated residual + RMSNorm + modulation row kernel
  for ``residual_out`` and the RMSNorm + modulation row kernel on that for the bf16 modulated rows.

The wiring into the model is the reference's protocol (:498-919): inside a planned DiT block (``make_block_forward``,
``block_plan``) the FP8 GEMM dispatcher's stash hook (``stash_hook``) keeps the operands of the qkv / out / fc2 GEMMs
and returns an uninitialised bf16 placeholder; the wrapped consumer (``make_qk_wrapper``, ``make_gate_rms_wrapper``,
``make_gate_wrapper``) recognises its placeholder (``qk_mismatch`` / ``rows_mismatch`` give the reason when not) and
runs the fused consumer instead.  A stash any other call meets first is materialised (the GEMM run into the
placeholder), and the first call per site and width is compared bit for bit on its first rows with the plain GEMM +
the stock consumer; a mismatch disables the site for the process.
"""
from __future__ import annotations

import functools
import logging
import threading
from typing import Any

import torch

from . import ops

logger = logging.getLogger("h3b.fp8_consumers")

SITES = ("qkv", "out", "fc2")


class Stash:
    """The operands of one FP8 GEMM whose output a fused consumer reads (reference ``Stash``: the fp32 product)."""
    __slots__ = ("a", "w", "sa", "sb", "bias", "ph")

    def __init__(self, a: torch.Tensor, w: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor,
                 bias: torch.Tensor | None, ph: torch.Tensor | None = None):
        self.a, self.w, self.sa, self.sb, self.bias, self.ph = a, w, sa, sb, bias, ph

    def materialize(self) -> torch.Tensor:
        """The ordinary bf16 output (into the placeholder when one was given)."""
        if self.ph is None:
            return torch.ops.h3b.fp8_gemm(self.a, self.w, self.sa, self.sb, self.bias, torch.bfloat16)
        torch.ops.h3b.fp8_gemm_out(self.a, self.w, self.sa, self.sb, self.bias, self.ph)
        return self.ph

    def rows(self, r: int) -> "Stash":
        return Stash(self.a[:r], self.w, self.sa[:r], self.sb, self.bias, None)


def qk_norm_rope_fused(st: Stash, num_heads: int, num_kv_heads: int, head_dim: int, q_weight: torch.Tensor,
                       k_weight: torch.Tensor, rope_table: torch.Tensor, eps: float):
    """(q, k, v) [T, H, d] bf16: per-head RMSNorm + partial RoPE (rotary dims = rope_table's width, cos | sin) on q
    and k, v scale-passed, all in the qkv GEMM's epilogue."""
    if num_kv_heads != num_heads or head_dim != 128:
        raise ValueError("qk_norm_rope_fused: equal q/kv heads of 128 dims only")
    if st.bias is not None:
        raise ValueError("qk_norm_rope_fused: the norm epilogue takes no bias")
    q, k, v = ops.fp8_gemm_qkv_send(st.a, st.w, st.sa, st.sb, num_heads, 1,
                                    qk_norm=(q_weight, k_weight, rope_table.float(), eps))
    T = st.a.shape[0]
    return tuple(t.view(T, num_heads, head_dim) for t in (q, k, v))


def qkv_into_send(st: Stash, num_heads: int, ws: int, q_weight: torch.Tensor, k_weight: torch.Tensor,
                  rope_table: torch.Tensor, eps: float, sends=None):  # noqa: ANN001
    """The qkv GEMM of ``st`` with the norm + RoPE epilogue writing per destination (the producer ``ulysses_exact``'s
    redirection uses; h3_tp2/ulysses_exact.py:278 ``fused_into_send``): (send_q, send_k, send_v) [P, M, H/P, 128] bf16,
    q and k normalised and rotated, v the plain scale pass; into ``sends`` when given."""
    return ops.fp8_gemm_qkv_send(st.a, st.w, st.sa, st.sb, num_heads, ws, sends=sends,
                                 qk_norm=(q_weight, k_weight, rope_table.float(), eps))


def gate_fused(st: Stash, x: torch.Tensor, gate: torch.Tensor, indices: torch.Tensor,
               reuse_placeholder: bool = True) -> torch.Tensor:
    """``indexed_gate(x, gate, fc2_output, indices)`` with the fc2 GEMM: written into the placeholder when ``x`` is
    contiguous (stock: ``empty_like(x)``)."""
    out = st.ph if (reuse_placeholder and st.ph is not None and x.is_contiguous()) else None
    if x.shape[0] == 0:
        return out if out is not None else torch.empty_like(x)
    if out is None:
        return torch.ops.h3b.fp8_gemm_gate(st.a, st.w, st.sa, st.sb, x, gate, indices, st.bias)
    torch.ops.h3b.fp8_gemm_gate_out(st.a, st.w, st.sa, st.sb, x, gate, indices, st.bias, out)
    return out


def gate_rms_fused(st: Stash, residual: torch.Tensor, gate: torch.Tensor, weight: torch.Tensor, shift: torch.Tensor,
                   scale: torch.Tensor, indices: torch.Tensor, eps: float, reuse_placeholder: bool = True):
    """``indexed_gate_rms_norm_scale_shift(residual, gate, branch, ...)`` with branch = the out projection of ``st``
    (h3_tp2/fp8_consumers.py:445): returns (residual_out = bf16(residual + gate[indices] * branch), modulated_out =
    bf16 RMSNorm(residual_out) * weight * (1 + scale[indices]) + shift[indices]); ``residual_out`` goes into the
    placeholder when ``reuse_placeholder`` and the stash has one."""
    rows = residual.shape[0]
    residual_out = st.ph if (reuse_placeholder and st.ph is not None) else torch.empty_like(residual)
    modulated_out = torch.empty_like(residual)
    if rows == 0:
        return residual_out, modulated_out
    branch = torch.ops.h3b.fp8_gemm(st.a, st.w, st.sa, st.sb, st.bias, torch.bfloat16)
    r_out, _, _ = torch.ops.h3b.gate_rms_quant(residual, gate, branch, weight, shift, scale, indices, float(eps))
    torch.ops.h3b.rms_quant(r_out, weight, shift, scale, indices, float(eps), modulated_out)
    if residual_out is not r_out:
        residual_out.copy_(r_out)
    return residual_out, modulated_out


def epilogue_bf16_torch(acc: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    """The bf16 epilogue in eager torch on broadcastable fp32 tensors (h3_tp2/fp8_consumers.py:305): column scale,
    row scale (bias by an fma carried out in float64), rounded to bf16 and returned as fp32."""
    t = sb * acc
    y = sa * t if bias is None else (sa.double() * t.double() + bias.double()).float()
    return y.to(torch.bfloat16).float()


def scale_pass_into(x32: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, bias: torch.Tensor | None,
                    y: torch.Tensor) -> torch.Tensor:
    """The ordinary two-pass scale pass into ``y`` (h3_tp2/fp8_consumers.py:373): the scale-pass kernel on the GPU.
    CPU tensors raise (the reference's eager CPU branch is ``fp8_gemm.epilogue_torch``, called explicitly)."""
    y.copy_(ops.scale_bias_cast(x32, sa, sb, bias, y.dtype))
    return y


def parse_sites(value: str | None) -> tuple[str, ...]:
    """``H3_TP2_FP8_CONSUMER_FUSE`` (h3_tp2/fp8_consumers.py:813): "1"/"all"/"on"/"true" = every site, a comma list of
    qkv,out,fc2 selects sites, anything else or empty = none."""
    v = (value or "").strip().lower()
    if v in ("1", "all", "on", "true"):
        return SITES
    if v in ("", "0", "off", "false"):
        return ()
    chosen = {part.strip() for part in v.split(",")}
    return tuple(site for site in SITES if site in chosen)


# --------------------------------------------------------------------------------------------------------------------
# the wiring: stash hook, block plan, consumer wrappers (h3_tp2/fp8_consumers.py:498-919)
# --------------------------------------------------------------------------------------------------------------------

_SELFCHECK_ROWS = 64
_ROTARY_DIMS = (32, 64, 96, 128)      # what the norm + RoPE epilogue rotates (the reference's Triton copy: 96 only)
_tls = threading.local()              # ctx: the _Ctx of the DiT block whose forward is running in this thread
_state: dict[str, Any] = {"sites": (), "checked": {}, "disabled": set(), "device_types": ("cuda",)}
_stats: dict[str, int] = {k: 0 for k in ("stash", "materialize", "fused_qkv", "fused_out", "fused_fc2",
                                         "selfcheck_pass", "selfcheck_fail")}
_warned: set = set()


def stats() -> dict[str, int]:
    return dict(_stats)


def _warn_once(key: str, msg: str, *args) -> None:  # noqa: ANN002
    if key not in _warned:
        _warned.add(key)
        logger.warning("h3b fp8 consumer fuse: " + msg, *args)


class _Ctx:
    __slots__ = ("want", "pending")

    def __init__(self, want: dict):
        self.want = want                            # (weight data_ptr, weight shape) -> site
        self.pending: dict[str, Stash] = {}


def _vec(scale: torch.Tensor, n: int) -> torch.Tensor:
    s = scale.reshape(-1).float()
    return (s.expand(n) if s.numel() == 1 else s).contiguous()


def stash_hook(a, b, scale_a, scale_b, out_dtype, bias):  # noqa: ANN001,ANN201
    """FP8 GEMM dispatcher hook (:531): when ``b`` ([K, N], the layer's stored weight) is the qkv / out / fc2 weight of
    the running DiT block, keep the GEMM's operands and return an uninitialised bf16 placeholder for the consumer."""
    ctx = getattr(_tls, "ctx", None)
    if ctx is None or out_dtype is not torch.bfloat16:
        return None
    site = ctx.want.pop((b.data_ptr(), tuple(b.shape)), None)
    if site is None:
        return None
    if ctx.pending:                       # a stash that was never consumed: make it real before the next one
        _materialize_all(ctx, f"unconsumed stash before {site}")
    M, N = a.shape[0], b.shape[1]
    ph = torch.empty((M, N), device=a.device, dtype=out_dtype)
    ctx.pending[site] = Stash(a, b.t(), _vec(scale_a, M), _vec(scale_b, N), bias, ph)
    _stats["stash"] += 1
    return ph


def _materialize_all(ctx: _Ctx, reason: str) -> None:
    for site, st in list(ctx.pending.items()):
        st.materialize()
        _stats["materialize"] += 1
        _warn_once("mat-" + reason, "%s: stash of %s materialised, stock consumer", reason, site)
    ctx.pending.clear()


def _bits(t: torch.Tensor) -> torch.Tensor:
    t = t.contiguous()
    return t.view({1: torch.uint8, 2: torch.int16, 4: torch.int32}[t.element_size()])


def _selfcheck(key, fused_fn, stock_fn) -> bool:  # noqa: ANN001
    """Once per (site, shape): fused against the plain GEMM + stock consumer on the first rows, bit for bit; a mismatch
    (or a raising fused kernel) disables the site for the process (:561)."""
    ok = _state["checked"].get(key)
    if ok is not None:
        return ok
    try:
        fused, stock = fused_fn(), stock_fn()
        ok = len(fused) == len(stock) and all(f.shape == t.shape and f.dtype == t.dtype
                                              and torch.equal(_bits(f), _bits(t)) for f, t in zip(fused, stock))
    except Exception as exc:  # noqa: BLE001
        logger.warning("h3b fp8 consumer fuse: self-check %s raised %s", key, exc)
        ok = False
    _state["checked"][key] = ok
    _stats["selfcheck_pass" if ok else "selfcheck_fail"] += 1
    if not ok:
        _state["disabled"].add(key[0])
        logger.warning("h3b fp8 consumer fuse: self-check %s not bit-identical to the GEMM + stock consumer; site %s "
                       "disabled for this process", key, key[0])
    return ok


def _device_ok(*ts: torch.Tensor) -> bool:
    dev = ts[0].device
    return all(t.device == dev for t in ts) and dev.type in _state["device_types"]


def _stash_ok(st: Stash) -> bool:
    ph = st.ph
    return (ph is not None and ph.dim() == 2 and ph.is_contiguous() and ph.dtype == torch.bfloat16
            and st.a.shape[0] == ph.shape[0] and st.w.shape[0] == ph.shape[1])


def qk_mismatch(st: Stash, q, k, q_weight, k_weight, rope_table, head_dim, rotary_dim, interleaved) -> str | None:  # noqa: ANN001
    """None when (q, k) are exactly the q/k views of the stash's placeholder and the norm + RoPE epilogue covers the
    call (:591), else the reason."""
    ph = st.ph
    if interleaved:
        return "interleaved"
    if q.dim() != 3 or k.dim() != 3 or q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16:
        return "q/k rank or dtype"
    T, H, D = q.shape
    Hk = k.shape[1]
    if ph is None or T == 0 or ph.dim() != 2 or ph.shape[0] != T or k.shape != (T, Hk, D) \
            or ph.shape[1] != (H + 2 * Hk) * D:
        return "shapes"
    if Hk != H:
        return "grouped kv heads"
    if not _stash_ok(st):
        return "placeholder/operand layout"
    eq, ek = ph[:, :H * D].view(T, H, D), ph[:, H * D:(H + Hk) * D].view(T, Hk, D)   # upstream's split + view
    if q.data_ptr() != eq.data_ptr() or k.data_ptr() != ek.data_ptr() or q.stride() != eq.stride() \
            or k.stride() != ek.stride():
        return "q/k are not the split views of the qkv placeholder"
    if D != 128 or head_dim not in (None, D):
        return "head_dim"
    rot = rope_table.shape[-1] if rope_table.dim() == 2 else -1
    if rot not in _ROTARY_DIMS or rotary_dim not in (None, rot) or rope_table.shape != (T, rot):
        return "rotary"
    if rope_table.dtype not in (torch.bfloat16, torch.float32) or q_weight.shape != (D,) or k_weight.shape != (D,) \
            or q_weight.dtype != torch.bfloat16 or k_weight.dtype != torch.bfloat16:
        return "rope table or norm weight dtype/shape"
    if st.bias is not None:
        return "bias (the norm epilogue has none)"
    if not _device_ok(q, k, q_weight, k_weight, rope_table, st.a):
        return "device"
    return None


def rows_mismatch(st: Stash, x: torch.Tensor, branch: torch.Tensor, *others: torch.Tensor) -> str | None:
    """None when ``branch`` is exactly the stash's placeholder and ``x`` (the residual) a contiguous bf16 tensor of the
    same shape on the same device as the other operands (gate / shift / scale, then the indices last) (:622)."""
    ph = st.ph
    if ph is None or branch.data_ptr() != ph.data_ptr() or branch.shape != ph.shape or branch.stride() != ph.stride():
        return "branch is not the placeholder"
    if x.dim() != 2 or x.shape != ph.shape or x.dtype != torch.bfloat16 or not x.is_contiguous() \
            or not _stash_ok(st):
        return "residual shape/dtype/layout"
    if x.shape[0] == 0:
        return "no rows"
    if any(o.dim() != 2 or o.stride(1) != 1 or o.dtype != torch.bfloat16 or o.shape[1] != x.shape[1]
           for o in others[:-1]):
        return "gate/shift/scale layout"
    if others[-1].dim() != 1 or others[-1].shape[0] != x.shape[0]:
        return "indices"
    if not _device_ok(x, st.a, *others):
        return "device"
    return None


def _take(site: str):  # noqa: ANN202
    ctx = getattr(_tls, "ctx", None)
    if ctx is None or not ctx.pending:
        return ctx, None
    st = ctx.pending.get(site)
    if st is None:
        _materialize_all(ctx, f"{site} consumer saw another site's stash")
    return ctx, st


def make_qk_wrapper(orig):  # noqa: ANN001,ANN201
    """Wrap the transformer's ``fused_qk_norm_rope`` (:652): on the qkv stash's q/k views, the qkv GEMM with the norm +
    RoPE epilogue (``qk_norm_rope_fused``, looked up at call time so the Ulysses producer can replace it)."""
    def fused_qk_norm_rope(q, k, q_weight, k_weight, rope_table, eps, *, head_dim=None, rotary_dim=None,  # noqa: ANN001,ANN202
                           interleaved=False):
        ctx, st = _take("qkv")
        if st is not None:
            reason = "qkv disabled by self-check" if "qkv" in _state["disabled"] else \
                qk_mismatch(st, q, k, q_weight, k_weight, rope_table, head_dim, rotary_dim, interleaved)
            if reason is None:
                H, Hk, D = q.shape[1], k.shape[1], q.shape[-1]
                r = min(_SELFCHECK_ROWS, q.shape[0])

                def _fused_sub():  # noqa: ANN202
                    return qk_norm_rope_fused(st.rows(r), H, Hk, D, q_weight, k_weight, rope_table[:r], eps)

                def _stock_sub():  # noqa: ANN202
                    p = st.rows(r).materialize()
                    qs, ks = p[:, :H * D].view(r, H, D), p[:, H * D:(H + Hk) * D].view(r, Hk, D)
                    oq, ok_ = orig(qs, ks, q_weight, k_weight, rope_table[:r], eps, head_dim=head_dim,
                                   rotary_dim=rotary_dim, interleaved=interleaved)
                    return oq, ok_, p[:, (H + Hk) * D:].view(r, Hk, D)

                if not _selfcheck(("qkv", tuple(st.ph.shape[1:]), rope_table.dtype), _fused_sub, _stock_sub):
                    reason = "qkv disabled by self-check"
            if reason is None:
                del ctx.pending["qkv"]
                out_q, out_k, v = qk_norm_rope_fused(st, H, Hk, D, q_weight, k_weight, rope_table, eps)
                v_view = st.ph[:, (H + Hk) * D:].view(q.shape[0], Hk, D)
                if v.data_ptr() != v_view.data_ptr():
                    v_view.copy_(v)       # the model reads v from its own view of the placeholder
                _stats["fused_qkv"] += 1
                return out_q, out_k
            _materialize_all(ctx, "qkv: " + reason)
        return orig(q, k, q_weight, k_weight, rope_table, eps, head_dim=head_dim, rotary_dim=rotary_dim,
                    interleaved=interleaved)

    fused_qk_norm_rope._h3b_consumer_fuse = True
    return fused_qk_norm_rope


def make_gate_rms_wrapper(orig):  # noqa: ANN001,ANN201
    """Wrap ``indexed_gate_rms_norm_scale_shift`` (:688): on the out stash's placeholder, ``gate_rms_fused``."""
    def indexed_gate_rms_norm_scale_shift(residual, gate, branch, weight, shift, scale, indices, eps):  # noqa: ANN001,ANN202
        ctx, st = _take("out")
        if st is not None:
            reason = "out disabled by self-check" if "out" in _state["disabled"] else \
                rows_mismatch(st, residual, branch, gate, shift, scale, indices)
            if reason is None and (weight.shape != (residual.shape[1],) or weight.device != residual.device
                                   or weight.dtype != torch.bfloat16):
                reason = "norm weight shape/device/dtype"
            if reason is None:
                r = min(_SELFCHECK_ROWS, residual.shape[0])

                def _fused_sub():  # noqa: ANN202
                    return gate_rms_fused(st.rows(r), residual[:r], gate, weight, shift, scale, indices[:r], eps)

                def _stock_sub():  # noqa: ANN202
                    p = st.rows(r).materialize()
                    return orig(residual[:r], gate, p, weight, shift, scale, indices[:r], eps)

                if not _selfcheck(("out", tuple(residual.shape[1:]), gate.dtype, weight.dtype), _fused_sub,
                                  _stock_sub):
                    reason = "out disabled by self-check"
            if reason is None:
                del ctx.pending["out"]
                res = gate_rms_fused(st, residual, gate, weight, shift, scale, indices, eps)
                _stats["fused_out"] += 1
                return res
            _materialize_all(ctx, "out: " + reason)
        return orig(residual, gate, branch, weight, shift, scale, indices, eps)

    indexed_gate_rms_norm_scale_shift._h3b_consumer_fuse = True
    return indexed_gate_rms_norm_scale_shift


def make_gate_wrapper(orig):  # noqa: ANN001,ANN201
    """Wrap ``indexed_gate`` (:720): on the fc2 stash's placeholder, the fc2 GEMM with the indexed-gate epilogue."""
    def indexed_gate(x, gate, other, indices):  # noqa: ANN001,ANN202
        ctx, st = _take("fc2")
        if st is not None:
            reason = "fc2 disabled by self-check" if "fc2" in _state["disabled"] else \
                rows_mismatch(st, x, other, gate, indices)
            if reason is None:
                r = min(_SELFCHECK_ROWS, x.shape[0])

                def _fused_sub():  # noqa: ANN202
                    return (gate_fused(st.rows(r), x[:r].contiguous(), gate, indices[:r], reuse_placeholder=False),)

                def _stock_sub():  # noqa: ANN202
                    p = st.rows(r).materialize()
                    return (orig(x[:r].contiguous(), gate, p, indices[:r]),)

                if not _selfcheck(("fc2", tuple(x.shape[1:]), gate.dtype), _fused_sub, _stock_sub):
                    reason = "fc2 disabled by self-check"
            if reason is None:
                del ctx.pending["fc2"]
                out = gate_fused(st, x, gate, indices)
                _stats["fused_fc2"] += 1
                return out
            _materialize_all(ctx, "fc2: " + reason)
        return orig(x, gate, other, indices)

    indexed_gate._h3b_consumer_fuse = True
    return indexed_gate


def _lora_types():  # noqa: ANN202
    try:
        from vllm.lora.layers import BaseLayerWithLoRA  # noqa: PLC0415
        return (BaseLayerWithLoRA,)
    except ImportError:
        return ()


def block_plan(block, rope_table, sites, lora_types=()) -> tuple[dict | None, str]:  # noqa: ANN001
    """{(weight data_ptr, weight shape): site} for this block's eligible GEMMs, or (None, reason) (:758)."""
    if rope_table is None:
        return None, "no rope table (q/k norm without fused rope)"
    compiling = getattr(getattr(torch, "compiler", None), "is_compiling", None)
    if compiling is not None and compiling():
        return None, "torch.compile tracing"
    attn, mlp = getattr(block, "attn", None), getattr(block, "mlp", None)
    layers = {"qkv": getattr(attn, "qkv_proj", None), "out": getattr(attn, "out_proj", None),
              "fc2": getattr(mlp, "fc2", None)}
    want: dict = {}
    for site in sites:
        if site in _state["disabled"]:
            continue
        layer = layers[site]
        if layer is None or (lora_types and isinstance(layer, lora_types)):
            return None, f"{site}: missing or LoRA-wrapped layer"
        if getattr(layer, "tp_size", 1) != 1:
            return None, f"{site}: tp_size != 1 (an all-reduce would read the placeholder)"
        w = getattr(layer, "weight", None)
        n = int(getattr(layer, "output_size_per_partition", 0) or 0)
        if not isinstance(w, torch.Tensor) or w.dtype != torch.float8_e4m3fn or w.dim() != 2 or w.shape[1] != n:
            return None, f"{site}: weight is not an unpadded FP8 [K, N] tensor"
        want[(w.data_ptr(), tuple(w.shape))] = site
    return (want or None), "no site left"


def make_block_forward(orig_forward, sites, lora_types=()):  # noqa: ANN001,ANN201
    """Wrap the DiT block's forward (:787): plan the sites, run the block with the context set, materialise a stash
    left at its end."""
    @functools.wraps(orig_forward)
    def forward(self, *args, **kwargs):  # noqa: ANN001,ANN202
        want, reason = block_plan(self, kwargs.get("rope_table"), sites, lora_types)
        if want is None:
            _warn_once("plan-" + reason, "block not fused (%s); stock path", reason)
            return orig_forward(self, *args, **kwargs)
        prev = getattr(_tls, "ctx", None)
        ctx = _Ctx(want)
        _tls.ctx = ctx
        ok = False
        try:
            out = orig_forward(self, *args, **kwargs)
            ok = True
            return out
        finally:
            _tls.ctx = prev
            if ctx.pending:
                if ok:   # make the placeholder real for whoever holds it
                    _materialize_all(ctx, "stash left at the end of the block")
                ctx.pending.clear()

    forward._h3b_consumer_fuse = True
    return forward


def install(sites: tuple[str, ...] = SITES, tr=None, *, check_source: bool = True, lora_types=None,  # noqa: ANN001
            level: str | None = None, nocopy: bool | None = None) -> list[str]:
    """Patch the transformer module ``tr`` (default: vLLM-Omni's MiniMax H3 transformer) for the given sites and
    register the stash hook (:859).  Returns the installed sites.  At the ``cutlass`` GEMM level the qkv / out GEMMs
    are routed by weight ahead of the stash hook (as the reference's DSL kernel is), so those consumers stay stock;
    beside the combined (nocopy) exchange the qkv site is skipped; with ``check_source`` a site whose upstream code
    (``sources.CONSUMER_SITE_SOURCES``) is not the reviewed source is skipped.  ``level`` / ``nocopy`` default to the
    installed state."""
    from . import fp8_gemm, sources  # noqa: PLC0415
    sites = tuple(s for s in SITES if s in sites)
    if not sites:
        return []
    level = fp8_gemm._state.get("level") if level is None else level
    if level not in ("tensor32", "cutlass"):
        logger.warning("h3b fp8 consumer fuse: needs the FP8 GEMM dispatcher at the tensor32 or cutlass level "
                       "(running: %s); skipped", level)
        return []
    if level == "cutlass":
        from .fp8_cutlass import SITES as routed  # noqa: PLC0415
        dropped = [s for s in sites if s in routed]
        sites = tuple(s for s in sites if s not in routed)
        if dropped:
            logger.warning("h3b fp8 consumer fuse: the cutlass level routes %s by weight; those consumers stay stock, "
                           "fused sites: %s", ", ".join(dropped), ", ".join(sites) or "none")
        if not sites:
            return []
    if tr is None:
        from vllm_omni.diffusion.models.minimax_h3 import minimax_h3_transformer as tr  # noqa: PLC0415
    block_cls = tr.MiniMaxH3DiTBlock
    if getattr(block_cls.forward, "_h3b_consumer_fuse", False):
        return list(_state["sites"])
    if nocopy is None:
        try:
            from vllm_omni.diffusion.attention import layer as layer_mod  # noqa: PLC0415
            nocopy = bool(getattr(layer_mod.Attention, "_h3b_nocopy", 0))
        except ImportError:
            nocopy = False
    if "qkv" in sites and nocopy:
        logger.warning("h3b fp8 consumer fuse: the Ulysses nocopy exchange wraps the rope producer; qkv site skipped")
        sites = tuple(s for s in sites if s != "qkv")
    if check_source:
        fps = sources.consumer_fingerprints(tr)
        keep = []
        for site in sites:
            bad = sources.changed(sources.CONSUMER_SITE_SOURCES[site], fps, sources.REVIEWED)
            if bad:
                logger.warning("h3b fp8 consumer fuse: site %s skipped, upstream source changed: %s", site,
                               ", ".join(bad))
            else:
                keep.append(site)
        sites = tuple(keep)
    if not sites:
        return []
    if "qkv" in sites:
        tr.fused_qk_norm_rope = make_qk_wrapper(tr.fused_qk_norm_rope)
    if "out" in sites:
        tr.indexed_gate_rms_norm_scale_shift = make_gate_rms_wrapper(tr.indexed_gate_rms_norm_scale_shift)
    if "fc2" in sites:
        tr.indexed_gate = make_gate_wrapper(tr.indexed_gate)
    block_cls.forward = make_block_forward(block_cls.forward, sites, _lora_types() if lora_types is None else lora_types)
    fp8_gemm.set_stash_hook(stash_hook)
    _state["sites"] = sites
    return list(sites)
