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

import logging
from typing import Any

import torch

from . import _fusewire as _fw
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
# the wiring (the reference's protocol, h3_tp2/fp8_consumers.py:498-919, on the shared machinery of h3b._fusewire)
# --------------------------------------------------------------------------------------------------------------------

_ROTARY_DIMS = (32, 64, 96, 128)      # what the norm + RoPE epilogue rotates (the reference's Triton copy: 96 only)
_state: dict[str, Any] = {"sites": (), "checked": {}, "disabled": set(), "device_types": ("cuda",)}
_stats: dict[str, int] = {k: 0 for k in ("stash", "materialize", "fused_qkv", "fused_out", "fused_fc2",
                                         "selfcheck_pass", "selfcheck_fail")}
_warned: set = set()


def stats() -> dict[str, int]:
    return dict(_stats)


def _note_realized(site: str, why: str) -> None:
    _stats["materialize"] += 1
    if why not in _warned:
        _warned.add(why)
        logger.warning("h3b fp8 consumer fuse: %s: stash of %s materialised, stock consumer", why, site)


_scopes = _fw.ScopeRegistry(lambda st: st.materialize(), _note_realized)
_tls = _scopes.local       # ``_tls.ctx``: the running block's scope (plan: (weight pointer, weight shape) -> site)
_verdicts = _fw.Verdicts(lambda: _state, lambda: _stats, logger, "fp8 consumer fuse")


def scope(block, want: dict) -> _fw.BlockScope:  # noqa: ANN001
    """The context in which a planned block's forward runs; ``want`` maps the planned GEMMs' weights to their sites."""
    return _fw.BlockScope(_scopes, block, want)


def _vec(scale: torch.Tensor, n: int) -> torch.Tensor:
    s = scale.reshape(-1).float()
    return (s.expand(n) if s.numel() == 1 else s).contiguous()


def stash_hook(a, b, scale_a, scale_b, out_dtype, bias):  # noqa: ANN001,ANN201
    """FP8 GEMM dispatcher hook (h3_tp2/fp8_consumers.py:531).  A bf16 GEMM whose weight ``b`` ([K, N], as the layer
    stores it) is one of the running block's planned qkv / out / fc2 weights is not run: its operands are kept (each
    planned weight once per block) and the model gets an uninitialised bf16 placeholder for the consumer."""
    sc = _scopes.current()
    if sc is None or out_dtype is not torch.bfloat16:
        return None
    site = sc.plan.pop((b.data_ptr(), tuple(b.shape)), None)
    if site is None:
        return None
    if sc.handoffs:
        _scopes.realize_all(sc, f"unconsumed stash before {site}")
    rows, cols = a.shape[0], b.shape[1]
    ph = torch.empty((rows, cols), device=a.device, dtype=out_dtype)
    sc.handoffs[site] = Stash(a, b.t(), _vec(scale_a, rows), _vec(scale_b, cols), bias, ph)
    _stats["stash"] += 1
    return ph


def _device_ok(*ts: torch.Tensor) -> bool:
    return _fw.same_device(_state["device_types"], *ts)


def _stash_ok(st: Stash) -> bool:
    ph = st.ph
    return (ph is not None and ph.dim() == 2 and ph.is_contiguous() and ph.dtype == torch.bfloat16
            and st.a.shape[0] == ph.shape[0] and st.w.shape[0] == ph.shape[1])


def _qkv_split(ph: torch.Tensor, T: int, H: int, Hk: int, D: int) -> tuple:
    """Upstream's split of the qkv output into q, k, v views [T, heads, D]."""
    return (ph[:, :H * D].view(T, H, D), ph[:, H * D:(H + Hk) * D].view(T, Hk, D), ph[:, (H + Hk) * D:].view(T, Hk, D))


def qk_mismatch(st: Stash, q, k, q_weight, k_weight, rope_table, head_dim, rotary_dim, interleaved) -> str | None:  # noqa: ANN001
    """None when (q, k) are exactly the q/k views of the stash's placeholder and the norm + RoPE epilogue covers the
    call (h3_tp2/fp8_consumers.py:591), else the first reason it does not (checked in this order: layout of the call,
    the placeholder, the views, the head and rotary sizes, the weights, bias, devices)."""
    ph = st.ph
    checks = (
        (lambda: not interleaved, "interleaved"),
        (lambda: q.dim() == 3 and k.dim() == 3 and q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16,
         "q/k rank or dtype"),
        (lambda: (ph is not None and q.shape[0] > 0 and ph.dim() == 2 and ph.shape[0] == q.shape[0]
                  and k.shape == (q.shape[0], k.shape[1], q.shape[2])
                  and ph.shape[1] == (q.shape[1] + 2 * k.shape[1]) * q.shape[2]), "shapes"),
        (lambda: k.shape[1] == q.shape[1], "grouped kv heads"),
        (lambda: _stash_ok(st), "placeholder/operand layout"),
        (lambda: _views_are_placeholder(ph, q, k), "q/k are not the split views of the qkv placeholder"),
        (lambda: q.shape[2] == 128 and head_dim in (None, 128), "head_dim"),
        (lambda: _rotary_ok(rope_table, rotary_dim, q.shape[0]), "rotary"),
        (lambda: (rope_table.dtype in (torch.bfloat16, torch.float32) and q_weight.shape == (128,)
                  and k_weight.shape == (128,) and q_weight.dtype == torch.bfloat16
                  and k_weight.dtype == torch.bfloat16), "rope table or norm weight dtype/shape"),
        (lambda: st.bias is None, "bias (the norm epilogue has none)"),
        (lambda: _device_ok(q, k, q_weight, k_weight, rope_table, st.a), "device"),
    )
    for holds, reason in checks:
        if not holds():
            return reason
    return None


def _views_are_placeholder(ph: torch.Tensor, q: torch.Tensor, k: torch.Tensor) -> bool:
    eq, ek, _ = _qkv_split(ph, q.shape[0], q.shape[1], k.shape[1], q.shape[2])
    return (q.data_ptr(), q.stride(), k.data_ptr(), k.stride()) == (eq.data_ptr(), eq.stride(), ek.data_ptr(),
                                                                    ek.stride())


def _rotary_ok(rope_table: torch.Tensor, rotary_dim, T: int) -> bool:  # noqa: ANN001
    rot = rope_table.shape[-1] if rope_table.dim() == 2 else -1
    return rot in _ROTARY_DIMS and rotary_dim in (None, rot) and tuple(rope_table.shape) == (T, rot)


def rows_mismatch(st: Stash, x: torch.Tensor, branch: torch.Tensor, *others: torch.Tensor) -> str | None:
    """None when ``branch`` is exactly the stash's placeholder and ``x`` (the residual) a contiguous bf16 tensor of its
    shape on the operands' device, with gate / shift / scale row-major bf16 of its width and the indices (last of
    ``others``) one per row (h3_tp2/fp8_consumers.py:622); else the reason."""
    ph = st.ph
    if ph is None or (branch.data_ptr(), branch.shape, branch.stride()) != (ph.data_ptr(), ph.shape, ph.stride()):
        return "branch is not the placeholder"
    if not (x.dim() == 2 and x.shape == ph.shape and x.dtype == torch.bfloat16 and x.is_contiguous()
            and _stash_ok(st)):
        return "residual shape/dtype/layout"
    if x.shape[0] == 0:
        return "no rows"
    *rowwise, indices = others
    if not all(o.dim() == 2 and o.stride(1) == 1 and o.dtype == torch.bfloat16 and o.shape[1] == x.shape[1]
               for o in rowwise):
        return "gate/shift/scale layout"
    if indices.dim() != 1 or indices.shape[0] != x.shape[0]:
        return "indices"
    return None if _device_ok(x, st.a, *others) else "device"


_STOCK = object()   # "not taken": the wrapper runs the stock consumer


class _Consumer:
    """One consumer site: ``call`` is the wrapped function's argument tuple and ``st`` the site's stash."""
    name = ""

    def __init__(self, orig):  # noqa: ANN001
        self.orig = orig

    def mismatch(self, st: Stash, call: tuple) -> str | None:
        raise NotImplementedError

    def key(self, st: Stash, call: tuple) -> tuple:
        raise NotImplementedError

    def fused(self, st: Stash, call: tuple, r: int) -> tuple:
        raise NotImplementedError

    def stock(self, st: Stash, call: tuple, r: int) -> tuple:
        raise NotImplementedError

    def run(self, st: Stash, call: tuple):  # noqa: ANN201
        raise NotImplementedError


def _consume(site: _Consumer, call: tuple):  # noqa: ANN202
    """The fused consumer's result when the running block holds this site's stash and the call is exactly its
    consumer (the first such call per key also matching the GEMM + stock consumer bit for bit); else ``_STOCK``, after
    making every stash real (another site's stash, an ineligible call, a failed comparison)."""
    sc = _scopes.current()
    if sc is None or not sc.handoffs:
        return _STOCK
    st = sc.handoffs.get(site.name)
    if st is None:
        _scopes.realize_all(sc, f"{site.name} consumer saw another site's stash")
        return _STOCK
    reason = f"{site.name} disabled by self-check" if _verdicts.off(site.name) else site.mismatch(st, call)
    if reason is None:
        r = min(_fw.CHECK_ROWS, st.a.shape[0])
        if not _verdicts.judge(site.key(st, call), lambda: site.fused(st.rows(r), call, r),
                               lambda: site.stock(st.rows(r), call, r)):
            reason = f"{site.name} disabled by self-check"
    if reason is not None:
        _scopes.realize_all(sc, f"{site.name}: {reason}")
        return _STOCK
    del sc.handoffs[site.name]
    out = site.run(st, call)
    _stats["fused_" + site.name] += 1
    return out


class _QkNormRope(_Consumer):
    """``fused_qk_norm_rope(q, k, q_weight, k_weight, rope_table, eps, head_dim, rotary_dim, interleaved)`` on the qkv
    placeholder's q/k views: the qkv GEMM with the norm + RoPE epilogue (``qk_norm_rope_fused``, looked up at call
    time so the Ulysses producer can replace it); v is written into the placeholder's v view, which the model reads."""
    name = "qkv"

    def mismatch(self, st, call):  # noqa: ANN001,ANN201
        q, k, qw, kw, table, _, head_dim, rotary_dim, interleaved = call
        return qk_mismatch(st, q, k, qw, kw, table, head_dim, rotary_dim, interleaved)

    def key(self, st, call):  # noqa: ANN001,ANN201
        return ("qkv", tuple(st.ph.shape[1:]), call[4].dtype)

    def _shape(self, call):  # noqa: ANN001,ANN202
        q, k = call[0], call[1]
        return q.shape[1], k.shape[1], q.shape[-1]

    def fused(self, st, call, r):  # noqa: ANN001,ANN201
        H, Hk, D = self._shape(call)
        _, _, qw, kw, table, eps, _, _, _ = call
        return qk_norm_rope_fused(st, H, Hk, D, qw, kw, table[:r], eps)

    def stock(self, st, call, r):  # noqa: ANN001,ANN201
        H, Hk, D = self._shape(call)
        _, _, qw, kw, table, eps, head_dim, rotary_dim, interleaved = call
        qs, ks, vs = _qkv_split(st.materialize(), r, H, Hk, D)
        oq, ok_ = self.orig(qs, ks, qw, kw, table[:r], eps, head_dim=head_dim, rotary_dim=rotary_dim,
                            interleaved=interleaved)
        return oq, ok_, vs

    def run(self, st, call):  # noqa: ANN001,ANN201
        H, Hk, D = self._shape(call)
        q, _, qw, kw, table, eps, _, _, _ = call
        out_q, out_k, v = qk_norm_rope_fused(st, H, Hk, D, qw, kw, table, eps)
        v_view = _qkv_split(st.ph, q.shape[0], H, Hk, D)[2]
        if v.data_ptr() != v_view.data_ptr():
            v_view.copy_(v)
        return out_q, out_k


class _GateRmsNorm(_Consumer):
    """``indexed_gate_rms_norm_scale_shift(residual, gate, branch, weight, shift, scale, indices, eps)`` on the out
    placeholder (branch): ``gate_rms_fused``."""
    name = "out"

    def mismatch(self, st, call):  # noqa: ANN001,ANN201
        residual, gate, branch, weight, shift, scale, indices, _ = call
        reason = rows_mismatch(st, residual, branch, gate, shift, scale, indices)
        if reason is None and (weight.shape != (residual.shape[1],) or weight.device != residual.device
                               or weight.dtype != torch.bfloat16):
            reason = "norm weight shape/device/dtype"
        return reason

    def key(self, st, call):  # noqa: ANN001,ANN201
        return ("out", tuple(call[0].shape[1:]), call[1].dtype, call[3].dtype)

    def fused(self, st, call, r):  # noqa: ANN001,ANN201
        residual, gate, _, weight, shift, scale, indices, eps = call
        return gate_rms_fused(st, residual[:r], gate, weight, shift, scale, indices[:r], eps)

    def stock(self, st, call, r):  # noqa: ANN001,ANN201
        residual, gate, _, weight, shift, scale, indices, eps = call
        return self.orig(residual[:r], gate, st.materialize(), weight, shift, scale, indices[:r], eps)

    def run(self, st, call):  # noqa: ANN001,ANN201
        residual, gate, _, weight, shift, scale, indices, eps = call
        return gate_rms_fused(st, residual, gate, weight, shift, scale, indices, eps)


class _IndexedGate(_Consumer):
    """``indexed_gate(x, gate, other, indices)`` on the fc2 placeholder (other): the fc2 GEMM with the indexed-gate
    epilogue."""
    name = "fc2"

    def mismatch(self, st, call):  # noqa: ANN001,ANN201
        x, gate, other, indices = call
        return rows_mismatch(st, x, other, gate, indices)

    def key(self, st, call):  # noqa: ANN001,ANN201
        return ("fc2", tuple(call[0].shape[1:]), call[1].dtype)

    def fused(self, st, call, r):  # noqa: ANN001,ANN201
        x, gate, _, indices = call
        return (gate_fused(st, x[:r].contiguous(), gate, indices[:r], reuse_placeholder=False),)

    def stock(self, st, call, r):  # noqa: ANN001,ANN201
        x, gate, _, indices = call
        return (self.orig(x[:r].contiguous(), gate, st.materialize(), indices[:r]),)

    def run(self, st, call):  # noqa: ANN001,ANN201
        x, gate, _, indices = call
        return gate_fused(st, x, gate, indices)


def make_qk_wrapper(orig):  # noqa: ANN001,ANN201
    """``fused_qk_norm_rope`` with the qkv consumer (h3_tp2/fp8_consumers.py:652)."""
    site = _QkNormRope(orig)

    def fused_qk_norm_rope(q, k, q_weight, k_weight, rope_table, eps, *, head_dim=None, rotary_dim=None,  # noqa: ANN001,ANN202
                           interleaved=False):
        out = _consume(site, (q, k, q_weight, k_weight, rope_table, eps, head_dim, rotary_dim, interleaved))
        if out is _STOCK:
            return orig(q, k, q_weight, k_weight, rope_table, eps, head_dim=head_dim, rotary_dim=rotary_dim,
                        interleaved=interleaved)
        return out

    fused_qk_norm_rope._h3b_consumer_fuse = True
    return fused_qk_norm_rope


def make_gate_rms_wrapper(orig):  # noqa: ANN001,ANN201
    """``indexed_gate_rms_norm_scale_shift`` with the out consumer (h3_tp2/fp8_consumers.py:688)."""
    site = _GateRmsNorm(orig)

    def indexed_gate_rms_norm_scale_shift(residual, gate, branch, weight, shift, scale, indices, eps):  # noqa: ANN001,ANN202
        call = (residual, gate, branch, weight, shift, scale, indices, eps)
        out = _consume(site, call)
        return orig(*call) if out is _STOCK else out

    indexed_gate_rms_norm_scale_shift._h3b_consumer_fuse = True
    return indexed_gate_rms_norm_scale_shift


def make_gate_wrapper(orig):  # noqa: ANN001,ANN201
    """``indexed_gate`` with the fc2 consumer (h3_tp2/fp8_consumers.py:720)."""
    site = _IndexedGate(orig)

    def indexed_gate(x, gate, other, indices):  # noqa: ANN001,ANN202
        out = _consume(site, (x, gate, other, indices))
        return orig(x, gate, other, indices) if out is _STOCK else out

    indexed_gate._h3b_consumer_fuse = True
    return indexed_gate


_lora_types = _fw.lora_types
_SITE_LAYER = {"qkv": ("attn", "qkv_proj"), "out": ("attn", "out_proj"), "fc2": ("mlp", "fc2")}


def _weight_key(site: str, layer, lora) -> tuple[tuple | None, str | None]:  # noqa: ANN001
    """((weight pointer, weight shape), None) for a layer whose GEMM the stash hook can take, else (None, reason)."""
    if layer is None or (lora and isinstance(layer, lora)):
        return None, f"{site}: missing or LoRA-wrapped layer"
    if getattr(layer, "tp_size", 1) != 1:
        return None, f"{site}: tp_size != 1 (an all-reduce would read the placeholder)"
    w = getattr(layer, "weight", None)
    n = int(getattr(layer, "output_size_per_partition", 0) or 0)
    if not (isinstance(w, torch.Tensor) and w.dtype == torch.float8_e4m3fn and w.dim() == 2 and w.shape[1] == n):
        return None, f"{site}: weight is not an unpadded FP8 [K, N] tensor"
    return (w.data_ptr(), tuple(w.shape)), None


def block_plan(block, rope_table, sites, lora_types=()) -> tuple[dict | None, str]:  # noqa: ANN001
    """{(weight data_ptr, weight shape): site} for this block's eligible GEMMs, or (None, reason)
    (h3_tp2/fp8_consumers.py:758)."""
    if rope_table is None:
        return None, "no rope table (q/k norm without fused rope)"
    if _fw.compiling():
        return None, "torch.compile tracing"
    want: dict = {}
    for site in (s for s in sites if s not in _state["disabled"]):
        owner, attr = _SITE_LAYER[site]
        key, why = _weight_key(site, getattr(getattr(block, owner, None), attr, None), lora_types)
        if key is None:
            return None, why
        want[key] = site
    return (want or None), "no site left"


def _unplanned(reason: str) -> None:
    key = "plan-" + reason
    if key not in _warned:
        _warned.add(key)
        logger.warning("h3b fp8 consumer fuse: block not fused (%s); stock path", reason)


def make_block_forward(orig_forward, sites, lora_types=()):  # noqa: ANN001,ANN201
    """The DiT block's forward, run in a scope with this block's planned weights (h3_tp2/fp8_consumers.py:787)."""
    return _fw.wrap_block_forward(
        orig_forward, _scopes, lambda blk, *a, **kw: block_plan(blk, kw.get("rope_table"), sites, lora_types),
        _unplanned, "_h3b_consumer_fuse")


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
    # each site's consumer in the transformer module
    for site, name, wrap in (("qkv", "fused_qk_norm_rope", make_qk_wrapper),
                             ("out", "indexed_gate_rms_norm_scale_shift", make_gate_rms_wrapper),
                             ("fc2", "indexed_gate", make_gate_wrapper)):
        if site in sites:
            setattr(tr, name, wrap(getattr(tr, name)))
    block_cls.forward = make_block_forward(block_cls.forward, sites, _lora_types() if lora_types is None else lora_types)
    fp8_gemm.set_stash_hook(stash_hook)
    _state["sites"] = sites
    return list(sites)
