"""Tensor-level entry points over the C ABI (``include/h3b.h``), and their ``torch.ops.h3b.*`` registrations.

Every function takes CUDA tensors, allocates its outputs with torch on the tensor's device (the caching allocator of
the current stream, as the reference does with ``torch.empty``) and enqueues one kernel on the current stream.
CPU tensors raise: there is no CPU fallback in the product path.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from ._lib import DIV_FULL, DIV_IEEE, EPI_PLAIN, EPI_QKV_SEND, EPI_SWIGLU, OUT_BF16, OUT_F16  # noqa: F401

E4M3 = torch.float8_e4m3fn
FP8_MAX = 448.0
MIN_SCALE = 1.0 / (FP8_MAX * 512.0)


def _need_cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("h3b kernels run on CUDA tensors only (no CPU fallback)")


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _addr(x) -> int | None:
    """Device address of a tensor, or an address given as an int (a peer's IPC mapping)."""
    if x is None:
        return None
    return x.data_ptr() if isinstance(x, torch.Tensor) else int(x)


def _dt(t: torch.Tensor, *dtypes: torch.dtype, what: str) -> None:
    if t.dtype not in dtypes:
        raise TypeError(f"{what}: dtype {t.dtype}, expected one of {dtypes}")


def _bias(bias: torch.Tensor | None, n: int, what: str) -> torch.Tensor | None:
    """A bias the kernels can read: None, or n bf16 values, contiguous (the kernels read it as bf16; an f16 bias
    would be misread, so it is refused rather than converted, which would round it)."""
    if bias is None:
        return None
    _dt(bias, torch.bfloat16, what=f"{what} bias")
    if bias.numel() != n:
        raise ValueError(f"{what}: bias has {bias.numel()} values, expected {n}")
    return bias.reshape(-1).contiguous()


def _out(out: torch.Tensor | None, shape: tuple[int, ...], dtype: torch.dtype, like: torch.Tensor, what: str, *,
         dense: bool = True) -> torch.Tensor:
    """A fresh output, or the caller's checked against the shape, dtype and device the kernel writes (``dense``: also
    contiguous; the kernels take a base pointer and write the whole extent)."""
    if out is None:
        return torch.empty(shape, dtype=dtype, device=like.device)
    if tuple(out.shape) != tuple(shape) or out.dtype != dtype or out.device != like.device or (
            dense and not out.is_contiguous()):
        raise ValueError(f"{what}: out must be {'contiguous ' if dense else ''}{tuple(shape)} {dtype} on "
                         f"{like.device}, got {tuple(out.shape)} {out.dtype} on {out.device}")
    return out


def _norm_rope_args(weights, table: torch.Tensor, m: int, what: str):  # noqa: ANN001,ANN202
    """Norm weights (128 bf16 values each) and the RoPE table [>= m, R] as fp32 with unit column stride: the kernels
    read 128 weights and table rows 0 .. m-1."""
    out = []
    for wt in weights:
        _need_cuda(wt)
        _dt(wt, torch.bfloat16, what=f"{what} norm weight")
        if wt.numel() != 128:
            raise ValueError(f"{what}: norm weight has {wt.numel()} values, expected 128 (head_dim)")
        out.append(wt.reshape(-1).contiguous())
    _need_cuda(table)
    if table.dim() != 2 or table.shape[0] < m or table.shape[1] > 128:
        raise ValueError(f"{what}: rope table must be [>= {m}, R <= 128], got {tuple(table.shape)}")
    table = table.float()
    if table.stride(-1) != 1:
        table = table.contiguous()
    return out, table


def _rows(t: torch.Tensor, rows: int, cols: int, what: str, dtype: torch.dtype = torch.bfloat16) -> None:
    """A [rows, cols] input of ``dtype`` with unit column stride (the row kernels take a base pointer and a row
    stride)."""
    _dt(t, dtype, what=what)
    if t.dim() != 2 or tuple(t.shape) != (rows, cols) or (t.numel() and t.stride(1) != 1):
        raise ValueError(f"{what}: must be [{rows}, {cols}] with unit column stride, got {tuple(t.shape)}")


def _weight(weight: torch.Tensor, n: int, what: str) -> torch.Tensor:
    _dt(weight, torch.bfloat16, what=f"{what} weight")
    if weight.numel() != n:
        raise ValueError(f"{what}: weight has {weight.numel()} values, expected {n}")
    return weight.reshape(-1).contiguous()


def _modulation(shift, scale, indices, rows: int, hidden: int, what: str, gate=None):  # noqa: ANN001,ANN202
    """AdaLN rows read as row ``indices[r]`` (row 0 without indices) of shift / scale (and gate): each [B, hidden] bf16
    ([B, 1, hidden] is viewed as [B, hidden]) with unit column stride; index values are the caller's contract, as in
    the reference's kernels.  Returns (shift, scale, gate, indices) as the kernels take them."""
    if (shift is None) != (scale is None):
        raise ValueError(f"{what}: shift and scale go together")
    out = []
    for name, t in (("shift", shift), ("scale", scale), ("gate", gate)):
        if t is not None:
            _dt(t, torch.bfloat16, what=f"{what} {name}")
            if t.dim() == 3 and t.shape[1] == 1:
                t = t[:, 0]
            if t.dim() != 2 or t.shape[1] != hidden or t.shape[0] < 1 or t.stride(1) != 1:
                raise ValueError(f"{what}: {name} must be [B >= 1, {hidden}] with unit column stride, got "
                                 f"{tuple(t.shape)}")
        out.append(t)
    if indices is not None:
        if indices.dtype.is_floating_point or indices.dtype == torch.bool or indices.numel() != rows:
            raise ValueError(f"{what}: indices must be {rows} integers, got {indices.numel()} {indices.dtype}")
        indices = indices.reshape(-1).to(torch.int64).contiguous()
    return (*out, indices)


def _span(t: torch.Tensor) -> int:
    """Elements reachable from ``t``'s data pointer through its shape and (non-negative) strides."""
    return 0 if t.numel() == 0 else 1 + sum((n - 1) * st for n, st in zip(t.shape, t.stride()))


def vec_scales(scale_a: torch.Tensor, scale_b: torch.Tensor, M: int, N: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row / per-column fp32 scale vectors (a scalar scale is broadcast), as fp8_gemm._vec_scales
    (h3_tp2/fp8_gemm.py:228-236)."""
    sa = scale_a.reshape(-1).float()
    sb = scale_b.reshape(-1).float()
    if sa.numel() not in (1, M) or sb.numel() not in (1, N):
        raise ValueError(f"scales: {sa.numel()} row and {sb.numel()} column scales for [{M}, {N}] (1 or one each)")
    if sa.numel() == 1:
        sa = sa.expand(M)
    if sb.numel() == 1:
        sb = sb.expand(N)
    return sa.contiguous(), sb.contiguous()


# ---------------------------------------------------------------------------------------------------------------
# per-token quant family
# ---------------------------------------------------------------------------------------------------------------


def quant_rows(base: torch.Tensor, m: int, p: int, seg: int, stride_p: int, stride_m: int, *,
               div_mode: int = DIV_IEEE) -> tuple[torch.Tensor, torch.Tensor]:
    """``ulysses_outq.quant_rows`` (h3_tp2/ulysses_outq.py:109): row m = concat_p base[p*stride_p + m*stride_m :][:seg]
    (element offsets from ``base``'s data pointer).  Returns (q [m, p*seg] e4m3, scale [m, 1] fp32)."""
    _need_cuda(base)
    _dt(base, torch.bfloat16, what="quant_rows")
    if m < 0 or p < 1 or seg < 0 or stride_p < 0 or stride_m < 0 or any(st < 0 for st in base.stride()):
        raise ValueError(f"quant_rows: m {m} p {p} seg {seg} strides {stride_p}, {stride_m}")
    if m and seg and (p - 1) * stride_p + (m - 1) * stride_m + seg > _span(base):
        raise ValueError(f"quant_rows: rows reach element {(p - 1) * stride_p + (m - 1) * stride_m + seg} of a base "
                         f"that spans {_span(base)}")
    q = torch.empty((m, p * seg), dtype=E4M3, device=base.device)
    s = torch.empty((m, 1), dtype=torch.float32, device=base.device)
    if m:
        _lib.call("h3b_quant_rows_e4m3", base.data_ptr(), m, p, seg, stride_p, stride_m, q.data_ptr(), s.data_ptr(),
                  div_mode, _stream(base))
    return q, s


def quant(h: torch.Tensor, *, div_mode: int = DIV_IEEE) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token dynamic e4m3 quant of a bf16 [M, K] tensor (``fp8_quant_fuse.quant``, h3_tp2/fp8_quant_fuse.py:318)."""
    if h.dim() != 2 or h.stride(1) != 1:
        raise ValueError("quant: h must be [M, K] with unit column stride")
    M, K = h.shape
    return quant_rows(h, M, 1, K, 0, h.stride(0), div_mode=div_mode)


def quant_from_recv(recv: torch.Tensor, *, div_mode: int = DIV_IEEE) -> tuple[torch.Tensor, torch.Tensor]:
    """recv [P, M, hl, d] contiguous -> quant of the [M, P*hl*d] rows stock's unpack would make
    (``ulysses_outq.quant_from_recv``, h3_tp2/ulysses_outq.py:138)."""
    if not recv.is_contiguous():
        raise ValueError("quant_from_recv: recv must be contiguous")
    p, m, hl, d = recv.shape
    seg = hl * d
    return quant_rows(recv, m, p, seg, m * seg, seg, div_mode=div_mode)


def rms_quant(x: torch.Tensor, weight: torch.Tensor, shift: torch.Tensor | None = None,
              scale: torch.Tensor | None = None, indices: torch.Tensor | None = None, eps: float = 1e-6,
              ph: torch.Tensor | None = None, *, div_mode: int = DIV_IEEE) -> tuple[torch.Tensor, torch.Tensor]:
    """RMSNorm (+ AdaLN modulation) + per-token quant (``fp8_quant_fuse.rms_quant``, h3_tp2/fp8_quant_fuse.py:330)."""
    _need_cuda(x, weight, shift, scale, indices, ph)
    if x.dim() != 2:
        raise ValueError("rms_quant: x must be [rows, hidden]")
    rows, hidden = x.shape
    _rows(x, rows, hidden, "rms_quant x")
    weight = _weight(weight, hidden, "rms_quant")
    shift, scale, _, indices = _modulation(shift, scale, indices, rows, hidden, "rms_quant")
    if ph is not None:
        _out(ph, (rows, hidden), torch.bfloat16, x, "rms_quant placeholder")
    q = torch.empty((rows, hidden), dtype=E4M3, device=x.device)
    s = torch.empty((rows, 1), dtype=torch.float32, device=x.device)
    _lib.call("h3b_rms_quant_e4m3", x.data_ptr(), rows, hidden, x.stride(0), weight.data_ptr(),
              _ptr(shift), shift.stride(0) if shift is not None else 0, _ptr(scale),
              scale.stride(0) if scale is not None else 0, _ptr(indices), float(eps), _ptr(ph), q.data_ptr(),
              s.data_ptr(), div_mode, _stream(x))
    return q, s


def gate_rms_quant(residual: torch.Tensor, gate: torch.Tensor, branch: torch.Tensor, weight: torch.Tensor,
                   shift: torch.Tensor | None, scale: torch.Tensor | None, indices: torch.Tensor | None, eps: float,
                   *, div_mode: int = DIV_IEEE) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Gated residual + RMSNorm + modulation + quant (``fp8_quant_fuse.gate_rms_quant``,
    h3_tp2/fp8_quant_fuse.py:350).  Returns (residual_out bf16, q e4m3, scale [M, 1])."""
    _need_cuda(residual, gate, branch, weight, shift, scale, indices)
    if residual.dim() != 2:
        raise ValueError("gate_rms_quant: residual must be [rows, hidden]")
    rows, hidden = residual.shape
    _rows(residual, rows, hidden, "gate_rms_quant residual")
    _rows(branch, rows, hidden, "gate_rms_quant branch")
    weight = _weight(weight, hidden, "gate_rms_quant")
    if gate is None:
        raise ValueError("gate_rms_quant: gate is required")
    shift, scale, gate, indices = _modulation(shift, scale, indices, rows, hidden, "gate_rms_quant", gate=gate)
    res_out = torch.empty((rows, hidden), dtype=torch.bfloat16, device=residual.device)
    q = torch.empty((rows, hidden), dtype=E4M3, device=residual.device)
    s = torch.empty((rows, 1), dtype=torch.float32, device=residual.device)
    _lib.call("h3b_gate_rms_quant_e4m3", residual.data_ptr(), residual.stride(0), gate.data_ptr(), gate.stride(0),
              branch.data_ptr(), branch.stride(0), weight.data_ptr(), _ptr(shift),
              shift.stride(0) if shift is not None else 0, _ptr(scale), scale.stride(0) if scale is not None else 0,
              _ptr(indices), rows, hidden, float(eps), res_out.data_ptr(), q.data_ptr(), s.data_ptr(), div_mode,
              _stream(residual))
    return res_out, q, s


def silu_mul_quant(x: torch.Tensor, *, div_mode: int = DIV_IEEE) -> tuple[torch.Tensor, torch.Tensor]:
    """silu_and_mul on bf16 [M, 2d] + per-token quant (``fp8_quant_fuse.silu_mul_quant``, :392)."""
    _need_cuda(x)
    if x.dim() != 2 or x.shape[1] % 2:
        raise ValueError(f"silu_mul_quant: x must be [rows, 2d], got {tuple(x.shape)}")
    rows, width = x.shape
    _rows(x, rows, width, "silu_mul_quant x")
    d = width // 2
    q = torch.empty((rows, d), dtype=E4M3, device=x.device)
    s = torch.empty((rows, 1), dtype=torch.float32, device=x.device)
    _lib.call("h3b_silu_mul_quant_e4m3", x.data_ptr(), rows, d, x.stride(0), q.data_ptr(), s.data_ptr(), div_mode,
              _stream(x))
    return q, s


def scale_bias_cast(x32: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, bias: torch.Tensor | None,
                    out_dtype: torch.dtype) -> torch.Tensor:
    """The two-pass path's scale pass (``fp8_gemm._scale_bias_cast``, h3_tp2/fp8_gemm.py:38)."""
    _need_cuda(x32, sa, sb, bias)
    _dt(x32, torch.float32, what="scale_bias_cast x32")
    M, N = x32.shape
    sa, sb = vec_scales(sa, sb, M, N)
    bias = _bias(bias, N, "scale_bias_cast")
    if out_dtype not in (torch.bfloat16, torch.float16):
        raise TypeError(f"scale_bias_cast: out_dtype {out_dtype}, expected bf16 or f16")
    y = torch.empty((M, N), dtype=out_dtype, device=x32.device)
    _lib.call("h3b_scale_bias_cast", x32.contiguous().data_ptr(), sa.data_ptr(), sb.data_ptr(), _ptr(bias),
              y.data_ptr(), M, N, OUT_BF16 if out_dtype == torch.bfloat16 else OUT_F16, _stream(x32))
    return y


def scale_swiglu(x32: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    """``fp8_swiglu.scale_swiglu`` (h3_tp2/fp8_swiglu.py:180): fp32 fc1 product -> bf16 SwiGLU [M, half]."""
    _need_cuda(x32, sa, sb, bias)
    _dt(x32, torch.float32, what="scale_swiglu x32")
    if x32.dim() != 2 or x32.shape[1] % 2:
        raise ValueError(f"scale_swiglu: x32 must be [M, 2 * half], got {tuple(x32.shape)}")
    M, width = x32.shape
    half = width // 2
    sa, sb = vec_scales(sa, sb, M, width)
    bias = _bias(bias, width, "scale_swiglu")
    y = torch.empty((M, half), dtype=torch.bfloat16, device=x32.device)
    _lib.call("h3b_scale_swiglu", x32.contiguous().data_ptr(), sa.data_ptr(), sb.data_ptr(), _ptr(bias),
              y.data_ptr(), M, half, _stream(x32))
    return y


def scale_swiglu_quant(x32: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, bias: torch.Tensor | None, *,
                       div_mode: int = DIV_IEEE) -> tuple[torch.Tensor, torch.Tensor]:
    """``fp8_swiglu.scale_swiglu_quant`` (h3_tp2/fp8_swiglu.py:191): SwiGLU + per-token quant for fc2."""
    _need_cuda(x32, sa, sb, bias)
    _dt(x32, torch.float32, what="scale_swiglu x32")
    if x32.dim() != 2 or x32.shape[1] % 2:
        raise ValueError(f"scale_swiglu: x32 must be [M, 2 * half], got {tuple(x32.shape)}")
    M, width = x32.shape
    half = width // 2
    sa, sb = vec_scales(sa, sb, M, width)
    bias = _bias(bias, width, "scale_swiglu")
    q = torch.empty((M, half), dtype=E4M3, device=x32.device)
    s = torch.empty((M, 1), dtype=torch.float32, device=x32.device)
    _lib.call("h3b_scale_swiglu_quant", x32.contiguous().data_ptr(), sa.data_ptr(), sb.data_ptr(), _ptr(bias),
              q.data_ptr(), s.data_ptr(), M, half, div_mode, _stream(x32))
    return q, s


# ---------------------------------------------------------------------------------------------------------------
# FP8 GEMM
# ---------------------------------------------------------------------------------------------------------------


def _gemm_operands(a: torch.Tensor, w: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, N: int):
    _need_cuda(a, w, sa, sb)
    _dt(a, E4M3, what="fp8_gemm a")
    _dt(w, E4M3, what="fp8_gemm w")
    if a.dim() != 2 or w.dim() != 2 or a.stride(1) != 1 or w.stride(1) != 1 or a.shape[1] != w.shape[1]:
        raise ValueError("fp8_gemm: a [M, K] and w [N, K] with unit column strides")
    M = a.shape[0]
    return vec_scales(sa, sb, M, N)


def fp8_gemm(a: torch.Tensor, w: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, bias: torch.Tensor | None = None,
             out_dtype: torch.dtype = torch.bfloat16, out: torch.Tensor | None = None) -> torch.Tensor:
    """y [M, N] = out_dtype(sa[m] * (sb[n] * (a @ w.T))) (bias by fma): the fused tcgen05 FP8 GEMM.  ``w`` is the
    weight [N, K] (the reference's ``b`` is ``w.t()``)."""
    N = w.shape[0]
    sa, sb = _gemm_operands(a, w, sa, sb, N)
    M, K = a.shape
    bias = _bias(bias, N, "fp8_gemm")
    if out is not None:
        _need_cuda(out)
        _dt(out, torch.bfloat16, torch.float16, what="fp8_gemm out")
        if out.shape != (M, N) or out.stride(1) != 1:
            raise ValueError(f"fp8_gemm: out must be [{M}, {N}] with unit column stride, got {tuple(out.shape)}")
    elif out_dtype not in (torch.bfloat16, torch.float16):
        raise TypeError(f"fp8_gemm: out_dtype {out_dtype}, expected bf16 or f16 (the epilogue writes the scaled output)")
    y = out if out is not None else torch.empty((M, N), dtype=out_dtype, device=a.device)
    _lib.call("h3b_fp8_gemm", a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), sa.data_ptr(), sb.data_ptr(),
              _ptr(bias), y.data_ptr(), y.stride(0), M, N, K, OUT_BF16 if y.dtype == torch.bfloat16 else OUT_F16,
              EPI_PLAIN, None, _stream(a))
    return y


def fp8_gemm_swiglu(a: torch.Tensor, w: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor,
                    bias: torch.Tensor | None = None) -> torch.Tensor:
    """fc1 + SwiGLU in one kernel (``fp8_swiglu.gemm_swiglu``, h3_tp2/fp8_swiglu.py:230): w [2F, K] holds the gate
    rows then the up rows; returns bf16 [M, F]."""
    N = w.shape[0]
    sa, sb = _gemm_operands(a, w, sa, sb, N)
    M, K = a.shape
    bias = _bias(bias, N, "fp8_gemm_swiglu")
    y = torch.empty((M, N // 2), dtype=torch.bfloat16, device=a.device)
    _lib.call("h3b_fp8_gemm", a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), sa.data_ptr(), sb.data_ptr(),
              _ptr(bias), y.data_ptr(), y.stride(0), M, N, K, OUT_BF16, EPI_SWIGLU, None, _stream(a))
    return y


def fp8_gemm_gate(a: torch.Tensor, w: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, x: torch.Tensor,
                  gate: torch.Tensor, indices: torch.Tensor, bias: torch.Tensor | None = None,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """fc2 with the indexed gated residual in the epilogue: ``x + gate[indices] * bf16(sa * (sb * (a @ w^T)))``
    (``fp8_consumers.gate_fused`` / ``_scale_indexed_gate_kernel``, h3_tp2/fp8_consumers.py:203-239,468).  x, gate
    bf16 with unit column stride (gate may be a row-strided view); indices [M] integer."""
    N = w.shape[0]
    sa, sb = _gemm_operands(a, w, sa, sb, N)
    _need_cuda(x, gate, indices)
    M, K = a.shape
    _dt(x, torch.bfloat16, what="fp8_gemm_gate x")
    _dt(gate, torch.bfloat16, what="fp8_gemm_gate gate")
    if x.shape != (M, N) or x.stride(1) != 1 or gate.shape[-1] != N or gate.stride(-1) != 1:
        raise ValueError(f"fp8_gemm_gate: x {tuple(x.shape)} / gate {tuple(gate.shape)} against [{M}, {N}]")
    bias = _bias(bias, N, "fp8_gemm_gate")
    if out is not None:
        _need_cuda(out)
        _dt(out, torch.bfloat16, what="fp8_gemm_gate out")
        if out.shape != (M, N) or out.stride(1) != 1:
            raise ValueError(f"fp8_gemm_gate: out must be [{M}, {N}] with unit column stride, got {tuple(out.shape)}")
    idx = indices.to(torch.int64).contiguous()
    y = out if out is not None else torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    _lib.call("h3b_fp8_gemm_gate", a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), sa.data_ptr(), sb.data_ptr(),
              _ptr(bias), x.data_ptr(), x.stride(0), gate.data_ptr(), gate.stride(0), gate.shape[0], idx.data_ptr(),
              y.data_ptr(), y.stride(0), M, N, K, _stream(a))
    return y


def fp8_gemm_qkv_send(a: torch.Tensor, w: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, heads: int, ws: int, *,
                      bias: torch.Tensor | None = None, v_f16: bool = False, sends=None,
                      range_flag: torch.Tensor | None = None, groups: int = 1, qk_norm=None, p2p=None,
                      interleaved: bool = False):
    """qkv projection whose epilogue writes q, k, v straight into the Ulysses send buffers (the producer redirection
    of ulysses_exact.fused_into_send, h3_tp2/ulysses_exact.py:278, moved into the GEMM).  groups = 1: each buffer is
    stock's [P, M, H/P, d]; groups = G > 1: [G, P, M, H/(G*P), d], head h = g*(H/G) + p*(H/(G*P)) + j, one
    contiguous all-to-all per group (the head-group overlap layout).  ``qk_norm = (q_weight, k_weight, rope_table,
    eps)`` applies the per-(token, head) RMSNorm + partial RoPE of the upstream producer to q and k in the epilogue
    (rope_table [M, R] fp32, cos | sin, R in {0, 32, 64, 96, 128}).

    ``p2p = (rank, peer_recv, peer_range_flag)``: no send buffers; the slab for rank p goes straight into
    ``peer_recv[p] = (q, k, v)`` (device tensors or addresses of rank p's [P, M, H/P, d] receive buffers, slot
    ``rank``) and a v overflow raises every rank's ``peer_range_flag[p]`` (so all ranks agree once the stores are
    ordered by the exchange's barrier).  Returns None then.

    ``interleaved``: one send buffer [G, P, M, 3, H/(G*P), d] (q, k, v of a token side by side, the combined-exchange
    layout of ulysses_nocopy) is returned instead of three; its v slots hold f16 bits when ``v_f16``."""
    N = w.shape[0]
    sa, sb = _gemm_operands(a, w, sa, sb, N)
    M, K = a.shape
    bias = _bias(bias, N, "fp8_gemm_qkv_send")
    if N != 3 * heads * 128 or heads % (ws * groups):
        raise ValueError(f"fp8_gemm_qkv_send: N {N} != 3 * {heads} * 128 or heads % (ws * groups)")
    shape = (ws, M, heads // ws, 128) if groups == 1 else (groups, ws, M, heads // (ws * groups), 128)
    if p2p is not None:
        rank, peer_recv, peer_rf = p2p
        if groups != 1 or len(peer_recv) != ws or ws > _lib.MAX_RANKS:
            raise ValueError("fp8_gemm_qkv_send: p2p needs groups 1 and one (q, k, v) triple per rank")
        desc = _lib.QkvSend()
        desc.heads, desc.head_dim, desc.ws, desc.v_f16, desc.groups = heads, 128, ws, int(bool(v_f16)), 1
        desc.p2p, desc.rank = 1, int(rank)
        for r in range(ws):
            for i in range(3):
                desc.peer_recv[r][i] = _addr(peer_recv[r][i])
            desc.peer_range_flag[r] = None if peer_rf is None else _addr(peer_rf[r])
        _lib.call("h3b_fp8_gemm", a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), sa.data_ptr(),
                  sb.data_ptr(), _ptr(bias), None, 0, M, N, K, OUT_BF16, EPI_QKV_SEND, ctypes.byref(desc), _stream(a))
        return None
    desc = _lib.QkvSend()
    if interleaved:
        ishape = (groups, ws, M, 3, heads // (ws * groups), 128)
        buf = _out(sends, ishape, torch.bfloat16, a, "fp8_gemm_qkv_send interleaved send buffer")
        desc.send[0] = buf.data_ptr()
        desc.qkv_interleaved = 1
        result = buf
    else:
        if sends is None:
            sends = [torch.empty(shape, dtype=torch.bfloat16, device=a.device) for _ in range(2)]
            sends.append(torch.empty(shape, dtype=torch.float16 if v_f16 else torch.bfloat16, device=a.device))
        if len(sends) != 3:
            raise ValueError("fp8_gemm_qkv_send: three send buffers (q, k, v)")
        for i in range(3):
            dt = torch.float16 if (i == 2 and v_f16) else torch.bfloat16
            _out(sends[i], shape, dt, a, f"fp8_gemm_qkv_send send buffer {'qkv'[i]}")
            desc.send[i] = sends[i].data_ptr()
        result = sends
    desc.heads, desc.head_dim, desc.ws, desc.v_f16 = heads, 128, ws, int(bool(v_f16))
    desc.groups = int(groups)
    if qk_norm is not None:
        qw, kw, table, eps = qk_norm
        if bias is not None:
            raise ValueError("fp8_gemm_qkv_send: the norm + RoPE epilogue has no bias term (q and k would drop it)")
        (qw, kw), table = _norm_rope_args((qw, kw), table, M, "fp8_gemm_qkv_send")
        desc.q_norm_weight, desc.k_norm_weight = qw.data_ptr(), kw.data_ptr()
        desc.rope_table, desc.rope_stride, desc.rot = table.data_ptr(), table.stride(0), table.shape[-1]
        desc.eps = float(eps)
        keep = (qw, kw, table)  # alive until the launch below returns
    desc.range_flag = _ptr(range_flag)
    _lib.call("h3b_fp8_gemm", a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), sa.data_ptr(), sb.data_ptr(),
              _ptr(bias), None, 0, M, N, K, OUT_BF16, EPI_QKV_SEND, ctypes.byref(desc), _stream(a))
    return result


# ---------------------------------------------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------------------------------------------


def _as3(t: torch.Tensor) -> torch.Tensor:
    if t.dim() == 4:
        if t.shape[0] != 1:
            raise ValueError("flash_attn: batch 1 only (strict Ulysses at batch 1)")
        t = t[0]
    if t.dim() != 3 or t.stride(2) != 1:
        raise ValueError("flash_attn: [S, H, d] (or [1, S, H, d]) with unit innermost stride")
    return t


def bf16_to_f16(x: torch.Tensor, range_flag: torch.Tensor | None = None) -> torch.Tensor:
    _need_cuda(x)
    _dt(x, torch.bfloat16, what="bf16_to_f16 x")
    y = torch.empty(x.shape, dtype=torch.float16, device=x.device)
    _lib.call("h3b_bf16_to_f16", x.contiguous().data_ptr(), y.data_ptr(), x.numel(), _ptr(range_flag), _stream(x))
    return y


def _v16_scratch(v16: torch.Tensor | None, rows: int, heads: int, ref: torch.Tensor) -> torch.Tensor:
    """The f16 copy of v that the bf16-v attention writes: [rows, heads, 128] f16, contiguous (given or allocated)."""
    if v16 is None:
        return torch.empty((rows, heads, 128), dtype=torch.float16, device=ref.device)
    _need_cuda(v16)
    _dt(v16, torch.float16, what="flash_attn v16 scratch")
    if v16.numel() < rows * heads * 128 or not v16.is_contiguous() or v16.device != ref.device:
        raise ValueError(f"flash_attn: v16 scratch needs {rows * heads * 128} contiguous f16 values on {ref.device}")
    return v16


def attn_ctl_words(heads: int) -> int:
    """int32 words of the control buffer of the bf16-v attention (H3B_ATTN_CTL_BYTES(heads) bytes): the range flag in
    word 0 (1 after a call whose v did not fit f16), the per (head, column) maxima of the scaled pass from word 4."""
    return 4 + 128 * heads


def attn_ctl(heads: int, device) -> torch.Tensor:
    return torch.zeros(attn_ctl_words(heads), dtype=torch.int32, device=device)


def _ctl(ctl: torch.Tensor | None, heads: int, ref: torch.Tensor) -> torch.Tensor:
    if ctl is None:
        return attn_ctl(heads, ref.device)
    _need_cuda(ctl)
    _dt(ctl, torch.int32, what="flash_attn ctl")
    if ctl.numel() < attn_ctl_words(heads) or not ctl.is_contiguous() or ctl.device != ref.device:
        raise ValueError(f"flash_attn: ctl needs {attn_ctl_words(heads)} contiguous int32 words on {ref.device}")
    return ctl


def flash_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, scale: float | None = None,
               valid_kv: int | None = None, out: torch.Tensor | None = None, pv_f16: bool = True,
               range_flag: torch.Tensor | None = None, v16: torch.Tensor | None = None,
               ctl: torch.Tensor | None = None) -> torch.Tensor:
    """softmax(q k^T * scale) v, non-causal, head_dim 128, batch 1: q/k/v [S, H, d] or [1, S, H, d] (any token/head
    strides that are multiples of 8).  Returns o with q's shape (bf16, contiguous).

    A bf16 v is taken in its whole range, as the reference's cuDNN SDPA takes it (h3_tp2/ulysses_exact.py:495-496):
    its valid rows are converted to f16 (into ``v16``, allocated if not given) and the device runs the f16 P.V
    product on that copy when every value fits f16, else on a copy scaled by a power of two per (head, column) whose
    output columns are scaled back (``h3b_flash_attn_fwd_bf16v``).  ``ctl`` (``attn_ctl(heads)``, allocated if not
    given) then holds 1 in word 0 when the scaled pass ran.  ``pv_f16=False`` runs bf16 P.V directly.  An f16 v (a
    producer's exact f16 copy) is used as is; a ``range_flag`` holding 1 then makes the kernel write nothing and
    record H3B_ERANGE in the device status word."""
    _need_cuda(q, k, v)
    q3, k3, v3 = _as3(q), _as3(k), _as3(v)
    _dt(q3, torch.bfloat16, what="flash_attn q")
    _dt(k3, torch.bfloat16, what="flash_attn k")
    s_q, heads, d = q3.shape
    s_kv = k3.shape[0]
    if k3.shape != (s_kv, heads, d) or v3.shape != k3.shape:
        raise ValueError(f"flash_attn: k and v must be [S_kv, {heads}, {d}] like q's heads, got {tuple(k3.shape)} "
                         f"and {tuple(v3.shape)}")
    _dt(v3, torch.bfloat16, torch.float16, what="flash_attn v")
    o = _out(out, tuple(q.shape), torch.bfloat16, q, "flash_attn", dense=False)
    o3 = _as3(o)
    sc = float(scale) if scale is not None else 1.0 / math.sqrt(d)
    vk = -1 if valid_kv is None else int(valid_kv)
    common = (q3.data_ptr(), q3.stride(0), q3.stride(1), k3.data_ptr(), k3.stride(0), k3.stride(1), v3.data_ptr(),
              v3.stride(0), v3.stride(1), o3.data_ptr(), o3.stride(0), o3.stride(1), s_q, s_kv, vk, heads, d, sc)
    if v3.dtype == torch.bfloat16 and pv_f16:
        rows = s_kv if valid_kv is None else max(0, min(int(valid_kv), s_kv))
        scratch = _v16_scratch(v16, rows, heads, q)
        c = _ctl(ctl, heads, q)
        _lib.call("h3b_flash_attn_fwd_bf16v", *common, scratch.data_ptr(), c.data_ptr(), _stream(q))
        return o
    f16 = v3.dtype == torch.float16
    _lib.call("h3b_flash_attn_fwd", *common, int(f16), _ptr(range_flag) if f16 else None, _stream(q))
    return o


def flash_attn_p2p(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, peer_back, rank: int, *,
                   scale: float | None = None, valid_kv: int | None = None,
                   range_flag: torch.Tensor | None = None, v16: torch.Tensor | None = None,
                   ctl: torch.Tensor | None = None) -> None:
    """Attention of this rank's heads over the gathered sequence (q/k/v [P*M, H/P, d]) whose output row t is stored
    into rank t // M's reverse receive buffer ``peer_back[t // M]`` ([P, M, H/P, d] bf16, slot ``rank``; tensors or
    device addresses): the head->seq all-to-all folded into the epilogue.  A bf16 v is taken in its whole range as in
    ``flash_attn`` (``v16`` / ``ctl`` as there); an f16 v is used as is (a set ``range_flag`` refuses it)."""
    _need_cuda(q, k, v)
    q3, k3, v3 = _as3(q), _as3(k), _as3(v)
    _dt(q3, torch.bfloat16, what="flash_attn_p2p q")
    _dt(k3, torch.bfloat16, what="flash_attn_p2p k")
    _dt(v3, torch.bfloat16, torch.float16, what="flash_attn_p2p v")
    s_q, heads, d = q3.shape
    ws = len(peer_back)
    if ws < 1 or ws > _lib.MAX_RANKS or s_q % ws:
        raise ValueError(f"flash_attn_p2p: {ws} peers for {s_q} query rows")
    if k3.shape[1:] != (heads, d) or v3.shape != k3.shape:
        raise ValueError(f"flash_attn_p2p: k and v must be [S_kv, {heads}, {d}], got {tuple(k3.shape)} and "
                         f"{tuple(v3.shape)}")
    for b in peer_back:
        if isinstance(b, torch.Tensor):
            _out(b, (ws, s_q // ws, heads, d), torch.bfloat16, b, "flash_attn_p2p reverse receive buffer")
    ptrs = (ctypes.c_void_p * ws)(*[_addr(b) for b in peer_back])
    sc = float(scale) if scale is not None else 1.0 / math.sqrt(d)
    s_kv = k3.shape[0]
    vk = -1 if valid_kv is None else int(valid_kv)
    common = (q3.data_ptr(), q3.stride(0), q3.stride(1), k3.data_ptr(), k3.stride(0), k3.stride(1), v3.data_ptr(),
              v3.stride(0), v3.stride(1), ptrs, ws, int(rank), s_q // ws, s_q, s_kv, vk, heads, d, sc)
    if v3.dtype == torch.bfloat16:
        rows = s_kv if valid_kv is None else max(0, min(int(valid_kv), s_kv))
        scratch = _v16_scratch(v16, rows, heads, q)
        c = _ctl(ctl, heads, q)
        _lib.call("h3b_flash_attn_fwd_p2p_bf16v", *common, scratch.data_ptr(), c.data_ptr(), _stream(q))
        return
    _lib.call("h3b_flash_attn_fwd_p2p", *common, 1, _ptr(range_flag), _stream(q))


def p2p_signal_wait(peer_flags, my_flags, rank: int, epoch: int, stream: int) -> None:
    """Epoch barrier over peer memory (one kernel): publish ``epoch`` into slot ``rank`` of every rank's flags,
    then wait (bounded) until this rank's flags all reach it."""
    ws = len(peer_flags)
    ptrs = (ctypes.c_void_p * ws)(*[_addr(f) for f in peer_flags])
    e32 = ((int(epoch) + 2 ** 31) % 2 ** 32) - 2 ** 31
    _lib.call("h3b_p2p_signal_wait", ptrs, _addr(my_flags), ws, int(rank), e32, stream)


# ---------------------------------------------------------------------------------------------------------------
# Ulysses layout kernels
# ---------------------------------------------------------------------------------------------------------------


def pack_by_dest(x: torch.Tensor, ws: int, out: torch.Tensor | None = None, *, to_f16: bool = False,
                 range_flag: torch.Tensor | None = None) -> torch.Tensor:
    """x [M, H, d] (strided) -> send [P, M, H/P, d] contiguous (``ulysses_exact.pack_into``, :119)."""
    _need_cuda(x)
    m, h, d = x.shape
    if x.stride(2) != 1:
        raise ValueError("pack_by_dest: unit innermost stride needed")
    _dt(x, torch.bfloat16, torch.float16, what="pack_by_dest x")
    if to_f16 and x.dtype != torch.bfloat16:
        raise TypeError("pack_by_dest: to_f16 converts bf16 input")
    if ws <= 0 or h % ws:
        raise ValueError(f"pack_by_dest: {h} heads over {ws} ranks")
    dt = torch.float16 if to_f16 else x.dtype
    send = _out(out, (ws, m, h // ws, d), dt, x, "pack_by_dest")
    _lib.call("h3b_pack_by_dest", x.data_ptr(), m, h, d, x.stride(0), x.stride(1), ws, send.data_ptr(),
              int(bool(to_f16)), _ptr(range_flag), _stream(x))
    return send


def norm_rope_send(x: torch.Tensor, weight: torch.Tensor, table: torch.Tensor, eps: float, ws: int,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """qk RMSNorm + partial RoPE of x [M, H, 128] (strided) written into send [P, M, H/P, 128] (the upstream
    norm+RoPE producer as ``ulysses_exact.rope_into_send`` launches it per destination, h3_tp2/ulysses_exact.py:264).
    table [M, R] fp32 holds cos[:R/2] | sin[R/2:] per token."""
    _need_cuda(x, weight, table)
    m, h, d = x.shape
    if d != 128 or x.stride(2) != 1:
        raise ValueError("norm_rope_send: x must be [M, H, 128] with unit innermost stride")
    _dt(x, torch.bfloat16, what="norm_rope_send x")
    if ws <= 0 or h % ws:
        raise ValueError(f"norm_rope_send: {h} heads over {ws} ranks")
    (weight,), table = _norm_rope_args((weight,), table, m, "norm_rope_send")
    send = _out(out, (ws, m, h // ws, d), torch.bfloat16, x, "norm_rope_send")
    _lib.call("h3b_norm_rope_send", x.data_ptr(), m, h, x.stride(0), x.stride(1), weight.data_ptr(),
              table.data_ptr(), table.stride(0), table.shape[-1], float(eps), ws, send.data_ptr(), _stream(x))
    return send


def unpack_recv(recv: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """recv [P, M, hl, d] -> [M, P*hl, d] contiguous (copy 5 of the reverse exchange, :181-183)."""
    _need_cuda(recv)
    _dt(recv, torch.bfloat16, torch.float16, what="unpack_recv recv")
    p, m, hl, d = recv.shape
    o = _out(out, (m, p * hl, d), recv.dtype, recv, "unpack_recv")
    _lib.call("h3b_unpack_recv", recv.contiguous().data_ptr(), p, m, hl, d, o.data_ptr(), _stream(recv))
    return o


def device_status() -> int:
    """Read and clear the library's sticky device status word (0 = no device-side failure since the last read)."""
    return _lib.device_status()


def set_wait_timeout_ns(ns: int) -> None:
    """Bound of every device-side wait in the library (nanoseconds; default 4e9); a wait that runs out records
    H3B_ETIMEOUT in the device status word and its kernel returns.  Bounds below 1 ms are refused."""
    if ns <= 0:
        raise ValueError("set_wait_timeout_ns: the bound must be positive")
    _lib.call("h3b_set_wait_timeout_ns", int(ns))


# ---------------------------------------------------------------------------------------------------------------
# torch.ops.h3b: the op surface the drop-in shims call (registered once, when this module is imported)
# ---------------------------------------------------------------------------------------------------------------
# The reference reaches its GEMM through vLLM's custom op (``ops.cutlass_scaled_mm``, h3_tp2/fp8_gemm.py:386) and its
# quant through ``QuantFP8``; the shims here call these ops, whose CUDA kernels are the functions above.  Only the
# CUDA dispatch key has a kernel: a CPU tensor raises (no CPU fallback).  Each op also has a fake (meta) kernel that
# gives its output shapes, so the ops trace.  Ops that write into a caller's tensor say so in their schema (``a!``).

SCHEMAS = {
    "quant": "quant(Tensor h, int div_mode=0) -> (Tensor, Tensor)",
    "quant_rows": "quant_rows(Tensor base, int m, int p, int seg, int stride_p, int stride_m, int div_mode=0) "
                  "-> (Tensor, Tensor)",
    "quant_from_recv": "quant_from_recv(Tensor recv, int div_mode=0) -> (Tensor, Tensor)",
    "rms_quant": "rms_quant(Tensor x, Tensor weight, Tensor? shift, Tensor? scale, Tensor? indices, float eps, "
                 "Tensor(a!)? ph, int div_mode=0) -> (Tensor, Tensor)",
    "gate_rms_quant": "gate_rms_quant(Tensor residual, Tensor gate, Tensor branch, Tensor weight, Tensor? shift, "
                      "Tensor? scale, Tensor? indices, float eps, int div_mode=0) -> (Tensor, Tensor, Tensor)",
    "silu_mul_quant": "silu_mul_quant(Tensor x, int div_mode=0) -> (Tensor, Tensor)",
    "fp8_gemm": "fp8_gemm(Tensor a, Tensor w, Tensor sa, Tensor sb, Tensor? bias, ScalarType out_dtype) -> Tensor",
    "fp8_gemm_out": "fp8_gemm_out(Tensor a, Tensor w, Tensor sa, Tensor sb, Tensor? bias, Tensor(a!) out) -> ()",
    "fp8_gemm_swiglu": "fp8_gemm_swiglu(Tensor a, Tensor w, Tensor sa, Tensor sb, Tensor? bias) -> Tensor",
    "fp8_gemm_gate": "fp8_gemm_gate(Tensor a, Tensor w, Tensor sa, Tensor sb, Tensor x, Tensor gate, Tensor indices, "
                     "Tensor? bias) -> Tensor",
    "fp8_gemm_gate_out": "fp8_gemm_gate_out(Tensor a, Tensor w, Tensor sa, Tensor sb, Tensor x, Tensor gate, "
                         "Tensor indices, Tensor? bias, Tensor(a!) out) -> ()",
    "flash_attn": "flash_attn(Tensor q, Tensor k, Tensor v, float? scale=None, int? valid_kv=None) -> Tensor",
    "flash_attn_scratch": "flash_attn_scratch(Tensor q, Tensor k, Tensor v, float? scale, int? valid_kv, "
                          "Tensor(a!) v16, Tensor(b!) ctl) -> Tensor",
}


def _kernels() -> dict:
    return {
        "quant": lambda h, div_mode=DIV_IEEE: quant(h, div_mode=div_mode),
        "quant_rows": lambda base, m, p, seg, sp, sm, div_mode=DIV_IEEE: quant_rows(base, m, p, seg, sp, sm,
                                                                                     div_mode=div_mode),
        "quant_from_recv": lambda recv, div_mode=DIV_IEEE: quant_from_recv(recv, div_mode=div_mode),
        "rms_quant": lambda x, w, sh, sc, idx, eps, ph, div_mode=DIV_IEEE: rms_quant(x, w, sh, sc, idx, eps, ph,
                                                                                   div_mode=div_mode),
        "gate_rms_quant": lambda r, g, b, w, sh, sc, idx, eps, div_mode=DIV_IEEE: gate_rms_quant(
            r, g, b, w, sh, sc, idx, eps, div_mode=div_mode),
        "silu_mul_quant": lambda x, div_mode=DIV_IEEE: silu_mul_quant(x, div_mode=div_mode),
        "fp8_gemm": lambda a, w, sa, sb, bias, dt: fp8_gemm(a, w, sa, sb, bias, dt),
        "fp8_gemm_out": lambda a, w, sa, sb, bias, out: (fp8_gemm(a, w, sa, sb, bias, out=out), None)[1],
        "fp8_gemm_swiglu": lambda a, w, sa, sb, bias: fp8_gemm_swiglu(a, w, sa, sb, bias),
        "fp8_gemm_gate": lambda a, w, sa, sb, x, g, idx, bias: fp8_gemm_gate(a, w, sa, sb, x, g, idx, bias),
        "fp8_gemm_gate_out": lambda a, w, sa, sb, x, g, idx, bias, out: (
            fp8_gemm_gate(a, w, sa, sb, x, g, idx, bias, out=out), None)[1],
        "flash_attn": lambda q, k, v, scale=None, valid_kv=None: flash_attn(q, k, v, scale=scale, valid_kv=valid_kv),
        "flash_attn_scratch": lambda q, k, v, scale, valid_kv, v16, ctl: flash_attn(q, k, v, scale=scale,
                                                                                    valid_kv=valid_kv, v16=v16,
                                                                                    ctl=ctl),
    }


def _fakes() -> dict:
    f32 = torch.float32

    def q_and_s(rows, cols, like):
        return like.new_empty((rows, cols), dtype=E4M3), like.new_empty((rows, 1), dtype=f32)

    def attn_out(q):
        return q.new_empty(q.shape, dtype=torch.bfloat16)

    return {
        "quant": lambda h, div_mode=0: q_and_s(h.shape[0], h.shape[1], h),
        "quant_rows": lambda base, m, p, seg, sp, sm, div_mode=0: q_and_s(m, p * seg, base),
        "quant_from_recv": lambda recv, div_mode=0: q_and_s(recv.shape[1], recv.shape[0] * recv.shape[2] *
                                                            recv.shape[3], recv),
        "rms_quant": lambda x, w, sh, sc, idx, eps, ph, div_mode=0: q_and_s(x.shape[0], x.shape[1], x),
        "gate_rms_quant": lambda r, g, b, w, sh, sc, idx, eps, div_mode=0: (
            r.new_empty(r.shape, dtype=torch.bfloat16), *q_and_s(r.shape[0], r.shape[1], r)),
        "silu_mul_quant": lambda x, div_mode=0: q_and_s(x.shape[0], x.shape[1] // 2, x),
        "fp8_gemm": lambda a, w, sa, sb, bias, dt: a.new_empty((a.shape[0], w.shape[0]), dtype=dt),
        "fp8_gemm_out": lambda a, w, sa, sb, bias, out: None,
        "fp8_gemm_swiglu": lambda a, w, sa, sb, bias: a.new_empty((a.shape[0], w.shape[0] // 2),
                                                                  dtype=torch.bfloat16),
        "fp8_gemm_gate": lambda a, w, sa, sb, x, g, idx, bias: x.new_empty((a.shape[0], w.shape[0]),
                                                                           dtype=torch.bfloat16),
        "fp8_gemm_gate_out": lambda a, w, sa, sb, x, g, idx, bias, out: None,
        "flash_attn": lambda q, k, v, scale=None, valid_kv=None: attn_out(q),
        "flash_attn_scratch": lambda q, k, v, scale, valid_kv, v16, ctl: attn_out(q),
    }


def _register() -> None:
    if hasattr(torch.ops, "h3b") and hasattr(torch.ops.h3b, "flash_attn"):
        return   # a second import of this module in the same process (the ops are process-wide)
    lib = torch.library.Library("h3b", "DEF")
    kernels, fakes = _kernels(), _fakes()
    for name, schema in SCHEMAS.items():
        lib.define(schema)
        lib.impl(name, kernels[name], "CUDA")
        torch.library.register_fake(f"h3b::{name}", fakes[name], lib=lib)
    globals()["_LIBRARY"] = lib   # the registrations live as long as the library object


_register()
