"""Fused FP8 fc1 epilogue + SwiGLU (mirrors ``h3_tp2/fp8_swiglu.py``).

``gemm_swiglu`` is the fc1 GEMM whose CTA tile holds gate columns n and up columns F + n in two halves of one TMEM
accumulator; the epilogue applies the scaled epilogue to both, rounds each to bf16, sets up = -0 to +0, computes
silu(g) = g / (1 + exp(-g)) in fp32 (CUDA's ``expf``, IEEE division) rounded to bf16, and writes bf16(silu * up).
``scale_swiglu`` / ``scale_swiglu_quant`` are the same arithmetic over an fp32 product (the two-pass form).
"""
from __future__ import annotations

import logging
import threading

import torch

from . import fp8_gemm, ops

logger = logging.getLogger("h3b.fp8_swiglu")


def scale_swiglu(x32: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    """h3_tp2/fp8_swiglu.py:180."""
    return ops.scale_swiglu(x32, sa, sb, bias)


def scale_swiglu_quant(x32: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, bias: torch.Tensor | None):
    """h3_tp2/fp8_swiglu.py:191: (fp8 [M, F], scale [M, 1])."""
    return ops.scale_swiglu_quant(x32, sa, sb, bias)


def gemm_swiglu(a: torch.Tensor, b: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, bias: torch.Tensor | None,
                cfg=None) -> torch.Tensor:  # noqa: ANN001
    """h3_tp2/fp8_swiglu.py:230: fc1 + epilogue + SwiGLU in one kernel; b [K, 2F] with b.t() contiguous."""
    del cfg
    return torch.ops.h3b.fp8_gemm_swiglu(a, b.t(), sa, sb, bias)


def ffn(x: torch.Tensor, norm_weight: torch.Tensor, w1: torch.Tensor, s1: torch.Tensor, w2: torch.Tensor,
        s2: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """BASELINE config 4's FFN: RMSNorm + per-token quant -> fc1 (gate/up, SwiGLU epilogue) -> per-token quant ->
    fc2.  x [M, C] bf16, w1 [2F, C] e4m3 with per-channel s1, w2 [C, F] e4m3 with s2 -> [M, C] bf16."""
    q, sq = torch.ops.h3b.rms_quant(x, norm_weight, None, None, None, float(eps), None)
    h = torch.ops.h3b.fp8_gemm_swiglu(q, w1, sq, s1, None)
    hq, sh = torch.ops.h3b.quant(h)
    return torch.ops.h3b.fp8_gemm(hq, w2, sh, s2, None, torch.bfloat16)


def swiglu_epilogue_torch(acc: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    """The SwiGLU epilogue in eager torch on an fp32 fc1 product [M, 2*half] (h3_tp2/fp8_swiglu.py:203): the scaled
    epilogue rounded to bf16 for the gate and up halves, up -0 -> +0, silu(g) = g / (1 + exp(-g)) in fp32 rounded to
    bf16, the product rounded to bf16.  torch's exp here, CUDA's expf in the kernel (within 1 bf16 ulp)."""
    h = fp8_gemm.epilogue_torch(acc, sa, sb, bias, torch.bfloat16).float()
    gate, up = h.chunk(2, dim=1)
    up = torch.where(up == 0, torch.zeros_like(up), up)
    silu = (gate / (1.0 + torch.exp(-gate))).to(torch.bfloat16).float()
    return (silu * up).to(torch.bfloat16)


def swiglu_config() -> tuple[int, int, int, int, int]:
    """(BLOCK_M, BLOCK_N, BLOCK_K, warps, stages) of the fc1 + SwiGLU kernel (h3_tp2/fp8_swiglu.py:247 returns the
    Triton kernel's): the FP8 GEMM's CTA-pair tile, whose 256 accumulator columns hold 128 gate and 128 up columns."""
    return fp8_gemm.fused_config()


def probe_gemm_swiglu(device) -> bool:  # noqa: ANN001
    """True when the fused fc1 + SwiGLU kernel serves on ``device`` and equals the eager epilogue on integer inputs
    (exact accumulators in any summation order) within 1 bf16 ulp (torch's exp against CUDA's expf)
    (h3_tp2/fp8_swiglu.py:258)."""
    dev = torch.device(device)
    if dev.type != "cuda" or not torch.cuda.is_available() or torch.cuda.get_device_capability(dev) != (10, 0):
        return False
    g = torch.Generator(device=dev).manual_seed(0)
    a = torch.randint(-3, 4, (130, 64), device=dev, generator=g).to(torch.float8_e4m3fn)
    w = torch.randint(-3, 4, (512, 64), device=dev, generator=g).to(torch.float8_e4m3fn)
    sa = torch.full((130,), 0.5, device=dev)
    sb = torch.full((512,), 0.03125, device=dev)
    y = torch.ops.h3b.fp8_gemm_swiglu(a, w, sa, sb, None)
    ref = swiglu_epilogue_torch(a.float().cpu() @ w.float().cpu().t(), sa.cpu(), sb.cpu(), None)
    diff = (y.cpu().view(torch.int16).int() - ref.view(torch.int16).int()).abs()
    return bool(diff.max().item() <= 1)



# --------------------------------------------------------------------------------------------------------------------
# the MLP wiring (h3_tp2/fp8_swiglu.py:215-421): fc1's GEMM is stashed as its operands, the MLP forward runs fc1 +
# SwiGLU as one kernel from them (no fp32 product exists on this path); level 2 also quantises the SwiGLU output per
# token and runs fc2 on it directly
# --------------------------------------------------------------------------------------------------------------------

_tls = threading.local()   # stash_next / expect_n: fc1's dispatch is to be stashed; stash: (operands, sa, sb, bias)


class GemmOperands:
    """Stashed in place of fc1's product (h3_tp2/fp8_swiglu.py:215): a [M, K] e4m3 and b [K, N] e4m3 (``b.t()``
    contiguous, vLLM's weight layout); the fused GEMM + SwiGLU kernel computes from them."""

    __slots__ = ("a", "b")

    def __init__(self, a: torch.Tensor, b: torch.Tensor):
        self.a, self.b = a, b

    @property
    def shape(self) -> tuple[int, int]:
        return (self.a.shape[0], self.b.shape[1])


def _stash_hook(a, b, scale_a, scale_b, out_dtype, bias):  # noqa: ANN001,ANN202
    """Registered with ``fp8_gemm.set_stash_hook``: while an MLP forward requests it, fc1's dispatch stashes its
    operands and scales and returns an uninitialised bf16 placeholder [M, N] (h3_tp2/fp8_swiglu.py:399)."""
    if not getattr(_tls, "stash_next", False) or out_dtype is not torch.bfloat16:
        return None
    M, N = a.shape[0], b.shape[1]
    expect = getattr(_tls, "expect_n", 0)
    if N % 2 or (expect and N != expect):      # a padded fc1 (N != the logical width) stays on the ordinary path
        _tls.stash_next = False
        return None
    sa, sb = ops.vec_scales(scale_a, scale_b, M, N)
    _tls.stash = (GemmOperands(a, b), sa, sb, bias)
    _tls.stash_next = False
    return torch.empty((M, N), device=a.device, dtype=out_dtype)


def _quant(h: torch.Tensor):  # noqa: ANN202
    return torch.ops.h3b.quant(h)


def _gemm(a: torch.Tensor, w: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor) -> torch.Tensor:
    return torch.ops.h3b.fp8_gemm(a, w, sa, sb, None, torch.bfloat16)


def _fc2_direct(fc2, q: torch.Tensor, scale: torch.Tensor, lead) -> torch.Tensor | None:  # noqa: ANN001
    """fc2 on a pre-quantised input through the tcgen05 GEMM (h3_tp2/fp8_swiglu.py:297): only the plain case this model
    uses (tp 1, no bias, an e4m3 weight [K, N] with its per-channel ``weight_scale``); otherwise None (the caller falls
    back)."""
    w, w_s = getattr(fc2, "weight", None), getattr(fc2, "weight_scale", None)
    if (not isinstance(w, torch.Tensor) or not isinstance(w_s, torch.Tensor) or getattr(fc2, "tp_size", 1) != 1
            or getattr(fc2, "bias", None) is not None or getattr(fc2, "skip_bias_add", False)
            or w.dtype != torch.float8_e4m3fn or w.dim() != 2 or w.shape[0] != q.shape[1]):
        return None
    return _gemm(q, w.t(), scale, w_s.reshape(-1)).view(*lead, w.shape[1])


def make_mlp_forward(orig_forward, *, level: int = 1, lora_layer_type=()):  # noqa: ANN001,ANN201
    """The MLP forward (h3_tp2/fp8_swiglu.py:345): fc1 through the dispatcher with its operands stashed, then fc1 +
    SwiGLU in one kernel (the placeholder fc1 returned is never read); ``level`` 2 also quantises the SwiGLU output
    per token and feeds fc2's GEMM directly.  If nothing was stashed (the dispatch took another route) the stock
    activation runs; LoRA-wrapped layers keep the ordinary forward."""
    def forward(self, x):  # noqa: ANN001,ANN202
        if lora_layer_type and (isinstance(self.fc1, lora_layer_type) or isinstance(self.fc2, lora_layer_type)):
            return orig_forward(self, x)
        _tls.stash_next, _tls.stash = True, None
        _tls.expect_n = int(getattr(self.fc1, "output_size_per_partition", 0) or 0)
        stash = None
        try:
            hidden, _ = self.fc1(x)
            stash = _tls.stash
        finally:
            _tls.stash_next, _tls.stash, _tls.expect_n = False, None, 0
        if stash is None:
            hidden = self.act_fn(hidden)
        else:
            lead = hidden.shape[:-1]
            del hidden
            operands, sa, sb, bias = stash
            del stash
            h = gemm_swiglu(operands.a, operands.b, sa, sb, bias)
            if level >= 2:
                q, scale = _quant(h)
                out = _fc2_direct(self.fc2, q, scale, lead)
                if out is not None:
                    return out
            hidden = h.view(*lead, operands.shape[1] // 2)
        out, _ = self.fc2(hidden)
        return out

    forward._h3b_fused_swiglu = True
    return forward


def _install_on(cls, *, level: int, lora_layer_type) -> bool:  # noqa: ANN001
    if getattr(cls, "_h3b_fused_swiglu", False):
        return False
    cls.forward = make_mlp_forward(cls.forward, level=level, lora_layer_type=lora_layer_type)
    cls._h3b_fused_swiglu = True
    return True


def install(level: int = 1) -> None:
    """Patch vLLM-Omni's ``MiniMaxH3MLP.forward`` and register the stash hook with the FP8 dispatcher
    (h3_tp2/fp8_swiglu.py:315); needs vLLM-Omni."""
    try:
        from vllm_omni.diffusion.models.minimax_h3 import minimax_h3_transformer as tr  # noqa: PLC0415
    except ImportError as exc:  # pragma: no cover - vLLM-Omni is not part of this image
        raise RuntimeError("h3b.fp8_swiglu.install needs vLLM-Omni (not installed)") from exc
    if not fp8_gemm._state.get("installed"):
        logger.warning("h3b: fused FP8 SwiGLU needs the FP8 GEMM dispatcher installed; skipped")
        return
    if torch.cuda.is_available() and not probe_gemm_swiglu("cuda"):
        logger.warning("h3b: the fc1 + SwiGLU kernel does not serve on this device; fused FP8 SwiGLU skipped")
        return
    try:
        from vllm.lora.layers import BaseLayerWithLoRA  # noqa: PLC0415
        lora = (BaseLayerWithLoRA,)
    except ImportError:
        lora = ()
    if _install_on(tr.MiniMaxH3MLP, level=level, lora_layer_type=lora):
        fp8_gemm.set_stash_hook(_stash_hook)
