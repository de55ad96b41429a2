"""The reviewed-upstream-source gate of the model wiring (mirrors ``h3_tp2/step_cache.py:72-86`` and the tables of
``h3_tp2/fp8_consumers.py:67-89``, ``h3_tp2/fp8_quant_fuse.py:856-877``, ``h3_tp2/ulysses_outq.py:57-65``).

The consumer fuse, the quant fuse and the out-projection deferral hand the model uninitialised placeholders and rely
on the upstream code between producer and consumer calling exactly the wrapped functions in between.  They install a
site only when every upstream function on its path has the source the protocol was reviewed against: vLLM-Omni
v0.30.0 (a8576ccb7) and vLLM 0.30.0.  A function's fingerprint is the first 16 hex digits of the sha256 of its source
lines, stripped, without blank, comment and decorator lines; a wrapper made with ``functools.wraps`` is followed to
the function it wraps.  The reviewed values are identifiers of that upstream version and therefore the reference's own.
"""
from __future__ import annotations

import hashlib
import inspect

# fp8_consumers: the block, attention and MLP forwards and the consumer kernels and launchers
REVIEWED = {
    "attn_forward": "b2a25e0b45bea674",                # MiniMaxH3Attention.forward
    "block_forward": "c052863b435652b7",               # MiniMaxH3DiTBlock.forward
    "mlp_forward": "ac9fa6ab2762a4bb",                 # MiniMaxH3MLP.forward (or the fused SwiGLU forward)
    "rms_norm_rope_kernel": "dde848323d52afbd",        # fused_qk_norm_rope._rms_norm_rope_kernel
    "launch_fused_rms_norm_rope": "06631d16d022e0ef",  # fused_qk_norm_rope._launch_fused_rms_norm_rope
    "fused_qk_norm_rope_impl": "dbc570960f4b3a99",     # fused_qk_norm_rope._fused_qk_norm_rope_impl
    "fused_qk_norm_rope": "38d2d10a3af2d594",          # fused_qk_norm_rope.fused_qk_norm_rope
    "fused_cuda_supported": "979429af70cdbf7b",        # fused_qk_norm_rope._fused_cuda_supported
    "indexed_gate_kernel": "9273a7807bd876ab",         # indexed_modulation._indexed_gate_kernel
    "indexed_gate": "0c16c223345767c7",                # indexed_modulation.indexed_gate
    "gate_rms_kernel": "7d239874d6fcab35",             # indexed_modulation._indexed_gate_rms_norm_scale_shift_kernel
    "gate_rms": "b0d503b521d61c64",                    # indexed_modulation.indexed_gate_rms_norm_scale_shift
    "launch_row_chunks": "9260a692db6402e3",           # indexed_modulation._launch_row_chunks
}
CONSUMER_SITE_SOURCES = {
    "qkv": ("block_forward", "attn_forward", "rms_norm_rope_kernel", "launch_fused_rms_norm_rope",
            "fused_qk_norm_rope_impl", "fused_qk_norm_rope", "fused_cuda_supported"),
    "out": ("block_forward", "attn_forward", "gate_rms_kernel", "gate_rms", "launch_row_chunks"),
    "fc2": ("block_forward", "mlp_forward", "indexed_gate_kernel", "indexed_gate", "launch_row_chunks"),
}

# fp8_quant_fuse: the code between each producer and its quant that the table above does not cover
REVIEWED_EXTRA = {
    "rms_kernel": "b791a0e3dec74b2e",          # indexed_modulation._rms_norm_indexed_scale_shift_kernel
    "rms": "373f4b3620d23b43",                 # indexed_modulation.rms_norm_indexed_scale_shift
    "run_packed": "89368785eed0feec",          # MiniMaxH3Attention._run_packed_attention
    "attn_layer_forward": "101199f5a077548b",  # vllm_omni attention layer Attention.forward
    "silu_forward_cuda": "cc7021d08b7cfd95",   # vllm_omni SiluAndMul.forward_cuda
    "col_forward": "af4d0eb5573d0dc6",         # vllm ColumnParallelLinear.forward
    "row_forward": "693d179dcadc13ff",         # vllm RowParallelLinear.forward
    "apply_weights": "54ad02f4f844454d",       # vllm FP8ScaledMMLinearKernel.apply_weights
}
QUANT_SITE_SOURCES = {
    "qkv": ("block_forward", "attn_forward", "rms_kernel", "rms", "launch_row_chunks", "col_forward",
            "apply_weights"),
    "out": ("block_forward", "attn_forward", "run_packed", "attn_layer_forward", "row_forward", "apply_weights"),
    "fc1": ("block_forward", "mlp_forward", "gate_rms_kernel", "gate_rms", "launch_row_chunks", "col_forward",
            "apply_weights"),
    "fc2": ("block_forward", "mlp_forward", "silu_forward_cuda", "row_forward", "apply_weights"),
}

# ulysses_outq: every function between the attention output and the out-projection's quant
OUTQ_REVIEWED = {
    "attn_forward": "b2a25e0b45bea674",   # MiniMaxH3Attention.forward
    "row_forward": "693d179dcadc13ff",    # vllm RowParallelLinear.forward
    "online_apply": "5cbe04cd0e39db60",   # vllm Fp8PerTensorOnlineLinearMethod.apply
    "apply_weights": "54ad02f4f844454d",  # vllm FP8ScaledMMLinearKernel.apply_weights
    "quant_native": "7a11e52df04d77be",   # vllm QuantFP8.forward_native
}


def fingerprint_source(src: str) -> str:
    """sha256 (first 16 hex) of the stripped source lines, blank, comment and decorator lines left out."""
    kept = []
    for line in src.splitlines():
        s = line.strip()
        if s and not s.startswith("#") and not s.startswith("@"):
            kept.append(s)
    return hashlib.sha256("\n".join(kept).encode()).hexdigest()[:16]


def fingerprint(fn) -> str | None:  # noqa: ANN001
    """The fingerprint of ``fn``'s source (a ``functools.wraps`` wrapper is followed), None when it has none."""
    try:
        return fingerprint_source(inspect.getsource(fn))
    except (OSError, TypeError):
        return None


def changed(names, fps: dict, expected: dict) -> list[str]:  # noqa: ANN001
    """The names among ``names`` whose fingerprint is not the reviewed one, as "name got (reviewed want)"."""
    return [f"{n} {fps.get(n)} (reviewed {expected.get(n)})" for n in names if fps.get(n) != expected.get(n)]


def consumer_fingerprints(tr) -> dict[str, str | None]:  # noqa: ANN001
    """The fingerprints the consumer sites need (h3_tp2/fp8_consumers.py:824); the upstream kernels and launchers are
    looked up in vLLM-Omni when it is importable, and a module-level name of ``tr`` that is no longer upstream's own
    function (someone else's wrapper) reads "wrapped"."""
    fps = {"attn_forward": fingerprint(tr.MiniMaxH3Attention.forward),
           "block_forward": fingerprint(tr.MiniMaxH3DiTBlock.forward)}
    fps["mlp_forward"] = REVIEWED["mlp_forward"] if getattr(tr.MiniMaxH3MLP, "_h3b_fused_swiglu", False) \
        else fingerprint(tr.MiniMaxH3MLP.forward)   # the fused SwiGLU forward returns fc2's output unchanged too
    try:
        from vllm_omni.diffusion.layers import fused_qk_norm_rope as fq  # noqa: PLC0415
        from vllm_omni.diffusion.layers import indexed_modulation as im  # noqa: PLC0415
    except ImportError:
        return fps
    src = {"rms_norm_rope_kernel": getattr(fq._rms_norm_rope_kernel, "fn", fq._rms_norm_rope_kernel),
           "launch_fused_rms_norm_rope": fq._launch_fused_rms_norm_rope,
           "fused_qk_norm_rope_impl": fq._fused_qk_norm_rope_impl,
           "fused_qk_norm_rope": fq.fused_qk_norm_rope,
           "fused_cuda_supported": fq._fused_cuda_supported,
           "indexed_gate_kernel": getattr(im._indexed_gate_kernel, "fn", im._indexed_gate_kernel),
           "indexed_gate": im.indexed_gate,
           "gate_rms_kernel": getattr(im._indexed_gate_rms_norm_scale_shift_kernel, "fn",
                                      im._indexed_gate_rms_norm_scale_shift_kernel),
           "gate_rms": im.indexed_gate_rms_norm_scale_shift,
           "launch_row_chunks": im._launch_row_chunks}
    fps.update({k: fingerprint(v) for k, v in src.items()})
    if tr.fused_qk_norm_rope is not fq.fused_qk_norm_rope:
        fps["fused_qk_norm_rope"] = "wrapped"
    if tr.indexed_gate is not im.indexed_gate:
        fps["indexed_gate"] = "wrapped"
    if tr.indexed_gate_rms_norm_scale_shift is not im.indexed_gate_rms_norm_scale_shift:
        fps["gate_rms"] = "wrapped"
    return fps


def quant_fingerprints(tr) -> dict[str, str | None]:  # noqa: ANN001
    """The fingerprints the quant-fuse sites need (h3_tp2/fp8_quant_fuse.py:880): the consumer table's plus the
    producers, the attention layer, the activation and vLLM's linear path."""
    fps = consumer_fingerprints(tr)
    fps["run_packed"] = fingerprint(getattr(tr.MiniMaxH3Attention, "_run_packed_attention", None))
    srcs: dict = {}
    try:
        from vllm_omni.diffusion.layers import indexed_modulation as im  # noqa: PLC0415
        srcs["rms_kernel"] = getattr(im._rms_norm_indexed_scale_shift_kernel, "fn",
                                     im._rms_norm_indexed_scale_shift_kernel)
        srcs["rms"] = im.rms_norm_indexed_scale_shift if tr.rms_norm_indexed_scale_shift is \
            im.rms_norm_indexed_scale_shift else None
    except ImportError:
        pass
    try:
        from vllm_omni.diffusion.attention import layer as layer_mod  # noqa: PLC0415
        srcs["attn_layer_forward"] = layer_mod.Attention.forward
    except ImportError:
        pass
    try:
        from vllm_omni.diffusion.layers.activation import SiluAndMul  # noqa: PLC0415
        srcs["silu_forward_cuda"] = SiluAndMul.forward_cuda
    except ImportError:
        pass
    try:
        from vllm.model_executor.kernels.linear.scaled_mm.ScaledMMLinearKernel import (  # noqa: PLC0415
            FP8ScaledMMLinearKernel)
        from vllm.model_executor.layers import linear as lin  # noqa: PLC0415
        srcs.update(col_forward=lin.ColumnParallelLinear.forward, row_forward=lin.RowParallelLinear.forward,
                    apply_weights=FP8ScaledMMLinearKernel.apply_weights)
    except ImportError:
        pass
    for name, fn in srcs.items():
        fps[name] = fingerprint(fn) if fn is not None else "wrapped"
    return fps


def quant_expected(name: str) -> str | None:
    return REVIEWED_EXTRA[name] if name in REVIEWED_EXTRA else REVIEWED.get(name)


def outq_fingerprints(attn_forward) -> dict[str, str | None]:  # noqa: ANN001
    """The fingerprints of the deferral's path (h3_tp2/ulysses_outq.py:300); ``attn_forward`` is the attention's
    forward as upstream wrote it (before any wrapping)."""
    fps: dict[str, str | None] = {"attn_forward": fingerprint(attn_forward)}
    try:
        from vllm.model_executor.kernels.linear.scaled_mm.ScaledMMLinearKernel import (  # noqa: PLC0415
            FP8ScaledMMLinearKernel)
        from vllm.model_executor.layers.linear import RowParallelLinear  # noqa: PLC0415
        from vllm.model_executor.layers.quantization.input_quant_fp8 import QuantFP8  # noqa: PLC0415
        from vllm.model_executor.layers.quantization.online.fp8 import Fp8PerTensorOnlineLinearMethod  # noqa: PLC0415
    except ImportError:
        return fps
    fps.update(row_forward=fingerprint(RowParallelLinear.forward),
               online_apply=fingerprint(Fp8PerTensorOnlineLinearMethod.apply),
               apply_weights=fingerprint(FP8ScaledMMLinearKernel.apply_weights),
               quant_native=fingerprint(QuantFP8.forward_native))
    return fps
