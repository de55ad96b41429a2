"""Plugin entry point with the reference's environment switches (mirrors the hot-path parts of ``h3_tp2/plugin.py``:
``register`` :74, the Ulysses block :272-308 and the FP8 block :429-505).

``register()`` is a no-op unless ``H3_TP2_ROLE`` is set; a required patch that fails exits the process with code 70,
as the reference does.  The patches themselves need vLLM / vLLM-Omni in the serving environment.
"""
from __future__ import annotations

import logging
import os
import sys
from types import ModuleType

logger = logging.getLogger("h3b.plugin")

_H3_MODULE = "vllm_omni.diffusion.models.minimax_h3.minimax_h3_transformer"


def fused_swiglu_marker() -> str:
    """The fused-SwiGLU class marker of the MiniMax H3 MLP as a startup diagnostic (h3_tp2/plugin.py:34): "present"
    (this plugin patched it), "absent" (not patched) or "unknown" (the module or class is not loaded, or the marker has
    an unexpected value).  Reads only an already-imported module's own dictionary: never imports the model and never
    triggers a lazy module attribute lookup."""
    module = sys.modules.get(_H3_MODULE)
    cls = vars(module).get("MiniMaxH3MLP") if isinstance(module, ModuleType) else None
    if not isinstance(cls, type):
        return "unknown"
    marker = cls.__dict__.get("_h3b_fused_swiglu")
    if marker is True:
        return "present"
    return "absent" if marker in (None, False) else "unknown"


def vllm_strategy_info(layer, attn_metadata):  # noqa: ANN001,ANN201
    """(pg, ws) when vLLM-Omni would run strict Ulysses for ``layer`` with nothing this path does not handle, else None
    (h3_tp2/ulysses_nocopy.py:336-362): the active strategy is plain Ulysses (no ring, no synchronous or permuting
    all-to-all, no ring group), strict mode with scatter 2 / gather 1, no paged KV and no custom attention on the
    layer, no mask, joint tensors or VSA gate in the metadata, and more than one rank."""
    from vllm_omni.diffusion.attention.parallel.ulysses import UlyssesParallelAttention  # noqa: PLC0415
    from vllm_omni.diffusion.forward_context import get_ulysses_mode  # noqa: PLC0415
    import torch.distributed as dist  # noqa: PLC0415

    strategy = layer._get_active_parallel_strategy()
    if not isinstance(strategy, UlyssesParallelAttention) or getattr(layer, "use_ring", False):
        return None
    if get_ulysses_mode(default="strict") != "strict" or (strategy._scatter_idx, strategy._gather_idx) != (2, 1):
        return None
    if strategy._use_sync or getattr(strategy, "_ulysses_a2a_permute", False) or strategy._sp_group.ring_world_size > 1:
        return None
    if getattr(layer, "_scheduler_paged_kv", False) or getattr(layer, "_has_custom_attention", False):
        return None
    if layer._active_paged_kv_adapter() is not None:
        return None
    if attn_metadata is not None and (
            any(getattr(attn_metadata, n, None) is not None for n in
                ("attn_mask", "joint_query", "joint_key", "joint_value", "joint_attn_mask"))
            or "gate_compress" in (getattr(attn_metadata, "extra", None) or {})):
        return None
    pg = strategy._ulysses_pg
    ws = dist.get_world_size(pg)
    return (pg, ws) if ws > 1 else None


def plan(env: dict | None = None) -> dict:
    """The patches ``_apply`` would install for an environment (pure; used by tests)."""
    env = os.environ if env is None else env
    out = {"ulysses": None, "fp8_gemm": None, "swiglu": 0, "consumer_fuse": None, "quant_fuse": None, "overlap": None,
           "nocopy": None, "a2a_timing": False}
    # the reference's precedence (h3_tp2/plugin.py:278-308): the combined exchange only when forced (it runs the
    # overlap's head groups itself), else the exact exchange (default "2"; replaces the overlap when both are set),
    # else the overlap
    ov = env.get("H3_TP2_A2A_OVERLAP", "").strip()
    ov_groups = int(ov) if ov and int(ov) > 1 else 1
    exact = env.get("H3_TP2_ULYSSES_EXACT", "2").strip().lower()
    if env.get("H3_TP2_ULYSSES_NOCOPY", "0") == "force":
        out["nocopy"] = ov_groups
    elif exact not in ("", "0"):
        out["ulysses"] = exact
    elif ov_groups > 1:
        out["overlap"] = ov_groups
    level = env.get("H3_TP2_FP8_GEMM", "cutlass").strip().lower()
    if level not in ("", "0", "off"):
        out["fp8_gemm"] = level
        # the fused SwiGLU MLP rides on the FP8 GEMM dispatcher (h3_tp2/plugin.py:461-469): level 1 by default, 2 also
        # quantises the SwiGLU output for fc2
        sw = env.get("H3_TP2_FP8_FUSE_SWIGLU", "1").strip()
        out["swiglu"] = int(sw) if sw in ("1", "2") else 0
        # consumers fused with the qkv / out / fc2 GEMMs (h3_tp2/plugin.py:479-481): tensor32 and cutlass levels only
        cf = env.get("H3_TP2_FP8_CONSUMER_FUSE", "1").strip().lower()
        if level in ("tensor32", "cutlass") and cf not in ("", "0"):
            out["consumer_fuse"] = cf
    fuse = env.get("H3_TP2_FP8_QUANT_FUSE", "1").strip().lower()
    if fuse not in ("", "0", "off"):
        out["quant_fuse"] = fuse
    out["a2a_timing"] = env.get("H3_TP2_A2A_TIMING", "0").strip() == "1"
    return out


def _apply(role: str) -> None:
    p = plan()
    logger.warning("h3b plugin (%s): %s", role, p)
    if p["a2a_timing"]:
        from . import a2a_timing  # noqa: PLC0415
        a2a_timing.install()
    if p["nocopy"]:
        from . import ulysses_nocopy  # noqa: PLC0415
        ulysses_nocopy.install(p["nocopy"])
    elif p["ulysses"]:
        from . import ulysses_exact  # noqa: PLC0415
        ulysses_exact.install(p["ulysses"])
    elif p["overlap"]:
        from . import ulysses_overlap  # noqa: PLC0415
        ulysses_overlap.install(p["overlap"])
    if p["fp8_gemm"]:
        from . import fp8_gemm  # noqa: PLC0415
        fp8_gemm.install(p["fp8_gemm"])
        level = fp8_gemm._state["level"]          # the level actually running ("stock": the kernel did not serve)
        if level == "cutlass":   # the block's qkv / out / fc1 GEMMs routed by weight (h3_tp2/plugin.py:446-456)
            from . import fp8_cutlass  # noqa: PLC0415
            try:
                fp8_cutlass.install_sites()
            except Exception:  # noqa: BLE001  (the dispatcher's own path stays)
                logger.warning("h3b plugin: FP8 GEMM block wiring failed; the dispatcher's path", exc_info=True)
                fp8_gemm._routers.clear()
        if p["swiglu"] and level != "stock":
            from . import fp8_swiglu  # noqa: PLC0415
            fp8_swiglu.install(level=p["swiglu"])
        if p["consumer_fuse"] and level in ("tensor32", "cutlass"):
            from . import fp8_consumers  # noqa: PLC0415
            try:
                cdone = fp8_consumers.install(fp8_consumers.parse_sites(p["consumer_fuse"]))
            except Exception:  # noqa: BLE001  (an optional fusion must not take the rank down: stock consumers)
                logger.warning("h3b plugin: FP8 consumer fuse install failed; stock consumers", exc_info=True)
                cdone = []
            logger.warning("h3b plugin: FP8 consumer fuse sites installed: %s", ", ".join(cdone) or "none")
    if p["quant_fuse"]:
        from . import fp8_quant_fuse  # noqa: PLC0415
        sites = fp8_quant_fuse.parse_sites(p["quant_fuse"])
        try:
            done = fp8_quant_fuse.install(sites, explicit=fp8_quant_fuse.is_explicit(p["quant_fuse"]))
        except Exception:  # noqa: BLE001  (a failing optional fusion keeps the stock quant, as the reference does)
            logger.warning("h3b plugin: FP8 quant fuse install failed; separate quant kernels", exc_info=True)
            done = []
        logger.warning("h3b plugin: FP8 quant fuse sites installed: %s", ", ".join(done) or "none")


def register() -> None:
    role = os.environ.get("H3_TP2_ROLE", "").strip()
    if not role:
        return
    try:
        _apply(role)
    except Exception:  # noqa: BLE001
        logger.exception("h3b plugin: a required patch failed; exiting (70)")
        os._exit(70)
    logger.warning("h3b plugin (%s): fused SwiGLU marker %s (H3_TP2_FP8_GEMM=%s)", role, fused_swiglu_marker(),
                   os.environ.get("H3_TP2_FP8_GEMM", "<default>"))
