"""Opt-in CUDA-event timing of the Ulysses all-to-alls (``H3_TP2_A2A_TIMING=1``; mirrors ``h3_tp2/a2a_timing.py``).

Wraps the collective ``torch.distributed.all_to_all_single`` (every exchange of this package goes through it, as does
stock's) and, when vLLM-Omni is loaded, its ``comm.all_to_all_4D`` (the permute copies plus the collective) with
events on the current stream, and reports the totals at the end of every ``diffuse`` phase of the MiniMax H3
pipeline.  Measurement only: no tensor is touched.
"""
from __future__ import annotations

import logging

import torch
import torch.distributed as dist

logger = logging.getLogger("h3b.a2a_timing")

_outer: list = []   # (start event, end event, input bytes) per all_to_all_4D call
_inner: list = []   # the same per collective call
_undo: list = []    # (object, attribute, original) to restore


def _event():  # noqa: ANN202
    return torch.cuda.Event(enable_timing=True)


def _sync() -> None:
    torch.cuda.synchronize()


def _timed(orig, record: list, input_pos: int):  # noqa: ANN001,ANN202
    def timed(*args, **kwargs):  # noqa: ANN002,ANN003,ANN202
        s, e = _event(), _event()
        s.record()
        try:
            return orig(*args, **kwargs)
        finally:
            e.record()
            x = args[input_pos] if len(args) > input_pos else kwargs.get("input")
            record.append((s, e, x.numel() * x.element_size() if isinstance(x, torch.Tensor) else 0))

    timed._h3b_a2a_timing = True
    return timed


def _patch(obj, name: str, value) -> None:  # noqa: ANN001
    _undo.append((obj, name, getattr(obj, name)))
    setattr(obj, name, value)


def install(comm=None, pipeline_cls=None) -> None:  # noqa: ANN001
    """Wrap the collective (``dist.all_to_all_single``, and ``comm.dist``'s name for it, which ``comm`` looks up at
    call time), ``comm.all_to_all_4D`` and ``pipeline_cls.diffuse`` (h3_tp2/a2a_timing.py:19).  ``comm`` /
    ``pipeline_cls`` default to vLLM-Omni's when it is importable; without it only the collective is timed."""
    if _undo:
        return
    if comm is None:
        try:
            from vllm_omni.diffusion.distributed import comm  # noqa: PLC0415
        except ImportError:
            comm = None
    if pipeline_cls is None:
        try:
            from vllm_omni.diffusion.models.minimax_h3 import pipeline_minimax_h3 as pp  # noqa: PLC0415
            pipeline_cls = pp.MiniMaxH3Pipeline
        except ImportError:
            pipeline_cls = None
    inner = _timed(dist.all_to_all_single, _inner, 1)
    _patch(dist, "all_to_all_single", inner)
    if comm is not None:
        _patch(comm, "all_to_all_4D", _timed(comm.all_to_all_4D, _outer, 0))
        comm_dist = getattr(comm, "dist", None)
        if comm_dist is not None and comm_dist is not dist:
            _patch(comm_dist, "all_to_all_single", _timed(comm_dist.all_to_all_single, _inner, 1))
    if pipeline_cls is not None:
        orig_diffuse = pipeline_cls.diffuse

        def diffuse(self, *a, **kw):  # noqa: ANN001,ANN002,ANN003,ANN202
            try:
                return orig_diffuse(self, *a, **kw)
            finally:
                try:
                    report("diffuse")
                except Exception:  # noqa: BLE001  (measurement must not fail the request)
                    logger.exception("h3b a2a report failed")

        _patch(pipeline_cls, "diffuse", diffuse)
    logger.info("h3b: all-to-all timing installed")


def uninstall() -> None:
    while _undo:
        obj, name, orig = _undo.pop()
        setattr(obj, name, orig)
    _outer.clear()
    _inner.clear()


def _sum(record: list) -> dict:
    return {"calls": len(record), "s": sum(s.elapsed_time(e) for s, e, _ in record) / 1000.0,
            "bytes": sum(b for _, _, b in record)}


def report(phase: str = "diffuse") -> dict | None:
    """Synchronise, sum the recorded events, log them and clear the record (h3_tp2/a2a_timing.py:73); returns
    {"outer": ..., "inner": ...} with calls, seconds and input bytes, or None when nothing was recorded."""
    if not (_outer or _inner):
        return None
    try:
        _sync()
        out = {"outer": _sum(_outer), "inner": _sum(_inner)}
        logger.info("h3b a2a %s: all_to_all_4D calls=%d %.3f s (%.2f GB in); collective calls=%d %.3f s (%.2f GB in)",
                    phase, out["outer"]["calls"], out["outer"]["s"], out["outer"]["bytes"] / 1e9,
                    out["inner"]["calls"], out["inner"]["s"], out["inner"]["bytes"] / 1e9)
        return out
    finally:
        _outer.clear()
        _inner.clear()
