"""CUDA-event timing of the Ulysses all-to-alls (mirrors ``h3_tp2/a2a_timing.py``): wraps
``torch.distributed.all_to_all_single`` and records (start, end, bytes) per call; ``report()`` sums them."""
from __future__ import annotations

import torch
import torch.distributed as dist

_calls: list = []
_orig = {"fn": None}


def install() -> None:
    if _orig["fn"] is not None:
        return
    orig = dist.all_to_all_single
    _orig["fn"] = orig

    def timed(output, input, *a, **kw):  # noqa: A002,ANN001
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        try:
            return orig(output, input, *a, **kw)
        finally:
            e.record()
            _calls.append((s, e, input.numel() * input.element_size()))

    dist.all_to_all_single = timed


def uninstall() -> None:
    if _orig["fn"] is not None:
        dist.all_to_all_single = _orig["fn"]
        _orig["fn"] = None


def report(reset: bool = True) -> dict:
    """Total milliseconds, bytes and calls since the last report (synchronises on the last event)."""
    if not _calls:
        return {"calls": 0, "ms": 0.0, "bytes": 0}
    _calls[-1][1].synchronize()
    ms = sum(s.elapsed_time(e) for s, e, _ in _calls)
    out = {"calls": len(_calls), "ms": ms, "bytes": sum(b for _, _, b in _calls)}
    if reset:
        _calls.clear()
    return out
