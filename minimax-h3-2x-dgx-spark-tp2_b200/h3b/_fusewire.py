"""The machinery the two fusion wirings share (``h3b.fp8_quant_fuse``: producers that also quantise;
``h3b.fp8_consumers``: consumers that also run the GEMM's epilogue).

Both wirings follow one contract, the reference's (h3_tp2/fp8_quant_fuse.py:404-700, h3_tp2/fp8_consumers.py:498-919):

* a fusion acts only while a planned DiT block's forward runs in the calling thread (``BlockScope``);
* the fused kernel's result is handed from the call that produces it to the call that consumes it through an
  uninitialised placeholder the model holds meanwhile; anything else that meets the placeholder first makes it real
  (runs the stock code into it) and the stock path continues;
* the first fused call per site and shape is compared bit for bit with the stock code on its first rows
  (``Verdicts``); a mismatch, or a fused kernel that raises, turns the site off for the process.

What differs between the wirings (which calls are wrapped, what a placeholder is, what the stock code is) stays in
their modules; this file holds only the parts that are the same.
"""
from __future__ import annotations

import functools
import logging
import threading
from typing import Any, Callable, Iterable

import torch

CHECK_ROWS = 64   # rows of the first-call comparison


def raw_bits(t: torch.Tensor) -> torch.Tensor:
    """The tensor's bytes as integers of its element size (so NaNs and signed zeros compare by their bits)."""
    t = t.contiguous()
    return t.view({1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}[t.element_size()])


def same_bits(fused: Iterable[torch.Tensor], stock: Iterable[torch.Tensor]) -> bool:
    fused, stock = list(fused), list(stock)
    if len(fused) != len(stock):
        return False
    for f, s in zip(fused, stock):
        if f.shape != s.shape or f.dtype != s.dtype or not torch.equal(raw_bits(f), raw_bits(s)):
            return False
    return True


class Verdicts:
    """First-call comparisons of one wiring.  The verdicts and the set of switched-off sites live in the wiring's
    ``state`` dict (keys ``checked`` and ``disabled``), looked up at every call, so a wiring's state can be replaced
    wholesale (as its tests do)."""

    def __init__(self, state: Callable[[], dict], stats: Callable[[], dict], log: logging.Logger, what: str):
        self._state, self._stats, self._log, self._what = state, stats, log, what

    def off(self, site: str) -> bool:
        return site in self._state()["disabled"]

    def judge(self, key: tuple, fused: Callable[[], tuple], stock: Callable[[], tuple], *, final: bool = True) -> bool:
        """The verdict for ``key`` (whose first element is the site), computed on its first occurrence.  A failed
        verdict on a ``final`` candidate switches the site off."""
        state = self._state()
        known = state["checked"].get(key)
        if known is not None:
            return known
        try:
            verdict = same_bits(fused(), stock())
        except Exception as exc:  # noqa: BLE001  (a fused kernel that raises fails its comparison)
            self._log.warning("h3b %s: comparison %s raised %s: %s", self._what, key, type(exc).__name__, exc)
            verdict = False
        state["checked"][key] = verdict
        self._stats()["selfcheck_pass" if verdict else "selfcheck_fail"] += 1
        if not verdict:
            if final:
                state["disabled"].add(key[0])
            self._log.warning("h3b %s: %s differs from the stock code%s", self._what, key,
                              f"; site {key[0]} off for this process" if final else "")
        return verdict

    def first_passing(self, key: tuple, candidates: tuple, fused_for: Callable[[Any], tuple],
                      stock_for: Callable[[Any], tuple]):
        """The first candidate (in order) whose comparison passes, or None; only the last one's failure switches the
        site off."""
        for i, c in enumerate(candidates):
            if self.judge(key + (c,), lambda c=c: fused_for(c), lambda c=c: stock_for(c),
                          final=i == len(candidates) - 1):
                return c
        return None


class BlockScope:
    """The planned DiT block whose forward runs in this thread, with the handoffs its fusions leave behind.

    ``with BlockScope(registry, block, plan) as scope`` makes ``registry.current()`` return it until the forward
    returns.  On a normal return, handoffs still outstanding are made real (``realize``) for whoever holds their
    placeholders; when the forward raises they are dropped.  Scopes nest (the outer one comes back on exit)."""

    __slots__ = ("block", "plan", "handoffs", "_registry", "_outer")

    def __init__(self, registry: "ScopeRegistry", block: Any, plan: Any):
        self.block, self.plan, self.handoffs = block, plan, {}
        self._registry, self._outer = registry, None

    def __enter__(self) -> "BlockScope":
        self._outer = self._registry.current()
        self._registry.set(self)
        return self

    def __exit__(self, exc_type, exc, tb) -> None:  # noqa: ANN001
        self._registry.set(self._outer)
        if exc_type is None and self.handoffs:
            self._registry.realize_all(self, "left at the end of the block")
        self.handoffs = {}


class ScopeRegistry:
    """Thread-local slot of the running ``BlockScope`` of one wiring, and how that wiring makes a handoff real."""

    def __init__(self, realize: Callable[[Any], None], on_realize: Callable[[str, str], None]):
        self._local = threading.local()
        self._realize, self._on_realize = realize, on_realize

    @property
    def local(self) -> threading.local:
        return self._local

    def current(self) -> BlockScope | None:
        return getattr(self._local, "ctx", None)

    def set(self, scope: BlockScope | None) -> None:
        self._local.ctx = scope

    def realize_all(self, scope: BlockScope, reason: str) -> None:
        pending, scope.handoffs = scope.handoffs, {}
        for site, handoff in pending.items():
            self._realize(handoff)
            self._on_realize(site, reason)


def wrap_block_forward(orig_forward: Callable, registry: ScopeRegistry, plan_for: Callable[..., tuple],
                       on_unplanned: Callable[[str], None], marker: str) -> Callable:
    """The DiT block's forward, run inside a ``BlockScope`` when ``plan_for(block, *args, **kwargs)`` gives a plan
    (``(plan, reason)``; plan None: the stock forward runs untouched)."""
    @functools.wraps(orig_forward)   # keeps __wrapped__: the source fingerprints see upstream's forward
    def forward(self, *args, **kwargs):  # noqa: ANN001,ANN202
        plan, reason = plan_for(self, *args, **kwargs)
        if plan is None:
            on_unplanned(reason)
            return orig_forward(self, *args, **kwargs)
        with BlockScope(registry, self, plan):
            return orig_forward(self, *args, **kwargs)

    setattr(forward, marker, True)
    return forward


def compiling() -> bool:
    fn = getattr(getattr(torch, "compiler", None), "is_compiling", None)
    return bool(fn is not None and fn())


def lora_types() -> tuple:
    try:
        from vllm.lora.layers import BaseLayerWithLoRA  # noqa: PLC0415
        return (BaseLayerWithLoRA,)
    except ImportError:
        return ()


def same_device(kinds: tuple, *ts: torch.Tensor) -> bool:
    """All tensors on one device, of a type in ``kinds``."""
    dev = ts[0].device
    return dev.type in kinds and all(t.device == dev for t in ts)
