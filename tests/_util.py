"""Shared helpers for the tests (fixture decoding, bit comparisons)."""
from __future__ import annotations

import numpy as np
import torch

BF16, F16, E4M3 = torch.bfloat16, torch.float16, torch.float8_e4m3fn


def t16(a: np.ndarray, dtype=BF16) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).view(dtype)


def t8(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).view(E4M3)


def tf(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).float()


def bits(t: torch.Tensor) -> torch.Tensor:
    t = t.detach().cpu().contiguous()
    if t.element_size() == 1:
        return t.view(torch.uint8)
    if t.element_size() == 2:
        return t.view(torch.int16)
    return t.view(torch.int32)


def same_bits(a: torch.Tensor, b: torch.Tensor) -> bool:
    return a.shape == b.shape and torch.equal(bits(a), bits(b))


def same_or_both_nan(a: torch.Tensor, b: torch.Tensor) -> bool:
    """Bitwise equal except that any NaN matches any NaN (NaN payloads differ between CPU and GPU arithmetic)."""
    a, b = a.detach().cpu(), b.detach().cpu()
    if a.shape != b.shape:
        return False
    na, nb = torch.isnan(a.float()), torch.isnan(b.float())
    if not torch.equal(na, nb):
        return False
    return torch.equal(bits(a)[~na], bits(b)[~nb])


def e4m3_same_or_both_nan(a: torch.Tensor, b: torch.Tensor) -> bool:
    ua, ub = bits(a), bits(b)
    na, nb = (ua & 0x7F) == 0x7F, (ub & 0x7F) == 0x7F
    return a.shape == b.shape and torch.equal(na, nb) and torch.equal(ua[~na], ub[~nb])


def ulp_diff_bf16(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """|ordinal(a) - ordinal(b)| for finite bf16 values (sign-magnitude to ordinal)."""
    def ordv(x):
        i = bits(x.to(BF16)).to(torch.int32)
        return torch.where(i < 0, -(i & 0x7FFF), i)
    return (ordv(a) - ordv(b)).abs()


def rel_l2(x: torch.Tensor, ref: torch.Tensor) -> float:
    x, ref = x.detach().double().cpu(), ref.detach().double().cpu()
    return float((x - ref).norm() / ref.norm().clamp_min(1e-300))


class CpuKernels:
    """Registers eager stand-ins as the CPU kernels of ``torch.ops.h3b`` ops for the duration of a test (the product
    registers CUDA kernels only, so a CPU tensor reaching an op otherwise raises).  Used by the host-wiring tests,
    which exercise the call protocol on the CPU, not the kernels."""

    def __init__(self, **impls):
        self.impls = impls
        self.lib = None

    def __enter__(self):
        import h3b.ops  # noqa: F401  (the op definitions)
        self.lib = torch.library.Library("h3b", "IMPL")
        for name, fn in self.impls.items():
            self.lib.impl(name, fn, "CPU")
        return self

    def __exit__(self, *exc):
        self.lib._destroy()
        self.lib = None
