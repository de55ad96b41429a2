"""The allocation-free attention entry point (h3b_flash_attn_fwd_noalloc), called through the C ABI.

Some callers cannot allocate device memory (a host framework that owns every byte of device memory and exposes no
allocator, a process that must not allocate after start-up); this entry point serves them from a fixed device array
inside the library.  Its output must match the regular entry point's (h3b_flash_attn_fwd on the f16 copy of v)
within the attention tolerance, on two calls in a row (the second reuses the array the first one left behind), and
must fall back to bf16 P.V when v does not fit f16.  This file is collected last so a stop-at-first-failure run has
already run every other test; it also passes alone in a fresh process."""
import math

import pytest
import torch

from _util import BF16, rel_l2
from h3b import _lib, ops

pytestmark = pytest.mark.gpu

MAX_V_ELEMS = 16 << 20


def _noalloc(q, k, v, o, valid_kv=-1):
    lib = _lib.load()
    s_q, heads, d = q.shape
    return lib.h3b_flash_attn_fwd_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0), k.stride(1), v.data_ptr(), v.stride(0),
        v.stride(1), o.data_ptr(), o.stride(0), o.stride(1), s_q, k.shape[0], valid_kv, heads, d,
        1.0 / math.sqrt(d), torch.cuda.current_stream().cuda_stream)


def _inputs(s, h, seed, dev):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(s, h, 128, generator=g).to(BF16).to(dev) for _ in range(3)]


def test_two_calls_match_the_regular_entry_point(dev):
    for call, (s, h) in enumerate(((1000, 3), (2048, 4))):
        q, k, v = _inputs(s, h, seed=100 + call, dev=dev)
        ref = ops.flash_attn(q, k, v)                                   # regular entry point, f16 copy of v
        o = torch.full_like(q, float("nan"))
        assert _noalloc(q, k, v, o) == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert rel_l2(o.float(), ref.float()) <= 2e-3
        assert (o.float() - ref.float()).abs().max().item() <= 2e-2
        assert torch.equal(o.view(torch.int16), ref.view(torch.int16))  # same kernel, same operands


def test_overflowing_v_takes_the_bf16_path(dev):
    q, k, v = _inputs(512, 2, seed=7, dev=dev)
    v[100, 1, 5] = 90000.0
    ref = ops.flash_attn(q, k, v, pv_f16=False)
    o = torch.empty_like(q)
    assert _noalloc(q, k, v, o) == 0
    torch.cuda.synchronize()
    assert rel_l2(o.float(), ref.float()) <= 2e-3
    q2, k2, v2 = _inputs(512, 2, seed=8, dev=dev)                        # the next call clears the flag again
    o2 = torch.empty_like(q2)
    assert _noalloc(q2, k2, v2, o2) == 0
    torch.cuda.synchronize()
    assert torch.equal(o2.view(torch.int16), ops.flash_attn(q2, k2, v2).view(torch.int16))


def test_sizes_beyond_the_fixed_array_are_rejected(dev):
    heads = 8
    s_kv = MAX_V_ELEMS // (128 * heads) + 1
    q = torch.empty(128, heads, 128, dtype=BF16, device=dev)
    kv = torch.empty(s_kv, heads, 128, dtype=BF16, device=dev)
    rc = _noalloc(q, kv, kv, torch.empty_like(q))
    assert rc == _lib.H3B_EUNSUPPORTED
    assert "exceeds the fixed scratch" in _lib.last_error()
