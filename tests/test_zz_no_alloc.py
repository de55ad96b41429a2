"""The allocation-free attention entry point (h3b_flash_attn_fwd_noalloc), called through the C ABI.

Some callers cannot allocate device memory (a host framework that owns every byte of device memory and exposes no
allocator, a process that must not allocate after start-up); this entry point serves them from a fixed device array
inside the library.  Its output must match the regular bf16-v entry point's (h3b_flash_attn_fwd_bf16v, the same
passes on caller-allocated scratch) and the fp32 SDPA oracle within the attention tolerance, on two calls in a row
(the second reuses the array the first one left behind), including a v beyond f16's range and padding rows beyond
valid_kv that hold values no pass may read.  Its status word reads back through h3b_noalloc_status.  This file is
collected last so a stop-at-first-failure run has already run every other test; it also passes alone in a fresh
process."""
import math

import pytest
import torch

from _util import BF16, rel_l2
from h3b import _lib, ops
from oracle import attention as oa

pytestmark = pytest.mark.gpu

MAX_V_ELEMS = 16 << 20
MAX_HEADS = 256


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


def _close_to_sdpa(o, q, k, v, valid=None):
    ref = oa.sdpa(q.cpu(), k.cpu(), v.cpu(), valid_kv=valid)
    o = o.float().cpu()
    assert rel_l2(o, ref) <= 2e-3, rel_l2(o, ref)
    colscale = ref.abs().amax(dim=0, keepdim=True).clamp_min(1.0)
    assert ((o - ref).abs() / colscale).max().item() <= 2e-2


def test_two_calls_match_the_regular_entry_point(dev):
    for call, (s, h) in enumerate(((1000, 3), (2048, 4))):
        q, k, v = _inputs(s, h, seed=100 + call, dev=dev)
        ref = ops.flash_attn(q, k, v)                                   # regular entry point, caller's scratch
        o = torch.full_like(q, float("nan"))
        assert _noalloc(q, k, v, o) == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert torch.equal(o.view(torch.int16), ref.view(torch.int16))  # same passes, same operands
        _close_to_sdpa(o, q, k, v)
    assert _lib.load().h3b_noalloc_status() == 0


def test_overflowing_v_and_padding_rows(dev):
    """A v beyond f16's range takes the scaled pass; rows beyond valid_kv (inf, nan, huge) are never read; the next
    call, on an ordinary v, starts from a cleared flag again."""
    q, k, v = _inputs(512, 2, seed=7, dev=dev)
    v[100, 1, 5] = 90000.0
    valid = 450
    v[valid:] = float("nan")
    v[valid + 1] = 3.0e20
    k[valid:] = float("inf")
    ctl = ops.attn_ctl(2, dev)
    ref = ops.flash_attn(q, k, v, valid_kv=valid, ctl=ctl)
    assert int(ctl[0].item()) == 1
    o = torch.full_like(q, float("nan"))
    assert _noalloc(q, k, v, o, valid_kv=valid) == 0, _lib.last_error()
    torch.cuda.synchronize()
    assert torch.equal(o.view(torch.int16), ref.view(torch.int16))
    _close_to_sdpa(o, q, k[:valid], v[:valid])
    q2, k2, v2 = _inputs(512, 2, seed=8, dev=dev)
    o2 = torch.full_like(q2, float("nan"))
    assert _noalloc(q2, k2, v2, o2) == 0
    torch.cuda.synchronize()
    assert torch.equal(o2.view(torch.int16), ops.flash_attn(q2, k2, v2).view(torch.int16))
    _close_to_sdpa(o2, q2, k2, v2)
    assert _lib.load().h3b_noalloc_status() == 0


def test_sizes_beyond_the_fixed_array_are_rejected(dev):
    heads = 8
    s_kv = MAX_V_ELEMS // (128 * heads) + 1
    q = torch.empty(128, heads, 128, dtype=BF16, device=dev)
    kv = torch.empty(s_kv, heads, 128, dtype=BF16, device=dev)
    rc = _noalloc(q, kv, kv, torch.empty_like(q))
    assert rc == _lib.H3B_EUNSUPPORTED
    assert "exceeds the fixed scratch" in _lib.last_error()
    # the limit counts the rows the attention reads: the same k/v with valid_kv inside the limit is served
    q, k, v = _inputs(128, heads, seed=9, dev=dev)
    big = torch.zeros(s_kv, heads, 128, dtype=BF16, device=dev)
    big[:128] = k
    bigv = torch.zeros_like(big)
    bigv[:128] = v
    o = torch.empty_like(q)
    assert _noalloc(q, big, bigv, o, valid_kv=128) == 0, _lib.last_error()
    torch.cuda.synchronize()
    _close_to_sdpa(o, q, k, v)
    wide = torch.empty(4, MAX_HEADS + 1, 128, dtype=BF16, device=dev)
    assert _noalloc(wide, wide, wide, torch.empty_like(wide)) == _lib.H3B_EUNSUPPORTED
    assert _lib.load().h3b_noalloc_status() == 0
