"""Attention at BASELINE's full per-rank shapes, checked on sampled query rows against the fp32 oracle (the full fp32
reference would be minutes of CPU work): cfg2 at SP=1 (124,992 tokens x 40 heads), cfg3 at SP=4 (366,912 tokens x 10
heads).  Also size-independent properties: every output lies within the per-column range of v (a convex combination)
and heads are independent bit for bit.

The qkv projection at cfg2's full M = 124,992 (a 489 x 60 tile schedule) with its send-layout epilogue, on integer
inputs so every output is exact whatever the summation order: all 1.9e9 outputs against the oracle's formula (fp32
accumulation of integers below 2^24 is exact, so the check may run it on the device in row chunks), sampled rows
against the oracle on the CPU, and guard bands around the send buffers."""
import pytest
import torch

from _util import BF16, E4M3, F16, rel_l2, same_bits
from h3b import ops
from oracle import attention as oa
from oracle import gemm as og
from oracle import ulysses as ou

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tokens,heads", [(124_992, 40), (366_912, 10)])
def test_full_shape_sampled_rows(dev, tokens, heads):
    g = torch.Generator(device=dev).manual_seed(tokens)
    q = torch.randn(tokens, heads, 128, device=dev, generator=g).to(BF16)
    k = torch.randn(tokens, heads, 128, device=dev, generator=g).to(BF16)
    v = torch.randn(tokens, heads, 128, device=dev, generator=g).to(BF16)
    o = ops.flash_attn(q, k, v)
    assert ops.device_status() == 0
    rows = torch.tensor([0, 1, 127, 128, 4095, tokens // 2, tokens - 129, tokens - 2, tokens - 1])
    for h in (0, heads - 1):
        ref = oa.sdpa(q[rows, h:h + 1].cpu(), k[:, h:h + 1].cpu(), v[:, h:h + 1].cpu(), chunk=16)
        got = o[rows, h:h + 1].float().cpu()
        assert rel_l2(got, ref) <= 2e-3
        assert (got - ref).abs().max().item() <= 2e-2
    # convexity: each output element lies within [min v, max v] of its head and column
    vmin = v.float().amin(dim=0)
    vmax = v.float().amax(dim=0)
    of = o.float()
    assert bool(((of >= vmin - 1e-2) & (of <= vmax + 1e-2)).all())
    # head independence: recomputing one head alone gives the same bytes
    o1 = ops.flash_attn(q[:, 1:2], k[:, 1:2], v[:, 1:2])
    assert torch.equal(o1.view(torch.int16), o[:, 1:2].contiguous().view(torch.int16))


@pytest.mark.parametrize("ws,v_f16", [(1, False), (8, True)])
def test_qkv_send_epilogue_full_m_integer_exact(dev, ws, v_f16):
    M, heads, K = 124_992, 40, 5120
    N = 3 * heads * 128
    g = torch.Generator(device=dev).manual_seed(ws + 11)
    a = torch.randint(-4, 5, (M, K), device=dev, generator=g).to(E4M3)
    w = torch.randint(-2, 3, (N, K), device=dev, generator=g).to(E4M3)
    sa = torch.rand(M, device=dev, generator=g) * 0.05 + 1e-3
    sb = torch.rand(N, device=dev, generator=g) * 0.05 + 1e-3
    # the three send buffers inside one guarded allocation
    per = M * heads * 128
    guard = 4096
    buf = torch.full((3 * per + 4 * guard,), -1, dtype=torch.int16, device=dev)
    sends = []
    for i in range(3):
        off = guard + i * (per + guard)
        dt = F16 if (i == 2 and v_f16) else BF16
        sends.append(buf[off:off + per].view(dt).view(ws, M, heads // ws, 128))
    out = ops.fp8_gemm_qkv_send(a, w, sa, sb, heads, ws, v_f16=v_f16, sends=sends)
    assert all(o is s_ for o, s_ in zip(out, sends))
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    for i in range(4):
        off = i * (per + guard)
        assert bool((buf[off:off + guard] == -1).all()), f"guard band {i} written"
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False     # fp32 products of integers: exact
    try:
        wf = w.float()
        for r0 in range(0, M, 16_384):
            r1 = min(M, r0 + 16_384)
            y = og.epilogue(a[r0:r1].float() @ wf.t(), sa[r0:r1], sb, None, BF16)
            q, k, v = (t.reshape(r1 - r0, heads, 128) for t in y.split(heads * 128, dim=1))
            v = v.to(F16) if v_f16 else v
            for got, ref in zip(sends, (q, k, v)):
                assert torch.equal(got[:, r0:r1].contiguous().view(torch.int16), ou.pack(ref, ws).view(torch.int16))
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    # the same rows from the CPU oracle (pins the device-side check to it)
    rows = torch.tensor([0, 127, 128, 255, 4096, M // 2, M - 129, M - 128, M - 1])
    y = og.scaled_mm(a[rows.to(dev)].cpu(), w.cpu(), sa[rows.to(dev)].cpu(), sb.cpu())
    q, k, v = (t.reshape(len(rows), heads, 128) for t in y.split(heads * 128, dim=1))
    v = v.to(F16) if v_f16 else v
    hl = heads // ws
    for got, ref in zip(sends, (q, k, v)):
        sampled = got[:, rows.to(dev)].cpu()                                  # [ws, rows, hl, d]
        assert same_bits(sampled, ref.reshape(len(rows), ws, hl, 128).permute(1, 0, 2, 3))
