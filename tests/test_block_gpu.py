"""The whole attention block (quant -> FP8 qkv with send-layout epilogue -> exchange -> attention -> exchange ->
quant from the receive buffer -> FP8 out projection) against the CPU oracle, and Ulysses ranks (threads on one GPU,
byte-copy collective) against the single-rank block."""
import pytest
import torch

from _util import BF16, rel_l2
from h3b import ops
from h3b.block import AttentionBlock
from oracle import block as ob
from oracle import ulysses as ou

pytestmark = pytest.mark.gpu


def test_block_matches_oracle(dev):
    n, hidden, heads = 1024, 512, 4
    weights = ob.make_weights(hidden, heads, seed=1)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(n, hidden, generator=g).to(BF16)
    blk = AttentionBlock(hidden, heads, device=dev, weights=weights)
    y = blk(x.to(dev))
    ref = ob.fp8_block_local(x, *weights, heads)
    assert y.shape == (n, hidden) and y.dtype == BF16
    assert rel_l2(y.float(), ref.float()) <= 1e-2
    assert ops.device_status() == 0


@pytest.mark.parametrize("ws", [2, 4])
def test_ulysses_ranks_equal_single_rank_bitwise(dev, ws):
    n, hidden, heads = 1024, 512, 8
    weights = ob.make_weights(hidden, heads, seed=2)
    x = torch.randn(n, hidden, generator=torch.Generator().manual_seed(1)).to(BF16).to(dev)
    full = AttentionBlock(hidden, heads, device=dev, weights=weights)(x)
    m = n // ws
    torch.cuda.synchronize()

    def body(r, a2a):
        blk = AttentionBlock(hidden, heads, device=dev, weights=weights, ws=ws, a2a=a2a)
        out = blk(x[r * m:(r + 1) * m].contiguous())
        torch.cuda.synchronize()
        return out

    outs = ou.run_ranks(body, ws)
    y = torch.cat(outs, dim=0)
    assert torch.equal(y.view(torch.int16), full.view(torch.int16))


@pytest.mark.parametrize("ws,groups", [(2, 2), (2, 4), (4, 2)])
def test_head_group_overlap_bitwise(dev, ws, groups):
    """The head-group overlap (grouped send layout, per-group exchanges on the communication stream, quant from the
    grouped reverse buffer) gives the same bytes as the single-rank block."""
    n, hidden, heads = 1024, 512, 8
    weights = ob.make_weights(hidden, heads, seed=3)
    x = torch.randn(n, hidden, generator=torch.Generator().manual_seed(4)).to(BF16).to(dev)
    full = AttentionBlock(hidden, heads, device=dev, weights=weights)(x)
    m = n // ws
    torch.cuda.synchronize()

    def body(r, a2a):
        blk = AttentionBlock(hidden, heads, device=dev, weights=weights, ws=ws, a2a=a2a, groups=groups)
        out = blk(x[r * m:(r + 1) * m].contiguous())
        torch.cuda.synchronize()
        return out

    y = torch.cat(ou.run_ranks(body, ws), dim=0)
    assert torch.equal(y.view(torch.int16), full.view(torch.int16))


def test_grouped_forward_stock_layout_matches_exact_forward(dev):
    from h3b import ulysses_exact, ulysses_overlap

    ws, m, heads = 2, 256, 8
    g = torch.Generator().manual_seed(8)
    qs, ks, vs = ([torch.randn(1, m, heads, 128, generator=g).to(BF16).to(dev) for _ in range(ws)] for _ in range(3))
    attn = ulysses_exact.local_attention
    torch.cuda.synchronize()

    def ref(r, a2a):
        out = ulysses_exact.exact_forward(qs[r], ks[r], vs[r], attn, ws=ws, a2a=a2a)
        torch.cuda.synchronize()
        return out

    def grouped(r, a2a):
        out = ulysses_overlap.grouped_forward(qs[r], ks[r], vs[r], attn, ws=ws, groups=2, a2a=a2a)
        torch.cuda.synchronize()
        return out

    a, b = ou.run_ranks(ref, ws), ou.run_ranks(grouped, ws)
    for r in range(ws):
        assert torch.equal(a[r].view(torch.int16), b[r].view(torch.int16))


def _weights_with_large_v(hidden, heads, seed):
    """Weights whose v channels of head 1 are scaled by 1e5: those v values leave f16's range (|v| > 65504) while q
    and k (and so the softmax) stay ordinary."""
    wqkv8, sqkv, wo8, so = ob.make_weights(hidden, heads, seed=seed)
    sqkv = sqkv.clone()
    hd = heads * 128
    sqkv[2 * hd + 128:2 * hd + 256] *= 1e5
    return wqkv8, sqkv, wo8, so


def test_block_serves_v_outside_f16_by_default(dev):
    """With default settings, a v outside f16's range takes the attention's scaled pass (decided on the device, no
    host read): the output is written and matches the oracle block."""
    n, hidden, heads = 1024, 512, 4
    weights = _weights_with_large_v(hidden, heads, seed=5)
    x = torch.randn(n, hidden, generator=torch.Generator().manual_seed(6)).to(BF16)
    blk = AttentionBlock(hidden, heads, device=dev, weights=weights)
    y = blk(x.to(dev))
    assert int(blk.range_flag.item()) == 1
    assert ops.device_status() == 0
    ref = ob.fp8_block_local(x, *weights, heads)
    assert torch.isfinite(y.float()).all()
    assert rel_l2(y.float(), ref.float()) <= 1e-2
    y2 = blk(x.to(dev))
    assert torch.equal(y2.view(torch.int16), y.view(torch.int16))
    assert ops.device_status() == 0


def test_local_attention_of_the_ulysses_forward_serves_v_outside_f16(dev):
    """The local attention that ulysses_exact's wrapped forward calls (the cuDNN SDPA replacement) takes |v| = 80,000
    with its defaults and stays within rel-L2 2e-3 of fp32 SDPA."""
    from h3b import ulysses_exact
    from oracle import attention as oa
    g = torch.Generator().manual_seed(12)
    s, h = 640, 2
    q, k, v = (torch.randn(1, s, h, 128, generator=g).to(BF16) for _ in range(3))
    v[0, 17, 1, 100] = 80000.0
    v[0, 300, 0, :] = -80000.0
    o = ulysses_exact.local_attention(q.to(dev), k.to(dev), v.to(dev))
    ref = oa.sdpa(q[0], k[0], v[0])
    assert rel_l2(o[0].float().cpu(), ref) <= 2e-3
    assert ops.device_status() == 0


@pytest.mark.parametrize("ws,groups", [(2, 1), (2, 2)])
def test_ulysses_ranks_with_v_outside_f16(dev, ws, groups):
    """Only some ranks' heads see a v beyond f16's range; each rank decides for the v it received, and the ranks'
    rows still equal the single-rank block's bit for bit (a head whose v fits is scaled by 2^0 on the scaled pass)."""
    n, hidden, heads = 1024, 512, 8
    weights = _weights_with_large_v(hidden, heads, seed=7)
    x = torch.randn(n, hidden, generator=torch.Generator().manual_seed(8)).to(BF16)
    x[: n // 2] *= 1e-3
    x = x.to(dev)
    full_blk = AttentionBlock(hidden, heads, device=dev, weights=weights)
    full = full_blk(x)
    assert int(full_blk.range_flag.item()) == 1
    m = n // ws
    torch.cuda.synchronize()

    def body(r, a2a):
        blk = AttentionBlock(hidden, heads, device=dev, weights=weights, ws=ws, a2a=a2a, groups=groups)
        out = blk(x[r * m:(r + 1) * m].contiguous())
        torch.cuda.synchronize()
        return out

    y = torch.cat(ou.run_ranks(body, ws), dim=0)
    assert torch.equal(y.view(torch.int16), full.view(torch.int16))
    assert ops.device_status() == 0


def test_kernel_launches_per_forward_match_the_bench_claim(dev):
    """bench.py reports AttentionBlock.KERNELS_PER_FORWARD launches of this library's kernels per forward: count them
    in a CUDA activity trace of one forward (the library's kernels live in the h3b, attn and gemm namespaces)."""
    from torch.profiler import ProfilerActivity, profile
    n, hidden, heads = 1024, 512, 4
    blk = AttentionBlock(hidden, heads, device=dev, weights=ob.make_weights(hidden, heads, seed=1))
    x = torch.randn(n, hidden, generator=torch.Generator().manual_seed(0)).to(BF16).to(dev)
    blk(x)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        blk(x)
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    ours = [s for s in names if any(ns in s for ns in ("h3b::", "attn::", "gemm::"))]
    assert len(ours) == AttentionBlock.KERNELS_PER_FORWARD, ours
