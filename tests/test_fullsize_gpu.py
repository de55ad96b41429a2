"""Attention at BASELINE's full per-rank shapes, checked on sampled query rows against the fp32 oracle (the full fp32
reference would be minutes of CPU work): cfg2 at SP=1 (124,992 tokens x 40 heads), cfg3 at SP=4 (366,912 tokens x 10
heads).  Also size-independent properties: every output lies within the per-column range of v (a convex combination)
and heads are independent bit for bit."""
import pytest
import torch

from _util import BF16, rel_l2
from h3b import ops
from oracle import attention as oa

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
