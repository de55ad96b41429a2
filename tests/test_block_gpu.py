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
