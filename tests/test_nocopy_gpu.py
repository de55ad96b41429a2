"""The combined q/k/v exchange (h3b.ulysses_nocopy): the qkv GEMM writes the interleaved [G, P, M, 3, hl, d] layout
bit for bit; the mirror's forward reproduces the reference's nocopy_forward (golden vectors, layout-revealing
attention); and the block run with one combined exchange per group equals the single-rank block bitwise."""
import math

import pytest
import torch

from _util import BF16, F16, same_bits, t16
from h3b import ops, ulysses_nocopy
from h3b.block import AttentionBlock
from oracle import block as ob
from oracle import ulysses as ou

pytestmark = pytest.mark.gpu


def _weights(hidden, heads, seed, dev):
    from h3b.block import quant_weight
    g = torch.Generator().manual_seed(seed)
    return (t.to(dev) for t in quant_weight(torch.randn(3 * heads * 128, hidden, generator=g) * 0.02))


@pytest.mark.parametrize("ws,groups,v_f16", [(2, 1, False), (2, 2, True), (4, 1, True), (4, 2, False)])
def test_interleaved_epilogue_equals_separate_sends(dev, ws, groups, v_f16):
    m, hidden, heads = 300, 512, 16
    w8, sw = _weights(hidden, heads, ws + groups, dev)
    x = torch.randn(m, hidden, generator=torch.Generator().manual_seed(3)).to(BF16).to(dev)
    q8, sx = ops.quant(x)
    sends = ops.fp8_gemm_qkv_send(q8, w8, sx, sw, heads, ws, v_f16=v_f16, groups=groups)
    buf = ops.fp8_gemm_qkv_send(q8, w8, sx, sw, heads, ws, v_f16=v_f16, groups=groups, interleaved=True)
    assert buf.shape == (groups, ws, m, 3, heads // (groups * ws), 128)
    for which in range(3):
        want = sends[which] if groups > 1 else sends[which].unsqueeze(0)
        got = buf[:, :, :, which]
        if which == 2 and v_f16:
            got = got.view(F16)
        assert same_bits(got.contiguous().cpu(), want.cpu()), which
    assert ops.device_status() == 0


def test_mirror_forward_matches_reference_golden(dev, golden):
    g = golden("nocopy")

    def attn(q, k, v):
        return (q.float() + 2.0 * k.float() - 0.5 * v.float()).to(q.dtype).contiguous()

    for ws, groups in ((2, 1), (2, 2), (4, 1), (4, 2)):
        key = f"ws{ws}_g{groups}"
        qs = [t16(g[f"{key}_q{r}"]).to(dev) for r in range(ws)]
        ks = [t16(g[f"{key}_k{r}"]).to(dev) for r in range(ws)]
        vs = [t16(g[f"{key}_v{r}"]).to(dev) for r in range(ws)]

        def body(r, a2a):
            out = ulysses_nocopy.nocopy_forward(qs[r], ks[r], vs[r], attn, ws=ws, groups=groups, a2a=a2a)
            torch.cuda.synchronize()
            return out.cpu()

        outs = ou.run_ranks(body, ws)
        for r in range(ws):
            assert same_bits(outs[r], t16(g[f"{key}_out{r}"])), (key, r)


@pytest.mark.parametrize("ws,groups", [(2, 1), (2, 2), (4, 1)])
def test_block_combined_exchange_bitwise(dev, ws, groups):
    n, hidden, heads = 1024, 512, 8
    weights = ob.make_weights(hidden, heads, seed=4)
    x = torch.randn(n, hidden, generator=torch.Generator().manual_seed(9)).to(BF16).to(dev)
    full = AttentionBlock(hidden, heads, device=dev, weights=weights)(x)
    m = n // ws
    torch.cuda.synchronize()

    def body(r, a2a):
        blk = AttentionBlock(hidden, heads, device=dev, weights=weights, ws=ws, a2a=a2a, groups=groups,
                             exchange="nocopy")
        out = blk(x[r * m:(r + 1) * m].contiguous())
        torch.cuda.synchronize()
        return out

    y = torch.cat(ou.run_ranks(body, ws), dim=0)
    assert same_bits(y.cpu(), full.cpu())
    assert ops.device_status() == 0
