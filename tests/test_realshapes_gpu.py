"""The reference's real MiniMax-H3 shapes (56 heads x 128, hidden 5376, FFN 14336, Ulysses P = 2), the shapes its own
GPU tests pin (tests/test_fp8_cutlass_gpu.py:20 SHAPES, tests/test_ulysses_exact.py:19 heads): GEMMs against the
reference's two-pass arithmetic, attention against fp32 SDPA, and the P = 2 block against one rank, bit for bit."""
import pytest
import torch

from _util import BF16, E4M3, rel_l2, ulp_diff_bf16
from h3b import ops
from h3b.block import AttentionBlock
from oracle import attention as oa
from oracle import block as ob
from oracle import ulysses as ou

pytestmark = pytest.mark.gpu

REAL = {"qkv": (21504, 5376), "out": (5376, 7168), "fc1": (28672, 5376), "fc2": (5376, 14336)}


def _quant_rows(rows, cols, std, g, dev):
    x = (torch.randn(rows, cols, generator=g, device=dev) * std).to(BF16).float()
    s = torch.clamp(x.abs().amax(dim=1) / 448.0, min=1.0 / (448.0 * 512.0))
    return torch.clamp(x / s[:, None], -448.0, 448.0).to(E4M3), s


@pytest.mark.parametrize("shape", list(REAL))
def test_real_gemm_shapes(dev, shape):
    N, K = REAL[shape]
    M = 4100
    g = torch.Generator(device=dev).manual_seed(N + K)
    a, sa = _quant_rows(M, K, torch.exp(torch.randn(M, 1, device=dev, generator=g) * 1.5), g, dev)
    w, sb = _quant_rows(N, K, 0.02, g, dev)
    y = ops.fp8_gemm(a, w, sa, sb)
    one = torch.ones((), device=dev)
    ref = ((sb.view(1, -1) * torch._scaled_mm(a, w.t(), scale_a=one, scale_b=one, out_dtype=torch.float32))
           * sa.view(-1, 1)).to(BF16)
    assert rel_l2(y.float(), ref.float()) <= 1e-3
    assert int(ulp_diff_bf16(y.cpu(), ref.cpu()).max()) <= 2


def test_real_attention_28_heads(dev):
    g = torch.Generator().manual_seed(28)
    q, k, v = (torch.randn(2048, 28, 128, generator=g).to(BF16) for _ in range(3))
    o = ops.flash_attn(q.to(dev), k.to(dev), v.to(dev))
    ref = oa.sdpa(q, k, v)
    assert rel_l2(o.float().cpu(), ref) <= 2e-3


def test_real_block_two_ranks_bitwise(dev):
    n, hidden, heads = 512, 5376, 56
    weights = ob.make_weights(hidden, heads, seed=5)
    x = torch.randn(n, hidden, generator=torch.Generator().manual_seed(6)).to(BF16).to(dev)
    full = AttentionBlock(hidden, heads, device=dev, weights=weights)(x)
    torch.cuda.synchronize()

    def body(r, a2a):
        out = AttentionBlock(hidden, heads, device=dev, weights=weights, ws=2, a2a=a2a)(x[r * 256:(r + 1) * 256].contiguous())
        torch.cuda.synchronize()
        return out

    y = torch.cat(ou.run_ranks(body, 2), dim=0)
    assert torch.equal(y.view(torch.int16), full.view(torch.int16))
    ref = ob.fp8_block_local(x.cpu(), *weights, heads)
    assert rel_l2(full.float().cpu(), ref.float()) <= 1e-2
