"""The torch.ops.h3b ops on the GPU against the CPU oracle: attention (fp32 SDPA, rel-L2 <= 2e-3, max-abs <= 2e-2),
the FP8 GEMM (bit-exact on integer inputs; the reference's two-pass arithmetic elsewhere) and the quant (bit-exact)."""
import pytest
import torch

from _util import BF16, E4M3, rel_l2, same_bits
from oracle import attention as oa
from oracle import gemm as og
from oracle import quant as oq

pytestmark = pytest.mark.gpu


def test_flash_attn_op(dev):
    g = torch.Generator().manual_seed(31)
    q, k, v = (torch.randn(1, 777, 3, 128, generator=g).to(BF16) for _ in range(3))
    o = torch.ops.h3b.flash_attn(q.to(dev), k.to(dev), v.to(dev), None, 600).float().cpu()
    ref = oa.sdpa(q[0], k[0], v[0], valid_kv=600)
    assert rel_l2(o[0], ref) <= 2e-3 and (o[0] - ref).abs().max().item() <= 2e-2


def test_fp8_gemm_op(dev):
    g = torch.Generator().manual_seed(32)
    a = torch.randint(-4, 5, (300, 512), generator=g).to(E4M3)
    w = torch.randint(-4, 5, (768, 512), generator=g).to(E4M3)
    sa, sb = torch.rand(300, generator=g) + 0.5, torch.rand(768, generator=g) + 0.5
    y = torch.ops.h3b.fp8_gemm(a.to(dev), w.to(dev), sa.to(dev), sb.to(dev), None, BF16)
    assert same_bits(y, og.scaled_mm(a, w, sa, sb))       # integer inputs: every summation order is exact
    out = torch.empty(300, 768, dtype=BF16, device=dev)
    torch.ops.h3b.fp8_gemm_out(a.to(dev), w.to(dev), sa.to(dev), sb.to(dev), None, out)
    assert same_bits(out, y)
    x = (torch.randn(300, 512, generator=g)).to(BF16)
    q8, sx = torch.ops.h3b.quant(x.to(dev))
    rq, rs = oq.quant(x)
    assert same_bits(q8, rq) and same_bits(sx, rs)
    y2 = torch.ops.h3b.fp8_gemm(q8, w.to(dev), sx, sb.to(dev), None, BF16)
    assert rel_l2(y2.float(), og.scaled_mm(rq, w, rs, sb).float()) <= 1e-2
