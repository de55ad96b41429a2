"""BASELINE config 4, the FP8 SwiGLU FFN at its real widths (hidden 5120 -> gate/up 2 x 13824 -> 5120): RMSNorm +
per-token quant -> fc1 with the SwiGLU epilogue -> per-token quant -> fc2, against the CPU oracle composition of the
reference's eager arithmetic (h3_tp2/fp8_quant_fuse.py rms_quant + quant_torch, h3_tp2/fp8_swiglu.py
swiglu_epilogue_torch, h3_tp2/fp8_gemm.py epilogue_torch)."""
import pytest
import torch

from _util import BF16, rel_l2, ulp_diff_bf16
from h3b import fp8_swiglu, ops
from oracle import gemm as og
from oracle import quant as oq
from oracle import rms as orms

pytestmark = pytest.mark.gpu

C, F = 5120, 13824


@pytest.fixture(scope="module")
def ffn_weights():
    g = torch.Generator().manual_seed(1)
    w1 = torch.randn(2 * F, C, generator=g) * 0.02
    w2 = torch.randn(C, F, generator=g) * 0.02
    nw = (1 + 0.1 * torch.randn(C, generator=g)).to(BF16)
    w1_8, s1 = og.quant_weight(w1)
    w2_8, s2 = og.quant_weight(w2)
    return nw, w1_8, s1, w2_8, s2


@pytest.mark.parametrize("M", [300, 1000])
def test_ffn_real_widths_against_oracle(dev, ffn_weights, M):
    nw, w1_8, s1, w2_8, s2 = ffn_weights
    x = torch.randn(M, C, generator=torch.Generator().manual_seed(M)).to(BF16)
    y = fp8_swiglu.ffn(x.to(dev), nw.to(dev), w1_8.to(dev), s1.to(dev), w2_8.to(dev), s2.to(dev), eps=1e-6)
    # oracle: the same chain on the CPU
    q, sq = orms.rms_quant(x, nw, eps=1e-6)
    h = og.swiglu_epilogue(og.accumulate(q, w1_8), sq, s1, None)
    hq, sh = oq.quant(h)
    ref = og.scaled_mm(hq, w2_8, sh, s2)
    assert y.shape == (M, C) and y.dtype == BF16
    assert rel_l2(y.float(), ref.float()) <= 1e-2


def test_fc1_swiglu_stage_against_oracle(dev, ffn_weights):
    nw, w1_8, s1, _, _ = ffn_weights
    M = 512
    x = torch.randn(M, C, generator=torch.Generator().manual_seed(3)).to(BF16)
    q, sq = ops.rms_quant(x.to(dev), nw.to(dev), eps=1e-6)
    h = ops.fp8_gemm_swiglu(q, w1_8.to(dev), sq, s1.to(dev)).cpu()
    ref = og.swiglu_epilogue(og.accumulate(q.cpu(), w1_8), sq.cpu(), s1, None)
    ud = ulp_diff_bf16(h, ref)
    assert rel_l2(h.float(), ref.float()) <= 2e-3
    assert (ud <= 1).float().mean().item() > 0.99
