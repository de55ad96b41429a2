"""The fused-SwiGLU MLP wiring (h3_tp2/fp8_swiglu.py:215-421) on the CPU with a fake MLP: fc1's dispatch is stashed
as its operands and the MLP runs fc1 + SwiGLU from them (level 1), or also quantises the SwiGLU output and feeds fc2
directly (level 2); the output equals the stock MLP's bit for bit.  The kernels are replaced by eager equivalents (the
oracle's) for these host-logic tests."""
from types import SimpleNamespace

import pytest
import torch

from h3b import fp8_gemm, fp8_swiglu
from oracle import gemm as og
from oracle import quant as oq

BF16 = torch.bfloat16


def _two_pass(a, b, sa, sb, out_dtype, bias=None):
    return og.epilogue(og.accumulate(a, b.t()), sa, sb, bias, out_dtype)


class _Linear:
    """A per-token FP8 linear as vLLM runs it: quantise the input, dispatch the scaled GEMM (weight stored [K, N])."""

    def __init__(self, k, n, seed):
        w8, sb = og.quant_weight(torch.randn(n, k, generator=torch.Generator().manual_seed(seed)) * 0.05)
        self.weight, self.weight_scale = w8.t(), sb
        self.output_size_per_partition, self.tp_size, self.bias = n, 1, None

    def __call__(self, x):
        q, s = oq.quant(x)
        return fp8_gemm.route(q, self.weight, s, self.weight_scale, BF16, None, two_pass=_two_pass), None


def _mlp(c=64, f=96):
    return SimpleNamespace(fc1=_Linear(c, 2 * f, 1), fc2=_Linear(f, c, 2), act_fn=og.silu_and_mul)


def _stock_forward(self, x):
    hidden, _ = self.fc1(x)
    out, _ = self.fc2(self.act_fn(hidden))
    return out


@pytest.fixture
def eager(monkeypatch):
    monkeypatch.setattr(fp8_gemm, "_stash_hooks", [fp8_swiglu._stash_hook])
    monkeypatch.setattr(fp8_gemm, "_routers", [])
    monkeypatch.setattr(fp8_swiglu, "gemm_swiglu",
                        lambda a, b, sa, sb, bias=None, cfg=None: og.swiglu_epilogue(og.accumulate(a, b.t()), sa, sb, bias))
    monkeypatch.setattr(fp8_swiglu, "_quant", oq.quant)
    monkeypatch.setattr(fp8_swiglu, "_gemm", lambda a, w, sa, sb: og.epilogue(og.accumulate(a, w), sa, sb, None, BF16))


@pytest.mark.parametrize("level", [1, 2])
def test_fused_mlp_equals_stock(eager, level, monkeypatch):
    mlp = _mlp()
    x = torch.randn(50, 64, generator=torch.Generator().manual_seed(3)).to(BF16)
    monkeypatch.setattr(fp8_gemm, "_stash_hooks", [])
    ref = _stock_forward(mlp, x)                                     # no stash requested: the two-pass path
    monkeypatch.setattr(fp8_gemm, "_stash_hooks", [fp8_swiglu._stash_hook])
    calls = []
    monkeypatch.setattr(mlp, "act_fn", lambda h: calls.append(1) or og.silu_and_mul(h))
    got = fp8_swiglu.make_mlp_forward(_stock_forward, level=level)(mlp, x)
    assert calls == []                                               # the stock activation never ran
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
    assert getattr(fp8_swiglu._tls, "stash", None) is None


def test_unstashed_dispatch_and_padded_fc1_run_stock(eager):
    """When the dispatch does not stash (another route took fc1, or fc1 is padded) the stock activation runs."""
    mlp = _mlp()
    mlp.fc1.output_size_per_partition = 100                          # the logical width differs: a padded fc1
    x = torch.randn(20, 64, generator=torch.Generator().manual_seed(4)).to(BF16)
    ran = []
    act = mlp.act_fn
    mlp.act_fn = lambda h: ran.append(1) or act(h)
    out = fp8_swiglu.make_mlp_forward(_stock_forward, level=1)(mlp, x)
    assert ran == [1] and out.shape == (20, 64)


def test_fc2_direct_refuses_layers_it_cannot_run():
    q, s = torch.zeros(4, 96, dtype=torch.float8_e4m3fn), torch.ones(4, 1)
    layer = _Linear(96, 64, 5)
    layer.bias = torch.zeros(64)
    assert fp8_swiglu._fc2_direct(layer, q, s, (4,)) is None
    layer.bias, layer.tp_size = None, 2
    assert fp8_swiglu._fc2_direct(layer, q, s, (4,)) is None


def test_stash_hook_takes_fc1_only_when_asked(eager):
    """The hook stashes only while an MLP forward asks for it, only bf16 outputs of the expected even width, once."""
    lin = _Linear(64, 192, 6)
    a, s = oq.quant(torch.randn(8, 64).to(BF16))
    hook = fp8_swiglu._stash_hook
    assert hook(a, lin.weight, s, lin.weight_scale, BF16, None) is None             # not asked
    fp8_swiglu._tls.stash_next, fp8_swiglu._tls.expect_n = True, 192
    try:
        assert hook(a, lin.weight, s, lin.weight_scale, torch.float16, None) is None
        ph = hook(a, lin.weight, s, lin.weight_scale, BF16, None)
        assert ph.shape == (8, 192) and ph.dtype == BF16 and not fp8_swiglu._tls.stash_next
        ops_, sa, sb, bias = fp8_swiglu._tls.stash
        assert ops_.a is a and ops_.b is lin.weight and ops_.shape == (8, 192) and sa.shape == (8,) and bias is None
        assert hook(a, lin.weight, s, lin.weight_scale, BF16, None) is None         # once
        fp8_swiglu._tls.stash_next, fp8_swiglu._tls.expect_n = True, 100             # a padded fc1
        assert hook(a, lin.weight, s, lin.weight_scale, BF16, None) is None and not fp8_swiglu._tls.stash_next
    finally:
        fp8_swiglu._tls.stash_next, fp8_swiglu._tls.stash, fp8_swiglu._tls.expect_n = False, None, 0


def test_mlp_forward_clears_state_on_exception_and_keeps_lora_stock(eager):
    x = torch.randn(10, 64).to(BF16)

    def failing(_x):
        raise RuntimeError("fc1 failed")
    fwd = fp8_swiglu.make_mlp_forward(lambda self, x: (_ for _ in ()).throw(AssertionError()), level=1)
    mlp_fail = SimpleNamespace(fc1=failing, fc2=None, act_fn=None)
    with pytest.raises(RuntimeError, match="fc1 failed"):
        fwd(mlp_fail, x)
    assert not fp8_swiglu._tls.stash_next and fp8_swiglu._tls.stash is None and fp8_swiglu._tls.expect_n == 0
    lora = _mlp()
    stock = []
    fwd = fp8_swiglu.make_mlp_forward(lambda self, x: stock.append(1) or "stock", level=2, lora_layer_type=(_Linear,))
    assert fwd(lora, x) == "stock" and stock == [1]
