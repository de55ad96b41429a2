"""The reference's eager (CPU) helpers mirrored in the h3b modules, pinned to the golden vectors the reference itself
produced, and its site switches parsed the same way."""
import pytest
import torch

from _util import BF16, same_bits, same_or_both_nan, t8, t16, tf
from h3b import fp8_consumers, fp8_gemm, fp8_quant_fuse, fp8_swiglu, ulysses_outq
from oracle import ulysses as ou


def test_epilogue_torch_matches_the_reference_epilogue(golden):
    g = golden("gemm")
    acc = t8(g["int_a"]).float() @ t8(g["int_w"]).float().t()
    sa, sb, bias = tf(g["int_sa"]), tf(g["int_sb"]), t16(g["int_bias"])
    assert same_bits(fp8_gemm.epilogue_torch(acc, sa, sb, None, BF16), t16(g["int_y"]))
    assert same_bits(fp8_gemm.epilogue_torch(acc, sa, sb, bias, BF16), t16(g["int_ybias"]))
    assert same_bits(fp8_gemm.epilogue_torch(acc, sa.view(-1, 1), sb, None, torch.float16),
                     t16(g["int_yf16"], torch.float16))
    # without a bias the two-pass scale pass is the same arithmetic; with one it adds in fp32 instead of an fma
    assert same_bits(fp8_gemm.scale_bias_cast_torch(acc, sa, sb, None, BF16), t16(g["int_y"]))
    direct = ((sb.view(1, -1) * acc) * sa.view(-1, 1) + bias.view(1, -1).float()).to(BF16)
    assert same_bits(fp8_gemm.scale_bias_cast_torch(acc, sa, sb, bias, BF16), direct)


def test_swiglu_epilogue_torch_matches_the_reference(golden):
    g = golden("swiglu")
    x32, sa, sb, bias = tf(g["x32"]), tf(g["sa"]), tf(g["sb"]), t16(g["bias"])
    assert same_bits(fp8_swiglu.swiglu_epilogue_torch(x32, sa, sb, None), t16(g["y"]))
    assert same_bits(fp8_swiglu.swiglu_epilogue_torch(x32, sa, sb, bias), t16(g["ybias"]))
    assert fp8_swiglu.swiglu_config() == fp8_gemm.fused_config()


def test_quant_torch_and_quant_reference_eager_match_the_reference(golden):
    g = golden("quant")
    for k in ("rand", "dir", "max"):
        x = t16(g[f"{k}_x"])
        for q, s in (fp8_quant_fuse.quant_torch(x), ulysses_outq.quant_reference_eager(x)):
            assert same_bits(q, t8(g[f"{k}_q"]))
            assert same_or_both_nan(s, tf(g[f"{k}_s"]))
    x = t16(g["rand_x"])
    out = (torch.empty(x.shape, dtype=torch.float8_e4m3fn), torch.empty(x.shape[0], 1))
    assert ulysses_outq.quant_reference_eager(x, out=out) is out
    assert same_bits(out[0], t8(g["rand_q"])) and torch.equal(out[1], tf(g["rand_s"]))


def test_epilogue_bf16_torch_broadcasts_like_the_gemm_epilogue(golden):
    g = golden("gemm")
    acc = t8(g["int_a"]).float() @ t8(g["int_w"]).float().t()
    sa, sb, bias = tf(g["int_sa"]), tf(g["int_sb"]), t16(g["int_bias"])
    y = fp8_consumers.epilogue_bf16_torch(acc, sa.view(-1, 1), sb.view(1, -1), bias.view(1, -1).float())
    assert y.dtype == torch.float32
    assert same_bits(y.to(BF16), t16(g["int_ybias"]))


def test_unpack_stock_is_the_reverse_unpack():
    ws, m, hl, d = 2, 5, 3, 8
    recv = torch.randn(ws, m, hl, d, generator=torch.Generator().manual_seed(1)).to(BF16)
    out = fp8_quant_fuse.unpack_stock(recv, ws * hl)
    assert out.shape == (1, m, ws * hl, d) and out.is_contiguous()
    assert torch.equal(out[0].view(torch.int16), ou.unpack(recv).view(torch.int16))
    with pytest.raises(ValueError):
        fp8_quant_fuse.unpack_stock(recv, 5)


@pytest.mark.parametrize("value,sites,explicit", [
    (None, (), False), ("", (), False), ("0", (), False), ("off", (), False), ("1", ("qkv", "out", "fc1", "fc2"), False),
    ("ALL", ("qkv", "out", "fc1", "fc2"), False), ("fc2, qkv", ("qkv", "fc2"), True), ("bogus", (), True)])
def test_quant_fuse_site_switch(value, sites, explicit):
    assert fp8_quant_fuse.parse_sites(value) == sites
    assert fp8_quant_fuse.is_explicit(value) is explicit


def test_consumer_site_switch():
    assert fp8_consumers.parse_sites("true") == ("qkv", "out", "fc2")
    assert fp8_consumers.parse_sites("out,fc1") == ("out",)
    assert fp8_consumers.parse_sites("false") == ()
