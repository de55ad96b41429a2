"""Row kernels on the B200 against the reference's golden vectors and the CPU oracle: per-token quant (bit-exact),
RMSNorm/gated producers, SiLU-mul and SwiGLU scale passes."""
import pytest
import torch

from _util import BF16, E4M3, e4m3_same_or_both_nan, same_bits, same_or_both_nan, t8, t16, tf, ulp_diff_bf16
from h3b import ops
from oracle import gemm as og
from oracle import quant as oq
from oracle import rms as orms

pytestmark = pytest.mark.gpu


def _cmp_quant(q, s, gq, gs):
    assert e4m3_same_or_both_nan(q.cpu(), gq)
    assert same_or_both_nan(s.cpu(), gs)


@pytest.mark.parametrize("case", ["rand", "dir", "max"])
def test_quant_golden(dev, golden, case):
    g = golden("quant")
    q, s = ops.quant(t16(g[f"{case}_x"]).to(dev))
    _cmp_quant(q, s, t8(g[f"{case}_q"]), tf(g[f"{case}_s"]))


def test_quant_recv_and_segmented_rows_golden(dev, golden):
    g = golden("quant")
    q, s = ops.quant_from_recv(t16(g["recv_x"]).to(dev))
    _cmp_quant(q, s, t8(g["recv_q"]), tf(g["recv_s"]))
    m, p, seg, sp, sm = (int(v) for v in g["seg_args"])
    q, s = ops.quant_rows(t16(g["seg_base"]).to(dev), m, p, seg, sp, sm)
    _cmp_quant(q, s, t8(g["seg_q"]), tf(g["seg_s"]))


def test_every_row_maximum_bitwise(dev):
    """Every non-negative bf16 bit pattern 0x0000..0x7F80 (and NaN) as a row's abs-max, K = 7168 read from a
    two-source receive buffer: covers every scale and reciprocal the quant can compute."""
    vals = torch.arange(0, 0x7F81, dtype=torch.int32).to(torch.int16).view(BF16).float()
    vals = torch.cat([vals, torch.tensor([float("nan")])])
    g = torch.Generator().manual_seed(11)
    K, P = 7168, 2
    for c in range(0, vals.numel(), 4096):
        v = vals[c:c + 4096]
        m = v.numel()
        x = ((torch.rand(m, K, generator=g) * 2 - 1) * v[:, None]).to(BF16)
        x = torch.where(torch.isfinite(x.float()) | torch.isnan(v[:, None]), x, torch.zeros_like(x))
        pos = torch.randint(0, K, (m,), generator=g)
        sign = torch.where(torch.rand(m, generator=g) < 0.5, -1.0, 1.0)
        x[torch.arange(m), pos] = (v * sign).to(BF16)
        recv = x.view(m, P, K // P).transpose(0, 1).contiguous()        # [P, M, K/P]: row m = concat_p recv[p, m]
        rq, rs = oq.quant(x)
        q, s = ops.quant_rows(recv.to(dev), m, P, K // P, m * (K // P), K // P)
        _cmp_quant(q, s, rq, rs)


@pytest.mark.parametrize("K", [16, 200, 5120, 13824, 27648, 40000])
def test_quant_widths(dev, K):
    g = torch.Generator().manual_seed(K)
    x = (torch.randn(37, K, generator=g) * torch.rand(37, 1, generator=g) * 30).to(BF16)
    q, s = ops.quant(x.to(dev))
    rq, rs = oq.quant(x)
    _cmp_quant(q, s, rq, rs)


def test_quant_strided_rows_and_empty(dev):
    big = (torch.randn(64, 5120 + 64) * 3).to(BF16)
    h = big.to(dev)[:, :5120]
    q, s = ops.quant(h)
    rq, rs = oq.quant(big[:, :5120])
    _cmp_quant(q, s, rq, rs)
    q, s = ops.quant(torch.empty(0, 128, dtype=BF16, device=dev))
    assert q.shape == (0, 128) and s.shape == (0, 1)


def test_div_full_mode_close_to_ieee(dev):
    x = (torch.randn(4096, 1024) * torch.rand(4096, 1) * 100).to(BF16).to(dev)
    q0, s0 = ops.quant(x)
    q1, s1 = ops.quant(x, div_mode=ops.DIV_FULL)
    d = (s0.view(torch.int32) - s1.view(torch.int32)).abs().max().item()
    assert d <= 2
    # div.full differs from IEEE division by at most 2 ulp: a scale one ulp off moves a few e4m3 roundings
    assert (q0.view(torch.uint8) != q1.view(torch.uint8)).float().mean().item() < 1e-2


def test_rms_quant_golden(dev, golden):
    g = golden("rms")
    x, w, shift, scale = (t16(g[k]).to(dev) for k in ("x", "w", "shift", "scale"))
    idx = torch.from_numpy(g["idx"]).to(dev)
    ph = torch.empty_like(x)
    q, s = ops.rms_quant(x, w, shift, scale, idx, 1e-6, ph)
    h_ref = t16(g["h"])
    ud = ulp_diff_bf16(ph.cpu(), h_ref)
    assert int(ud.max()) <= 1 and (ud == 0).float().mean().item() > 0.99
    rq, rs = oq.quant(ph.cpu())            # the quant of the row it produced is bit-exact
    _cmp_quant(q, s, rq, rs)


def test_rms_quant_plain_dit_width(dev):
    g = torch.Generator().manual_seed(5)
    x = (torch.randn(300, 5120, generator=g) * 2).to(BF16)
    w = (1 + 0.1 * torch.randn(5120, generator=g)).to(BF16)
    ph = torch.empty(300, 5120, dtype=BF16, device=dev)
    q, s = ops.rms_quant(x.to(dev), w.to(dev), eps=1e-6, ph=ph)
    ref = orms.rms_norm_scale_shift(x, w, eps=1e-6)
    ud = ulp_diff_bf16(ph.cpu(), ref)
    assert int(ud.max()) <= 1 and (ud == 0).float().mean().item() > 0.99
    rq, rs = oq.quant(ph.cpu())
    _cmp_quant(q, s, rq, rs)


def test_gate_rms_quant_golden(dev, golden):
    g = golden("rms")
    args = [t16(g[k]).to(dev) for k in ("res", "gate", "branch", "w", "shift", "scale")]
    idx = torch.from_numpy(g["idx"]).to(dev)
    r, q, s = ops.gate_rms_quant(*args, idx, 1e-6)
    ud = ulp_diff_bf16(r.cpu(), t16(g["r_out"]))
    assert int(ud.max()) <= 1 and (ud == 0).float().mean().item() > 0.99
    assert (q.cpu().view(torch.uint8) == t8(g["q2"]).view(torch.uint8)).float().mean().item() > 0.97
    rel = ((s.cpu() - tf(g["s2"])).abs() / tf(g["s2"])).max().item()
    assert rel < 1e-2


def test_silu_mul_quant_golden(dev, golden):
    g = golden("swiglu")
    q, s = ops.silu_mul_quant(t16(g["silu_x"]).to(dev))
    assert (q.cpu().view(torch.uint8) == t8(g["silu_q"]).view(torch.uint8)).float().mean().item() > 0.995
    rel = ((s.cpu() - tf(g["silu_s"])).abs() / tf(g["silu_s"])).max().item()
    assert rel < 1e-2


def test_scale_swiglu_golden(dev, golden):
    g = golden("swiglu")
    x32, sa, sb, bias = tf(g["x32"]).to(dev), tf(g["sa"]).to(dev), tf(g["sb"]).to(dev), t16(g["bias"]).to(dev)
    for b, key in ((None, "y"), (bias, "ybias")):
        y = ops.scale_swiglu(x32, sa, sb, b).cpu()
        ud = ulp_diff_bf16(y, t16(g[key]))
        assert int(ud.max()) <= 1 and (ud == 0).float().mean().item() > 0.99
    d = tf(g["dir_x32"]).to(dev)
    y = ops.scale_swiglu(d, torch.ones(d.shape[0], device=dev), torch.ones(d.shape[1], device=dev), None).cpu()
    ref = t16(g["dir_y"])
    nan = torch.isnan(ref.float())
    assert torch.equal(torch.isnan(y.float()), nan)
    assert int(ulp_diff_bf16(y[~nan], ref[~nan]).max()) <= 1


def test_scale_swiglu_quant(dev, golden):
    g = golden("swiglu")
    q, s = ops.scale_swiglu_quant(tf(g["x32"]).to(dev), tf(g["sa"]).to(dev), tf(g["sb"]).to(dev), None)
    assert (q.cpu().view(torch.uint8) == t8(g["q"]).view(torch.uint8)).float().mean().item() > 0.99
    assert ((s.cpu() - tf(g["s"])).abs() / tf(g["s"])).max().item() < 1e-2


def test_scale_bias_cast(dev):
    g = torch.Generator().manual_seed(9)
    x = torch.randn(77, 400, generator=g) * 1000
    sa, sb = torch.rand(77, generator=g) * 1e-2, torch.rand(400, generator=g) * 1e-2
    bias = (torch.randn(400, generator=g) * 0.1).to(BF16)
    y = ops.scale_bias_cast(x.to(dev), sa.to(dev), sb.to(dev), None, BF16).cpu()
    assert same_bits(y, og.epilogue(x, sa, sb, None, BF16))
    y = ops.scale_bias_cast(x.to(dev), sa.to(dev), sb.to(dev), bias.to(dev), torch.float16).cpu()
    ref = og.epilogue(x, sa, sb, bias, torch.float16)
    assert (y.view(torch.int16) != ref.view(torch.int16)).float().mean().item() < 1e-3


def test_scale_passes_vector_and_scalar_forms_agree(dev, golden):
    """The launchers read sb / bias as 16-byte vectors when aligned and element by element otherwise; both forms give
    the same bits (sb and bias passed at an odd element offset take the element-wise form)."""
    g = golden("swiglu")
    x32, sa, sb, bias = tf(g["x32"]).to(dev), tf(g["sa"]).to(dev), tf(g["sb"]).to(dev), t16(g["bias"]).to(dev)
    sb_odd = torch.empty(sb.numel() + 1, device=dev)[1:]
    sb_odd.copy_(sb)
    b_odd = torch.empty(bias.numel() + 1, dtype=BF16, device=dev)[1:]
    b_odd.copy_(bias)
    assert sb_odd.data_ptr() % 16 and b_odd.data_ptr() % 16
    for b, bo in ((None, None), (bias, b_odd)):
        assert same_bits(ops.scale_swiglu(x32, sa, sb, b), ops.scale_swiglu(x32, sa, sb_odd, bo))
    q1, s1 = ops.scale_swiglu_quant(x32, sa, sb, bias)
    q2, s2 = ops.scale_swiglu_quant(x32, sa, sb_odd, b_odd)
    assert torch.equal(q1.view(torch.uint8), q2.view(torch.uint8)) and torch.equal(s1, s2)


@pytest.mark.parametrize("n", [403, 400])
def test_scale_bias_cast_any_width(dev, n):
    """N % 8 != 0 takes the element-wise kernel, N % 8 == 0 the vector one: both match the eager epilogue."""
    g = torch.Generator().manual_seed(10)
    x = torch.randn(65, n, generator=g) * 100
    sa, sb = torch.rand(65, generator=g) * 1e-2, torch.rand(n, generator=g) * 1e-2
    bias = (torch.randn(n, generator=g) * 0.1).to(BF16)
    y = ops.scale_bias_cast(x.to(dev), sa.to(dev), sb.to(dev), None, BF16).cpu()
    assert same_bits(y, og.epilogue(x, sa, sb, None, BF16))
    # with a bias the oracle adds in double and rounds twice, the kernel rounds one fma: rare last-bit differences
    y = ops.scale_bias_cast(x.to(dev), sa.to(dev), sb.to(dev), bias.to(dev), BF16).cpu()
    ref = og.epilogue(x, sa, sb, bias, BF16)
    assert (y.view(torch.int16) != ref.view(torch.int16)).float().mean().item() < 1e-3
