"""The CPU oracle against golden vectors produced by the reference itself (tests/golden/make_golden.py)."""
import numpy as np
import torch

from _util import BF16, E4M3, same_bits, same_or_both_nan, t8, t16, tf, ulp_diff_bf16
from oracle import gemm as og
from oracle import quant as oq
from oracle import rms as orms
from oracle import ulysses as ou


def test_min_scale_constant_is_the_fp32_division():
    assert np.float32(oq.MIN_SCALE) == np.float32(1.0) / np.float32(229376.0)


def _check_quant(q, s, gq, gs):
    assert same_bits(q, t8(gq))
    assert same_or_both_nan(s, tf(gs))


def test_quant_random_directed_and_rowmax(golden):
    g = golden("quant")
    for k in ("rand", "dir", "max"):
        q, s = oq.quant(t16(g[f"{k}_x"]))
        _check_quant(q, s, g[f"{k}_q"], g[f"{k}_s"])


def test_quant_from_recv_and_segments(golden):
    g = golden("quant")
    q, s = oq.quant_from_recv(t16(g["recv_x"]))
    _check_quant(q, s, g["recv_q"], g["recv_s"])
    m, p, seg, sp, sm = (int(v) for v in g["seg_args"])
    q, s = oq.quant_rows(t16(g["seg_base"]), m, p, seg, sp, sm)
    _check_quant(q, s, g["seg_q"], g["seg_s"])


def test_gemm_integer_inputs_exact(golden):
    g = golden("gemm")
    a, w = t8(g["int_a"]), t8(g["int_w"])
    sa, sb, bias = tf(g["int_sa"]), tf(g["int_sb"]), t16(g["int_bias"])
    assert same_bits(og.scaled_mm(a, w, sa, sb), t16(g["int_y"]))
    assert same_bits(og.scaled_mm(a, w, sa, sb, bias), t16(g["int_ybias"]))
    assert same_bits(og.scaled_mm(a, w, sa, sb, None, torch.float16), t16(g["int_yf16"], torch.float16))


def test_indexed_gate_fc2_epilogue(golden):
    """x + gate[idx] * bf16(fc2 epilogue): the oracle equals the reference's eager mirror bit for bit."""
    g = golden("gate")
    a, w, sa, sb, bias = t8(g["a"]), t8(g["w"]), tf(g["sa"]), tf(g["sb"]), t16(g["bias"])
    x, gate6, idx = t16(g["x"]), t16(g["gate6"]), torch.from_numpy(g["idx"])
    gate = gate6.chunk(6, dim=-1)[5]
    acc = og.accumulate(a, w)
    assert same_bits(og.indexed_gate(x, gate, og.epilogue(acc, sa, sb, None, BF16), idx), t16(g["y"]))
    assert same_bits(og.indexed_gate(x, gate, og.epilogue(acc, sa, sb, bias, BF16), idx), t16(g["ybias"]))


def test_gemm_random_inputs_close(golden):
    g = golden("gemm")
    y = og.scaled_mm(t8(g["rnd_a"]), t8(g["rnd_w"]), tf(g["rnd_sa"]), tf(g["rnd_sb"]))
    ref = t16(g["rnd_y"])
    assert int(ulp_diff_bf16(y, ref).max()) <= 1


def test_swiglu_epilogue(golden):
    g = golden("swiglu")
    x32, sa, sb, bias = tf(g["x32"]), tf(g["sa"]), tf(g["sb"]), t16(g["bias"])
    assert same_bits(og.swiglu_epilogue(x32, sa, sb, None), t16(g["y"]))
    assert same_bits(og.swiglu_epilogue(x32, sa, sb, bias), t16(g["ybias"]))
    q, s = oq.quant(t16(g["y"]))
    assert same_bits(q, t8(g["q"])) and same_bits(s, tf(g["s"]))
    d = tf(g["dir_x32"])
    y = og.swiglu_epilogue(d, torch.ones(d.shape[0]), torch.ones(d.shape[1]), None)
    assert same_or_both_nan(y, t16(g["dir_y"]))


def test_silu_and_mul_and_quant(golden):
    g = golden("swiglu")
    h = og.silu_and_mul(t16(g["silu_x"]))
    assert same_bits(h, t16(g["silu_h"]))
    q, s = oq.quant(h)
    assert same_bits(q, t8(g["silu_q"])) and same_bits(s, tf(g["silu_s"]))


def test_rms_producers(golden):
    g = golden("rms")
    x, w, shift, scale = t16(g["x"]), t16(g["w"]), t16(g["shift"]), t16(g["scale"])
    idx = torch.from_numpy(g["idx"])
    h = orms.rms_norm_scale_shift(x, w, shift, scale, idx, 1e-6)
    assert same_bits(h, t16(g["h"]))
    q, s = oq.quant(h)
    assert same_bits(q, t8(g["q"])) and same_bits(s, tf(g["s"]))
    r, h2 = orms.gate_rms_norm_scale_shift(t16(g["res"]), t16(g["gate"]), t16(g["branch"]), w, shift, scale, idx, 1e-6)
    assert same_bits(r, t16(g["r_out"])) and same_bits(h2, t16(g["h2"]))
    q2, s2 = oq.quant(h2)
    assert same_bits(q2, t8(g["q2"])) and same_bits(s2, tf(g["s2"]))


def _layout_attn(q, k, v):
    return (q.float() + 2.0 * k.float() - 0.5 * v.float()).to(q.dtype)


def test_ulysses_layouts(golden):
    g = golden("ulysses")
    for ws in (2, 4):
        m, heads, d = (int(v) for v in g[f"ws{ws}_shape"])
        qs = [t16(g[f"ws{ws}_q{r}"]) for r in range(ws)]
        ks = [t16(g[f"ws{ws}_k{r}"]) for r in range(ws)]
        vs = [t16(g[f"ws{ws}_v{r}"]) for r in range(ws)]
        for r in range(ws):
            assert same_bits(ou.pack(qs[r][0], ws), t16(g[f"ws{ws}_send{r}"]))

        def body(r, a2a):
            sends = [ou.pack(t[r][0], ws) for t in (qs, ks, vs)]
            recv = []
            for snd in sends:
                rv = torch.empty_like(snd)
                a2a(rv, snd)
                recv.append(rv.view(1, ws * m, heads // ws, d))
            o = _layout_attn(*recv)[0].contiguous()
            back = torch.empty((ws, m, heads // ws, d), dtype=o.dtype)
            a2a(back, o)
            stock_q = ou.stock_all_to_all_4d(qs[r], 2, 1, ws, a2a)
            return ou.unpack(back).view(1, m, heads, d), stock_q

        res = ou.run_ranks(body, ws)
        for r in range(ws):
            assert same_bits(res[r][0], t16(g[f"ws{ws}_out{r}"]))
            assert same_bits(res[r][1], t16(g[f"ws{ws}_stockq{r}"]))


def test_a2a_reference_matches_fake_collective():
    ws, m, h, d = 4, 6, 8, 16
    xs = [torch.randn(ws, m, h // ws, d) for _ in range(ws)]
    got = ou.run_ranks(lambda r, a2a: (lambda out: (a2a(out, xs[r]), out)[1])(torch.empty_like(xs[r])), ws)
    ref = ou.a2a_reference(xs)
    for r in range(ws):
        assert torch.equal(got[r], ref[r])


def test_quant_dtype_contract():
    q, s = oq.quant(torch.randn(4, 64).to(BF16))
    assert q.dtype == E4M3 and s.shape == (4, 1) and s.dtype == torch.float32


def test_norm_rope_into_send(golden):
    g = golden("rope")
    for ws in (2, 4):
        m, heads = (int(v) for v in g[f"ws{ws}_shape"])
        qkv = t16(g[f"ws{ws}_qkv"])
        q, k, _ = (t.view(m, heads, 128) for t in qkv.split([heads * 128] * 3, dim=-1))
        table = tf(g[f"ws{ws}_table"])
        assert same_bits(ou.norm_rope_into_send(q, t16(g[f"ws{ws}_wq"]), table, 1e-6, ws), t16(g[f"ws{ws}_sendq"]))
        assert same_bits(ou.norm_rope_into_send(k, t16(g[f"ws{ws}_wk"]), table, 1e-6, ws), t16(g[f"ws{ws}_sendk"]))


def test_nocopy_combined_exchange(golden):
    """The combined q/k/v exchange (pack [G, P, M, 3, hl, d], one a2a per group, strided views, reverse a2a + unpack)
    restated in the oracle equals the reference's nocopy_forward and pack_qkv bit for bit, over threads."""
    g = golden("nocopy")

    def attn(q, k, v):
        return (q.float() + 2.0 * k.float() - 0.5 * v.float()).to(q.dtype).contiguous()

    for ws, groups in ((2, 1), (2, 2), (4, 1), (4, 2)):
        key = f"ws{ws}_g{groups}"
        m, heads, d = (int(x) for x in g[f"{key}_shape"])
        qs = [t16(g[f"{key}_q{r}"]) for r in range(ws)]
        ks = [t16(g[f"{key}_k{r}"]) for r in range(ws)]
        vs = [t16(g[f"{key}_v{r}"]) for r in range(ws)]
        for r in range(ws):
            assert same_bits(ou.pack_qkv(qs[r][0], ks[r][0], vs[r][0], ws, groups), t16(g[f"{key}_send{r}"]))
        outs = ou.run_ranks(lambda r, a2a: ou.nocopy_forward(qs[r], ks[r], vs[r], attn, ws=ws, groups=groups,
                                                              a2a=a2a), ws)
        for r in range(ws):
            assert same_bits(outs[r], t16(g[f"{key}_out{r}"])), (key, r)


def test_consumer_mirrors(golden):
    """The oracle's norm + RoPE and gated RMS on the bf16 GEMM output equal the reference's eager mirrors of its
    consumer kernels (h3_tp2/fp8_consumers.py:316 _qk_rope_torch, :354 _gate_rms_torch) bit for bit, on exact integer
    products, with the rope table in fp32 and in bf16."""
    g = golden("consumers")
    T, H, D = (int(v) for v in g["qk_shape"])
    y = og.scaled_mm(t8(g["qk_a"]), t8(g["qk_w"]), tf(g["qk_sa"]), tf(g["qk_sb"]))
    q, k = y[:, :H * D].reshape(T, H, D), y[:, H * D:2 * H * D].reshape(T, H, D)
    table = tf(g["qk_table"])
    for tag, tab in (("f32", table), ("bf16", table.to(BF16))):
        for name, x, wt in (("q", q, t16(g["qk_qw"])), ("k", k, t16(g["qk_kw"]))):
            assert same_bits(ou.norm_rope(x, wt, tab, 1e-6), t16(g[f"qk_{name}_{tag}"])), (name, tag)
    branch = og.scaled_mm(t8(g["gr_a"]), t8(g["gr_w"]), tf(g["gr_sa"]), tf(g["gr_sb"]))
    r_out, m_out = orms.gate_rms_norm_scale_shift(t16(g["gr_res"]), t16(g["gr_gate"]), branch, t16(g["gr_nw"]),
                                                  t16(g["gr_shift"]), t16(g["gr_scale"]),
                                                  torch.from_numpy(g["gr_idx"]), 1e-6)
    assert same_bits(r_out, t16(g["gr_res_out"])) and same_bits(m_out, t16(g["gr_mod_out"]))
