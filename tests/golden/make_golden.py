"""Generate the golden vectors that pin the oracle (and, on the GPU, the kernels) to the reference itself.

Runs IN THIS CONTAINER ONLY: it imports the reference package ``h3_tp2`` (and its CPU test fakes) from the read-only
reference checkout given by ``--reference`` (or the ``H3_TP2_REFERENCE`` environment variable), executes the reference's
own CPU/eager functions on seeded inputs built from the recipes of the reference's tests, and writes small ``.npz``
fixtures next to this script.  The GPU box never needs the reference: the fixtures are committed.

    python tests/golden/make_golden.py --reference PATH

Reference functions exercised (paths inside the reference project):
  quant:    h3_tp2/fp8_quant_fuse.py:302 quant_torch, h3_tp2/ulysses_outq.py:109 quant_rows (CPU path),
            h3_tp2/ulysses_outq.py:138 quant_from_recv
  gemm:     h3_tp2/fp8_gemm.py:149 scaled_mm_tensor32 (CPU: torch._scaled_mm + eager scale pass),
            h3_tp2/fp8_gemm.py:174 epilogue_torch
  swiglu:   h3_tp2/fp8_swiglu.py:203 swiglu_epilogue_torch
  rms:      h3_tp2/fp8_quant_fuse.py:330 rms_quant, :350 gate_rms_quant (stock = tests/fake_h3_consumers.py mirrors)
  ulysses:  h3_tp2/ulysses_exact.py:187 exact_forward, :108 send_shape, :119 pack_into, :156 exchange_back, and the
            stock exchange tests/test_ulysses_exact.py:74 stock_all_to_all_4d, with FakeA2A (:25)
  rope:     h3_tp2/ulysses_exact.py:264 rope_into_send with the eager norm+RoPE stand-in tests/test_ulysses_exact.py:107
  nocopy:   h3_tp2/ulysses_nocopy.py:74 send_shape, :84 pack_qkv, :105 qkv_views, :112 back_into, :124 nocopy_forward
            (one combined q/k/v exchange per head group) with FakeA2A, and the stock exchange for comparison
  sources:  h3_tp2/step_cache.py:72 fingerprint_source on sample texts, and the reviewed-source tables
            (h3_tp2/fp8_consumers.py:67-89, h3_tp2/fp8_quant_fuse.py:856-877, h3_tp2/ulysses_outq.py:59) -> sources.json
  consumers: h3_tp2/fp8_consumers.py:316 _qk_rope_torch (q and k blocks, rope table fp32 and bf16) and :354
            _gate_rms_torch on exact integer fp32 products
  gate:     h3_tp2/fp8_consumers.py:367 _gate_torch (the eager mirror of _scale_indexed_gate_kernel) on an exact
            integer fp32 product, gate rows as a row-strided chunk view (recipe of tests/test_fp8_consumer_fuse.py:118)
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
BF16, E4M3 = torch.bfloat16, torch.float8_e4m3fn


def bits16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().copy()


def bits8(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.uint8).numpy().copy()


def f32(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().float().numpy().copy()


def directed_rows(k: int, seg: int, g: torch.Generator) -> torch.Tensor:
    """Edge-case rows after the recipe of tests/test_ulysses_outq_gpu.py:93-113 (zeros, -0, bf16 subnormals, huge
    values, +-inf, NaN, maxima on both sides of a segment boundary, bf16 max, one empty segment, exactly 448, a ramp)."""
    x = (torch.randn(16, k, generator=g) * 2).to(BF16)
    x[0] = 0
    x[1] = -0.0
    x[2] = (torch.randn(k, generator=g) * 1e-38).to(BF16)
    x[3] = (torch.randn(k, generator=g) * 1e36).to(BF16)
    x[4, 17] = float("inf")
    x[5, k - 3] = float("nan")
    x[6, 9] = float("-inf")
    x[7, seg - 1] = 900.0
    x[8, seg] = -900.0
    x[9] = torch.finfo(BF16).max
    x[10, :seg] = 0
    x[11, seg:] = 0
    x[12] = 448.0
    x[13] = ((torch.arange(k) % 448 - 224).float() * 0.01).to(BF16)
    x[14] = (torch.rand(k, generator=g) * 1e-3).to(BF16)
    x[15] = -(torch.rand(k, generator=g) * 3e4).to(BF16)
    return x


def rowmax_rows(k: int, step: int, g: torch.Generator) -> torch.Tensor:
    """Rows whose abs-max runs over every ``step``-th non-negative finite bf16 bit pattern (plus NaN), random
    elements below it, after tests/test_ulysses_outq_gpu.py:115-132."""
    vals = torch.arange(0, 0x7F81, step, dtype=torch.int32).to(torch.int16).view(BF16).float()
    vals = torch.cat([vals, torch.tensor([float("nan")])])
    m = vals.numel()
    x = ((torch.rand(m, k, generator=g) * 2 - 1) * vals[:, None]).to(BF16)
    x = torch.where(torch.isfinite(x.float()) | torch.isnan(vals[:, None]), x, torch.zeros_like(x))
    pos = torch.randint(0, k, (m,), generator=g)
    sign = torch.where(torch.rand(m, generator=g) < 0.5, -1.0, 1.0)
    x[torch.arange(m), pos] = (vals * sign).to(BF16)
    return x


def gen_quant(fq, oq) -> dict:
    g = torch.Generator().manual_seed(0)
    out = {}
    x = (torch.randn(96, 640, generator=g) * torch.rand(96, 1, generator=g) * 8).to(BF16)
    q, s = fq.quant_torch(x)
    out.update(rand_x=bits16(x), rand_q=bits8(q), rand_s=f32(s))
    x = directed_rows(512, 256, g)
    q, s = fq.quant_torch(x)
    out.update(dir_x=bits16(x), dir_q=bits8(q), dir_s=f32(s))
    x = rowmax_rows(256, 64, g)
    q, s = fq.quant_torch(x)
    out.update(max_x=bits16(x), max_q=bits8(q), max_s=f32(s))
    recv = (torch.randn(2, 40, 2, 128, generator=g) * 3).to(BF16)       # [P, M, hl, d] receive buffer
    q, s = oq.quant_from_recv(recv)
    out.update(recv_x=bits16(recv), recv_q=bits8(q), recv_s=f32(s))
    base = (torch.randn(3 * 24 * 96 + 64, generator=g)).to(BF16)        # generic segmented addressing
    q, s = oq.quant_rows(base, 24, 3, 80, 24 * 96, 96)
    out.update(seg_base=bits16(base), seg_q=bits8(q), seg_s=f32(s), seg_args=np.array([24, 3, 80, 24 * 96, 96]))
    return out


def _quant_rows_t(rows, cols, std, g):
    x = (torch.randn(rows, cols, generator=g) * std).to(BF16).float()
    s = torch.clamp(x.abs().amax(dim=1) / 448.0, min=1.0 / (448.0 * 512.0))
    return torch.clamp(x / s[:, None], -448.0, 448.0).to(E4M3), s


def gen_gemm(fg) -> dict:
    g = torch.Generator().manual_seed(1)
    fg._state["triton"] = False   # eager scale pass on the CPU (h3_tp2/fp8_gemm.py:160-163)
    out = {}
    M, N, K = 200, 400, 512       # partial row / column tiles for a 128 x 256 tile
    a = torch.randint(-4, 5, (M, K), generator=g).to(E4M3)
    w = torch.randint(-2, 3, (N, K), generator=g).to(E4M3)
    sa = torch.exp(torch.empty(M).uniform_(-9.0, -2.0, generator=g))
    sb = torch.exp(torch.empty(N).uniform_(-9.5, -7.5, generator=g))
    bias = (torch.randn(N, generator=g) * 0.1).to(BF16)
    y = fg.scaled_mm_tensor32(a, w.t(), sa.view(M, 1), sb, BF16)
    acc = a.float() @ w.float().t()
    yb = fg.epilogue_torch(acc, sa, sb, bias, BF16)
    y16 = fg.epilogue_torch(acc, sa, sb, None, torch.float16)
    out.update(int_a=bits8(a), int_w=bits8(w), int_sa=f32(sa), int_sb=f32(sb), int_bias=bits16(bias),
               int_y=bits16(y), int_ybias=bits16(yb), int_yf16=bits16(y16))
    M, N, K = 130, 272, 384
    a, sa = _quant_rows_t(M, K, 1.0, g)
    w, sb = _quant_rows_t(N, K, 0.02, g)
    y = fg.scaled_mm_tensor32(a, w.t(), sa.view(M, 1), sb, BF16)
    out.update(rnd_a=bits8(a), rnd_w=bits8(w), rnd_sa=f32(sa), rnd_sb=f32(sb), rnd_y=bits16(y))
    return out


def gen_swiglu(fs, fq) -> dict:
    g = torch.Generator().manual_seed(2)
    out = {}
    M, width = 48, 512
    x32 = torch.randn(M, width, generator=g) * 3000
    sa = torch.rand(M, generator=g) * 0.01 + 0.001
    sb = torch.rand(width, generator=g) * 0.01 + 0.001
    bias = (torch.randn(width, generator=g) * 0.1).to(BF16)
    y = fs.swiglu_epilogue_torch(x32, sa, sb, None)
    yb = fs.swiglu_epilogue_torch(x32, sa, sb, bias)
    q, s = fq.quant_torch(y)
    out.update(x32=f32(x32), sa=f32(sa), sb=f32(sb), bias=bits16(bias), y=bits16(y), ybias=bits16(yb), q=bits8(q),
               s=f32(s))
    vals = torch.tensor([0.0, -0.0, 1e-40, -1e-40, 1.0, -1.0, 88.0, -88.0, 1e4, -1e4, 0.5000001, 1.9999999,
                         float("inf"), -float("inf"), float("nan")])
    width = 2 * 1504
    d = vals.repeat(1, width // vals.numel() + 1)[:, :width].clone()
    d = torch.cat([d, torch.randn(7, width, generator=g) * 100])
    ones_a, ones_b = torch.ones(d.shape[0]), torch.ones(width)
    out.update(dir_x32=f32(d), dir_y=bits16(fs.swiglu_epilogue_torch(d, ones_a, ones_b, None)))
    # silu_and_mul of a bf16 [M, 2d] input (= the epilogue with unit scales) and its per-token quant
    xb = (torch.randn(32, 2 * 384, generator=g) * 4).to(BF16)
    h = fs.swiglu_epilogue_torch(xb.float(), torch.ones(32), torch.ones(768), None)
    q, s = fq.quant_torch(h)
    out.update(silu_x=bits16(xb), silu_h=bits16(h), silu_q=bits8(q), silu_s=f32(s))
    return out


def gen_rms(fq, fake) -> dict:
    g = torch.Generator().manual_seed(3)
    M, H = 32, 512
    x = (torch.randn(M, H, generator=g) * 2).to(BF16)
    w = (1 + 0.1 * torch.randn(H, generator=g)).to(BF16)
    shift = (torch.randn(4, H, generator=g) * 0.1).to(BF16)
    scale = (torch.randn(4, H, generator=g) * 0.1).to(BF16)
    idx = torch.randint(0, 4, (M,), generator=g)
    h = fake.rms_norm_indexed_scale_shift(x, w, shift, scale, idx, 1e-6)
    q, s = fq.rms_quant(x, w, shift, scale, idx, 1e-6, stock=fake.rms_norm_indexed_scale_shift)
    res = (torch.randn(M, H, generator=g) * 2).to(BF16)
    gate = (torch.randn(4, H, generator=g) * 0.5).to(BF16)
    branch = (torch.randn(M, H, generator=g)).to(BF16)
    r_out, h2 = fake.indexed_gate_rms_norm_scale_shift(res, gate, branch, w, shift, scale, idx, 1e-6)
    r2, q2, s2 = fq.gate_rms_quant(res, gate, branch, w, shift, scale, idx, 1e-6,
                                   stock=fake.indexed_gate_rms_norm_scale_shift)
    assert torch.equal(r2.view(torch.int16), r_out.view(torch.int16))
    return dict(x=bits16(x), w=bits16(w), shift=bits16(shift), scale=bits16(scale), idx=idx.numpy(), h=bits16(h),
                q=bits8(q), s=f32(s), res=bits16(res), gate=bits16(gate), branch=bits16(branch), r_out=bits16(r_out),
                h2=bits16(h2), q2=bits8(q2), s2=f32(s2))


def gen_ulysses(ux, tue) -> dict:
    out = {}
    heads, d = 8, 128
    for ws, m in ((2, 16), (4, 8)):
        g = torch.Generator().manual_seed(10 + ws)
        qs = [(torch.randn(1, m, heads, d, generator=g)).to(BF16) for _ in range(ws)]
        ks = [(torch.randn(1, m, heads, d, generator=g)).to(BF16) for _ in range(ws)]
        vs = [(torch.randn(1, m, heads, d, generator=g)).to(BF16) for _ in range(ws)]

        def attn(q, k, v):  # layout-revealing, elementwise (any misplaced row or head changes the result)
            return (q.float() + 2.0 * k.float() - 0.5 * v.float()).to(q.dtype)

        def body(r, a2a):
            res = ux.exact_forward(qs[r], ks[r], vs[r], attn, ws=ws, a2a=a2a)
            send = torch.empty(ux.send_shape(m, heads, d, ws), dtype=BF16)
            ux.pack_into(send, qs[r][0], ws)
            stock_q = tue.stock_all_to_all_4d(qs[r], 2, 1, ws, a2a)
            return res, send, stock_q

        fake = tue.FakeA2A(ws)
        import threading
        results = [None] * ws

        def run(r):
            results[r] = body(r, fake.bind(r))
        ts = [threading.Thread(target=run, args=(r,)) for r in range(ws)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        for r in range(ws):
            res, send, stock_q = results[r]
            out[f"ws{ws}_q{r}"] = bits16(qs[r])
            out[f"ws{ws}_k{r}"] = bits16(ks[r])
            out[f"ws{ws}_v{r}"] = bits16(vs[r])
            out[f"ws{ws}_out{r}"] = bits16(res)
            out[f"ws{ws}_send{r}"] = bits16(send)
            out[f"ws{ws}_stockq{r}"] = bits16(stock_q)
        out[f"ws{ws}_shape"] = np.array([m, heads, d])
    return out


def gen_rope(ux, tue) -> dict:
    """The upstream norm+RoPE producer's eager stand-in (tests/test_ulysses_exact.py:107-116) written per destination
    by ulysses_exact.rope_into_send (h3_tp2/ulysses_exact.py:264), on the reference's own input recipe
    (tests/test_ulysses_exact.py:123-130: q/k from a random qkv, weights 1 + 0.1 N(0,1), table N(0,1) [M, 96])."""
    out = {}
    for ws, m, heads in ((2, 24, 8), (4, 16, 8)):
        g = torch.Generator().manual_seed(20 + ws)
        qkv = torch.randn(m, 3 * heads * 128, generator=g).to(BF16)
        q, k, v = (t.view(m, heads, 128) for t in qkv.split([heads * 128] * 3, dim=-1))
        w_q = (1 + 0.1 * torch.randn(128, generator=g)).to(BF16)
        w_k = (1 + 0.1 * torch.randn(128, generator=g)).to(BF16)
        table = torch.randn(m, 96, generator=g)
        sq = torch.empty(ux.send_shape(m, heads, 128, ws), dtype=BF16)
        sk = torch.empty_like(sq)
        ux.rope_into_send(sq, sk, q, k, w_q, w_k, table, 1e-6, tue.eager_launch)
        out.update({f"ws{ws}_qkv": bits16(qkv), f"ws{ws}_wq": bits16(w_q), f"ws{ws}_wk": bits16(w_k),
                    f"ws{ws}_table": f32(table), f"ws{ws}_sendq": bits16(sq), f"ws{ws}_sendk": bits16(sk),
                    f"ws{ws}_shape": np.array([m, heads])})
    return out


def gen_nocopy(nc, tue) -> dict:
    import threading
    out = {}
    heads, d = 8, 128
    for ws, m, groups in ((2, 16, 1), (2, 16, 2), (4, 8, 1), (4, 8, 2)):
        g = torch.Generator().manual_seed(100 + 10 * ws + groups)
        qs = [(torch.randn(1, m, heads, d, generator=g)).to(BF16) for _ in range(ws)]
        ks = [(torch.randn(1, m, heads, d, generator=g)).to(BF16) for _ in range(ws)]
        vs = [(torch.randn(1, m, heads, d, generator=g)).to(BF16) for _ in range(ws)]

        def attn(q, k, v):  # layout-revealing and elementwise; returns a dense [1, S, hl, d] like cuDNN
            return (q.float() + 2.0 * k.float() - 0.5 * v.float()).to(q.dtype).contiguous()

        def body(r, a2a):
            res = nc.nocopy_forward(qs[r], ks[r], vs[r], attn, ws=ws, groups=groups, a2a=a2a)
            send = torch.empty(nc.send_shape(m, heads, d, ws, groups), dtype=BF16)
            nc.pack_qkv(send, qs[r][0], ks[r][0], vs[r][0], ws, groups)
            return res, send

        fake = tue.FakeA2A(ws)
        results = [None] * ws

        def run(r):
            results[r] = body(r, fake.bind(r))
        ts = [threading.Thread(target=run, args=(r,)) for r in range(ws)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        key = f"ws{ws}_g{groups}"
        for r in range(ws):
            res, send = results[r]
            out[f"{key}_q{r}"], out[f"{key}_k{r}"], out[f"{key}_v{r}"] = bits16(qs[r]), bits16(ks[r]), bits16(vs[r])
            out[f"{key}_out{r}"] = bits16(res)
            out[f"{key}_send{r}"] = bits16(send)
        out[f"{key}_shape"] = np.array([m, heads, d])
    return out


def gen_gate(fc) -> dict:
    g = torch.Generator().manual_seed(7)
    M, N, K = 200, 272, 256        # partial row / column tiles
    a = torch.randint(-4, 5, (M, K), generator=g).to(E4M3)
    w = torch.randint(-2, 3, (N, K), generator=g).to(E4M3)
    sa = torch.exp(torch.empty(M).uniform_(-9.0, -2.0, generator=g))
    sb = torch.exp(torch.empty(N).uniform_(-9.5, -7.5, generator=g))
    bias = (torch.randn(N, generator=g) * 0.1).to(BF16)
    x32 = a.float() @ w.float().t()                 # exact (integer products, |sum| < 2^24)
    x = torch.randn(M, N, generator=g).to(BF16)
    gate6 = torch.randn(3, 6 * N, generator=g).to(BF16)
    gate = gate6.chunk(6, dim=-1)[5]                # [3, N] view with row stride 6N
    idx = torch.randint(0, 3, (M,), generator=g)
    y = torch.empty(M, N, dtype=BF16)
    fc._gate_torch(x, gate, x32, sa, sb, None, idx, y)
    yb = torch.empty(M, N, dtype=BF16)
    fc._gate_torch(x, gate, x32, sa, sb, bias, idx, yb)
    return dict(a=bits8(a), w=bits8(w), sa=f32(sa), sb=f32(sb), bias=bits16(bias), x=bits16(x), gate6=bits16(gate6),
                idx=idx.numpy().copy(), y=bits16(y), ybias=bits16(yb))


def gen_consumers(fc) -> dict:
    """The consumer-fused qkv norm + RoPE and out-projection gated RMS of h3_tp2/fp8_consumers.py:316 _qk_rope_torch
    and :354 _gate_rms_torch (the eager mirrors of its Triton consumer kernels) on exact integer fp32 products, the
    rope table fp32 and bf16 (recipe of tests/test_fp8_consumer_fuse.py:78-116: rotary 96, head_dim 128)."""
    g = torch.Generator().manual_seed(8)
    T, H, D, K = 160, 2, 128, 256
    N = 3 * H * D
    a = torch.randint(-4, 5, (T, K), generator=g).to(E4M3)
    w = torch.randint(-2, 3, (N, K), generator=g).to(E4M3)
    sa = torch.exp(torch.empty(T).uniform_(-6.0, -3.0, generator=g))
    sb = torch.exp(torch.empty(N).uniform_(-6.5, -4.5, generator=g))
    x32 = a.float() @ w.float().t()                 # exact (integer products, |sum| < 2^24)
    qw, kw = ((1 + 0.1 * torch.randn(D, generator=g)).to(BF16) for _ in range(2))
    pos = torch.arange(T, dtype=torch.float32)[:, None] * torch.exp(-torch.arange(48, dtype=torch.float32) / 8.0)
    table = torch.cat((torch.cos(pos), torch.sin(pos)), dim=-1)
    out = dict(qk_a=bits8(a), qk_w=bits8(w), qk_sa=f32(sa), qk_sb=f32(sb), qk_qw=bits16(qw), qk_kw=bits16(kw),
               qk_table=f32(table), qk_shape=np.array([T, H, D]))
    for tag, tab in (("f32", table), ("bf16", table.to(BF16))):
        for name, col0, wt in (("q", 0, qw), ("k", H * D, kw)):
            y = torch.empty(T, H, D, dtype=BF16)
            fc._qk_rope_torch(x32, col0, sa, sb, None, wt, tab, 1e-6, H, D, (x32.stride(0), D, 1), y)
            out[f"qk_{name}_{tag}"] = bits16(y)
    Tg, C, Kg = 96, 512, 256
    a = torch.randint(-4, 5, (Tg, Kg), generator=g).to(E4M3)
    w = torch.randint(-2, 3, (C, Kg), generator=g).to(E4M3)
    sa = torch.exp(torch.empty(Tg).uniform_(-6.0, -3.0, generator=g))
    sb = torch.exp(torch.empty(C).uniform_(-6.5, -4.5, generator=g))
    x32 = a.float() @ w.float().t()
    res = torch.randn(Tg, C, generator=g).to(BF16)
    gate, shift, scale = ((0.2 * torch.randn(4, C, generator=g)).to(BF16) for _ in range(3))
    nw = (1 + 0.1 * torch.randn(C, generator=g)).to(BF16)
    idx = torch.randint(0, 4, (Tg,), generator=g)
    r_out, m_out = torch.empty(Tg, C, dtype=BF16), torch.empty(Tg, C, dtype=BF16)
    fc._gate_rms_torch(res, gate, x32, sa, sb, None, nw, shift, scale, idx, 1e-6, r_out, m_out)
    out.update(gr_a=bits8(a), gr_w=bits8(w), gr_sa=f32(sa), gr_sb=f32(sb), gr_res=bits16(res), gr_gate=bits16(gate),
               gr_shift=bits16(shift), gr_scale=bits16(scale), gr_nw=bits16(nw), gr_idx=idx.numpy().copy(),
               gr_res_out=bits16(r_out), gr_mod_out=bits16(m_out))
    return out


SOURCE_SAMPLES = [
    "",
    "def f(x):\n    return x\n",
    "@decorator\ndef f(x):  # trailing comment stays\n\n    # a comment line\n    y = x * 2\t \n    return y\n",
    '    @functools.wraps(g)\n    def wrapper(*a, **kw):\n        """doc # not a comment"""\n        return g(*a, **kw)\n',
    "x = 'été'\n   \n#\n@\nz = 1",
]


def gen_sources(step_cache, fc, fq, outq) -> dict:
    """The upstream-source fingerprint (h3_tp2/step_cache.py:72 fingerprint_source) of a few source texts, and the
    reviewed tables of h3_tp2/fp8_consumers.py:67-89, h3_tp2/fp8_quant_fuse.py:856-877, h3_tp2/ulysses_outq.py:59."""
    return {"samples": SOURCE_SAMPLES, "fingerprints": [step_cache.fingerprint_source(t) for t in SOURCE_SAMPLES],
            "consumer_expected": fc.EXPECTED, "consumer_sites": {k: list(v) for k, v in fc.SITE_SOURCES.items()},
            "quant_expected_extra": fq.EXPECTED_EXTRA, "quant_sites": {k: list(v) for k, v in fq.SITE_SOURCES.items()},
            "outq_expected": outq.EXPECTED}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("H3_TP2_REFERENCE"),
                    help="checkout of the reference project (the directory holding h3_tp2/ and tests/)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or H3_TP2_REFERENCE) is required")
    ref = Path(args.reference)
    sys.path.insert(0, str(ref))
    sys.path.insert(0, str(ref / "tests"))
    from h3_tp2 import fp8_consumers, fp8_gemm, fp8_quant_fuse, fp8_swiglu, ulysses_exact, ulysses_nocopy, ulysses_outq  # noqa: PLC0415,E501
    from h3_tp2 import step_cache  # noqa: PLC0415
    import fake_h3_consumers  # noqa: PLC0415
    import test_ulysses_exact  # noqa: PLC0415

    torch.manual_seed(0)
    np.savez_compressed(HERE / "quant.npz", **gen_quant(fp8_quant_fuse, ulysses_outq))
    np.savez_compressed(HERE / "gemm.npz", **gen_gemm(fp8_gemm))
    np.savez_compressed(HERE / "swiglu.npz", **gen_swiglu(fp8_swiglu, fp8_quant_fuse))
    np.savez_compressed(HERE / "rms.npz", **gen_rms(fp8_quant_fuse, fake_h3_consumers))
    np.savez_compressed(HERE / "ulysses.npz", **gen_ulysses(ulysses_exact, test_ulysses_exact))
    np.savez_compressed(HERE / "rope.npz", **gen_rope(ulysses_exact, test_ulysses_exact))
    np.savez_compressed(HERE / "gate.npz", **gen_gate(fp8_consumers))
    np.savez_compressed(HERE / "consumers.npz", **gen_consumers(fp8_consumers))
    np.savez_compressed(HERE / "nocopy.npz", **gen_nocopy(ulysses_nocopy, test_ulysses_exact))
    (HERE / "sources.json").write_text(json.dumps(gen_sources(step_cache, fp8_consumers, fp8_quant_fuse, ulysses_outq),
                                                  indent=1, sort_keys=True) + "\n")
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
