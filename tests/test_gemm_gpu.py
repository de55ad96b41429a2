"""The tcgen05 FP8 GEMM against the reference's golden vectors (integer inputs: exact in any summation order) and the
reference's two-pass arithmetic (torch._scaled_mm fp32 product + the eager scale pass) on DiT shapes."""
import pytest
import torch

from _util import BF16, E4M3, F16, rel_l2, same_bits, t8, t16, tf, ulp_diff_bf16
from h3b import fp8_consumers, fp8_gemm, ops
from oracle import gemm as og
from oracle import ulysses as ou

pytestmark = pytest.mark.gpu

# BASELINE shapes (N, K): qkv, out, fc1 (gate|up), fc2
SHAPES = {"qkv": (15360, 5120), "out": (5120, 5120), "fc1": (27648, 5120), "fc2": (5120, 13824)}


def _quant_rows(rows, cols, std, g, dev):
    x = (torch.randn(rows, cols, generator=g, device=dev) * std).to(BF16).float()
    s = torch.clamp(x.abs().amax(dim=1) / 448.0, min=1.0 / (448.0 * 512.0))
    return torch.clamp(x / s[:, None], -448.0, 448.0).to(E4M3), s


def _serving_like(M, N, K, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    a, sa = _quant_rows(M, K, torch.exp(torch.randn(M, 1, device=dev, generator=g) * 1.5), g, dev)
    w, sb = _quant_rows(N, K, 0.02, g, dev)
    return a, w, sa, sb


def _two_pass(a, w, sa, sb, out_dtype=BF16):
    one = torch.ones((), device=a.device)
    acc = torch._scaled_mm(a, w.t(), scale_a=one, scale_b=one, out_dtype=torch.float32)
    return ((sb.view(1, -1) * acc) * sa.view(-1, 1)).to(out_dtype)


def test_integer_inputs_golden_exact_with_guards(dev, golden):
    g = golden("gemm")
    a, w = t8(g["int_a"]).to(dev), t8(g["int_w"]).to(dev)
    sa, sb = tf(g["int_sa"]).to(dev), tf(g["int_sb"]).to(dev)
    M, N = a.shape[0], w.shape[0]
    guard = 4096
    buf = torch.full((M * N + 2 * guard,), float("nan"), device=dev, dtype=BF16)
    buf[:guard] = 7.0
    buf[-guard:] = 7.0
    y = buf[guard:guard + M * N].view(M, N)
    ops.fp8_gemm(a, w, sa, sb, out=y)
    assert same_bits(y.cpu(), t16(g["int_y"]))
    assert bool((buf[:guard] == 7.0).all()) and bool((buf[-guard:] == 7.0).all())
    yb = ops.fp8_gemm(a, w, sa, sb, t16(g["int_bias"]).to(dev))
    assert (yb.cpu().view(torch.int16) != t16(g["int_ybias"]).view(torch.int16)).sum().item() <= 2
    y16 = ops.fp8_gemm(a, w, sa, sb, out_dtype=F16)
    assert same_bits(y16.cpu(), t16(g["int_yf16"], F16))
    assert ops.device_status() == 0


def test_random_golden_close(dev, golden):
    g = golden("gemm")
    y = ops.fp8_gemm(t8(g["rnd_a"]).to(dev), t8(g["rnd_w"]).to(dev), tf(g["rnd_sa"]).to(dev), tf(g["rnd_sb"]).to(dev))
    assert int(ulp_diff_bf16(y.cpu(), t16(g["rnd_y"])).max()) <= 1


@pytest.mark.parametrize("M", [1, 200, 1000, 4100])
@pytest.mark.parametrize("shape", list(SHAPES))
def test_dit_shapes_against_two_pass(dev, shape, M):
    N, K = SHAPES[shape]
    a, w, sa, sb = _serving_like(M, N, K, seed=M * 7 + N, dev=dev)
    y = fp8_gemm.scaled_mm(a, w.t(), sa.view(M, 1), sb, BF16)
    ref = _two_pass(a, w, sa, sb)
    assert rel_l2(y.float(), ref.float()) <= 1e-3          # the contract is 1e-2; the epilogue is the reference's
    ud = ulp_diff_bf16(y.cpu(), ref.cpu())
    assert int(ud.max()) <= 2 and (ud == 0).float().mean().item() > 0.95


@pytest.mark.parametrize("M,N,K", [(1, 128, 64), (200, 400, 512), (333, 272, 1024), (129, 5376, 7168),
                                   (8200, 144, 320)])
def test_integer_partial_tiles_exact(dev, M, N, K):
    g = torch.Generator(device=dev).manual_seed(M + N + K)
    a = torch.randint(-4, 5, (M, K), device=dev, generator=g).to(E4M3)
    w = torch.randint(-2, 3, (N, K), device=dev, generator=g).to(E4M3)
    sa = torch.exp(torch.empty(M, device=dev).uniform_(-9.0, -2.0, generator=g))
    sb = torch.exp(torch.empty(N, device=dev).uniform_(-9.5, -7.5, generator=g))
    y = ops.fp8_gemm(a, w, sa, sb)
    ref = og.scaled_mm(a.cpu(), w.cpu(), sa.cpu(), sb.cpu())
    assert same_bits(y.cpu(), ref)


def test_swiglu_epilogue_integer_inputs(dev):
    M, F, K = 300, 384, 512
    g = torch.Generator(device=dev).manual_seed(3)
    a = torch.randint(-4, 5, (M, K), device=dev, generator=g).to(E4M3)
    w = torch.randint(-2, 3, (2 * F, K), device=dev, generator=g).to(E4M3)
    sa = torch.rand(M, device=dev, generator=g) * 0.05 + 0.01
    sb = torch.rand(2 * F, device=dev, generator=g) * 0.05 + 0.01
    y = ops.fp8_gemm_swiglu(a, w, sa, sb).cpu()
    ref = og.swiglu_epilogue(og.accumulate(a.cpu(), w.cpu()), sa.cpu(), sb.cpu(), None)
    ud = ulp_diff_bf16(y, ref)
    assert int(ud.max()) <= 1 and (ud == 0).float().mean().item() > 0.99


@pytest.mark.parametrize("ws", [1, 2, 4, 8])
def test_qkv_send_epilogue_layout(dev, ws):
    M, heads, K = 150, 8, 256
    N = 3 * heads * 128
    g = torch.Generator(device=dev).manual_seed(ws)
    a = torch.randint(-4, 5, (M, K), device=dev, generator=g).to(E4M3)
    w = torch.randint(-2, 3, (N, K), device=dev, generator=g).to(E4M3)
    sa = torch.rand(M, device=dev, generator=g) * 0.05
    sb = torch.rand(N, device=dev, generator=g) * 0.05
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    sq, sk, sv = ops.fp8_gemm_qkv_send(a, w, sa, sb, heads, ws, v_f16=True, range_flag=flag)
    y = ops.fp8_gemm(a, w, sa, sb).cpu()
    q, k, v = (t.reshape(M, heads, 128) for t in y.split(heads * 128, dim=1))
    assert same_bits(sq.cpu(), ou.pack(q, ws)) and same_bits(sk.cpu(), ou.pack(k, ws))
    # v: the bf16 value converted to f16 (round to nearest even; tiny values become f16 subnormals)
    assert sv.dtype == F16 and same_bits(sv.cpu(), ou.pack(v, ws).to(F16))
    assert int(flag.item()) == 0


def test_side_stream(dev):
    a, w, sa, sb = _serving_like(1000, 5120, 5120, seed=5, dev=dev)
    ref = ops.fp8_gemm(a, w, sa, sb)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        y = ops.fp8_gemm(a, w, sa, sb)
    torch.cuda.current_stream().wait_stream(s)
    assert same_bits(y.cpu(), ref.cpu())


def test_deterministic_repeat(dev):
    a, w, sa, sb = _serving_like(4100, 15360, 5120, seed=9, dev=dev)
    y0 = ops.fp8_gemm(a, w, sa, sb)
    for _ in range(3):
        assert torch.equal(ops.fp8_gemm(a, w, sa, sb).view(torch.int16), y0.view(torch.int16))


@pytest.mark.parametrize("ws", [1, 2])
def test_qkv_send_epilogue_with_qk_norm_rope(dev, ws):
    """The norm+RoPE producer fused into the qkv epilogue equals the oracle producer applied to the GEMM's own bf16
    output (a bf16 ulp at most: rsqrt and the sum order)."""
    from oracle import ulysses as oul
    M, heads, K = 200, 4, 256
    N = 3 * heads * 128
    g = torch.Generator(device=dev).manual_seed(7)
    a = torch.randint(-4, 5, (M, K), device=dev, generator=g).to(E4M3)
    w = torch.randint(-2, 3, (N, K), device=dev, generator=g).to(E4M3)
    sa = torch.rand(M, device=dev, generator=g) * 0.05
    sb = torch.rand(N, device=dev, generator=g) * 0.05
    qw = (1 + 0.1 * torch.randn(128, device=dev, generator=g)).to(BF16)
    kw = (1 + 0.1 * torch.randn(128, device=dev, generator=g)).to(BF16)
    table = torch.randn(M, 96, device=dev, generator=g)
    sq, sk, sv = ops.fp8_gemm_qkv_send(a, w, sa, sb, heads, ws, qk_norm=(qw, kw, table, 1e-6))
    y = ops.fp8_gemm(a, w, sa, sb).cpu()
    q, k, v = (t.reshape(M, heads, 128) for t in y.split(heads * 128, dim=1))
    for got, x, wt in ((sq, q, qw), (sk, k, kw)):
        ref = oul.norm_rope_into_send(x, wt.cpu(), table.cpu(), 1e-6, ws)
        ud = ulp_diff_bf16(got.cpu(), ref)
        assert (ud == 0).float().mean().item() > 0.98 and int(ud.max()) <= 8
        assert rel_l2(got.float().cpu(), ref.float()) <= 2e-3
    assert same_bits(sv.cpu(), ou.pack(v, ws))


def test_gate_epilogue_golden_exact(dev, golden):
    """fc2 + indexed gated residual in one kernel: bit-exact against the reference's eager mirror on exact integer
    products, gate rows given as a row-strided view."""
    g = golden("gate")
    a, w = t8(g["a"]).to(dev), t8(g["w"]).to(dev)
    sa, sb, bias = tf(g["sa"]).to(dev), tf(g["sb"]).to(dev), t16(g["bias"]).to(dev)
    x, gate6 = t16(g["x"]).to(dev), t16(g["gate6"]).to(dev)
    idx = torch.from_numpy(g["idx"]).to(dev)
    gate = gate6.chunk(6, dim=-1)[5]
    assert same_bits(ops.fp8_gemm_gate(a, w, sa, sb, x, gate, idx).cpu(), t16(g["y"]))
    assert same_bits(ops.fp8_gemm_gate(a, w, sa, sb, x, gate, idx, bias).cpu(), t16(g["ybias"]))
    assert ops.device_status() == 0


@pytest.mark.parametrize("M", [1, 333, 2000])
def test_gate_epilogue_fc2_shape(dev, M):
    """The fc2 shape (N = 5120, K = 13824) against the two-pass product + the oracle's indexed gate."""
    N, K = SHAPES["fc2"]
    a, w, sa, sb = _serving_like(M, N, K, seed=M + 11, dev=dev)
    g = torch.Generator(device=dev).manual_seed(M)
    x = torch.randn(M, N, device=dev, generator=g).to(BF16)
    gate = torch.randn(4, N, device=dev, generator=g).to(BF16)
    idx = torch.randint(0, 4, (M,), device=dev, generator=g)
    y = ops.fp8_gemm_gate(a, w, sa, sb, x, gate, idx)
    ref = og.indexed_gate(x.cpu(), gate.cpu(), _two_pass(a, w, sa, sb).cpu(), idx.cpu())
    ud = ulp_diff_bf16(y.cpu(), ref)
    assert int(ud.max()) <= 2 and (ud == 0).float().mean().item() > 0.95
    assert ops.device_status() == 0


def test_gate_index_out_of_range_is_reported(dev):
    """A token whose gate row does not exist leaves its output row alone and records H3B_EINVAL."""
    from h3b import _lib
    M, N, K = 130, 256, 128
    a = torch.randint(-2, 3, (M, K), device=dev).to(E4M3)
    w = torch.randint(-2, 3, (N, K), device=dev).to(E4M3)
    sa, sb = torch.full((M,), 1e-3, device=dev), torch.full((N,), 1e-3, device=dev)
    x = torch.zeros(M, N, device=dev, dtype=BF16)
    gate = torch.ones(2, N, device=dev, dtype=BF16)
    idx = torch.zeros(M, device=dev, dtype=torch.int64)
    idx[7] = 2
    y = torch.full((M, N), 5.0, device=dev, dtype=BF16)
    ops.fp8_gemm_gate(a, w, sa, sb, x, gate, idx, out=y)
    torch.cuda.synchronize()
    assert ops.device_status() == _lib.H3B_EINVAL
    assert bool((y[7] == 5.0).all())


def test_consumers_mirror(dev):
    """h3b.fp8_consumers (the reference's stash consumers): the qk norm + RoPE consumer is the qkv GEMM with the norm
    epilogue (v = the plain scale pass), the fc2 gate consumer the gated GEMM, written into the placeholder."""
    M, H, K = 300, 4, 512
    a, w, sa, sb = _serving_like(M, 3 * H * 128, K, seed=5, dev=dev)
    g = torch.Generator(device=dev).manual_seed(6)
    qw = (1.0 + 0.1 * torch.randn(128, device=dev, generator=g)).to(BF16)
    kw = (1.0 + 0.1 * torch.randn(128, device=dev, generator=g)).to(BF16)
    pos = torch.arange(M, device=dev, dtype=torch.float32)[:, None] * torch.exp(-torch.arange(48, device=dev) / 8.0)
    table = torch.cat((torch.cos(pos), torch.sin(pos)), dim=-1).to(BF16)
    st = fp8_consumers.Stash(a, w, sa, sb, None)
    q, k, v = fp8_consumers.qk_norm_rope_fused(st, H, H, 128, qw, kw, table, 1e-6)
    sends = ops.fp8_gemm_qkv_send(a, w, sa, sb, H, 1, qk_norm=(qw, kw, table.float(), 1e-6))
    assert same_bits(q.cpu(), sends[0].view(M, H, 128).cpu()) and same_bits(k.cpu(), sends[1].view(M, H, 128).cpu())
    y = st.materialize()
    assert same_bits(v.cpu(), y[:, 2 * H * 128:].reshape(M, H, 128).cpu())
    N2, K2 = 512, 1024
    a2, w2, sa2, sb2 = _serving_like(M, N2, K2, seed=7, dev=dev)
    x = torch.randn(M, N2, device=dev, generator=g).to(BF16)
    gate = torch.randn(3, N2, device=dev, generator=g).to(BF16)
    idx = torch.randint(0, 3, (M,), device=dev, generator=g)
    ph = torch.empty(M, N2, device=dev, dtype=BF16)
    out = fp8_consumers.gate_fused(fp8_consumers.Stash(a2, w2, sa2, sb2, None, ph), x, gate, idx)
    assert out.data_ptr() == ph.data_ptr()
    assert same_bits(out.cpu(), ops.fp8_gemm_gate(a2, w2, sa2, sb2, x, gate, idx).cpu())
    assert ops.device_status() == 0


def test_wrappers_refuse_what_the_kernels_would_misread(dev):
    """An f16 bias (the kernels read bf16) and an fp32 output are refused before any launch."""
    a = torch.zeros(4, 64, dtype=E4M3, device=dev)
    w = torch.zeros(32, 64, dtype=E4M3, device=dev)
    sa, sb = torch.ones(4, device=dev), torch.ones(32, device=dev)
    with pytest.raises(TypeError, match="bias"):
        ops.fp8_gemm(a, w, sa, sb, torch.zeros(32, dtype=torch.float16, device=dev))
    with pytest.raises(TypeError, match="out_dtype"):
        ops.fp8_gemm(a, w, sa, sb, None, torch.float32)
    with pytest.raises(TypeError, match="out"):
        ops.fp8_gemm(a, w, sa, sb, None, out=torch.empty(4, 32, device=dev))
    with pytest.raises(ValueError, match="unit column stride"):
        ops.fp8_gemm(a, w, sa, sb, None, out=torch.empty(32, 4, dtype=torch.bfloat16, device=dev).t())
    assert ops.device_status() == 0


def test_gate_rms_consumer(dev):
    """fp8_consumers.gate_rms_fused: (residual + gate[idx] * out-projection, its modulated RMSNorm) as bf16, the
    residual written into the placeholder; within 1 bf16 ulp of the eager oracle (fma against separate roundings)."""
    from oracle import rms as orms
    M, N, K = 300, 512, 256
    a, w, sa, sb = _serving_like(M, N, K, seed=11, dev=dev)
    g = torch.Generator(device=dev).manual_seed(12)
    residual = torch.randn(M, N, device=dev, generator=g).to(BF16)
    gate = (0.1 * torch.randn(4, N, device=dev, generator=g)).to(BF16)
    weight = (1.0 + 0.1 * torch.randn(N, device=dev, generator=g)).to(BF16)
    shift = (0.1 * torch.randn(4, N, device=dev, generator=g)).to(BF16)
    scale = (0.1 * torch.randn(4, N, device=dev, generator=g)).to(BF16)
    idx = torch.randint(0, 4, (M,), device=dev, generator=g)
    ph = torch.empty(M, N, device=dev, dtype=BF16)
    st = fp8_consumers.Stash(a, w, sa, sb, None, ph)
    r_out, mod = fp8_consumers.gate_rms_fused(st, residual, gate, weight, shift, scale, idx, 1e-6)
    assert r_out.data_ptr() == ph.data_ptr() and mod.shape == (M, N) and mod.dtype == BF16
    branch = ops.fp8_gemm(a, w, sa, sb).cpu()
    ref_r, _ = orms.gate_rms_norm_scale_shift(residual.cpu(), gate.cpu(), branch, weight.cpu(), shift.cpu(),
                                              scale.cpu(), idx.cpu(), 1e-6)
    ud = ulp_diff_bf16(r_out.cpu(), ref_r)
    assert int(ud.max()) <= 1 and (ud == 0).float().mean().item() > 0.99
    # the modulated rows against the oracle's modulated RMSNorm of the residual the kernel wrote: a residual element one
    # ulp off (fma against separate roundings) moves its modulated value by up to ~2^-8 of n(1 + scale), which near a
    # cancellation with the shift is many ulps of a small result; compared on that stage alone it stays within 1 ulp
    _check_modulated(mod.cpu(), orms.rms_norm_scale_shift(r_out.cpu(), weight.cpu(), shift.cpu(), scale.cpu(), idx.cpu(),
                                                          1e-6))
    assert ops.device_status() == 0


def _check_modulated(got, ref):
    """Modulated RMSNorm rows: within 1 bf16 ulp except where the shift cancels most of n(1 + scale) (there an fp32 ulp
    of the normalised value is many bf16 ulps of the small result): 99.9 % of the elements within 1 ulp, every error
    below 2^-7 of the row's largest value, rel-L2 <= 1e-3."""
    ud = ulp_diff_bf16(got, ref)
    assert (ud <= 1).float().mean().item() > 0.999 and (ud == 0).float().mean().item() > 0.99
    err = (got.float() - ref.float()).abs()
    assert bool((err <= ref.float().abs().amax(dim=1, keepdim=True) * 2.0 ** -7).all())
    assert rel_l2(got.float(), ref.float()) <= 1e-3


def test_consumers_against_the_reference_mirrors(dev, golden):
    """The qkv GEMM with the norm + RoPE epilogue and the out-projection gated-RMS consumer against the reference's
    eager mirrors of its consumer kernels (h3_tp2/fp8_consumers.py:316, :354; tests/golden/consumers.npz) on exact
    integer products: the GEMM output is the mirror's bf16 epilogue exactly, the norm differs by rsqrt and summation
    order (the bounds of the oracle comparisons above)."""
    g = golden("consumers")
    T, H, D = (int(v) for v in g["qk_shape"])
    st = fp8_consumers.Stash(t8(g["qk_a"]).to(dev), t8(g["qk_w"]).to(dev), tf(g["qk_sa"]).to(dev),
                             tf(g["qk_sb"]).to(dev), None)
    qw, kw = t16(g["qk_qw"]).to(dev), t16(g["qk_kw"]).to(dev)
    table = tf(g["qk_table"])
    for tag, tab in (("f32", table), ("bf16", table.to(BF16))):
        q, k, _ = fp8_consumers.qk_norm_rope_fused(st, H, H, D, qw, kw, tab.to(dev), 1e-6)
        for name, got in (("q", q), ("k", k)):
            ref = t16(g[f"qk_{name}_{tag}"])
            ud = ulp_diff_bf16(got.cpu(), ref)
            # a normalised value one bf16 ulp off (rsqrt, summation order) is many ulps of a rotated output where
            # a cos and b sin cancel: bounded against the head's largest value there
            assert (ud == 0).float().mean().item() > 0.98 and (ud <= 8).float().mean().item() > 0.999, (name, tag)
            err = (got.cpu().float() - ref.float()).abs()
            assert bool((err <= ref.float().abs().amax(dim=-1, keepdim=True) * 2.0 ** -7).all()), (name, tag)
            assert rel_l2(got.float().cpu(), ref.float()) <= 2e-3
    st = fp8_consumers.Stash(t8(g["gr_a"]).to(dev), t8(g["gr_w"]).to(dev), tf(g["gr_sa"]).to(dev),
                             tf(g["gr_sb"]).to(dev), None)
    args = [t16(g[k]).to(dev) for k in ("gr_res", "gr_gate", "gr_nw", "gr_shift", "gr_scale")]
    r_out, mod = fp8_consumers.gate_rms_fused(st, *args, torch.from_numpy(g["gr_idx"]).to(dev), 1e-6)
    ud = ulp_diff_bf16(r_out.cpu(), t16(g["gr_res_out"]))
    assert int(ud.max()) <= 1 and (ud == 0).float().mean().item() > 0.99
    _check_modulated(mod.cpu(), t16(g["gr_mod_out"]))
    assert ops.device_status() == 0


def test_tma_store_epilogue_equals_plain_stores(dev, tmp_path):
    """The staged output blocks leave through TMA stores by default; H3B_GEMM_TMA_STORE=0 keeps them on plain stores.
    Both write the same bytes: plain and f16 outputs, the SwiGLU output, and the q/k/v send layouts (head groups,
    interleaved, q/k RMSNorm + RoPE) on shapes with partial row and column tiles, each computed in a fresh process
    per setting.  (With TMA stores the SwiGLU epilogue runs its 8-warp form, without them the 4-warp one, so this also
    compares the two.)"""
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    code = (
        "import sys, torch\n"
        f"sys.path[:0] = [{str(root / 'minimax-h3-2x-dgx-spark-tp2_b200')!r}, {str(root)!r}]\n"
        "from h3b import ops\n"
        "E4M3 = torch.float8_e4m3fn\n"
        "def inputs(M, N, K, seed):\n"
        "    g = torch.Generator(device='cuda').manual_seed(seed)\n"
        "    a = torch.randint(-4, 5, (M, K), device='cuda', generator=g).to(E4M3)\n"
        "    w = torch.randint(-2, 3, (N, K), device='cuda', generator=g).to(E4M3)\n"
        "    sa = torch.rand(M, device='cuda', generator=g) * 0.05 + 1e-3\n"
        "    sb = torch.rand(N, device='cuda', generator=g) * 0.05 + 1e-3\n"
        "    return a, w, sa, sb\n"
        "out = {}\n"
        "a, w, sa, sb = inputs(333, 400, 256, 1)\n"
        "out['plain'] = ops.fp8_gemm(a, w, sa, sb)\n"
        "out['f16'] = ops.fp8_gemm(a, w, sa, sb, out_dtype=torch.float16)\n"
        "a, w, sa, sb = inputs(300, 768, 512, 2)\n"
        "out['swiglu'] = ops.fp8_gemm_swiglu(a, w, sa, sb)\n"
        "a, w, sa, sb = inputs(150, 3 * 8 * 128, 256, 3)\n"
        "for i, t in enumerate(ops.fp8_gemm_qkv_send(a, w, sa, sb, 8, 2, groups=2, v_f16=True)):\n"
        "    out[f'grouped{i}'] = t\n"
        "out['inter'] = ops.fp8_gemm_qkv_send(a, w, sa, sb, 8, 2, interleaved=True)\n"
        "g = torch.Generator(device='cuda').manual_seed(4)\n"
        "qw, kw = (torch.rand(128, device='cuda', generator=g) + 0.5).to(torch.bfloat16), (torch.rand(128, device='cuda', generator=g) + 0.5).to(torch.bfloat16)\n"
        "tab = torch.rand(150, 96, device='cuda', generator=g) * 2 - 1\n"
        "for i, t in enumerate(ops.fp8_gemm_qkv_send(a, w, sa, sb, 8, 2, qk_norm=(qw, kw, tab, 1e-6))):\n"
        "    out[f'norm{i}'] = t\n"
        "torch.cuda.synchronize()\n"
        "assert ops.device_status() == 0\n"
        "torch.save({k: v.cpu() for k, v in out.items()}, sys.argv[1])\n")
    res = {}
    for setting in ("0", "1"):
        path = tmp_path / f"out{setting}.pt"
        env = dict(os.environ, H3B_GEMM_TMA_STORE=setting)
        run = subprocess.run([sys.executable, "-c", code, str(path)], env=env, capture_output=True, text=True,
                             timeout=300)
        assert run.returncode == 0, run.stderr[-3000:]
        res[setting] = torch.load(path)
    assert res["0"].keys() == res["1"].keys()
    for key in res["0"]:
        assert same_bits(res["0"][key], res["1"][key]), key


def test_strided_output_rows_keep_their_gaps(dev):
    """An output view with a row stride above N (the caller's wider buffer): every row gets its N values and the
    columns between rows stay untouched (the TMA stores clip at N; partial row and column tiles included)."""
    M, N, K = 333, 400, 256
    g = torch.Generator(device=dev).manual_seed(11)
    a = torch.randint(-4, 5, (M, K), device=dev, generator=g).to(E4M3)
    w = torch.randint(-2, 3, (N, K), device=dev, generator=g).to(E4M3)
    sa = torch.rand(M, device=dev, generator=g) * 0.05 + 1e-3
    sb = torch.rand(N, device=dev, generator=g) * 0.05 + 1e-3
    buf = torch.full((M, N + 72), 7.0, dtype=BF16, device=dev)
    y = ops.fp8_gemm(a, w, sa, sb, out=buf[:, :N])
    ref = ops.fp8_gemm(a, w, sa, sb)
    assert same_bits(y.cpu(), ref.cpu())
    assert bool((buf[:, N:] == 7.0).all())
    assert ops.device_status() == 0
