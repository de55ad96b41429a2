"""The consumer-fuse wiring on the CPU (h3_tp2/fp8_consumers.py:498-919): inside a planned DiT block the FP8 GEMM
dispatcher's stash hook keeps the qkv / out / fc2 operands behind placeholders, the wrapped consumers run the fused
consumer on exactly their placeholder, the first call per site is compared bit for bit with GEMM + stock consumer
(a planted mismatch disables the site), and every call the wiring cannot take materialises the stash and runs stock.

The fused consumers and the GEMM are CUDA kernels; here they are replaced for the duration of each test by eager
restatements from ``oracle/`` (the test exercises the protocol, not the kernels, which the GPU tests pin)."""
from types import SimpleNamespace

import pytest
import torch

from h3b import fp8_consumers as fc
from _util import CpuKernels
from h3b import fp8_gemm, ops
from oracle import gemm as og
from oracle import quant as oq
from oracle import rms as orms
from oracle import ulysses as ou

BF16, E4M3 = torch.bfloat16, torch.float8_e4m3fn
T, H, D, C, F = 96, 2, 128, 256, 512


def _gemm(a, w, sa, sb, bias=None, out_dtype=BF16, out=None):
    y = og.scaled_mm(a, w, sa, sb, bias, out.dtype if out is not None else out_dtype)
    return y if out is None else out.copy_(y)


def _stock_qk(q, k, qw, kw, table, eps, *, head_dim=None, rotary_dim=None, interleaved=False):  # noqa: ARG001
    return ou.norm_rope(q, qw, table, eps), ou.norm_rope(k, kw, table, eps)


def _stock_gate_rms(residual, gate, branch, weight, shift, scale, indices, eps):
    return orms.gate_rms_norm_scale_shift(residual, gate, branch, weight, shift, scale, indices, eps)


def _fused_qk(st, heads, kv_heads, head_dim, qw, kw, table, eps):
    q, k, v = _gemm(st.a, st.w, st.sa, st.sb, st.bias).split(heads * head_dim, dim=1)
    q, k, v = (t.reshape(-1, heads, head_dim) for t in (q, k, v))
    return ou.norm_rope(q, qw, table, eps), ou.norm_rope(k, kw, table, eps), v.contiguous()


def _fused_gate_rms(st, residual, gate, weight, shift, scale, indices, eps, reuse_placeholder=True):  # noqa: ARG001
    return orms.gate_rms_norm_scale_shift(residual, gate, _gemm(st.a, st.w, st.sa, st.sb, st.bias), weight, shift,
                                          scale, indices, eps)


def _fused_gate(st, x, gate, indices, reuse_placeholder=True):  # noqa: ARG001
    return og.indexed_gate(x, gate, _gemm(st.a, st.w, st.sa, st.sb, st.bias), indices)


@pytest.fixture(autouse=True)
def _eager(monkeypatch):
    kernels = CpuKernels(fp8_gemm=lambda a, w, sa, sb, bias, dt: _gemm(a, w, sa, sb, bias, dt),
                         fp8_gemm_out=lambda a, w, sa, sb, bias, out: (_gemm(a, w, sa, sb, bias, out=out), None)[1])
    kernels.__enter__()
    monkeypatch.setattr(ops, "fp8_gemm", _gemm)
    monkeypatch.setattr(fc, "qk_norm_rope_fused", _fused_qk)
    monkeypatch.setattr(fc, "gate_rms_fused", _fused_gate_rms)
    monkeypatch.setattr(fc, "gate_fused", _fused_gate)
    monkeypatch.setattr(fc, "_state", {"sites": (), "checked": {}, "disabled": set(), "device_types": ("cpu",)})
    monkeypatch.setattr(fc, "_stats", dict.fromkeys(fc._stats, 0))
    monkeypatch.setattr(fp8_gemm, "_stash_hooks", [])
    monkeypatch.setattr(fp8_gemm, "_routers", [])
    yield
    fc._tls.ctx = None
    kernels.__exit__()


def _layer(n, k, seed):
    w8, sb = og.quant_weight(torch.randn(n, k, generator=torch.Generator().manual_seed(seed)) * 0.05)
    return SimpleNamespace(weight=w8.t(), weight_scale=sb, output_size_per_partition=n, tp_size=1)


def _linear(layer, x):
    a8, sa = oq.quant(x)
    return fp8_gemm.route(a8, layer.weight, sa, layer.weight_scale, BF16, None)


def _module():
    """A stand-in for the MiniMax H3 transformer module: its block calls the module-level consumers by name."""
    tr = SimpleNamespace(fused_qk_norm_rope=_stock_qk, indexed_gate_rms_norm_scale_shift=_stock_gate_rms,
                         indexed_gate=og.indexed_gate)

    class MiniMaxH3DiTBlock:
        def __init__(self):
            self.attn = SimpleNamespace(qkv_proj=_layer(3 * H * D, C, 1), out_proj=_layer(C, H * D, 2))
            self.mlp = SimpleNamespace(fc2=_layer(C, F, 3))
            g = torch.Generator().manual_seed(4)
            self.qw, self.kw, self.nw = ((1 + 0.1 * torch.randn(n, generator=g)).to(BF16) for n in (D, D, C))
            self.gate, self.shift, self.scale, self.gate2 = (
                (0.1 * torch.randn(3, C, generator=g)).to(BF16) for _ in range(4))

        def forward(self, x, idx, rope_table=None, skip_qk=False):
            qkv = _linear(self.attn.qkv_proj, x)
            q, k, v = (t.view(T, H, D) for t in qkv.split(H * D, dim=1))
            if not skip_qk:
                q, k = tr.fused_qk_norm_rope(q, k, self.qw, self.kw, rope_table, 1e-6)
                o = (q.float() * 0.5 + k.float() * 0.25 + v.float()).to(BF16).reshape(T, H * D)
            else:                         # a consumer outside the wiring: its input is not the qkv output
                o = (x[:, :H * D].float() * 0.5).to(BF16)
            branch = _linear(self.attn.out_proj, o)
            res, mod = tr.indexed_gate_rms_norm_scale_shift(x, self.gate, branch, self.nw, self.shift, self.scale,
                                                            idx, 1e-6)
            h = _linear(self.mlp.fc2, torch.cat((mod, mod), dim=1))
            return tr.indexed_gate(res, self.gate2, h, idx)

    tr.MiniMaxH3DiTBlock = MiniMaxH3DiTBlock
    return tr


def _inputs(seed=9):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, C, generator=g).to(BF16)
    idx = torch.randint(0, 3, (T,), generator=g)
    pos = torch.arange(T, dtype=torch.float32)[:, None] * torch.exp(-torch.arange(48, dtype=torch.float32) / 8)
    return x, idx, torch.cat((torch.cos(pos), torch.sin(pos)), dim=-1)


def _install(tr, sites=fc.SITES, **kw):
    kw.setdefault("level", "tensor32")
    kw.setdefault("nocopy", False)
    kw.setdefault("check_source", False)          # the stand-in module is not the reviewed upstream source
    kw.setdefault("lora_types", ())
    return fc.install(sites, tr, **kw)


def test_installed_block_equals_stock():
    tr = _module()
    block = tr.MiniMaxH3DiTBlock()
    x, idx, table = _inputs()
    ref = block.forward(x, idx, rope_table=table)
    assert _install(tr) == list(fc.SITES)
    got = tr.MiniMaxH3DiTBlock.forward(block, x, idx, rope_table=table)
    assert torch.equal(got, ref)
    st = fc.stats()
    assert (st["stash"], st["fused_qkv"], st["fused_out"], st["fused_fc2"]) == (3, 1, 1, 1)
    assert st["selfcheck_pass"] == 3 and st["materialize"] == 0
    assert torch.equal(tr.MiniMaxH3DiTBlock.forward(block, x, idx, rope_table=table), ref)   # self-checks cached
    assert fc.stats()["selfcheck_pass"] == 3 and fc.stats()["fused_fc2"] == 2


def test_planted_mismatch_disables_the_site(monkeypatch):
    """A fused fc2 consumer one bf16 ulp off on its first row fails the self-check: the site turns off for the process
    and the stash is materialised for the stock consumer, so the block's output is still stock's."""
    def off_by_one(st, x, gate, indices, reuse_placeholder=True):
        y = _fused_gate(st, x, gate, indices)
        y.view(torch.int16)[0, 0] += 1
        return y

    monkeypatch.setattr(fc, "gate_fused", off_by_one)
    tr = _module()
    block = tr.MiniMaxH3DiTBlock()
    x, idx, table = _inputs()
    ref = block.forward(x, idx, rope_table=table)
    _install(tr)
    assert torch.equal(tr.MiniMaxH3DiTBlock.forward(block, x, idx, rope_table=table), ref)
    st = fc.stats()
    assert "fc2" in fc._state["disabled"] and st["selfcheck_fail"] == 1 and st["materialize"] == 1
    assert st["fused_fc2"] == 0 and st["fused_qkv"] == 1
    assert torch.equal(tr.MiniMaxH3DiTBlock.forward(block, x, idx, rope_table=table), ref)
    assert fc.stats()["stash"] == 3 + 2                             # the second block plans qkv and out only


def test_unconsumed_stashes_are_materialised():
    """A block whose q/k never reach the wrapped producer: the qkv stash is made real before the out GEMM's, and the
    output is stock's; without a rope table the block is not planned at all."""
    tr = _module()
    block = tr.MiniMaxH3DiTBlock()
    x, idx, table = _inputs()
    ref = block.forward(x, idx, rope_table=table, skip_qk=True)
    _install(tr)
    assert torch.equal(tr.MiniMaxH3DiTBlock.forward(block, x, idx, rope_table=table, skip_qk=True), ref)
    assert fc.stats()["materialize"] == 1 and fc.stats()["fused_qkv"] == 0 and fc.stats()["fused_out"] == 1
    before = fc.stats()["stash"]
    tr.fused_qk_norm_rope = _stock_qk                             # the unplanned block runs the stock consumers
    tr.MiniMaxH3DiTBlock.forward(block, x, idx, rope_table=None, skip_qk=True)
    assert fc.stats()["stash"] == before


def test_mismatch_reasons():
    t, h = 8, 2
    a8, sa = oq.quant(torch.randn(t, C).to(BF16))
    w8, sb = og.quant_weight(torch.randn(3 * h * D, C))
    ph = torch.empty(t, 3 * h * D, dtype=BF16)
    st = fc.Stash(a8, w8, sa.reshape(-1), sb, None, ph)
    q, k = ph[:, :h * D].view(t, h, D), ph[:, h * D:2 * h * D].view(t, h, D)
    w = torch.ones(D, dtype=BF16)
    tab = torch.zeros(t, 96)
    assert fc.qk_mismatch(st, q, k, w, w, tab, None, None, False) is None
    assert fc.qk_mismatch(st, q, k, w, w, tab, None, None, True) == "interleaved"
    assert fc.qk_mismatch(st, q.clone(), k, w, w, tab, None, None, False).startswith("q/k are not")
    assert fc.qk_mismatch(st, q, k, w, w, torch.zeros(t, 48), None, None, False) == "rotary"
    assert fc.qk_mismatch(st, q, k, w, w, tab, None, 64, False) == "rotary"
    assert fc.qk_mismatch(st, q, k, w.float(), w, tab, None, None, False).startswith("rope table or norm weight")
    biased = fc.Stash(a8, w8, sa.reshape(-1), sb, torch.zeros(3 * h * D, dtype=BF16), ph)
    assert fc.qk_mismatch(biased, q, k, w, w, tab, None, None, False).startswith("bias")
    ph_gqa = torch.empty(t, (h + 2) * D, dtype=BF16)
    st_gqa = fc.Stash(a8, w8[:(h + 2) * D], sa.reshape(-1), sb[:(h + 2) * D], None, ph_gqa)
    assert fc.qk_mismatch(st_gqa, ph_gqa[:, :h * D].view(t, h, D), ph_gqa[:, h * D:(h + 1) * D].view(t, 1, D), w, w,
                          tab, None, None, False) == "grouped kv heads"
    fc._state["device_types"] = ("cuda",)
    assert fc.qk_mismatch(st, q, k, w, w, tab, None, None, False) == "device"
    fc._state["device_types"] = ("cpu",)

    w2, sb2 = og.quant_weight(torch.randn(C, C))
    ph2 = torch.empty(t, C, dtype=BF16)
    st2 = fc.Stash(a8, w2, sa.reshape(-1), sb2, None, ph2)
    x, g = torch.zeros(t, C, dtype=BF16), torch.zeros(3, C, dtype=BF16)
    idx = torch.zeros(t, dtype=torch.int64)
    assert fc.rows_mismatch(st2, x, ph2, g, idx) is None
    assert fc.rows_mismatch(st2, x, ph2.clone(), g, idx) == "branch is not the placeholder"
    assert fc.rows_mismatch(st2, x.float(), ph2, g, idx) == "residual shape/dtype/layout"
    assert fc.rows_mismatch(st2, x, ph2, g.float(), idx) == "gate/shift/scale layout"
    assert fc.rows_mismatch(st2, x, ph2, g, idx[:4]) == "indices"


def test_install_rules():
    tr = _module()
    assert _install(tr, level="cutlass") == ["fc2"]               # qkv / out are routed by weight at that level
    assert _install(tr) == ["fc2"]                                # installed once
    assert fp8_gemm._stash_hooks == [fc.stash_hook]
    assert tr.indexed_gate._h3b_consumer_fuse and not hasattr(tr.fused_qk_norm_rope, "_h3b_consumer_fuse")
    tr2 = _module()
    assert _install(tr2, nocopy=True) == ["out", "fc2"]           # the combined exchange owns the rope producer
    assert _install(_module(), sites=()) == []
    assert _install(_module(), ("qkv", "out"), level="cutlass") == []


def test_install_skips_sites_whose_upstream_source_is_not_the_reviewed_one():
    """With the source check (the default) a stand-in transformer is not vLLM-Omni's reviewed code: no site installs
    and nothing is wrapped."""
    tr = _module()
    tr.MiniMaxH3Attention = type("MiniMaxH3Attention", (), {"forward": lambda self, x: x})
    tr.MiniMaxH3MLP = type("MiniMaxH3MLP", (), {"forward": lambda self, x: x})
    stock = (tr.fused_qk_norm_rope, tr.indexed_gate, tr.MiniMaxH3DiTBlock.forward)
    assert _install(tr, check_source=True) == []
    assert stock == (tr.fused_qk_norm_rope, tr.indexed_gate, tr.MiniMaxH3DiTBlock.forward)
    assert fp8_gemm._stash_hooks == []


@pytest.mark.parametrize("sites", [("qkv",), ("out",), ("fc2",), ("out", "fc2")])
def test_site_subsets(sites):
    tr = _module()
    block = tr.MiniMaxH3DiTBlock()
    x, idx, table = _inputs(11)
    ref = block.forward(x, idx, rope_table=table)
    assert _install(tr, sites) == list(sites)
    assert torch.equal(tr.MiniMaxH3DiTBlock.forward(block, x, idx, rope_table=table), ref)
    st = fc.stats()
    assert [st[f"fused_{s}"] for s in fc.SITES] == [int(s in sites) for s in fc.SITES] and st["materialize"] == 0


def test_plan_rejections_and_lora():
    tr = _module()
    block = tr.MiniMaxH3DiTBlock()
    table = torch.zeros(4, 96)
    want, _ = fc.block_plan(block, table, fc.SITES)
    assert sorted(want.values()) == sorted(fc.SITES)
    assert fc.block_plan(block, None, fc.SITES)[0] is None                          # no rope table
    assert fc.block_plan(block, table, fc.SITES, lora_types=(SimpleNamespace,))[0] is None
    block.mlp.fc2.tp_size = 2
    assert "tp_size" in fc.block_plan(block, table, fc.SITES)[1]                    # an all-reduce reads the output
    block.mlp.fc2.tp_size = 1
    block.attn.out_proj.output_size_per_partition += 16                             # a padded N is sliced and copied
    assert fc.block_plan(block, table, fc.SITES)[0] is None
    block.attn.out_proj.output_size_per_partition -= 16
    fc._state["disabled"].add("qkv")
    assert sorted(fc.block_plan(block, table, fc.SITES)[0].values()) == ["fc2", "out"]

    x, idx, table = _inputs(12)
    ref = block.forward(x, idx, rope_table=table)
    _install(tr, lora_types=(SimpleNamespace,))                                     # every layer counts as wrapped
    assert torch.equal(tr.MiniMaxH3DiTBlock.forward(block, x, idx, rope_table=table), ref)
    assert fc.stats()["stash"] == 0


def test_foreign_site_stash_and_calls_outside_a_block():
    """A consumer that meets another site's stash makes it real first; with no block context nothing is stashed."""
    t = 6
    a8, sa = oq.quant(torch.randn(t, C).to(BF16))
    w8, sb = og.quant_weight(torch.randn(C, C))
    ph = torch.empty(t, C, dtype=BF16)
    x, gate = torch.randn(t, C).to(BF16), (0.1 * torch.randn(1, C)).to(BF16)
    idx = torch.zeros(t, dtype=torch.int64)
    with fc.scope(None, {}) as sc:
        sc.handoffs["out"] = fc.Stash(a8, w8, sa.reshape(-1), sb, None, ph)
        out = fc.make_gate_wrapper(og.indexed_gate)(x, gate, ph, idx)              # fc2's consumer, out's stash
        branch = og.scaled_mm(a8, w8, sa.reshape(-1), sb)
        assert torch.equal(out, og.indexed_gate(x, gate, branch, idx)) and torch.equal(ph, branch)
        assert fc.stats()["materialize"] == 1 and not sc.handoffs and fc.stats()["fused_fc2"] == 0
    assert fc._tls.ctx is None
    layer = _layer(C, C, 5)
    _install(_module())
    y = _linear(layer, x)                                                          # a GEMM outside any block
    assert fc.stats()["stash"] == 0 and y.shape == (t, C)


def test_stash_hook_takes_only_the_planned_weights_once():
    mine, other = _layer(64, C, 6), _layer(64, C, 7)
    a8, sa = oq.quant(torch.randn(4, C).to(BF16))
    sc = fc.scope(None, {(mine.weight.data_ptr(), tuple(mine.weight.shape)): "fc2"}).__enter__()
    assert fc.stash_hook(a8, other.weight, sa, other.weight_scale, BF16, None) is None
    assert fc.stash_hook(a8, mine.weight, sa, mine.weight_scale, torch.float16, None) is None   # bf16 outputs only
    ph = fc.stash_hook(a8, mine.weight, sa, mine.weight_scale, BF16, None)
    assert ph.shape == (4, 64) and ph.dtype == BF16 and set(sc.handoffs) == {"fc2"}
    st = sc.handoffs["fc2"]
    assert st.a is a8 and st.w.shape == (64, C) and st.w.data_ptr() == mine.weight.data_ptr() and st.sa.shape == (4,)
    assert fc.stash_hook(a8, mine.weight, sa, mine.weight_scale, BF16, None) is None             # once per block
