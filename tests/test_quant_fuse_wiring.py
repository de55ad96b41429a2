"""The quant-fuse wiring (h3_tp2/fp8_quant_fuse.py:404-1002) on the CPU with a fake DiT block: the planned producers
stash (fp8, scale) behind placeholders that the layers' quants consume, the block's output is the stock one bit for
bit, a stash met by another quant is materialised, and a fused producer that differs from the stock pair disables its
site.  The fused kernels are replaced by eager equivalents (the oracle's) for these host-logic tests."""
from types import SimpleNamespace

import pytest
import torch

from h3b import fp8_quant_fuse as fq
from oracle import gemm as og
from oracle import quant as oq
from oracle import rms as orms

BF16 = torch.bfloat16
C = 64          # hidden width
F = 96          # ffn width


def _make_classes():
    """Fresh stand-ins for vLLM's QuantFP8 and vLLM-Omni's SiluAndMul (install patches their forward)."""
    class Quant:
        static = False
        use_per_token_if_dynamic = True
        is_group_quant = False
        num_token_padding = None

        def forward(self, x, scale=None, scale_ub=None):
            return oq.quant(x)

        def __call__(self, x, scale=None, scale_ub=None):
            return type(self).forward(self, x, scale, scale_ub)

    class Act:
        def forward(self, x):
            return og.silu_and_mul(x)

        def __call__(self, x):
            return type(self).forward(self, x)

    return Quant, Act


class Linear(torch.nn.Module):
    """A per-token FP8 linear: its kernel quantises the input with ``quant_fp8`` and multiplies (fp32, then bf16)."""

    def __init__(self, k, n, quant, seed):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.weight = torch.randn(k, n, generator=g) * 0.05        # vLLM stores [K, N]
        self.quant_method = SimpleNamespace(fp8_linear=SimpleNamespace(quant_fp8=quant))
        self.tp_size = 1

    def forward(self, x):
        k = self.weight.shape[0]
        q, s = self.quant_method.fp8_linear.quant_fp8(x.reshape(-1, k))
        return (q.float() * s @ self.weight).to(BF16), None


def _tr(Quant, Act):
    """A fake transformer module: the block reads its producers from the module at call time."""
    tr = SimpleNamespace(rms_norm_indexed_scale_shift=orms.rms_norm_scale_shift,
                         indexed_gate_rms_norm_scale_shift=orms.gate_rms_norm_scale_shift)

    class Block:
        def __init__(self):
            self.attn = SimpleNamespace(qkv_proj=Linear(C, 3 * C, Quant(), 1), out_proj=None, to_gate_compress=None)
            self.mlp = SimpleNamespace(fc1=Linear(C, 2 * F, Quant(), 2), fc2=Linear(F, C, Quant(), 3), act_fn=Act())
            self.norm1 = SimpleNamespace(weight=(1 + 0.1 * torch.randn(C)).to(BF16))
            self.norm2 = SimpleNamespace(weight=(1 + 0.1 * torch.randn(C)).to(BF16))

        def forward(self, x, shift, scale, gate, idx):
            h = tr.rms_norm_indexed_scale_shift(x, self.norm1.weight, shift, scale, idx, 1e-6)
            qkv, _ = self.attn.qkv_proj(h)
            branch = qkv[:, :C]
            res, mod = tr.indexed_gate_rms_norm_scale_shift(x, gate, branch, self.norm2.weight, shift, scale, idx, 1e-6)
            hidden, _ = self.mlp.fc1(mod)
            out, _ = self.mlp.fc2(self.mlp.act_fn(hidden))
            return res, out

    tr.MiniMaxH3DiTBlock = Block
    return tr


def _eager_site_kernels(monkeypatch):
    def rms_quant(x, weight, shift, scale, indices, eps, stock=None, ph=None):
        h = stock(x, weight, shift, scale, indices, eps)
        if ph is not None:
            ph.copy_(h)
        return oq.quant(h)

    def gate_rms_quant(residual, gate, branch, weight, shift, scale, indices, eps, stock=None, ph=None):
        res, mod = stock(residual, gate, branch, weight, shift, scale, indices, eps)
        if ph is not None:
            ph.copy_(mod)
        return (res, *oq.quant(mod))

    monkeypatch.setattr(fq, "rms_quant", rms_quant)
    monkeypatch.setattr(fq, "gate_rms_quant", gate_rms_quant)
    monkeypatch.setattr(fq, "silu_mul_quant", lambda x, stock=None: oq.quant(og.silu_and_mul(x)))


# the stand-in module is not the reviewed upstream source, fc1's output reaches the activation as at the cutlass level
_AS_REVIEWED = {"check_source": False, "level": "cutlass", "env": {}}


@pytest.fixture
def fuse(monkeypatch):
    """Fresh module state, CPU tensors admitted, eager site kernels."""
    for key, val in (("sites", ()), ("checked", {}), ("disabled", set()), ("orig_quant", None), ("quant_cls", None),
                     ("act_cls", None), ("verify", False), ("modes", (0, 1)), ("device_types", ("cpu",))):
        monkeypatch.setitem(fq._state, key, val)
    for k in fq._stats:
        monkeypatch.setitem(fq._stats, k, 0)
    _eager_site_kernels(monkeypatch)


def _inputs(m, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, C, generator=g).to(BF16)
    shift, scale, gate = ((0.1 * torch.randn(4, C, generator=g)).to(BF16) for _ in range(3))
    idx = torch.randint(0, 4, (m,), generator=g)
    return x, shift, scale, gate, idx


def test_fused_block_equals_stock_bit_for_bit(fuse):
    Quant, Act = _make_classes()
    tr = _tr(Quant, Act)
    torch.manual_seed(0)
    blk = tr.MiniMaxH3DiTBlock()
    args = _inputs(100)
    ref = blk.forward(*args)                                    # the stock block
    installed = fq.install(("qkv", "fc1", "fc2"), tr, quant_cls=Quant, act_cls=Act, lora_types=(), **_AS_REVIEWED)
    assert installed == ["qkv", "fc1", "fc2"]
    got = tr.MiniMaxH3DiTBlock.forward(blk, *args)
    for a, b in zip(got, ref):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    st = fq.stats()
    assert (st["fused_qkv"], st["fused_fc1"], st["fused_fc2"], st["consumed"]) == (1, 1, 1, 3)
    assert st["selfcheck_pass"] == 3 and st["materialize"] == 0


def test_stash_met_by_another_quant_is_materialised(fuse):
    """A producer output read by something other than its layer's quant gets the stock bytes."""
    Quant, Act = _make_classes()
    tr = _tr(Quant, Act)
    blk = tr.MiniMaxH3DiTBlock()
    fq.install(("qkv",), tr, quant_cls=Quant, act_cls=Act, lora_types=(), **_AS_REVIEWED)
    x, shift, scale, gate, idx = _inputs(80, 1)
    with fq.scope(blk, fq.block_plan(blk, ("qkv",))[0]) as sc:
        ph = tr.rms_norm_indexed_scale_shift(x, blk.norm1.weight, shift, scale, idx, 1e-6)
        assert fq.pending_placeholder(ph)
        Quant()(torch.zeros(3, C).to(BF16))                      # another tensor's quant first
        assert not sc.handoffs and fq.stats()["materialize"] == 1
        ref = orms.rms_norm_scale_shift(x, blk.norm1.weight, shift, scale, idx, 1e-6)
        assert torch.equal(ph.view(torch.int16), ref.view(torch.int16))
    assert fq._tls.ctx is None


def test_a_fused_producer_that_differs_disables_its_site(fuse, monkeypatch):
    Quant, Act = _make_classes()
    tr = _tr(Quant, Act)
    blk = tr.MiniMaxH3DiTBlock()
    monkeypatch.setattr(fq, "silu_mul_quant", lambda x, stock=None: (oq.quant(og.silu_and_mul(x))[0],
                                                                    oq.quant(og.silu_and_mul(x))[1] * 2))
    fq.install(("fc2",), tr, quant_cls=Quant, act_cls=Act, lora_types=(), **_AS_REVIEWED)
    args = _inputs(70, 2)
    got = tr.MiniMaxH3DiTBlock.forward(blk, *args)
    assert "fc2" in fq._state["disabled"] and fq.stats()["fused_fc2"] == 0
    Quant2, Act2 = _make_classes()                         # an unpatched block with the same layers
    stock = _tr(Quant2, Act2).MiniMaxH3DiTBlock
    b2 = stock.__new__(stock)
    b2.__dict__.update(blk.__dict__)
    for a, b in zip(got, stock.forward(b2, *args)):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_plan_refuses_blocks_it_cannot_fuse(fuse):
    Quant, Act = _make_classes()
    tr = _tr(Quant, Act)
    fq._state["quant_cls"] = Quant
    blk = tr.MiniMaxH3DiTBlock()
    assert fq.block_plan(blk, ("qkv", "fc1"))[0] is not None
    blk.attn.qkv_proj.tp_size = 2
    assert fq.block_plan(blk, ("qkv",)) == (None, "qkv: tp_size != 1")
    blk.attn.qkv_proj.tp_size = 1
    blk.attn.qkv_proj.quant_method.fp8_linear.quant_fp8.static = True
    assert fq.block_plan(blk, ("qkv",))[0] is None


def test_install_rules(fuse, monkeypatch):
    """The reference's skip rules: the source check, fc2 below the cutlass level, fc1 beside the consumer fuse's out
    site, the out site outside mode 1, everything under VLLM_BATCH_INVARIANT."""
    import sys
    from h3b import fp8_consumers
    monkeypatch.setitem(sys.modules, "vllm", None)          # vLLM's linear path is not looked up (a slow import)
    Quant, Act = _make_classes()
    tr = _tr(Quant, Act)
    tr.MiniMaxH3Attention = type("MiniMaxH3Attention", (), {"forward": lambda self, x: x})
    tr.MiniMaxH3MLP = type("MiniMaxH3MLP", (), {"forward": lambda self, x: x})
    kw = {"quant_cls": Quant, "act_cls": Act, "lora_types": ()}
    assert fq.install(("qkv", "fc1", "fc2"), tr, level="cutlass", env={}, **kw) == []        # not reviewed source
    assert fq.install(("qkv", "fc1", "fc2"), tr, env={"VLLM_BATCH_INVARIANT": "1"}, check_source=False, **kw) == []
    assert fq.install(("out",), tr, ulysses_mode="2", **_AS_REVIEWED, **kw) == []
    assert fq.install(("out",), tr, ulysses_mode=None, **_AS_REVIEWED, **kw) == []
    owned = _tr(Quant, Act)

    def consumer_fused(*a):
        return orms.gate_rms_norm_scale_shift(*a)
    consumer_fused._h3b_consumer_fuse = True
    owned.indexed_gate_rms_norm_scale_shift = consumer_fused
    assert fq.install(("fc1", "fc2"), owned, check_source=False, level="tensor32", env={}, **kw) == []
    assert "out" not in fp8_consumers._state["sites"]
    assert fq.install(("fc1", "fc2"), tr, check_source=False, level="tensor32", env={}, **kw) == ["fc1"]


def _installed(sites=("qkv", "fc1", "fc2")):
    Quant, Act = _make_classes()
    tr = _tr(Quant, Act)
    blk = tr.MiniMaxH3DiTBlock()
    ref_tr = _tr(*_make_classes())
    ref_blk = ref_tr.MiniMaxH3DiTBlock.__new__(ref_tr.MiniMaxH3DiTBlock)
    ref_blk.__dict__.update(blk.__dict__)
    assert fq.install(sites, tr, quant_cls=Quant, act_cls=Act, lora_types=(), **_AS_REVIEWED) == list(sites)
    return tr, blk, ref_tr, ref_blk, Quant


def _equal(got, ref):
    return all(torch.equal(a.view(torch.int16), b.view(torch.int16)) for a, b in zip(got, ref))


def test_mode_with_the_stored_row_when_registers_differ(fuse, monkeypatch):
    """A producer whose register-only mode (no bf16 row stored) differs from stock falls back to the mode that stores
    the row (the reference's reload mode); the site stays on."""
    tr, blk, ref_tr, ref_blk, _ = _installed(("qkv",))
    real = fq.rms_quant

    def regs_differ(x, weight, shift, scale, indices, eps, stock=None, ph=None):
        q, s = real(x, weight, shift, scale, indices, eps, stock, ph)
        return (q, s * 2) if ph is None else (q, s)

    monkeypatch.setattr(fq, "rms_quant", regs_differ)
    args = _inputs(90, 4)
    ref = ref_tr.MiniMaxH3DiTBlock.forward(ref_blk, *args)
    assert _equal(tr.MiniMaxH3DiTBlock.forward(blk, *args), ref)
    st = fq.stats()
    assert st["selfcheck_fail"] == 1 and st["selfcheck_pass"] == 1 and st["fused_qkv"] == 1
    assert "qkv" not in fq._state["disabled"] and fq._state["checked"][("qkv", C, BF16, BF16, 1)]


def test_layer_that_never_quantises_is_rerun(fuse):
    """A planned layer that returns without its quant consuming the stash ran on the placeholder: it is materialised
    and the layer run again."""
    tr, blk, ref_tr, ref_blk, _ = _installed(("qkv",))

    def unquantised(x, _w=blk.attn.qkv_proj.weight):
        return (x.float() @ _w).to(BF16), None

    blk.attn.qkv_proj.forward = unquantised
    args = _inputs(90, 5)
    ref = ref_tr.MiniMaxH3DiTBlock.forward(ref_blk, *args)
    assert _equal(tr.MiniMaxH3DiTBlock.forward(blk, *args), ref)
    assert fq.stats()["rerun"] == 1 and fq.stats()["materialize"] == 1 and fq.stats()["consumed"] == 0


@pytest.mark.parametrize("how", ["static_scale", "other_shape"])
def test_quant_calls_that_do_not_match_the_stash_get_real_rows(fuse, how):
    """A quant with a static scale, or on another shape than the placeholder's, is not the planned call: the stash is
    materialised first, so the layer's own quant sees the stock rows."""
    tr, blk, _, _, _ = _installed(("qkv",))
    lin = blk.attn.qkv_proj
    quant = lin.quant_method.fp8_linear.quant_fp8

    def forward(x, _lin=lin):
        k = _lin.weight.shape[0]
        if how == "static_scale":
            q, s = quant(x.reshape(-1, k), torch.ones(1))
        else:
            q, s = quant(x.reshape(-1, k)[:-1])
            q, s = torch.cat((q, q[-1:])), torch.cat((s, s[-1:]))
        return (q.float() * s @ _lin.weight).to(BF16), None

    lin.forward = forward
    args = _inputs(70, 6)
    got = tr.MiniMaxH3DiTBlock.forward(blk, *args)
    h = orms.rms_norm_scale_shift(args[0], blk.norm1.weight, args[1], args[2], args[4], 1e-6)
    q_ref, _ = forward(h)
    assert torch.equal(got[0], orms.gate_rms_norm_scale_shift(args[0], args[3], q_ref[:, :C], blk.norm2.weight,
                                                              args[1], args[2], args[4], 1e-6)[0])
    assert fq.stats()["materialize"] == 1 and fq.stats()["consumed"] == 0


def test_plan_exclusions(fuse):
    Quant, Act = _make_classes()
    tr = _tr(Quant, Act)
    fq._state["quant_cls"] = Quant
    blk = tr.MiniMaxH3DiTBlock()
    blk.attn.to_gate_compress = object()                       # a VSA gate reads the qkv input a second time
    assert sorted(fq.block_plan(blk, ("qkv", "fc1"))[0]) == ["fc1"]
    blk.attn.to_gate_compress = None
    assert fq.block_plan(blk, ("qkv",), lora_types=(Linear,)) == (None, "qkv: missing or LoRA-wrapped layer")
    for attr, val in (("static", True), ("is_group_quant", True), ("use_per_token_if_dynamic", False),
                      ("num_token_padding", 16)):
        q = blk.attn.qkv_proj.quant_method.fp8_linear.quant_fp8
        old = getattr(q, attr)
        setattr(q, attr, val)
        assert fq.block_plan(blk, ("qkv",))[0] is None, attr
        setattr(q, attr, old)
    blk.attn.qkv_proj.input_scale = torch.ones(1)              # a static input scale
    assert fq.block_plan(blk, ("qkv",))[0] is None
    del blk.attn.qkv_proj.input_scale
    assert fq.block_plan(blk, ("qkv",))[0] is not None


def test_producers_outside_a_block_and_verify_mode(fuse):
    tr, blk, ref_tr, ref_blk, _ = _installed()
    x, shift, scale, gate, idx = _inputs(40, 7)
    h = tr.rms_norm_indexed_scale_shift(x, blk.norm1.weight, shift, scale, idx, 1e-6)   # no block context: stock
    assert torch.equal(h, orms.rms_norm_scale_shift(x, blk.norm1.weight, shift, scale, idx, 1e-6))
    assert fq.stats()["fused_qkv"] == 0
    fq._state["verify"] = True
    args = _inputs(80, 8)
    assert _equal(tr.MiniMaxH3DiTBlock.forward(blk, *args), ref_tr.MiniMaxH3DiTBlock.forward(ref_blk, *args))
    assert fq.stats()["verify_calls"] == 3 and fq.stats()["verify_mismatch"] == 0
