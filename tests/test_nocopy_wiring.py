"""The drop-in wiring of the combined q/k/v exchange on the CPU (fakes for the model, threads for the ranks): the
redirected norm + RoPE producer writes q and k per destination into one send buffer behind placeholders, the wrapped
attention forward packs v into that buffer's third slot and runs one exchange per head group, and every call it
cannot take runs stock with real q and k -- the reference's wiring (h3_tp2/ulysses_nocopy.py:190-430).

The product's ``pack_qkv`` / ``fill_slot`` refuse CPU tensors and the groups = 1 unpack is a CUDA kernel; these tests
lift that guard and substitute the eager unpack for the duration of each test only."""
from types import SimpleNamespace

import pytest
import torch

from h3b import ops, ulysses_nocopy as nc
from oracle import attention as oa
from oracle import ulysses as ou

WS = 2
INFO = lambda layer, md: (None, WS)  # noqa: E731  strict Ulysses over WS ranks for every layer


@pytest.fixture(autouse=True)
def _cpu_plumbing(monkeypatch):
    monkeypatch.setattr(ops, "_need_cuda", lambda *ts: None)

    def unpack_recv(recv, out=None):
        p, m, hl, d = recv.shape
        o = out if out is not None else torch.empty((m, p * hl, d), dtype=recv.dtype)
        o.view(m, p, hl, d).copy_(recv.permute(1, 0, 2, 3))
        return o

    monkeypatch.setattr(ops, "unpack_recv", unpack_recv)
    yield
    nc._tls.armed = None
    nc._tls.pending = None


def _attn(q, k, v, md=None):  # noqa: ARG001
    return oa.sdpa(q[0], k[0], v[0]).to(q.dtype).unsqueeze(0)


def _launch(x_block, weight, table, eps, out):
    out.copy_(ou.norm_rope(x_block, weight, table, eps))


def _inputs(m, heads, d, rot, seed):
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(m, heads, d, generator=g).to(torch.bfloat16) for _ in range(3))
    wq, wk = ((1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16) for _ in range(2))
    pos = torch.arange(m, dtype=torch.float32)[:, None] * torch.exp(-torch.arange(rot // 2, dtype=torch.float32))
    return q, k, v, wq, wk, torch.cat((torch.cos(pos), torch.sin(pos)), dim=-1)


def _owner(layer=None):
    return SimpleNamespace(attention=layer or object(), to_gate_compress=None)


def _fail(*a, **kw):  # noqa: ARG001
    raise AssertionError("the stock path ran")


def _stock_forward(q, k, v, a2a):
    sq, sk, sv = (ou.stock_all_to_all_4d(t, 2, 1, WS, a2a) for t in (q, k, v))
    return ou.stock_all_to_all_4d(_attn(sq, sk, sv), 1, 2, WS, a2a)


@pytest.mark.parametrize("groups", [1, 2])
def test_rope_redirect_ranks_equal_stock(groups):
    m, heads, d = 64, 8, 16
    ins = [_inputs(m, heads, d, 8, 70 + r) for r in range(WS)]
    before = nc.stats()

    def stock(r, a2a):
        q, k, v, wq, wk, table = ins[r]
        q, k = ou.norm_rope(q, wq, table, 1e-6), ou.norm_rope(k, wk, table, 1e-6)
        return _stock_forward(q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0), a2a)

    def ours(r, a2a):
        q, k, v, wq, wk, table = ins[r]
        rope = nc.make_rope(_fail, groups, INFO, _launch, lambda *a: True)
        fwd = nc.make_forward_impl(_fail, groups, INFO, a2a=a2a, attn=_attn)

        def body(self_, x):  # noqa: ARG001
            qp, kp = rope(q, k, wq, wk, table, 1e-6)
            assert nc._is_placeholder(qp) and nc._is_placeholder(kp)
            return fwd(object(), qp.unsqueeze(0), kp.unsqueeze(0), v.unsqueeze(0))

        return nc.make_armed_forward(body)(_owner(), torch.empty(m, 8))

    ref, got = ou.run_ranks(stock, WS), ou.run_ranks(ours, WS)
    for r in range(WS):
        assert torch.equal(ref[r], got[r]), r
    assert nc.stats()["redirect"] - before["redirect"] == WS


@pytest.mark.parametrize("groups", [1, 2])
def test_packed_path_equals_the_oracle(groups):
    """q/k that did not come through the redirect are packed (all three slots) and give the oracle's forward."""
    m, heads, d = 48, 8, 16
    ins = [_inputs(m, heads, d, 8, 90 + r) for r in range(WS)]
    before = nc.stats()

    def oracle(r, a2a):
        q, k, v = (t.unsqueeze(0) for t in ins[r][:3])
        return ou.nocopy_forward(q, k, v, _attn, ws=WS, groups=groups, a2a=a2a)

    def ours(r, a2a):
        q, k, v = (t.unsqueeze(0) for t in ins[r][:3])
        return nc.make_forward_impl(_fail, groups, INFO, a2a=a2a, attn=_attn)(object(), q, k, v)

    ref, got = ou.run_ranks(oracle, WS), ou.run_ranks(ours, WS)
    for r in range(WS):
        assert torch.equal(ref[r], got[r]), r
    assert nc.stats()["pack"] - before["pack"] == WS


def test_send_box_v_slot():
    """A box filled with q and k only gets v packed from ``value``; with ``v_in_box`` slot 2 is the producer's."""
    m, heads, d, groups = 32, 4, 8, 1
    q, k, v = (t.unsqueeze(0) for t in _inputs(m, heads, d, 8, 5)[:3])

    def run(box_fill, v_in, v_arg):
        def fn(r, a2a):
            send = torch.full(nc.send_shape(m, heads, d, WS, groups), float("nan"), dtype=q.dtype)
            for slot, x in box_fill.items():
                nc.fill_slot(send, x[0], slot, WS, groups)
            return nc.nocopy_forward(q, k, v_arg, _attn, ws=WS, groups=groups, a2a=a2a, send_box=[send],
                                     v_in_box=v_in)
        return ou.run_ranks(fn, WS)

    ref = run({0: q, 1: k, 2: v}, True, torch.zeros_like(v))
    assert torch.equal(run({0: q, 1: k}, False, v)[0], ref[0])
    assert not torch.isnan(ref[0]).any()


def test_fallback_materializes_q_and_k():
    """The rope wrapper redirected, but the attention call is not eligible (its metadata rules Ulysses out): stock
    ``_forward_impl`` gets real q and k, equal to the stock producer's."""
    m, heads, d = 16, 4, 8
    q, k, v, wq, wk, table = _inputs(m, heads, d, 8, 11)
    info = lambda layer, md: None if md == "no-ulysses" else (None, WS)  # noqa: E731
    seen = {}

    def orig(self_, qq, kk, vv, md=None):  # noqa: ARG001
        seen.update(q=qq, k=kk, v=vv)
        return "stock"

    rope = nc.make_rope(_fail, 1, info, _launch, lambda *a: True)
    fwd = nc.make_forward_impl(orig, 1, info, attn=_fail)
    before = nc.stats()

    def body(self_):  # noqa: ARG001
        qp, kp = rope(q, k, wq, wk, table, 1e-6)
        return fwd(object(), qp.unsqueeze(0), kp.unsqueeze(0), v.unsqueeze(0), "no-ulysses")

    assert nc.make_armed_forward(body)(_owner()) == "stock"
    assert torch.equal(seen["q"][0], ou.norm_rope(q, wq, table, 1e-6))
    assert torch.equal(seen["k"][0], ou.norm_rope(k, wk, table, 1e-6))
    assert seen["v"].data_ptr() == v.data_ptr()
    after = nc.stats()
    assert after["materialize"] - before["materialize"] == 1
    assert after["fallback"] - before["fallback"] == 1


def test_calls_the_wiring_cannot_take_run_stock():
    m, heads, d = 16, 4, 8
    q, k, v, wq, wk, table = _inputs(m, heads, d, 8, 12)
    calls = []

    def orig_rope(*a, **kw):  # noqa: ARG001
        calls.append("rope")
        return a[0], a[1]

    ok = lambda *a: True  # noqa: E731
    armed = lambda fn, owner=None: nc.make_armed_forward(lambda self_: fn())(owner or _owner())  # noqa: E731
    rope = nc.make_rope(orig_rope, 1, INFO, _launch, ok)
    rope(q, k, wq, wk, table, 1e-6)                                   # not armed
    armed(lambda: rope(q, k, wq, wk, table, 1e-6),
          SimpleNamespace(attention=object(), to_gate_compress=object()))  # gated attention
    armed(lambda: nc.make_rope(orig_rope, 1, INFO, _launch, lambda *a: False)(q, k, wq, wk, table, 1e-6))
    armed(lambda: nc.make_rope(orig_rope, 3, INFO, _launch, ok)(q, k, wq, wk, table, 1e-6))  # 4 heads, 3*2 ranks
    armed(lambda: rope(q, k, wq, wk, table, 1e-6, head_dim=d + 1))
    armed(lambda: rope(q, k, wq, wk, table[:-1], 1e-6))               # table rows != tokens
    assert calls == ["rope"] * 6
    assert getattr(nc._tls, "pending", None) is None

    def one_redirect():                                                # one redirect per armed forward
        first = rope(q, k, wq, wk, table, 1e-6)
        nc._tls.pending = None
        rope(q, k, wq, wk, table, 1e-6)
        return first
    qp, _ = armed(one_redirect)
    assert nc._is_placeholder(qp) and calls == ["rope"] * 7

    stock = []
    fwd = nc.make_forward_impl(lambda *a: stock.append(1) or "stock", 1, INFO, attn=_fail)
    b2 = torch.zeros(2, m, heads, d, dtype=torch.bfloat16)
    assert fwd(object(), b2, b2, b2) == "stock"                        # batch 2
    q3 = torch.zeros(1, m, 3, d, dtype=torch.bfloat16)
    assert fwd(object(), q3, q3, q3) == "stock"                        # heads not divisible by the ranks
    assert nc.make_forward_impl(lambda *a: "stock", 1, lambda *a: None)(object(), q3, q3, q3) == "stock"
    assert len(stock) == 2


def test_placeholders_never_outlive_their_forward():
    m, heads, d = 16, 4, 8
    q, k, v, wq, wk, table = _inputs(m, heads, d, 8, 13)
    rope = nc.make_rope(_fail, 1, INFO, _launch, lambda *a: True)
    kept = nc.make_armed_forward(lambda self_: rope(q, k, wq, wk, table, 1e-6))(_owner())
    assert getattr(nc._tls, "pending", None) is None
    with pytest.raises(RuntimeError, match="placeholder"):
        nc.take_pending(kept[0].unsqueeze(0), kept[1].unsqueeze(0))
    assert nc.take_pending(q.unsqueeze(0), k.unsqueeze(0)) is None


def test_install_on_fakes():
    class Attention:
        def _forward_impl(self, q, k, v, md=None):  # noqa: ARG002
            return "stock"

    class MiniMaxH3Attention:
        def forward(self, x):
            return x

    def fused_qk_norm_rope(q, k, *a, **kw):  # noqa: ARG001
        return q, k

    tr = SimpleNamespace(fused_qk_norm_rope=fused_qk_norm_rope, MiniMaxH3Attention=MiniMaxH3Attention)
    nc._install_on(Attention, tr, 2, INFO)
    wrapped = (Attention._forward_impl, tr.fused_qk_norm_rope, MiniMaxH3Attention.forward)
    assert Attention._h3b_nocopy == 2 and tr.fused_qk_norm_rope._h3b_nocopy
    assert MiniMaxH3Attention.forward._h3b_nocopy_armed
    nc._install_on(Attention, tr, 2, INFO)                             # idempotent
    assert wrapped == (Attention._forward_impl, tr.fused_qk_norm_rope, MiniMaxH3Attention.forward)
    with pytest.raises(RuntimeError, match="groups=2"):
        nc._install_on(Attention, tr, 4, INFO)

    class Overlapped:
        _h3b_overlap = 2
    with pytest.raises(RuntimeError, match="overlap"):
        nc._install_on(Overlapped, None, 1, INFO)
