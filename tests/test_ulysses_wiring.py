"""The drop-in wiring of the Ulysses exchange on the CPU (fakes for the model, threads for the ranks): the redirected
producers (norm + RoPE, and the consumer-fused qkv projection) write per destination into send buffers behind
placeholders, the wrapped attention forward exchanges those buffers, and every call it cannot take (unarmed, a
consumer's self-check, ineligible shapes) runs stock -- the reference's wiring (h3_tp2/ulysses_exact.py:313-505)."""
from types import SimpleNamespace

import pytest
import torch

from h3b import fp8_consumers, fp8_gemm, ulysses_exact as ux
from oracle import attention as oa
from oracle import gemm as og
from oracle import ulysses as ou

WS = 2
INFO = lambda layer, md: (None, WS)  # noqa: E731  strict Ulysses over WS ranks for every layer


@pytest.fixture(autouse=True)
def _clean_thread_state():
    yield
    ux._tls.armed = None
    ux._tls.pending = None


def _attn(q, k, v, md=None):  # noqa: ARG001
    return oa.sdpa(q[0], k[0], v[0]).to(q.dtype).unsqueeze(0)


def _launch(x_block, weight, table, eps, out):
    out.copy_(ou.norm_rope(x_block, weight, table, eps))


def _stock_forward(q, k, v, a2a):
    sq, sk, sv = (ou.stock_all_to_all_4d(t, 2, 1, WS, a2a) for t in (q, k, v))
    return ou.stock_all_to_all_4d(_attn(sq, sk, sv), 1, 2, WS, a2a)


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


@pytest.mark.parametrize("mode", ["1", "fwd"])
def test_rope_redirect_ranks_equal_stock(mode):
    m, heads, d = 96, 4, 16
    ins = [_inputs(m, heads, d, 8, 40 + r) for r in range(WS)]

    def stock(r, a2a):
        q, k, v, wq, wk, table = ins[r]
        q, k = ou.norm_rope(q, wq, table, 1e-6), ou.norm_rope(k, wk, table, 1e-6)
        return _stock_forward(q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0), a2a)

    def ours(r, a2a):
        q, k, v, wq, wk, table = ins[r]
        rope = ux.make_rope(_fail, INFO, _launch, lambda *a: True, unpack_fn=ou.unpack)
        fwd = ux.make_forward_impl(_fail, mode, INFO, a2a=a2a, attn=_attn, pack=ou.pack, unpack_fn=ou.unpack,
                                   stock_back=lambda t: ou.stock_all_to_all_4d(t, 1, 2, WS, a2a))

        def body(self_, x):  # noqa: ARG001
            qp, kp = rope(q, k, wq, wk, table, 1e-6)
            assert ux._is_placeholder(qp) and ux._is_placeholder(kp)
            return fwd(object(), qp.unsqueeze(0), kp.unsqueeze(0), v.unsqueeze(0))

        return ux.make_armed_forward(body)(_owner(), torch.empty(m, 8))

    ref, got = ou.run_ranks(stock, WS), ou.run_ranks(ours, WS)
    for r in range(WS):
        assert torch.equal(ref[r], got[r]), r


def _stash(t, heads, seed):
    g = torch.Generator().manual_seed(seed)
    a, sa = og.quant_weight(torch.randn(t, 256, generator=g))
    w, sb = og.quant_weight(torch.randn(3 * heads * 128, 256, generator=g) * 0.02)
    ph = torch.empty(t, 3 * heads * 128, dtype=torch.bfloat16)
    return fp8_consumers.Stash(a, w, sa, sb, None, ph)


def _eager_qkv(st, heads):
    x = fp8_gemm.epilogue_torch(og.accumulate(st.a, st.w), st.sa, st.sb, None, torch.bfloat16)
    return [c.reshape(-1, heads, 128) for c in x.split(heads * 128, dim=1)]


def _fake_fc(heads):
    def qkv_into_send(st, num_heads, ws, qw, kw, table, eps):
        q, k, v = _eager_qkv(st, num_heads)
        return (ou.pack(ou.norm_rope(q, qw, table, eps), ws), ou.pack(ou.norm_rope(k, kw, table, eps), ws),
                ou.pack(v, ws))
    return SimpleNamespace(qkv_into_send=qkv_into_send)


def test_fused_producer_ranks_equal_stock():
    """The consumer-fused producer writes q, k and v per destination; the model's v view stays unwritten."""
    t, heads = 72, 4
    ins = [(_stash(t, heads, 70 + r), *_inputs(t, heads, 128, 32, 80 + r)[3:]) for r in range(WS)]

    def stock(r, a2a):
        st, wq, wk, table = ins[r]
        q, k, v = _eager_qkv(st, heads)
        q, k = ou.norm_rope(q, wq, table, 1e-6), ou.norm_rope(k, wk, table, 1e-6)
        return _stock_forward(q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0), a2a)

    def ours(r, a2a):
        st, wq, wk, table = ins[r]
        prod = ux.make_fused_producer(_fail, _fake_fc(heads), INFO, unpack_fn=ou.unpack)
        fwd = ux.make_forward_impl(_fail, "1", INFO, a2a=a2a, attn=_attn, pack=ou.pack, unpack_fn=ou.unpack)

        def body(self_, x):  # noqa: ARG001
            qp, kp, v = prod(st, heads, heads, 128, wq, wk, table, 1e-6)
            model_v = st.ph[:, 2 * heads * 128:].view(t, heads, 128)
            assert v.data_ptr() == model_v.data_ptr()
            return fwd(object(), qp.unsqueeze(0), kp.unsqueeze(0), model_v.unsqueeze(0))

        return ux.make_armed_forward(body)(_owner(), torch.empty(t, 8))

    ref, got = ou.run_ranks(stock, WS), ou.run_ranks(ours, WS)
    for r in range(WS):
        assert torch.equal(ref[r], got[r]), r


def test_fallback_materializes_q_k_and_v():
    """A redirected call whose attention then cannot run the exchange gets real q, k and (in the model's view) v."""
    t, heads = 72, 4
    st = _stash(t, heads, 11)
    _, _, _, wq, wk, table = _inputs(t, heads, 128, 32, 12)
    calls = []
    prod = ux.make_fused_producer(_fail, _fake_fc(heads), INFO, unpack_fn=ou.unpack)
    fwd = ux.make_forward_impl(lambda self_, q, k, v, md=None: calls.append((q, k, v)) or "stock", "1",
                               lambda layer, md: None)

    def body(self_, x):  # noqa: ARG001
        qp, kp, v = prod(st, heads, heads, 128, wq, wk, table, 1e-6)
        return fwd(object(), qp.unsqueeze(0), kp.unsqueeze(0), v.unsqueeze(0))

    assert ux.make_armed_forward(body)(_owner(), torch.empty(t, 8)) == "stock"
    (q, k, v), = calls
    rq, rk, rv = _eager_qkv(st, heads)
    assert torch.equal(q[0], ou.norm_rope(rq, wq, table, 1e-6)) and torch.equal(k[0], ou.norm_rope(rk, wk, table, 1e-6))
    assert torch.equal(v[0], rv)


def test_calls_the_wiring_cannot_take_run_stock():
    m, heads, d = 96, 4, 16
    q, k, v, wq, wk, table = _inputs(m, heads, d, 8, 4)
    rope = ux.make_rope(lambda *a, **kw: "stock", INFO, _launch, lambda *a: True)
    assert rope(q, k, wq, wk, table, 1e-6) == "stock"                      # no armed attention forward
    gated = _owner()
    gated.to_gate_compress = object()                                      # a VSA gate
    assert ux.make_armed_forward(lambda s, x: rope(q, k, wq, wk, table, 1e-6))(gated, torch.empty(m, 8)) == "stock"
    odd = ux.make_rope(lambda *a, **kw: "stock", lambda layer, md: (None, 3), _launch, lambda *a: True)
    assert ux.make_armed_forward(lambda s, x: odd(q, k, wq, wk, table, 1e-6))(_owner(), torch.empty(m, 8)) == "stock"
    # a consumer's self-check sized call (<= 64 rows) stays stock and leaves the arm for the full call
    st = _stash(80, heads, 9)
    _, _, _, wq2, wk2, table2 = _inputs(80, heads, 128, 32, 10)
    seen = []
    prod = ux.make_fused_producer(lambda st_, *a: seen.append(st_.a.shape[0]) or ("q", "k", "v"), _fake_fc(heads),
                                  INFO)

    def body(self_, x):  # noqa: ARG001
        sub = fp8_consumers.Stash(st.a[:64], st.w, st.sa[:64], st.sb, None, st.ph[:64].clone())
        assert prod(sub, heads, heads, 128, wq2, wk2, table2[:64], 1e-6) == ("q", "k", "v")
        qp, _, _ = prod(st, heads, heads, 128, wq2, wk2, table2, 1e-6)
        assert ux._is_placeholder(qp)
        return seen

    assert ux.make_armed_forward(body)(_owner(), torch.empty(80, 8)) == [64]


def test_placeholder_without_buffers_and_bad_mode_raise():
    ph = ux._placeholder(torch.randn(64, 4, 16)).unsqueeze(0)
    with pytest.raises(RuntimeError):
        ux.take_pending(ph, ph, ph)
    with pytest.raises(ValueError):
        ux.make_forward_impl(lambda *a: None, "3", INFO)


def test_fused_into_send_fills_the_given_buffers():
    """``fused_into_send`` (the reference's consumer-fused producer) writes the projection of the stash into the send
    buffers it is given, q and k normalised and rotated; a bias or another head size is refused."""
    t, heads = 24, 4
    st = _stash(t, heads, 3)
    _, _, _, wq, wk, table = _inputs(t, heads, 128, 32, 4)
    seen = {}

    def qkv_into_send(st_, num_heads, ws, qw, kw, tab, eps, sends=None):
        packed = _fake_fc(heads).qkv_into_send(st_, num_heads, ws, qw, kw, tab, eps)
        for dst, src in zip(sends, packed):
            dst.copy_(src)
        seen["ws"] = ws

    fc = SimpleNamespace(qkv_into_send=qkv_into_send)
    sends = [torch.empty(ux.send_shape(t, heads, 128, WS), dtype=torch.bfloat16) for _ in range(3)]
    ux.fused_into_send(fc, st, heads, 128, wq, wk, table, 1e-6, sends)
    q, k, v = _eager_qkv(st, heads)
    assert seen["ws"] == WS
    assert torch.equal(sends[0], ou.pack(ou.norm_rope(q, wq, table, 1e-6), WS))
    assert torch.equal(sends[1], ou.pack(ou.norm_rope(k, wk, table, 1e-6), WS))
    assert torch.equal(sends[2], ou.pack(v, WS))
    with pytest.raises(ValueError, match="head_dim"):
        ux.fused_into_send(fc, st, heads, 64, wq, wk, table, 1e-6, sends)
    biased = fp8_consumers.Stash(st.a, st.w, st.sa, st.sb, torch.zeros(3 * heads * 128, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="bias"):
        ux.fused_into_send(fc, biased, heads, 128, wq, wk, table, 1e-6, sends)
