"""The tensor wrappers over the C ABI refuse, before any launch, every argument the kernels would misread: the C entry
points take base pointers and trust the caller for extents and element types, so a wrong-sized output, a short RoPE
table, a wrong-typed input or a bias the norm epilogue would drop must stop in the wrapper.  Run on the CPU with the
CUDA-tensor guard lifted, the stream stubbed and the library call recorded instead of made."""
import pytest
import torch

from h3b import _lib, ops

BF16, F16, E4M3 = torch.bfloat16, torch.float16, torch.float8_e4m3fn


@pytest.fixture
def calls(monkeypatch):
    made = []
    monkeypatch.setattr(ops, "_need_cuda", lambda *ts: None)
    monkeypatch.setattr(ops, "_stream", lambda t: 0)
    monkeypatch.setattr(_lib, "call", lambda name, *a: made.append(name))
    return made


def _refused(calls, exc, fn, match=None):
    n = len(calls)
    with pytest.raises(exc, match=match):
        fn()
    assert len(calls) == n, "a refused call reached the library"


def test_unpack_recv(calls):
    recv = torch.zeros(2, 8, 3, 128, dtype=BF16)
    _refused(calls, ValueError, lambda: ops.unpack_recv(recv, out=torch.empty(8, 5, 128, dtype=BF16)), "out must")
    _refused(calls, ValueError, lambda: ops.unpack_recv(recv, out=torch.empty(8, 6, 128, dtype=F16)), "out must")
    _refused(calls, ValueError, lambda: ops.unpack_recv(recv, out=torch.empty(8, 128, 6, dtype=BF16).transpose(1, 2)))
    _refused(calls, TypeError, lambda: ops.unpack_recv(recv.float()))
    assert ops.unpack_recv(recv, out=torch.empty(8, 6, 128, dtype=BF16)).shape == (8, 6, 128)
    assert ops.unpack_recv(recv.to(F16)).dtype == F16
    assert calls == ["h3b_unpack_recv"] * 2


def test_pack_by_dest(calls):
    x = torch.zeros(8, 6, 128, dtype=BF16)
    _refused(calls, TypeError, lambda: ops.pack_by_dest(x.float(), 2))
    _refused(calls, TypeError, lambda: ops.pack_by_dest(x.to(F16), 2, to_f16=True))
    _refused(calls, ValueError, lambda: ops.pack_by_dest(x, 4), "heads")
    _refused(calls, ValueError, lambda: ops.pack_by_dest(x, 2, out=torch.empty(2, 8, 3, 64, dtype=BF16)))
    _refused(calls, ValueError, lambda: ops.pack_by_dest(x, 2, out=torch.empty(2, 8, 3, 128, dtype=BF16), to_f16=True))
    assert ops.pack_by_dest(x, 2, out=torch.empty(2, 8, 3, 128, dtype=F16), to_f16=True).dtype == F16
    assert ops.pack_by_dest(x, 3).shape == (3, 8, 2, 128)
    assert calls == ["h3b_pack_by_dest"] * 2


def test_norm_rope_send(calls):
    m, h = 8, 4
    x = torch.zeros(m, h, 128, dtype=BF16)
    w = torch.ones(128, dtype=BF16)
    tab = torch.zeros(m, 64)
    _refused(calls, ValueError, lambda: ops.norm_rope_send(x, w, tab[:m - 1], 1e-6, 2), "rope table")
    _refused(calls, ValueError, lambda: ops.norm_rope_send(x, w, torch.zeros(m, 160), 1e-6, 2), "rope table")
    _refused(calls, ValueError, lambda: ops.norm_rope_send(x, w[:64], tab, 1e-6, 2), "128")
    _refused(calls, TypeError, lambda: ops.norm_rope_send(x, w.float(), tab, 1e-6, 2))
    _refused(calls, TypeError, lambda: ops.norm_rope_send(x.to(F16), w, tab, 1e-6, 2))
    _refused(calls, ValueError, lambda: ops.norm_rope_send(x, w, tab, 1e-6, 3), "heads")
    _refused(calls, ValueError, lambda: ops.norm_rope_send(x, w, tab, 1e-6, 2, out=torch.empty(2, m, 2, 64, dtype=BF16)))
    assert ops.norm_rope_send(x, w, tab.to(BF16), 1e-6, 2).shape == (2, m, 2, 128)   # a longer or bf16 table is fine
    ops.norm_rope_send(x, w, torch.zeros(2 * m, 32), 1e-6, 4, out=torch.empty(4, m, 1, 128, dtype=BF16))
    assert calls == ["h3b_norm_rope_send"] * 2


def _gemm_args(m, heads, k=64):
    n = 3 * heads * 128
    return torch.zeros(m, k, dtype=E4M3), torch.zeros(n, k, dtype=E4M3), torch.ones(m), torch.ones(n)


def test_qkv_send(calls):
    m, heads, ws = 16, 4, 2
    a, w, sa, sb = _gemm_args(m, heads)
    qw, kw = torch.ones(128, dtype=BF16), torch.ones(128, dtype=BF16)
    tab = torch.zeros(m, 64)
    bias = torch.zeros(3 * heads * 128, dtype=BF16)
    send = lambda **kw_: ops.fp8_gemm_qkv_send(a, w, sa, sb, heads, ws, **kw_)  # noqa: E731
    _refused(calls, ValueError, lambda: send(bias=bias, qk_norm=(qw, kw, tab, 1e-6)), "bias")
    _refused(calls, ValueError, lambda: send(qk_norm=(qw, kw, tab[:m // 2], 1e-6)), "rope table")
    _refused(calls, ValueError, lambda: send(qk_norm=(qw[:100], kw, tab, 1e-6)), "128")
    shape = (ws, m, heads // ws, 128)
    bf = lambda: torch.empty(shape, dtype=BF16)  # noqa: E731
    _refused(calls, ValueError, lambda: send(sends=[bf(), bf()]), "three")
    _refused(calls, ValueError, lambda: send(sends=[bf(), bf(), bf()], v_f16=True), "send buffer v")
    _refused(calls, ValueError, lambda: send(sends=[bf(), bf(), torch.empty(shape, dtype=F16)]), "send buffer v")
    _refused(calls, ValueError, lambda: send(sends=torch.empty(1, ws, m, 3, 1, 128, dtype=BF16), interleaved=True))
    _refused(calls, ValueError, lambda: send(sends=[bf(), torch.empty(ws, m, 128, heads // ws, dtype=BF16).transpose(2, 3),
                                                    bf()]))
    send(sends=[bf(), bf(), torch.empty(shape, dtype=F16)], v_f16=True)
    send(qk_norm=(qw, kw, tab, 1e-6))
    send(bias=bias)
    assert send(interleaved=True, groups=2).shape == (2, ws, m, 3, 1, 128)
    assert calls == ["h3b_fp8_gemm"] * 4


def test_flash_attn(calls):
    s, h = 32, 2
    q = torch.zeros(s, h, 128, dtype=BF16)
    _refused(calls, ValueError, lambda: ops.flash_attn(q, torch.zeros(s, 1, 128, dtype=BF16), q), "k and v")
    _refused(calls, ValueError, lambda: ops.flash_attn(q, q, torch.zeros(s - 8, h, 128, dtype=BF16)), "k and v")
    _refused(calls, ValueError, lambda: ops.flash_attn(q, q, q, out=torch.empty(s - 8, h, 128, dtype=BF16)), "out must")
    _refused(calls, ValueError, lambda: ops.flash_attn(q, q, q, out=torch.empty(s, h, 128, dtype=F16)), "out must")
    _refused(calls, TypeError, lambda: ops.bf16_to_f16(q.float()))
    # the bf16-v pass's scratch: an f16 copy of the valid rows of v and the control words, each checked for size
    _refused(calls, ValueError, lambda: ops.flash_attn(q, q, q, v16=torch.empty(s - 1, h, 128, dtype=F16)), "v16")
    _refused(calls, TypeError, lambda: ops.flash_attn(q, q, q, v16=torch.empty(s, h, 128, dtype=BF16)))
    _refused(calls, ValueError, lambda: ops.flash_attn(q, q, q, ctl=torch.empty(ops.attn_ctl_words(h) - 1,
                                                                                 dtype=torch.int32)), "ctl")
    ops.flash_attn(q, q, q, valid_kv=20, v16=torch.empty(20, h, 128, dtype=F16))   # v16 holds the valid rows only
    kv = torch.zeros(2 * s, h, 128, dtype=BF16)
    ops.flash_attn(q, kv, kv.to(F16))                              # more keys than queries, f16 v as is
    wide = torch.empty(s, h + 1, 128, dtype=BF16)
    ops.flash_attn(q.unsqueeze(0), q, q, out=wide[:, :h].unsqueeze(0))  # a strided output view, bf16 v
    ops.flash_attn(q, q, q, pv_f16=False)                          # bf16 P.V asked for
    assert calls == ["h3b_flash_attn_fwd_bf16v", "h3b_flash_attn_fwd", "h3b_flash_attn_fwd_bf16v",
                     "h3b_flash_attn_fwd"]


def test_flash_attn_p2p(calls):
    ws, m, hl = 2, 16, 2
    q = torch.zeros(ws * m, hl, 128, dtype=BF16)
    good = [torch.empty(ws, m, hl, 128, dtype=BF16) for _ in range(ws)]
    _refused(calls, ValueError, lambda: ops.flash_attn_p2p(q, q, q, [good[0], torch.empty(ws, m, hl, 64, dtype=BF16)],
                                                          0), "reverse receive buffer")
    _refused(calls, ValueError, lambda: ops.flash_attn_p2p(q, q, q[:-8], good, 0), "k and v")
    _refused(calls, ValueError, lambda: ops.flash_attn_p2p(q[:-1], q, q, good, 0), "peers")
    ops.flash_attn_p2p(q, q, q.to(F16), good, 1)
    ops.flash_attn_p2p(q, q, q.to(F16), [4096, 8192], 0)           # device addresses are the caller's to size
    ops.flash_attn_p2p(q, q, q, good, 0)                           # bf16 v: the pass that takes any range
    assert calls == ["h3b_flash_attn_fwd_p2p"] * 2 + ["h3b_flash_attn_fwd_p2p_bf16v"]


def test_quant_rows_span(calls):
    recv = torch.zeros(2, 8, 3, 128, dtype=BF16)
    seg = 3 * 128
    ops.quant_rows(recv, 8, 2, seg, 8 * seg, seg)                           # exactly the buffer
    _refused(calls, ValueError, lambda: ops.quant_rows(recv, 9, 2, seg, 8 * seg, seg), "reach")
    _refused(calls, ValueError, lambda: ops.quant_rows(recv, 8, 2, seg + 8, 8 * seg, seg), "reach")
    _refused(calls, ValueError, lambda: ops.quant_rows(recv, 8, 2, seg, -seg, seg))
    _refused(calls, TypeError, lambda: ops.quant_rows(recv.to(F16), 8, 2, seg, 8 * seg, seg))
    big = torch.zeros(8, 1024, dtype=BF16)
    ops.quant(big[:, :512])                                                 # a strided row view: its span is enough
    ops.quant_from_recv(recv)
    assert calls == ["h3b_quant_rows_e4m3"] * 3


def test_rms_family(calls):
    rows, hid = 8, 64
    x = torch.zeros(rows, hid, dtype=BF16)
    w = torch.ones(hid, dtype=BF16)
    sh, sc, gt = (torch.zeros(4, hid, dtype=BF16) for _ in range(3))
    idx = torch.zeros(rows, dtype=torch.int32)
    _refused(calls, ValueError, lambda: ops.rms_quant(x, w, sh, None, idx), "together")
    _refused(calls, ValueError, lambda: ops.rms_quant(x, w[:32], sh, sc, idx), "weight")
    _refused(calls, ValueError, lambda: ops.rms_quant(x, w, sh[:, :32], sc, idx), "shift")
    _refused(calls, ValueError, lambda: ops.rms_quant(x, w, sh, sc, idx[:4]), "indices")
    _refused(calls, ValueError, lambda: ops.rms_quant(x, w, sh, sc, idx.float()), "indices")
    _refused(calls, ValueError, lambda: ops.rms_quant(x, w, ph=torch.empty(rows, hid + 8, dtype=BF16)), "placeholder")
    _refused(calls, TypeError, lambda: ops.rms_quant(x.float(), w))
    _refused(calls, ValueError, lambda: ops.rms_quant(torch.zeros(hid, rows, dtype=BF16).t(), w))
    ops.rms_quant(x, w, sh, sc, idx, 1e-6, torch.empty(rows, hid, dtype=BF16))
    ops.rms_quant(x, w, sh.unsqueeze(1), sc.unsqueeze(1), idx)              # [B, 1, hidden] modulation rows
    ops.rms_quant(x, w)
    r = torch.zeros(rows, hid, dtype=BF16)
    _refused(calls, ValueError, lambda: ops.gate_rms_quant(r, gt, r[:4], w, sh, sc, idx, 1e-6), "branch")
    _refused(calls, ValueError, lambda: ops.gate_rms_quant(r, gt[:, :8], r, w, sh, sc, idx, 1e-6), "gate")
    _refused(calls, ValueError, lambda: ops.gate_rms_quant(r, None, r, w, sh, sc, idx, 1e-6), "gate")
    ops.gate_rms_quant(r, gt, r, w, sh, sc, idx, 1e-6)
    ops.gate_rms_quant(r, gt[:1], r, w, None, None, None, 1e-6)
    _refused(calls, ValueError, lambda: ops.silu_mul_quant(torch.zeros(rows, 65, dtype=BF16)))
    _refused(calls, TypeError, lambda: ops.silu_mul_quant(torch.zeros(rows, 64)))
    ops.silu_mul_quant(x)
    assert calls == ["h3b_rms_quant_e4m3"] * 3 + ["h3b_gate_rms_quant_e4m3"] * 2 + ["h3b_silu_mul_quant_e4m3"]


def test_scale_passes(calls):
    m, n = 8, 64
    x32 = torch.zeros(m, n)
    sa, sb = torch.ones(m), torch.ones(n)
    _refused(calls, TypeError, lambda: ops.scale_bias_cast(x32.to(BF16), sa, sb, None, BF16))
    _refused(calls, ValueError, lambda: ops.scale_bias_cast(x32, sa[:4], sb, None, BF16), "scales")
    _refused(calls, ValueError, lambda: ops.scale_bias_cast(x32, sa, sb[:8], None, BF16), "scales")
    _refused(calls, TypeError, lambda: ops.scale_swiglu(x32.to(BF16), sa, sb, None))
    _refused(calls, ValueError, lambda: ops.scale_swiglu_quant(torch.zeros(m, 63), sa, torch.ones(63), None))
    ops.scale_bias_cast(x32, torch.ones(1), sb, None, F16)                  # a scalar scale broadcasts
    ops.scale_swiglu(x32, sa, sb, None)
    ops.scale_swiglu_quant(x32, sa, sb, torch.zeros(n, dtype=BF16))
    assert calls == ["h3b_scale_bias_cast", "h3b_scale_swiglu", "h3b_scale_swiglu_quant"]
