"""Host-side logic of the drop-in modules on the CPU: the Ulysses orchestration with injected layout functions and a
threaded collective, the plugin's switch plan, and the no-CPU-fallback rule."""
import pytest
import torch

from _util import same_bits, t16
from h3b import fp8_gemm, ops, plugin, ulysses_exact, ulysses_outq
from oracle import quant as oq
from oracle import ulysses as ou


def _layout_attn(q, k, v):
    return (q.float() + 2.0 * k.float() - 0.5 * v.float()).to(q.dtype)


@pytest.mark.parametrize("ws", [2, 4])
def test_exact_forward_matches_reference_outputs(golden, ws):
    g = golden("ulysses")
    m, heads, d = (int(v) for v in g[f"ws{ws}_shape"])
    qs, ks, vs = ([t16(g[f"ws{ws}_{n}{r}"]) for r in range(ws)] for n in ("q", "k", "v"))

    def body(r, a2a):
        return ulysses_exact.exact_forward(qs[r], ks[r], vs[r], _layout_attn, ws=ws, a2a=a2a, pack=ou.pack,
                                           unpack_fn=ou.unpack)

    res = ou.run_ranks(body, ws)
    for r in range(ws):
        assert same_bits(res[r], t16(g[f"ws{ws}_out{r}"]))


class _Quant:
    """Stands in for vLLM's QuantFP8 (dynamic, per token): the oracle's quant."""
    static = False
    is_group_quant = False
    use_per_token_if_dynamic = True
    num_token_padding = None

    def __init__(self):
        self.calls = 0

    def __call__(self, x, scale=None, scale_ub=None):
        self.calls += 1
        return oq.quant(x)


def _owner(heads, d):
    """An attention whose out-projection reaches ``quant_method.fp8_linear.quant_fp8`` (the prepared path)."""
    from types import SimpleNamespace
    kernel = SimpleNamespace(quant_fp8=_Quant())
    layer = SimpleNamespace(tp_size=1, input_size_per_partition=heads * d, quant_method=SimpleNamespace(fp8_linear=kernel))
    return SimpleNamespace(out_proj=layer, num_heads=heads, head_dim=d), kernel


@pytest.fixture
def outq_cpu(monkeypatch):
    """The deferral's two kernels on the CPU (the oracle's), and a fresh self-check state."""
    monkeypatch.setitem(ulysses_outq._kernels, "quant_from_recv", oq.quant_from_recv)
    monkeypatch.setitem(ulysses_outq._kernels, "unpack_rows", lambda recv: ou.unpack(recv).reshape(recv.shape[1], -1))
    monkeypatch.setitem(ulysses_outq._state, "checked", False)
    monkeypatch.setitem(ulysses_outq._state, "disabled", None)
    monkeypatch.setitem(ulysses_outq._state, "sources", None)


def test_exact_forward_with_presupplied_sends_and_defer(outq_cpu):
    """Mode 2: an armed forward's reverse exchange returns a stride-0 placeholder; the prepared out-projection quant
    recognises it and quantises the receive buffer (after the first call's self-check), bit-equal to copy 5 + quant."""
    ws, m, heads, d = 2, 4, 4, 8
    qs = [torch.randn(1, m, heads, d).to(torch.bfloat16) for _ in range(ws)]
    ks = [torch.randn(1, m, heads, d).to(torch.bfloat16) for _ in range(ws)]
    vs = [torch.randn(1, m, heads, d).to(torch.bfloat16) for _ in range(ws)]

    def body(r, a2a):
        owner, kernel = _owner(heads, d)
        prev = ulysses_outq.arm(owner, m)
        sends = [ou.pack(t[r][0], ws) for t in (qs, ks, vs)]
        ph = ulysses_exact.exact_forward(qs[r], ks[r], vs[r], _layout_attn, ws=ws, a2a=a2a, sends=sends,
                                         back="defer", unpack_fn=ou.unpack)
        assert sends == []
        assert ulysses_outq.is_placeholder(ph) and ph.shape == (1, m, heads, d)
        out = kernel.quant_fp8(ph.view(m, heads * d))
        ulysses_outq.disarm(prev, check=True)
        return out

    res = ou.run_ranks(lambda r, a2a: body(r, a2a), ws)
    ref = ou.run_ranks(lambda r, a2a: ulysses_exact.exact_forward(qs[r], ks[r], vs[r], _layout_attn, ws=ws, a2a=a2a,
                                                                  pack=ou.pack, unpack_fn=ou.unpack), ws)
    for r in range(ws):
        rq, rs = oq.quant(ref[r].reshape(m, heads * d))
        assert same_bits(res[r][0], rq) and torch.equal(res[r][1], rs)
    assert ulysses_outq._state["checked"] and ulysses_outq._state["disabled"] is None


def test_deferral_needs_the_reviewed_upstream_path(outq_cpu, monkeypatch):
    """Mode 2's producer hook checks the upstream sources on the attention forward as upstream wrote it: a changed
    path keeps the reverse unpack (``prepare`` refuses every attention); the reviewed path lets it through."""
    import sys
    from types import SimpleNamespace

    from h3b import sources
    monkeypatch.setitem(sys.modules, "vllm", None)              # vLLM's linear path is not looked up (a slow import)

    class MiniMaxH3Attention:
        def forward(self, x):
            return x

    def rope(*a, **kw):
        return a[:2]
    upstream = MiniMaxH3Attention.forward
    tr = SimpleNamespace(MiniMaxH3Attention=MiniMaxH3Attention, fused_qk_norm_rope=rope)
    ulysses_exact._hook_producers_on(tr, lambda layer, md: None, "2")
    assert MiniMaxH3Attention.forward._h3b_exact_armed and tr.fused_qk_norm_rope._h3b_exact
    assert ulysses_outq._state["sources"].startswith("upstream source changed: attn_forward")
    owner, kernel = _owner(4, 8)
    assert not ulysses_outq.prepare(owner) and not isinstance(kernel.quant_fp8, ulysses_outq.OutQuant)
    assert sources.outq_fingerprints(upstream) == {"attn_forward": sources.fingerprint(upstream)}
    monkeypatch.setattr(sources, "outq_fingerprints", lambda fwd: dict(sources.OUTQ_REVIEWED))
    assert ulysses_outq.check_sources(upstream) is None
    owner, kernel = _owner(4, 8)
    assert ulysses_outq.prepare(owner) and isinstance(kernel.quant_fp8, ulysses_outq.OutQuant)


def test_deferral_guards_and_self_check_failure(outq_cpu, monkeypatch):
    m, heads, d, ws = 4, 4, 8, 2
    recv = torch.randn(ws, m, heads // ws, d).to(torch.bfloat16)
    # not armed: no placeholder (the caller unpacks)
    assert ulysses_outq.defer(recv, heads) is None
    owner, kernel = _owner(heads, d)
    prev = ulysses_outq.arm(owner, m)
    ph = ulysses_outq.defer(recv, heads)
    # an armed forward that returns without consuming its deferral raises
    with pytest.raises(RuntimeError, match="without its out-projection"):
        ulysses_outq.disarm(prev, check=True)
    # a placeholder reaching a quant with no pending deferral raises
    with pytest.raises(RuntimeError, match="placeholder"):
        kernel.quant_fp8(ph.view(m, heads * d))
    # a receive-buffer quant that differs from copy 5 + quant disables the path for the process: stock result returned
    monkeypatch.setitem(ulysses_outq._kernels, "quant_from_recv",
                        lambda r: (oq.quant_from_recv(r)[0], oq.quant_from_recv(r)[1] * 2))
    prev = ulysses_outq.arm(owner, m)
    ph = ulysses_outq.defer(recv, heads)
    q, s = kernel.quant_fp8(ph.view(m, heads * d))
    ulysses_outq.disarm(prev, check=True)
    rq, rs = oq.quant(ou.unpack(recv).reshape(m, -1))
    assert same_bits(q, rq) and torch.equal(s, rs)
    assert ulysses_outq._state["disabled"]
    prev = ulysses_outq.arm(owner, m)
    assert ulysses_outq.defer(recv, heads) is None
    ulysses_outq.disarm(prev, check=True)


def test_send_shape_and_by_dest_views():
    x = torch.arange(6 * 8 * 4).float().view(6, 8, 4)
    assert ulysses_exact.send_shape(6, 8, 4, 2) == (2, 6, 4, 4)
    assert torch.equal(ulysses_exact.by_dest(x, 2).contiguous(), ou.pack(x, 2))


def test_eligibility():
    q = torch.zeros(1, 4, 8, 16)
    assert ulysses_exact.eligible_shape(q, q, q, 2)
    assert not ulysses_exact.eligible_shape(q, q, q, 1)
    assert not ulysses_exact.eligible_shape(q, q, q, 3)
    assert not ulysses_exact.eligible_shape(torch.zeros(2, 4, 8, 16), q, q, 2)


def test_plugin_plan_defaults_and_switches():
    p = plugin.plan({})
    assert p["ulysses"] == "2" and p["fp8_gemm"] == "cutlass" and p["overlap"] is None
    assert p["swiglu"] == 1 and p["quant_fuse"] == "1"
    assert plugin.plan({"H3_TP2_FP8_FUSE_SWIGLU": "2"})["swiglu"] == 2
    assert plugin.plan({"H3_TP2_FP8_FUSE_SWIGLU": "0"})["swiglu"] == 0
    assert plugin.plan({"H3_TP2_FP8_GEMM": "0"})["swiglu"] == 0      # the MLP fusion rides on the GEMM dispatcher
    assert p["consumer_fuse"] == "1"
    assert plugin.plan({"H3_TP2_FP8_GEMM": "tensor32", "H3_TP2_FP8_CONSUMER_FUSE": "fc2,out"})["consumer_fuse"] == "fc2,out"
    assert plugin.plan({"H3_TP2_FP8_GEMM": "fused"})["consumer_fuse"] is None     # no stash at the fused level
    assert plugin.plan({"H3_TP2_FP8_CONSUMER_FUSE": "0"})["consumer_fuse"] is None
    p = plugin.plan({"H3_TP2_A2A_OVERLAP": "2", "H3_TP2_FP8_GEMM": "0", "H3_TP2_A2A_TIMING": "1"})
    assert p["ulysses"] == "2" and p["overlap"] is None and p["fp8_gemm"] is None and p["a2a_timing"]  # exact wins
    p = plugin.plan({"H3_TP2_A2A_OVERLAP": "2", "H3_TP2_ULYSSES_EXACT": "0"})
    assert p["overlap"] == 2 and p["ulysses"] is None and p["nocopy"] is None
    p = plugin.plan({"H3_TP2_A2A_OVERLAP": "4", "H3_TP2_ULYSSES_NOCOPY": "force"})
    assert p["nocopy"] == 4 and p["ulysses"] is None and p["overlap"] is None
    assert plugin.plan({"H3_TP2_ULYSSES_NOCOPY": "1"})["nocopy"] is None      # the reference requires "force"
    plugin.register()  # no H3_TP2_ROLE: a no-op


def test_gemm_dispatch_guards():
    a = torch.zeros(8, 32, dtype=torch.float8_e4m3fn)
    b = torch.zeros(16, 32, dtype=torch.float8_e4m3fn).t()
    sa, sb = torch.ones(8, 1), torch.ones(16)
    assert fp8_gemm.eligible(a, b, sa, sb, torch.bfloat16, None)
    assert not fp8_gemm.eligible(a, b, torch.ones(1), torch.ones(1), torch.bfloat16, None)   # per-tensor: stock
    assert not fp8_gemm.eligible(a, b.contiguous(), sa, sb, torch.bfloat16, None)            # b.t() not contiguous
    assert not fp8_gemm.eligible(a, b, sa, sb, torch.float32, None)
    # a bias is read as bf16 by the kernels: bf16 is taken, an f16 bias falls through to the stock dispatch
    assert fp8_gemm.eligible(a, b, sa, sb, torch.float16, torch.zeros(16, dtype=torch.bfloat16))
    assert not fp8_gemm.eligible(a, b, sa, sb, torch.float16, torch.zeros(16, dtype=torch.float16))


def test_launch_fused_signature_and_raw_accumulator_refusal():
    """launch_fused takes the reference's cfg argument; the raw fp32 accumulator form is refused, not faked."""
    a = torch.zeros(8, 32, dtype=torch.float8_e4m3fn)
    b = torch.zeros(16, 32, dtype=torch.float8_e4m3fn).t()
    y = torch.empty(8, 16)
    with pytest.raises(NotImplementedError, match="raw accumulator"):
        fp8_gemm.launch_fused(a, b, torch.ones(8), torch.ones(16), None, y, (128, 128, 64, 8, 3))


def test_route_order_routers_then_hooks():
    calls = []
    fp8_gemm._routers.clear(), fp8_gemm._stash_hooks.clear()
    fp8_gemm.set_router(lambda *a: calls.append("router"))
    fp8_gemm.set_stash_hook(lambda *a: (calls.append("hook"), "ph")[1])
    assert fp8_gemm.route(None, None, None, None, None) == "ph"
    assert calls == ["router", "hook"]
    fp8_gemm._routers.clear(), fp8_gemm._stash_hooks.clear()


def test_kernels_refuse_cpu_tensors():
    x = torch.zeros(4, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        ops.quant(x)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        ops.flash_attn(torch.zeros(8, 1, 128, dtype=torch.bfloat16), torch.zeros(8, 1, 128, dtype=torch.bfloat16),
                       torch.zeros(8, 1, 128, dtype=torch.bfloat16))


def test_new_entry_points_refuse_cpu_tensors():
    z8 = torch.zeros(4, 64, dtype=torch.float8_e4m3fn)
    s = torch.ones(4)
    x = torch.zeros(4, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        ops.fp8_gemm_gate(z8, z8, s, s, x, x, torch.zeros(4, dtype=torch.int64))
    q = torch.zeros(8, 1, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        ops.flash_attn_p2p(q, q, q, [q, q], 0)
    from h3b import ulysses_nocopy
    send = torch.zeros(ulysses_nocopy.send_shape(4, 4, 128, 2, 1), dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        ulysses_nocopy.pack_qkv(send, torch.zeros(4, 4, 128), torch.zeros(4, 4, 128), torch.zeros(4, 4, 128), 2, 1)


def test_nocopy_layout_helpers_match_the_oracle():
    """send_shape / qkv_views of the mirror against the oracle's restatement (pure views, no kernel)."""
    from h3b import ulysses_nocopy
    assert ulysses_nocopy.send_shape(16, 8, 128, 2, 2) == ou.nocopy_send_shape(16, 8, 128, 2, 2) == (2, 2, 16, 3, 2, 128)
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(16, 8, 128, generator=g).to(torch.bfloat16) for _ in range(3))
    send = ou.pack_qkv(q, k, v, 2, 1)
    a = ulysses_nocopy.qkv_views(send[0])
    b = ou.qkv_views(send[0])
    for x, y in zip(a, b):
        assert x.stride() == y.stride() and same_bits(x.contiguous(), y.contiguous())
    v16 = ulysses_nocopy.qkv_views(send[0], v_f16=True)[2]
    assert v16.dtype == torch.float16 and v16.data_ptr() == a[2].data_ptr()


def test_p2p_epoch_is_passed_as_int32_serial_number(monkeypatch):
    """Epochs grow without bound on the host; the barrier kernel compares them as 32-bit serial numbers."""
    seen = []
    monkeypatch.setattr(ops._lib, "call", lambda name, *args: seen.append(args[4]))
    for e in (1, 2 ** 31 - 1, 2 ** 31, 2 ** 32 + 5):
        ops.p2p_signal_wait([16, 32], 16, 0, e, 0)
    assert seen == [1, 2 ** 31 - 1, -2 ** 31, 5]


def test_block_exchange_options_are_validated():
    from h3b.block import AttentionBlock
    w = (torch.zeros(3 * 2 * 128, 64, dtype=torch.float8_e4m3fn), torch.ones(768),
         torch.zeros(64, 256, dtype=torch.float8_e4m3fn), torch.ones(64))
    with pytest.raises(ValueError, match="exchange"):
        AttentionBlock(64, 2, device="cpu", ws=2, weights=w, exchange="rdma", groups=1)
    with pytest.raises(ValueError, match="head groups"):
        AttentionBlock(64, 4, device="cpu", ws=2, weights=(torch.zeros(3 * 4 * 128, 64, dtype=torch.float8_e4m3fn),
                                                           torch.ones(1536), torch.zeros(64, 512,
                                                                                        dtype=torch.float8_e4m3fn),
                                                           torch.ones(64)), exchange="p2p", groups=2, rank=0)


@pytest.mark.parametrize("M,N", [(1, 16), (255, 256), (257, 272), (62_496, 15_360), (15_624, 5_120), (3_000, 27_648)])
def test_gemm_tile_raster_covers_every_tile_once(M, N):
    """The pair-tile raster of the persistent GEMM (mirrored by fp8_gemm.tile_coords) visits each (256-row block,
    256-column block) exactly once, GROUP_M row blocks at a time."""
    bm, bn, _, _, _ = fp8_gemm.fused_config()
    num_mb, num_nb = -(-M // bm), -(-N // bn)
    seen = [fp8_gemm.tile_coords(t, M, N) for t in range(num_mb * num_nb)]
    assert sorted(seen) == [(i, j) for i in range(num_mb) for j in range(num_nb)]
    # within a group of GROUP_M row blocks, consecutive tiles walk down the rows of one column block first
    if num_mb >= 2 and num_nb >= 2:
        assert seen[1] == (1, 0)


def test_exact_forward_hooks_and_counters():
    """set_key_hook sees each rank's packed keys before their exchange; set_unpack_hook replaces the reverse unpack;
    stats() counts the packed forwards (h3_tp2/ulysses_exact.py:88,144,151)."""
    ws, m, heads, d = 2, 4, 4, 8
    qs, ks, vs = ([torch.randn(1, m, heads, d) for _ in range(ws)] for _ in range(3))
    seen = []
    ulysses_exact.set_key_hook(lambda send_k: seen.append(tuple(send_k.shape)))
    ulysses_exact.set_unpack_hook(lambda recv, h: torch.full((1, recv.shape[1], h, recv.shape[3]), 7.0))
    before = ulysses_exact.stats()
    try:
        res = ou.run_ranks(lambda r, a2a: ulysses_exact.exact_forward(qs[r], ks[r], vs[r], _layout_attn, ws=ws,
                                                                      a2a=a2a, pack=ou.pack, unpack_fn=ou.unpack), ws)
    finally:
        ulysses_exact.set_key_hook(None)
        ulysses_exact.set_unpack_hook(None)
    after = ulysses_exact.stats()
    assert seen == [(ws, m, heads // ws, d)] * ws
    assert all(t.shape == (1, m, heads, d) and bool((t == 7.0).all()) for t in res)
    assert after["pack"] - before["pack"] == ws and after["unpack_hook"] - before["unpack_hook"] == ws


def test_verify_forward_compares_with_the_stock_exchange():
    """verify_forward runs the stock all-to-alls and the exact exchange on the same tensors: all equal for a correct
    layout, and a stock side that differs is reported (h3_tp2/ulysses_exact.py:232)."""
    ws, m, heads, d = 2, 4, 4, 8
    qs, ks, vs = ([torch.randn(1, m, heads, d) for _ in range(ws)] for _ in range(3))

    def body(r, a2a, skew=0.0):
        return ulysses_exact.verify_forward(
            qs[r], ks[r], vs[r], _layout_attn, ws=ws, a2a=a2a, pack=ou.pack, unpack_fn=ou.unpack,
            stock_fwd=lambda t: ou.stock_all_to_all_4d(t, 2, 1, ws, a2a),
            stock_back=lambda t: ou.stock_all_to_all_4d(t, 1, 2, ws, a2a) + skew)

    for res, eq in ou.run_ranks(body, ws):
        assert eq == {"q": True, "k": True, "v": True, "attn": True, "result": True}
        assert res.shape == (1, m, heads, d)
    for _, eq in ou.run_ranks(lambda r, a2a: body(r, a2a, skew=1.0), ws):
        assert eq["q"] and eq["attn"] and not eq["result"]


def test_cutlass_block_wiring_registers_the_running_block_weights(monkeypatch):
    """fp8_cutlass: inside a wrapped DiT block forward the router knows the block's qkv / out / fc1 weights by pointer
    and shape ([K, N] as vLLM stores them); outside it nothing is routed (h3_tp2/fp8_cutlass.py:252-294)."""
    from types import SimpleNamespace
    from h3b import fp8_cutlass
    lin = lambda k, n: SimpleNamespace(weight=torch.zeros(k, n, dtype=torch.float8_e4m3fn))  # noqa: E731
    block = SimpleNamespace(attn=SimpleNamespace(qkv_proj=lin(32, 96), out_proj=lin(32, 32)),
                            mlp=SimpleNamespace(fc1=lin(32, 128)))
    want = fp8_cutlass.block_want(block)
    assert sorted(want.values()) == ["fc1", "out", "qkv"]
    assert want[(block.attn.qkv_proj.weight.data_ptr(), (32, 96))] == "qkv"
    seen = []
    fwd = fp8_cutlass.make_block_forward(lambda self, x: seen.append(dict(fp8_cutlass._tls.want)) or x)
    assert fwd(block, 7) == 7 and seen == [want]
    assert getattr(fp8_cutlass._tls, "want", None) is None
    tr = SimpleNamespace(MiniMaxH3DiTBlock=type("Block", (), {"forward": lambda self, x: x}))
    monkeypatch.setattr(fp8_gemm, "_routers", [])
    assert fp8_cutlass.install_sites(tr) and tr.MiniMaxH3DiTBlock.forward._h3b_cutlass
    assert fp8_gemm._routers == [fp8_cutlass.route]


def test_dispatcher_install_levels(monkeypatch):
    """``fp8_gemm.install``: the kernel's probe decides whether the dispatcher goes in at all (stock stays otherwise);
    the cutlass level registers the block router after its own check, else runs as tensor32 (h3_tp2/fp8_gemm.py:344)."""
    from types import SimpleNamespace
    from h3b import fp8_cutlass
    monkeypatch.setattr(fp8_gemm, "_routers", [])
    monkeypatch.setattr(fp8_gemm, "_state", {"level": "tcgen05", "installed": False})

    def stock(a, b, scale_a, scale_b, out_dtype, bias=None):
        return "stock"
    vops = SimpleNamespace(cutlass_scaled_mm=stock)
    fp8_gemm._install_into(vops, "cutlass", probe=lambda dev: False)
    assert vops.cutlass_scaled_mm is stock and fp8_gemm._state == {"level": "stock", "installed": False}
    fp8_gemm._install_into(vops, "cutlass", probe=lambda dev: True, cutlass_probe=lambda dev: False)
    assert fp8_gemm._state["level"] == "tensor32" and fp8_gemm._routers == []
    mm = vops.cutlass_scaled_mm
    a = torch.zeros(4, 32, dtype=torch.float8_e4m3fn)
    assert mm(a, a.t(), torch.ones(4, 1), torch.ones(4), torch.bfloat16) == "stock"     # CPU tensors: stock
    assert mm.stats == {"two_pass": 0, "stock": 1}
    fp8_gemm._install_into(vops, "cutlass", probe=lambda dev: True, cutlass_probe=lambda dev: True)
    assert vops.cutlass_scaled_mm is mm                                                  # installed once
    vops2 = SimpleNamespace(cutlass_scaled_mm=stock)
    fp8_gemm._install_into(vops2, "cutlass", probe=lambda dev: True, cutlass_probe=lambda dev: True)
    assert fp8_gemm._state["level"] == "cutlass" and fp8_gemm._routers == [fp8_cutlass.route]
    with pytest.raises(ValueError, match="unknown"):
        fp8_gemm._install_into(SimpleNamespace(cutlass_scaled_mm=stock), "int8")


def test_cutlass_router_order_failure_and_verify(monkeypatch):
    """The block router runs before the stash hooks and only for the running block's weights; a launch that raises
    turns it off for the process; verify mode compares each routed output with the two-pass arithmetic."""
    from h3b import fp8_cutlass
    a = torch.randint(-3, 4, (6, 32)).to(torch.float8_e4m3fn)
    w = torch.randint(-3, 4, (48, 32)).to(torch.float8_e4m3fn)
    b, other = w.t(), torch.zeros(48, 32, dtype=torch.float8_e4m3fn).t()
    sa, sb = torch.full((6, 1), 0.5), torch.full((48,), 0.25)
    monkeypatch.setattr(fp8_cutlass, "_state", {"ok": True, "verify": True})
    monkeypatch.setattr(fp8_cutlass, "_stats", {"dsl": 0, "fallthrough": 0})
    monkeypatch.setattr(fp8_gemm, "_routers", [fp8_cutlass.route])
    monkeypatch.setattr(fp8_gemm, "_stash_hooks", [lambda *args: "stashed"])
    mm = lambda a_, b_, sa_, sb_, dt, bias: fp8_cutlass._two_pass(a_, b_, sa_, sb_, dt, bias)  # noqa: E731
    monkeypatch.setattr(fp8_cutlass, "scaled_mm", mm)
    fp8_cutlass._tls.want = {(b.data_ptr(), tuple(b.shape)): "qkv"}
    try:
        y = fp8_gemm.route(a, b, sa, sb, torch.bfloat16)
        assert isinstance(y, torch.Tensor) and fp8_cutlass.stats()["dsl"] == 1
        assert fp8_cutlass.stats()["verify_calls"] == 1 and "verify_mismatch" not in fp8_cutlass.stats()
        assert fp8_gemm.route(a, other, sa, sb, torch.bfloat16) == "stashed"             # not the block's weight
        monkeypatch.setattr(fp8_cutlass, "scaled_mm", lambda *args: (_ for _ in ()).throw(RuntimeError("launch")))
        assert fp8_gemm.route(a, b, sa, sb, torch.bfloat16) == "stashed" and not fp8_cutlass._state["ok"]
        assert fp8_cutlass.stats()["fallthrough"] == 1
        off_by_one = lambda *args: mm(*args).view(torch.int16).add(1).view(torch.bfloat16)  # noqa: E731
        monkeypatch.setattr(fp8_cutlass, "scaled_mm", off_by_one)
        fp8_cutlass._state["ok"] = True
        fp8_gemm.route(a, b, sa, sb, torch.bfloat16)
        assert fp8_cutlass.stats()["verify_mismatch"] == 1
    finally:
        fp8_cutlass._tls.want = None


def test_deferral_refusals_once_only_views_and_passthrough(outq_cpu):
    """``defer`` refuses an unarmed forward, other rows, non-bf16 receive buffers, another head count and an
    out-projection ``prepare`` refused; one deferral per armed forward; the model's views of the placeholder still
    match; other inputs pass to the wrapped quant (attributes too); a placeholder in another shape raises
    (h3_tp2/ulysses_outq.py:191-421)."""
    m, heads, d, ws = 16, 4, 8, 2
    k = heads * d
    recv = torch.randn(ws, m, heads // ws, d).to(torch.bfloat16)
    assert ulysses_outq.defer(recv, heads) is None                               # not armed
    owner, kernel = _owner(heads, d)
    for rows, buf, h in ((m + 1, recv, heads), (m, recv.float(), heads), (m, recv, heads + 2)):
        prev = ulysses_outq.arm(owner, rows)
        assert ulysses_outq.defer(buf, h) is None
        ulysses_outq.disarm(prev, check=True)
    refused, _ = _owner(heads, d)
    refused.out_proj._h3b_outq = False                                            # prepare() said no
    prev = ulysses_outq.arm(refused, m)
    assert ulysses_outq.defer(recv, heads) is None
    ulysses_outq.disarm(prev, check=True)

    prev = ulysses_outq.arm(owner, m)
    ph = ulysses_outq.defer(recv, heads)
    assert ph.shape == (1, m, heads, d) and ulysses_outq.defer(recv, heads) is None      # once per armed forward
    x = ph.squeeze(0).reshape(m, k).view(-1, k)                                   # the model's views
    assert x.data_ptr() == ph.data_ptr() and x.stride() == (0, 0) and ulysses_outq._tls.pending.matches(x)
    with pytest.raises(RuntimeError, match="another shape"):
        kernel.quant_fp8(ph.reshape(m * k)[None].expand(1, m * k))
    q, s = kernel.quant_fp8(x)
    rq, rs = oq.quant(ou.unpack(recv).reshape(m, k))
    assert same_bits(q, rq) and torch.equal(s, rs)
    ulysses_outq.disarm(prev, check=True)

    y = torch.randn(8, k).to(torch.bfloat16)
    calls = kernel.quant_fp8._orig.calls
    q, s = kernel.quant_fp8(y)                                                    # an ordinary input: the layer's quant
    assert kernel.quant_fp8._orig.calls == calls + 1 and same_bits(q, oq.quant(y)[0])
    assert kernel.quant_fp8.use_per_token_if_dynamic and not kernel.quant_fp8.static   # attributes reach the quant
    prev = ulysses_outq.arm(owner, m)
    ulysses_outq.defer(recv, heads)
    ulysses_outq.disarm(prev, check=False)                                        # an exception is propagating
    assert getattr(ulysses_outq._tls, "pending", None) is None


def test_fused_swiglu_marker_never_imports_the_model(monkeypatch):
    """The startup diagnostic reads the MLP class marker of an already-loaded module only (h3_tp2/plugin.py:34)."""
    import sys
    from types import ModuleType
    name = "vllm_omni.diffusion.models.minimax_h3.minimax_h3_transformer"
    monkeypatch.setitem(sys.modules, name, None)
    assert plugin.fused_swiglu_marker() == "unknown"
    monkeypatch.setitem(sys.modules, name, object())
    assert plugin.fused_swiglu_marker() == "unknown"
    lazy = ModuleType(name)

    def fail_if_queried(_name):
        raise AssertionError("the diagnostic looked an attribute up lazily")
    lazy.__getattr__ = fail_if_queried
    monkeypatch.setitem(sys.modules, name, lazy)
    assert plugin.fused_swiglu_marker() == "unknown"
    module = ModuleType(name)

    class MiniMaxH3MLP:
        pass
    module.MiniMaxH3MLP = MiniMaxH3MLP
    monkeypatch.setitem(sys.modules, name, module)
    assert plugin.fused_swiglu_marker() == "absent"
    MiniMaxH3MLP._h3b_fused_swiglu = True
    assert plugin.fused_swiglu_marker() == "present"
    MiniMaxH3MLP._h3b_fused_swiglu = "unexpected"
    assert plugin.fused_swiglu_marker() == "unknown"


def test_a2a_timing_wraps_the_collective_the_4d_exchange_and_reports_per_diffuse(monkeypatch):
    """``a2a_timing`` (h3_tp2/a2a_timing.py): the collective and ``comm.all_to_all_4D`` are timed with events, the totals
    are reported (and cleared) at the end of each ``diffuse``, and uninstall restores everything."""
    from types import SimpleNamespace
    import torch.distributed as dist
    from h3b import a2a_timing

    class Event:
        def record(self):
            pass

        def elapsed_time(self, end):  # noqa: ARG002
            return 2.0                                              # ms

    monkeypatch.setattr(a2a_timing, "_event", Event)
    monkeypatch.setattr(a2a_timing, "_sync", lambda: None)
    calls = []
    monkeypatch.setattr(dist, "all_to_all_single", lambda out, inp, group=None: calls.append("a2a") or out.copy_(inp))
    comm_dist = SimpleNamespace(all_to_all_single=dist.all_to_all_single)

    def all_to_all_4d(x, *a, **kw):  # noqa: ARG001  (stock: permute copies around the collective comm looks up)
        out = torch.empty_like(x)
        comm_dist.all_to_all_single(out, x)
        return out
    comm = SimpleNamespace(dist=comm_dist, all_to_all_4D=all_to_all_4d)
    reports = []

    class Pipeline:
        def diffuse(self, x):
            comm.all_to_all_4D(x)
            dist.all_to_all_single(torch.empty_like(x), x)
            return "latents"

    orig_diffuse = Pipeline.diffuse
    a2a_timing.install(comm=comm, pipeline_cls=Pipeline)
    real_report = a2a_timing.report
    monkeypatch.setattr(a2a_timing, "report", lambda phase="diffuse": reports.append(real_report(phase)))
    try:
        assert Pipeline().diffuse(torch.zeros(4, 8)) == "latents"
        assert calls == ["a2a", "a2a"]
        assert reports == [{"outer": {"calls": 1, "s": 0.002, "bytes": 128},
                            "inner": {"calls": 2, "s": 0.004, "bytes": 256}}]
        assert real_report() is None                                  # cleared by the diffuse report
    finally:
        a2a_timing.uninstall()
    assert Pipeline.diffuse is orig_diffuse and not getattr(dist.all_to_all_single, "_h3b_a2a_timing", False)


def test_probes_answer_false_without_a_gpu(monkeypatch):
    """The install probes never raise on a host without a GPU: the dispatcher then leaves the stock kernel in place.
    The host is made GPU-less here, so the test means the same on a GPU box."""
    import torch
    from h3b import fp8_swiglu
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    assert fp8_gemm.probe_fused("cuda") is False and fp8_gemm.probe_fused("cpu") is False
    assert fp8_swiglu.probe_gemm_swiglu("cuda") is False
