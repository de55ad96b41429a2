"""The plugin's ``_apply`` against stand-in vLLM / vLLM-Omni modules on the CPU: the switches install the modules in the
reference's order, the FP8 dispatcher resolves its level, and the interplay rules hold (the cutlass level routes qkv /
out ahead of the consumer fuse, the combined exchange owns the rope producer, the consumer fuse's out site owns the
gated RMS, the quant fuse's out site needs the exact exchange in mode 1, its fc2 site the cutlass level).  Kernel
probes and the upstream source fingerprints are stubbed as passing (the stand-ins are not vLLM-Omni's code)."""
import sys
from types import ModuleType

import pytest

from h3b import (fp8_consumers, fp8_cutlass, fp8_gemm, fp8_quant_fuse, fp8_swiglu, plugin, sources, ulysses_exact,
                 ulysses_nocopy)


def _stock(*a, **kw):  # noqa: ARG001
    return "stock"


def _modules():
    """Fresh stand-ins for the modules the plugin patches (package modules with the classes and functions it reads)."""
    mods = {}

    def mod(name, **attrs):
        m = ModuleType(name)
        m.__dict__.update(attrs)
        mods[name] = m
        return m

    class QuantFP8:
        def forward(self, x, scale=None, scale_ub=None):  # noqa: ARG002
            return "stock quant"

    class SiluAndMul:
        def forward(self, x):
            return x

    class Attention:
        def _forward_impl(self, q, k, v, md=None):  # noqa: ARG002
            return "stock attention"

    class MiniMaxH3DiTBlock:
        def forward(self, x):
            return x

    class MiniMaxH3Attention:
        def forward(self, x):
            return x

    class MiniMaxH3MLP:
        def forward(self, x):
            return x

    mod("vllm")
    mod("vllm._custom_ops", cutlass_scaled_mm=_stock)
    mod("vllm.model_executor")
    mod("vllm.model_executor.layers")
    mod("vllm.model_executor.layers.quantization")
    mod("vllm.model_executor.layers.quantization.input_quant_fp8", QuantFP8=QuantFP8)
    for name in ("vllm_omni", "vllm_omni.diffusion", "vllm_omni.diffusion.attention", "vllm_omni.diffusion.models",
                 "vllm_omni.diffusion.models.minimax_h3", "vllm_omni.diffusion.layers"):
        mod(name)
    mod("vllm_omni.diffusion.attention.layer", Attention=Attention)
    mod("vllm_omni.diffusion.layers.activation", SiluAndMul=SiluAndMul)
    mod("vllm_omni.diffusion.models.minimax_h3.minimax_h3_transformer", MiniMaxH3DiTBlock=MiniMaxH3DiTBlock,
        MiniMaxH3Attention=MiniMaxH3Attention, MiniMaxH3MLP=MiniMaxH3MLP, fused_qk_norm_rope=_stock,
        indexed_gate=_stock, indexed_gate_rms_norm_scale_shift=_stock, rms_norm_indexed_scale_shift=_stock)
    return mods


@pytest.fixture
def stack(monkeypatch):
    mods = _modules()
    for name, m in mods.items():
        monkeypatch.setitem(sys.modules, name, m)
    for name in ("vllm_omni.diffusion.layers.fused_qk_norm_rope", "vllm_omni.diffusion.layers.indexed_modulation",
                 "vllm.lora", "vllm.lora.layers"):
        monkeypatch.setitem(sys.modules, name, None)       # absent: imports of them fail at once
    monkeypatch.setattr(fp8_gemm, "_state", {"level": "tcgen05", "installed": False})
    monkeypatch.setattr(fp8_gemm, "_routers", [])
    monkeypatch.setattr(fp8_gemm, "_stash_hooks", [])
    monkeypatch.setattr(fp8_gemm, "probe_fused", lambda device: True)
    monkeypatch.setattr(fp8_cutlass, "probe", lambda device="cuda": True)
    monkeypatch.setattr(fp8_consumers, "_state", {"sites": (), "checked": {}, "disabled": set(),
                                                  "device_types": ("cuda",)})
    for key, val in (("sites", ()), ("checked", {}), ("disabled", set()), ("orig_quant", None), ("quant_cls", None),
                     ("act_cls", None)):
        monkeypatch.setitem(fp8_quant_fuse._state, key, val)
    reviewed = dict(sources.REVIEWED, **sources.REVIEWED_EXTRA)
    monkeypatch.setattr(sources, "consumer_fingerprints", lambda tr: dict(reviewed))
    monkeypatch.setattr(sources, "quant_fingerprints", lambda tr: dict(reviewed))
    for key in [k for k in __import__("os").environ if k.startswith("H3_TP2_") or k == "VLLM_BATCH_INVARIANT"]:
        monkeypatch.delenv(key)
    return mods


def _tr(mods):
    return mods["vllm_omni.diffusion.models.minimax_h3.minimax_h3_transformer"]


def test_defaults(stack):
    """Defaults: exact exchange mode 2, FP8 GEMM at the cutlass level with the block router, fused SwiGLU level 1,
    the consumer fuse on fc2 only (the router takes qkv / out), the quant fuse on qkv / fc1 / fc2 (out: mode 2)."""
    plugin._apply("dit")
    tr, attn = _tr(stack), stack["vllm_omni.diffusion.attention.layer"].Attention
    assert attn._h3b_exact == "2" and not getattr(attn, "_h3b_nocopy", 0)
    assert stack["vllm._custom_ops"].cutlass_scaled_mm._h3b and fp8_gemm._state == {"level": "cutlass",
                                                                                    "installed": True}
    assert fp8_gemm._routers == [fp8_cutlass.route]
    assert tr.MiniMaxH3MLP._h3b_fused_swiglu and plugin.fused_swiglu_marker() == "present"
    assert fp8_consumers._state["sites"] == ("fc2",) and tr.indexed_gate._h3b_consumer_fuse
    assert not getattr(tr.indexed_gate_rms_norm_scale_shift, "_h3b_consumer_fuse", False)
    assert fp8_quant_fuse._state["sites"] == ("qkv", "fc1", "fc2")
    assert fp8_gemm._stash_hooks == [fp8_swiglu._stash_hook, fp8_consumers.stash_hook]
    block_fwd = tr.MiniMaxH3DiTBlock.forward
    assert block_fwd._h3b_quant_fuse and block_fwd.__wrapped__._h3b_consumer_fuse
    assert block_fwd.__wrapped__.__wrapped__._h3b_cutlass


def test_nocopy_at_tensor32(stack, monkeypatch):
    """The combined exchange owns the rope producer (no consumer qkv site); the consumer fuse's out site owns the gated
    RMS (no quant-fuse fc1); without the exact exchange the quant fuse has no out site; fc2 needs the cutlass level."""
    monkeypatch.setenv("H3_TP2_ULYSSES_NOCOPY", "force")
    monkeypatch.setenv("H3_TP2_A2A_OVERLAP", "2")
    monkeypatch.setenv("H3_TP2_FP8_GEMM", "tensor32")
    plugin._apply("dit")
    tr, attn = _tr(stack), stack["vllm_omni.diffusion.attention.layer"].Attention
    assert attn._h3b_nocopy == 2 and not getattr(attn, "_h3b_exact", None)
    assert tr.fused_qk_norm_rope._h3b_nocopy and tr.MiniMaxH3Attention.forward._h3b_nocopy_armed
    assert fp8_gemm._state["level"] == "tensor32" and fp8_gemm._routers == []
    assert fp8_consumers._state["sites"] == ("out", "fc2")
    assert fp8_quant_fuse._state["sites"] == ("qkv",)
    with pytest.raises(RuntimeError, match="exact replaces it"):
        ulysses_exact.install("2")
    with pytest.raises(RuntimeError, match="groups=2"):
        ulysses_nocopy.install(4)


def test_kernel_that_does_not_serve_keeps_stock(stack, monkeypatch):
    """When the GEMM kernel's probe fails the stock dispatch stays and nothing rides on it."""
    monkeypatch.setattr(fp8_gemm, "probe_fused", lambda device: False)
    monkeypatch.setenv("H3_TP2_FP8_QUANT_FUSE", "0")
    plugin._apply("dit")
    tr = _tr(stack)
    assert stack["vllm._custom_ops"].cutlass_scaled_mm is _stock and fp8_gemm._state["level"] == "stock"
    assert fp8_gemm._routers == [] and fp8_gemm._stash_hooks == []
    assert not getattr(tr.MiniMaxH3MLP, "_h3b_fused_swiglu", False) and fp8_consumers._state["sites"] == ()


def test_first_attention_call_hooks_the_producer(stack, monkeypatch):
    """The exact exchange hooks its producer on the first attention call: at tensor32 the consumer-fused qkv (which the
    consumer fuse installed) becomes the per-destination producer; in mode 2 the deferral's upstream path is checked
    first (the stand-in attention forward is not the reviewed one, so the reverse unpack stays)."""
    from h3b import ulysses_outq
    monkeypatch.setattr(fp8_consumers, "qk_norm_rope_fused", fp8_consumers.qk_norm_rope_fused)   # restored after
    monkeypatch.setitem(ulysses_outq._state, "sources", None)
    monkeypatch.setenv("H3_TP2_FP8_GEMM", "tensor32")
    plugin._apply("dit")
    monkeypatch.setitem(sys.modules, "vllm", None)           # the source check finds no vLLM linear path to look up
    tr = _tr(stack)
    assert fp8_consumers._state["sites"] == ("qkv", "out", "fc2") and tr.fused_qk_norm_rope._h3b_consumer_fuse
    ulysses_exact._hook_producers_on(tr, lambda layer, md: None, "2")
    assert fp8_consumers.qk_norm_rope_fused._h3b_exact                 # the consumer-fused producer, redirected
    assert not getattr(tr.fused_qk_norm_rope, "_h3b_exact", False)     # the wrapper itself stays the consumer's
    assert tr.MiniMaxH3Attention.forward._h3b_exact_armed
    assert ulysses_outq._state["sources"].startswith("upstream source changed")


def test_strategy_info_takes_only_plain_strict_ulysses(monkeypatch):
    """``vllm_strategy_info``: (pg, ws) for plain strict Ulysses over more than one rank, None for everything the stock
    path must keep (h3_tp2/ulysses_nocopy.py:336-362)."""
    from types import SimpleNamespace
    import torch.distributed as dist

    class UlyssesParallelAttention:
        def __init__(self, **kw):
            self.__dict__.update(dict(_scatter_idx=2, _gather_idx=1, _use_sync=False, _ulysses_pg="pg",
                                      _sp_group=SimpleNamespace(ring_world_size=1)), **kw)

    mode = {"m": "strict"}
    for name, attrs in (("vllm_omni", {}), ("vllm_omni.diffusion", {}), ("vllm_omni.diffusion.attention", {}),
                        ("vllm_omni.diffusion.attention.parallel", {}),
                        ("vllm_omni.diffusion.attention.parallel.ulysses",
                         {"UlyssesParallelAttention": UlyssesParallelAttention}),
                        ("vllm_omni.diffusion.forward_context", {"get_ulysses_mode": lambda default: mode["m"]})):
        m = ModuleType(name)
        m.__dict__.update(attrs)
        monkeypatch.setitem(sys.modules, name, m)
    ws = {"n": 2}
    monkeypatch.setattr(dist, "get_world_size", lambda pg: ws["n"])

    def layer(strategy=None, **kw):
        s = strategy or UlyssesParallelAttention()
        ns = SimpleNamespace(_get_active_parallel_strategy=lambda: s, _active_paged_kv_adapter=lambda: None)
        ns.__dict__.update(kw)
        return ns

    md = SimpleNamespace(attn_mask=None, joint_query=None, joint_key=None, joint_value=None, joint_attn_mask=None,
                         extra={})
    info = plugin.vllm_strategy_info
    assert info(layer(), md) == ("pg", 2) and info(layer(), None) == ("pg", 2)
    assert info(layer(strategy=object()), md) is None                              # not Ulysses
    assert info(layer(use_ring=True), md) is None
    for kw in ({"_use_sync": True}, {"_ulysses_a2a_permute": True}, {"_scatter_idx": 1},
               {"_sp_group": SimpleNamespace(ring_world_size=2)}):
        assert info(layer(strategy=UlyssesParallelAttention(**kw)), md) is None, kw
    assert info(layer(_scheduler_paged_kv=True), md) is None
    assert info(layer(_has_custom_attention=True), md) is None
    paged = layer()
    paged._active_paged_kv_adapter = lambda: object()
    assert info(paged, md) is None
    for field in ("attn_mask", "joint_query", "joint_attn_mask"):
        assert info(layer(), SimpleNamespace(**dict(vars(md), **{field: object()}))) is None, field
    assert info(layer(), SimpleNamespace(**dict(vars(md), extra={"gate_compress": 1}))) is None
    mode["m"] = "relaxed"
    assert info(layer(), md) is None
    mode["m"], ws["n"] = "strict", 1
    assert info(layer(), md) is None                                               # one rank: nothing to exchange
