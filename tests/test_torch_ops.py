"""The torch.ops.h3b op surface: every op is registered when h3b.ops is imported, with the schema the shims call,
a fake (meta) kernel that gives the output shapes, no CPU kernel (a CPU tensor raises: no CPU fallback), and the
drop-in shims reach the kernels through these ops."""
import inspect

import pytest
import torch

from h3b import ops

BF16, F16, E4M3 = torch.bfloat16, torch.float16, torch.float8_e4m3fn


def test_every_op_is_registered_with_its_schema():
    for name, schema in ops.SCHEMAS.items():
        op = getattr(torch.ops.h3b, name).default
        assert str(op._schema) == "h3b::" + schema, name
    # writes into caller tensors are declared
    assert "Tensor(a!) out" in ops.SCHEMAS["fp8_gemm_out"] and "Tensor(a!)? ph" in ops.SCHEMAS["rms_quant"]


def test_fake_kernels_give_the_output_shapes():
    m = lambda *s, dt=BF16: torch.empty(s, dtype=dt, device="meta")  # noqa: E731
    q, s = torch.ops.h3b.quant(m(300, 640))
    assert q.shape == (300, 640) and q.dtype == E4M3 and s.shape == (300, 1) and s.dtype == torch.float32
    q, s = torch.ops.h3b.quant_from_recv(m(4, 100, 5, 128))
    assert q.shape == (100, 4 * 5 * 128) and s.shape == (100, 1)
    q, s = torch.ops.h3b.quant_rows(m(4, 100, 5, 128), 100, 4, 640, 64000, 640)
    assert q.shape == (100, 2560)
    q, s = torch.ops.h3b.silu_mul_quant(m(8, 512))
    assert q.shape == (8, 256)
    q, s = torch.ops.h3b.rms_quant(m(8, 512), m(512), None, None, None, 1e-6, None)
    assert q.shape == (8, 512) and q.dtype == E4M3
    r, q, s = torch.ops.h3b.gate_rms_quant(m(8, 512), m(1, 512), m(8, 512), m(512), None, None, None, 1e-6)
    assert r.shape == (8, 512) and r.dtype == BF16 and q.dtype == E4M3
    a, w = m(300, 512, dt=E4M3), m(768, 512, dt=E4M3)
    sa, sb = m(300, dt=torch.float32), m(768, dt=torch.float32)
    y = torch.ops.h3b.fp8_gemm(a, w, sa, sb, None, F16)
    assert y.shape == (300, 768) and y.dtype == F16
    assert torch.ops.h3b.fp8_gemm_swiglu(a, w, sa, sb, None).shape == (300, 384)
    assert torch.ops.h3b.fp8_gemm_gate(a, w, sa, sb, m(300, 768), m(2, 768), m(300, dt=torch.int64),
                                       None).shape == (300, 768)
    qq = m(1, 1000, 2, 128)
    assert torch.ops.h3b.flash_attn(qq, qq, qq).shape == (1, 1000, 2, 128)
    assert torch.ops.h3b.flash_attn_scratch(qq, qq, qq, None, 700, m(700, 2, 128, dt=F16),
                                            m(ops.attn_ctl_words(2), dt=torch.int32)).shape == (1, 1000, 2, 128)


def test_cpu_tensors_raise():
    if torch.cuda.is_available():
        pytest.skip("the CPU-key check needs no GPU; on a GPU host the CUDA kernel would be found for CUDA tensors only")
    x = torch.zeros(8, 1, 128, dtype=BF16)
    with pytest.raises(NotImplementedError):
        torch.ops.h3b.flash_attn(x, x, x)
    with pytest.raises(NotImplementedError):
        torch.ops.h3b.quant(torch.zeros(4, 64, dtype=BF16))


def test_shims_call_the_ops():
    """The hot call of every drop-in shim is a torch.ops.h3b op (the scatter epilogues into send / peer buffers, which
    take pointer tables, stay direct calls of h3b.ops)."""
    from h3b import (block, fp8_consumers, fp8_cutlass, fp8_gemm, fp8_quant_fuse, fp8_swiglu, ulysses_exact,
                     ulysses_nocopy, ulysses_outq, ulysses_overlap)
    wants = {
        fp8_gemm.scaled_mm: "torch.ops.h3b.fp8_gemm(", fp8_gemm.launch_fused: "torch.ops.h3b.fp8_gemm_out(",
        fp8_cutlass.DslGemm.run: "torch.ops.h3b.fp8_gemm_out(", fp8_quant_fuse.quant: "torch.ops.h3b.quant(",
        fp8_quant_fuse.rms_quant: "torch.ops.h3b.rms_quant(", fp8_quant_fuse.gate_rms_quant:
        "torch.ops.h3b.gate_rms_quant(", fp8_quant_fuse.unpack_quant: "torch.ops.h3b.quant_from_recv(",
        fp8_quant_fuse.silu_mul_quant: "torch.ops.h3b.silu_mul_quant(",
        fp8_swiglu.gemm_swiglu: "torch.ops.h3b.fp8_gemm_swiglu(", fp8_consumers.gate_fused:
        "torch.ops.h3b.fp8_gemm_gate", ulysses_exact.local_attention: "torch.ops.h3b.flash_attn(",
        ulysses_nocopy.local_attention: "torch.ops.h3b.flash_attn(", ulysses_outq.quant_rows:
        "torch.ops.h3b.quant_rows(", ulysses_outq.quant_from_recv: "torch.ops.h3b.quant_from_recv(",
        ulysses_overlap.quant_grouped_back: "torch.ops.h3b.quant_rows(",
        block.AttentionBlock.forward: "torch.ops.h3b.flash_attn_scratch(",
    }
    for fn, call in wants.items():
        assert call in inspect.getsource(fn), fn.__qualname__
