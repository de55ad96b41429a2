"""Per-kernel timing sweep of the library at DiT shapes: every kernel once per row, CUDA-event timed, with its
algorithmic bytes (HBM-bound kernels) or FLOPs (tensor kernels) against the measured peaks.

    python -m h3b.kernel_bench [--rows M] [--iters N] [--once] [--only NAME,...]
    python -m h3b.kernel_bench --ffn [--iters N]
    python -m h3b.kernel_bench --cublas [--rows M] [--iters N]

``--once`` launches each kernel exactly once after its inputs are built (the form an ncu launch capture wants).
``--ffn`` times the FFN of the DiT block (RMSNorm + quant -> fc1 with the SwiGLU epilogue -> quant -> fc2) at the token
counts of the FFN sweep config, M = 124,992 / P for P = 8, 4, 2, 1, stage by stage.  ``--cublas`` times cuBLASLt's FP8
GEMM (``torch._scaled_mm``, tensor-wise and row-wise scales, bf16 out) at the qkv and fc1 shapes as a library
reference point for the tcgen05 GEMM; it is not on the product path.
Inputs of the HBM-bound kernels exceed the 126 MB L2 at the default sizes, so no flush is needed between iterations.
"""
from __future__ import annotations

import argparse
import json
import math
from pathlib import Path

import torch

from . import _lib, ops

BF16, F16, E4M3 = torch.bfloat16, torch.float16, torch.float8_e4m3fn
HIDDEN, HEADS, D, FFN = 5120, 40, 128, 13824


def _peaks() -> dict:
    p = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    out = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}
    if p.exists():
        d = json.loads(p.read_text())
        for k in ("hbm_gbs", "bf16_tflops"):
            v = d.get(k)
            if isinstance(v, dict):
                v = v.get("value", v.get("median"))
            if isinstance(v, (int, float)):
                out[k] = float(v)
        out["source"] = "measured"
    return out


def _rand(shape, dtype, g, dev, scale=1.0):
    return (torch.randn(shape, generator=g, device=dev) * scale).to(dtype)


def _wq(n, k, g, dev):
    w = torch.randn(n, k, generator=g, device=dev) * 0.02
    s = torch.clamp(w.abs().amax(dim=1) / 448.0, min=1.0 / (448.0 * 512.0))
    return torch.clamp(w / s[:, None], -448.0, 448.0).to(E4M3), s


def _aq(m, k, g, dev):
    x = torch.randn(m, k, generator=g, device=dev)
    s = torch.clamp(x.abs().amax(dim=1) / 448.0, min=1.0 / (448.0 * 512.0))
    return torch.clamp(x / s[:, None], -448.0, 448.0).to(E4M3), s


def cases(M: int, dev):
    """(name, bound, work per launch, setup() -> run callable).  work: bytes for "hbm", FLOPs for "tensor"."""
    g = torch.Generator(device=dev).manual_seed(0)
    mf = max(M // 4, 1)          # the FFN and fp32 two-pass kernels run at a quarter of the rows (SP=4 share)
    out = []

    def add(name, bound, work, setup):
        out.append((name, bound, work, setup))

    def s_quant():
        x = _rand((M, HIDDEN), BF16, g, dev)
        return lambda: ops.quant(x)
    add("quant_rows_vec (x quant)", "hbm", 3 * M * HIDDEN + 4 * M, s_quant)

    def s_rms():
        x = _rand((M, HIDDEN), BF16, g, dev)
        w = _rand((HIDDEN,), BF16, g, dev)
        sh, sc = _rand((4, HIDDEN), BF16, g, dev, 0.1), _rand((4, HIDDEN), BF16, g, dev, 0.1)
        idx = torch.randint(0, 4, (M,), device=dev, generator=g)
        return lambda: ops.rms_quant(x, w, sh, sc, idx, 1e-6)
    add("rms_quant (norm + modulation + quant)", "hbm", 3 * M * HIDDEN + 4 * M, s_rms)

    def s_grms():
        r, b = _rand((M, HIDDEN), BF16, g, dev), _rand((M, HIDDEN), BF16, g, dev)
        gt, w = _rand((4, HIDDEN), BF16, g, dev, 0.1), _rand((HIDDEN,), BF16, g, dev)
        sh, sc = _rand((4, HIDDEN), BF16, g, dev, 0.1), _rand((4, HIDDEN), BF16, g, dev, 0.1)
        idx = torch.randint(0, 4, (M,), device=dev, generator=g)
        return lambda: ops.gate_rms_quant(r, gt, b, w, sh, sc, idx, 1e-6)
    add("gate_rms_quant (gated residual + norm + quant)", "hbm", 7 * M * HIDDEN + 4 * M, s_grms)

    def s_silu():
        x = _rand((mf, 2 * FFN), BF16, g, dev)
        return lambda: ops.silu_mul_quant(x)
    add("silu_mul_quant", "hbm", 5 * mf * FFN + 4 * mf, s_silu)

    def s_sbc():
        x32 = torch.randn(mf, HIDDEN, generator=g, device=dev)
        sa, sb = torch.rand(mf, device=dev, generator=g), torch.rand(HIDDEN, device=dev, generator=g)
        return lambda: ops.scale_bias_cast(x32, sa, sb, None, BF16)
    add("scale_bias_cast (two-pass scale pass)", "hbm", 6 * mf * HIDDEN, s_sbc)

    def s_sw():
        x32 = torch.randn(mf, 2 * FFN, generator=g, device=dev)
        sa, sb = torch.rand(mf, device=dev, generator=g), torch.rand(2 * FFN, device=dev, generator=g)
        return lambda: ops.scale_swiglu(x32, sa, sb, None)
    add("scale_swiglu (two-pass fc1 epilogue)", "hbm", 10 * mf * FFN, s_sw)

    def s_swq():
        x32 = torch.randn(mf, 2 * FFN, generator=g, device=dev)
        sa, sb = torch.rand(mf, device=dev, generator=g), torch.rand(2 * FFN, device=dev, generator=g)
        return lambda: ops.scale_swiglu_quant(x32, sa, sb, None)
    add("scale_swiglu_quant", "hbm", 9 * mf * FFN + 4 * mf, s_swq)

    def s_pack():
        x = _rand((M, HEADS, D), BF16, g, dev)
        return lambda: ops.pack_by_dest(x, 8)
    add("pack_by_dest (P = 8)", "hbm", 4 * M * HEADS * D, s_pack)

    def s_unpack():
        r = _rand((8, M // 8, HEADS // 8, D), BF16, g, dev)
        return lambda: ops.unpack_recv(r)
    add("unpack_recv (P = 8)", "hbm", 4 * (M // 8) * 8 * HEADS // 8 * D, s_unpack)

    def s_f16():
        x = _rand((M, HEADS, D), BF16, g, dev)
        return lambda: ops.bf16_to_f16(x)
    add("bf16_to_f16", "hbm", 4 * M * HEADS * D, s_f16)

    def s_rope():
        x = _rand((M, HEADS, D), BF16, g, dev)
        w = _rand((D,), BF16, g, dev)
        tab = torch.randn(M, 96, generator=g, device=dev)
        return lambda: ops.norm_rope_send(x, w, tab, 1e-6, 8)
    add("norm_rope_send (qk norm + RoPE into the send layout, P = 8)", "hbm", 4 * M * HEADS * D + 4 * M * 96,
        s_rope)

    def s_noalloc():
        s_kv, h = 16384, 8                      # the fixed scratch holds s_kv * heads <= 131,072
        q, k, v = (_rand((s_kv, h, D), BF16, g, dev) for _ in range(3))
        o = torch.empty_like(q)
        st = torch.cuda.current_stream(dev).cuda_stream

        def run():
            _lib.call("h3b_flash_attn_fwd_noalloc", q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(),
                      k.stride(0), k.stride(1), v.data_ptr(), v.stride(0), v.stride(1), o.data_ptr(), o.stride(0),
                      o.stride(1), s_kv, s_kv, -1, h, D, 1.0 / math.sqrt(D), st)
        return run
    add("flash_attn_noalloc (v -> f16 + attention, 16,384 x 8 heads)", "tensor", 4.0 * 16384 ** 2 * D * 8, s_noalloc)

    def s_qkv():
        a, sa = _aq(M, HIDDEN, g, dev)
        w, sb = _wq(3 * HEADS * D, HIDDEN, g, dev)
        return lambda: ops.fp8_gemm_qkv_send(a, w, sa, sb, HEADS, 8, v_f16=True)
    add("fp8_gemm qkv -> send layout (P = 8)", "tensor", 2.0 * M * 3 * HEADS * D * HIDDEN, s_qkv)

    def s_qkvn():
        a, sa = _aq(M, HIDDEN, g, dev)
        w, sb = _wq(3 * HEADS * D, HIDDEN, g, dev)
        qw, kw = _rand((D,), BF16, g, dev), _rand((D,), BF16, g, dev)
        tab = torch.randn(M, 96, generator=g, device=dev)
        return lambda: ops.fp8_gemm_qkv_send(a, w, sa, sb, HEADS, 8, v_f16=True, qk_norm=(qw, kw, tab, 1e-6))
    add("fp8_gemm qkv + qk norm + RoPE -> send layout (P = 8)", "tensor", 2.0 * M * 3 * HEADS * D * HIDDEN, s_qkvn)

    def s_fc1():
        a, sa = _aq(mf, HIDDEN, g, dev)
        w, sb = _wq(2 * FFN, HIDDEN, g, dev)
        return lambda: ops.fp8_gemm_swiglu(a, w, sa, sb)
    add("fp8_gemm fc1 + SwiGLU", "tensor", 2.0 * mf * 2 * FFN * HIDDEN, s_fc1)

    def s_fc2():
        a, sa = _aq(mf, FFN, g, dev)
        w, sb = _wq(HIDDEN, FFN, g, dev)
        x = _rand((mf, HIDDEN), BF16, g, dev)
        gate = _rand((4, HIDDEN), BF16, g, dev, 0.1)
        idx = torch.randint(0, 4, (mf,), device=dev, generator=g)
        return lambda: ops.fp8_gemm_gate(a, w, sa, sb, x, gate, idx)
    add("fp8_gemm fc2 + indexed gated residual", "tensor", 2.0 * mf * HIDDEN * FFN, s_fc2)

    def s_sig():
        flags = torch.zeros(8, dtype=torch.int32, device=dev)
        state = {"e": 0}
        st = torch.cuda.current_stream(dev).cuda_stream

        def run():
            state["e"] += 1
            ops.p2p_signal_wait([flags], flags, 0, state["e"], st)
        return run
    add("p2p signal_wait (one rank)", "latency", 0, s_sig)
    return out


def ffn_sweep(dev, iters: int) -> None:
    """FFN sweep: hidden 5120 -> gate/up 2 x 13,824 -> 5120, bf16 x ~ N(0,1), weights N(0, 0.02) quantised per output
    channel to e4m3, RMSNorm eps 1e-6; one line per M with each stage's CUDA-event time."""
    from .block import quant_weight  # noqa: PLC0415
    g = torch.Generator(device=dev).manual_seed(1)
    w1, s1 = quant_weight(torch.randn(2 * FFN, HIDDEN, device=dev, generator=g) * 0.02)
    w2, s2 = quant_weight(torch.randn(HIDDEN, FFN, device=dev, generator=g) * 0.02)
    nw = (1 + 0.1 * torch.randn(HIDDEN, device=dev, generator=g)).to(BF16)
    for M in (15_624, 31_248, 62_496, 124_992):
        x = torch.randn(M, HIDDEN, device=dev, generator=g).to(BF16)

        def stages():
            q, sq = ops.rms_quant(x, nw, eps=1e-6)
            yield
            h = ops.fp8_gemm_swiglu(q, w1, sq, s1)
            yield
            hq, sh = ops.quant(h)
            yield
            ops.fp8_gemm(hq, w2, sh, s2)
            yield

        for _ in range(3):
            for _ in stages():
                pass
        torch.cuda.synchronize()
        tot = [0.0] * 4
        for _ in range(iters):
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
            ev[0].record()
            for i, _ in enumerate(stages()):
                ev[i + 1].record()
            torch.cuda.synchronize()
            for i in range(4):
                tot[i] += ev[i].elapsed_time(ev[i + 1]) / iters
        fl1, fl2 = 2.0 * M * HIDDEN * 2 * FFN, 2.0 * M * FFN * HIDDEN
        print(json.dumps({"ffn_rows": M, "ms": round(sum(tot), 3), "rms_quant_ms": round(tot[0], 4),
                          "fc1_swiglu_ms": round(tot[1], 4), "quant_ms": round(tot[2], 4), "fc2_ms": round(tot[3], 4),
                          "fc1_tflops": round(fl1 / tot[1] / 1e9, 1), "fc2_tflops": round(fl2 / tot[3] / 1e9, 1),
                          "ffn_tflops": round((fl1 + fl2) / sum(tot) / 1e9, 1)}), flush=True)
        del x
        torch.cuda.empty_cache()


def cublas_reference(rows: int, dev, iters: int) -> None:
    """cuBLASLt FP8 at the qkv (rows x 15,360 x 5,120) and fc1 (rows/4 x 27,648 x 5,120) shapes: the device's library
    FP8 GEMM with tensor-wise scales (its fastest form) and with the row-wise scales this path needs."""
    g = torch.Generator(device=dev).manual_seed(0)
    for name, (M, N, K) in {"qkv": (rows, 3 * HEADS * D, HIDDEN), "fc1": (max(rows // 4, 1), 2 * FFN, HIDDEN)}.items():
        a = (torch.randn(M, K, device=dev, generator=g) * 0.5).to(E4M3)
        w = (torch.randn(N, K, device=dev, generator=g) * 0.5).to(E4M3)
        one = torch.ones((), device=dev)
        sa = torch.rand(M, 1, device=dev, generator=g) + 0.5
        sb = torch.rand(1, N, device=dev, generator=g) + 0.5
        for mode, (s_a, s_b) in {"tensorwise": (one, one), "rowwise": (sa, sb)}.items():
            def run():
                return torch._scaled_mm(a, w.t(), scale_a=s_a, scale_b=s_b, out_dtype=BF16)
            try:
                for _ in range(2):
                    run()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(iters):
                    run()
                e1.record()
                torch.cuda.synchronize()
                ms = e0.elapsed_time(e1) / iters
                print(json.dumps({"library_gemm": f"cuBLASLt FP8 {name}", "scales": mode, "ms": round(ms, 4),
                                  "tflops": round(2.0 * M * N * K / (ms * 1e-3) / 1e12, 1)}), flush=True)
            except RuntimeError as exc:  # a scaling mode this torch build does not offer
                print(json.dumps({"library_gemm": f"cuBLASLt FP8 {name}", "scales": mode, "error": str(exc)[:200]}))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=62496, help="token rows M (default: cfg2 at SP=2)")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--once", action="store_true", help="launch each kernel once (for an ncu launch capture)")
    ap.add_argument("--only", default="", help="comma-separated substrings of kernel names")
    ap.add_argument("--ffn", action="store_true", help="time the FFN sweep instead of the single kernels")
    ap.add_argument("--cublas", action="store_true", help="time cuBLASLt's FP8 GEMM at the qkv / fc1 shapes")
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if args.cublas:
        cublas_reference(args.rows, dev, args.iters)
        return
    if args.ffn:
        ffn_sweep(dev, args.iters)
        status = ops.device_status()
        if status != 0:
            raise SystemExit(f"device status {status}")
        return
    peaks = _peaks()
    only = [s.strip() for s in args.only.split(",") if s.strip()]
    for name, bound, work, setup in cases(args.rows, dev):
        if only and not any(s in name for s in only):
            continue
        run = setup()
        torch.cuda.synchronize()
        if args.once:
            run()
            torch.cuda.synchronize()
            continue
        for _ in range(2):
            run()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iters):
            run()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.iters
        line = {"kernel": name, "bound": bound, "ms": round(ms, 4)}
        if bound == "hbm":
            gbs = work / (ms * 1e-3) / 1e9
            line.update(gb_per_s=round(gbs, 1), frac_of_hbm=round(gbs / peaks["hbm_gbs"], 3))
        elif bound == "tensor":
            tf = work / (ms * 1e-3) / 1e12
            # FP8 against twice the measured dense bf16 rate (the e4m3 tensor rate is twice bf16's on B200)
            peak = peaks["bf16_tflops"] * (2.0 if "fp8_gemm" in name else 1.0)
            line.update(tflops=round(tf, 1), frac_of_tensor=round(tf / peak, 3))
        line["peaks"] = peaks["source"]
        print(json.dumps(line), flush=True)
        del run
        torch.cuda.empty_cache()
    status = ops.device_status()
    if status != 0:
        raise SystemExit(f"device status {status}")


if __name__ == "__main__":
    main()
