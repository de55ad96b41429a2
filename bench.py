"""Benchmark of the DiT attention block (BASELINE metric: ms per block and TFLOP/s at 124,992 tokens, SP=1/2/4/8).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl h3b|reference] [--tokens T]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU, NCCL over NVLink)

Workload: 124,992 tokens (31 x 48 x 84), hidden 5120, 40 heads x 128, B = 1, bf16 activations
x ~ N(0,1) (seed = rank), weights N(0, 0.02) quantised per output channel to e4m3 (seed 1), dynamic per-token e4m3
activation quant; Ulysses degree P = number of ranks (each rank holds 124,992 / P rows).  One step = one block
forward on every rank.  Inputs are larger than L2 (x is 1.28 GB / P, the attention streams 2.6 GB of K/V per head
group), so no explicit flush is needed.  Rank 0 prints one JSON line.

After the timed regions every rank checks its part of one more forward against the CPU oracle on 64 sampled rows
(``parity`` in the JSON line, the worst over ranks): the qkv projection rows it received from every rank, the
attention of its heads for those rows (the device's q against the device's K/V), the reverse exchange, and the whole block's output
rows through the oracle's attention, quant and out projection.  ``other_configs`` then runs BASELINE configs[1]
(66,960 tokens) and configs[3] (366,912 tokens) through the same block at this SP (3 timed steps each, 32 sampled
rows of parity per rank; ``--no-configs`` skips them).  Then the ``ffn`` section times BASELINE configs[4],
the block's FFN over the same M = 124,992 / SP rows per rank (RMSNorm + quant, fc1 with the SwiGLU epilogue, quant,
fc2; no communication), with its own sampled-row parity.

``--impl reference`` times the reference's CPU path for the same workload on the host cores (the oracle port of
h3_tp2's eager arithmetic: per-token quant, FP8 GEMM epilogue, fp32 SDPA) on a bounded per-head sample, as the
driver's reference arm; its ``ms_per_step`` is the measured sample time and ``block_ms_extrapolated`` the whole
block scaled from it.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "minimax-h3-2x-dgx-spark-tp2_b200"
for _p in (str(PKG), str(ROOT)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "DiT attn-block ms/layer & TFLOP/s at 125k tokens, SP=1/2/4/8 B200"
TOKENS, HIDDEN, HEADS, HEAD_DIM = 124_992, 5120, 40, 128


def block_flops(tokens: int, hidden: int = HIDDEN, heads: int = HEADS, d: int = HEAD_DIM) -> dict:
    hd = heads * d
    return {"attention": 4.0 * tokens * tokens * d * heads, "qkv": 2.0 * tokens * hidden * 3 * hd,
            "out": 2.0 * tokens * hd * hidden}


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return {"hbm_gbs": d["hbm_gbs"], "bf16": d["bf16_tflops"], "bf16_sustained": d["bf16_tflops_sustained"],
                    "sustained_sm_mhz": (d.get("clocks_under_load") or {}).get("sm_mhz_median"), "source": "measured"}
        except Exception:  # noqa: BLE001
            pass
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "sustained_sm_mhz": 1300.0,
            "source": "fallback"}


def clock_normalised(achieved: float, peak: float, peak_mhz, run_mhz) -> dict:
    """The roofline fraction with the peak moved to the kernel's own SM clock.  The sustained peak was measured at the
    median SM clock ``peak_mhz`` (a cuBLAS loop under the power cap) and tensor throughput scales with the clock, so
    against ``run_mhz`` (the median sampled over the timed region) the attainable rate is peak * run_mhz / peak_mhz."""
    if not peak_mhz or not run_mhz:
        return {"frac_at_run_clock": None, "peak_sm_mhz": peak_mhz, "run_sm_mhz": run_mhz}
    at_clock = peak * float(run_mhz) / float(peak_mhz)
    return {"frac_at_run_clock": achieved / at_clock, "peak_at_run_clock": at_clock, "peak_sm_mhz": peak_mhz,
            "run_sm_mhz": run_mhz}


class ClockSampler:
    """SM clock and throttle reasons of this rank's GPU, sampled every 10 ms through NVML while the timed region runs
    (read-only queries; falls back to `nvidia-smi -lms 50` when NVML is unavailable)."""

    def __init__(self, device: torch.device):
        self.device = device
        self.samples = []
        self.max_mhz = None
        self._stop = None
        self._thread = None
        self._proc = None

    def _nvml_handle(self):
        import pynvml  # noqa: PLC0415 (nvidia-ml-py)

        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(self.device)
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())

    def __enter__(self):
        import threading  # noqa: PLC0415

        try:
            nv, h = self._nvml_handle()
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            reasons_fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            self._stop = threading.Event()
            masks = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
                     "sw_power_cap": 0x4}

            def run():
                while not self._stop.is_set():
                    try:
                        mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                        r = reasons_fn(h)
                        self.samples.append((mhz, {k for k, m in masks.items() if r & m}))
                    except Exception:  # noqa: BLE001
                        pass
                    self._stop.wait(0.01)

            self._thread = threading.Thread(target=run, daemon=True)
            self._thread.start()
        except Exception:  # noqa: BLE001
            try:
                self._proc = subprocess.Popen(
                    ["nvidia-smi", "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
                     "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                     "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits", "-lms", "50",
                     "-i", str(self.device.index or 0)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            except (OSError, ValueError):
                self._proc = None
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
        if self._proc is not None:
            self._proc.terminate()
            try:
                out, _ = self._proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
                out, _ = self._proc.communicate()
            names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
            for line in (out or "").splitlines():
                parts = [x.strip() for x in line.split(",")]
                try:
                    mhz, self.max_mhz = float(parts[0]), float(parts[1])
                except (ValueError, IndexError):
                    continue
                self.samples.append((mhz, {n for n, v in zip(names, parts[2:]) if v.lower() in ("active", "1")}))

    def summary(self) -> dict:
        sm = [m for m, _ in self.samples]
        reasons = set().union(*[r for _, r in self.samples]) if self.samples else set()
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------------------------------------------
# CPU baseline (oracle port of the reference's eager path), bounded per-head sample scaled to the whole block
# ---------------------------------------------------------------------------------------------------------------


def cpu_sample(tokens: int, q_rows: int = 1024, threads: int | None = None) -> dict:
    """Time one head's attention for ``q_rows`` queries against all ``tokens`` keys (fp32 SDPA) plus that slice's
    share of the FP8 projections (per-token quant + the eager GEMM epilogue); the block figure scales it to 40 heads x
    all rows."""
    from oracle import attention as oa  # noqa: PLC0415
    from oracle import gemm as og  # noqa: PLC0415
    from oracle import quant as oq  # noqa: PLC0415

    if threads:
        torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    d = HEAD_DIM
    x = torch.randn(q_rows, HIDDEN, generator=g).to(torch.bfloat16)
    wq = og.quant_weight(torch.randn(3 * d, HIDDEN, generator=g) * 0.02)
    wo = og.quant_weight(torch.randn(HIDDEN, d, generator=g) * 0.02)
    k = torch.randn(tokens, 1, d, generator=g).to(torch.bfloat16)
    v = torch.randn(tokens, 1, d, generator=g).to(torch.bfloat16)
    t0 = time.perf_counter()
    q8, sx = oq.quant(x)                                  # the whole rows' quant, counted once per head (an
    qkv = og.scaled_mm(q8, wq[0], sx, wq[1])              # overestimate of this head's share of it)
    q = qkv[:, :d].reshape(q_rows, 1, d)
    t1 = time.perf_counter()
    o = oa.sdpa(q, k, v, chunk=256).to(torch.bfloat16)
    t2 = time.perf_counter()
    o8, so = oq.quant(o.reshape(q_rows, d))
    og.scaled_mm(o8, wo[0], so, wo[1])
    t3 = time.perf_counter()
    sample_s = t3 - t0
    scale = tokens / q_rows * HEADS
    # the sample's own work: one head of attention for q_rows rows + its projection share
    sample_fl = 4.0 * q_rows * tokens * d + 2.0 * q_rows * HIDDEN * 3 * d + 2.0 * q_rows * d * HIDDEN
    return {"seconds": sample_s, "block_seconds": sample_s * scale, "tflops": sample_fl / sample_s / 1e12,
            "attn_seconds": t2 - t1, "threads": torch.get_num_threads(),
            "sample": f"1 of {HEADS} heads, {q_rows} of {tokens} query rows vs all {tokens} keys (fp32 SDPA) + that "
                      f"slice's FP8 projection share; the block time scales it x{scale:.0f}"}


def _cfg0_worker(rank: int, ws: int, port: int, threads: int, reps: int, out: str) -> None:
    """One rank of BASELINE configs[0] (fp32, gloo): the reference's exact_forward data flow with fp32 projections
    (the oracle port, oracle.block.fp32_block), timed reps times after one warm-up."""
    import datetime  # noqa: PLC0415
    for pth in (str(PKG), str(ROOT)):
        if pth not in sys.path:
            sys.path.insert(0, pth)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.set_num_threads(threads)
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=120))
    try:
        from oracle import block as ob  # noqa: PLC0415
        g = torch.Generator().manual_seed(0)
        x = torch.randn(4096, 1024, generator=g)
        wqkv = torch.randn(3 * 1024, 1024, generator=g) * 0.02
        wo = torch.randn(1024, 1024, generator=g) * 0.02
        m = x.shape[0] // ws
        xl = x[rank * m:(rank + 1) * m].contiguous()

        def a2a(o, i):
            dist.all_to_all_single(o, i)

        times = []
        for it in range(reps + 1):
            dist.barrier()
            t0 = time.perf_counter()
            ob.fp32_block(xl, wqkv, wo, 8, ws, a2a)
            dist.barrier()
            if it:
                times.append(time.perf_counter() - t0)
        if rank == 0:
            Path(out).write_text(json.dumps(times))
    finally:
        dist.destroy_process_group()


def cpu_cfg0(cores: int, reps: int = 5) -> dict:
    """BASELINE configs[0] whole: 2 gloo processes x cores/2 threads, median of ``reps`` after one warm-up."""
    import socket  # noqa: PLC0415
    import tempfile  # noqa: PLC0415

    import torch.multiprocessing as mp  # noqa: PLC0415
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    per = max(1, cores // 2)
    with tempfile.TemporaryDirectory() as tmp:
        out = str(Path(tmp) / "t.json")
        mp.start_processes(_cfg0_worker, args=(2, port, per, reps, out), nprocs=2, start_method="spawn")
        times = json.loads(Path(out).read_text())
    return {"ms": statistics.median(times) * 1e3, "cores": 2 * per, "processes": 2, "reps": reps}


def cpu_cfg1_slice(cores: int) -> dict:
    """BASELINE configs[1] (66,960 tokens), one head: the whole head's fp32 SDPA (all queries, all keys) plus its share
    of the FP8 projections (quant of all rows, 3 x 128 qkv columns, 128 rows of the out projection), timed once; the
    block figure scales it x40 (all heads)."""
    from oracle import attention as oa  # noqa: PLC0415
    from oracle import gemm as og  # noqa: PLC0415
    from oracle import quant as oq  # noqa: PLC0415
    torch.set_num_threads(cores)
    n, d = 66_960, HEAD_DIM
    g = torch.Generator().manual_seed(0)
    x = torch.randn(n, HIDDEN, generator=g).to(torch.bfloat16)
    wq = og.quant_weight(torch.randn(3 * d, HIDDEN, generator=g) * 0.02)
    wo = og.quant_weight(torch.randn(HIDDEN, d, generator=g) * 0.02)
    t0 = time.perf_counter()
    q8, sx = oq.quant(x)
    qkv = og.scaled_mm(q8, wq[0], sx, wq[1]).reshape(n, 3, 1, d)
    o = oa.sdpa(qkv[:, 0], qkv[:, 1], qkv[:, 2], chunk=1024).to(torch.bfloat16)
    o8, so = oq.quant(o.reshape(n, d))
    og.scaled_mm(o8, wo[0], so, wo[1])
    sec = time.perf_counter() - t0
    return {"ms": sec * 1e3, "ms_scaled": sec * 1e3 * HEADS, "cores": cores,
            "sample": f"configs[1] one head of {HEADS}: all {n} queries x {n} keys fp32 SDPA + its projection share, "
                      f"scaled x{HEADS}"}


def config_dict(tokens: int, world: int) -> dict:
    """The workload both arms print (identical dicts: the reference arm runs the same configuration)."""
    return {"workload": f"cfg2 DiT attention block: {tokens} tokens (31x48x84), hidden {HIDDEN}, {HEADS} heads x "
                        f"{HEAD_DIM}, Ulysses SP={world}", "tokens": tokens, "rows_per_rank": tokens // world,
            "hidden": HIDDEN, "heads": HEADS, "head_dim": HEAD_DIM, "sp": world,
            "l2": "inputs larger than L2 (no flush)"}


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    tokens = args.tokens or TOKENS
    for _ in range(args.warmup):
        cpu_sample(tokens, q_rows=args.ref_rows, threads=threads)
    samples = [cpu_sample(tokens, q_rows=args.ref_rows, threads=threads) for _ in range(args.steps)]
    value = statistics.median(s["tflops"] for s in samples)
    step_ms = statistics.median(s["seconds"] for s in samples) * 1e3
    block_ms = statistics.median(s["block_seconds"] for s in samples) * 1e3
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp32 (CPU eager path)", "data": "synthetic",
            "config": config_dict(tokens, world),
            "step": "one bounded sample of the block (the cpu_baseline sample), timed on the host cores",
            "block_ms_extrapolated": block_ms,
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": samples[0]["threads"], "kind": "port",
                             "sample": samples[0]["sample"]},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------------------------
# parity at the benchmark's shape: sampled rows of one more forward against the CPU oracle, on every rank
# ---------------------------------------------------------------------------------------------------------------


def make_x(rank: int, m: int, dev) -> torch.Tensor:
    """Rank ``rank``'s input rows (any rank can regenerate any other's from its seed)."""
    g = torch.Generator(device=dev).manual_seed(rank)
    return torch.randn(m, HIDDEN, device=dev, generator=g).to(torch.bfloat16)


def block_parity(blk, keep: dict, rank: int, world: int, m: int, dev, pg, rows: int = 64) -> dict:
    """This rank's share of the block at ``rows`` sampled local rows (the same rows on every rank), against the CPU
    oracle (oracle.quant / oracle.gemm / oracle.attention):
      qkv       the q/k/v rows this rank received from every rank (its head group's columns) against the oracle's
                quant + FP8 projection of those ranks' inputs (regenerated from their seeds);
      attention every rank's oracle attention for its head group at those query rows (the device's q rows against
                the device's K/V of all tokens, so that this stage measures the attention alone), exchanged back,
                against this rank's reverse receive buffer;
      out       the device's y rows against the oracle's quant + out projection of the device's reverse buffer rows;
      block     the device's y rows against the oracle's quant + out projection of the oracle's attention rows.
    Thresholds: GEMM-based stages rel-L2 <= 1e-2 (the FP8 GEMM contract); attention rel-L2 <= 2e-3 and max-abs <=
    2e-2 after dividing each column by max(1, its largest |ref|), as the attention tests measure it (the raw max-abs
    is reported beside it); block rel-L2 <= 1e-2."""
    from oracle import attention as oa  # noqa: PLC0415
    from oracle import gemm as og  # noqa: PLC0415
    from oracle import quant as oq  # noqa: PLC0415

    def rel(a, b):
        a, b = a.double(), b.double()
        return float((a - b).norm() / b.norm().clamp_min(1e-300))

    H, d = HEADS, HEAD_DIM
    hl = H // world
    idx = torch.linspace(0, m - 1, rows).round().long()
    idx_d = idx.to(dev)
    xs = torch.stack([make_x(p, m, dev)[idx_d].cpu() for p in range(world)])            # [P, R, C]
    cols = torch.cat([torch.arange(w * H * d + rank * hl * d, w * H * d + (rank + 1) * hl * d) for w in range(3)])
    wq8, sq = blk.wqkv8[cols.to(dev)].cpu(), blk.sqkv[cols.to(dev)].cpu()
    q8, sx = oq.quant(xs.reshape(world * rows, HIDDEN))
    qkv = og.scaled_mm(q8, wq8, sx, sq).reshape(world * rows, 3, hl, d)                 # bf16
    tok = (torch.arange(world)[:, None] * m + idx[None, :]).reshape(-1).to(dev)         # [P*R] gathered rows
    got = torch.stack([keep[n][tok].float().cpu() for n in ("q", "k", "v")], dim=1)
    r_qkv = rel(got, qkv.float())
    # oracle attention of this rank's heads for all P*R sampled tokens, against the device's K/V (one head at a time)
    o_or = torch.empty(world * rows, hl, d)
    for h in range(hl):
        kh = keep["k"][:, h:h + 1].contiguous().cpu()
        vh = keep["v"][:, h:h + 1].contiguous().cpu()
        o_or[:, h:h + 1] = oa.sdpa(got[:, 0, h:h + 1].to(torch.bfloat16), kh, vh, chunk=world * rows)
    o_or = o_or.reshape(world, rows, hl, d)                                              # [dest rank, R, hl, d]
    if world > 1:
        recv = torch.empty_like(o_or, device=dev)
        dist.all_to_all_single(recv, o_or.to(dev).contiguous(), group=pg)
        attn_or = recv.cpu()                                                             # [head group, R, hl, d]
    else:
        attn_or = o_or
    back = keep["back"][:, idx_d].float().cpu()                                          # [head group, R, hl, d]
    r_attn = rel(back, attn_or)
    err = (back - attn_or).abs()
    a_attn = float(err.max())
    worst = int(err.argmax())
    # the attention tests' max-abs measure: each column's error over max(1, that column's largest |ref|)
    colscale = attn_or.abs().amax(dim=1, keepdim=True).clamp_min(1.0)
    s_attn = float((err / colscale).max())
    w_ref, w_got = float(attn_or.reshape(-1)[worst]), float(back.reshape(-1)[worst])
    wo8, so_w = blk.wo8.cpu(), blk.so.cpu()
    y = keep["y"][idx_d].float().cpu()
    ob8, obs = oq.quant(back.permute(1, 0, 2, 3).reshape(rows, H * d).to(torch.bfloat16))
    r_out = rel(y, og.scaled_mm(ob8, wo8, obs, so_w).float())
    oa8, oas = oq.quant(attn_or.permute(1, 0, 2, 3).reshape(rows, H * d).to(torch.bfloat16))
    r_block = rel(y, og.scaled_mm(oa8, wo8, oas, so_w).float())
    print(f"[rank {rank}] attention parity: worst |err| {a_attn:.4g} at ref {w_ref:.4g} (got {w_got:.4g}), "
          f"column-scaled {s_attn:.4g}", file=sys.stderr, flush=True)
    vals = [r_qkv, r_attn, a_attn, r_out, r_block, s_attn]
    if world > 1:
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=pg)
        vals = t.tolist()
    r_qkv, r_attn, a_attn, r_out, r_block, s_attn = vals
    ok = r_qkv <= 1e-2 and r_attn <= 2e-3 and s_attn <= 2e-2 and r_out <= 1e-2 and r_block <= 1e-2
    return {"rows": rows, "tokens_checked": rows * world, "rel_l2": {"qkv": r_qkv, "attention": r_attn,
            "out": r_out, "block": r_block}, "max_abs": {"attention": a_attn},
            "max_abs_colscaled": {"attention": s_attn},
            "tolerance": {"qkv": 1e-2, "attention": [2e-3, 2e-2], "out": 1e-2, "block": 1e-2},
            "oracle": "oracle.quant + oracle.gemm + oracle.attention (fp32 SDPA) on the CPU", "ok": bool(ok)}


# ---------------------------------------------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------------------------------------------


FFN = 13_824   # hidden 5120 -> gate/up 2 x 13,824 -> 5120


def ffn_flops(m: int) -> float:
    return 2.0 * m * HIDDEN * 2 * FFN + 2.0 * m * FFN * HIDDEN


def ffn_weights(dev):
    """The cfg4 FFN's weights (seed 2): W1 [2F, C] (gate rows, then up rows) and W2 [C, F] ~ N(0, 0.02), quantised per
    output channel to e4m3, and the RMSNorm weight (bf16, around 1)."""
    from h3b.block import quant_weight  # noqa: PLC0415
    g = torch.Generator(device=dev).manual_seed(2)
    w1 = torch.randn(2 * FFN, HIDDEN, device=dev, generator=g) * 0.02
    w2 = torch.randn(HIDDEN, FFN, device=dev, generator=g) * 0.02
    norm_w = (1.0 + 0.1 * torch.randn(HIDDEN, device=dev, generator=g)).to(torch.bfloat16)
    return (norm_w, *quant_weight(w1), *quant_weight(w2))


FFN_STAGES = ("rms_quant", "fc1_swiglu", "quant_h", "fc2")


def ffn_forward(x, norm_w, w1, s1, w2, s2, marks=None, keep=None):
    """RMSNorm (eps 1e-6) + per-token quant -> fc1 with the SwiGLU epilogue -> per-token quant -> fc2 (the torch ops
    the plugin's MLP path calls); ``marks`` gets a CUDA event before and after each stage."""
    def mark():
        if marks is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            marks.append(ev)
    mark()
    q, sq = torch.ops.h3b.rms_quant(x, norm_w, None, None, None, 1e-6, None)
    mark()
    h = torch.ops.h3b.fp8_gemm_swiglu(q, w1, sq, s1, None)
    mark()
    hq, sh = torch.ops.h3b.quant(h)
    mark()
    y = torch.ops.h3b.fp8_gemm(hq, w2, sh, s2, None, torch.bfloat16)
    mark()
    if keep is not None:
        keep.update(h=h, y=y)
    return y


def ffn_parity(x, weights, keep, rows: int = 64) -> dict:
    """The FFN's sampled rows against the CPU oracle: the SwiGLU output h (the fc1 GEMM with its epilogue; CUDA's expf
    against torch's exp) and the FFN output y.  Threshold rel-L2 <= 1e-2 (the FP8 GEMM contract) for both."""
    from oracle import gemm as og  # noqa: PLC0415
    from oracle import quant as oq  # noqa: PLC0415
    from oracle import rms as orms  # noqa: PLC0415
    norm_w, w1, s1, w2, s2 = (t.cpu() for t in weights)
    idx = torch.linspace(0, x.shape[0] - 1, rows).round().long()
    xr = x[idx.to(x.device)].cpu()
    q, sq = orms.rms_quant(xr, norm_w, eps=1e-6)
    h = og.swiglu_epilogue(og.accumulate(q, w1), sq, s1, None)
    hq, sh = oq.quant(h)
    y = og.scaled_mm(hq, w2, sh, s2)

    def rel(a, b):
        a, b = a.double(), b.double()
        return float((a - b).norm() / b.norm().clamp_min(1e-300))
    r_h = rel(keep["h"][idx.to(x.device)].float().cpu(), h.float())
    r_y = rel(keep["y"][idx.to(x.device)].float().cpu(), y.float())
    return {"rows": rows, "rel_l2": {"swiglu_h": r_h, "ffn_y": r_y}, "tolerance": 1e-2,
            "ok": bool(r_h <= 1e-2 and r_y <= 1e-2)}


def run_ffn(args, rank: int, world: int, dev, pg, m: int) -> dict:
    """BASELINE configs[4] at this SP: the FFN over this rank's M = 124,992 / SP rows (replicas: the FFN is row-local,
    no communication), device-timed over --steps steps after --warmup, the worst rank's time."""
    from h3b import ops  # noqa: PLC0415
    weights = ffn_weights(dev)
    x = make_x(rank, m, dev)
    for _ in range(args.warmup):
        ffn_forward(x, *weights)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier(group=pg, device_ids=[dev.index])
    marks_all = []
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        marks = []
        ffn_forward(x, *weights, marks=marks)
        marks_all.append(marks)
    end.record()
    torch.cuda.synchronize(dev)
    vals = [start.elapsed_time(end) / args.steps] + [
        statistics.mean(mk[i].elapsed_time(mk[i + 1]) for mk in marks_all) for i in range(len(FFN_STAGES))]
    if world > 1:
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=pg)
        vals = t.tolist()
    ms = vals[0]
    keep = {}
    ffn_forward(x, *weights, keep=keep)
    torch.cuda.synchronize(dev)
    status = ops.device_status()
    if status != 0:
        raise RuntimeError(f"device status {status} in the FFN")
    par = ffn_parity(x, weights, keep)
    if world > 1:
        t = torch.tensor([par["rel_l2"]["swiglu_h"], par["rel_l2"]["ffn_y"]], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=pg)
        par["rel_l2"] = {"swiglu_h": t[0].item(), "ffn_y": t[1].item()}
        par["ok"] = bool(t.max().item() <= 1e-2)
    fl = ffn_flops(m)
    return {"workload": f"cfg4 FFN: M = {m} rows per rank (124,992 / SP), hidden {HIDDEN} -> 2 x {FFN} -> {HIDDEN}, "
                        "RMSNorm eps 1e-6 + per-token e4m3 quant, fc1 with the SwiGLU epilogue, quant, fc2",
            "rows_per_rank": m, "ms_per_step": ms, "tflops": world * fl / (ms * 1e-3) / 1e12,
            "tflops_per_gpu": fl / (ms * 1e-3) / 1e12, "ms_per_stage": dict(zip(FFN_STAGES, vals[1:])),
            "scaling": "weak (replicas: no communication)", "parity": par}


OTHER_CONFIGS = (("cfg1", 66_960, "31x36x60"), ("cfg3", 366_912, "91x48x84"))


def run_configs(args, blk, rank: int, world: int, dev, pg) -> list:
    """BASELINE configs[1] and configs[3] through the same block at this SP: device-timed ms per block over 3 steps
    after 2 warm-up forwards (the worst rank's time), and the sampled-row parity of one more forward against the CPU
    oracle (32 rows per rank)."""
    from h3b import ops  # noqa: PLC0415
    out = []
    for name, tokens, grid in OTHER_CONFIGS:
        if tokens % world:
            continue
        m = tokens // world
        x = make_x(rank, m, dev)
        for _ in range(2):
            blk(x)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier(group=pg, device_ids=[dev.index])
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(3):
            blk(x)
        e1.record()
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / 3
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=pg)
            ms = t.item()
        keep = {}
        blk.forward(x, keep=keep)
        torch.cuda.synchronize(dev)
        status = ops.device_status()
        if status != 0:
            raise RuntimeError(f"device status {status} in {name}")
        par = block_parity(blk, keep, rank, world, m, dev, pg, rows=32)
        del keep, x
        fl = sum(block_flops(tokens).values())
        out.append({"config": f"{name}: {tokens} tokens ({grid}), SP={world}", "tokens": tokens, "rows_per_rank": m,
                    "ms_per_block": ms, "tflops": fl / (ms * 1e-3) / 1e12, "steps": 3, "warmup": 2,
                    "parity_ok": par["ok"], "parity_rel_l2": par["rel_l2"]})
    return out


def run_h3b(args, rank: int, world: int, local_rank: int, pg) -> None:
    import h3b  # noqa: PLC0415
    from h3b.block import AttentionBlock  # noqa: PLC0415

    h3b.load_library()
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    tokens = args.tokens or TOKENS
    if tokens % world:
        raise SystemExit(f"tokens {tokens} not divisible by {world} ranks")
    m = tokens // world
    p2p = args.exchange == "p2p" and world > 1
    exchange = args.exchange if world > 1 else "nccl"
    if p2p:
        from h3b.ulysses_p2p import probe  # noqa: PLC0415
        ok, why = probe(pg, dev)
        if not ok:   # every rank agreed: take the collective path instead, and say so in the JSON line
            print(f"bench.py: peer memory unavailable ({why}); NCCL exchange instead", file=sys.stderr)
            p2p, exchange = False, "nccl"
            args.exchange = "nccl"
    blk = AttentionBlock(HIDDEN, HEADS, device=dev, ws=world, pg=pg, init_device=dev, seed=1,
                         groups=1 if p2p else (args.groups or None), exchange=exchange)
    try:
        _timed(args, blk, rank, world, local_rank, pg, dev, tokens, m, p2p)
    finally:
        blk.close()


def _timed(args, blk, rank, world, local_rank, pg, dev, tokens, m, p2p) -> None:
    from h3b import ops  # noqa: PLC0415

    x = make_x(rank, m, dev)

    def barrier():
        if world > 1:
            dist.barrier(group=pg, device_ids=[local_rank])
        torch.cuda.synchronize(dev)

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=pg)
        return float(t.item())

    for _ in range(args.warmup):
        blk(x)
    barrier()
    status = ops.device_status()
    if status != 0:
        raise RuntimeError(f"device status {status} after warm-up")

    # ---- device-timed region: K steps, inputs resident in HBM ----
    marks_all = []
    with ClockSampler(dev) as clocks:
        barrier()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            marks = []
            blk.forward(x, marks=marks)
            marks_all.append(marks)
        end.record()
        barrier()
    ms = start.elapsed_time(end) / args.steps
    ms = max_over_ranks(ms)
    stage_ms = {}
    for i, name in enumerate(blk.STAGES):
        vals = [mk[i].elapsed_time(mk[i + 1]) for mk in marks_all]
        stage_ms[name] = max_over_ranks(statistics.mean(vals))
    status = ops.device_status()
    if status != 0:
        raise RuntimeError(f"device status {status} in the timed region")

    # ---- end to end through the public API: every step copies its x from pinned host memory to the device and
    # reads its y back to pinned host memory.  The copies run on a side stream: step i+1's input and step i-1's output
    # cross PCIe while step i's block computes (two device input buffers, two host output buffers). ----
    hx = x.cpu().pin_memory()
    hy = [torch.empty((m, HIDDEN), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    xd = [torch.empty_like(x) for _ in range(2)]
    comp = torch.cuda.current_stream(dev)
    copy = torch.cuda.Stream(dev)
    blk(hx.to(dev, non_blocking=True))
    barrier()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    copy.wait_stream(comp)
    with torch.cuda.stream(copy):
        xd[0].copy_(hx, non_blocking=True)
        ev_in[0].record(copy)
    for i in range(args.steps):
        if i + 1 < args.steps:
            with torch.cuda.stream(copy):
                if i >= 1:
                    copy.wait_event(ev_used[(i + 1) % 2])   # step i-1 is done with that buffer
                xd[(i + 1) % 2].copy_(hx, non_blocking=True)
                ev_in[(i + 1) % 2].record(copy)
        comp.wait_event(ev_in[i % 2])
        y = blk(xd[i % 2])
        ev_used[i % 2].record(comp)
        copy.wait_stream(comp)
        with torch.cuda.stream(copy):
            y.record_stream(copy)
            hy[i % 2].copy_(y, non_blocking=True)
    comp.wait_stream(copy)
    e1.record(comp)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)

    fl = block_flops(tokens)
    total_fl = sum(fl.values())
    value = total_fl / (ms * 1e-3) / 1e12
    peaks = measured_peaks()
    attn_ms = stage_ms["attention"]
    attn_fl_per_launch = fl["attention"] / world
    achieved = attn_fl_per_launch / (attn_ms * 1e-3) / 1e12
    peak = peaks["bf16_sustained"]
    clk = clocks.summary()
    # ---- parity: one more forward, its sampled rows against the CPU oracle on every rank (outside the timings) ----
    keep = {}
    blk.forward(x, keep=keep)
    torch.cuda.synchronize(dev)
    status = ops.device_status()
    if status != 0:
        raise RuntimeError(f"device status {status} in the parity forward")
    if world > 1:
        torch.set_num_threads(max(1, (os.cpu_count() or 1) // world))
    parity = block_parity(blk, keep, rank, world, m, dev, pg)
    del keep
    configs = None if args.no_configs else run_configs(args, blk, rank, world, dev, pg)
    ffn = None if args.no_ffn else run_ffn(args, rank, world, dev, pg, m)

    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "e4m3 projections (f32 acc), bf16 attention (f16 P.V, f32 softmax)",
        "data": "synthetic", "config": config_dict(tokens, world),
        "exchange": {"p2p": "peer memory (epilogue stores over NVLink + epoch barriers)",
                     "nccl": "NCCL all_to_all_single (q, k, v, out)",
                     "nocopy": "NCCL all_to_all_single (combined q/k/v per head group, out)"}[args.exchange]
                    if world > 1 else "none (SP=1)",
        "head_groups": blk.groups,
        "ms_per_stage": stage_ms,
        "roofline": {"bound": "tensor", "kernel": "flash_attn", "achieved": achieved, "peak": peak,
                     "unit": "TFLOP/s", "frac": achieved / peak,
                     "peak_source": f"{peaks['source']} bf16 dense, sustained (kernel timed inside a long step)",
                     "traffic": None,
                     "traffic_source": "not measured by this run (DRAM bytes need an ncu capture; the committed "
                                       "profiles hold them)",
                     **clock_normalised(achieved, peak, peaks.get("sustained_sm_mhz"), clk.get("sm_mhz"))},
        "e2e": {"value": total_fl / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": m * HIDDEN * 2, "d2h_bytes_per_step": m * HIDDEN * 2},
        "gpu_launches": (blk.KERNELS_PER_FORWARD + (blk.P2P_BARRIERS if p2p else 0)) * args.steps,
        "clocks": clk,
        "parity": parity,
    }
    if configs is not None:
        line["other_configs"] = configs
    if ffn is not None:
        line["ffn"] = ffn
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cores = os.cpu_count() or 1
        cpu_sample(tokens, q_rows=256, threads=cores)            # warm-up (thread pool, page faults)
        cbs = [cpu_sample(tokens, q_rows=args.ref_rows, threads=cores) for _ in range(3)]
        c0 = cpu_cfg0(cores)
        c1 = cpu_cfg1_slice(cores)
        line["cpu_baseline"] = {
            "value": statistics.median(c["tflops"] for c in cbs), "unit": "TFLOP/s", "cores": cbs[0]["threads"],
            "kind": "port", "sample": cbs[0]["sample"] + " (median of 3 after a warm-up)",
            "ms_per_block": statistics.median(c["block_seconds"] for c in cbs) * 1e3,
            "cfg0_ms": c0["ms"], "cfg0_cores": c0["cores"],
            "cfg0": f"configs[0] whole: 4096 tokens, hidden 1024, 8 x 128, fp32, 2 gloo processes x "
                    f"{c0['cores'] // 2} threads, median of {c0['reps']} after 1 warm-up",
            "cfg1_slice_ms": c1["ms"], "cfg1_slice_ms_scaled": c1["ms_scaled"], "cfg1_cores": c1["cores"],
            "cfg1": c1["sample"]}
    if rank == 0:
        print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    # 10 steps: the end-to-end loop's first input copy and last output copy (no block to overlap them with) weigh
    # 1/10 of a step each instead of 1/5
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("h3b", "reference"), default="h3b")
    ap.add_argument("--tokens", type=int, default=0, help="override the token count (tests / small runs)")
    ap.add_argument("--ref-rows", type=int, default=1024, help="query rows of the CPU sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ffn", action="store_true", help="skip the cfg4 FFN section of the JSON line")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the cfg1 / cfg3 block timings (other_configs) of the JSON line")
    ap.add_argument("--groups", type=int, default=0,
                    help="Ulysses head groups overlapped with attention (NCCL exchange; 0: the measured default)")
    ap.add_argument("--exchange", choices=("nccl", "nocopy", "p2p"), default="p2p",
                    help="Ulysses exchange at SP > 1: NCCL all-to-alls (three per block, or one combined q/k/v "
                         "exchange with nocopy), or the kernels' stores into peer memory")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"bench.py: WORLD_SIZE {world} != --gpus {args.gpus}", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if not torch.cuda.is_available():
        raise SystemExit("bench.py: the h3b arm needs a CUDA GPU (there is no CPU fallback); --impl reference times "
                         "the CPU path")
    pg = None
    if world > 1:
        import datetime  # noqa: PLC0415
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))
        pg = dist.group.WORLD
    try:
        run_h3b(args, rank, world, local_rank, pg)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
