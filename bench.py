"""Benchmark of the DiT attention block (BASELINE metric: ms per block and TFLOP/s at 124,992 tokens, SP=1/2/4/8).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl h3b|reference] [--tokens T]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU, NCCL over NVLink)

Workload: 124,992 tokens (31 x 48 x 84), hidden 5120, 40 heads x 128, B = 1, bf16 activations
x ~ N(0,1) (seed 0 + rank), weights N(0, 0.02) quantised per output channel to e4m3 (seed 1), dynamic per-token e4m3
activation quant; Ulysses degree P = number of ranks (each rank holds 124,992 / P rows).  One step = one block
forward on every rank.  Inputs are larger than L2 (x is 1.28 GB / P, the attention streams 2.6 GB of K/V per head
group), so no explicit flush is needed.  Rank 0 prints one JSON line.

``--impl reference`` times the reference's CPU path for the same workload on the host cores (the oracle port of
h3_tp2's eager arithmetic: per-token quant, FP8 GEMM epilogue, fp32 SDPA) on a bounded per-head sample scaled to the
whole block, as the driver's reference arm.
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
                    "source": "measured"}
        except Exception:  # noqa: BLE001
            pass
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


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
    share of the FP8 projections (per-token quant + the eager GEMM epilogue), then scale to 40 heads x all rows."""
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
    q8, sx = oq.quant(x)                                  # the whole row's quant (shared by all heads; counted once
    qkv = og.scaled_mm(q8, wq[0], sx, wq[1])              # per head below as 1/40 of it is an underestimate: keep)
    q = qkv[:, :d].reshape(q_rows, 1, d)
    t1 = time.perf_counter()
    o = oa.sdpa(q, k, v, chunk=256).to(torch.bfloat16)
    t2 = time.perf_counter()
    o8, so = oq.quant(o.reshape(q_rows, d))
    og.scaled_mm(o8, wo[0], so, wo[1])
    t3 = time.perf_counter()
    scale_rows = tokens / q_rows
    proj_s = ((t1 - t0) + (t3 - t2)) * scale_rows * HEADS
    attn_s = (t2 - t1) * scale_rows * HEADS
    total_s = proj_s + attn_s
    fl = sum(block_flops(tokens).values())
    return {"seconds_per_block": total_s, "tflops": fl / total_s / 1e12, "sample_seconds": t3 - t0,
            "threads": torch.get_num_threads(),
            "sample": f"1 of {HEADS} heads, {q_rows} of {tokens} query rows vs all {tokens} keys (fp32 SDPA) + that "
                      f"slice's FP8 projection share; scaled x{scale_rows * HEADS:.0f}"}


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    tokens = args.tokens or TOKENS
    for _ in range(args.warmup):
        cpu_sample(tokens, q_rows=256, threads=threads)
    samples = [cpu_sample(tokens, q_rows=args.ref_rows, threads=threads) for _ in range(args.steps)]
    sec = statistics.median(s["seconds_per_block"] for s in samples)
    fl = sum(block_flops(tokens).values())
    value = fl / sec / 1e12
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp32 (CPU eager path)", "data": "synthetic",
            "config": {"workload": f"cfg2 DiT attention block, {tokens} tokens, hidden {HIDDEN}, {HEADS}x{HEAD_DIM}",
                       "tokens": tokens, "sp": world},
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": samples[0]["threads"], "kind": "port",
                             "sample": samples[0]["sample"]},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------------------------------------------


# DRAM bytes (read + write) of one attention launch at cfg2 SP=1, from the ncu launch list of this bench
ATTN_TRAFFIC_BYTES = 33.82e9


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

    g = torch.Generator(device=dev).manual_seed(rank)
    x = torch.randn(m, HIDDEN, device=dev, generator=g).to(torch.bfloat16)

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
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "e4m3 projections (f32 acc), bf16 attention (f16 P.V, f32 softmax)",
        "data": "synthetic",
        "config": {"workload": f"cfg2 DiT attention block: {tokens} tokens (31x48x84), hidden {HIDDEN}, "
                               f"{HEADS} heads x {HEAD_DIM}, Ulysses SP={world}", "tokens": tokens,
                   "rows_per_rank": m, "hidden": HIDDEN, "heads": HEADS, "head_dim": HEAD_DIM, "sp": world,
                   "head_groups": blk.groups, "l2": "inputs larger than L2 (no flush)",
                   "exchange": {"p2p": "peer memory (epilogue stores over NVLink + epoch barriers)",
                                "nccl": "NCCL all_to_all_single (q, k, v, out)",
                                "nocopy": "NCCL all_to_all_single (combined q/k/v per head group, out)"}[args.exchange]
                               if world > 1 else "none (SP=1)"},
        "ms_per_stage": stage_ms,
        "roofline": {"bound": "tensor", "kernel": "flash_attn", "achieved": achieved, "peak": peak,
                     "unit": "TFLOP/s", "frac": achieved / peak,
                     "peak_source": f"{peaks['source']} bf16 dense, sustained (kernel timed inside a long step)",
                     "traffic": ATTN_TRAFFIC_BYTES if (world == 1 and tokens == TOKENS) else None,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one attention launch "
                                       "in the launch-list capture of this bench at cfg2 SP=1"},
        "e2e": {"value": total_fl / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": m * HIDDEN * 2, "d2h_bytes_per_step": m * HIDDEN * 2},
        "gpu_launches": (blk.KERNELS_PER_FORWARD + (blk.P2P_BARRIERS if p2p else 0)) * args.steps,
        "clocks": clocks.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = cpu_sample(tokens, q_rows=args.ref_rows, threads=os.cpu_count())
        line["cpu_baseline"] = {"value": cb["tflops"], "unit": "TFLOP/s", "cores": cb["threads"], "kind": "port",
                                "sample": cb["sample"], "ms_per_block": cb["seconds_per_block"] * 1e3}
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
