"""bench.py's JSON contract on the CPU: the reference arm prints one line with every key the driver reads, and the
h3b arm refuses to run without a GPU (no CPU fallback)."""
import json
import subprocess
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

ROOT = Path(__file__).resolve().parents[1]
KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config"}


def _run(*args, timeout=300):
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                          timeout=timeout, cwd=ROOT)


def test_reference_arm_prints_the_driver_line():
    res = _run("--impl", "reference", "--tokens", "4096", "--steps", "2", "--warmup", "1", "--ref-rows", "64")
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert KEYS <= d.keys() and d["impl"] == "reference"
    assert d["steps"] == 2 and d["warmup"] == 1 and d["n_gpus"] == 1 and d["higher_is_better"] is True
    assert d["value"] > 0 and d["unit"] == "TFLOP/s" and d["config"]["tokens"] == 4096
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_gpu_arm_fails_loudly_without_a_gpu():
    if torch.cuda.is_available():
        return
    res = _run("--tokens", "4096", "--steps", "1", "--warmup", "1", "--no-cpu-baseline")
    assert res.returncode != 0
    assert not [ln for ln in res.stdout.splitlines() if ln.startswith("{")]


def test_reference_arm_times_the_sample_it_ran():
    """ms_per_step is the measured sample time (it must fit in the run), the whole-block figure is a separate,
    labelled extrapolation, and the config dict is the GPU arm's (same workload)."""
    import bench
    res = _run("--impl", "reference", "--tokens", "4096", "--steps", "3", "--warmup", "1", "--ref-rows", "64")
    d = json.loads([ln for ln in res.stdout.splitlines() if ln.startswith("{")][0])
    assert d["ms_per_step"] * d["steps"] < 60_000
    assert d["block_ms_extrapolated"] > d["ms_per_step"]
    assert d["config"] == bench.config_dict(4096, 1)


def _fake_block_run(m, world_rows=None, plant=None):
    """The GPU arm's parity inputs built on the CPU from the oracle (rank 0 of 1): weights, x from bench.make_x, and
    the forward's kept tensors as the oracle computes them; ``plant`` corrupts one of them."""
    import bench
    from oracle import attention as oa
    from oracle import block as ob
    from oracle import gemm as og
    from oracle import quant as oq
    H, d, C = bench.HEADS, bench.HEAD_DIM, bench.HIDDEN
    wqkv8, sqkv, wo8, so = ob.make_weights(C, H, seed=1)
    blk = type("Blk", (), {"wqkv8": wqkv8, "sqkv": sqkv, "wo8": wo8, "so": so})()
    x = bench.make_x(0, m, torch.device("cpu"))
    q8, sx = oq.quant(x)
    qkv = og.scaled_mm(q8, wqkv8, sx, sqkv)
    q, k, v = (t.reshape(m, H, d) for t in qkv.split(H * d, dim=1))
    o = oa.sdpa(q, k, v).to(torch.bfloat16)
    o8, so_ = oq.quant(o.reshape(m, H * d))
    y = og.scaled_mm(o8, wo8, so_, so)
    keep = {"q": q, "k": k, "v": v, "back": o.reshape(1, m, H, d), "y": y}
    if plant is not None:
        plant(keep)
    return blk, keep


def test_block_parity_passes_on_oracle_data_and_catches_a_planted_error():
    import bench
    m = 192
    blk, keep = _fake_block_run(m)
    par = bench.block_parity(blk, keep, 0, 1, m, torch.device("cpu"), None, rows=16)
    assert par["ok"], par
    # the kept attention rows are bf16 (the oracle's fp32 rows rounded): that rounding is all that differs
    assert par["rel_l2"]["attention"] < 2e-3 and par["rel_l2"]["block"] < 1e-6 and par["rel_l2"]["qkv"] == 0

    def plant(keep):   # one value of the kept K: every sampled query row's attention moves
        keep["k"][5, 3] += 40.0
    blk, keep = _fake_block_run(m, plant=plant)
    par = bench.block_parity(blk, keep, 0, 1, m, torch.device("cpu"), None, rows=16)
    assert not par["ok"]

    def plant_y(keep):  # one output row of the block
        keep["y"][0] *= 1.5
    blk, keep = _fake_block_run(m, plant=plant_y)
    par = bench.block_parity(blk, keep, 0, 1, m, torch.device("cpu"), None, rows=16)
    assert not par["ok"] and par["rel_l2"]["out"] > 1e-2


def test_ffn_parity_passes_on_oracle_data_and_catches_a_planted_error():
    """The FFN section's parity check, fed the oracle's own h and y (built on the CPU), passes; one changed output row
    fails it."""
    import bench
    from oracle import gemm as og
    from oracle import quant as oq
    from oracle import rms as orms
    m = 96
    g = torch.Generator().manual_seed(5)
    norm_w = (1.0 + 0.1 * torch.randn(bench.HIDDEN, generator=g)).to(torch.bfloat16)
    w1, s1 = og.quant_weight(torch.randn(2 * 256, bench.HIDDEN, generator=g) * 0.02)
    w2, s2 = og.quant_weight(torch.randn(bench.HIDDEN, 256, generator=g) * 0.02)
    x = torch.randn(m, bench.HIDDEN, generator=g).to(torch.bfloat16)
    q, sq = orms.rms_quant(x, norm_w, eps=1e-6)
    h = og.swiglu_epilogue(og.accumulate(q, w1), sq, s1, None)
    hq, sh = oq.quant(h)
    y = og.scaled_mm(hq, w2, sh, s2)
    par = bench.ffn_parity(x, (norm_w, w1, s1, w2, s2), {"h": h, "y": y}, rows=16)
    assert par["ok"] and par["rel_l2"]["ffn_y"] < 5e-3     # CPU matmuls of a row subset may round differently
    y2 = y.clone()
    y2[0] *= 2
    assert not bench.ffn_parity(x, (norm_w, w1, s1, w2, s2), {"h": h, "y": y2}, rows=16)["ok"]


def test_other_configs_shard_at_every_driver_n():
    """The cfg1 / cfg3 token counts of the JSON line's other_configs split evenly over 1, 2, 4 and 8 ranks, as the
    heads do, so the driver's scaling runs carry them at every N."""
    import bench
    for _, tokens, _grid in bench.OTHER_CONFIGS:
        for n in (1, 2, 4, 8):
            assert tokens % n == 0 and bench.HEADS % n == 0


def test_roofline_fraction_at_the_kernels_own_clock():
    """The clock-normalised roofline: the sustained peak, measured at one median SM clock, is moved to the clock the
    timed region ran at before the kernel's rate is divided by it; missing clocks give no fraction, not a guess."""
    import bench

    r = bench.clock_normalised(1100.0, 1363.1, 1312.0, 1560.0)
    assert abs(r["peak_at_run_clock"] - 1363.1 * 1560.0 / 1312.0) < 1e-9
    assert abs(r["frac_at_run_clock"] - 1100.0 / (1363.1 * 1560.0 / 1312.0)) < 1e-12
    assert r["peak_sm_mhz"] == 1312.0 and r["run_sm_mhz"] == 1560.0
    assert bench.clock_normalised(1100.0, 1363.1, None, 1560.0)["frac_at_run_clock"] is None
    assert bench.clock_normalised(1100.0, 1363.1, 1312.0, None)["frac_at_run_clock"] is None
    peaks = bench.measured_peaks()
    assert "sustained_sm_mhz" in peaks
