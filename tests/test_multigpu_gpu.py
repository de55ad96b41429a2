"""Ulysses over NCCL and through peer memory on 2 (and, when visible, 4 or 8) GPUs, one process per GPU: the ranks'
rows of the attention block are bit-identical to the single-GPU block (each head's attention sees the same keys in the
same order), forward after forward."""
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("n,groups,exchange", [(2, 1, "nccl"), (2, 2, "nccl"), (4, 1, "nccl"), (4, 2, "nccl"),
                                               (8, 1, "nccl"), (2, 1, "p2p"), (4, 1, "p2p"), (8, 1, "p2p"),
                                               (2, 1, "nocopy"), (4, 2, "nocopy")])
def test_ulysses_ranks_equal_single_gpu(dev, tmp_path, n, groups, exchange):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs, {torch.cuda.device_count()} visible")
    iters = 3 if exchange == "p2p" else 1
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", str(n), "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           str(ROOT / "tests" / "mgpu_worker.py"), "--out", str(tmp_path), "--heads", "16", "--groups", str(groups),
           "--exchange", exchange, "--iters", str(iters)]
    res = subprocess.run(cmd, capture_output=True, text=True, env={**__import__("os").environ, "NCCL_NVLS_ENABLE": "0"})
    assert res.returncode == 0, res.stderr[-4000:]
    for it in range(iters):
        full = torch.load(tmp_path / f"full_{it}.pt")
        parts = torch.cat([torch.load(tmp_path / f"rank{r}_{it}.pt") for r in range(n)])
        assert torch.equal(parts.view(torch.int16), full.view(torch.int16)), it
