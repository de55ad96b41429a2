"""Worker for tests/test_multigpu_gpu.py (launched by torchrun, one process per GPU, NCCL): every rank runs its rows
of the cfg-like attention block with the Ulysses exchange over NCCL (--exchange nccl) or through peer memory
(--exchange p2p); rank 0 also runs the single-GPU block.  Results are written to --out for the test to compare."""
import argparse
import datetime
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT / "minimax-h3-2x-dgx-spark-tp2_b200"), str(ROOT)]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--hidden", type=int, default=1024)
    ap.add_argument("--heads", type=int, default=8)
    ap.add_argument("--groups", type=int, default=0)
    ap.add_argument("--exchange", default="nccl")
    ap.add_argument("--iters", type=int, default=1)
    args = ap.parse_args()
    rank, ws, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        from h3b import ops
        from h3b.block import AttentionBlock

        m = args.tokens // ws
        if args.exchange == "p2p":
            from h3b.ulysses_p2p import probe
            ok, why = probe(dist.group.WORLD, dev)
            assert ok, why
        blk = AttentionBlock(args.hidden, args.heads, device=dev, ws=ws, pg=dist.group.WORLD, seed=1,
                             groups=args.groups or None, exchange=args.exchange)
        full_blk = AttentionBlock(args.hidden, args.heads, device=dev, ws=1, seed=1) if rank == 0 else None
        for it in range(args.iters):   # several forwards back to back: buffer reuse across steps
            g = torch.Generator().manual_seed(it)
            x = torch.randn(args.tokens, args.hidden, generator=g).to(torch.bfloat16)
            y = blk(x[rank * m:(rank + 1) * m].contiguous().to(dev))
            torch.save(y.cpu(), Path(args.out) / f"rank{rank}_{it}.pt")
            if rank == 0:
                torch.save(full_blk(x.to(dev)).cpu(), Path(args.out) / f"full_{it}.pt")
        torch.cuda.synchronize()
        assert ops.device_status() == 0
        blk.close()
        dist.barrier(device_ids=[local])
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
