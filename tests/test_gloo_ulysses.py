"""BASELINE config 0 on two CPU processes over gloo (world size 2): the Ulysses block with a real collective equals
the single-process block, through both the oracle and the h3b orchestration (``ulysses_exact.exact_forward`` with
``torch.distributed.all_to_all_single``), and the combined q/k/v exchange (``ulysses_nocopy.nocopy_forward``, one and two
head groups; its layout runs in torch in these CPU processes).  A rank that dies before the exchange makes the survivor's collective fail
within the process-group timeout (failure detection on the host, no GPU involved)."""
import datetime
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _cfg0(seed=0):
    """B=1, 4096 tokens, hidden 1024, 8 heads x 128, fp32, x ~ N(0,1), Wqkv/Wo ~ N(0, 0.02), no bias."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(4096, 1024, generator=g)
    wqkv = torch.randn(3 * 1024, 1024, generator=g) * 0.02
    wo = torch.randn(1024, 1024, generator=g) * 0.02
    return x, wqkv, wo


def _worker(rank, ws, port, mode, out_dir):
    sys.path[:0] = [str(ROOT / "minimax-h3-2x-dgx-spark-tp2_b200"), str(ROOT), str(ROOT / "tests")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.set_num_threads(2)
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=10))
    try:
        from oracle import attention as oa
        from oracle import block as ob
        from oracle import ulysses as ou
        from h3b import ulysses_exact

        x, wqkv, wo = _cfg0()
        m = x.shape[0] // ws
        xl = x[rank * m:(rank + 1) * m]
        if mode == "die":
            if rank == 1:
                os._exit(3)
            send = torch.zeros(ws, 4)
            try:
                dist.all_to_all_single(torch.empty_like(send), send)
                torch.save({"raised": False}, Path(out_dir) / f"r{rank}.pt")
            except Exception as exc:  # noqa: BLE001
                torch.save({"raised": True, "what": type(exc).__name__}, Path(out_dir) / f"r{rank}.pt")
            return

        def a2a(out, inp, group=None):
            dist.all_to_all_single(out, inp, group=group)

        if mode == "nocopy":      # the combined q/k/v exchange, one and two head groups, over the real collective
            from h3b import ops, ulysses_nocopy

            ops._need_cuda = lambda *ts: None                   # this CPU process runs the layout in torch

            def unpack_recv(recv, out=None):
                p_, m_, hl, d = recv.shape
                o_ = out if out is not None else torch.empty((m_, p_ * hl, d), dtype=recv.dtype)
                o_.view(m_, p_, hl, d).copy_(recv.permute(1, 0, 2, 3))
                return o_
            ops.unpack_recv = unpack_recv
            qkv = xl @ wqkv.t()
            q, k, v = (t.reshape(1, m, 8, 128) for t in qkv.split(1024, dim=1))
            res = {}
            for groups in (1, 2):
                o = ulysses_nocopy.nocopy_forward(q, k, v, lambda a, b, c: oa.sdpa(a[0], b[0], c[0]).unsqueeze(0),
                                                  ws=ws, groups=groups, a2a=a2a)
                res[f"g{groups}"] = o.reshape(m, 1024) @ wo.t()
            torch.save(res, Path(out_dir) / f"r{rank}.pt")
            return

        y_oracle = ob.fp32_block(xl, wqkv, wo, 8, ws, a2a)
        qkv = xl @ wqkv.t()
        q, k, v = (t.reshape(1, m, 8, 128) for t in qkv.split(1024, dim=1))
        o = ulysses_exact.exact_forward(q, k, v, lambda a, b, c: oa.sdpa(a[0], b[0], c[0]).unsqueeze(0), ws=ws,
                                        pack=ou.pack, unpack_fn=ou.unpack)
        y_h3b = o.reshape(m, 1024) @ wo.t()
        torch.save({"oracle": y_oracle, "h3b": y_h3b}, Path(out_dir) / f"r{rank}.pt")
    finally:
        if mode != "die" or rank == 0:
            dist.destroy_process_group()


def _spawn(mode, tmp_path, ws=2):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, ws, port, mode, str(tmp_path))) for r in range(ws)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        if p.is_alive():
            p.kill()
            pytest.fail("gloo worker hung")
    return procs


def test_config0_two_ranks_equal_single_process(tmp_path):
    from oracle import attention as oa

    procs = _spawn("block", tmp_path)
    assert all(p.exitcode == 0 for p in procs)
    x, wqkv, wo = _cfg0()
    qkv = x @ wqkv.t()
    q, k, v = (t.reshape(4096, 8, 128) for t in qkv.split(1024, dim=1))
    ref = oa.sdpa(q, k, v).reshape(4096, 1024) @ wo.t()
    for r in range(2):
        got = torch.load(tmp_path / f"r{r}.pt")
        rows = ref[r * 2048:(r + 1) * 2048]
        for key in ("oracle", "h3b"):
            err = float((got[key] - rows).norm() / rows.norm())
            assert err < 1e-5, (key, r, err)


def test_config0_combined_exchange_two_ranks(tmp_path):
    """The combined q/k/v exchange (one all-to-all per head group, attention on strided views of the receive buffer)
    over gloo equals the single-process block for one and two head groups."""
    from oracle import attention as oa

    procs = _spawn("nocopy", tmp_path)
    assert all(p.exitcode == 0 for p in procs)
    x, wqkv, wo = _cfg0()
    qkv = x @ wqkv.t()
    q, k, v = (t.reshape(4096, 8, 128) for t in qkv.split(1024, dim=1))
    ref = oa.sdpa(q, k, v).reshape(4096, 1024) @ wo.t()
    for r in range(2):
        got = torch.load(tmp_path / f"r{r}.pt")
        rows = ref[r * 2048:(r + 1) * 2048]
        for key in ("g1", "g2"):
            err = float((got[key] - rows).norm() / rows.norm())
            assert err < 1e-5, (key, r, err)


def test_dead_rank_fails_the_survivors_collective(tmp_path):
    procs = _spawn("die", tmp_path)
    assert procs[1].exitcode == 3
    res = torch.load(tmp_path / "r0.pt")
    assert res["raised"], "the surviving rank's all_to_all must fail, not hang"
