"""The peer-memory Ulysses exchange on one GPU: the kernels' peer-store epilogues (ranks emulated one after another,
every "peer" buffer a local tensor, so nothing waits on anything) give exactly the bytes the all-to-all would deliver;
a one-rank PeerExchange runs the whole block; the epoch barrier gives up with H3B_ETIMEOUT when a flag never
arrives; a v overflow on one rank reaches every rank's flag; and the peer attention serves a v beyond f16."""
import math

import pytest
import torch

from _util import BF16, F16, same_bits
from h3b import _lib, ops
from h3b.block import AttentionBlock, quant_weight
from oracle import block as ob
from oracle import ulysses as ou

pytestmark = pytest.mark.gpu


def _weights(hidden, heads, seed):
    g = torch.Generator().manual_seed(seed)
    wqkv = torch.randn(3 * heads * 128, hidden, generator=g) * 0.02
    return quant_weight(wqkv)


@pytest.mark.parametrize("ws,m,heads", [(2, 256, 4), (4, 200, 8), (8, 128, 8)])
def test_qkv_peer_stores_equal_all_to_all(dev, ws, m, heads):
    """Rank r's GEMM with p2p targets writes, into every rank p's receive buffers at slot r, exactly the slab its
    send-buffer GEMM gives for destination p; recv[p] then equals the all-to-all of all ranks' send buffers."""
    hidden = 512
    w8, sw = (t.to(dev) for t in _weights(hidden, heads, seed=ws))
    hl = heads // ws
    recv = [[torch.full((ws, m, hl, 128), -1, dtype=dt, device=dev) for dt in (BF16, BF16, F16)] for _ in range(ws)]
    flags = [torch.zeros(1, dtype=torch.int32, device=dev) for _ in range(ws)]
    sends = []
    for r in range(ws):
        x = torch.randn(m, hidden, generator=torch.Generator().manual_seed(100 + r)).to(BF16).to(dev)
        q8, sx = ops.quant(x)
        sends.append(ops.fp8_gemm_qkv_send(q8, w8, sx, sw, heads, ws, v_f16=True))
        ops.fp8_gemm_qkv_send(q8, w8, sx, sw, heads, ws, v_f16=True, p2p=(r, recv, flags))
    torch.cuda.synchronize()
    for p in range(ws):
        for i in range(3):
            want = torch.stack([sends[r][i][p] for r in range(ws)])   # what all_to_all_single delivers to p
            assert same_bits(recv[p][i], want), (p, i)
    assert all(int(f.item()) == 0 for f in flags)
    assert ops.device_status() == 0


def test_qkv_peer_stores_raise_the_destination_flags(dev):
    """A v that overflows f16 on one source raises the range flag of every destination it was stored to."""
    ws, m, heads, hidden = 2, 128, 4, 256
    w8, sw = (t.to(dev) for t in _weights(hidden, heads, seed=9))
    recv = [[torch.empty((ws, m, heads // ws, 128), dtype=dt, device=dev) for dt in (BF16, BF16, F16)]
            for _ in range(ws)]
    flags = [torch.zeros(1, dtype=torch.int32, device=dev) for _ in range(ws)]
    x = (torch.randn(m, hidden, generator=torch.Generator().manual_seed(3)) * 1e7).to(BF16).to(dev)
    q8, sx = ops.quant(x)
    ops.fp8_gemm_qkv_send(q8, w8, sx, sw, heads, ws, v_f16=True, p2p=(1, recv, flags))
    torch.cuda.synchronize()
    assert [int(f.item()) for f in flags] == [1, 1]
    assert ops.device_status() == 0


@pytest.mark.parametrize("ws,m,hl", [(2, 256, 2), (4, 160, 1), (8, 128, 2)])
def test_attention_peer_stores_equal_reverse_all_to_all(dev, ws, m, hl):
    """Rank r's attention with peer targets stores output row t at slot r of rank t // m's back buffer: the bytes the
    head->seq all-to-all of its plain output delivers."""
    n = ws * m
    g = torch.Generator().manual_seed(ws)
    back = [torch.full((ws, m, hl, 128), -1, dtype=BF16, device=dev) for _ in range(ws)]
    outs = []
    for r in range(ws):
        q, k, v = (torch.randn(n, hl, 128, generator=g).to(BF16).to(dev) for _ in range(3))
        v16 = v.to(F16)
        outs.append(ops.flash_attn(q, k, v16, scale=1 / math.sqrt(128)).view(ws, m, hl, 128))
        ops.flash_attn_p2p(q, k, v16, back, r, scale=1 / math.sqrt(128))
    torch.cuda.synchronize()
    for p in range(ws):
        assert same_bits(back[p], torch.stack([outs[r][p] for r in range(ws)])), p
    assert ops.device_status() == 0


def test_one_rank_peer_exchange_runs_the_block(dev):
    """P = 1 through PeerExchange (its own buffer is the only peer; each barrier waits for its own flag): quant ->
    GEMM into the receive buffers -> barrier -> attention into the back buffer -> barrier -> quant -> out GEMM equals
    the plain block, forward after forward."""
    from h3b.ulysses_p2p import PeerExchange

    n, hidden, heads = 512, 512, 4
    weights = ob.make_weights(hidden, heads, seed=5)
    blk = AttentionBlock(hidden, heads, device=dev, weights=weights)
    px = PeerExchange(n, heads, 1, 0, dev, allgather=lambda b: [b])
    try:
        for it in range(3):
            x = torch.randn(n, hidden, generator=torch.Generator().manual_seed(it)).to(BF16).to(dev)
            want = blk(x)
            q8, sx = ops.quant(x)
            px.forward_qkv(q8, blk.wqkv8, sx, blk.sqkv)
            px.barrier()
            px.attention(1 / math.sqrt(128))
            px.barrier()
            o8, so = ops.quant_from_recv(px.back)
            y = ops.fp8_gemm(o8, blk.wo8, so, blk.so)
            assert same_bits(y, want), it
        assert px.epoch == 6
        assert int(px._flags[0].item()) == 6
        assert ops.device_status() == 0
    finally:
        px.close()


def test_barrier_gives_up_on_a_missing_peer(dev):
    """A flag that nothing sets: the barrier kernel returns after the wait bound with H3B_ETIMEOUT, having published
    its own epoch to both ranks; the context stays usable."""
    lib = _lib.load()
    flags = [torch.zeros(8, dtype=torch.int32, device=dev) for _ in range(2)]
    _lib.check(lib.h3b_set_wait_timeout_ns(20_000_000), "h3b_set_wait_timeout_ns")
    try:
        ops.p2p_signal_wait(flags, flags[0], 0, 7, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert ops.device_status() == _lib.H3B_ETIMEOUT
    finally:
        _lib.check(lib.h3b_set_wait_timeout_ns(4_000_000_000), "h3b_set_wait_timeout_ns")
    assert flags[0][0].item() == 7 and flags[1][0].item() == 7
    assert flags[0][1].item() == 0
    # both slots present: the same barrier passes
    flags[0][1] = 7
    ops.p2p_signal_wait(flags, flags[0], 0, 7, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert ops.device_status() == 0


def test_peer_attention_serves_v_outside_f16(dev):
    """The peer-memory attention with a bf16 v beyond f16's range (the scaled pass, chosen on the device) stores into
    every owner's reverse buffer exactly the rows the local attention computes."""
    ws, m, hl = 2, 192, 2
    g = torch.Generator().manual_seed(21)
    q, k, v = (torch.randn(ws * m, hl, 128, generator=g).to(BF16).to(dev) for _ in range(3))
    v[40, 1, 7] = 2.0e6
    back = [torch.full((ws, m, hl, 128), -1, dtype=BF16, device=dev) for _ in range(ws)]
    ctl = ops.attn_ctl(hl, dev)
    ops.flash_attn_p2p(q, k, v, back, 1, ctl=ctl)
    o = ops.flash_attn(q, k, v)
    torch.cuda.synchronize()
    assert int(ctl[0].item()) == 1
    for t in range(ws):
        assert same_bits(back[t][1], o[t * m:(t + 1) * m]), t
    assert ops.device_status() == 0
