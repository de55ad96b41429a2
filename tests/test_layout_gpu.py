"""Ulysses layout kernels against the oracle layouts (bit-exact)."""
import pytest
import torch

from _util import BF16, rel_l2, same_bits
from h3b import ops, ulysses_exact
from oracle import ulysses as ou

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("ws", [1, 2, 4, 8])
def test_pack_from_strided_qkv_view_and_unpack(dev, ws):
    m, heads, d = 37, 8, 128
    qkv = (torch.randn(m, 3 * heads * d) * 3).to(BF16)
    k = qkv[:, heads * d:2 * heads * d].view(m, heads, d)          # row stride 3*H*d, like the qkv GEMM output
    send = ops.pack_by_dest(qkv.to(dev)[:, heads * d:2 * heads * d].view(m, heads, d), ws)
    assert same_bits(send.cpu(), ou.pack(k, ws))
    assert same_bits(ops.unpack_recv(send).cpu(), ou.unpack(ou.pack(k, ws)))
    assert same_bits(ulysses_exact.unpack(send).cpu(), k.contiguous())


def test_pack_to_f16_exact_and_range_flag(dev):
    x = (torch.randn(16, 4, 128) * 100).to(BF16)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    send = ops.pack_by_dest(x.to(dev), 2, to_f16=True, range_flag=flag)
    assert send.dtype == torch.float16 and int(flag.item()) == 0
    assert torch.equal(send.cpu().float(), ou.pack(x, 2).float())
    x[3, 1, 7] = 70000.0
    ops.pack_by_dest(x.to(dev), 2, to_f16=True, range_flag=flag)
    assert int(flag.item()) == 1


def test_bf16_to_f16(dev):
    x = (torch.randn(4096) * 50).to(BF16)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    y = ops.bf16_to_f16(x.to(dev), flag)
    assert torch.equal(y.cpu().float(), x.float()) and int(flag.item()) == 0


def test_norm_rope_send_against_reference_vectors(dev, golden):
    from _util import t16, tf, ulp_diff_bf16
    g = golden("rope")
    for ws in (2, 4):
        m, heads = (int(v) for v in g[f"ws{ws}_shape"])
        qkv = t16(g[f"ws{ws}_qkv"]).to(dev)
        q, k, _ = (t.view(m, heads, 128) for t in qkv.split([heads * 128] * 3, dim=-1))
        table = tf(g[f"ws{ws}_table"]).to(dev)
        sq = torch.empty((ws, m, heads // ws, 128), dtype=BF16, device=dev)
        sk = torch.empty_like(sq)
        ulysses_exact.rope_into_send(sq, sk, q, k, t16(g[f"ws{ws}_wq"]).to(dev), t16(g[f"ws{ws}_wk"]).to(dev), table,
                                     1e-6)
        for got, key in ((sq, "sendq"), (sk, "sendk")):
            ud = ulp_diff_bf16(got.cpu(), t16(g[f"ws{ws}_{key}"]))
            # rsqrt on the GPU vs the CPU's moves a normalised value by a bf16 ulp at most; the rotation
            # a cos - b sin can cancel and turn that into a few ulps of a smaller result, on few elements
            assert (ud == 0).float().mean().item() > 0.98 and int(ud.max()) <= 8
            assert rel_l2(got.float().cpu(), t16(g[f"ws{ws}_{key}"]).float()) <= 2e-3


def test_norm_rope_send_dit_shape(dev):
    from oracle import ulysses as oul
    from _util import ulp_diff_bf16
    m, heads, ws = 300, 40, 4
    gen = torch.Generator().manual_seed(2)
    qkv = torch.randn(m, 3 * heads * 128, generator=gen).to(BF16)
    q = qkv[:, :heads * 128].view(m, heads, 128)
    w = (1 + 0.1 * torch.randn(128, generator=gen)).to(BF16)
    table = torch.randn(m, 96, generator=gen)
    got = ops.norm_rope_send(qkv.to(dev)[:, :heads * 128].view(m, heads, 128), w.to(dev), table.to(dev), 1e-6, ws)
    ref = oul.norm_rope_into_send(q, w, table, 1e-6, ws)
    ud = ulp_diff_bf16(got.cpu(), ref)
    assert (ud == 0).float().mean().item() > 0.98 and int(ud.max()) <= 8
    assert rel_l2(got.float().cpu(), ref.float()) <= 2e-3
