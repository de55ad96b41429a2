"""Ulysses layout kernels against the oracle layouts (bit-exact)."""
import pytest
import torch

from _util import BF16, same_bits
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
