"""tcgen05 flash attention against an fp32 SDPA on the same bf16 inputs: rel-L2 <= 2e-3 and max-abs <= 2e-2."""
import pytest
import torch

from _util import BF16, F16, rel_l2
from h3b import ops
from oracle import attention as oa

pytestmark = pytest.mark.gpu


def _qkv(s_q, s_kv, h, seed, vscale=1.0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(s_q, h, 128, generator=g).to(BF16)
    k = torch.randn(s_kv, h, 128, generator=g).to(BF16)
    v = (torch.randn(s_kv, h, 128, generator=g) * vscale).to(BF16)
    return q, k, v


def _check(o, ref, tol_rel=2e-3, tol_abs=2e-2):
    o = o.float().cpu()
    assert rel_l2(o, ref) <= tol_rel, rel_l2(o, ref)
    assert (o - ref).abs().max().item() <= tol_abs


@pytest.mark.parametrize("s,h", [(128, 1), (256, 2), (300, 2), (1000, 3), (4096, 2)])
def test_self_attention_shapes(dev, s, h):
    q, k, v = _qkv(s, s, h, seed=s + h)
    o = ops.flash_attn(q.to(dev), k.to(dev), v.to(dev))
    _check(o, oa.sdpa(q, k, v))
    assert ops.device_status() == 0


def test_cross_lengths_and_valid_kv(dev):
    q, k, v = _qkv(200, 777, 2, seed=1)
    o = ops.flash_attn(q.to(dev), k.to(dev), v.to(dev))
    _check(o, oa.sdpa(q, k, v))
    o = ops.flash_attn(q.to(dev), k.to(dev), v.to(dev), valid_kv=517)
    _check(o, oa.sdpa(q, k, v, valid_kv=517))


def test_peaked_scores_rescale_path(dev):
    # large q scale: the running max jumps by many binades between key tiles (exercises the O rescale)
    g = torch.Generator().manual_seed(3)
    q = (torch.randn(512, 2, 128, generator=g) * 4).to(BF16)
    k = (torch.randn(2048, 2, 128, generator=g)).to(BF16)
    k[1500:1510] *= 3
    v = torch.randn(2048, 2, 128, generator=g).to(BF16)
    o = ops.flash_attn(q.to(dev), k.to(dev), v.to(dev))
    _check(o, oa.sdpa(q, k, v))


def test_bf16_pv_variant(dev):
    q, k, v = _qkv(1024, 1024, 2, seed=7)
    o = ops.flash_attn(q.to(dev), k.to(dev), v.to(dev), pv_f16=False)
    _check(o, oa.sdpa(q, k, v), tol_rel=4e-3)


def test_ulysses_receive_views_and_head_independence(dev):
    # q/k/v as the [1, P*M, hl, d] receive views; heads computed alone equal heads computed together (bitwise)
    s, h = 640, 4
    q, k, v = _qkv(s, s, h, seed=11)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    o_all = ops.flash_attn(qd.unsqueeze(0), kd.unsqueeze(0), vd.unsqueeze(0))
    for h0 in range(0, h, 2):
        o_part = ops.flash_attn(qd[:, h0:h0 + 2].contiguous(), kd[:, h0:h0 + 2].contiguous(),
                                vd[:, h0:h0 + 2].contiguous())
        assert torch.equal(o_part.view(torch.int16), o_all[0, :, h0:h0 + 2].contiguous().view(torch.int16))
    _check(o_all[0], oa.sdpa(q, k, v))
    # strided (non-contiguous head slice) inputs
    o_str = ops.flash_attn(qd[:, 1:3], kd[:, 1:3], vd[:, 1:3])
    assert torch.equal(o_str.view(torch.int16), o_all[0, :, 1:3].contiguous().view(torch.int16))


def test_f16_v_with_raised_flag_refuses(dev):
    """An f16 v comes from a producer that converted it; with that producer's range flag raised the kernel writes
    nothing and records H3B_ERANGE (the caller asked for f16 P.V on an f16 copy that is not v)."""
    q, k, v = _qkv(128, 128, 1, seed=2)
    flag = torch.ones(1, dtype=torch.int32, device=dev)
    o = torch.full((128, 1, 128), 7.0, dtype=BF16, device=dev)
    ops.flash_attn(q.to(dev), k.to(dev), v.to(F16).to(dev), range_flag=flag, out=o)
    assert ops.device_status() == ops._lib.H3B_ERANGE
    assert (o.float() == 7.0).all()


@pytest.mark.parametrize("big", [80000.0, -3.0e9, 1.0e30])
def test_bf16_v_outside_f16_is_served(dev, big):
    """A bf16 v with values beyond f16's range takes the scaled pass (decided on the device): the output is written
    and stays within the f16 path's tolerance of fp32 SDPA.  Max-abs is measured relative to the output's scale."""
    q, k, v = _qkv(300, 777, 3, seed=4)
    v[5, 0, 3] = big            # one huge value in one column
    v[100:110, 2, :] = big / 2  # whole rows of another head
    ctl = ops.attn_ctl(3, dev)
    o = ops.flash_attn(q.to(dev), k.to(dev), v.to(dev), ctl=ctl)
    assert int(ctl[0].item()) == 1 and ops.device_status() == 0
    ref = oa.sdpa(q, k, v)
    o = o.float().cpu()
    assert rel_l2(o, ref) <= 2e-3, rel_l2(o, ref)
    # per (head, column): error against that column's scale (the scale is exact: ordinary columns keep f16 accuracy)
    colscale = ref.abs().amax(dim=0, keepdim=True).clamp_min(1.0)
    assert ((o - ref).abs() / colscale).max().item() <= 2e-2
    # ordinary heads and columns equal the plain f16 pass bit for bit (their scale is 2^0)
    o_plain = ops.flash_attn(q[:, 1:2].to(dev), k[:, 1:2].to(dev), v[:, 1:2].to(dev)).cpu()
    assert torch.equal(o[:, 1:2].to(BF16).view(torch.int16), o_plain.view(torch.int16))


def test_bf16_v_padding_rows_are_never_read(dev):
    """Rows of v (and k) beyond valid_kv may hold anything (here inf, nan and values beyond f16): the attention
    neither reads them nor takes the scaled pass because of them."""
    q, k, v = _qkv(256, 700, 2, seed=6)
    valid = 517
    v[valid:] = float("nan")
    v[valid + 3] = 1e30
    k[valid:] = float("inf")
    ctl = ops.attn_ctl(2, dev)
    o = ops.flash_attn(q.to(dev), k.to(dev), v.to(dev), valid_kv=valid, ctl=ctl)
    assert int(ctl[0].item()) == 0
    _check(o, oa.sdpa(q[:, :], k[:valid], v[:valid]))
    assert ops.device_status() == 0


def test_bf16_pv_variant_direct(dev):
    q, k, v = _qkv(512, 512, 2, seed=8)
    o = ops.flash_attn(q.to(dev), k.to(dev), v.to(dev), pv_f16=False)
    _check(o, oa.sdpa(q, k, v), tol_rel=4e-3)


@pytest.mark.parametrize("poly", ["0", "2", "3", "4"])
def test_poly_exp2_variants_in_a_fresh_process(dev, poly):
    """H3B_ATTN_EXP2_POLY=n (n of every 8 exponential pairs on the FMA pipe) stays within the attention tolerance."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    code = (
        "import sys, torch\n"
        f"sys.path[:0] = [{str(root / 'minimax-h3-2x-dgx-spark-tp2_b200')!r}, {str(root)!r}, {str(root / 'tests')!r}]\n"
        "from h3b import ops\n"
        "from oracle import attention as oa\n"
        "from _util import rel_l2\n"
        "g = torch.Generator().manual_seed(5)\n"
        "q, k, v = (torch.randn(1000, 2, 128, generator=g).to(torch.bfloat16) for _ in range(3))\n"
        "o = ops.flash_attn(q.cuda(), k.cuda(), v.cuda()).float().cpu()\n"
        "ref = oa.sdpa(q, k, v)\n"
        "print(rel_l2(o, ref), (o - ref).abs().max().item(), ops.device_status())\n")
    env = dict(os.environ, H3B_ATTN_EXP2_POLY=poly)
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    rel, mabs, status = out.stdout.split()
    assert float(rel) <= 2e-3 and float(mabs) <= 2e-2 and int(status) == 0


def test_pair_kernel_in_a_fresh_process(dev):
    """H3B_ATTN_PAIR=1 selects the CTA-pair kernel (2-SM MMAs): within the attention tolerance of fp32 SDPA on odd
    lengths, valid_kv, the scaled pass for a v beyond f16, and the peer-store epilogue equal to the local output."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    code = (
        "import sys, torch\n"
        f"sys.path[:0] = [{str(root / 'minimax-h3-2x-dgx-spark-tp2_b200')!r}, {str(root)!r}, {str(root / 'tests')!r}]\n"
        "from h3b import ops\n"
        "from oracle import attention as oa\n"
        "from _util import rel_l2\n"
        "worst = 0.0\n"
        "for s, h, vk, big in [(1000, 2, None, None), (300, 3, 129, None), (777, 2, 600, 90000.0), (4096, 1, None, None)]:\n"
        "    g = torch.Generator().manual_seed(s)\n"
        "    q, k, v = (torch.randn(s, h, 128, generator=g).to(torch.bfloat16) for _ in range(3))\n"
        "    if big: v[5, 0, 3] = big\n"
        "    o = ops.flash_attn(q.cuda(), k.cuda(), v.cuda(), valid_kv=vk).float().cpu()\n"
        "    ref = oa.sdpa(q, k, v, valid_kv=vk)\n"
        "    worst = max(worst, rel_l2(o, ref))\n"
        "ws, m = 2, 192\n"
        "g = torch.Generator().manual_seed(3)\n"
        "q, k, v = (torch.randn(ws * m, 2, 128, generator=g).to(torch.bfloat16).cuda() for _ in range(3))\n"
        "back = [torch.full((ws, m, 2, 128), -1.0, dtype=torch.bfloat16, device='cuda') for _ in range(ws)]\n"
        "ops.flash_attn_p2p(q, k, v, back, 1)\n"
        "o = ops.flash_attn(q, k, v)\n"
        "same = all(torch.equal(back[t][1].view(torch.int16), o[t * m:(t + 1) * m].view(torch.int16)) for t in range(ws))\n"
        "print(worst, int(same), ops.device_status())\n")
    env = dict(os.environ, H3B_ATTN_PAIR="1")
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    worst, same, status = out.stdout.split()
    assert float(worst) <= 2e-3 and same == "1" and int(status) == 0
