"""The C-ABI library loads without a GPU and exports exactly what include/h3b.h declares; argument errors are
reported on the host before any CUDA call."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from h3b import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "h3b.h"


def declared():
    text = HEADER.read_text()
    return set(re.findall(r"^H3B_API\s+[^(]*?\b(h3b_\w+)\s*\(", text, flags=re.M))


def exported():
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T h3b_" in line}


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared()
    assert len(names) >= 17
    for n in names:
        assert hasattr(lib, n), n
    assert exported() == names


def test_binding_signatures_cover_the_header():
    assert set(_lib.SIGNATURES) == declared()


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.h3b_abi_version() == _lib.ABI_VERSION == 4
    assert lib.h3b_status_string(0) == b"ok"
    assert lib.h3b_status_string(_lib.H3B_ETIMEOUT) == b"device wait timed out"


_PEERS2 = (ctypes.c_void_p * 2)(16, 32)
_PEERS2_BAD = (ctypes.c_void_p * 2)(16, 33)


def _qkv_p2p(rank=0, groups=1, null_peer=False):
    d = _lib.QkvSend()
    d.heads, d.head_dim, d.ws, d.groups, d.p2p, d.rank = 2, 128, 2, groups, 1, rank
    for r in range(2):
        for i in range(3):
            d.peer_recv[r][i] = None if (null_peer and r == 1) else 4096 * (1 + 3 * r + i)
    return d


def _qkv_norm():
    d = _lib.QkvSend()
    d.heads, d.head_dim, d.ws, d.groups = 2, 128, 2, 1
    for i in range(3):
        d.send[i] = 4096 * (1 + i)
    d.q_norm_weight, d.k_norm_weight, d.rope_table = 8192, 8448, 8704
    d.rope_stride, d.rot, d.eps = 64, 64, 1e-6
    return d


@pytest.mark.parametrize("call,status", [
    (lambda L: L.h3b_quant_rows_e4m3(None, -1, 1, 8, 0, 8, None, None, 0, None), _lib.H3B_EINVAL),
    (lambda L: L.h3b_quant_rows_e4m3(None, 4, 1, 8, 0, 8, None, None, 7, None), _lib.H3B_EINVAL),
    (lambda L: L.h3b_quant_rows_e4m3(None, 0, 1, 8, 0, 8, None, None, 0, None), _lib.H3B_OK),
    (lambda L: L.h3b_fp8_gemm(1, 16, 1, 16, 1, 1, None, 1, 16, 4, 24, 16, 0, 0, None, None), _lib.H3B_EUNSUPPORTED),
    (lambda L: L.h3b_fp8_gemm(1, 16, 1, 16, 1, 1, None, 1, 16, 4, 32, 16, 0, 9, None, None), _lib.H3B_EINVAL),
    (lambda L: L.h3b_fp8_gemm(None, 16, 1, 16, 1, 1, None, 1, 16, 4, 32, 16, 0, 0, None, None), _lib.H3B_EINVAL),
    (lambda L: L.h3b_flash_attn_fwd(1, 8, 8, 1, 8, 8, 1, 8, 8, 1, 8, 8, 4, 4, -1, 1, 64, 1.0, 0, None, None),
     _lib.H3B_EUNSUPPORTED),
    (lambda L: L.h3b_flash_attn_fwd(1, 8, 8, 1, 8, 8, 1, 8, 8, 1, 8, 8, 4, 4, 9, 1, 128, 1.0, 0, None, None),
     _lib.H3B_EINVAL),
    (lambda L: L.h3b_flash_attn_fwd(1, 8, 8, 1, 12, 8, 1, 8, 8, 1, 8, 8, 4, 4, -1, 1, 128, 1.0, 0, None, None),
     _lib.H3B_EALIGN),
    (lambda L: L.h3b_pack_by_dest(1, 4, 6, 128, 768, 128, 4, 1, 0, None, None), _lib.H3B_EINVAL),
    (lambda L: L.h3b_rms_quant_e4m3(1, 4, 64, 64, 1, 1, 64, None, 0, None, 1e-6, None, 1, 1, 0, None),
     _lib.H3B_EINVAL),
    (lambda L: L.h3b_fp8_gemm_gate(16, 16, 16, 16, 16, 16, None, None, 256, 16, 256, 2, 16, 16, 256, 4, 256, 16, None),
     _lib.H3B_EINVAL),
    (lambda L: L.h3b_fp8_gemm_gate(16, 16, 16, 16, 16, 16, None, 16, 250, 16, 256, 2, 16, 16, 256, 4, 256, 16, None),
     _lib.H3B_EALIGN),
    (lambda L: L.h3b_fp8_gemm_gate(16, 16, 16, 16, 16, 16, None, 16, 256, 16, 256, 0, 16, 16, 256, 4, 256, 16, None),
     _lib.H3B_EINVAL),
    # peer-memory exchange: bad rank / world, row split, sizes
    (lambda L: L.h3b_p2p_signal_wait(None, None, 2, 0, 1, None), _lib.H3B_EINVAL),
    (lambda L: L.h3b_p2p_signal_wait(_PEERS2, 1, 9, 0, 1, None), _lib.H3B_EINVAL),
    (lambda L: L.h3b_p2p_signal_wait(_PEERS2, 1, 2, 2, 1, None), _lib.H3B_EINVAL),
    (lambda L: L.h3b_p2p_alloc(0, ctypes.byref(ctypes.c_void_p()), ctypes.byref(_lib.IpcHandle())), _lib.H3B_EINVAL),
    (lambda L: L.h3b_p2p_open(None, ctypes.byref(ctypes.c_void_p())), _lib.H3B_EINVAL),
    (lambda L: L.h3b_p2p_close(None), _lib.H3B_OK),
    (lambda L: L.h3b_p2p_free(None), _lib.H3B_OK),
    (lambda L: L.h3b_flash_attn_fwd_p2p(16, 8, 8, 16, 8, 8, 16, 8, 8, _PEERS2, 2, 0, 100, 256, 256, -1, 1, 128, 1.0,
                                        0, None, None), _lib.H3B_EINVAL),
    (lambda L: L.h3b_flash_attn_fwd_p2p(16, 8, 8, 16, 8, 8, 16, 8, 8, _PEERS2, 2, 3, 128, 256, 256, -1, 1, 128, 1.0,
                                        0, None, None), _lib.H3B_EINVAL),
    (lambda L: L.h3b_flash_attn_fwd_p2p(16, 8, 8, 16, 8, 8, 16, 8, 8, _PEERS2_BAD, 2, 0, 128, 256, 256, -1, 1, 128,
                                        1.0, 0, None, None), _lib.H3B_EALIGN),
    (lambda L: L.h3b_fp8_gemm(16, 16, 16, 16, 16, 16, None, None, 0, 4, 3 * 2 * 128, 16, 0, 1,
                              ctypes.byref(_qkv_p2p(rank=2)), None), _lib.H3B_EINVAL),
    (lambda L: L.h3b_fp8_gemm(16, 16, 16, 16, 16, 16, None, None, 0, 4, 3 * 2 * 128, 16, 0, 1,
                              ctypes.byref(_qkv_p2p(groups=2)), None), _lib.H3B_EUNSUPPORTED),
    (lambda L: L.h3b_fp8_gemm(16, 16, 16, 16, 16, 16, None, None, 0, 4, 3 * 2 * 128, 16, 0, 1,
                              ctypes.byref(_qkv_p2p(null_peer=True)), None), _lib.H3B_EALIGN),
    # the norm + RoPE epilogue has no bias term: a bias with norm weights is refused, not dropped
    (lambda L: L.h3b_fp8_gemm(16, 16, 16, 16, 16, 16, 16, None, 0, 4, 3 * 2 * 128, 16, 0, 1,
                              ctypes.byref(_qkv_norm()), None), _lib.H3B_EUNSUPPORTED),
])
def test_host_side_argument_errors(call, status):
    lib = _lib.load()
    assert call(lib) == status
    if status != _lib.H3B_OK:
        assert lib.h3b_last_error()


def test_check_raises_with_the_reason():
    lib = _lib.load()
    rc = lib.h3b_quant_rows_e4m3(None, -1, 1, 8, 0, 8, None, None, 0, None)
    with pytest.raises(_lib.H3BError, match="quant_rows"):
        _lib.check(rc, "h3b_quant_rows_e4m3")


def test_wait_timeout_bounds():
    """The device-wait bound is a host-side setting: below 1 ms the library refuses it, and the default is restored."""
    from h3b import ops
    with pytest.raises(ValueError):
        ops.set_wait_timeout_ns(0)
    with pytest.raises(_lib.H3BError, match="below 1 ms"):
        ops.set_wait_timeout_ns(999_999)
    ops.set_wait_timeout_ns(4_000_000_000)


def test_qkv_send_struct_layout(tmp_path):
    """The ctypes mirror matches the C compiler's layout of h3b_qkv_send field by field."""
    fields = [f[0] for f in _lib.QkvSend._fields_]
    src = tmp_path / "layout.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "h3b.h"\nint main(void) {\n'
                   '  printf("%zu\\n", sizeof(h3b_qkv_send));\n' +
                   "".join(f'  printf("%zu\\n", offsetof(h3b_qkv_send, {f}));\n' for f in fields) +
                   '  printf("%zu\\n", sizeof(h3b_ipc_handle));\n  return 0;\n}\n')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    want = [ctypes.sizeof(_lib.QkvSend)] + [getattr(_lib.QkvSend, f).offset for f in fields] + \
        [ctypes.sizeof(_lib.IpcHandle)]
    assert got == want
    assert ctypes.sizeof(_lib.QkvSend) == 368
