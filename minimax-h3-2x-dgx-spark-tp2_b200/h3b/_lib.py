"""ctypes binding of the C ABI in ``include/h3b.h`` (``libh3b.so``, built in-tree by ``build.py``).

There is no CPU fallback: if the library is missing or a call fails, this module raises.  Every call returns the
C status; ``check`` turns a non-zero status into ``RuntimeError`` carrying ``h3b_last_error()``.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libh3b.so"

H3B_OK, H3B_EINVAL, H3B_EALIGN, H3B_EUNSUPPORTED, H3B_ECUDA, H3B_ETIMEOUT, H3B_ERANGE = 0, -1, -2, -3, -4, -5, -6
DIV_IEEE, DIV_FULL = 0, 1
OUT_BF16, OUT_F16 = 0, 1
EPI_PLAIN, EPI_QKV_SEND, EPI_SWIGLU = 0, 1, 2

_p, _i32, _i64, _f32, _u64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_uint64
MAX_RANKS = 8   # H3B_MAX_RANKS
ABI_VERSION = 4


class QkvSend(ctypes.Structure):
    _fields_ = [("send", _p * 3), ("heads", _i32), ("head_dim", _i32), ("ws", _i32), ("v_f16", _i32),
                ("range_flag", _p), ("groups", _i32), ("q_norm_weight", _p), ("k_norm_weight", _p),
                ("rope_table", _p), ("rope_stride", _i64), ("rot", _i32), ("eps", _f32),
                ("p2p", _i32), ("rank", _i32), ("peer_recv", (_p * 3) * MAX_RANKS), ("peer_range_flag", _p * MAX_RANKS),
                ("qkv_interleaved", _i32)]


class IpcHandle(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_ubyte * 64)]


# name -> (restype, argtypes): exactly the declarations of include/h3b.h
SIGNATURES = {
    "h3b_abi_version": (ctypes.c_int, []),
    "h3b_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "h3b_last_error": (ctypes.c_char_p, []),
    "h3b_device_status": (ctypes.c_int, []),
    "h3b_set_wait_timeout_ns": (ctypes.c_int, [_u64]),
    "h3b_quant_rows_e4m3": (ctypes.c_int, [_p, _i64, _i32, _i64, _i64, _i64, _p, _p, _i32, _p]),
    "h3b_rms_quant_e4m3": (ctypes.c_int, [_p, _i64, _i64, _i64, _p, _p, _i64, _p, _i64, _p, _f32, _p, _p, _p, _i32,
                                          _p]),
    "h3b_gate_rms_quant_e4m3": (ctypes.c_int, [_p, _i64, _p, _i64, _p, _i64, _p, _p, _i64, _p, _i64, _p, _i64, _i64,
                                               _f32, _p, _p, _p, _i32, _p]),
    "h3b_silu_mul_quant_e4m3": (ctypes.c_int, [_p, _i64, _i64, _i64, _p, _p, _i32, _p]),
    "h3b_scale_bias_cast": (ctypes.c_int, [_p, _p, _p, _p, _p, _i64, _i64, _i32, _p]),
    "h3b_scale_swiglu": (ctypes.c_int, [_p, _p, _p, _p, _p, _i64, _i64, _p]),
    "h3b_scale_swiglu_quant": (ctypes.c_int, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i32, _p]),
    "h3b_fp8_gemm": (ctypes.c_int, [_p, _i64, _p, _i64, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i32, _i32,
                                    ctypes.POINTER(QkvSend), _p]),
    "h3b_flash_attn_fwd": (ctypes.c_int, [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i64, _i64,
                                          _i64, _i32, _i32, _f32, _i32, _p, _p]),
    "h3b_flash_attn_fwd_bf16v": (ctypes.c_int, [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i64,
                                                _i64, _i64, _i32, _i32, _f32, _p, _p, _p]),
    "h3b_flash_attn_fwd_noalloc": (ctypes.c_int, [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64,
                                                  _i64, _i64, _i64, _i32, _i32, _f32, _p]),
    "h3b_noalloc_status": (ctypes.c_int, []),
    "h3b_pack_by_dest": (ctypes.c_int, [_p, _i64, _i32, _i32, _i64, _i64, _i32, _p, _i32, _p, _p]),
    "h3b_unpack_recv": (ctypes.c_int, [_p, _i32, _i64, _i32, _i32, _p, _p]),
    "h3b_norm_rope_send": (ctypes.c_int, [_p, _i64, _i32, _i64, _i64, _p, _p, _i64, _i32, _f32, _i32, _p, _p]),
    "h3b_bf16_to_f16": (ctypes.c_int, [_p, _p, _i64, _p, _p]),
    "h3b_fp8_gemm_gate": (ctypes.c_int, [_p, _i64, _p, _i64, _p, _p, _p, _p, _i64, _p, _i64, _i64, _p, _p, _i64, _i64,
                                         _i64, _i64, _p]),
    "h3b_flash_attn_fwd_p2p": (ctypes.c_int, [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _p, _i32, _i32, _i64,
                                              _i64, _i64, _i64, _i32, _i32, _f32, _i32, _p, _p]),
    "h3b_flash_attn_fwd_p2p_bf16v": (ctypes.c_int, [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _p, _i32, _i32,
                                                    _i64, _i64, _i64, _i64, _i32, _i32, _f32, _p, _p, _p]),
    "h3b_p2p_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(_p), ctypes.POINTER(IpcHandle)]),
    "h3b_p2p_open": (ctypes.c_int, [ctypes.POINTER(IpcHandle), ctypes.POINTER(_p)]),
    "h3b_p2p_close": (ctypes.c_int, [_p]),
    "h3b_p2p_free": (ctypes.c_int, [_p]),
    "h3b_p2p_signal_wait": (ctypes.c_int, [_p, _p, _i32, _i32, _i32, _p]),
}

_lib = None


def load() -> ctypes.CDLL:
    """Load ``libh3b.so`` once (raises ``OSError`` with the build command when it is missing)."""
    global _lib
    if _lib is None:
        path = Path(os.environ.get("H3B_LIB", LIB_PATH))
        if not path.exists():
            raise OSError(f"h3b CUDA library not built: {path} is missing (run `python build.py` in "
                          f"{LIB_PATH.parent.parent})")
        lib = ctypes.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def last_error() -> str:
    return load().h3b_last_error().decode(errors="replace")


class H3BError(RuntimeError):
    def __init__(self, status: int, where: str, detail: str):
        super().__init__(f"{where}: {detail or 'h3b status ' + str(status)} (status {status})")
        self.status = status


def check(rc: int, where: str) -> None:
    if rc != H3B_OK:
        raise H3BError(rc, where, last_error())


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


def device_status() -> int:
    """Read and clear the sticky device status word (syncs the current device)."""
    return load().h3b_device_status()
