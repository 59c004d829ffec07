"""ctypes binding of libvmlx_cuda.so (the C ABI declared in include/vmlx_cuda.h).

The library is built in-tree (``vmlx-swift_b200/libvmlx_cuda.so``) by
``vmlx-swift_b200/csrc/Makefile``.  There is no fallback: if the library is
missing or fails to load, every op raises.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libvmlx_cuda.so")
CSRC = os.path.join(_HERE, "csrc")

VMLX_OK = 0
VMLX_E_INVALID = 1
VMLX_E_UNSUPPORTED = 2
VMLX_E_CUDA = 3
VMLX_E_PEER_TIMEOUT = 4
VMLX_E_STATE = 5

VMLX_BF16 = 0
VMLX_F32 = 1

_c = ctypes
_vp = _c.c_void_p
_i64 = _c.c_int64
_int = _c.c_int
_bool = _c.c_bool
_str = _c.c_char_p
_sz = _c.c_size_t

# name -> (restype, argtypes); every symbol of include/vmlx_cuda.h
SIGNATURES = {
    "vmlx_last_error": (_str, []),
    "vmlx_version": (_int, []),
    "vmlx_set_launch_overlap": (_int, [_int]),
    "vmlx_cuda_quantize": (_int, [_vp, _vp, _vp, _vp, _int, _i64, _i64, _int, _int, _str, _vp]),
    "vmlx_cuda_dequantize": (_int, [_vp, _int, _vp, _vp, _vp, _int, _i64, _i64, _int, _int, _str, _vp]),
    "vmlx_cuda_quantized_matmul": (
        _int, [_vp, _vp, _vp, _vp, _vp, _bool, _int, _int, _str, _i64, _i64, _i64, _vp]),
    "vmlx_cuda_quantized_matmul_fused": (
        _int, [_vp, _vp, _vp, _vp, _vp, _int, _int, _i64, _i64, _i64, _vp, _c.c_float, _vp, _vp]),
    "vmlx_cuda_gather_qmm": (
        _int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _bool, _int, _int, _str, _bool, _i64, _i64,
               _i64, _i64, _i64, _i64, _vp]),
    "vmlx_cuda_gather_qmm_workspace_size": (_sz, [_i64, _i64, _i64, _i64]),
    "vmlx_cuda_gather_qmm_ws": (
        _int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _bool, _int, _int, _str, _bool, _i64, _i64,
               _i64, _i64, _i64, _i64, _vp, _sz, _vp]),
    "vmlx_cuda_moe_route": (_int, [_vp, _int, _i64, _int, _int, _bool, _vp, _vp, _vp]),
    "vmlx_cuda_moe_sort": (_int, [_vp, _i64, _int, _int, _vp, _vp, _vp, _vp, _vp]),
    "vmlx_cuda_moe_combine": (_int, [_vp, _vp, _vp, _int, _i64, _int, _i64, _vp, _vp]),
    "vmlx_cuda_rms_norm": (_int, [_vp, _vp, _vp, _c.c_float, _i64, _i64, _vp]),
    "vmlx_cuda_rope_qkv": (_int, [_vp, _vp, _vp, _vp, _i64, _int, _int, _int, _i64, _i64, _c.c_float,
                                  _c.c_float, _vp]),
    "vmlx_cuda_sdpa_decode_workspace": (_sz, [_i64, _int, _i64, _int]),
    "vmlx_cuda_sdpa_decode": (_int, [_vp, _vp, _vp, _vp, _i64, _int, _int, _int, _i64, _i64, _c.c_float, _vp,
                                     _sz, _vp]),
    "vmlx_cuda_sdpa_decode_noalloc": (_int, [_vp, _vp, _vp, _vp, _i64, _int, _int, _int, _i64, _i64,
                                             _c.c_float, _vp]),
    "vmlx_cuda_silu_mul": (_int, [_vp, _vp, _i64, _i64, _vp]),
    "vmlx_cuda_add": (_int, [_vp, _vp, _vp, _i64, _vp]),
    "vmlx_cuda_bias_add": (_int, [_vp, _vp, _vp, _i64, _i64, _vp]),
    "vmlx_cuda_fp_quantize": (_int, [_vp, _vp, _vp, _int, _i64, _i64, _int, _int, _str, _vp]),
    "vmlx_cuda_fp_dequantize": (_int, [_vp, _int, _vp, _vp, _i64, _i64, _int, _int, _str, _vp]),
    "vmlx_cuda_fp_quantized_matmul": (_int, [_vp, _vp, _vp, _vp, _int, _int, _str, _i64, _i64, _i64, _vp]),
    "vmlx_cuda_quantized_embedding": (_int, [_vp, _vp, _vp, _vp, _vp, _int, _int, _i64, _i64, _i64, _vp, _vp]),
    "vmlx_cuda_rope_qk_norm": (_int, [_vp, _vp, _vp, _vp, _i64, _int, _int, _int, _vp, _i64, _int, _i64, _vp, _vp,
                                      _c.c_float, _c.c_float, _c.c_float, _vp, _vp]),
    "vmlx_cuda_sdpa_decode_at": (_int, [_vp, _vp, _vp, _vp, _i64, _int, _int, _int, _vp, _i64, _c.c_float, _vp, _sz,
                                        _vp]),
    "vmlx_cuda_argmax": (_int, [_vp, _vp, _i64, _i64, _vp]),
    "vmlx_cuda_advance": (_int, [_vp, _c.c_int32, _vp]),
    "vmlx_tp_create": (_int, [_int, _int, _sz, _c.POINTER(_vp)]),
    "vmlx_tp_create_loopback": (_int, [_int, _sz, _c.POINTER(_vp)]),
    "vmlx_tp_moe_combine_all_sum": (_int, [_vp, _vp, _vp, _vp, _vp, _int, _i64, _int, _i64, _vp, _vp]),
    "vmlx_tp_rank": (_int, [_vp]),
    "vmlx_tp_size": (_int, [_vp]),
    "vmlx_tp_ipc_handle": (_int, [_vp, _vp]),
    "vmlx_tp_open_peers": (_int, [_vp, _vp]),
    "vmlx_tp_set_peer": (_int, [_vp, _int, _vp]),
    "vmlx_tp_buffer": (_vp, [_vp]),
    "vmlx_tp_set_timeout_us": (_int, [_vp, _c.c_uint64]),
    "vmlx_tp_all_sum": (_int, [_vp, _vp, _vp, _i64, _vp]),
    "vmlx_tp_quantized_matmul_all_sum": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _int, _int, _i64, _i64, _i64,
                                                _vp, _vp]),
    "vmlx_tp_quantized_matmul_swiglu_all_sum": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _int, _int, _i64, _i64,
                                                       _i64, _vp, _vp]),
    "vmlx_cuda_quantized_matmul_swiglu": (_int, [_vp, _vp, _vp, _vp, _vp, _int, _int, _i64, _i64, _i64, _vp, _vp]),
    "vmlx_tp_status": (_int, [_vp, _c.POINTER(_int)]),
    "vmlx_tp_destroy": (_int, [_vp]),
}

_lock = threading.Lock()
_lib = None


class VMLXError(RuntimeError):
    """Raised when a C-ABI call returns nonzero; carries the return code."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"vmlx error {code}: {msg}")
        self.code = code


def build(force: bool = False) -> str:
    """Compile libvmlx_cuda.so for sm_100a (nvcc cross-compiles without a GPU)."""
    args = ["make", "-s", "-j8", "-C", CSRC]
    if force:
        subprocess.run(["make", "-s", "-C", CSRC, "clean"], check=True)
    subprocess.run(args, check=True)
    return LIB_PATH


def lib():
    """Load (once) and return the ctypes handle of libvmlx_cuda.so."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `make -C {CSRC}` "
                    "(there is no CPU fallback)")
            h = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(h, name)
                fn.restype = res
                fn.argtypes = args
            _lib = h
    return _lib


def check(rc: int) -> None:
    if rc != VMLX_OK:
        msg = lib().vmlx_last_error()
        raise VMLXError(rc, msg.decode() if msg else "")
