"""ctypes binding of the C ABI in include/candelora_iq2.h (libcandelora_iq2.so).

There is no fallback: if the CUDA library is missing, loading fails loudly.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libcandelora_iq2.so"

# Status codes (enum iq2_status).
IQ2_OK = 0
IQ2_ERR_INVALID_ARGUMENT = 1
IQ2_ERR_ZERO_DIM = 2
IQ2_ERR_DEVICE = 3
IQ2_ERR_DTYPE = 4
IQ2_ERR_OVERFLOW = 5
IQ2_ERR_TOO_SMALL = 6
IQ2_ERR_UNSUPPORTED = 7
IQ2_ERR_WORKSPACE = 8
IQ2_ERR_CUDA = 9
IQ2_ERR_COMM = 10
IQ2_ERR_TIMEOUT = 11
IQ2_COMM_ID_BYTES = 128

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
ACT_QUANT_OFF, ACT_QUANT_W8A8, ACT_QUANT_W4A8 = 0, 1, 2

# Every symbol the headers (include/candelora_iq2.h, include/candelora_iq2_testing.h) declare,
# with its C signature.
_vp, _u32, _sz, _int = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_size_t, ctypes.c_int
SIGNATURES = {
    "iq2_last_error": ([], ctypes.c_char_p),
    "iq2_abi_version": ([], _int),
    "iq2_device_check": ([], _int),
    "iq2_testing_set_gemm_stall": ([ctypes.c_uint64, _u32], _int),
    "iq2_matmul_workspace_size": ([_u32, _u32, _u32, _int, _int], _sz),
    "iq2_matmul": ([_vp, _int, _u32, _vp, _sz, _vp, _sz, _u32, _u32, _int, _vp, _vp, _sz, _vp], _int),
    "iq2_matmul_with_activation_quant": (
        [_vp, _int, _u32, _vp, _sz, _vp, _sz, _u32, _u32, _int, _int, _int, _vp, _vp, _sz, _vp], _int),
    "iq2_matmul_with_activation_quant_workspace_size": ([_u32, _u32, _u32, _int, _int, _int], _sz),
    "iq2_matmul_grouped_workspace_size": ([_vp, _u32, _u32, _int], _sz),
    "iq2_matmul_grouped": ([_vp, _u32, _u32, _int, _vp, _sz, _vp], _int),
    "iq2_matmul_noalloc": ([_vp, _int, _u32, _vp, _sz, _vp, _sz, _u32, _u32, _vp, _vp], _int),
    "iq2_dequantize": ([_vp, _sz, _vp, _sz, _u32, _u32, _int, _vp, _int, _vp], _int),
    "iq2_gather_columns": ([_vp, _u32, _u32, _u32, _vp, _vp], _int),
    "iq2_split_interleaved": ([_vp, _sz, ctypes.c_uint64, _int, _vp, _vp, _vp], _int),
    "iq2_comm_unique_id": ([_vp], _int),
    "iq2_comm_init": ([_vp, _int, _int, _vp], _int),
    "iq2_comm_init_with_timeout": ([_vp, _int, _int, _u32, _vp], _int),
    "iq2_comm_destroy": ([_vp], _int),
    "iq2_comm_symmetric_alloc": ([_vp, _sz, _vp], _int),
    "iq2_comm_check": ([_vp], _int),
    "iq2_matmul_grouped_sharded_workspace_size": ([_vp, _u32, _u32, _int, _int], _sz),
    "iq2_matmul_grouped_sharded": ([_vp, _vp, _u32, _u32, _int, _vp, _sz, _vp], _int),
}


class Iq2MatmulProblem(ctypes.Structure):
    """struct iq2_matmul_problem."""

    _fields_ = [("x", ctypes.c_void_p), ("weight_bytes", ctypes.c_void_p), ("weight_bytes_len", ctypes.c_size_t),
                ("weight_scales", ctypes.c_void_p), ("weight_scales_len", ctypes.c_size_t),
                ("out_dim", ctypes.c_uint32), ("in_dim", ctypes.c_uint32), ("out", ctypes.c_void_p)]


class Iq2Error(RuntimeError):
    """A failed C ABI call: `code` is the iq2_status value, the message is iq2_last_error()."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load the CUDA library (once). Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.is_file():
                raise ImportError(
                    f"{LIB_PATH} is missing: build the CUDA library first "
                    "(python -m candelora_metal_kernels_b200.build). There is no CPU fallback.")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (args, res) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = res
            _lib = lib
    return _lib


def check(rc: int) -> None:
    if rc != IQ2_OK:
        msg = load().iq2_last_error().decode(errors="replace")
        raise Iq2Error(rc, msg)
