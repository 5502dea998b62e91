"""TEST INFRASTRUCTURE ONLY: numpy front end for the two CPU parity checkers.

* ``Oracle``    -- the C restatement of the reference's scalar CPU path (oracle/iq2xxs_oracle.c,
                   which cites the reference file:line of every function it restates).
* ``RefKernels`` -- the reference's own Metal kernels compiled from their source as C++
                   (oracle/ref_harness.cpp + oracle/metal_shim/), i.e. the reference itself run
                   on host cores. Present only where oracle/_ref/libiq2ref.so was built (it needs
                   the reference checkout at build time; the built file travels with the repo).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this module. The
library under candelora_metal_kernels_b200/ never does: its product path is CUDA only.

Also here: the reference's own test-fixture generators (src/iq2_matmul.rs:765-787), in numpy.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "libiq2oracle.so"
REF_SO = HERE / "_ref" / "libiq2ref.so"

QK = 256
# Where a checkout of the reference crate is looked for: $CANDELORA_REFERENCE_DIR, else a directory
# named "reference" beside this repository. It is needed only to (re)build oracle/_ref and to
# regenerate tables; nothing run on a GPU box reads it.
REFERENCE_ENV = "CANDELORA_REFERENCE_DIR"


def reference_dir() -> Path | None:
    """The reference checkout (see REFERENCE_ENV), or None when there is none."""
    cand = os.environ.get(REFERENCE_ENV) or str(HERE.parent.parent / "reference")
    p = Path(cand)
    return p if (p / "src/metal_src/iq2_matmul.metal").is_file() else None


DTYPE_CODE = {"f32": 0, "f16": 1, "bf16": 2}
VARIANT_CODE = {"iq2_xxs": 0, "iq2_xs": 1, "iq2_s": 2, "iq3_s": 3}
# (weight bytes, scale bytes) per 256-weight block (src/iq2_matmul.rs:15-29)
BLOCK_BYTES = {"iq2_xxs": (64, 2), "iq2_xs": (64, 10), "iq2_s": (72, 10), "iq3_s": (104, 6)}

_c_f32p = ctypes.POINTER(ctypes.c_float)
_c_u8p = ctypes.POINTER(ctypes.c_uint8)
_c_u16p = ctypes.POINTER(ctypes.c_uint16)
_c_i64p = ctypes.POINTER(ctypes.c_int64)


def _ptr(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def build(ref: str | None = None) -> None:
    """Compile the checkers (make -C oracle). `_ref` is built only when the reference exists."""
    targets = ["oracle"]
    ref_path = Path(ref) if ref else reference_dir()
    args = []
    if ref_path is not None and (ref_path / "src/metal_src/iq2_matmul.metal").is_file():
        targets.append("ref")
        args.append(f"REF={ref_path}")
    subprocess.run(["make", "-s", "-C", str(HERE), *args, *targets], check=True)


# ----------------------------------------------------------------------------- fixtures
def lcg_fill(length: int, seed: int) -> np.ndarray:
    """lcg_fill (src/iq2_matmul.rs:765-773): state = state*1664525 + 1013904223; byte = state>>24."""
    out = np.empty(length, dtype=np.uint8)
    state = seed & 0xFFFFFFFF
    for i in range(length):
        state = (state * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = state >> 24
    return out


def deterministic_x(m: int, in_dim: int) -> np.ndarray:
    """deterministic_x (src/iq2_matmul.rs:775-779): x[i] = ((i*17) % 41 - 20) / 13 in f32."""
    i = np.arange(m * in_dim, dtype=np.int64)
    v = ((i * 17) % 41).astype(np.float32) - np.float32(20.0)
    return (v / np.float32(13.0)).astype(np.float32).reshape(m, in_dim)


def force_f16_one_per_block(scales: np.ndarray, scales_per_block: int) -> np.ndarray:
    """force_f16_one_per_block (src/iq2_matmul.rs:781-787): every block's d := f16 1.0 (0x3C00)."""
    s = scales.copy()
    nblk = len(s) // scales_per_block
    s[: nblk * scales_per_block].reshape(nblk, scales_per_block)[:, 0] = 0x00
    s[: nblk * scales_per_block].reshape(nblk, scales_per_block)[:, 1] = 0x3C
    return s


def reference_parity_fixture(m=2, out_dim=7, in_dim=320, bytes_seed=0xA11CE5ED,
                             scales_seed=0xC0FFEE12, last_byte=0x5A, variant="iq2_xxs"):
    """The inputs of the reference's parity_case(variant) (src/iq2_matmul.rs:1065-1100): LCG
    weight bytes and scales, every d forced to 1.0, last weight byte forced, x from
    deterministic_x. Returns (x f32 [m,in_dim], weight_bytes u8, weight_scales u8)."""
    nb = (in_dim + QK - 1) // QK
    nblocks = out_dim * nb
    bpb, spb = BLOCK_BYTES[variant]
    wb = lcg_fill(nblocks * bpb, bytes_seed)
    ws = force_f16_one_per_block(lcg_fill(nblocks * spb, scales_seed), spb)
    if last_byte is not None and len(wb):
        wb[-1] = last_byte
    return deterministic_x(m, in_dim), wb, ws


# ----------------------------------------------------------------------------- C restatement
class Oracle:
    """The C restatement of the reference CPU path."""

    def __init__(self, path: Path = ORACLE_SO):
        if not path.is_file():
            raise FileNotFoundError(f"{path} not built (run make -C oracle)")
        lib = ctypes.CDLL(str(path))
        lib.oracle_iq2xxs_matmul_f32.argtypes = [_c_f32p, ctypes.c_size_t, ctypes.c_size_t,
                                                 ctypes.c_size_t, _c_u8p, _c_u8p, _c_i64p,
                                                 ctypes.c_size_t, _c_f32p, ctypes.c_int]
        lib.oracle_iq2xxs_dequantize.argtypes = [_c_u8p, _c_u8p, ctypes.c_size_t, ctypes.c_size_t,
                                                 ctypes.c_int, ctypes.c_void_p, ctypes.c_int]
        lib.oracle_widen_x.argtypes = [_c_u16p, ctypes.c_int, ctypes.c_size_t, _c_f32p]
        lib.oracle_iq2_matmul_f32.argtypes = [ctypes.c_int, _c_f32p, ctypes.c_size_t, ctypes.c_size_t,
                                              ctypes.c_size_t, _c_u8p, _c_u8p, _c_i64p, ctypes.c_size_t,
                                              _c_f32p, ctypes.c_int]
        lib.oracle_iq2_dequantize.argtypes = [ctypes.c_int, _c_u8p, _c_u8p, ctypes.c_size_t, ctypes.c_size_t,
                                              ctypes.c_int, ctypes.c_void_p, ctypes.c_int]
        lib.oracle_rowwise_qdq_w8a8.argtypes = [_c_f32p, ctypes.c_size_t, ctypes.c_size_t, _c_f32p]
        lib.oracle_f32_to_f16.argtypes = [ctypes.c_float]
        lib.oracle_f32_to_f16.restype = ctypes.c_uint16
        lib.oracle_f32_to_bf16.argtypes = [ctypes.c_float]
        lib.oracle_f32_to_bf16.restype = ctypes.c_uint16
        self.lib = lib

    @staticmethod
    def _check(wb, ws, out_dim, in_dim, variant="iq2_xxs"):
        nb = (in_dim + QK - 1) // QK
        bpb, spb = BLOCK_BYTES[variant]
        assert wb.dtype == np.uint8 and ws.dtype == np.uint8
        assert wb.size >= out_dim * nb * bpb and ws.size >= out_dim * nb * spb

    def widen_x(self, x16: np.ndarray, dtype: str) -> np.ndarray:
        """f16/bf16 bit patterns (uint16) -> f32, as the reference kernels' float(x)."""
        x16 = np.ascontiguousarray(x16, dtype=np.uint16)
        out = np.empty(x16.shape, dtype=np.float32)
        self.lib.oracle_widen_x(_ptr(x16, _c_u16p), DTYPE_CODE[dtype], x16.size, _ptr(out, _c_f32p))
        return out

    def matmul(self, x: np.ndarray, wb: np.ndarray, ws: np.ndarray, out_dim: int, in_dim: int,
               cols=None, threads: int = 0, x_dtype: str = "f32", variant: str = "iq2_xxs") -> np.ndarray:
        """Reference matmul: x [m, in_dim] (f32, or uint16 bit patterns for f16/bf16) -> f32
        [m, out_dim] (or [m, len(cols)] for a column sample)."""
        self._check(wb, ws, out_dim, in_dim, variant)
        if x_dtype != "f32":
            x = self.widen_x(x, x_dtype)
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, in_dim)
        m = x.shape[0]
        wb = np.ascontiguousarray(wb)
        ws = np.ascontiguousarray(ws)
        if cols is not None:
            cols = np.ascontiguousarray(cols, dtype=np.int64)
            out = np.empty((m, cols.size), dtype=np.float32)
            cp = _ptr(cols, _c_i64p)
            nc = cols.size
        else:
            out = np.empty((m, out_dim), dtype=np.float32)
            cp, nc = None, 0
        threads = threads or (os.cpu_count() or 1)
        self.lib.oracle_iq2_matmul_f32(VARIANT_CODE[variant], _ptr(x, _c_f32p), m, out_dim, in_dim,
                                       _ptr(wb, _c_u8p), _ptr(ws, _c_u8p), cp, nc, _ptr(out, _c_f32p), threads)
        return out

    def dequantize(self, wb, ws, out_dim, in_dim, out_dtype="f16", threads: int = 0,
                   variant: str = "iq2_xxs") -> np.ndarray:
        """Dense [out_dim, in_dim]: f32 values, or f16/bf16 RNE bit patterns (uint16)."""
        self._check(wb, ws, out_dim, in_dim, variant)
        code = DTYPE_CODE[out_dtype]
        out = np.empty((out_dim, in_dim), dtype=np.float32 if code == 0 else np.uint16)
        self.lib.oracle_iq2_dequantize(VARIANT_CODE[variant], _ptr(np.ascontiguousarray(wb), _c_u8p),
                                       _ptr(np.ascontiguousarray(ws), _c_u8p), out_dim, in_dim,
                                       code, out.ctypes.data, threads or (os.cpu_count() or 1))
        return out

    def rowwise_qdq_w8a8(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty_like(x)
        self.lib.oracle_rowwise_qdq_w8a8(_ptr(x, _c_f32p), x.shape[0], x.shape[1], _ptr(out, _c_f32p))
        return out


# ----------------------------------------------------------------------------- reference kernels
class RefKernels:
    """The reference's own Metal kernels, compiled from source as C++ and run on host cores."""

    def __init__(self, path: Path = REF_SO):
        if not path.is_file():
            raise FileNotFoundError(f"{path} not built (make -C oracle ref, needs the reference)")
        lib = ctypes.CDLL(str(path))
        lib.iq2ref_matmul.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_uint32,
                                      ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p, _c_u8p,
                                      _c_u8p, _c_f32p, ctypes.c_int]
        lib.iq2ref_dequantize_f16.argtypes = [ctypes.c_int, ctypes.c_uint32, ctypes.c_uint32,
                                              _c_u8p, _c_u8p, _c_u16p, ctypes.c_int]
        lib.iq2ref_max_threads.restype = ctypes.c_int
        self.lib = lib

    @staticmethod
    def available() -> bool:
        return REF_SO.is_file()

    def max_threads(self) -> int:
        return int(self.lib.iq2ref_max_threads())

    def matmul(self, x: np.ndarray, wb, ws, out_dim: int, in_dim: int, x_dtype="f32",
               variant="iq2_xxs", w8a8=False, threads: int = 0) -> np.ndarray:
        """x: f32 [m, in_dim], or uint16 bit patterns for x_dtype f16/bf16."""
        want = np.float32 if x_dtype == "f32" else np.uint16
        x = np.ascontiguousarray(x, dtype=want).reshape(-1, in_dim)
        out = np.zeros((x.shape[0], out_dim), dtype=np.float32)
        rc = self.lib.iq2ref_matmul(VARIANT_CODE[variant], int(w8a8), DTYPE_CODE[x_dtype],
                                    x.shape[0], out_dim, in_dim, x.ctypes.data,
                                    _ptr(np.ascontiguousarray(wb), _c_u8p),
                                    _ptr(np.ascontiguousarray(ws), _c_u8p), _ptr(out, _c_f32p),
                                    threads)
        if rc != 0:
            raise ValueError(f"iq2ref_matmul rc={rc}")
        return out

    def dequantize_f16(self, wb, ws, out_dim: int, in_dim: int, variant="iq2_xxs",
                       threads: int = 0) -> np.ndarray:
        out = np.zeros((out_dim, in_dim), dtype=np.uint16)
        rc = self.lib.iq2ref_dequantize_f16(VARIANT_CODE[variant], out_dim, in_dim,
                                            _ptr(np.ascontiguousarray(wb), _c_u8p),
                                            _ptr(np.ascontiguousarray(ws), _c_u8p),
                                            _ptr(out, _c_u16p), threads)
        if rc != 0:
            raise ValueError(f"iq2ref_dequantize_f16 rc={rc}")
        return out
