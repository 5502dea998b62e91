"""Tensor-level host API: the reference crate's IQ2 public functions, over the CUDA C ABI.

Mirrors src/iq2_matmul.rs of candelora-metal-kernels (same names, argument meaning, output
shape/dtype and error conditions), with torch CUDA tensors in place of candle Metal tensors:

  iq2_matmul(x, weight_bytes, weight_scales, out_dim, in_dim, variant)      :535-553
  iq2_matmul_with_activation_quant(..., variant, activation_quant)          :555-591
  iq2_dequantize_to_f16(weight_bytes, weight_scales, out_dim, in_dim, variant)  :593-602
  iq2_xxs_matmul / iq2_xs_matmul / iq2_s_matmul / iq3_s_matmul              :604-670
  Iq2MatmulVariant                                                          :31-37

`Iq2MatmulOp` is the op-struct form of the same call (candle's CustomOp3 shape: name /
cpu_fwd / cuda_fwd over (x, weight_bytes, weight_scales)); cpu_fwd refuses, there is no CPU
fallback. Every compute call goes through libcandelora_iq2.so on the current CUDA stream.

Errors raise `Iq2Error` carrying the reference's bail! message; the checks run in the
reference's order (iq2_matmul_metal, :210-259): non-zero dims, CUDA device, same device, U8
weights, x shape (parse_x_shape :170-195), size overflow, buffers too small.
"""
from __future__ import annotations

import ctypes
import enum

import torch

from . import _lib
from ._lib import Iq2Error
from .activation_quant import ActivationQuantConfig, ActivationQuantMode

QK = 256


class Iq2MatmulVariant(enum.IntEnum):
    """Iq2MatmulVariant (src/iq2_matmul.rs:31-37). Only Iq2Xxs has CUDA kernels."""

    Iq2Xxs = 0
    Iq2Xs = 1
    Iq2S = 2
    Iq3S = 3

    def bytes_per_block(self) -> int:      # src/iq2_matmul.rs:41-48
        return {0: 64, 1: 64, 2: 72, 3: 104}[int(self)]

    def scales_per_block(self) -> int:     # src/iq2_matmul.rs:50-57
        return {0: 2, 1: 10, 2: 10, 3: 6}[int(self)]


_X_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16}


def _bail(code: int, msg: str):
    raise Iq2Error(code, msg)


def _stream_handle(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _parse_x_shape(x: torch.Tensor, in_dim: int):
    """parse_x_shape (src/iq2_matmul.rs:170-195): [K] -> ([1, K], squeeze) or [M, K]."""
    if x.dim() == 1:
        if x.shape[0] != in_dim:
            _bail(_lib.IQ2_ERR_INVALID_ARGUMENT,
                  f"iq2_matmul input mismatch: x dim={x.shape[0]} expected in_dim={in_dim}")
        return x.reshape(1, in_dim), 1, True
    if x.dim() == 2:
        if x.shape[1] != in_dim:
            _bail(_lib.IQ2_ERR_INVALID_ARGUMENT,
                  f"iq2_matmul input mismatch: x last dim={x.shape[1]} expected in_dim={in_dim}")
        return x, x.shape[0], False
    _bail(_lib.IQ2_ERR_INVALID_ARGUMENT, f"iq2_matmul expects x rank 1 or 2, got shape {list(x.shape)}")


def _check_common(op: str, weight_bytes, weight_scales, out_dim, in_dim, x=None):
    if out_dim == 0 or in_dim == 0:
        _bail(_lib.IQ2_ERR_ZERO_DIM, f"{op} expects non-zero dimensions")
    first = x if x is not None else weight_bytes
    if first.device.type != "cuda":
        _bail(_lib.IQ2_ERR_DEVICE, f"{op} requires a CUDA device")
    if weight_bytes.device != first.device or weight_scales.device != first.device:
        if x is not None:
            _bail(_lib.IQ2_ERR_DEVICE, f"{op} device mismatch: x={x.device}, bytes={weight_bytes.device}, "
                                       f"scales={weight_scales.device}")
        _bail(_lib.IQ2_ERR_DEVICE, f"{op} device mismatch: bytes={weight_bytes.device}, "
                                   f"scales={weight_scales.device}")
    if weight_bytes.dtype != torch.uint8 or weight_scales.dtype != torch.uint8:
        _bail(_lib.IQ2_ERR_DTYPE, f"{op} expects U8 weight bytes/scales, got bytes={weight_bytes.dtype}, "
                                  f"scales={weight_scales.dtype}")


def _check_weight_layout(op, weight_bytes, weight_scales):
    if not weight_bytes.is_contiguous() or not weight_scales.is_contiguous():
        _bail(_lib.IQ2_ERR_INVALID_ARGUMENT, f"{op} expects contiguous layouts")


def workspace_bytes(m: int, out_dim: int, in_dim: int, x_dtype: torch.dtype,
                    variant: Iq2MatmulVariant = Iq2MatmulVariant.Iq2Xxs) -> int:
    """Device scratch the C ABI needs for this call (iq2_matmul_workspace_size)."""
    return int(_lib.load().iq2_matmul_workspace_size(m, out_dim, in_dim, _X_DTYPES[x_dtype], int(variant)))


def _matmul(x, weight_bytes, weight_scales, out_dim, in_dim, variant, act_mode=_lib.ACT_QUANT_OFF,
            strict=False, out=None, workspace=None):
    lib = _lib.load()
    op = "iq2_matmul"
    _check_common(op, weight_bytes, weight_scales, out_dim, in_dim, x)
    x2, m, squeeze = _parse_x_shape(x, in_dim)
    x2 = x2.contiguous()
    if x2.dtype not in _X_DTYPES:
        _bail(_lib.IQ2_ERR_DTYPE, f"iq2_matmul unsupported x dtype: {x2.dtype}")
    _check_weight_layout(op, weight_bytes, weight_scales)
    if out is None:
        out = torch.empty((m, out_dim), dtype=torch.float32, device=x.device)
    else:
        if out.shape != (m, out_dim) or out.dtype != torch.float32 or not out.is_contiguous() \
                or out.device != x.device:
            _bail(_lib.IQ2_ERR_INVALID_ARGUMENT, f"{op}: out must be a contiguous f32 [{m}, {out_dim}] tensor "
                                                 f"on {x.device}")
    ws_need = int(lib.iq2_matmul_with_activation_quant_workspace_size(m, out_dim, in_dim, _X_DTYPES[x2.dtype],
                                                                      int(variant), int(act_mode))) if m else 0
    if ws_need == 0:
        ws_ptr, ws_len = None, 0  # this call needs no scratch at all
    else:
        if workspace is None or workspace.numel() < ws_need:
            workspace = torch.empty(ws_need, dtype=torch.uint8, device=x.device)
        ws_ptr, ws_len = workspace.data_ptr(), workspace.numel()
    with torch.cuda.device(x.device):
        rc = lib.iq2_matmul_with_activation_quant(
            ctypes.c_void_p(x2.data_ptr()), _X_DTYPES[x2.dtype], m,
            ctypes.c_void_p(weight_bytes.data_ptr()), weight_bytes.numel(),
            ctypes.c_void_p(weight_scales.data_ptr()), weight_scales.numel(),
            out_dim, in_dim, int(variant), act_mode, int(bool(strict)),
            ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(ws_ptr), ws_len,
            _stream_handle(x.device))
    _lib.check(rc)
    return out.squeeze(0) if squeeze else out


def iq2_matmul(x: torch.Tensor, weight_bytes: torch.Tensor, weight_scales: torch.Tensor, out_dim: int,
               in_dim: int, variant: Iq2MatmulVariant = Iq2MatmulVariant.Iq2Xxs, *, out=None,
               workspace=None) -> torch.Tensor:
    """Generic entry point (src/iq2_matmul.rs:535-553): f32 [m, out_dim] (or [out_dim] for a
    rank-1 x) = x @ dequant(weights)^T. `out`/`workspace` let a caller reuse buffers."""
    return _matmul(x, weight_bytes, weight_scales, out_dim, in_dim, variant, out=out, workspace=workspace)


def iq2_matmul_with_activation_quant(x, weight_bytes, weight_scales, out_dim, in_dim,
                                     variant: Iq2MatmulVariant,
                                     activation_quant: ActivationQuantConfig, *, out=None, workspace=None):
    """src/iq2_matmul.rs:555-591. Off -> iq2_matmul. W4A8 -> error if strict, else iq2_matmul.
    W8A8 -> the reference's W8A8 numerics (each x row quantised to int8 with 127/max|x| and back,
    src/metal_src/iq2_matmul.metal:85-102), then the matmul."""
    mode = ActivationQuantMode(activation_quant.mode)
    return _matmul(x, weight_bytes, weight_scales, out_dim, in_dim, variant, act_mode=int(mode),
                   strict=activation_quant.strict, out=out, workspace=workspace)


def iq2_matmul_grouped(problems, *, workspace=None):
    """Several IQ2_XXS projections with the same m and x dtype in as few launches as possible
    (iq2_matmul_grouped in the C ABI; no reference counterpart -- the reference dispatches one
    projection at a time). `problems` is a sequence of (x, weight_bytes, weight_scales, out_dim,
    in_dim) or (..., out) tuples, x of shape [m, in_dim]; returns the list of f32 outputs."""
    lib = _lib.load()
    op = "iq2_matmul_grouped"
    if not problems:
        return []
    outs, keep = [], []
    arr = (_lib.Iq2MatmulProblem * len(problems))()
    m = dtype = device = None
    for i, pr in enumerate(problems):
        x, wb, ws, out_dim, in_dim = pr[:5]
        out = pr[5] if len(pr) > 5 else None
        _check_common(op, wb, ws, out_dim, in_dim, x)
        x2, mi, _ = _parse_x_shape(x, in_dim)
        x2 = x2.contiguous()
        _check_weight_layout(op, wb, ws)
        if x2.dtype not in _X_DTYPES:
            _bail(_lib.IQ2_ERR_DTYPE, f"iq2_matmul unsupported x dtype: {x2.dtype}")
        if m is None:
            m, dtype, device = mi, x2.dtype, x.device
        elif mi != m or x2.dtype != dtype or x.device != device:
            _bail(_lib.IQ2_ERR_INVALID_ARGUMENT, f"{op}: every problem needs the same m, x dtype and device")
        if out is None:
            out = torch.empty((mi, out_dim), dtype=torch.float32, device=x.device)
        keep.append(x2)
        outs.append(out)
        arr[i] = _lib.Iq2MatmulProblem(x2.data_ptr(), wb.data_ptr(), wb.numel(), ws.data_ptr(), ws.numel(),
                                       out_dim, in_dim, out.data_ptr())
    with torch.cuda.device(device):
        need = int(lib.iq2_matmul_grouped_workspace_size(arr, len(problems), m, _X_DTYPES[dtype]))
        if workspace is None or workspace.numel() < need:
            workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=device)
        rc = lib.iq2_matmul_grouped(arr, len(problems), m, _X_DTYPES[dtype], ctypes.c_void_p(workspace.data_ptr()),
                                    workspace.numel(), _stream_handle(device))
    _lib.check(rc)
    return outs


def grouped_workspace_bytes(problems) -> int:
    """Workspace iq2_matmul_grouped needs for these (x, weight_bytes, weight_scales, out_dim,
    in_dim[, out]) problems (the output pointers do not affect the size)."""
    lib = _lib.load()
    arr = (_lib.Iq2MatmulProblem * len(problems))()
    m = dtype = None
    for i, pr in enumerate(problems):
        x, wb, ws, out_dim, in_dim = pr[:5]
        x2, mi, _ = _parse_x_shape(x, in_dim)
        m, dtype = mi, x2.dtype
        arr[i] = _lib.Iq2MatmulProblem(x2.data_ptr(), wb.data_ptr(), wb.numel(), ws.data_ptr(), ws.numel(),
                                       out_dim, in_dim, None)
    return int(lib.iq2_matmul_grouped_workspace_size(arr, len(problems), m, _X_DTYPES[dtype]))


def device_check(device=None) -> None:
    """Raise Iq2Error (IQ2_ERR_TIMEOUT) if a kernel of this library on `device` (default: the
    current one) gave up on a bounded in-kernel wait since the previous check, i.e. some call's
    outputs are incomplete although the call returned. Synchronises the device; clears the status."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().iq2_device_check())


def iq2_dequantize(weight_bytes, weight_scales, out_dim, in_dim, variant=Iq2MatmulVariant.Iq2Xxs,
                   dtype: torch.dtype = torch.float16, out=None) -> torch.Tensor:
    """Dense [out_dim, in_dim] weights in f16 (reference-identical), bf16 (RNE) or f32 (exact)."""
    lib = _lib.load()
    op = "iq2_dequantize_to_f16"
    _check_common(op, weight_bytes, weight_scales, out_dim, in_dim)
    _check_weight_layout(op, weight_bytes, weight_scales)
    codes = {torch.float32: _lib.DTYPE_F32, torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16}
    if dtype not in codes:
        _bail(_lib.IQ2_ERR_DTYPE, f"{op} unsupported out dtype: {dtype}")
    if out is None:
        out = torch.empty((out_dim, in_dim), dtype=dtype, device=weight_bytes.device)
    with torch.cuda.device(weight_bytes.device):
        rc = lib.iq2_dequantize(ctypes.c_void_p(weight_bytes.data_ptr()), weight_bytes.numel(),
                                ctypes.c_void_p(weight_scales.data_ptr()), weight_scales.numel(),
                                out_dim, in_dim, int(variant), ctypes.c_void_p(out.data_ptr()), codes[dtype],
                                _stream_handle(weight_bytes.device))
    _lib.check(rc)
    return out


def iq2_dequantize_to_f16(weight_bytes, weight_scales, out_dim, in_dim,
                          variant: Iq2MatmulVariant = Iq2MatmulVariant.Iq2Xxs) -> torch.Tensor:
    """src/iq2_matmul.rs:593-602: dense F16 [out_dim, in_dim]."""
    return iq2_dequantize(weight_bytes, weight_scales, out_dim, in_dim, variant, torch.float16)


def iq2_xxs_matmul(x, weight_bytes, weight_scales, out_dim, in_dim, **kw):
    """src/iq2_matmul.rs:604-619."""
    return iq2_matmul(x, weight_bytes, weight_scales, out_dim, in_dim, Iq2MatmulVariant.Iq2Xxs, **kw)


def iq2_xs_matmul(x, weight_bytes, weight_scales, out_dim, in_dim, **kw):
    """src/iq2_matmul.rs:621-636 (no CUDA kernel: raises Iq2Error IQ2_ERR_UNSUPPORTED)."""
    return iq2_matmul(x, weight_bytes, weight_scales, out_dim, in_dim, Iq2MatmulVariant.Iq2Xs, **kw)


def iq2_s_matmul(x, weight_bytes, weight_scales, out_dim, in_dim, **kw):
    """src/iq2_matmul.rs:638-653 (no CUDA kernel: raises Iq2Error IQ2_ERR_UNSUPPORTED)."""
    return iq2_matmul(x, weight_bytes, weight_scales, out_dim, in_dim, Iq2MatmulVariant.Iq2S, **kw)


def iq3_s_matmul(x, weight_bytes, weight_scales, out_dim, in_dim, **kw):
    """src/iq2_matmul.rs:655-670 (no CUDA kernel: raises Iq2Error IQ2_ERR_UNSUPPORTED)."""
    return iq2_matmul(x, weight_bytes, weight_scales, out_dim, in_dim, Iq2MatmulVariant.Iq3S, **kw)


class Iq2MatmulOp:
    """Op-struct form of iq2_matmul over (x, weight_bytes, weight_scales), shaped like the candle
    CustomOp3 the Rust drop-in implements (name / cpu_fwd / cuda_fwd)."""

    def __init__(self, out_dim: int, in_dim: int, variant: Iq2MatmulVariant = Iq2MatmulVariant.Iq2Xxs,
                 activation_quant: ActivationQuantConfig = ActivationQuantConfig()):
        self.out_dim = out_dim
        self.in_dim = in_dim
        self.variant = Iq2MatmulVariant(variant)
        self.activation_quant = activation_quant

    def name(self) -> str:
        return "candelora_iq2_matmul"

    def cpu_fwd(self, *args, **kw):
        raise Iq2Error(_lib.IQ2_ERR_DEVICE, "iq2_matmul requires a CUDA device")

    def cuda_fwd(self, x, weight_bytes, weight_scales, **kw):
        return iq2_matmul_with_activation_quant(x, weight_bytes, weight_scales, self.out_dim, self.in_dim,
                                                self.variant, self.activation_quant, **kw)

    def __call__(self, x, weight_bytes, weight_scales, **kw):
        if x.device.type != "cuda":
            return self.cpu_fwd(x, weight_bytes, weight_scales)
        return self.cuda_fwd(x, weight_bytes, weight_scales, **kw)
