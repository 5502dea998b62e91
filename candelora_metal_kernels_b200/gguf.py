"""Ingest of IQ2/IQ3 weights stored the way llama.cpp stores them: ggml's interleaved blocks,
optionally inside a GGUF file, turned into the split (weight_bytes, weight_scales) tensors the
matmul takes (the reference's own layout, src/iq2_matmul.rs:197-259).

ggml block layouts per 256 weights (fields in order, `d` an fp16):
  block_iq2_xxs  66 B: d, qs[64]
  block_iq2_xs   74 B: d, qs[64], scales[8]
  block_iq2_s    82 B: d, qs[64], qh[8], scales[8]
  block_iq3_s   110 B: d, qs[64], qh[8], signs[32], scales[4]
The split layout keeps everything but `d` and the trailing scale bytes in weight_bytes, and `d`
followed by those scale bytes in weight_scales (the repack runs on the GPU: iq2_split_interleaved).

GGUF (version 2 or 3): "GGUF", version, tensor count, metadata count, metadata key/values,
tensor infos (name, dims with ne[0] the fastest, ggml type, offset), then the data section at the
next multiple of general.alignment (32 by default). A weight matrix [out_dim, in_dim] has
ne = (in_dim, out_dim), so each output row's blocks are contiguous, as the matmul expects.
"""
from __future__ import annotations

import ctypes
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from . import _lib
from .iq2_matmul import Iq2MatmulVariant, _bail, _stream_handle

QK = 256
# ggml type ids of the formats the matmul reads
GGML_TYPE = {16: Iq2MatmulVariant.Iq2Xxs, 17: Iq2MatmulVariant.Iq2Xs, 21: Iq2MatmulVariant.Iq3S,
             22: Iq2MatmulVariant.Iq2S}
# (split weight bytes, split scale bytes) per block; the interleaved block is their sum
SPLIT = {Iq2MatmulVariant.Iq2Xxs: (64, 2), Iq2MatmulVariant.Iq2Xs: (64, 10), Iq2MatmulVariant.Iq2S: (72, 10),
         Iq2MatmulVariant.Iq3S: (104, 6)}

_MAGIC = 0x46554747  # "GGUF" little-endian
_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
_STRING, _ARRAY = 8, 9


def block_bytes(variant: Iq2MatmulVariant) -> int:
    b, s = SPLIT[Iq2MatmulVariant(variant)]
    return b + s


def split_interleaved(blocks: torch.Tensor, nblocks: int, variant: Iq2MatmulVariant = Iq2MatmulVariant.Iq2Xxs):
    """Interleaved ggml blocks (u8 CUDA tensor) -> (weight_bytes, weight_scales) on the same device."""
    variant = Iq2MatmulVariant(variant)
    bpb, spb = SPLIT[variant]
    if blocks.dtype != torch.uint8 or not blocks.is_contiguous():
        _bail(_lib.IQ2_ERR_INVALID_ARGUMENT, "split_interleaved expects contiguous u8 blocks")
    if blocks.device.type != "cuda":
        _bail(_lib.IQ2_ERR_DEVICE, "split_interleaved requires a CUDA device")
    wb = torch.empty(nblocks * bpb, dtype=torch.uint8, device=blocks.device)
    ws = torch.empty(nblocks * spb, dtype=torch.uint8, device=blocks.device)
    with torch.cuda.device(blocks.device):
        rc = _lib.load().iq2_split_interleaved(ctypes.c_void_p(blocks.data_ptr()), blocks.numel(), nblocks,
                                               int(variant), ctypes.c_void_p(wb.data_ptr()),
                                               ctypes.c_void_p(ws.data_ptr()), _stream_handle(blocks.device))
    _lib.check(rc)
    return wb, ws


@dataclass
class TensorInfo:
    name: str
    shape: tuple        # ggml order: ne[0] (fastest) first
    ggml_type: int
    offset: int         # absolute file offset of the data
    nbytes: int | None  # for the IQ formats the matmul reads; None otherwise


class GGUFReader:
    """Reads the header, metadata and tensor directory of a GGUF file; tensor data is mapped on
    demand (numpy memmap)."""

    def __init__(self, path):
        self.path = Path(path)
        self.metadata: dict = {}
        self.tensors: dict[str, TensorInfo] = {}
        with open(self.path, "rb") as f:
            buf = f.read()
        self._buf = memoryview(buf)
        self._pos = 0
        if self._u32() != _MAGIC:
            raise ValueError(f"{self.path}: not a GGUF file")
        self.version = self._u32()
        if self.version not in (2, 3):
            raise ValueError(f"{self.path}: GGUF version {self.version} not supported")
        n_tensors, n_kv = self._u64(), self._u64()
        for _ in range(n_kv):
            key = self._str()
            self.metadata[key] = self._value(self._u32())
        infos = []
        for _ in range(n_tensors):
            name = self._str()
            ndim = self._u32()
            shape = tuple(self._u64() for _ in range(ndim))
            gtype, off = self._u32(), self._u64()
            infos.append((name, shape, gtype, off))
        align = int(self.metadata.get("general.alignment", 32))
        data_start = (self._pos + align - 1) // align * align
        for name, shape, gtype, off in infos:
            nbytes = None
            if gtype in GGML_TYPE:
                nrows = int(np.prod(shape[1:])) if len(shape) > 1 else 1
                nbytes = nrows * ((shape[0] + QK - 1) // QK) * block_bytes(GGML_TYPE[gtype])
            self.tensors[name] = TensorInfo(name, shape, gtype, data_start + off, nbytes)
        del self._buf

    # -- primitive readers
    def _take(self, n):
        b = self._buf[self._pos:self._pos + n]
        if len(b) != n:
            raise ValueError(f"{self.path}: truncated")
        self._pos += n
        return b

    def _u32(self):
        return struct.unpack("<I", self._take(4))[0]

    def _u64(self):
        return struct.unpack("<Q", self._take(8))[0]

    def _str(self):
        return bytes(self._take(self._u64())).decode("utf-8")

    def _value(self, vtype):
        if vtype in _SCALAR:
            fmt = _SCALAR[vtype]
            return struct.unpack(fmt, self._take(struct.calcsize(fmt)))[0]
        if vtype == _STRING:
            return self._str()
        if vtype == _ARRAY:
            etype, n = self._u32(), self._u64()
            return [self._value(etype) for _ in range(n)]
        raise ValueError(f"{self.path}: unknown metadata type {vtype}")

    def raw(self, name: str) -> np.ndarray:
        """The tensor's bytes as a read-only u8 memmap (IQ formats only)."""
        info = self.tensors[name]
        if info.nbytes is None:
            raise ValueError(f"{name}: ggml type {info.ggml_type} is not an IQ format this library reads")
        return np.memmap(self.path, dtype=np.uint8, mode="r", offset=info.offset, shape=(info.nbytes,))


def load_iq2_weight(path, name: str, device="cuda"):
    """One IQ2_XXS / IQ2_XS / IQ2_S / IQ3_S weight matrix of a GGUF file as
    (weight_bytes, weight_scales, out_dim, in_dim, variant), ready for iq2_matmul."""
    r = GGUFReader(path)
    if name not in r.tensors:
        raise KeyError(name)
    info = r.tensors[name]
    if info.ggml_type not in GGML_TYPE:
        raise ValueError(f"{name}: ggml type {info.ggml_type} is not IQ2_XXS/IQ2_XS/IQ2_S/IQ3_S")
    variant = GGML_TYPE[info.ggml_type]
    in_dim = info.shape[0]
    out_dim = int(np.prod(info.shape[1:])) if len(info.shape) > 1 else 1
    nblocks = out_dim * ((in_dim + QK - 1) // QK)
    blocks = torch.from_numpy(np.array(r.raw(name))).to(device)
    wb, ws = split_interleaved(blocks, nblocks, variant)
    return wb, ws, out_dim, in_dim, variant
