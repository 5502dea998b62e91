"""Seeded synthetic IQ2_XXS weights and activations with the benchmark distributions.

The reference has no public dataset on this path; the benchmark shapes are Llama-3-8B/70B-like
projections and the weight distribution is the one the benchmark plan states:
  * per 256-weight block: d = fp16(U[1e-3, 1e-2]);
  * per 32-weight sub-block: 4 grid indices ~U{0..255} (bytes 0..3), 4 sign indices ~U{0..127}
    and a 4-bit scale ~U{0..15} packed as aux_s = s0 | s1<<7 | s2<<14 | s3<<21 | scale<<28
    (bytes 4..7, little-endian), i.e. the ggml block_iq2_xxs fields, all uniform;
  * activations: f32/bf16 ~N(0, 1), optionally each row rescaled to unit RMS.

Weights come from a counter-based generator (splitmix64 of seed-derived stream bases plus the
sub-block / block index), written with plain int64 tensor ops, so the bytes are identical on the
CPU and on any GPU and any slice can be regenerated independently. A sub-block's 8 bytes are
exactly one 64-bit hash (low 32 bits = aux_g, high 32 bits = aux_s), which makes every field
uniform and independent.
"""
from __future__ import annotations

import torch

QK = 256


def _s64(v: int) -> int:
    v &= (1 << 64) - 1
    return v - (1 << 64) if v >= (1 << 63) else v


_GOLDEN = _s64(0x9E3779B97F4A7C15)
_M1 = _s64(0xBF58476D1CE4E5B9)
_M2 = _s64(0x94D049BB133111EB)


def _srl(z: torch.Tensor, k: int) -> torch.Tensor:
    return (z >> k) & ((1 << (64 - k)) - 1)


def splitmix64(x: torch.Tensor) -> torch.Tensor:
    """splitmix64 finaliser (Steele, Lea, Flood 2014) on int64 tensors, two's-complement wrap."""
    z = x + _GOLDEN
    z = (z ^ _srl(z, 30)) * _M1
    z = (z ^ _srl(z, 27)) * _M2
    return z ^ _srl(z, 31)


def _base(seed: int, stream: int) -> int:
    """A 64-bit stream base for (seed, stream), computed with Python ints (exact)."""
    z = (seed * 0x100000001B3 + stream * 0x9E3779B97F4A7C15 + 0x2545F4914F6CDD1D) & ((1 << 64) - 1)
    for _ in range(2):
        z = (z + 0x9E3779B97F4A7C15) & ((1 << 64) - 1)
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & ((1 << 64) - 1)
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & ((1 << 64) - 1)
        z ^= z >> 31
    return _s64(z)


def iq2xxs_weights(out_dim: int, in_dim: int, seed: int, device="cpu", d_lo: float = 1e-3,
                   d_hi: float = 1e-2, row_begin: int = 0, row_end: int | None = None):
    """(weight_bytes u8 [rows*nb*64], weight_scales u8 [rows*nb*2]) for rows [row_begin, row_end)
    of an out_dim x in_dim IQ2_XXS matrix; the full matrix by default. Slices of the same seed
    are byte-identical to the corresponding part of the full matrix."""
    nb = (in_dim + QK - 1) // QK
    row_end = out_dim if row_end is None else row_end
    rows = row_end - row_begin
    dev = torch.device(device)
    sb0 = row_begin * nb * 8
    idx = torch.arange(rows * nb * 8, dtype=torch.int64, device=dev) + (sb0 + _base(seed, 1))
    qs = splitmix64(idx).view(torch.uint8)
    b0 = row_begin * nb
    bidx = torch.arange(rows * nb, dtype=torch.int64, device=dev) + (b0 + _base(seed, 2))
    u = _srl(splitmix64(bidx), 40).to(torch.float32) * (1.0 / 16777216.0)
    d = (torch.tensor(d_lo, dtype=torch.float32) + u * torch.tensor(d_hi - d_lo, dtype=torch.float32))
    sc = d.to(torch.float16).view(torch.uint8)
    return qs.contiguous(), sc.contiguous()


def activations(m: int, in_dim: int, seed: int, dtype=torch.float32, device="cpu",
                rms_normalize: bool = False) -> torch.Tensor:
    """x ~ N(0, 1) of shape [m, in_dim] (drawn on the CPU with a seeded generator, then moved), in
    `dtype`; with rms_normalize each row is scaled to unit RMS in f32 first."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    x = torch.randn((m, in_dim), generator=g, dtype=torch.float32)
    if rms_normalize:
        x = x / x.pow(2).mean(dim=1, keepdim=True).sqrt()
    return x.to(dtype).to(device)


# Projection shapes (in_dim K, out_dim N) of the benchmark configurations.
LLAMA3_8B_PROJECTIONS = [  # name, K, N
    ("q", 4096, 4096),
    ("k", 4096, 1024),
    ("v", 4096, 1024),
    ("o", 4096, 4096),
    ("gate", 4096, 14336),
    ("up", 4096, 14336),
    ("down", 14336, 4096),
]

LLAMA3_70B_FFN = [("gate", 8192, 28672), ("up", 8192, 28672), ("down", 28672, 8192)]


def packed_bytes(out_dim: int, in_dim: int) -> int:
    """Algorithmic bytes of one IQ2_XXS matrix: 66 bytes per 256-weight block."""
    return out_dim * ((in_dim + QK - 1) // QK) * 66
