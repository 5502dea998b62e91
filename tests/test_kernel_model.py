"""CPU model of the decode GEMV's arithmetic (candelora_metal_kernels_b200/csrc/iq2xxs_gemv.cu),
checked against the oracle. It re-derives, in numpy, exactly what the kernel computes:
  * weights via `prmt` selectors: GRID_SEL[grid idx] | SIGN_SEL[sign idx] picking bytes out of
    {+8,+25,+43,0,-8,-25,-43,0};
  * x as four signed 7-bit limbs of a 28-bit fixed-point value per (token, 256-block);
  * s32 sums per 32-weight sub-block, scaled by (2s+1) in s32, f32 once per block.
so a design error in the tables or the limb algebra shows up here, without a GPU."""
import numpy as np
import pytest

from conftest import parse_codebook, rel_l2
from candelora_metal_kernels_b200 import synth

KPOS, KNEG = 0x002B1908, 0x00D5E7F8


def prmt(a: int, b: int, sel: int) -> int:
    src = [(a >> (8 * i)) & 0xFF for i in range(4)] + [(b >> (8 * i)) & 0xFF for i in range(4)]
    out = 0
    for i in range(4):
        nib = (sel >> (4 * i)) & 0xF
        byte = src[nib & 7]
        if nib & 8:
            byte = 0xFF if byte & 0x80 else 0x00
        out |= byte << (8 * i)
    return out


def decode_weights_int8(qs: np.ndarray, n: int, k: int, cb) -> np.ndarray:
    """Signed int8 weights [n, nb*256] (without d*(2s+1)/8) as the kernel's decode produces them."""
    nb = (k + 255) // 256
    words = qs.reshape(n, nb * 8, 8)
    out = np.zeros((n, nb * 256), dtype=np.int8)
    gsel, ssel = cb["IQ2XXS_GRID_SEL"], cb["IQ2XXS_SIGN_SEL"]
    for r in range(n):
        for sb in range(nb * 8):
            w = words[r, sb]
            aux_g = int.from_bytes(bytes(w[:4]), "little")
            aux_s = int.from_bytes(bytes(w[4:]), "little")
            for t in range(4):
                sel = gsel[(aux_g >> (8 * t)) & 0xFF] | ssel[(aux_s >> (7 * t)) & 0x7F]
                lo, hi = prmt(KPOS, KNEG, sel & 0xFFFF), prmt(KPOS, KNEG, sel >> 16)
                v = lo.to_bytes(4, "little") + hi.to_bytes(4, "little")
                out[r, sb * 32 + t * 8: sb * 32 + t * 8 + 8] = np.frombuffer(v, dtype=np.int8)
    return out


def test_selector_tables_decode_every_grid_and_sign_pattern():
    cb = parse_codebook()
    for e in range(256):
        g = cb["IQ2XXS_GRID"][e]
        mags = [(g >> (8 * j)) & 0xFF for j in range(8)]
        for s in range(128):
            signs = cb["IQ2_KSIGNS"][s]
            sel = cb["IQ2XXS_GRID_SEL"][e] | cb["IQ2XXS_SIGN_SEL"][s]
            got = prmt(KPOS, KNEG, sel & 0xFFFF).to_bytes(4, "little") + \
                prmt(KPOS, KNEG, sel >> 16).to_bytes(4, "little")
            want = bytes(((-mags[j]) & 0xFF) if (signs >> j) & 1 else mags[j] for j in range(8))
            assert got == want, (e, s)


def model_gemv(x: np.ndarray, qs: np.ndarray, sc: np.ndarray, n: int, k: int, cb) -> np.ndarray:
    m = x.shape[0]
    nb = (k + 255) // 256
    A = decode_weights_int8(qs, n, k, cb).astype(np.int64)          # [n, nb*256]
    words = qs.reshape(n, nb * 8, 8)
    aux_s = words[:, :, 4:].copy().view("<u4").reshape(n, nb * 8).astype(np.int64)
    c = ((aux_s >> 27) | 1)                                          # 2s+1 per (row, sub-block)
    d = sc.view(np.float16).astype(np.float32).reshape(n, nb)
    xp = np.zeros((m, nb * 256), dtype=np.float32)
    xp[:, :k] = x
    out = np.zeros((m, n), dtype=np.float32)
    for b in range(nb):
        xb = xp[:, b * 256:(b + 1) * 256]
        amax = np.abs(xb).max(axis=1)
        E = np.frexp(amax)[1]
        q = np.rint(np.ldexp(xb.astype(np.float64), (27 - E)[:, None])).astype(np.int64)
        assert np.abs(q).max() <= (1 << 27)
        mag, sgn = np.abs(q), np.sign(q)
        limbs = [sgn * ((mag >> (7 * l)) & 127) for l in range(3)] + [sgn * (mag >> 21)]
        for l in range(4):
            assert np.abs(limbs[l]).max() <= 127
        colscale = [np.ldexp(np.float32(1.0), E - 30 + 7 * l).astype(np.float32) for l in range(4)]
        for l in range(4):
            I = np.zeros((n, m), dtype=np.int64)
            for sbi in range(8):
                sb = b * 8 + sbi
                D = A[:, sb * 32:(sb + 1) * 32] @ limbs[l][:, sbi * 32:(sbi + 1) * 32].T   # [n, m]
                assert np.abs(D).max() < (1 << 31)
                I += c[:, sb:sb + 1] * D
            assert np.abs(I).max() < (1 << 31), "s32 block accumulator would overflow"
            scale = (d[:, b:b + 1] * colscale[l][None, :]).astype(np.float32)
            out += (I.astype(np.float32) * scale).T
    return out


@pytest.mark.parametrize("m,n,k", [(1, 6, 512), (2, 5, 320), (3, 4, 1000)])
def test_gemv_model_matches_oracle(oracle, m, n, k):
    cb = parse_codebook()
    qs, sc = synth.iq2xxs_weights(n, k, seed=7 * k + n)
    x = synth.activations(m, k, seed=m + 31).numpy()
    y_model = model_gemv(x, qs.numpy(), sc.numpy(), n, k, cb)
    y_ref = oracle.matmul(x, qs.numpy(), sc.numpy(), n, k)
    err = rel_l2(y_model, y_ref)
    assert err < 1e-6, err  # the bound in the tests of the CUDA path is 1e-4


def test_gemv_model_worst_case_magnitudes_fit_s32(oracle):
    """All weights at the largest magnitude (43) with the largest scale (2s+1 = 31) and x at
    the per-block maximum: the s32 block sums must not overflow."""
    n, k = 2, 256
    nb = 1
    qs = np.zeros(n * nb * 64, dtype=np.uint8)
    cb = parse_codebook()
    e43 = next(i for i, g in enumerate(cb["IQ2XXS_GRID"]) if g == 0x2B2B2B2B2B2B2B2B) \
        if 0x2B2B2B2B2B2B2B2B in cb["IQ2XXS_GRID"] else None
    # the grid has no all-43 word; use the entry with the largest byte sum instead
    if e43 is None:
        e43 = max(range(256), key=lambda e: sum((cb["IQ2XXS_GRID"][e] >> (8 * j)) & 0xFF for j in range(8)))
    words = qs.reshape(n * nb * 8, 8)
    words[:, 0:4] = e43
    words[:, 4:8] = np.frombuffer((0xF << 28).to_bytes(4, "little"), dtype=np.uint8)
    sc = np.full(n * nb, 0x3C00, dtype=np.uint16).view(np.uint8)
    x = np.ones((1, k), dtype=np.float32) * np.float32(0.999)
    y_model = model_gemv(x, qs, sc, n, k, cb)
    y_ref = oracle.matmul(x, qs, sc, n, k)
    assert rel_l2(y_model, y_ref) < 1e-6


def _bf16_bits(v: np.ndarray) -> np.ndarray:
    import torch
    return torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32)).to(torch.bfloat16).view(torch.int16).numpy() \
        .view(np.uint16)


def test_gemm_bf16_decode_tables_match_rounded_dequant(oracle):
    """The GEMM's weight decode (csrc/iq2xxs_gemm.cu): per sub-block the bf16 roundings of
    dl*{8,25,43}, a prmt by IQ2XXS_BF16_SEL and an XOR by the sign byte spread with one multiply,
    (S * K_i) & 0x80008000, must equal the bf16 rounding of every exact weight (the oracle's f32
    dequant). The spread is also checked against the mask table IQ2_SIGN_PAIR_MASK."""
    cb = parse_codebook()
    sel, smask = cb["IQ2XXS_BF16_SEL"], cb["IQ2_SIGN_PAIR_MASK"]
    K = [0x40008000, 0x10002000, 0x04000800, 0x01000200]
    for si in range(128):
        S = cb["IQ2_KSIGNS"][si]
        assert [((S * K[i]) & 0xFFFFFFFF) & 0x80008000 for i in range(4)] == smask[si * 4:si * 4 + 4]
    n, k = 12, 768
    qs, sc = synth.iq2xxs_weights(n, k, seed=21)
    qs, sc = qs.numpy(), sc.numpy()
    want = oracle.dequantize(qs, sc, n, k, "bf16")
    d = sc.view(np.float16).astype(np.float32).reshape(n, k // 256)
    words = qs.reshape(n, k // 32, 8)
    got = np.zeros((n, k), dtype=np.uint16)
    for r in range(n):
        for sb in range(k // 32):
            aux_g = int.from_bytes(bytes(words[r, sb, :4]), "little")
            aux_s = int.from_bytes(bytes(words[r, sb, 4:]), "little")
            dl = np.float32(d[r, sb // 8]) * np.float32((aux_s >> 27) | 1) * np.float32(0.125)
            b8, b25, b43 = _bf16_bits(np.array([dl * 8, dl * 25, dl * 43], dtype=np.float32))
            qlo, qhi = int(b8) | (int(b25) << 16), int(b43)
            for t in range(4):
                gi, si = (aux_g >> (8 * t)) & 0xFF, (aux_s >> (7 * t)) & 0x7F
                for i in range(4):
                    w = prmt(qlo, qhi, sel[gi * 4 + i]) ^ smask[si * 4 + i]
                    col = sb * 32 + t * 8 + 2 * i
                    got[r, col], got[r, col + 1] = w & 0xFFFF, w >> 16
    assert np.array_equal(got, want)


def test_variant_selector_rules_decode_the_xs_and_s_grids():
    """The IQ2_XS / IQ2_S matmul (csrc/iq2_variants.cu, decode8_sel) builds its tables at run time:
    grid selector nibble j = 0, 1, 2 for magnitude byte j = 8, 25, 43; sign selector nibble j = 4
    when bit j of the sign byte is set. Decoded through `prmt` of the IQ2_XXS magnitude words, every
    grid entry and sign pattern must give exactly grid * sign."""
    import re
    from pathlib import Path
    text = (Path(__file__).resolve().parent.parent / "candelora_metal_kernels_b200" / "csrc" /
            "iq2_variant_grids.h").read_text()

    def table(name):
        m = re.search(name + r"\[\d+\]\s*=\s*\{(.*?)\};", text, re.S)
        return [int(t, 16) for t in re.findall(r"0x[0-9a-fA-F]+", m.group(1))]

    code = {8: 0, 25: 1, 43: 2}
    ssel = [sum((((i >> j) & 1) << (4 * j + 2)) for j in range(8)) for i in range(256)]
    for name in ("IQ2XS_GRID", "IQ2S_GRID"):
        grid = table(name)
        gsel = [sum(code[(g >> (8 * j)) & 0xFF] << (4 * j) for j in range(8)) for g in grid]
        cases = [(e, s) for e in range(len(grid)) for s in (0x00, 0xFF, 0xA5, 0x5A, 0x01, 0x80, 0x3C, 0xC3)]
        cases += [(e, s) for e in range(0, len(grid), len(grid) // 32) for s in range(256)]
        for e, s in cases:
            sel = gsel[e] | ssel[s]
            got = prmt(KPOS, KNEG, sel & 0xFFFF).to_bytes(4, "little") + prmt(KPOS, KNEG, sel >> 16).to_bytes(4, "little")
            mags = [(grid[e] >> (8 * j)) & 0xFF for j in range(8)]
            want = bytes(((-mags[j]) & 0xFF) if (s >> j) & 1 else mags[j] for j in range(8))
            assert got == want, (name, e, s)
