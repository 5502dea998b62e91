"""The CPU oracle pinned against the reference: golden vectors from the reference's own kernels,
and (where oracle/_ref was built) direct comparison with those kernels on fresh inputs."""
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import GOLDEN, ROOT, parse_codebook, rel_l2
from oracle.oracle import (deterministic_x, force_f16_one_per_block, lcg_fill,
                           reference_dir, reference_parity_fixture)
from candelora_metal_kernels_b200 import synth

_REF = reference_dir()
REF_TABLES = _REF / "src/metal_src/iq2_tables.metal" if _REF is not None else Path("-missing-")


def _bits(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(x).view(np.uint32)


def test_fixture_generators_match_golden(golden):
    g = golden["ref_parity"]
    x, wb, ws = reference_parity_fixture()
    assert np.array_equal(wb, g["weight_bytes"]) and np.array_equal(ws, g["weight_scales"])
    assert np.array_equal(_bits(x), _bits(g["x_f32"]))
    # spot values of the LCG / deterministic_x definitions (src/iq2_matmul.rs:765-779)
    assert lcg_fill(3, 0)[0] == (1013904223 >> 24)
    assert deterministic_x(1, 3)[0, 0] == np.float32(-20.0) / np.float32(13.0)
    s = force_f16_one_per_block(np.zeros(6, np.uint8), 2)
    assert list(s) == [0x00, 0x3C] * 3


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
def test_oracle_matches_reference_golden_parity_fixture(oracle, golden, dtype):
    g = golden["ref_parity"]
    x = g["x_f32"] if dtype == "f32" else g[f"x_{dtype}_bits"]
    y = oracle.matmul(x, g["weight_bytes"], g["weight_scales"], 7, 320, x_dtype=dtype)
    assert np.array_equal(_bits(y), _bits(g[f"y_{dtype}"])), "oracle != reference kernel (bit-exact)"


def test_oracle_dequant_matches_reference_golden(oracle, golden):
    g = golden["ref_parity"]
    assert np.array_equal(oracle.dequantize(g["weight_bytes"], g["weight_scales"], 7, 320, "f16"),
                          g["deq_f16_bits"])
    b = golden["baseline_small"]
    assert np.array_equal(oracle.dequantize(b["b_weight_bytes"], b["b_weight_scales"], 9, 1000, "f16"),
                          b["b_deq_f16_bits"])


def test_oracle_matches_reference_golden_nonunit_scales(oracle, golden):
    b = golden["baseline_small"]
    ya = oracle.matmul(b["a_x_f32"], b["a_weight_bytes"], b["a_weight_scales"], 33, 4096)
    assert np.array_equal(_bits(ya), _bits(b["a_y"]))
    yb = oracle.matmul(b["b_x_bf16_bits"], b["b_weight_bytes"], b["b_weight_scales"], 9, 1000, x_dtype="bf16")
    assert np.array_equal(_bits(yb), _bits(b["b_y"]))


def test_oracle_column_sample_equals_full(oracle):
    qs, sc = synth.iq2xxs_weights(40, 512, seed=3)
    x = synth.activations(2, 512, seed=4).numpy()
    full = oracle.matmul(x, qs.numpy(), sc.numpy(), 40, 512)
    cols = np.array([0, 7, 39, 13])
    part = oracle.matmul(x, qs.numpy(), sc.numpy(), 40, 512, cols=cols)
    assert np.array_equal(_bits(part), _bits(np.ascontiguousarray(full[:, cols])))


def test_oracle_dequant_f32_is_exact_and_f16_is_its_rne(oracle):
    qs, sc = synth.iq2xxs_weights(5, 768, seed=9)
    f32 = oracle.dequantize(qs.numpy(), sc.numpy(), 5, 768, "f32")
    f16 = oracle.dequantize(qs.numpy(), sc.numpy(), 5, 768, "f16")
    bf16 = oracle.dequantize(qs.numpy(), sc.numpy(), 5, 768, "bf16")
    t = torch.from_numpy(f32)
    assert np.array_equal(f16, t.to(torch.float16).view(torch.int16).numpy().view(np.uint16))
    assert np.array_equal(bf16, t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16))
    # every value is d*(2s+1)/8 * {8,25,43}: exact in f64 too
    assert np.all(np.isfinite(f32)) and set(np.unique(np.abs(f32) > 0)) == {True}


@pytest.mark.parametrize("case", [(1, 5, 256), (2, 17, 320), (3, 31, 4096), (4, 9, 1000), (1, 3, 7)])
@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
def test_oracle_matches_reference_kernels_live(oracle, ref_kernels, case, dtype):
    m, n, k = case
    qs, sc = synth.iq2xxs_weights(n, k, seed=100 + k)
    x = synth.activations(m, k, seed=200 + n)
    if dtype == "f32":
        xin = x.numpy()
    else:
        xin = x.to(torch.float16 if dtype == "f16" else torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    a = oracle.matmul(xin, qs.numpy(), sc.numpy(), n, k, x_dtype=dtype)
    b = ref_kernels.matmul(xin, qs.numpy(), sc.numpy(), n, k, x_dtype=dtype)
    assert np.array_equal(_bits(a), _bits(b))
    assert np.array_equal(oracle.dequantize(qs.numpy(), sc.numpy(), n, k, "f16"),
                          ref_kernels.dequantize_f16(qs.numpy(), sc.numpy(), n, k))


def test_oracle_handles_extreme_scales_like_reference(oracle, ref_kernels):
    """d = inf, NaN, max normal, subnormal, +-0 (fp16 patterns) -- never exercised by the reference
    tests (they force d = 1.0)."""
    n, k = 6, 256
    qs, _ = synth.iq2xxs_weights(n, k, seed=5)
    d_bits = np.array([0x7C00, 0x7E00, 0x7BFF, 0x0001, 0x0000, 0x8000], dtype=np.uint16)
    sc = d_bits.view(np.uint8).copy()
    x = synth.activations(2, k, seed=6).numpy()
    a = oracle.matmul(x, qs.numpy(), sc, n, k)
    b = ref_kernels.matmul(x, qs.numpy(), sc, n, k)
    assert np.array_equal(_bits(a), _bits(b))
    assert np.array_equal(oracle.dequantize(qs.numpy(), sc, n, k, "f16"), ref_kernels.dequantize_f16(qs.numpy(), sc, n, k))


def test_product_codebook_matches_oracle_tables():
    """The kernels' codebook (csrc/iq2xxs_codebook.h) against the oracle's table header; both
    are generated independently from the reference's iq2_tables.metal."""
    import re
    cb = parse_codebook()
    text = (Path(__file__).resolve().parents[1] / "oracle" / "iq2_tables_ref.h").read_text()
    body = re.search(r"ref_iq2xxs_grid\[256\] = \{(.*?)\};", text, re.S).group(1)
    grid = [int(v.replace("ull", ""), 16) for v in re.findall(r"0x[0-9a-f]+ull", body)]
    assert cb["IQ2XXS_GRID"] == grid
    body = re.search(r"ref_ksigns_iq2xs\[128\] = \{(.*?)\};", text, re.S).group(1)
    ksigns = [int(v) for v in re.findall(r"(\d+)u", body)]
    assert cb["IQ2_KSIGNS"] == ksigns


@pytest.mark.skipif(not REF_TABLES.is_file(), reason="reference checkout not present")
def test_tables_match_reference_source():
    import subprocess
    import sys
    import tempfile
    root = Path(__file__).resolve().parents[1]
    with tempfile.TemporaryDirectory() as d:
        subprocess.run([sys.executable, str(root / "oracle" / "gen_tables.py"), "--ref", str(_REF),
                        "--out", f"{d}/t.h"], check=True)
        assert Path(f"{d}/t.h").read_text() == (root / "oracle" / "iq2_tables_ref.h").read_text()
        subprocess.run([sys.executable, str(root / "candelora_metal_kernels_b200" / "csrc" / "gen_codebook.py"),
                        "--tables", str(REF_TABLES), "--out", f"{d}/c.h", "--out-variants", f"{d}/v.h"], check=True)
        assert Path(f"{d}/c.h").read_text() == (root / "candelora_metal_kernels_b200" / "csrc" /
                                                "iq2xxs_codebook.h").read_text()
        assert Path(f"{d}/v.h").read_text() == (root / "candelora_metal_kernels_b200" / "csrc" /
                                                "iq2_variant_grids.h").read_text()


def test_oracle_w8a8_matches_reference_golden(oracle, golden):
    """W8A8 (src/metal_src/iq2_matmul.metal:85-102, :437-499): the restated row quant-dequant
    followed by the restated f32 matmul equals the reference's W8A8 kernel bit for bit, on the
    reference's parity fixture and on benchmark-distribution weights."""
    g = golden["ref_parity"]
    xq = oracle.rowwise_qdq_w8a8(g["x_f32"])
    assert np.array_equal(oracle.matmul(xq, g["weight_bytes"], g["weight_scales"], 7, 320), g["y_w8a8_f32"])
    x16 = g["x_f16_bits"].view(np.float16).astype(np.float32)
    xq16 = oracle.rowwise_qdq_w8a8(x16)
    assert np.array_equal(oracle.matmul(xq16, g["weight_bytes"], g["weight_scales"], 7, 320), g["y_w8a8_f16"])
    b = golden["baseline_small"]
    xq = oracle.rowwise_qdq_w8a8(b["a_x_f32"])
    assert np.array_equal(oracle.matmul(xq, b["a_weight_bytes"], b["a_weight_scales"], 33, 4096), b["a_y_w8a8"])


VARIANTS = ("iq2_xs", "iq2_s", "iq3_s")


@pytest.mark.parametrize("variant", VARIANTS)
def test_oracle_variants_match_reference_golden(oracle, variant):
    """IQ2_XS / IQ2_S / IQ3_S (src/iq2_matmul.rs:884-1016, iq2_matmul.metal:736-866): the
    restated dequantisation equals the reference kernels' bit for bit; the restated matmul
    follows the reference's CPU loop, which for IQ2_XS is also the Metal kernel's order (bit
    exact) while for IQ2_S / IQ3_S the Metal kernels interleave the two grid words of a group
    (iq2_matmul.metal:55-83): there the two agree to float rounding of the sum order."""
    v = dict(np.load(GOLDEN / "ref_variants.npz"))
    x, wb = v[f"{variant}_x"], v[f"{variant}_weight_bytes"]
    for sfx, ws_key, deq_key in (("", "weight_scales", "deq_f16_bits"), ("_d", "weight_scales_d", "deq_d_f16_bits")):
        ws = v[f"{variant}_{ws_key}"]
        assert np.array_equal(oracle.dequantize(wb, ws, 7, 320, "f16", variant=variant), v[f"{variant}_{deq_key}"])
        y = oracle.matmul(x, wb, ws, 7, 320, variant=variant)
        want = v[f"{variant}_y{sfx}"]
        if variant == "iq2_xs":
            assert np.array_equal(y, want)
        else:
            assert rel_l2(y, want) <= 1e-6
            assert np.abs(y - want).max() <= 2e-3 * max(1.0, float(np.abs(want).max()))


def test_variant_grids_header_matches_oracle_tables():
    """csrc/iq2_variant_grids.h (the product's copy) and oracle/iq2_tables_ref.h (the oracle's)
    hold the same values: both are generated from the reference's table source."""
    import re
    prod = (ROOT / "candelora_metal_kernels_b200" / "csrc" / "iq2_variant_grids.h").read_text()
    ref = (ROOT / "oracle" / "iq2_tables_ref.h").read_text()

    def table(text, name):
        m = re.search(name + r"\[\d+\]\s*=\s*\{(.*?)\};", text, re.S)
        return [int(t, 16) for t in re.findall(r"0x[0-9a-fA-F]+", m.group(1))]
    for p_name, r_name in (("IQ2XS_GRID", "ref_iq2xs_grid"), ("IQ2S_GRID", "ref_iq2s_grid"), ("IQ3S_GRID", "ref_iq3s_grid")):
        assert table(prod, p_name) == table(ref, r_name), p_name
