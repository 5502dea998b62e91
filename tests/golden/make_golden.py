#!/usr/bin/env python3
"""Writes the golden fixtures in tests/golden/ from the REFERENCE'S OWN KERNELS.

The reference's kernels (src/metal_src/iq2_matmul.metal, with its tables) are compiled from
source as C++ by oracle/Makefile into oracle/_ref/libiq2ref.so and run on host cores; this script
calls them on:
  ref_parity.npz   the reference test fixture of parity_case(Iq2Xxs) (src/iq2_matmul.rs:1065-1100:
                   m=2, out_dim=7, in_dim=320, LCG bytes 0xA11CE5ED / scales 0xC0FFEE12, every d
                   forced to 1.0, last byte 0x5A, x = deterministic_x) with x in f32, f16 and bf16,
                   plus the f16 dequantisation and the W8A8 outputs (f32 and f16 x; the
                   fixture of parity_case_w8a8, src/iq2_matmul.rs:1181-1253);
  baseline_small.npz  benchmark-distribution inputs (non-unit d ~U[1e-3,1e-2], N(0,1) x) that the
                   reference tests never cover: matmul m=3 x 4096 -> 33 (f32 x), m=2 x 1000 -> 9
                   (bf16 x, ragged K), the f16 dequantisation of the 9 x 1000 matrix, and the W8A8
                   output of the first case;
  ref_variants.npz the parity_case fixture for IQ2_XS, IQ2_S and IQ3_S (d = 1) and the same bytes
                   with non-unit d: f32 matmul and f16 dequantisation.
Needs oracle/_ref/libiq2ref.so (make -C oracle ref). Run from the repository root.
"""
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle.oracle import RefKernels, reference_parity_fixture  # noqa: E402
from candelora_metal_kernels_b200 import synth  # noqa: E402

OUT = Path(__file__).resolve().parent


def bits16(x: torch.Tensor) -> np.ndarray:
    return x.contiguous().view(torch.int16).numpy().view(np.uint16)


def main():
    ref = RefKernels()
    # --- the reference's own parity fixture
    x, wb, ws = reference_parity_fixture()
    xt = torch.from_numpy(x)
    out = {
        "x_f32": x, "weight_bytes": wb, "weight_scales": ws,
        "x_f16_bits": bits16(xt.to(torch.float16)), "x_bf16_bits": bits16(xt.to(torch.bfloat16)),
    }
    out["y_f32"] = ref.matmul(x, wb, ws, 7, 320, "f32")
    out["y_f16"] = ref.matmul(out["x_f16_bits"], wb, ws, 7, 320, "f16")
    out["y_bf16"] = ref.matmul(out["x_bf16_bits"], wb, ws, 7, 320, "bf16")
    out["deq_f16_bits"] = ref.dequantize_f16(wb, ws, 7, 320)
    out["y_w8a8_f32"] = ref.matmul(x, wb, ws, 7, 320, "f32", w8a8=True)
    out["y_w8a8_f16"] = ref.matmul(out["x_f16_bits"], wb, ws, 7, 320, "f16", w8a8=True)
    np.savez_compressed(OUT / "ref_parity.npz", **out)

    # --- benchmark-distribution cases (non-unit d)
    b = {}
    qs, sc = synth.iq2xxs_weights(33, 4096, seed=11)
    xa = synth.activations(3, 4096, seed=12)
    b["a_weight_bytes"], b["a_weight_scales"], b["a_x_f32"] = qs.numpy(), sc.numpy(), xa.numpy()
    b["a_y"] = ref.matmul(b["a_x_f32"], b["a_weight_bytes"], b["a_weight_scales"], 33, 4096, "f32")
    b["a_y_w8a8"] = ref.matmul(b["a_x_f32"], b["a_weight_bytes"], b["a_weight_scales"], 33, 4096, "f32", w8a8=True)
    qs, sc = synth.iq2xxs_weights(9, 1000, seed=13)
    xb = synth.activations(2, 1000, seed=14, dtype=torch.bfloat16)
    b["b_weight_bytes"], b["b_weight_scales"], b["b_x_bf16_bits"] = qs.numpy(), sc.numpy(), bits16(xb)
    b["b_y"] = ref.matmul(b["b_x_bf16_bits"], b["b_weight_bytes"], b["b_weight_scales"], 9, 1000, "bf16")
    b["b_deq_f16_bits"] = ref.dequantize_f16(b["b_weight_bytes"], b["b_weight_scales"], 9, 1000)
    np.savez_compressed(OUT / "baseline_small.npz", **b)

    # --- the other variants: the reference's parity_case(variant) fixture (d = 1) and the same
    # --- bytes with non-unit d ~U[1e-3, 1e-2] (f16), f32 matmul and f16 dequantisation
    v = {}
    rng = np.random.default_rng(17)
    for name in ("iq2_xs", "iq2_s", "iq3_s"):
        x, wb, ws = reference_parity_fixture(variant=name)
        v[f"{name}_x"], v[f"{name}_weight_bytes"], v[f"{name}_weight_scales"] = x, wb, ws
        v[f"{name}_y"] = ref.matmul(x, wb, ws, 7, 320, "f32", variant=name)
        v[f"{name}_deq_f16_bits"] = ref.dequantize_f16(wb, ws, 7, 320, variant=name)
        spb = {"iq2_xs": 10, "iq2_s": 10, "iq3_s": 6}[name]
        ws2 = ws.copy()
        d = rng.uniform(1e-3, 1e-2, ws2.size // spb).astype(np.float16).view(np.uint16)
        ws2.reshape(-1, spb)[:, 0] = (d & 0xFF).astype(np.uint8)
        ws2.reshape(-1, spb)[:, 1] = (d >> 8).astype(np.uint8)
        v[f"{name}_weight_scales_d"] = ws2
        v[f"{name}_y_d"] = ref.matmul(x, wb, ws2, 7, 320, "f32", variant=name)
        v[f"{name}_deq_d_f16_bits"] = ref.dequantize_f16(wb, ws2, 7, 320, variant=name)
    np.savez_compressed(OUT / "ref_variants.npz", **v)
    print("wrote", OUT / "ref_parity.npz", OUT / "baseline_small.npz", OUT / "ref_variants.npz")


if __name__ == "__main__":
    main()
