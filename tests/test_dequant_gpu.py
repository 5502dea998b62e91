"""GPU dequantisation: bit-exact against the reference (golden vectors from its own kernel) and
the oracle, for f16 (the reference's iq2_dequantize_to_f16), bf16 and f32 outputs."""
import numpy as np
import pytest
import torch

import candelora_metal_kernels_b200 as c
from candelora_metal_kernels_b200 import synth

pytestmark = pytest.mark.gpu


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def test_dequant_f16_matches_reference_golden(golden):
    g = golden["ref_parity"]
    y = c.iq2_dequantize_to_f16(torch.from_numpy(g["weight_bytes"]).cuda(),
                                torch.from_numpy(g["weight_scales"]).cuda(), 7, 320, c.Iq2MatmulVariant.Iq2Xxs)
    assert y.dtype == torch.float16 and y.shape == (7, 320)
    assert np.array_equal(_bits(y), g["deq_f16_bits"])
    b = golden["baseline_small"]
    y = c.iq2_dequantize_to_f16(torch.from_numpy(b["b_weight_bytes"]).cuda(),
                                torch.from_numpy(b["b_weight_scales"]).cuda(), 9, 1000)
    assert np.array_equal(_bits(y), b["b_deq_f16_bits"])


@pytest.mark.parametrize("n,k", [(7, 320), (33, 4096), (5, 1000), (300, 768), (1, 8), (2, 257)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_dequant_bit_exact_vs_oracle(oracle, n, k, dtype):
    qs, sc = synth.iq2xxs_weights(n, k, seed=n + k)
    y = c.iq2_dequantize(qs.cuda(), sc.cuda(), n, k, dtype=dtype)
    name = {torch.float16: "f16", torch.bfloat16: "bf16", torch.float32: "f32"}[dtype]
    ref = oracle.dequantize(qs.numpy(), sc.numpy(), n, k, name)
    got = y.cpu().numpy() if dtype == torch.float32 else _bits(y)
    if dtype == torch.float32:
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    else:
        assert np.array_equal(got, ref)


def test_dequant_extreme_scales_bit_exact(oracle):
    n, k = 6, 256
    qs, _ = synth.iq2xxs_weights(n, k, seed=5)
    sc = torch.from_numpy(np.array([0x7C00, 0x7E00, 0x7BFF, 0x0001, 0x0000, 0x8000], dtype=np.uint16)
                          .view(np.uint8).copy())
    y = c.iq2_dequantize_to_f16(qs.cuda(), sc.cuda(), n, k)
    got, want = _bits(y), oracle.dequantize(qs.numpy(), sc.numpy(), n, k, "f16")
    # NaN payloads carry no value (the GPU writes the canonical 0x7FFF, the host 0x7E00):
    # NaN must map to NaN, every other value bit for bit.
    nan_got = (got & 0x7C00) == 0x7C00
    nan_got &= (got & 0x03FF) != 0
    nan_want = ((want & 0x7C00) == 0x7C00) & ((want & 0x03FF) != 0)
    assert np.array_equal(nan_got, nan_want) and nan_want.any()
    assert np.array_equal(got[~nan_want], want[~nan_want])


def test_dequant_unaligned_buffers(oracle):
    n, k = 20, 512
    qs, sc = synth.iq2xxs_weights(n, k, seed=77)
    bq = torch.zeros(qs.numel() + 8, dtype=torch.uint8)
    bs = torch.zeros(sc.numel() + 8, dtype=torch.uint8)
    bq[5:5 + qs.numel()] = qs
    bs[3:3 + sc.numel()] = sc
    y = c.iq2_dequantize_to_f16(bq.cuda()[5:5 + qs.numel()], bs.cuda()[3:3 + sc.numel()], n, k)
    assert np.array_equal(_bits(y), oracle.dequantize(qs.numpy(), sc.numpy(), n, k, "f16"))
