"""Tensor-level host API (the mirror of src/iq2_matmul.rs's public functions): argument checks
that run before any CUDA call, with the reference's messages."""
import pytest
import torch

import candelora_metal_kernels_b200 as c
from candelora_metal_kernels_b200 import _lib


def _w(n=4, k=256, device="cpu"):
    nb = (k + 255) // 256
    return torch.zeros(n * nb * 64, dtype=torch.uint8, device=device), torch.zeros(n * nb * 2, dtype=torch.uint8,
                                                                                      device=device)


def test_zero_dims():
    wb, ws = _w()
    with pytest.raises(c.Iq2Error, match="expects non-zero dimensions") as e:
        c.iq2_xxs_matmul(torch.zeros(1, 256), wb, ws, 0, 256)
    assert e.value.code == _lib.IQ2_ERR_ZERO_DIM


def test_cpu_tensors_need_a_cuda_device():
    wb, ws = _w()
    with pytest.raises(c.Iq2Error, match="requires a CUDA device") as e:
        c.iq2_xxs_matmul(torch.zeros(1, 256), wb, ws, 4, 256)
    assert e.value.code == _lib.IQ2_ERR_DEVICE
    with pytest.raises(c.Iq2Error, match="iq2_dequantize_to_f16 requires a CUDA device"):
        c.iq2_dequantize_to_f16(wb, ws, 4, 256, c.Iq2MatmulVariant.Iq2Xxs)


def test_op_struct_refuses_cpu():
    wb, ws = _w()
    op = c.Iq2MatmulOp(4, 256)
    assert op.name() == "candelora_iq2_matmul"
    with pytest.raises(c.Iq2Error, match="requires a CUDA device"):
        op(torch.zeros(256), wb, ws)


def test_variant_geometry_matches_reference_constants():
    # src/iq2_matmul.rs:12-29
    v = c.Iq2MatmulVariant
    assert [x.bytes_per_block() for x in v] == [64, 64, 72, 104]
    assert [x.scales_per_block() for x in v] == [2, 10, 10, 6]


def test_activation_quant_config_defaults():
    cfg = c.ActivationQuantConfig()
    assert cfg.mode == c.ActivationQuantMode.Off and cfg.strict is False and not cfg.is_enabled()
    assert c.ActivationQuantConfig(c.ActivationQuantMode.W8A8).is_enabled()
