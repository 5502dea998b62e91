"""B200-native (sm_100a) IQ2_XXS quantised matmul: a drop-in for the IQ2 path of
candelora-metal-kernels (src/iq2_matmul.rs + src/metal_src/iq2_matmul.metal).

The compute path is libcandelora_iq2.so (hand-written CUDA, C ABI in include/candelora_iq2.h);
this package is its tensor-level host binding, mirroring the reference's public functions.
"""
from ._lib import Iq2Error, LIB_PATH
from .activation_quant import ActivationQuantConfig, ActivationQuantMode
from .iq2_matmul import (
    Iq2MatmulOp,
    Iq2MatmulVariant,
    device_check,
    iq2_dequantize,
    iq2_dequantize_to_f16,
    grouped_workspace_bytes,
    iq2_matmul,
    iq2_matmul_grouped,
    iq2_matmul_with_activation_quant,
    iq2_s_matmul,
    iq2_xs_matmul,
    iq2_xxs_matmul,
    iq3_s_matmul,
    workspace_bytes,
)

__all__ = [
    "ActivationQuantConfig",
    "ActivationQuantMode",
    "Iq2Error",
    "Iq2MatmulOp",
    "Iq2MatmulVariant",
    "LIB_PATH",
    "device_check",
    "iq2_dequantize",
    "iq2_dequantize_to_f16",
    "grouped_workspace_bytes",
    "iq2_matmul",
    "iq2_matmul_grouped",
    "iq2_matmul_with_activation_quant",
    "iq2_s_matmul",
    "iq2_xs_matmul",
    "iq2_xxs_matmul",
    "iq3_s_matmul",
    "workspace_bytes",
]
