"""Activation-quantisation contract types: a mirror of src/activation_quant.rs:7-44."""
from __future__ import annotations

import enum
from dataclasses import dataclass


class ActivationQuantMode(enum.IntEnum):
    """ActivationQuantMode (src/activation_quant.rs:7-15)."""

    Off = 0   # existing floating-point activation path
    W8A8 = 1  # INT8 activation kernels (contract target)
    W4A8 = 2  # W4A8 workflows (contract target; no kernel in the reference either)


@dataclass(frozen=True)
class ActivationQuantConfig:
    """ActivationQuantConfig (src/activation_quant.rs:23-44)."""

    mode: ActivationQuantMode = ActivationQuantMode.Off
    strict: bool = False

    def is_enabled(self) -> bool:
        return self.mode != ActivationQuantMode.Off
