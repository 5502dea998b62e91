"""Shared fixtures. `-m gpu` tests need a CUDA device (B200); everything else runs on CPU."""
import re
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"
HEADER = ROOT / "include" / "candelora_iq2.h"
CODEBOOK = ROOT / "candelora_metal_kernels_b200" / "csrc" / "iq2xxs_codebook.h"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a B200); run with -m gpu")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import ORACLE_SO, Oracle, build
    if not ORACLE_SO.is_file():
        build()
    return Oracle()


@pytest.fixture(scope="session")
def ref_kernels():
    from oracle.oracle import RefKernels
    if not RefKernels.available():
        pytest.skip("oracle/_ref/libiq2ref.so not built (needs the reference checkout at build time)")
    return RefKernels()


@pytest.fixture(scope="session")
def golden():
    return {name: dict(np.load(GOLDEN / f"{name}.npz")) for name in ("ref_parity", "baseline_small")}


def parse_codebook():
    """The product's generated codebook header, parsed back into Python lists."""
    text = CODEBOOK.read_text()
    tables = {}
    for m in re.finditer(r"(\w+)\s+(\w+)((?:\[\d+\])+)\s*=\s*\{(.*?)\};", text, re.S):
        vals = [int(v, 0) for v in re.findall(r"0x[0-9a-fA-F]+|\d+", m.group(4).replace("ull", "").replace("u", ""))]
        tables[m.group(2)] = vals  # multi-dimensional tables come back flattened
    return tables


def header_functions():
    """Names of every function the C ABI header declares."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w[\w\s\*]*?\b(iq2_\w+)\s*\(", text, re.M)))


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))
