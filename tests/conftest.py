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
HEADERS = [HEADER, ROOT / "include" / "candelora_iq2_testing.h"]
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


_C_TYPES = {"int": "i32", "uint32_t": "u32", "uint64_t": "u64", "size_t": "usize", "uint8_t": "u8", "float": "f32"}


def _canon_c(decl: str) -> str:
    """A C parameter or return type (name dropped) in canonical form: ptr, i32, u32, u64, usize."""
    decl = re.sub(r"\bconst\b", " ", decl)
    if "*" in decl:
        return "ptr"
    words = decl.split()
    if not words or words == ["void"]:
        return "void"
    for w in words:
        if w in _C_TYPES:
            return _C_TYPES[w]
    return "ptr" if words[0].endswith("_t") and words[0].startswith("iq2_") else "?" + words[0]


def header_prototypes():
    """Every function the C ABI headers declare: name -> (return type, [parameter types]), canonical."""
    protos = {}
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", " ", h.read_text(), flags=re.S)
        text = re.sub(r"//[^\n]*", " ", text)
        for m in re.finditer(r"([A-Za-z_][\w\s\*]*?)\b(iq2_\w+)\s*\(([^()]*)\)\s*;", text):
            ret, name, params = m.group(1), m.group(2), m.group(3).strip()
            if ret.strip().startswith("typedef"):
                continue
            args = []
            if params and params != "void":
                for prm in params.split(","):
                    prm = prm.strip()
                    # drop the parameter's name (the last identifier, unless the declaration is a bare type)
                    mm = re.match(r"(.*?[\s\*])(\w+)$", prm)
                    args.append(_canon_c(mm.group(1) if mm and mm.group(1).strip() not in ("", "const") else prm))
            protos[name] = (_canon_c(ret), args)
    return protos


def header_functions():
    """Names of every function the C ABI headers declare."""
    return sorted(header_prototypes())


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))
