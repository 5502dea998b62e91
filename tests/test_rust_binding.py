"""The Rust (candle) binding in candelora_metal_kernels_b200/rust/ against the C ABI, on CPU: the image
has no Rust toolchain, so the binding is checked as text. Every function the headers declare is
declared in the Rust extern block with the same return type and the same argument types in the
same order; the problem struct has the same fields; the status, dtype and activation-mode
constants have the header's values; build.rs compiles the same sources as build.py."""
import re

from conftest import HEADER, ROOT, header_prototypes

RUST = ROOT / "candelora_metal_kernels_b200" / "rust"
FFI = RUST / "src" / "iq2_cuda_ffi.rs"


def _canon_rust(t: str) -> str:
    t = t.strip()
    if t.startswith("*"):
        return "ptr"
    return {"c_int": "i32", "i32": "i32", "u32": "u32", "u64": "u64", "usize": "usize", "f32": "f32",
            "c_char": "i8", "": "void", "()": "void"}.get(t, "?" + t)


def rust_externs():
    text = re.sub(r"//[^\n]*", "", FFI.read_text())
    block = re.search(r'extern "C" \{(.*?)\n\}', text, re.S).group(1)
    out = {}
    for m in re.finditer(r"pub fn (iq2_\w+)\s*\((.*?)\)\s*(?:->\s*([^;]+))?;", block, re.S):
        name, params, ret = m.group(1), m.group(2), m.group(3) or ""
        args = [p.split(":", 1)[1] for p in (q.strip() for q in params.split(",")) if p]
        out[name] = (_canon_rust(ret), [_canon_rust(a) for a in args])
    return out


def test_every_header_function_is_declared_in_rust_with_the_same_signature():
    c_protos, rs = header_prototypes(), rust_externs()
    assert sorted(rs) == sorted(c_protos)
    for name, (ret, params) in c_protos.items():
        assert rs[name] == (ret, params), (name, rs[name], (ret, params))


def test_problem_struct_fields_match():
    h = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    body = re.search(r"typedef struct iq2_matmul_problem \{(.*?)\} iq2_matmul_problem;", h, re.S).group(1)
    c_fields = []
    for decl in (d.strip() for d in body.split(";") if d.strip()):
        *typ, names = decl.rsplit(None, 1) if "," not in decl else (decl.split(None, 1)[0], decl.split(None, 1)[1])
        for nm in names.split(","):
            nm = nm.strip()
            star = "*" in decl
            c_fields.append((nm.lstrip("*"), "ptr" if star else {"size_t": "usize", "uint32_t": "u32"}[typ[0].split()[-1]]))
    rs = re.search(r"pub struct Iq2MatmulProblem \{(.*?)\}", FFI.read_text(), re.S).group(1)
    r_fields = [(m.group(1), _canon_rust(m.group(2))) for m in re.finditer(r"pub (\w+):\s*([^,]+),", rs)]
    assert r_fields == c_fields


def test_constants_match_the_header():
    h = HEADER.read_text()
    consts = dict((k, int(v)) for k, v in re.findall(r"\b(IQ2_(?:ERR_\w+|OK|DTYPE_\w+|ACT_QUANT_\w+))\s*=\s*(\d+)", h))
    consts["IQ2_COMM_ID_BYTES"] = int(re.search(r"#define IQ2_COMM_ID_BYTES (\d+)", h).group(1))
    rs = dict((k, int(v)) for k, v in re.findall(r"pub const (IQ2_\w+): \w+ = (\d+);", FFI.read_text()))
    for k, v in consts.items():
        assert rs.get(k) == v, k


def test_build_rs_compiles_the_library_sources_for_sm_100a():
    from candelora_metal_kernels_b200.build import SOURCES
    text = (RUST / "build.rs").read_text()
    listed = re.findall(r'"(\w+\.cu)"', re.search(r"const SOURCES.*?\];", text, re.S).group(0))
    assert listed == SOURCES
    assert "arch=compute_100a,code=sm_100a" in text
