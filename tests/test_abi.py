"""The C ABI library: it loads, exports every symbol include/candelora_iq2.h declares, and its
argument checks that need no GPU behave like the reference's bail conditions."""
import ctypes

import pytest
import torch

from conftest import header_functions, header_prototypes
from candelora_metal_kernels_b200 import _lib
from candelora_metal_kernels_b200.build import LIB, build


@pytest.fixture(scope="module")
def lib():
    build()
    return _lib.load()


def test_header_declares_the_expected_entry_points():
    names = header_functions()
    assert names == sorted(_lib.SIGNATURES), names


# (on 64-bit Linux ctypes.c_size_t is ctypes.c_uint64: size_t and uint64_t compare equal here)
_CTYPES_CANON = {ctypes.c_void_p: "ptr", ctypes.c_char_p: "ptr", ctypes.c_uint32: "u32", ctypes.c_int: "i32",
                 ctypes.c_uint64: "u64"}


def test_python_binding_argument_lists_match_the_header():
    """Every ctypes signature has the header's argument count and types, in order."""
    protos = header_prototypes()
    as_ctypes = {"usize": "u64"}
    for name, (args, res) in _lib.SIGNATURES.items():
        ret, params = protos[name]
        assert [_CTYPES_CANON[a] for a in args] == [as_ctypes.get(t, t) for t in params], name
        assert _CTYPES_CANON.get(res, "?") == as_ctypes.get(ret, ret), name


def test_library_exports_every_header_symbol(lib):
    raw = ctypes.CDLL(str(LIB))
    for name in header_functions():
        assert hasattr(raw, name), f"{name} missing from {LIB.name}"


def test_abi_version(lib):
    assert lib.iq2_abi_version() == 2


def _matmul(lib, m=1, out_dim=4, in_dim=256, variant=0, x_dtype=0):
    return lib.iq2_matmul(None, x_dtype, m, None, 0, None, 0, out_dim, in_dim, variant, None, None, 0, None)


def test_zero_dims_rejected_first(lib):
    assert _matmul(lib, out_dim=0) == _lib.IQ2_ERR_ZERO_DIM
    assert b"expects non-zero dimensions" in lib.iq2_last_error()
    assert _matmul(lib, in_dim=0) == _lib.IQ2_ERR_ZERO_DIM
    rc = lib.iq2_dequantize(None, 0, None, 0, 0, 8, 0, None, 1, None)
    assert rc == _lib.IQ2_ERR_ZERO_DIM
    assert b"iq2_dequantize_to_f16 expects non-zero dimensions" in lib.iq2_last_error()


def test_unknown_variant_rejected(lib):
    assert _matmul(lib, variant=9) == _lib.IQ2_ERR_INVALID_ARGUMENT


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device path")
def test_no_device_is_a_device_error(lib):
    assert _matmul(lib) == _lib.IQ2_ERR_DEVICE
    assert b"requires a CUDA device" in lib.iq2_last_error()


def test_error_message_is_per_call(lib):
    _matmul(lib, out_dim=0)
    assert lib.iq2_last_error() != b""
    assert lib.iq2_gather_columns(None, 0, 0, 0, None, None) == _lib.IQ2_OK
    assert lib.iq2_last_error() == b""


def test_workspace_query_needs_no_device(lib):
    assert lib.iq2_matmul_workspace_size(16, 4096, 4096, 0, 0) > 0  # x limbs go through the workspace
    assert lib.iq2_matmul_workspace_size(1, 4096, 4096, 0, 0) == 0  # small K: limbs made in shared memory
    assert lib.iq2_matmul_workspace_size(0, 4096, 4096, 0, 0) == 0
    # IQ2_XS, IQ2_S and IQ3_S at m <= 32: their decode GEMV's x limbs (always through the
    # workspace); above, every format reports the tensor-core GEMM's
    assert lib.iq2_matmul_workspace_size(1, 4096, 4096, 0, 1) > 0
    assert lib.iq2_matmul_workspace_size(1, 4096, 4096, 0, 2) > 0
    assert lib.iq2_matmul_workspace_size(1, 4096, 4096, 0, 3) > 0
    assert lib.iq2_matmul_workspace_size(64, 4096, 4096, 0, 3) > 0


def test_activation_quant_modes_without_device(lib):
    args = (None, 0, 1, None, 0, None, 0, 4, 256, 0)
    tail = (None, None, 0, None)
    assert lib.iq2_matmul_with_activation_quant(*args, 1, 0, *tail) == _lib.IQ2_ERR_DEVICE  # W8A8 runs
    assert lib.iq2_matmul_with_activation_quant(*args, 2, 1, *tail) == _lib.IQ2_ERR_UNSUPPORTED
    assert b"strict" in lib.iq2_last_error()
    assert lib.iq2_matmul_with_activation_quant(*args, 7, 0, *tail) == _lib.IQ2_ERR_INVALID_ARGUMENT


def test_w8a8_workspace_query_needs_no_device(lib):
    off = lib.iq2_matmul_workspace_size(3, 4096, 4096, 0, 0)
    w8 = lib.iq2_matmul_with_activation_quant_workspace_size(3, 4096, 4096, 0, 0, 1)
    assert w8 >= off + 3 * 4096 * 4
    assert lib.iq2_matmul_with_activation_quant_workspace_size(3, 4096, 4096, 0, 0, 0) == off


def test_sharded_workspace_query_covers_the_exchange_buffers(lib):
    """A sharded call's scratch is sized without a device: this rank's packed output slices, every
    rank's gathered slices, and the largest GEMM scratch of its projections (for m > 32 the chunks of
    the pipelined exchange run one after another and share it; f32 x adds the chunk's bf16 copy)."""
    shapes = [(28672, 8192), (28672, 8192), (8192, 28672)]  # configuration 3: gate, up, down (N, K)
    arr = (_lib.Iq2MatmulProblem * len(shapes))()
    for i, (n, k) in enumerate(shapes):
        arr[i].out_dim, arr[i].in_dim = n, k
    f32, bf16 = 0, 2
    for world in (2, 8):
        for m in (1, 3, 300, 2048):
            slices = sum(m * (n // world) for n, _ in shapes) * 4
            need = lib.iq2_matmul_grouped_sharded_workspace_size(arr, len(shapes), m, bf16, world)
            assert need >= slices * (world + 1)
            if m > 32:
                need_f32 = lib.iq2_matmul_grouped_sharded_workspace_size(arr, len(shapes), m, f32, world)
                assert need_f32 >= slices * (world + 1) + m * 28672 * 2  # down's x rows as bf16
    assert lib.iq2_matmul_grouped_sharded_workspace_size(arr, len(shapes), 0, bf16, 2) == 0
    assert lib.iq2_matmul_grouped_sharded_workspace_size(arr, 0, 2048, bf16, 2) == 0
