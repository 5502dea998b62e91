"""iq2_matmul_noalloc, the decode matmul (m <= 16) that takes its scratch from the library's fixed
device array instead of a workspace, called through the C ABI and checked against iq2_matmul.

This file is collected last on purpose: it must pass both alone in a fresh process (where its
first call does the per-device set-up) and after every other test has used the library."""
import ctypes

import pytest
import torch

import candelora_metal_kernels_b200 as c
from candelora_metal_kernels_b200 import _lib, synth

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 8 * 1024 * 1024  # IQ2_NOALLOC_SCRATCH_BYTES in include/candelora_iq2.h

_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.float16: _lib.DTYPE_F16,
           torch.bfloat16: _lib.DTYPE_BF16}


def _ptr(t: torch.Tensor):
    return ctypes.c_void_p(t.data_ptr())


def _noalloc(lib, x, qs, sc, n, k, out):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.iq2_matmul_noalloc(_ptr(x), _DTYPES[x.dtype], x.shape[0], _ptr(qs), qs.numel(), _ptr(sc),
                                  sc.numel(), n, k, _ptr(out), ctypes.c_void_p(stream))


@pytest.mark.parametrize("m,n,k,dtype", [(1, 14336, 4096, torch.float32), (4, 4096, 14336, torch.float32),
                                         (16, 1000, 2304, torch.bfloat16), (3, 33, 300, torch.float16)])
def test_noalloc_matches_iq2_matmul_on_two_calls_in_a_row(m, n, k, dtype):
    lib = _lib.load()
    qs, sc = synth.iq2xxs_weights(n, k, seed=n + k)
    qs, sc = qs.cuda(), sc.cuda()
    xs = [synth.activations(m, k, seed=s, dtype=dtype, device="cuda") for s in (11, 12)]
    outs = [torch.full((m, n), float("nan"), device="cuda") for _ in xs]
    before = torch.cuda.memory_allocated()
    for x, out in zip(xs, outs):  # back to back on one stream: the second reuses the scratch
        rc = _noalloc(lib, x, qs, sc, n, k, out)
        assert rc == _lib.IQ2_OK, lib.iq2_last_error()
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() == before
    for x, out in zip(xs, outs):
        want = c.iq2_xxs_matmul(x, qs, sc, n, k)  # the existing entry point, iq2_matmul
        assert torch.isfinite(out).all()
        # the same kernels on the same inputs (deterministic: no atomics): identical bits
        assert torch.equal(out, want)


def _misaligned(t: torch.Tensor, offset: int = 1) -> torch.Tensor:
    """A copy of `t` whose data starts `offset` bytes past a 16-byte boundary."""
    buf = torch.empty(t.numel() + 16, dtype=torch.uint8, device=t.device)
    v = buf[offset:offset + t.numel()]
    v.copy_(t)
    return v


def test_noalloc_unaligned_weights_take_the_generic_kernel_twice_in_a_row():
    """Weight buffers that do not start on a 16-byte (bytes) / 4-byte (scales) boundary go to the
    generic decode kernel, which needs no scratch at all; the result equals iq2_matmul's."""
    lib = _lib.load()
    m, n, k = 2, 96, 320
    qs, sc = synth.iq2xxs_weights(n, k, seed=5)
    qs, sc = _misaligned(qs.cuda()), _misaligned(sc.cuda(), 2)
    assert qs.data_ptr() % 16 != 0 and sc.data_ptr() % 4 != 0
    for seed in (21, 22):
        x = synth.activations(m, k, seed=seed, device="cuda")
        out = torch.full((m, n), float("nan"), device="cuda")
        rc = _noalloc(lib, x, qs, sc, n, k, out)
        assert rc == _lib.IQ2_OK, lib.iq2_last_error()
        assert torch.equal(out, c.iq2_xxs_matmul(x, qs, sc, n, k))


def test_noalloc_rejects_problems_beyond_the_scratch():
    lib = _lib.load()
    m, n, k = 16, 256, 262144
    assert lib.iq2_matmul_workspace_size(m, n, k, _lib.DTYPE_F32, 0) > SCRATCH_BYTES
    qs = torch.zeros(n * k // 4, dtype=torch.uint8, device="cuda")
    sc = torch.zeros(n * k // 128, dtype=torch.uint8, device="cuda")
    x = torch.zeros(m, k, device="cuda")
    out = torch.zeros(m, n, device="cuda")
    assert _noalloc(lib, x, qs, sc, n, k, out) == _lib.IQ2_ERR_WORKSPACE
    assert b"more than the library's fixed" in lib.iq2_last_error()


def test_noalloc_rejects_prefill_sizes():
    lib = _lib.load()
    m, n, k = 17, 64, 256
    qs, sc = synth.iq2xxs_weights(n, k, seed=1)
    x = torch.zeros(m, k, device="cuda")
    out = torch.zeros(m, n, device="cuda")
    assert _noalloc(lib, x, qs.cuda(), sc.cuda(), n, k, out) == _lib.IQ2_ERR_UNSUPPORTED
    assert b"m <= 16" in lib.iq2_last_error()
