"""Error behaviour on a GPU box: the reference's bail conditions (src/iq2_matmul.rs:210-259,
:300-302, :581-589) and the C ABI's workspace contract."""
import ctypes

import pytest
import torch

import candelora_metal_kernels_b200 as c
from candelora_metal_kernels_b200 import _lib, synth

pytestmark = pytest.mark.gpu


def _setup(n=16, k=512, m=2):
    qs, sc = synth.iq2xxs_weights(n, k, seed=1)
    return synth.activations(m, k, seed=2, device="cuda"), qs.cuda(), sc.cuda()


def test_buffers_too_small():
    x, qs, sc = _setup()
    with pytest.raises(c.Iq2Error, match="weight_bytes too small: got 2047 expected at least 2048") as e:
        c.iq2_xxs_matmul(x, qs[:-1], sc, 16, 512)
    assert e.value.code == _lib.IQ2_ERR_TOO_SMALL
    with pytest.raises(c.Iq2Error, match="weight_scales too small: got 63 expected at least 64"):
        c.iq2_xxs_matmul(x, qs, sc[:-1], 16, 512)
    with pytest.raises(c.Iq2Error, match="weight_bytes too small"):
        c.iq2_dequantize_to_f16(qs[:100], sc, 16, 512)


def test_device_mismatch_and_host_tensors():
    x, qs, sc = _setup()
    with pytest.raises(c.Iq2Error, match="requires a CUDA device"):
        c.iq2_xxs_matmul(x.cpu(), qs, sc, 16, 512)
    with pytest.raises(c.Iq2Error, match="device mismatch"):
        c.iq2_xxs_matmul(x, qs.cpu(), sc, 16, 512)


def test_dtype_and_shape_errors():
    x, qs, sc = _setup()
    with pytest.raises(c.Iq2Error, match="expects U8 weight bytes/scales"):
        c.iq2_xxs_matmul(x, qs.to(torch.int32), sc, 16, 512)
    with pytest.raises(c.Iq2Error, match="unsupported x dtype"):
        c.iq2_xxs_matmul(x.double(), qs, sc, 16, 512)
    with pytest.raises(c.Iq2Error, match="x last dim=512 expected in_dim=256"):
        c.iq2_xxs_matmul(x, qs, sc, 16, 256)
    with pytest.raises(c.Iq2Error, match="rank 1 or 2"):
        c.iq2_xxs_matmul(x[None], qs, sc, 16, 512)


def test_other_variants_and_activation_modes():
    x, qs, sc = _setup()
    # IQ2_XS: its own block geometry (64 + 10 bytes per block); too-small scales are rejected
    with pytest.raises(c.Iq2Error, match="weight_scales too small") as e:
        c.iq2_xs_matmul(x, torch.zeros(16 * 2 * 64, dtype=torch.uint8, device="cuda"),
                        torch.zeros(16 * 2 * 2, dtype=torch.uint8, device="cuda"), 16, 512)
    assert e.value.code == _lib.IQ2_ERR_TOO_SMALL
    y = c.iq2_xs_matmul(x, torch.zeros(16 * 2 * 64, dtype=torch.uint8, device="cuda"),
                        torch.zeros(16 * 2 * 10, dtype=torch.uint8, device="cuda"), 16, 512)
    assert torch.equal(y, torch.zeros_like(y))  # d = 0 everywhere
    strict = c.ActivationQuantConfig(c.ActivationQuantMode.W4A8, strict=True)
    with pytest.raises(c.Iq2Error, match="strict mode"):
        c.iq2_matmul_with_activation_quant(x, qs, sc, 16, 512, c.Iq2MatmulVariant.Iq2Xxs, strict)
    lax = c.ActivationQuantConfig(c.ActivationQuantMode.W4A8, strict=False)
    y = c.iq2_matmul_with_activation_quant(x, qs, sc, 16, 512, c.Iq2MatmulVariant.Iq2Xxs, lax)
    assert torch.equal(y, c.iq2_xxs_matmul(x, qs, sc, 16, 512))


def test_c_abi_workspace_contract():
    # k = 14336 at m = 1: the x limbs go through the workspace (small k needs none)
    x, qs, sc = _setup(n=1024, k=14336, m=1)
    lib = _lib.load()
    out = torch.empty((1, 1024), device="cuda")
    need = lib.iq2_matmul_workspace_size(1, 1024, 14336, 0, 0)
    assert need > 0
    assert lib.iq2_matmul_workspace_size(1, 1024, 4096, 0, 0) == 0
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = [ctypes.c_void_p(x.data_ptr()), 0, 1, ctypes.c_void_p(qs.data_ptr()), qs.numel(),
            ctypes.c_void_p(sc.data_ptr()), sc.numel(), 1024, 14336, 0, ctypes.c_void_p(out.data_ptr())]
    assert lib.iq2_matmul(*args, None, 0, stream) == _lib.IQ2_ERR_WORKSPACE
    assert lib.iq2_matmul(*args, ctypes.c_void_p(ws.data_ptr()), need - 1, stream) == _lib.IQ2_ERR_WORKSPACE
    assert lib.iq2_matmul(*args, ctypes.c_void_p(ws.data_ptr()), need, stream) == _lib.IQ2_OK
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()


def test_gemm_wait_that_runs_out_is_reported_and_the_context_stays_usable():
    """The prefill GEMM's pipeline waits are bounded: with the test hook a stage's "weights
    written" arrival is withheld (a flag that nothing sets), the MMA thread's wait on it runs out
    after 20 ms, and iq2_device_check reports IQ2_ERR_TIMEOUT; afterwards the status is clear and
    the same call computes the right result again. No GPU fault is involved."""
    lib = _lib.load()
    m, n, k = 256, 512, 1024
    qs, sc = synth.iq2xxs_weights(n, k, seed=7)
    qs, sc = qs.cuda(), sc.cuda()
    x = synth.activations(m, k, seed=8, dtype=torch.bfloat16, device="cuda")
    want = c.iq2_xxs_matmul(x, qs, sc, n, k)
    c.device_check()  # nothing timed out so far
    assert lib.iq2_testing_set_gemm_stall(20_000_000, 2) == _lib.IQ2_OK
    try:
        c.iq2_xxs_matmul(x, qs, sc, n, k)  # returns at once: the kernel is asynchronous
        with pytest.raises(c.Iq2Error, match="decoded weights") as e:
            c.device_check()
        assert e.value.code == _lib.IQ2_ERR_TIMEOUT
    finally:
        lib.iq2_testing_set_gemm_stall(0, 0)
    c.device_check()  # the status was cleared by the check that reported it
    assert torch.equal(c.iq2_xxs_matmul(x, qs, sc, n, k), want)
    c.device_check()
