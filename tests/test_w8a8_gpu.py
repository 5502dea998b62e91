"""GPU parity of the W8A8 activation-quant mode (iq2_matmul_with_activation_quant with
ActivationQuantMode::W8A8): every x row quantised to int8 with 127/max|x| and back, as the
reference's W8A8 kernels do (src/metal_src/iq2_matmul.metal:85-102, :437-499), then the matmul.

Against the reference's own W8A8 kernel outputs (golden vectors, its parity fixture: the
reference test's 3e-3 absolute bound and our rel. L2 bound) and against the oracle restatement at
larger sizes: rel. L2 <= 1e-4 for m <= 32 (the int8 activations go straight into the decode GEMV:
exact integer products, f32 scaling), <= 2e-2 beyond (quant-dequant, then the bf16 tensor-core path)."""
import numpy as np
import pytest
import torch

import candelora_metal_kernels_b200 as c
from candelora_metal_kernels_b200 import synth
from conftest import rel_l2

pytestmark = pytest.mark.gpu

W8 = c.ActivationQuantConfig(c.ActivationQuantMode.W8A8)


def _w8a8(x, qs, sc, n, k):
    return c.iq2_matmul_with_activation_quant(x, qs, sc, n, k, c.Iq2MatmulVariant.Iq2Xxs, W8)


def test_w8a8_reference_fixture(golden):
    g = golden["ref_parity"]
    qs, sc = torch.from_numpy(g["weight_bytes"]).cuda(), torch.from_numpy(g["weight_scales"]).cuda()
    y = _w8a8(torch.from_numpy(g["x_f32"]).cuda(), qs, sc, 7, 320).cpu().numpy()
    assert np.abs(y - g["y_w8a8_f32"]).max() <= 3e-3  # the reference test's own bound (:1181-1253)
    assert rel_l2(y, g["y_w8a8_f32"]) <= 1e-6
    x16 = torch.from_numpy(g["x_f16_bits"].view(np.int16)).view(torch.float16).cuda()
    y16 = _w8a8(x16, qs, sc, 7, 320).cpu().numpy()
    assert rel_l2(y16, g["y_w8a8_f16"]) <= 1e-6


def test_w8a8_benchmark_distribution_golden(golden):
    b = golden["baseline_small"]
    qs, sc = torch.from_numpy(b["a_weight_bytes"]).cuda(), torch.from_numpy(b["a_weight_scales"]).cuda()
    y = _w8a8(torch.from_numpy(b["a_x_f32"]).cuda(), qs, sc, 33, 4096).cpu().numpy()
    assert rel_l2(y, b["a_y_w8a8"]) <= 1e-5


@pytest.mark.parametrize("m,n,k,tol", [(1, 4096, 4096, 1e-4), (5, 1000, 2304, 1e-4), (16, 333, 700, 1e-4),
                                       (32, 700, 1024, 1e-4), (9, 14336, 4096, 1e-4), (64, 512, 1024, 2e-2), (300, 1024, 4096, 2e-2)])
def test_w8a8_matches_oracle(oracle, m, n, k, tol):
    qs, sc = synth.iq2xxs_weights(n, k, seed=n + m)
    x = synth.activations(m, k, seed=m)
    x[0, 0] = 40.0  # one outlier row: a coarse int8 step for the rest of that row
    y = _w8a8(x.cuda(), qs.cuda(), sc.cuda(), n, k).cpu().numpy()
    cols = np.unique(np.concatenate([np.arange(min(n, 16)), [n - 1]]))
    ref = oracle.matmul(oracle.rowwise_qdq_w8a8(x.numpy()), qs.numpy(), sc.numpy(), n, k, cols=cols)
    assert rel_l2(y[:, cols], ref) <= tol


def test_w8a8_zero_row_uses_unit_scale(oracle):
    n, k = 64, 512
    qs, sc = synth.iq2xxs_weights(n, k, seed=3)
    x = torch.zeros(2, k)
    x[1] = synth.activations(1, k, seed=4)[0] * 1e-10  # max|x| < 1e-8: inv_scale = 1, everything rounds to 0
    y = _w8a8(x.cuda(), qs.cuda(), sc.cuda(), n, k).cpu().numpy()
    assert np.array_equal(y, np.zeros_like(y))


def test_w8a8_workspace_contract():
    import ctypes
    from candelora_metal_kernels_b200 import _lib
    lib = _lib.load()
    n, k, m = 256, 1024, 2
    qs, sc = (t.cuda() for t in synth.iq2xxs_weights(n, k, seed=1))
    x = synth.activations(m, k, seed=2, device="cuda")
    out = torch.empty(m, n, device="cuda")
    need = lib.iq2_matmul_with_activation_quant_workspace_size(m, n, k, 0, 0, 1)
    args = [ctypes.c_void_p(x.data_ptr()), 0, m, ctypes.c_void_p(qs.data_ptr()), qs.numel(),
            ctypes.c_void_p(sc.data_ptr()), sc.numel(), n, k, 0, 1, 1, ctypes.c_void_p(out.data_ptr())]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    assert lib.iq2_matmul_with_activation_quant(*args, ctypes.c_void_p(ws.data_ptr()), need - 1, stream) \
        == _lib.IQ2_ERR_WORKSPACE
    assert lib.iq2_matmul_with_activation_quant(*args, ctypes.c_void_p(ws.data_ptr()), need, stream) == _lib.IQ2_OK
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()


def test_w8a8_nonfinite_row_is_nan():
    """A row with an infinity: the reference's int8 step becomes 0 and its dequantised values NaN,
    so that row's outputs are NaN; the other rows are unaffected."""
    n, k = 64, 1024
    qs, sc = synth.iq2xxs_weights(n, k, seed=21)
    x = synth.activations(3, k, seed=22)
    x[1, 5] = float("inf")
    y = _w8a8(x.cuda(), qs.cuda(), sc.cuda(), n, k).cpu()
    assert torch.isnan(y[1]).all()
    assert torch.isfinite(y[0]).all() and torch.isfinite(y[2]).all()
