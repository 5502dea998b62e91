"""GPU parity of the IQ2_XS, IQ2_S and IQ3_S formats (iq2_xs_matmul / iq2_s_matmul / iq3_s_matmul
and iq2_dequantize with those variants): against the reference kernels' golden outputs on the
reference's parity fixture, and against the oracle restatement on larger random blocks.
Dequantisation is bit-exact (f32 exact value, f16/bf16 round to nearest even); the matmul
accumulates in f32 with FMA, rel. L2 <= 1e-4 (f32 x)."""
import numpy as np
import pytest
import torch

import candelora_metal_kernels_b200 as c
from conftest import GOLDEN, rel_l2

pytestmark = pytest.mark.gpu

VARIANTS = {"iq2_xs": (c.Iq2MatmulVariant.Iq2Xs, 64, 10), "iq2_s": (c.Iq2MatmulVariant.Iq2S, 72, 10),
            "iq3_s": (c.Iq2MatmulVariant.Iq3S, 104, 6)}


def _blocks(variant, n, k, seed):
    """Random bytes for every field, d ~U[1e-3, 1e-2] as f16 at the start of each block's scales."""
    _, bpb, spb = VARIANTS[variant]
    nb = (k + 255) // 256
    rng = np.random.default_rng(seed)
    wb = rng.integers(0, 256, n * nb * bpb, dtype=np.uint8)
    ws = rng.integers(0, 256, n * nb * spb, dtype=np.uint8)
    d = rng.uniform(1e-3, 1e-2, n * nb).astype(np.float16).view(np.uint16)
    ws.reshape(-1, spb)[:, 0] = (d & 0xFF).astype(np.uint8)
    ws.reshape(-1, spb)[:, 1] = (d >> 8).astype(np.uint8)
    return wb, ws


@pytest.mark.parametrize("variant", list(VARIANTS))
def test_variant_reference_fixture(variant):
    v = dict(np.load(GOLDEN / "ref_variants.npz"))
    var = VARIANTS[variant][0]
    x = torch.from_numpy(v[f"{variant}_x"]).cuda()
    wb = torch.from_numpy(v[f"{variant}_weight_bytes"]).cuda()
    for sfx, ws_key, deq_key in (("", "weight_scales", "deq_f16_bits"), ("_d", "weight_scales_d", "deq_d_f16_bits")):
        ws = torch.from_numpy(v[f"{variant}_{ws_key}"]).cuda()
        y = c.iq2_matmul(x, wb, ws, 7, 320, var).cpu().numpy()
        want = v[f"{variant}_y{sfx}"]
        assert np.abs(y - want).max() <= 2e-3 * max(1.0, float(np.abs(want).max()))  # the reference test's bound
        assert rel_l2(y, want) <= 1e-5
        deq = c.iq2_dequantize_to_f16(wb, ws, 7, 320, var).cpu().view(torch.int16).numpy().view(np.uint16)
        assert np.array_equal(deq, v[f"{variant}_{deq_key}"])


@pytest.mark.parametrize("variant", list(VARIANTS))
@pytest.mark.parametrize("m,n,k,xdt", [(1, 300, 4096, torch.float32), (5, 64, 1000, torch.float32),
                                       (20, 96, 2304, torch.float32), (3, 40, 512, torch.bfloat16)])
def test_variant_matmul_matches_oracle(oracle, variant, m, n, k, xdt):
    var = VARIANTS[variant][0]
    wb, ws = _blocks(variant, n, k, seed=n + k)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(m)).to(xdt)
    y = c.iq2_matmul(x.cuda(), torch.from_numpy(wb).cuda(), torch.from_numpy(ws).cuda(), n, k, var).cpu().numpy()
    ref = oracle.matmul(x.float().numpy(), wb, ws, n, k, variant=variant)
    assert rel_l2(y, ref) <= 1e-4


@pytest.mark.parametrize("variant", list(VARIANTS))
@pytest.mark.parametrize("m,offset,xdt", [(1, 0, torch.float32), (1, 1, torch.float32), (9, 3, torch.float32),
                                          (1, 0, torch.float16)])
def test_variant_matmul_chunks_and_unaligned(oracle, variant, m, offset, xdt):
    """Rows of more blocks than the kernel stages at a time (17 blocks, ragged K), weight buffers
    that start off any alignment (byte-wise loads), one token and a masked 8-token pass."""
    var = VARIANTS[variant][0]
    n, k = 40, 17 * 256 - 96
    wb, ws = _blocks(variant, n, k, seed=11 + m + offset)

    def dev(a):
        b = torch.zeros(a.size + offset, dtype=torch.uint8)
        b[offset:] = torch.from_numpy(a)
        return b.cuda()[offset:]
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(m)).to(xdt)
    y = c.iq2_matmul(x.cuda(), dev(wb), dev(ws), n, k, var).cpu().numpy()
    assert rel_l2(y, oracle.matmul(x.float().numpy(), wb, ws, n, k, variant=variant)) <= 1e-4


@pytest.mark.parametrize("variant", list(VARIANTS))
@pytest.mark.parametrize("dtype,name", [(torch.float32, "f32"), (torch.float16, "f16"), (torch.bfloat16, "bf16")])
def test_variant_dequant_bit_exact(oracle, variant, dtype, name):
    var = VARIANTS[variant][0]
    n, k = 33, 1000  # ragged K
    wb, ws = _blocks(variant, n, k, seed=7)
    got = c.iq2_dequantize(torch.from_numpy(wb).cuda(), torch.from_numpy(ws).cuda(), n, k, var, dtype=dtype).cpu()
    want = oracle.dequantize(wb, ws, n, k, name, variant=variant)
    if name == "f32":
        assert np.array_equal(got.numpy(), want)
    else:
        assert np.array_equal(got.view(torch.int16).numpy().view(np.uint16), want)


@pytest.mark.parametrize("variant", list(VARIANTS))
def test_variant_w8a8(oracle, variant):
    var = VARIANTS[variant][0]
    n, k, m = 48, 768, 3
    wb, ws = _blocks(variant, n, k, seed=3)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(5))
    cfg = c.ActivationQuantConfig(c.ActivationQuantMode.W8A8)
    y = c.iq2_matmul_with_activation_quant(x.cuda(), torch.from_numpy(wb).cuda(), torch.from_numpy(ws).cuda(),
                                           n, k, var, cfg).cpu().numpy()
    ref = oracle.matmul(oracle.rowwise_qdq_w8a8(x.numpy()), wb, ws, n, k, variant=variant)
    assert rel_l2(y, ref) <= 1e-4


# ---- m > 32: the tcgen05 GEMM (weights decoded to bf16 in shared memory), selected when the call
# ---- has the workspace iq2_matmul_workspace_size asks for
GEMM_FP32_TOL = 1e-4    # against a plain fp32 matmul of the same bf16 operands
GEMM_ORACLE_TOL = 2e-2  # against the oracle (the GEMM rounds x and the weights to bf16)


def _cuda_core(x, wb, ws, n, k, var):
    """The CUDA-core kernel: the C call with no workspace (the path a caller without one gets)."""
    import ctypes
    from candelora_metal_kernels_b200 import _lib
    lib = _lib.load()
    out = torch.empty(x.shape[0], n, dtype=torch.float32, device="cuda")
    dt = {torch.float32: _lib.DTYPE_F32, torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16}[x.dtype]
    rc = lib.iq2_matmul(ctypes.c_void_p(x.data_ptr()), dt, x.shape[0], ctypes.c_void_p(wb.data_ptr()), wb.numel(),
                        ctypes.c_void_p(ws.data_ptr()), ws.numel(), n, k, int(var), ctypes.c_void_p(out.data_ptr()),
                        None, 0, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc)
    return out


@pytest.mark.parametrize("variant", list(VARIANTS))
@pytest.mark.parametrize("m,n,k,xdt", [
    (33, 72, 1000, torch.float32),     # one 256-token tile, ragged K, a part-filled weight tile
    (300, 520, 4096, torch.bfloat16),  # paired CTAs, the odd one part-filled
    (600, 256, 2304, torch.float16),   # two pairs, the last pair's odd CTA without tokens
    (2048, 1024, 4096, torch.bfloat16),  # every pair tile split over K (fewer tiles than SMs)
])
def test_variant_gemm(oracle, variant, m, n, k, xdt):
    var = VARIANTS[variant][0]
    wb, ws = _blocks(variant, n, k, seed=m + n)
    assert c.workspace_bytes(m, n, k, xdt, var) > 0  # (the size query routes these to the GEMM)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(m)).to(xdt).cuda()
    wbd, wsd = torch.from_numpy(wb).cuda(), torch.from_numpy(ws).cuda()
    y = c.iq2_matmul(x, wbd, wsd, n, k, var)
    assert bool(torch.isfinite(y).all())
    w = c.iq2_dequantize(wbd, wsd, n, k, var, dtype=torch.bfloat16).float()
    exact = x.to(torch.bfloat16).float() @ w.T
    assert rel_l2(y.double().cpu().numpy(), exact.double().cpu().numpy()) <= GEMM_FP32_TOL
    cols = np.unique(np.concatenate([np.arange(4), np.random.default_rng(n).integers(0, n, 24), [n - 1]]))
    ref = oracle.matmul(x.float().cpu().numpy(), wb, ws, n, k, cols=cols, variant=variant)
    assert rel_l2(y.cpu().numpy()[:, cols], ref) <= GEMM_ORACLE_TOL
    assert rel_l2(y.cpu().numpy(), _cuda_core(x, wbd, wsd, n, k, var).cpu().numpy()) <= GEMM_ORACLE_TOL


@pytest.mark.parametrize("variant", list(VARIANTS))
def test_variant_w8a8_gemm(oracle, variant):
    """W8A8 at m > 32: the int8-rounded activations through the tensor-core GEMM."""
    var = VARIANTS[variant][0]
    n, k, m = 64, 1024, 48
    wb, ws = _blocks(variant, n, k, seed=9)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(6))
    cfg = c.ActivationQuantConfig(c.ActivationQuantMode.W8A8)
    y = c.iq2_matmul_with_activation_quant(x.cuda(), torch.from_numpy(wb).cuda(), torch.from_numpy(ws).cuda(),
                                           n, k, var, cfg).cpu().numpy()
    ref = oracle.matmul(oracle.rowwise_qdq_w8a8(x.numpy()), wb, ws, n, k, variant=variant)
    assert rel_l2(y, ref) <= GEMM_ORACLE_TOL


@pytest.mark.parametrize("variant", ["iq2_xs", "iq2_s", "iq3_s"])
@pytest.mark.parametrize("m", [1, 3, 8, 16, 32])
def test_variant_decode_gemv(oracle, variant, m):
    """IQ2_XS, IQ2_S and IQ3_S at m <= 32 on the IQ2_XXS decode GEMV (int8 tensor-core decode;
    IQ2_XS / IQ2_S: two MMAs per sub-block, one per 16-weight scale; IQ3_S: magnitudes 1..15 signed
    by a byte mask), selected when the call has the workspace the size query reports: against the
    oracle and the CUDA-core kernel (no workspace), f32 x, ragged K."""
    var = VARIANTS[variant][0]
    n, k = 1000, 4096 + 256 + 96
    wb, ws = _blocks(variant, n, k, seed=40 + m)
    assert c.workspace_bytes(m, n, k, torch.float32, var) > 0
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(50 + m)).cuda()
    wbd, wsd = torch.from_numpy(wb).cuda(), torch.from_numpy(ws).cuda()
    y = c.iq2_matmul(x, wbd, wsd, n, k, var)
    ref = oracle.matmul(x.cpu().numpy(), wb, ws, n, k, variant=variant)
    assert rel_l2(y.cpu().numpy(), ref) <= 1e-4
    assert rel_l2(y.cpu().numpy(), _cuda_core(x, wbd, wsd, n, k, var).cpu().numpy()) <= 1e-4
