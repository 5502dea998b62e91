"""GPU parity of the matmul path (C ABI via the host binding) against the CPU oracle and the
reference's golden vectors. Tolerance (from the benchmark specification) for the decode path with
f32/f16/bf16 activations: relative L2 <= 1e-4 for every m <= 32, plus the reference test's own
criterion, every |diff| <= 2e-3 on its fixture (src/iq2_matmul.rs:1107-1125). For m <= 4 x is
held in four 7-bit limbs (28-bit fixed point per 256-block); for 5 <= m <= 32 in a 16-bit fixed
point value split into a signed high and an unsigned low byte (error ~4e-5)."""
import numpy as np
import pytest
import torch

import candelora_metal_kernels_b200 as c
from candelora_metal_kernels_b200 import synth
from conftest import rel_l2

pytestmark = pytest.mark.gpu

GEMV_TOL = 1e-4
WIDE_TOL = GEMV_TOL  # 16 < m <= 32 (the 16-bit split, as for 5 <= m <= 16)


def _dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _x16(bits: np.ndarray, dtype) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(dtype).cuda()


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
def test_reference_parity_fixture(golden, dtype):
    g = golden["ref_parity"]
    if dtype == "f32":
        x = _dev(g["x_f32"])
    else:
        x = _x16(g[f"x_{dtype}_bits"], torch.float16 if dtype == "f16" else torch.bfloat16)
    y = c.iq2_xxs_matmul(x, _dev(g["weight_bytes"]), _dev(g["weight_scales"]), 7, 320)
    torch.cuda.synchronize()
    ref = g[f"y_{dtype}"]
    yh = y.cpu().numpy()
    assert y.shape == (2, 7) and y.dtype == torch.float32
    assert np.max(np.abs(yh - ref)) <= 2e-3
    assert rel_l2(yh, ref) <= GEMV_TOL


def test_baseline_golden_nonunit_scales(golden):
    b = golden["baseline_small"]
    y = c.iq2_xxs_matmul(_dev(b["a_x_f32"]), _dev(b["a_weight_bytes"]), _dev(b["a_weight_scales"]), 33, 4096)
    assert rel_l2(y.cpu().numpy(), b["a_y"]) <= GEMV_TOL
    y = c.iq2_xxs_matmul(_x16(b["b_x_bf16_bits"], torch.bfloat16), _dev(b["b_weight_bytes"]),
                         _dev(b["b_weight_scales"]), 9, 1000)
    assert rel_l2(y.cpu().numpy(), b["b_y"]) <= GEMV_TOL


CASES = [  # m, n, k -- includes split-K (k=4096/14336), ragged k, odd n, every m tile width
    (1, 4096, 4096), (1, 14336, 4096), (1, 4096, 14336), (1, 1024, 4096),
    (2, 7, 320), (3, 33, 4096), (4, 100, 1000), (5, 64, 512), (8, 200, 2048), (16, 130, 4096),
    (12, 50, 768), (1, 1, 256), (7, 31, 300),
]


@pytest.mark.parametrize("m,n,k", CASES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_gemv_matches_oracle(oracle, m, n, k, dtype):
    qs, sc = synth.iq2xxs_weights(n, k, seed=n * 131 + k)
    x = synth.activations(m, k, seed=m * 7 + n, dtype=dtype)
    y = c.iq2_xxs_matmul(x.cuda(), qs.cuda(), sc.cuda(), n, k).cpu().numpy()
    cols = np.unique(np.concatenate([np.arange(min(n, 24)), np.random.default_rng(n).integers(0, n, 40),
                                     [n - 1]]))
    xo = x.float().numpy() if dtype == torch.float32 else x.view(torch.int16).numpy().view(np.uint16)
    ref = oracle.matmul(xo, qs.numpy(), sc.numpy(), n, k, cols=cols,
                        x_dtype="f32" if dtype == torch.float32 else "bf16")
    assert rel_l2(y[:, cols], ref) <= GEMV_TOL


WIDE_CASES = [(17, 33, 4096), (20, 100, 1000), (24, 4096, 4096), (31, 7, 300), (32, 14336, 4096),
              (32, 4096, 14336)]


@pytest.mark.parametrize("m,n,k", WIDE_CASES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_gemv_wide_m_matches_oracle(oracle, m, n, k, dtype):
    qs, sc = synth.iq2xxs_weights(n, k, seed=n * 17 + k)
    x = synth.activations(m, k, seed=m * 3 + n, dtype=dtype)
    y = c.iq2_xxs_matmul(x.cuda(), qs.cuda(), sc.cuda(), n, k).cpu().numpy()
    cols = np.unique(np.concatenate([np.arange(min(n, 16)), np.random.default_rng(n).integers(0, n, 24),
                                     [n - 1]]))
    xo = x.float().numpy() if dtype == torch.float32 else x.view(torch.int16).numpy().view(np.uint16)
    ref = oracle.matmul(xo, qs.numpy(), sc.numpy(), n, k, cols=cols,
                        x_dtype="f32" if dtype == torch.float32 else "bf16")
    assert rel_l2(y[:, cols], ref) <= WIDE_TOL


def test_gemv_wide_m_grouped_and_full_output():
    """m = 32 through one grouped launch (four projections sharing x, the prep kernel writing the
    split 16-bit x once) equals the single calls, and the whole output is within the bound of the
    exact product (f32 dequant x f64)."""
    m, k = 32, 4096
    shapes = [4096, 1024, 14336, 96]
    W = [tuple(t.cuda() for t in synth.iq2xxs_weights(n, k, seed=50 + i)) for i, n in enumerate(shapes)]
    x = synth.activations(m, k, seed=51, device="cuda")
    ys = c.iq2_matmul_grouped([(x, W[i][0], W[i][1], n, k) for i, n in enumerate(shapes)])
    for i, n in enumerate(shapes):
        single = c.iq2_xxs_matmul(x, W[i][0], W[i][1], n, k)
        assert rel_l2(ys[i].double().cpu().numpy(), single.double().cpu().numpy()) <= 1e-6
        w = c.iq2_dequantize(W[i][0], W[i][1], n, k, dtype=torch.float32)
        exact = x.double() @ w.double().T
        assert rel_l2(ys[i].double().cpu().numpy(), exact.cpu().numpy()) <= WIDE_TOL


@pytest.mark.parametrize("m,n,k", [(1, 14336, 4096), (4, 4096, 14336), (16, 1024, 4096)])
def test_gemv_full_output_against_exact_dequant(m, n, k):
    """Whole-output check at benchmark sizes: the exact weights (f32 dequant, itself bit-exact
    against the oracle) times x in f64 on the GPU is the exact product; the GEMV must be within
    the tolerance of it everywhere."""
    qs, sc = synth.iq2xxs_weights(n, k, seed=99 + n)
    qs, sc = qs.cuda(), sc.cuda()
    x = synth.activations(m, k, seed=5, device="cuda")
    y = c.iq2_xxs_matmul(x, qs, sc, n, k)
    w = c.iq2_dequantize(qs, sc, n, k, dtype=torch.float32)
    exact = x.double() @ w.double().T
    assert rel_l2(y.double().cpu().numpy(), exact.cpu().numpy()) <= GEMV_TOL


def test_gemv_deterministic_and_reusable_buffers():
    n, k, m = 4096, 14336, 1
    qs, sc = synth.iq2xxs_weights(n, k, seed=1)
    qs, sc = qs.cuda(), sc.cuda()
    x = synth.activations(m, k, seed=2, device="cuda")
    y1 = c.iq2_xxs_matmul(x, qs, sc, n, k)
    ws = torch.empty(c.workspace_bytes(m, n, k, torch.float32), dtype=torch.uint8, device="cuda")
    out = torch.empty((m, n), dtype=torch.float32, device="cuda")
    for _ in range(3):
        y2 = c.iq2_xxs_matmul(x, qs, sc, n, k, out=out, workspace=ws)
    assert y2.data_ptr() == out.data_ptr()
    assert torch.equal(y1, y2)


def test_rank1_x_and_empty_m():
    n, k = 64, 512
    qs, sc = synth.iq2xxs_weights(n, k, seed=3)
    qs, sc = qs.cuda(), sc.cuda()
    x = synth.activations(1, k, seed=4, device="cuda")
    y1 = c.iq2_xxs_matmul(x[0], qs, sc, n, k)
    assert y1.shape == (n,)
    assert torch.equal(y1, c.iq2_xxs_matmul(x, qs, sc, n, k)[0])
    y0 = c.iq2_xxs_matmul(torch.empty(0, k, device="cuda"), qs, sc, n, k)
    assert y0.shape == (0, n)


def test_noncontiguous_x_and_misaligned_weights(oracle):
    """A strided x is made contiguous (src/iq2_matmul.rs:235); weight buffers at odd byte offsets
    (allowed by the reference's byte-offset views) take the unaligned path and agree."""
    n, k, m = 48, 1024, 3
    qs, sc = synth.iq2xxs_weights(n, k, seed=8)
    x = synth.activations(k, m, seed=9).T  # [m, k], non-contiguous
    big_q = torch.zeros(qs.numel() + 16, dtype=torch.uint8)
    big_s = torch.zeros(sc.numel() + 16, dtype=torch.uint8)
    big_q[3:3 + qs.numel()] = qs
    big_s[1:1 + sc.numel()] = sc
    qd, sd = big_q.cuda()[3:3 + qs.numel()], big_s.cuda()[1:1 + sc.numel()]
    y = c.iq2_xxs_matmul(x.cuda(), qd, sd, n, k).cpu().numpy()
    ref = oracle.matmul(x.contiguous().numpy(), qs.numpy(), sc.numpy(), n, k)
    assert rel_l2(y, ref) <= GEMV_TOL


def test_oversized_buffers_are_accepted():
    """Buffers longer than needed are fine (the reference checks elem_count >= expected)."""
    n, k = 32, 512
    qs, sc = synth.iq2xxs_weights(n, k, seed=10)
    x = synth.activations(2, k, seed=11, device="cuda")
    y = c.iq2_xxs_matmul(x, torch.cat([qs, qs]).cuda(), torch.cat([sc, sc]).cuda(), n, k)
    assert torch.equal(y, c.iq2_xxs_matmul(x, qs.cuda(), sc.cuda(), n, k))


def test_nonfinite_activation_block_gives_nan_row():
    n, k = 16, 512
    qs, sc = synth.iq2xxs_weights(n, k, seed=12)
    x = synth.activations(2, k, seed=13, device="cuda")
    x[1, 300] = float("inf")
    y = c.iq2_xxs_matmul(x, qs.cuda(), sc.cuda(), n, k)
    assert torch.isfinite(y[0]).all() and not torch.isfinite(y[1]).any()


def test_grouped_matches_oracle_and_single_calls(oracle):
    """iq2_matmul_grouped over projections of different shapes, two of them sharing x."""
    m = 2
    shapes = [(4096, 4096), (1024, 4096), (1024, 4096), (14336, 1024), (300, 320), (4096, 14336)]
    xs = {k: synth.activations(m, k, seed=k, device="cuda") for k in {k for _, k in shapes}}
    probs, refs = [], []
    for i, (n, k) in enumerate(shapes):
        qs, sc = synth.iq2xxs_weights(n, k, seed=500 + i)
        probs.append((xs[k], qs.cuda(), sc.cuda(), n, k))
        cols = np.unique(np.concatenate([np.arange(min(n, 16)), np.random.default_rng(i).integers(0, n, 24), [n - 1]]))
        refs.append((cols, oracle.matmul(xs[k].cpu().numpy(), qs.numpy(), sc.numpy(), n, k, cols=cols)))
    outs = c.iq2_matmul_grouped(probs)
    for (cols, ref), y, pr in zip(refs, outs, probs):
        assert rel_l2(y.cpu().numpy()[:, cols], ref) <= GEMV_TOL
        single = c.iq2_xxs_matmul(*pr[:5])
        assert rel_l2(y.cpu().numpy(), single.cpu().numpy()) <= 1e-6


@pytest.mark.parametrize("m", [1, 4, 8])
def test_grouped_ragged_mix_every_cursor_width(oracle, m):
    """One grouped launch over projections with ragged rows (N not a multiple of the row tile),
    ragged K, a one-block K and a one-row N, for the n8-tile widths whose issue side keeps a
    running cursor: tile and problem changes fall inside warps' ranges."""
    shapes = [(97, 2816), (64, 256), (1, 4096), (130, 320), (33, 768), (512, 1000), (45, 256)]
    probs, refs = [], []
    for i, (n, k) in enumerate(shapes):
        x = synth.activations(m, k, seed=40 + i, device="cuda")
        qs, sc = synth.iq2xxs_weights(n, k, seed=900 + 10 * m + i)
        probs.append((x, qs.cuda(), sc.cuda(), n, k))
        refs.append(oracle.matmul(x.cpu().numpy(), qs.numpy(), sc.numpy(), n, k))
    outs = c.iq2_matmul_grouped(probs)
    for (n, k), y, ref in zip(shapes, outs, refs):
        assert rel_l2(y.cpu().numpy(), ref) <= GEMV_TOL, (m, n, k)


def test_grouped_many_problems_beyond_one_launch(oracle):
    """More projections than one launch holds (256): split into several launches."""
    m, n, k = 1, 64, 512
    x = synth.activations(m, k, seed=3, device="cuda")
    probs = []
    for i in range(300):
        qs, sc = synth.iq2xxs_weights(n, k, seed=i)
        probs.append((x, qs.cuda(), sc.cuda(), n, k))
    outs = c.iq2_matmul_grouped(probs)
    for i in (0, 255, 256, 299):
        qs, sc = probs[i][1].cpu().numpy(), probs[i][2].cpu().numpy()
        assert rel_l2(outs[i].cpu().numpy(), oracle.matmul(x.cpu().numpy(), qs, sc, n, k)) <= GEMV_TOL


def test_stream_k_boundaries_all_m(oracle):
    """Shapes whose step counts split unevenly over the warps, for every n8-tile width."""
    for m in (1, 2, 3, 4, 6, 8, 11, 16):
        n, k = 97, 2816  # 11 blocks per row
        qs, sc = synth.iq2xxs_weights(n, k, seed=m)
        x = synth.activations(m, k, seed=m + 100, device="cuda")
        y = c.iq2_xxs_matmul(x, qs.cuda(), sc.cuda(), n, k)
        assert rel_l2(y.cpu().numpy(), oracle.matmul(x.cpu().numpy(), qs.numpy(), sc.numpy(), n, k)) <= GEMV_TOL, m
