"""Parity at the benchmark configurations' own shapes, against the CPU oracle (the reference's CPU
path restated, src/iq2_matmul.rs:833-883, pinned to the reference's kernels in test_oracle.py):

* configuration 3, the Llama-3-70B FFN projections (gate/up 8192x28672, down 28672x8192: K = 28672 is
  112 blocks per row): M = 1 through the decode GEMV (single and grouped calls, f32 x) and M = 2048
  through the tcgen05 GEMM (bf16 x), on sampled output columns (the oracle's column sample);
* configuration 4, the Llama-3-8B linear stack with the benchmark's fixed dataflow (q, k, v, gate, up
  on x; o on q; down on up; the next layer's x = RMS-normalised down), two layers at M = 1 and
  M = 32: every projection against the oracle on the same input, and the chain's final output
  against the oracle's own chain.

Tolerances: the decode GEMV (m <= 32) relative L2 <= 1e-4; the GEMM <= 2e-2 against the oracle
(its weights are rounded to bf16) and <= 1e-4 against a plain fp32 matmul of the same bf16
operands; the two-layer chain <= 3e-4 (two layers of 1e-4-class errors, each layer's input
already carrying the previous layer's)."""
import numpy as np
import pytest
import torch

import candelora_metal_kernels_b200 as c
from candelora_metal_kernels_b200 import synth
from conftest import rel_l2

pytestmark = pytest.mark.gpu

GEMV_TOL = 1e-4
GEMM_ORACLE_TOL = 2e-2
GEMM_FP32_TOL = 1e-4
CHAIN_TOL = 3e-4
QS, SC = 64, 2


def _sample_cols(n: int, seed: int, count: int = 48) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return np.unique(np.concatenate([np.arange(8), rng.integers(0, n, count), [n - 1]]))


def _rows(qs: torch.Tensor, sc: torch.Tensor, cols: np.ndarray, k: int):
    """The packed weight rows `cols` of a matrix, as a smaller matrix of len(cols) rows."""
    nb = (k + 255) // 256
    idx = torch.as_tensor(cols, device=qs.device)
    return (qs.view(-1, nb * QS)[idx].reshape(-1).contiguous(), sc.view(-1, nb * SC)[idx].reshape(-1).contiguous())


@pytest.fixture(scope="module")
def ffn70b():
    return [(name, k, n, *synth.iq2xxs_weights(n, k, seed=700 + i, device="cuda"))
            for i, (name, k, n) in enumerate(synth.LLAMA3_70B_FFN)]


def test_config3_ffn70b_decode_m1_single_and_grouped(oracle, ffn70b):
    xs = [synth.activations(1, k, seed=800 + i, device="cuda") for i, (_, k, _, _, _) in enumerate(ffn70b)]
    grouped = c.iq2_matmul_grouped([(xs[i], qs, sc, n, k) for i, (_, k, n, qs, sc) in enumerate(ffn70b)])
    for i, (name, k, n, qs, sc) in enumerate(ffn70b):
        y = c.iq2_xxs_matmul(xs[i], qs, sc, n, k)
        # (the grouped launch splits K over other warps, so only the partial-sum order differs)
        assert rel_l2(grouped[i].double().cpu().numpy(), y.double().cpu().numpy()) <= 1e-6, name
        cols = _sample_cols(n, i)
        ref = oracle.matmul(xs[i].cpu().numpy(), qs.cpu().numpy(), sc.cpu().numpy(), n, k, cols=cols)
        assert rel_l2(y.cpu().numpy()[:, cols], ref) <= GEMV_TOL, name


def test_config3_ffn70b_prefill_m2048(oracle, ffn70b):
    m = 2048
    for i, (name, k, n, qs, sc) in enumerate(ffn70b):
        x = synth.activations(m, k, seed=900 + i, dtype=torch.bfloat16, device="cuda")
        y = c.iq2_xxs_matmul(x, qs, sc, n, k)
        assert bool(torch.isfinite(y).all()), name
        cols = _sample_cols(n, 10 + i, count=24)
        ys = y[:, torch.as_tensor(cols, device="cuda")].double().cpu().numpy()
        # the same bf16 operands in fp32: x and the sampled weight rows rounded to bf16
        qr, sr = _rows(qs, sc, cols, k)
        w = c.iq2_dequantize(qr, sr, len(cols), k, dtype=torch.bfloat16).float()
        exact = (x.float() @ w.T).double().cpu().numpy()
        assert rel_l2(ys, exact) <= GEMM_FP32_TOL, name
        ref = oracle.matmul(x.view(torch.int16).cpu().numpy().view(np.uint16), qs.cpu().numpy(), sc.cpu().numpy(),
                            n, k, cols=cols, x_dtype="bf16")
        assert rel_l2(ys, ref) <= GEMM_ORACLE_TOL, name


def _rms_norm(d):
    return d / np.sqrt(np.mean(d.astype(np.float64) ** 2, axis=1, keepdims=True) + 1e-6).astype(np.float32)


@pytest.mark.parametrize("m", [1, 32])
def test_config4_two_layer_chain(oracle, m):
    layers = 2
    W = [{name: (k, n, *synth.iq2xxs_weights(n, k, seed=layer * 16 + pi, device="cuda"))
          for pi, (name, k, n) in enumerate(synth.LLAMA3_8B_PROJECTIONS)} for layer in range(layers)]
    Wh = [{name: (k, n, qs.cpu().numpy(), sc.cpu().numpy()) for name, (k, n, qs, sc) in lay.items()} for lay in W]
    x0 = synth.activations(m, 4096, seed=4242, rms_normalize=True)

    # the GPU chain (as the benchmark's forward pass: three calls per layer)
    x = x0.cuda()
    gpu_outs = []
    for lay in W:
        first = ("q", "k", "v", "gate", "up")
        ys = c.iq2_matmul_grouped([(x, lay[nm][2], lay[nm][3], lay[nm][1], lay[nm][0]) for nm in first])
        outs = dict(zip(first, ys))
        outs["o"] = c.iq2_matmul_grouped([(outs["q"], lay["o"][2], lay["o"][3], lay["o"][1], lay["o"][0])])[0]
        outs["down"] = c.iq2_matmul_grouped(
            [(outs["up"], lay["down"][2], lay["down"][3], lay["down"][1], lay["down"][0])])[0]
        gpu_outs.append({k_: v.cpu().numpy() for k_, v in outs.items()} | {"x": x.cpu().numpy()})
        d = outs["down"]
        x = d * torch.rsqrt((d * d).mean(dim=1, keepdim=True) + 1e-6)
    gpu_final = x.cpu().numpy()

    # every projection against the oracle on the very input the GPU used
    for li, (lay, g) in enumerate(zip(Wh, gpu_outs)):
        inputs = {"q": g["x"], "k": g["x"], "v": g["x"], "gate": g["x"], "up": g["x"], "o": g["q"], "down": g["up"]}
        for nm, (k, n, qs, sc) in lay.items():
            cols = _sample_cols(n, 100 * li + len(nm))
            ref = oracle.matmul(inputs[nm], qs, sc, n, k, cols=cols)
            assert rel_l2(g[nm][:, cols], ref) <= GEMV_TOL, (li, nm)

    # the oracle's own chain, end to end (the next layer's x depends on up -> down only)
    xo = x0.numpy()
    for lay in Wh:
        def mm(nm, inp):
            k, n, qs, sc = lay[nm]
            return oracle.matmul(inp, qs, sc, n, k)
        xo = _rms_norm(mm("down", mm("up", xo)))
    assert rel_l2(gpu_final, xo) <= CHAIN_TOL
