"""GPU parity of the column-sharded path (iq2_matmul_grouped_sharded: local slices, one NCCL
all-gather, one scatter kernel) against the single-GPU iq2_matmul on the full weights. Needs two
GPUs of one node; skipped otherwise."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = 2
TOL = 1e-5  # same kernels per row; only the order of the per-warp partial sums can differ


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, port: int, q):
    try:
        import numpy as np
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=WORLD)  # carries the NCCL id only
        import candelora_metal_kernels_b200 as c
        from candelora_metal_kernels_b200 import synth
        from candelora_metal_kernels_b200.sharded import (Iq2Comm, iq2_matmul_grouped_sharded, iq2_matmul_sharded,
                                                          shard_rows)
        comm = Iq2Comm()
        dev = torch.device("cuda", rank)

        def rel(a, b):
            a, b = a.double().cpu().numpy(), b.double().cpu().numpy()
            return float(np.linalg.norm(a - b) / np.linalg.norm(b))

        errs = {}
        shapes = [(4096, 4096), (1024, 14336), (14336, 4096)]
        full = [tuple(t.to(dev) for t in synth.iq2xxs_weights(n, k, seed=i)) for i, (n, k) in enumerate(shapes)]
        for m in (1, 3):
            xs = [synth.activations(m, k, seed=20 + i, device=dev) for i, (n, k) in enumerate(shapes)]
            # one projection per call (m = 1: all-gathered straight into the output)
            for i, (n, k) in enumerate(shapes):
                qs_r, sc_r = shard_rows(full[i][0], full[i][1], n, k, rank, WORLD)
                y = iq2_matmul_sharded(comm, xs[i], qs_r, sc_r, n, k)
                errs[f"single m={m} {n}x{k}"] = rel(y, c.iq2_xxs_matmul(xs[i], full[i][0], full[i][1], n, k))
            # all of them in one call
            probs = [(xs[i], *shard_rows(full[i][0], full[i][1], n, k, rank, WORLD), n, k)
                     for i, (n, k) in enumerate(shapes)]
            ys = iq2_matmul_grouped_sharded(comm, probs)
            for i, (n, k) in enumerate(shapes):
                errs[f"grouped m={m} {n}x{k}"] = rel(ys[i], c.iq2_xxs_matmul(xs[i], full[i][0], full[i][1], n, k))
        torch.cuda.synchronize()
        comm.close()
        dist.destroy_process_group()
        q.put((rank, errs))
    except Exception as e:
        q.put((rank, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs two GPUs")
def test_sharded_matches_single_gpu():
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    try:
        res = [q.get(timeout=300) for _ in range(WORLD)]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, errs in res:
        assert isinstance(errs, dict), (rank, errs)
        for name, e in errs.items():
            assert e <= TOL, (rank, name, e)
