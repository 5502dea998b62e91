"""Column sharding on the host (no GPU): two gloo ranks on CPU. Each takes its row slice with
shard_rows, computes its output slice with the CPU oracle, and the all-gathered slices must equal
the unsharded oracle output bit for bit (rows are independent). Also pins shard_rows against the
synthetic generator's own row-slice mode."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

N, K = 96, 640  # K not a multiple of 256: the partial last block
WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, port: int, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=WORLD)
        from oracle.oracle import Oracle
        from candelora_metal_kernels_b200 import synth
        from candelora_metal_kernels_b200.sharded import shard_rows
        qs, sc = synth.iq2xxs_weights(N, K, seed=5)
        qs_r, sc_r = shard_rows(qs, sc, N, K, rank, WORLD)
        rows = N // WORLD
        q2, s2 = synth.iq2xxs_weights(N, K, seed=5, row_begin=rank * rows, row_end=(rank + 1) * rows)
        same_slice = torch.equal(qs_r, q2) and torch.equal(sc_r, s2)
        x = synth.activations(3, K, seed=9)
        o = Oracle()
        part = torch.from_numpy(np.ascontiguousarray(o.matmul(x.numpy(), qs_r.numpy(), sc_r.numpy(), rows, K)))
        parts = [torch.empty_like(part) for _ in range(WORLD)]
        dist.all_gather(parts, part)
        full = torch.cat(parts, dim=1)  # rank-major column slices -> [m, N]
        want = torch.from_numpy(o.matmul(x.numpy(), qs.numpy(), sc.numpy(), N, K))
        q.put((rank, same_slice, bool(torch.equal(full, want))))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), False))


def test_sharded_slices_reassemble_the_unsharded_output(oracle):
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    try:
        res = sorted(q.get(timeout=180) for _ in range(WORLD))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for rank, same_slice, equal in res:
        assert same_slice is True, (rank, same_slice)
        assert equal, rank


def test_shard_rows_checks():
    from candelora_metal_kernels_b200 import Iq2Error, synth
    from candelora_metal_kernels_b200.sharded import shard_rows
    qs, sc = synth.iq2xxs_weights(6, 256, seed=1)
    with pytest.raises(Iq2Error, match="not a multiple of the world size"):
        shard_rows(qs, sc, 6, 256, 0, 4)
    with pytest.raises(Iq2Error, match="rank 2 of world 2"):
        shard_rows(qs, sc, 6, 256, 2, 2)
    a, b = shard_rows(qs, sc, 6, 256, 1, 3)
    assert a.numel() == 2 * 64 and b.numel() == 2 * 2
    assert torch.equal(a, qs[128:256]) and torch.equal(b, sc[4:8])
