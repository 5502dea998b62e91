"""GPU parity of the column-sharded path (iq2_matmul_grouped_sharded: local slices, one NCCL
all-gather, one scatter kernel; or, with outputs in the communicator's symmetric region, the
decode GEMV storing into every rank's copy) against the single-GPU iq2_matmul on the full
weights. Needs two GPUs of one node; skipped otherwise. A rank that skips a call makes the other
rank's bounded waits run out: the status says so and no GPU is faulted."""
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
        for m in (1, 3, 300):  # (300: the tensor-core GEMM, paired CTAs, on each rank's slice)
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
        # m > 32 exchanges chunk by chunk while the next chunk computes: a projection whose gathered
        # output exceeds one chunk is split along m (4608 x 14336 f32 = 264 MB: chunks of 2304)
        m = 4608
        n, k = shapes[2]
        xb = synth.activations(m, k, seed=40, dtype=torch.bfloat16, device=dev)
        pb = [(xb, *shard_rows(full[2][0], full[2][1], n, k, rank, WORLD), n, k)]
        errs[f"grouped m={m} {n}x{k} (split along m)"] = rel(iq2_matmul_grouped_sharded(comm, pb)[0],
                                                            c.iq2_xxs_matmul(xb, full[2][0], full[2][1], n, k))
        # ... and under CUDA-graph capture (the side streams fork from and join the capturing stream)
        m = 300
        xs = [synth.activations(m, k, seed=50 + i, device=dev) for i, (n, k) in enumerate(shapes)]
        outs = [torch.empty(m, n, device=dev) for (n, k) in shapes]
        probs = [(xs[i], *shard_rows(full[i][0], full[i][1], n, k, rank, WORLD), n, k, outs[i])
                 for i, (n, k) in enumerate(shapes)]
        st = torch.cuda.Stream()
        with torch.cuda.stream(st):
            iq2_matmul_grouped_sharded(comm, probs)
        st.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            iq2_matmul_grouped_sharded(comm, probs)
        for i in range(len(outs)):
            outs[i].zero_()
        with torch.cuda.stream(st):
            g.replay()
        st.synchronize()
        for i, (n, k) in enumerate(shapes):
            errs[f"graph m={m} {n}x{k}"] = rel(outs[i], c.iq2_xxs_matmul(xs[i], full[i][0], full[i][1], n, k))
        del g
        torch.cuda.synchronize()
        comm.close()
        dist.destroy_process_group()
        q.put((rank, errs))
    except Exception as e:
        q.put((rank, repr(e)))


def _rank_fused(rank: int, port: int, q):
    try:
        import numpy as np
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=WORLD)
        import candelora_metal_kernels_b200 as c
        from candelora_metal_kernels_b200 import synth
        from candelora_metal_kernels_b200 import _lib
        from candelora_metal_kernels_b200.sharded import Iq2Comm, iq2_matmul_grouped_sharded, shard_rows
        comm = Iq2Comm()
        comm.alloc_symmetric(64 << 20)
        dev = torch.device("cuda", rank)

        def rel(a, b):
            a, b = a.double().cpu().numpy(), b.double().cpu().numpy()
            return float(np.linalg.norm(a - b) / np.linalg.norm(b))

        res = {}
        shapes = [(4096, 4096), (1024, 14336), (14336, 4096), (96, 512)]
        full = [tuple(t.to(dev) for t in synth.iq2xxs_weights(n, k, seed=i)) for i, (n, k) in enumerate(shapes)]
        slices = [shard_rows(full[i][0], full[i][1], n, k, rank, WORLD) for i, (n, k) in enumerate(shapes)]
        for m in (1, 3, 16):
            xs = [synth.activations(m, k, seed=30 + i, device=dev) for i, (n, k) in enumerate(shapes)]
            outs = [comm.symmetric_empty(m, n) for (n, k) in shapes]
            probs = [(xs[i], *slices[i], n, k, outs[i]) for i, (n, k) in enumerate(shapes)]
            ys = iq2_matmul_grouped_sharded(comm, probs)  # fused exchange
            ref_nccl = iq2_matmul_grouped_sharded(comm, [p[:5] for p in probs])  # NCCL all-gather
            for i, (n, k) in enumerate(shapes):
                res[f"m={m} {n}x{k} vs single"] = rel(ys[i], c.iq2_xxs_matmul(xs[i], full[i][0], full[i][1], n, k))
                res[f"m={m} {n}x{k} same as nccl"] = 0.0 if torch.equal(ys[i], ref_nccl[i]) else 1.0
            # one projection per call, then a CUDA graph of three calls replayed with new x
            y1 = iq2_matmul_grouped_sharded(comm, [probs[2]])[0]
            res[f"m={m} single call"] = rel(y1, c.iq2_xxs_matmul(xs[2], full[2][0], full[2][1], *shapes[2]))
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                iq2_matmul_grouped_sharded(comm, probs[:3])
            s.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for _ in range(3):
                    iq2_matmul_grouped_sharded(comm, probs[:3])
            for rep in range(3):
                for i, (n, k) in enumerate(shapes[:3]):
                    xs[i].copy_(synth.activations(m, k, seed=100 * rep + i, device=dev))
                with torch.cuda.stream(s):
                    g.replay()
                s.synchronize()
                for i, (n, k) in enumerate(shapes[:3]):
                    res[f"m={m} graph replay {rep} {n}x{k}"] = rel(
                        outs[i], c.iq2_xxs_matmul(xs[i], full[i][0], full[i][1], n, k))
            del g
        torch.cuda.synchronize()
        comm.check()
        # failure detection: rank 1 skips one call, so rank 0's entry wait runs out (bounded)
        x = synth.activations(1, 4096, seed=5, device=dev)
        out = comm.symmetric_empty(1, 4096)
        if rank == 0:
            iq2_matmul_grouped_sharded(comm, [(x, *slices[0], 4096, 4096, out)])
            torch.cuda.synchronize()
            try:
                comm.check()
                res["timeout reported"] = 1.0
            except c.Iq2Error as e:
                res["timeout reported"] = 0.0 if e.code == _lib.IQ2_ERR_COMM else 1.0
        dist.barrier()
        # one more call on both ranks: their call numbers now differ by one, so neither rank may
        # return the other's stale columns as a success; each rank's own columns are still right
        out2 = comm.symmetric_empty(1, 4096)
        iq2_matmul_grouped_sharded(comm, [(x, *slices[0], 4096, 4096, out2)])
        torch.cuda.synchronize()
        try:
            comm.check()
            res["error reported after the mismatched call"] = 1.0
        except c.Iq2Error as e:
            res["error reported after the mismatched call"] = 0.0 if e.code == _lib.IQ2_ERR_COMM else 1.0
        own = slice(rank * 2048, (rank + 1) * 2048)
        res["own columns after the error"] = rel(out2[:, own], c.iq2_xxs_matmul(x, *full[0], 4096, 4096)[:, own])
        dist.barrier()
        comm.close()
        dist.destroy_process_group()
        q.put((rank, res))
    except Exception as e:
        import traceback
        q.put((rank, repr(e) + traceback.format_exc()))


def _lonely_init(q):
    # rank 0 of a world of two, whose partner never calls iq2_comm_init
    try:
        import ctypes
        import time
        torch.cuda.set_device(0)
        from candelora_metal_kernels_b200 import _lib
        lib = _lib.load()
        uid = (ctypes.c_uint8 * _lib.IQ2_COMM_ID_BYTES)()
        _lib.check(lib.iq2_comm_unique_id(uid))
        h = ctypes.c_void_p()
        t0 = time.monotonic()
        rc = lib.iq2_comm_init_with_timeout(uid, 2, 0, 3000, ctypes.byref(h))
        q.put((rc, time.monotonic() - t0, lib.iq2_last_error().decode(), h.value))
    except Exception as e:
        q.put(repr(e))


def test_comm_init_gives_up_when_a_rank_never_joins():
    """A non-blocking communicator: the rank that waits for a partner that never comes gets
    IQ2_ERR_COMM after its timeout (3 s here) instead of hanging; no GPU kernel is involved."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_init, args=(q,))
    p.start()
    try:
        res = q.get(timeout=240)
    finally:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    from candelora_metal_kernels_b200 import _lib
    assert isinstance(res, tuple), res
    rc, dt, msg, handle = res
    assert rc == _lib.IQ2_ERR_COMM, (rc, msg)
    assert "not every rank joined within 3000 ms" in msg
    assert 2.5 <= dt < 120, dt
    assert handle is None


def _spawn(target):
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    try:
        return [q.get(timeout=300) for _ in range(WORLD)]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs two GPUs")
def test_fused_exchange_matches_single_gpu_and_nccl():
    for rank, res in _spawn(_rank_fused):
        assert isinstance(res, dict), (rank, res)
        for name, e in res.items():
            assert e <= TOL, (rank, name, e)
        if rank == 0:
            assert "timeout reported" in res


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
