"""Column-sharded IQ2_XXS matmul over the GPUs of one node (one process per GPU).

Rank r of a world of g holds rows [r*N/g, (r+1)*N/g) of each projection's weights -- a contiguous
slice of the reference's split tensors (row n's blocks are contiguous, src/metal_src/iq2_matmul.metal:211-213),
so sharding is plain slicing -- computes its [m, N/g] slice with the single-GPU kernels, and one NCCL
all-gather over NVLink gives every rank the full [m, N] output (iq2_matmul_grouped_sharded in the C
ABI). The reference is single-device; this is the multi-GPU layout the benchmark specification asks for.

The communicator is the library's own NCCL communicator; torch.distributed (any backend) only
carries its 128-byte id from rank 0 to the others.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .iq2_matmul import _X_DTYPES, _bail, _check_common, _parse_x_shape, _stream_handle

QK = 256
QS_BYTES, SC_BYTES = 64, 2


def shard_rows(weight_bytes: torch.Tensor, weight_scales: torch.Tensor, out_dim: int, in_dim: int, rank: int,
               world: int):
    """Views of rank `rank`'s rows [rank*N/world, (rank+1)*N/world) of the split IQ2_XXS tensors."""
    if out_dim % world != 0:
        _bail(_lib.IQ2_ERR_INVALID_ARGUMENT, f"shard_rows: out_dim {out_dim} is not a multiple of the world size {world}")
    if not 0 <= rank < world:
        _bail(_lib.IQ2_ERR_INVALID_ARGUMENT, f"shard_rows: rank {rank} of world {world}")
    nb = (in_dim + QK - 1) // QK
    rows = out_dim // world
    qb, sb = rows * nb * QS_BYTES, rows * nb * SC_BYTES
    if weight_bytes.numel() < world * qb or weight_scales.numel() < world * sb:
        _bail(_lib.IQ2_ERR_TOO_SMALL, "shard_rows: weight tensors smaller than out_dim x in_dim")
    return weight_bytes[rank * qb:(rank + 1) * qb], weight_scales[rank * sb:(rank + 1) * sb]


class Iq2Comm:
    """The library's NCCL communicator over the ranks of a torch.distributed group (one GPU per
    rank, each rank's device current). Collective: every rank constructs it."""

    def __init__(self, group=None, timeout_ms: int = 120_000):
        """`timeout_ms` bounds every wait on the other ranks (joining, NCCL calls, barriers): a wait
        that runs out aborts the communicator and raises Iq2Error(IQ2_ERR_COMM)."""
        import torch.distributed as dist
        lib = _lib.load()
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.device = torch.device("cuda", torch.cuda.current_device())
        buf = (ctypes.c_uint8 * _lib.IQ2_COMM_ID_BYTES)()
        if self.rank == 0:
            _lib.check(lib.iq2_comm_unique_id(buf))
        obj = [bytes(buf)]
        dist.broadcast_object_list(obj, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        uid = (ctypes.c_uint8 * _lib.IQ2_COMM_ID_BYTES).from_buffer_copy(obj[0])
        handle = ctypes.c_void_p()
        _lib.check(lib.iq2_comm_init_with_timeout(uid, self.world, self.rank, int(timeout_ms), ctypes.byref(handle)))
        self._h = handle
        self._symm = None  # (base address, bytes) of the symmetric region
        self._symm_used = 0

    def alloc_symmetric(self, nbytes: int):
        """Collective: give this communicator a symmetric output region of `nbytes` (same on every
        rank). Outputs carved from it with symmetric_empty let the sharded decode (m <= 32)
        store straight into every rank's copy instead of going through an NCCL all-gather."""
        ptr = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(_lib.load().iq2_comm_symmetric_alloc(self._h, int(nbytes), ctypes.byref(ptr)))
        self._symm = (int(ptr.value), int(nbytes))
        self._symm_used = 0

    def symmetric_empty(self, *shape, dtype=torch.float32) -> torch.Tensor:
        """A tensor in the symmetric region (bump allocation, 256-byte aligned). Every rank must
        carve the same shapes in the same order, so that offsets agree."""
        if self._symm is None:
            _bail(_lib.IQ2_ERR_INVALID_ARGUMENT, "symmetric_empty: call alloc_symmetric first")
        shape = tuple(int(d) for d in (shape[0] if len(shape) == 1 and isinstance(shape[0], (tuple, list)) else shape))
        itemsize = torch.empty((), dtype=dtype).element_size()
        nbytes = itemsize
        for d in shape:
            nbytes *= d
        base, cap = self._symm
        off = (self._symm_used + 255) // 256 * 256
        if off + nbytes > cap:
            _bail(_lib.IQ2_ERR_TOO_SMALL, f"symmetric_empty: region of {cap} bytes is full")
        self._symm_used = off + nbytes
        return _device_view(base + off, shape, dtype, self.device, owner=self)

    @property
    def has_symmetric(self) -> bool:
        return self._symm is not None

    def check(self):
        """Raise if a fused exchange of this communicator failed, NCCL reported an asynchronous
        error or the communicator was aborted (synchronises the device)."""
        with torch.cuda.device(self.device):
            _lib.check(_lib.load().iq2_comm_check(self._h))

    def close(self):
        if self._h:
            _lib.check(_lib.load().iq2_comm_destroy(self._h))
            self._h = ctypes.c_void_p()
            self._symm = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class _CudaArray:
    """Exposes raw device memory to torch through the CUDA array interface (no copy)."""

    _TYPESTR = {torch.float32: "<f4", torch.float16: "<f2", torch.uint8: "|u1", torch.int32: "<i4"}

    def __init__(self, ptr, shape, dtype, owner):
        self.owner = owner  # keeps the communicator (and its region) alive
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": self._TYPESTR[dtype],
                                         "data": (ptr, False), "version": 3, "strides": None}


def _device_view(ptr, shape, dtype, device, owner):
    if dtype not in _CudaArray._TYPESTR:
        _bail(_lib.IQ2_ERR_DTYPE, f"symmetric_empty: unsupported dtype {dtype}")
    t = torch.as_tensor(_CudaArray(ptr, shape, dtype, owner), device=device)
    t._iq2_owner = owner
    return t


def _problems(op, comm: Iq2Comm, problems):
    arr = (_lib.Iq2MatmulProblem * len(problems))()
    outs, keep = [], []
    m = dtype = None
    for i, pr in enumerate(problems):
        x, wb, ws, out_dim, in_dim = pr[:5]
        out = pr[5] if len(pr) > 5 else None
        if out_dim % comm.world != 0:
            _bail(_lib.IQ2_ERR_INVALID_ARGUMENT,
                  f"{op}: problem {i}: out_dim {out_dim} is not a multiple of the world size {comm.world}")
        _check_common(op, wb, ws, out_dim // comm.world, in_dim, x)
        x2, mi, _ = _parse_x_shape(x, in_dim)
        x2 = x2.contiguous()
        if x2.dtype not in _X_DTYPES:
            _bail(_lib.IQ2_ERR_DTYPE, f"iq2_matmul unsupported x dtype: {x2.dtype}")
        if m is None:
            m, dtype = mi, x2.dtype
        elif mi != m or x2.dtype != dtype:
            _bail(_lib.IQ2_ERR_INVALID_ARGUMENT, f"{op}: every problem needs the same m and x dtype")
        if out is None:
            out = torch.empty((mi, out_dim), dtype=torch.float32, device=x.device)
        keep.append(x2)
        outs.append(out)
        arr[i] = _lib.Iq2MatmulProblem(x2.data_ptr(), wb.data_ptr(), wb.numel(), ws.data_ptr(), ws.numel(),
                                       out_dim, in_dim, out.data_ptr())
    return arr, outs, keep, m, dtype


def sharded_workspace_bytes(comm: Iq2Comm, problems) -> int:
    """Workspace iq2_matmul_grouped_sharded needs for these (x, shard_bytes, shard_scales, out_dim,
    in_dim[, out]) problems (out_dim: the full N)."""
    arr, _, _, m, dtype = _problems("iq2_matmul_grouped_sharded", comm, problems)
    return int(_lib.load().iq2_matmul_grouped_sharded_workspace_size(arr, len(problems), m, _X_DTYPES[dtype],
                                                                     comm.world))


def iq2_matmul_grouped_sharded(comm: Iq2Comm, problems, *, workspace=None):
    """Collective: every rank passes its row slices (see shard_rows) of the same projections;
    each rank gets the full [m, out_dim] outputs. `problems`: (x, shard_bytes, shard_scales,
    out_dim, in_dim[, out]) with out_dim the full N."""
    op = "iq2_matmul_grouped_sharded"
    if not problems:
        return []
    lib = _lib.load()
    arr, outs, keep, m, dtype = _problems(op, comm, problems)
    with torch.cuda.device(comm.device):
        need = int(lib.iq2_matmul_grouped_sharded_workspace_size(arr, len(problems), m, _X_DTYPES[dtype], comm.world))
        if workspace is None or workspace.numel() < need:
            workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=comm.device)
        rc = lib.iq2_matmul_grouped_sharded(comm._h, arr, len(problems), m, _X_DTYPES[dtype],
                                            ctypes.c_void_p(workspace.data_ptr()), workspace.numel(),
                                            _stream_handle(comm.device))
    _lib.check(rc)
    return outs


def iq2_matmul_sharded(comm: Iq2Comm, x, shard_bytes, shard_scales, out_dim: int, in_dim: int, *, out=None,
                       workspace=None) -> torch.Tensor:
    """One projection, column-sharded: x [m, in_dim] (or [in_dim]) on every rank, this rank's
    row slice of the weights, the full [m, out_dim] output on every rank."""
    _, m, squeeze = _parse_x_shape(x, in_dim)
    pr = (x, shard_bytes, shard_scales, out_dim, in_dim) + ((out,) if out is not None else ())
    y = iq2_matmul_grouped_sharded(comm, [pr], workspace=workspace)[0]
    return y.squeeze(0) if squeeze else y
