"""Column sharding of a quantized projection across ranks, one process per GPU.

A large-N projection (the vocab head, an FFN up projection) splits its N weight rows -- the output
columns -- into one contiguous block per rank. Every rank runs the product for its block on its own
GPU, then one all-gather assembles the f32 outputs. This path has no counterpart in the reference
(which runs on one device); it is the multi-GPU layout of the same product.

Layout of the gathered result: rank-major, ``gathered[r]`` is rank r's ``[m, n_r]`` block (the
all-gather writes each rank's contiguous output once, with no transposing copy).
``logical_columns`` gives the ``[m, world, n_r]`` view of it whose flattened last two dimensions
are the output columns in order, without copying.
"""
from __future__ import annotations

from .formats import block

# Shard boundaries are multiples of this many weight rows: the product's weight tiles are 128 rows,
# and 64 keeps every shard a legal matrix shape (n % 64 == 0) for all block types.
SHARD_ALIGN = 64


def column_shard(n_total: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [lo, hi) of the weight matrix (output columns) owned by `rank`.

    Shards are as equal as SHARD_ALIGN allows; the first ranks take one extra unit when the
    units do not divide evenly. Raises ValueError if n_total is not a multiple of SHARD_ALIGN or a
    rank would get no rows."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world size {world}")
    if n_total % SHARD_ALIGN:
        raise ValueError(f"n={n_total} is not a multiple of {SHARD_ALIGN}")
    units = n_total // SHARD_ALIGN
    if units < world:
        raise ValueError(f"n={n_total} has fewer than {world} shards of {SHARD_ALIGN} rows")
    base, extra = divmod(units, world)
    lo = rank * base + min(rank, extra)
    hi = lo + base + (1 if rank < extra else 0)
    return lo * SHARD_ALIGN, hi * SHARD_ALIGN


def shard_rows(raw: bytes | memoryview, kind: int, n_total: int, k: int, lo: int, hi: int):
    """The GGUF bytes of weight rows [lo, hi) of an [n_total, k] matrix of block type `kind`
    (GGUF stores rows contiguously, each k / block_elems blocks long)."""
    bk = block(kind)
    if bk is None:
        raise ValueError(f"unknown block type {kind}")
    elems, nbytes = bk
    if k % elems:
        raise ValueError(f"k={k} is not a multiple of the {elems}-element block")
    row_bytes = k // elems * nbytes
    if len(raw) != n_total * row_bytes:
        raise ValueError(f"{len(raw)} bytes for [{n_total}, {k}] (expected {n_total * row_bytes})")
    return memoryview(raw)[lo * row_bytes: hi * row_bytes]


def gather_shards(local_out, out=None, group=None, async_op: bool = False):
    """All-gathers every rank's ``[m, n_r]`` f32 output (all ranks the same n_r) into a rank-major
    ``[world, m, n_r]`` tensor (allocated if `out` is None). Every rank must call it in the same
    order. Returns (gathered, work) where work is the async handle when async_op is set."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    m, n_r = local_out.shape
    if out is None:
        out = torch.empty((world, m, n_r), dtype=local_out.dtype, device=local_out.device)
    if tuple(out.shape) != (world, m, n_r) or not out.is_contiguous() or not local_out.is_contiguous():
        raise ValueError("gather_shards needs contiguous [m, n_r] input and [world, m, n_r] output")
    # The concatenated-along-dim-0 form is accepted by every backend (gloo and NCCL).
    work = dist.all_gather_into_tensor(out.view(world * m, n_r), local_out, group=group, async_op=async_op)
    return out, work


def logical_columns(gathered):
    """``[m, world, n_r]`` view of a rank-major gathered output: element [i, r, j] is output
    column r * n_r + j of row i."""
    return gathered.permute(1, 0, 2)


class PeerGather:
    """Buffers for jk_sharded_matmul_allgather on one rank: `buffers` rank-major gathered outputs
    [world, m, n_r] f32 and one array of `world` u32 counter words, allocated with jk_ipc_alloc on
    this rank's GPU and mapped into every other rank (jk_ipc_open) through one exchange of the
    64-byte IPC handles over the process group. The copy engines of each rank write its shard into
    the peers' buffers; nothing here launches a collective kernel. Every rank must create it and
    call `run` / `wait` in the same order."""

    def __init__(self, gpu, m: int, n_r: int, buffers: int = 2, group=None):
        import ctypes
        import torch.distributed as dist
        from ._lib import check, load
        self.gpu, self.m, self.n_r, self.buffers = gpu, int(m), int(n_r), int(buffers)
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        lib = load()
        dev = gpu.device
        self._own, handles = [], []
        sizes = [self.world * self.m * self.n_r * 4] * self.buffers + [max(self.world * 4, 256)]
        for nbytes in sizes:
            ptr = ctypes.c_void_p()
            h = (ctypes.c_uint8 * 64)()
            check(lib.jk_ipc_alloc(dev, nbytes, ctypes.byref(ptr), h))
            self._own.append(ptr.value)
            handles.append(bytes(h))
        everyone = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(everyone, handles, group=group)
        else:
            everyone = [handles]
        self._opened = []
        # tables[i]: pointer arrays [world] of buffer i (the last entry: the flag words) per rank
        self.tables = []
        for i in range(len(sizes)):
            arr = (ctypes.c_void_p * self.world)()
            for p in range(self.world):
                if p == self.rank:
                    arr[p] = self._own[i]
                    continue
                ptr = ctypes.c_void_p()
                h = (ctypes.c_uint8 * 64).from_buffer_copy(everyone[p][i])
                check(lib.jk_ipc_open(dev, h, ctypes.byref(ptr)))
                self._opened.append(ptr.value)
                arr[p] = ptr.value
            self.tables.append(arr)
        self.flags = self.tables[-1]

    def output(self, i: int):
        """Gathered output buffer i as a torch tensor [world, m, n_r] (no copy)."""
        n = self.world * self.m * self.n_r
        return _tensor_from_ptr(self.tables[i][self.rank], n, self.gpu.device).view(self.world, self.m, self.n_r)

    def run(self, w_shard, x, i: int = 0, wait: bool = True, chunks: int = 4, scratch=None, stream=None):
        """One jk_sharded_matmul_allgather call into gathered buffer i."""
        import ctypes
        import torch
        from ._lib import check, load
        st = stream if stream is not None else torch.cuda.current_stream().cuda_stream
        check(load().jk_sharded_matmul_allgather(
            w_shard.handle, ctypes.c_void_p(x.data_ptr()), _DT[x.dtype], x.numel(), self.m, self.rank, self.world,
            ctypes.cast(self.tables[i], ctypes.c_void_p), ctypes.cast(self.flags, ctypes.c_void_p), int(chunks),
            1 if wait else 0, scratch.handle if scratch is not None else None, ctypes.c_void_p(st)))

    def wait(self, stream=None):
        """jk_allgather_wait: ends the exchange of every product made with wait=False since the
        last wait (this rank's copies are signalled to the peers, the peers' shards have landed)."""
        import ctypes
        import torch
        from ._lib import check, load
        st = stream if stream is not None else torch.cuda.current_stream().cuda_stream
        check(load().jk_allgather_wait(self.gpu.device, ctypes.cast(self.flags, ctypes.c_void_p), self.world,
                                       self.rank, ctypes.c_void_p(st)))

    def close(self):
        from ._lib import load
        lib = load()
        for p in getattr(self, "_opened", []):
            lib.jk_ipc_close(self.gpu.device, p)
        for p in getattr(self, "_own", []):
            lib.jk_ipc_free(self.gpu.device, p)
        self._opened, self._own = [], []


def _tensor_from_ptr(ptr: int, numel: int, device: int):
    """A float32 CUDA tensor viewing `numel` values at device pointer `ptr` (memory owned elsewhere)."""
    import torch

    class _Cai:
        def __init__(self):
            self.__cuda_array_interface__ = {"shape": (numel,), "typestr": "<f4", "data": (ptr, False),
                                             "version": 3, "strides": None}
    with torch.cuda.device(device):
        return torch.as_tensor(_Cai(), device=f"cuda:{device}")


def _dtypes():
    import torch
    return {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


class _DtMap(dict):
    def __missing__(self, key):
        self.update(_dtypes())
        return dict.__getitem__(self, key)


_DT = _DtMap()
