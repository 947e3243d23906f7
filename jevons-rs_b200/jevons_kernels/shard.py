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
