"""Row sharding across ranks (one process per GPU, torch.distributed).

The hot path partitions cleanly: elementwise ranges, matmul output rows and
sweep a-rows are independent, so a rank computes its block with no exchange
and only results meet: event counts are summed (all-reduce), row blocks are
gathered (all-gather of equal, padded blocks), and device times take the max
over ranks.  Every rank calls these in the same order.  The functions take
the process group's module (``torch.distributed``) so the same code runs
over NCCL on GPUs and over gloo on CPU tensors.
"""
from __future__ import annotations


def _nccl_type(dt) -> bool:
    import torch
    return dt in (torch.uint8, torch.int8, torch.int32, torch.int64, torch.float16, torch.bfloat16, torch.float32,
                  torch.float64)


def row_cuts(n: int, world: int, start: int = 0) -> list[int]:
    """world + 1 cut points splitting [start, start + n) into near-equal blocks."""
    return [start + (n * r) // world for r in range(world + 1)]


def block(n: int, world: int, rank: int, start: int = 0) -> tuple[int, int]:
    c = row_cuts(n, world, start)
    return c[rank], c[rank + 1]


def sum_counts(counts, dist=None, world: int = 1):
    """Event counts summed over ranks, in place."""
    if dist is not None and world > 1:
        dist.all_reduce(counts)
    return counts


def max_over_ranks(value: float, device, dist=None, world: int = 1) -> float:
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    if dist is not None and world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_rows(local, cuts, dist=None, world: int = 1):
    """Concatenate every rank's row block (dim 0; blocks sized by ``cuts``),
    on every rank."""
    import torch
    if dist is None or world == 1:
        return local
    sizes = [cuts[r + 1] - cuts[r] for r in range(world)]
    if len(set(sizes)) == 1 and local.is_cuda and dist.get_backend() == "nccl":
        # equal blocks: NCCL writes every rank's block straight into place
        full = torch.empty((sizes[0] * world,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
        src, dst = local.contiguous().reshape(-1), full.reshape(-1)
        if not _nccl_type(local.dtype):              # NCCL has no int16: send the bytes
            src, dst = src.view(torch.uint8), dst.view(torch.uint8)
        dist.all_gather_into_tensor(dst, src)
        return full
    rows_max = max(sizes)
    pad = torch.zeros((rows_max,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[:local.shape[0]] = local
    wire = pad
    if not _nccl_type(pad.dtype):                    # NCCL has no int16: send the bytes
        wire = pad.reshape(rows_max, -1).view(torch.uint8)
    parts = [torch.empty_like(wire) for _ in range(world)]
    dist.all_gather(parts, wire)
    if wire is not pad:
        parts = [p.view(pad.dtype).reshape(pad.shape) for p in parts]
    return torch.cat([parts[r][:cuts[r + 1] - cuts[r]] for r in range(world)])


def cyclic_pieces(n: int, world: int, parts: int, rank: int) -> list[tuple[int, int]]:
    """Rows of ``rank`` when n rows go to the ranks block-cyclically in
    ``parts`` pieces of P = n / (world parts) rows: piece j is global rows
    [(j world + rank) P, (j world + rank + 1) P).  The pieces j of all ranks
    then form rows [j world P, (j + 1) world P) in rank order, so gathering
    piece j needs no reordering."""
    if n % (world * parts):
        raise ValueError(f"{n} rows do not split into {world} x {parts} equal pieces")
    P = n // (world * parts)
    return [((j * world + rank) * P, (j * world + rank + 1) * P) for j in range(parts)]


def gather_piece(full, piece, j: int, dist=None, world: int = 1, async_op: bool = False):
    """All-gather every rank's piece j (P rows, block-cyclic order) into rows
    [j world P, (j + 1) world P) of ``full`` (contiguous, every rank).
    Returns the collective's work handle when ``async_op`` (NCCL runs it on
    its own stream beside later kernels), else None."""
    import torch
    P = piece.shape[0]
    dst = full[j * world * P:(j + 1) * world * P]
    if dist is None or world == 1:
        dst.copy_(piece)
        return None
    src = piece.contiguous()
    if not _nccl_type(piece.dtype):                  # NCCL has no int16: send the bytes
        dst, src = dst.view(torch.uint8), src.view(torch.uint8)
    return dist.all_gather_into_tensor(dst, src, async_op=async_op)


def sharded_matmul(compute, A, B, rank: int, world: int, dist=None):
    """Row-sharded matmul: this rank computes rows [lo, hi) of A @ B with
    ``compute(A_block, B) -> (codes, flags, counts)`` (B replicated), then
    the codes and flags are gathered and the counts summed, so every rank
    ends with the whole result."""
    M = A.shape[-2]
    cuts = row_cuts(M, world)
    lo, hi = cuts[rank], cuts[rank + 1]
    codes, flags, counts = compute(A[..., lo:hi, :], B)
    if A.dim() > 2:       # batched: rows are the second-to-last dim, gather along it
        codes = gather_rows(codes.movedim(-2, 0).contiguous(), cuts, dist, world).movedim(0, -2)
        flags = gather_rows(flags.movedim(-2, 0).contiguous(), cuts, dist, world).movedim(0, -2)
    else:
        codes = gather_rows(codes, cuts, dist, world)
        flags = gather_rows(flags, cuts, dist, world)
    return codes, flags, sum_counts(counts, dist, world)
