"""Multi-GPU layout of the coding path: one process per GPU, streams sharded across ranks.

Streams are independent (each is one serial rANS chain), so a batch shards by stream with no
exchange on the data path: rank r codes a contiguous range of streams on its own GPU.  The only
collective is the placement of each rank's records in the job-wide concatenated bitstream (the
container of merge_bytes, torch_ans/utils.py:47-72): ranks all-gather their record byte counts,
and an exclusive scan gives each rank the offset at which its records start.  On decode every
rank finds its own byte range by walking the record prefixes (split_merged_bytes semantics,
torch_ans/utils.py:74-101) and loads only its records.  No payload crosses GPUs.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch
import torch.distributed as dist


def shard_streams(num_streams: int, world_size: int, rank: int) -> Tuple[int, int]:
    """Contiguous stream range [lo, hi) of `rank`: sizes differ by at most one, lower ranks first."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError("bad world_size / rank")
    base, extra = divmod(int(num_streams), world_size)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shard_ragged(row_starts: torch.Tensor, world_size: int, rank: int) -> Tuple[int, int]:
    """Contiguous stream range [lo, hi) of `rank` for ragged streams, balanced by symbol count:
    stream b goes to the rank whose share [r T / W, (r + 1) T / W) holds the stream's midpoint."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError("bad world_size / rank")
    rs = row_starts.to(torch.int64).cpu()
    B = rs.numel() - 1
    if B <= 0:
        return 0, 0
    total = int(rs[-1] - rs[0])
    mid2 = (rs[:-1] - rs[0]) + (rs[1:] - rs[0])  # twice the midpoint of each stream
    owner = torch.clamp((mid2 * world_size) // max(2 * total, 1), 0, world_size - 1) if total > 0 else \
        torch.tensor([shard_owner(b, B, world_size) for b in range(B)], dtype=torch.int64)
    # owners are non-decreasing, so each rank's streams form one contiguous range
    lo = int(torch.searchsorted(owner, torch.tensor(rank), right=False))
    hi = int(torch.searchsorted(owner, torch.tensor(rank), right=True))
    return lo, hi


def shard_owner(b: int, num_streams: int, world_size: int) -> int:
    """Rank that shard_streams assigns stream b to."""
    base, extra = divmod(num_streams, world_size)
    cut = extra * (base + 1)
    return b // (base + 1) if b < cut else extra + (b - cut) // max(base, 1)


def record_offsets(local_bytes: int, group: Optional[dist.ProcessGroup] = None,
                   device: Optional[torch.device] = None) -> Tuple[int, int, List[int]]:
    """All-gather of every rank's record byte count; returns (this rank's byte offset in the
    job-wide bitstream, the job's total bytes, the per-rank sizes).  `device` is where the
    collective's tensors live (a CUDA device for NCCL, the CPU for gloo)."""
    ws = dist.get_world_size(group)
    me = dist.get_rank(group)
    dev = device if device is not None else torch.device("cpu")
    n = torch.tensor([int(local_bytes)], dtype=torch.int64, device=dev)
    sizes = [torch.zeros_like(n) for _ in range(ws)]
    dist.all_gather(sizes, n, group=group)
    sz = [int(s.item()) for s in sizes]
    return sum(sz[:me]), sum(sz), sz


def rank_byte_range(data: torch.Tensor, rows_per_rank: List[int], rank: int, num_bytes_length: int = 4
                    ) -> Tuple[int, int]:
    """Byte range [start, end) of `rank`'s records in the job-wide bitstream `data` (uint8 CPU
    tensor), given how many stream records each rank wrote, in rank order."""
    from . import _C
    total_rows = int(sum(rows_per_rank))
    r0 = int(sum(rows_per_rank[:rank]))
    r1 = r0 + int(rows_per_rank[rank])
    if r1 == r0:
        offs, lens = _C.parse_merged(data, num_bytes_length, max(r0, 1))
        at = int(offs[r0 - 1] + lens[r0 - 1]) if r0 > 0 else 0
        return at, at
    offs, lens = _C.parse_merged(data, num_bytes_length, total_rows)
    return int(offs[r0]) - num_bytes_length, int(offs[r1 - 1] + lens[r1 - 1])
