"""Multi-GPU layout of the coding path: one process per GPU, streams sharded across ranks.

Streams are independent (each is one serial rANS chain), so a batch shards by stream with no
exchange on the data path: rank r codes the contiguous stream range ``shard_streams(B, W, r)`` on
its own GPU.  The one collective is the placement of every stream's record in the job-wide
concatenated bitstream (the container of merge_bytes, torch_ans/utils.py:47-72: per stream a
little-endian length prefix, then the payload, in stream order):

1. each rank all-gathers the int32 payload byte length of every stream of its shard
   (``gather_stream_lengths``; over NCCL / NVLink on GPUs, gloo on CPUs);
2. every rank exclusive-scans ``prefix + length`` over the job's streams
   (``record_offsets_from_lengths``) and so knows where its first record starts;
3. each rank writes its records, assembled on its own GPU, at that offset into the job bitstream
   (``JobBitstream``, a file every rank of the host maps; no payload crosses GPUs).

On decode a rank takes its byte range straight from the gathered lengths (``rank_byte_range``
parses the prefixes instead, for a bitstream read back without them).
"""
from __future__ import annotations

import os
import tempfile
from typing import List, Optional, Sequence, Tuple

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


def gather_stream_lengths(local_lengths: torch.Tensor, shards: Sequence[Tuple[int, int]],
                          group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
    """All-gather of the payload byte length of every stream of the job.

    ``local_lengths``: int32 tensor with one entry per stream of this rank's shard (column 0 of
    its stream rows), on the collective's device (a CUDA device for NCCL, the CPU for gloo).
    ``shards``: every rank's [lo, hi) stream range, in rank order.  Returns the lengths of all
    streams in stream order (int64, CPU).  Shards of different sizes are padded to the largest."""
    ws = dist.get_world_size(group)
    if len(shards) != ws:
        raise ValueError("one shard range per rank expected")
    me = dist.get_rank(group)
    width = max(1, max(hi - lo for lo, hi in shards))
    if local_lengths.numel() != shards[me][1] - shards[me][0]:
        raise ValueError("local_lengths does not match this rank's shard")
    buf = torch.zeros(width, dtype=torch.int32, device=local_lengths.device)
    buf[: local_lengths.numel()] = local_lengths.to(torch.int32)
    parts = [torch.empty_like(buf) for _ in range(ws)]
    dist.all_gather(parts, buf, group=group)
    host = torch.stack(parts).cpu()
    return torch.cat([host[r, : hi - lo] for r, (lo, hi) in enumerate(shards)]).to(torch.int64)


def record_offsets_from_lengths(lengths: torch.Tensor, prefix_bytes: int = 4) -> Tuple[torch.Tensor, int]:
    """Byte offset of every stream's record in the job bitstream (exclusive scan of prefix +
    length, the layout merge_bytes writes) and the bitstream's total size."""
    rec = lengths.to(torch.int64) + int(prefix_bytes)
    offs = torch.zeros_like(rec)
    if rec.numel() > 1:
        offs[1:] = torch.cumsum(rec[:-1], 0)
    total = int(offs[-1] + rec[-1]) if rec.numel() else 0
    return offs, total


def record_offsets(local_bytes: int, group: Optional[dist.ProcessGroup] = None,
                   device: Optional[torch.device] = None) -> Tuple[int, int, List[int]]:
    """All-gather of every rank's total record bytes; returns (this rank's byte offset in the
    job-wide bitstream, the job's total bytes, the per-rank sizes).  For callers that hold their
    shard's container already; the per-stream form is ``gather_stream_lengths``."""
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
    tensor), given how many stream records each rank wrote, in rank order, by walking the length
    prefixes (split_merged_bytes semantics, torch_ans/utils.py:74-101)."""
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


class JobBitstream:
    """The job-wide concatenated bitstream as one host file that every rank of the node opens.

    Rank 0 creates it with the job's total size (known to every rank after the length all-gather).
    Each rank then either maps its own byte range (``map_range``: a uint8 tensor over the shared
    pages, page-locked for the GPU when the driver accepts the registration, so device copies go
    straight in and out of the job bitstream) or writes and reads it with ``write`` / ``read``.
    ``path`` must be the same on every rank (broadcast it).  The file lives in /dev/shm when that
    has room (host memory), else in the temporary directory."""

    def __init__(self, path: str):
        self.path = path
        self.fd = None
        self._maps = []

    @staticmethod
    def default_path(tag: str, size_hint: int) -> str:
        for d in ("/dev/shm", tempfile.gettempdir()):
            try:
                st = os.statvfs(d)
                if st.f_bavail * st.f_frsize > 2 * size_hint + (256 << 20):
                    return os.path.join(d, f"tans_job_{tag}.bin")
            except OSError:
                continue
        return os.path.join(tempfile.gettempdir(), f"tans_job_{tag}.bin")

    def create(self, total: int) -> None:
        """Create (or resize) the file to `total` bytes; call on one rank, then barrier."""
        with open(self.path, "wb") as f:
            f.truncate(int(total))

    def open(self) -> "JobBitstream":
        if self.fd is None:
            self.fd = os.open(self.path, os.O_RDWR)
        return self

    def write(self, offset: int, data: torch.Tensor) -> None:
        """Write a contiguous uint8 CPU tensor at `offset`."""
        mv = memoryview(data.numpy()).cast("B")
        done = 0
        while done < len(mv):
            done += os.pwrite(self.fd, mv[done:], int(offset) + done)

    def read(self, offset: int, out: torch.Tensor) -> torch.Tensor:
        """Fill a contiguous uint8 CPU tensor from `offset`."""
        mv = memoryview(out.numpy()).cast("B")
        done = 0
        while done < len(mv):
            n = os.preadv(self.fd, [mv[done:]], int(offset) + done)
            if n <= 0:
                raise IOError("job bitstream shorter than expected")
            done += n
        return out

    def map_range(self, offset: int, length: int) -> torch.Tensor:
        """A uint8 tensor over bytes [offset, offset + length) of the file, shared with every rank
        that maps them.  The pages are registered with the CUDA driver (page-locked) when possible,
        so copies between the tensor and a GPU run asynchronously at full host-link speed;
        ``registered`` tells whether that succeeded."""
        import mmap
        page = mmap.ALLOCATIONGRANULARITY
        lo = (int(offset) // page) * page
        n = int(offset) + int(length) - lo
        mm = mmap.mmap(self.fd, max(n, 1), mmap.MAP_SHARED, mmap.PROT_READ | mmap.PROT_WRITE, offset=lo)
        whole = torch.frombuffer(mm, dtype=torch.uint8)
        registered = False
        if torch.cuda.is_available() and n > 0:
            rc = torch.cuda.cudart().cudaHostRegister(whole.data_ptr(), n, 0)
            registered = int(rc) == 0
        self._maps.append((mm, whole, registered))
        self.registered = registered
        return whole[int(offset) - lo: int(offset) - lo + int(length)]

    def close(self, unlink: bool = False) -> None:
        while self._maps:
            mm, whole, registered = self._maps.pop()
            if registered:
                torch.cuda.cudart().cudaHostUnregister(whole.data_ptr())
            del whole
            try:
                mm.close()
            except BufferError:  # a caller still holds a view; the mapping closes with the last one
                pass
        if self.fd is not None:
            os.close(self.fd)
            self.fd = None
        if unlink:
            try:
                os.unlink(self.path)
            except FileNotFoundError:
                pass
