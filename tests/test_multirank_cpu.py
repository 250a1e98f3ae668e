"""Multi-rank host logic on CPU (gloo, world size 2): stream sharding, the all-gather of record
sizes that places each rank's records in the job-wide bitstream, and each rank finding its own
records again on decode.  Streams are coded by the oracle here, so no GPU is needed; the GPU run
(bench.py under torchrun) uses the same functions over NCCL."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O
from torch_ans_b200.sharding import (JobBitstream, gather_stream_lengths, rank_byte_range, record_offsets,
                                     record_offsets_from_lengths, shard_owner, shard_ragged, shard_streams)


def _free_port():
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _batch(variant, B, N):
    rng = np.random.default_rng(11)
    fp = 15 if variant == "rans32_16" else 16
    K, A = 4, 20
    pm = rng.integers(1, 512, (K, A)).astype(np.float32)
    cdfs = O.pmf_to_quantized_cdf(pm / pm.sum(1, keepdims=True), fp)
    sizes = np.full(K, A + 1, np.int32)
    idx = rng.integers(0, K, (B, N)).astype(np.int32)
    sym = np.clip(rng.integers(0, A, (B, N)), 0, A - 1).astype(np.int32)
    return fp, cdfs, sizes, idx, sym


def _rank_main(rank, ws, port, variant, B, N):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=60))
    try:
        from torch_ans_b200.utils import merge_bytes
        fp, cdfs, sizes, idx, sym = _batch(variant, B, N)
        lo, hi = shard_streams(B, ws, rank)
        st, err = O.push(variant, O.init_stream(variant, hi - lo), sym[lo:hi], idx[lo:hi], cdfs, sizes, None, fp,
                         False)
        assert err == 0
        mine = merge_bytes(O.stream_to_byte_strings(st), num_bytes_length=4)
        off, total, sizes_all = record_offsets(len(mine))
        assert sizes_all[rank] == len(mine) and total == sum(sizes_all)
        parts = [None] * ws
        dist.all_gather_object(parts, mine)  # test only: the product never moves payload between ranks
        job = bytearray(total)
        pos = 0
        for r in range(ws):
            job[pos:pos + len(parts[r])] = parts[r]
            if r == rank:
                assert pos == off
            pos += len(parts[r])
        full, _ = O.push(variant, O.init_stream(variant, B), sym, idx, cdfs, sizes, None, fp, False)
        assert bytes(job) == merge_bytes(O.stream_to_byte_strings(full), num_bytes_length=4)
        rows = [shard_streams(B, ws, r)[1] - shard_streams(B, ws, r)[0] for r in range(ws)]
        a, b = rank_byte_range(torch.frombuffer(bytearray(job), dtype=torch.uint8), rows, rank)
        assert bytes(job[a:b]) == mine
        # this rank decodes its own records back to its symbols
        from torch_ans_b200.utils import split_merged_bytes
        if hi > lo:
            seg = O.byte_strings_to_stream(split_merged_bytes(bytes(job[a:b]), num_bytes_length=4))
            dec, derr = O.pop(variant, seg, idx[lo:hi], cdfs, sizes, None, fp, False)
            assert derr == 0 and np.array_equal(dec, sym[lo:hi])
        else:
            assert a == b
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("variant", ["rans64", "rans32_16"])
@pytest.mark.parametrize("B", [7, 2, 1])
def test_two_rank_job_bitstream(variant, B):
    """World size 2 over gloo: each rank codes its shard, places its records with the size
    all-gather, and the job bitstream equals the single-process container of the whole batch; each
    rank then finds and decodes exactly its own records (including a rank with no streams)."""
    mp.spawn(_rank_main, args=(2, _free_port(), variant, B, 64), nprocs=2, join=True)


def test_shard_streams_partition():
    for B in [0, 1, 5, 64, 1000, 8192]:
        for ws in [1, 2, 3, 8]:
            ranges = [shard_streams(B, ws, r) for r in range(ws)]
            assert ranges[0][0] == 0 and ranges[-1][1] == B
            assert all(ranges[r][1] == ranges[r + 1][0] for r in range(ws - 1))
            sizes = [h - l for l, h in ranges]
            assert max(sizes) - min(sizes) <= 1
            for b in range(0, B, max(1, B // 50)):
                r = shard_owner(b, B, ws)
                assert ranges[r][0] <= b < ranges[r][1]


def test_shard_ragged_balances_symbols():
    rng = np.random.default_rng(3)
    lengths = np.clip(np.round(np.exp(rng.normal(np.log(300), 1.0, 500))), 10, 5000).astype(np.int64)
    rs = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]))
    for ws in [1, 2, 4, 8]:
        ranges = [shard_ragged(rs, ws, r) for r in range(ws)]
        assert ranges[0][0] == 0 and ranges[-1][1] == len(lengths)
        assert all(ranges[r][1] == ranges[r + 1][0] for r in range(ws - 1))
        loads = [int(lengths[l:h].sum()) for l, h in ranges]
        assert max(loads) - min(loads) <= 2 * int(lengths.max())


def _rank_job_file(rank, ws, port, variant, B, N, path):
    """One rank of the per-stream length protocol: code the shard, all-gather one length per
    stream, write this rank's records into the shared job file at the scanned offset, read its
    own byte range back and decode it."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=60))
    try:
        from torch_ans_b200.utils import merge_bytes, split_merged_bytes
        fp, cdfs, sizes, idx, sym = _batch(variant, B, N)
        shards = [shard_streams(B, ws, r) for r in range(ws)]
        lo, hi = shards[rank]
        st, err = O.push(variant, O.init_stream(variant, hi - lo), sym[lo:hi], idx[lo:hi], cdfs, sizes, None, fp,
                         False)
        assert err == 0
        lens = gather_stream_lengths(torch.from_numpy(st[:, 0].copy()), shards)
        assert lens.shape == (B,)
        offs, total = record_offsets_from_lengths(lens)
        start = int(offs[lo]) if hi > lo else (int(offs[lo]) if lo < B else total)
        mine = merge_bytes(O.stream_to_byte_strings(st), num_bytes_length=4)
        job = JobBitstream(path)
        if rank == 0:
            job.create(total)
        dist.barrier()
        job.open()
        if mine:
            if rank == 0:  # rank 0 writes through the file, rank 1 through its mapped range
                job.write(start, torch.frombuffer(bytearray(mine), dtype=torch.uint8))
            else:
                view = job.map_range(start, len(mine))
                view.copy_(torch.frombuffer(bytearray(mine), dtype=torch.uint8))
                del view
        dist.barrier()
        if rank == 0:
            whole = job.read(0, torch.empty(total, dtype=torch.uint8)).numpy().tobytes()
            full, _ = O.push(variant, O.init_stream(variant, B), sym, idx, cdfs, sizes, None, fp, False)
            assert whole == merge_bytes(O.stream_to_byte_strings(full), num_bytes_length=4)
        if hi > lo:
            data = job.read(start, torch.empty(len(mine), dtype=torch.uint8)).numpy().tobytes()
            seg = O.byte_strings_to_stream(split_merged_bytes(data, num_bytes_length=4))
            dec, derr = O.pop(variant, seg, idx[lo:hi], cdfs, sizes, None, fp, False)
            assert derr == 0 and np.array_equal(dec, sym[lo:hi])
        dist.barrier()
        job.close(unlink=rank == 0)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("B", [9, 1])
def test_two_rank_job_file_from_stream_lengths(tmp_path, B):
    """World size 2 over gloo: the per-stream length all-gather places every record; the job file
    the ranks write equals the single-process container of the whole batch (a rank with no
    streams included)."""
    mp.spawn(_rank_job_file, args=(2, _free_port(), "rans32", B, 40, str(tmp_path / "job.bin")), nprocs=2, join=True)


def test_record_offsets_from_lengths():
    offs, total = record_offsets_from_lengths(torch.tensor([3, 0, 5], dtype=torch.int64), prefix_bytes=4)
    assert offs.tolist() == [0, 7, 11] and total == 20
    offs, total = record_offsets_from_lengths(torch.zeros(0, dtype=torch.int64))
    assert offs.numel() == 0 and total == 0


def _rank_leaves(rank, ws, port, out_path):
    """Rank 1 leaves before the length all-gather (between steps, nothing in flight); rank 0 must
    get an error from the collective within the process group's timeout, not wait for ever."""
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=5))
    dist.barrier()
    if rank == 1:
        os._exit(0)  # leaves without taking part in the next collective
    t0 = time.monotonic()
    raised = None
    try:
        gather_stream_lengths(torch.tensor([7, 9], dtype=torch.int32), [(0, 2), (2, 4)])
    except Exception as e:  # noqa: BLE001  (gloo reports a closed peer or a timeout)
        raised = type(e).__name__
    with open(out_path, "w") as f:
        f.write(f"{raised}\n{time.monotonic() - t0:.3f}\n")
    os._exit(0)


def test_rank_leaving_before_gather_surfaces_an_error(tmp_path):
    out = tmp_path / "rank0.txt"
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_leaves, args=(r, 2, port, str(out))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert out.exists(), "rank 0 did not finish"
    name, secs = out.read_text().split()
    assert name != "None", "the all-gather returned although a rank had left"
    assert float(secs) < 30.0
