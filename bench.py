"""Benchmark of the rANS coding path: encode + decode Gsymbols/s on 1..8 B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload mixture_invcdf] [--impl ours|reference]
                    [--scaling strong|weak]

A step is one pass of the coding path over one batch: push (encode) of every stream from a fresh
stream tensor, then pop (decode) of every stream, through the `_C` op surface, with inputs
resident in HBM.  ``value`` = symbols of the whole job / max-over-ranks device time of K steps
(each symbol is encoded once and decoded once per step), in Gsymbols/s.  The default workload is
the 2^31-symbol rans64 push + inverse-cdf pop configuration: 8,192 streams x 262,144 symbols over
256 tables of 1,024 symbols.

Scaling (``--scaling``):
  * ``strong`` (default): the configuration's batch is the job; rank r of N codes the contiguous
    stream range ``shard_streams(8192, N, r)`` (1,024 streams per GPU at N = 8).  With N > 1 the
    line also carries ``weak_scaling``: every rank coding a whole batch, timed the same way.
  * ``weak``: every rank codes a whole batch (N batches per job).

Also reported:
  * ``e2e``: the same round trip through the public host API (``HostStreamCoder``) from pinned
    host memory: H2D of symbols and indexes overlapped with the push; NCCL all-gather of every
    stream's byte length (N > 1); device assembly of this rank's records and D2H of them into the
    job-wide concatenated bitstream at the offsets the lengths give (a host file shared by the
    ranks, N > 1); then this rank's byte range back in, device parse, pop overlapped with the D2H
    of the decoded symbols.  Host wall clock, max over ranks.  ``e2e.host_link`` gives the time
    of plain pinned copies of the same bytes on all ranks at once (the ceiling the e2e can reach).
  * ``roofline``: the dominant kernel's algorithmic bytes (symbol + index + compressed bytes per
    symbol, plus its tables) over its CUDA-event time, against the measured HBM copy bandwidth.
  * ``cpu_baseline`` (N = 1): the reference CPU implementation (compiled from the reference's
    sources by oracle/build_ref.py) on a bounded sample of the same workload, all host threads,
    with the same steps and warm-up as ``--impl reference``.
  * ``parity``: the GPU's bytes, lengths and decoded symbols against that reference on the same
    sample (rank 0; at N > 1 a smaller sample).
``--impl reference`` times only the reference CPU implementation (rank 0), on the same workload
and metric; that process loads none of this library's native code.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import struct
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "encode & decode Gsymbols/s at 1/2/4/8 B200, bit-exact vs reference CPU"
UNIT = "Gsymbols/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="mixture_invcdf")
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"])
    ap.add_argument("--scale", type=float, default=1.0, help="fraction of the configuration's streams")
    ap.add_argument("--length-scale", type=float, default=1.0, help="fraction of the configuration's stream length")
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--e2e-chunk", type=int, default=4096, help="symbols per column chunk of the host pipeline")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--parity-streams", type=int, default=64,
                    help="streams of the byte-parity sample when no CPU-baseline sample is run (N > 1)")
    ap.add_argument("--no-other-configs", action="store_true",
                    help="skip the short runs of the metric's other configurations (single-GPU default run only)")
    ap.add_argument("--probe", action="store_true",
                    help="instead of the benchmark: the latency probes (cycles of one dependent step, tans_probe)")
    ap.add_argument("--clocks-dir", default=None,
                    help="folder that keeps the nvidia-smi samples of the timed region (default: a temporary folder)")
    return ap.parse_args()


def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        from datetime import timedelta
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo", timeout=timedelta(seconds=180))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return ws, rank, local


def max_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(ws):
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()


def reference_steps(steps, warmup):
    """Seconds of reference CPU work per step, the same for the reference arm and the CPU leg."""
    return min(10.0, max(2.0, 120.0 / max(1, steps + warmup)))


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index, folder=None, tag=""):
        try:
            self.gpu = "GPU-" + str(torch.cuda.get_device_properties(gpu_index).uuid)
        except Exception:
            self.gpu = str(gpu_index)
        self.proc = None
        if folder is None:
            import tempfile
            folder = tempfile.mkdtemp(prefix="tans_clocks_")
        self.path = os.path.join(folder, f"clocks_rank{gpu_index}{tag}.csv")

    def __enter__(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        out = {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        try:
            rows = [l.split(",") for l in open(self.path).read().strip().splitlines() if l.strip()]
        except Exception:
            return out
        rows = [[c.strip() for c in r] for r in rows if len(r) >= 9]
        if not rows:
            return out
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        out.update(sm_mhz=statistics.median(sm) if sm else None, sm_max_mhz=max(mx) if mx else None,
                   reasons=sorted(reasons), samples=len(rows))
        return out


def measured_peak_hbm():
    try:
        d = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def reference_lib():
    """The compiled reference CPU extension (oracle/_ref), or None."""
    from oracle import build_ref
    return build_ref.load()


def port_alias_builder():
    """The oracle's restatement of rans_alias_build_table (for hosts without oracle/_ref)."""
    from oracle import oracle as O

    def build(cdfs, sizes, symbol_precision=8, freq_precision=16):
        remap, table, _ = O.alias_build_table(cdfs.numpy(), sizes.numpy(), symbol_precision, freq_precision)
        return torch.from_numpy(remap), torch.from_numpy(table)
    return build


def build_workload(name, device, scale, length_scale, seed_offset=0, alias_builder=None):
    from torch_ans_b200 import workloads as W
    fn = W.BUILDERS[name]
    kw = dict(device=device, scale=scale)
    if name != "gaussian_latent":
        kw["length_scale"] = length_scale
    if name == "zipf_alias" and alias_builder is not None:
        kw["alias_builder"] = alias_builder
    if seed_offset:
        import inspect
        kw["seed"] = inspect.signature(fn).parameters["seed"].default + seed_offset
    return fn(**kw)


def shard_of(w, lo, hi):
    """The workload restricted to streams [lo, hi) (the same object when that is all of them)."""
    import dataclasses
    if lo == 0 and hi == w.symbols.shape[0]:
        return w
    return dataclasses.replace(w, symbols=w.symbols[lo:hi].contiguous(), indexes=w.indexes[lo:hi].contiguous())


# ----------------------------------------------------------------------------- our GPU path
def time_round_trips(args, w, ws, local, tag=""):
    """Warm-up, then K timed push + pop steps of the rank's batch `w` (all ranks take part)."""
    from torch_ans_b200 import _C
    dev = torch.device("cuda", local)
    B, N = w.symbols.shape
    push = getattr(_C, w.push_op)
    pop = getattr(_C, w.pop_op)
    init = getattr(_C, f"{w.variant}_init_stream")
    kw = dict(freq_precision=w.fp, bypass_coding=w.bypass, bypass_precision=w.bp)
    push_t, pop_t = w.tables_for_push(), w.tables_for_pop()

    def step(ev=None):
        st = init(B, device=str(dev))  # made on the device: the push resizes without a device read
        if ev:
            ev[0].record()
        push(st, w.symbols, w.indexes, push_t, w.cdfs_sizes, w.offsets, **kw)
        if ev:
            ev[1].record()
        comp = st[:, 0].clone()
        dec = pop(st, w.indexes, pop_t, w.cdfs_sizes, w.offsets, **kw)
        if ev:
            ev[2].record()
        return dec, comp

    for _ in range(args.warmup):
        dec, comp = step()
    torch.cuda.synchronize()
    ok = bool(torch.equal(dec, w.symbols))
    sb = 8 if w.variant == "rans64" else 4
    comp_bytes = float((comp.to(torch.int64) - sb).sum().item())
    del dec
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local, args.clocks_dir, tag) as clk:
        barrier(ws)
        n_launch0 = _C.launch_count()
        t0.record()
        for k in range(args.steps):
            dec, comp = step(evs[k])
        t1.record()
        n_launch = _C.launch_count() - n_launch0
        barrier(ws)
    ok = ok and bool(torch.equal(dec, w.symbols)) and _C.device_status() == 0
    del dec
    ms = t0.elapsed_time(t1) / args.steps
    push_ms = sum(e[0].elapsed_time(e[1]) for e in evs) / args.steps
    pop_ms = sum(e[1].elapsed_time(e[2]) for e in evs) / args.steps
    return dict(ms=max_over_ranks(ms, ws), push_ms=max_over_ranks(push_ms, ws), pop_ms=max_over_ranks(pop_ms, ws),
                push_ms_local=push_ms, pop_ms_local=pop_ms, ok=max_over_ranks(0.0 if ok else 1.0, ws) == 0.0,
                comp_bytes=comp_bytes, n_launch=int(n_launch), clocks=clk.summary(), B=B, N=N)


def roofline(args, w, r, nsym):
    """Roofline of the dominant kernel on this rank (algorithmic bytes / CUDA-event time)."""
    push_t, pop_t = w.tables_for_push(), w.tables_for_pop()
    c = r["comp_bytes"] / nsym
    table_bytes = {"push": push_t.numel() * 4 + 16 * push_t.shape[0], "pop": pop_t.numel() * 4 + 16 * pop_t.shape[0]}
    alg = {"push": nsym * (8 + c) + table_bytes["push"], "pop": nsym * (8 + c) + table_bytes["pop"]}
    dom = "pop" if r["pop_ms_local"] >= r["push_ms_local"] else "push"
    dom_ms = r["pop_ms_local"] if dom == "pop" else r["push_ms_local"]
    peak, peak_kind = measured_peak_hbm()
    achieved = alg[dom] / (dom_ms / 1e3) / 1e9
    traffic = None
    try:
        prof = json.load(open(os.path.join(ROOT, "profiles", "traffic.json")))
        ent = prof.get(f"{args.workload}:{dom}")
        if ent:
            traffic = ent["dram_bytes_per_symbol"] * nsym
    except Exception:
        pass
    # the kernels are bound by the latency of one serial step per stream: report it beside the
    # bandwidth roofline (every stream runs its N steps concurrently with the others)
    step_ns = dom_ms * 1e6 / max(r["N"], 1)
    mhz = r["clocks"].get("sm_mhz")
    return {"bound": "hbm", "kernel": f"{w.pop_op if dom == 'pop' else w.push_op}", "achieved": achieved, "peak": peak,
            "unit": "GB/s", "frac": achieved / peak, "peak_kind": peak_kind, "traffic": traffic,
            "algorithmic_bytes_per_launch": alg[dom], "launch_ms": dom_ms, "serial_step_ns": step_ns,
            "serial_step_cycles": step_ns * mhz / 1e3 if mhz else None, "streams_in_flight": r["B"]}


def run_ours(args, ws, rank, local):
    from torch_ans_b200.sharding import shard_streams
    dev = torch.device("cuda", local)
    # every rank builds the configuration's whole batch from the same seed: in strong scaling it
    # codes its shard of it, in weak scaling all of it
    w_full = build_workload(args.workload, dev, args.scale, args.length_scale)
    B_cfg, N = w_full.symbols.shape
    if args.scaling == "strong":
        shards = [shard_streams(B_cfg, ws, r) for r in range(ws)]
        lo, hi = shards[rank]
        w = shard_of(w_full, lo, hi)
        job_streams = B_cfg
    else:
        shards = [(0, B_cfg) for _ in range(ws)]
        w = w_full
        job_streams = B_cfg * ws
    r = time_round_trips(args, w, ws, local)
    total = job_streams * N
    res = dict(value=total / (r["ms"] / 1e3) / 1e9, ms=r["ms"], gpu_launches=r["n_launch"], push_ms=r["push_ms"],
               pop_ms=r["pop_ms"], ok=r["ok"], nsym=total, B=w.symbols.shape[0], N=N, job_streams=job_streams,
               comp_bytes_per_symbol=r["comp_bytes"] / max(w.symbols.numel(), 1), clocks=r["clocks"],
               roofline=roofline(args, w, r, w.symbols.numel()),
               encode_gsym_s=total / (r["push_ms"] / 1e3) / 1e9, decode_gsym_s=total / (r["pop_ms"] / 1e3) / 1e9)
    if ws > 1 and args.scaling == "strong":
        # the weak-scaling view: every rank codes the whole batch
        rw = time_round_trips(args, w_full, ws, local, tag="_weak")
        tw = B_cfg * N * ws
        res["weak_scaling"] = {"value": tw / (rw["ms"] / 1e3) / 1e9, "unit": UNIT, "ms_per_step": rw["ms"],
                               "streams_per_gpu": B_cfg, "push_ms": rw["push_ms"], "pop_ms": rw["pop_ms"],
                               "bit_exact_roundtrip": rw["ok"], "clocks": rw["clocks"]}
        res["ok"] = res["ok"] and rw["ok"]
    if not args.no_e2e:
        res["e2e"] = run_e2e(args, w, w_full, shards, ws, rank, dev)
    del w, w_full
    torch.cuda.empty_cache()
    return res


def host_link_ceiling(h2d_bytes, d2h_bytes, ws, dev, reps=2):
    """Time of plain pinned H2D + D2H copies of the given sizes on every rank at once (one copy
    per direction on two CUDA streams): the host link's ceiling for the e2e step's traffic."""
    chunk = 1 << 30
    nh, nd = max(1, min(h2d_bytes, chunk)), max(1, min(d2h_bytes, chunk))
    hs = torch.empty(nh, dtype=torch.uint8, pin_memory=True)
    hd = torch.empty(nd, dtype=torch.uint8, pin_memory=True)
    ds = torch.empty(nh, dtype=torch.uint8, device=dev)
    dd = torch.empty(nd, dtype=torch.uint8, device=dev)
    s1, s2 = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def once():
        with torch.cuda.stream(s1):
            left = h2d_bytes
            while left > 0:
                n = min(left, nh)
                ds[:n].copy_(hs[:n], non_blocking=True)
                left -= n
        with torch.cuda.stream(s2):
            left = d2h_bytes
            while left > 0:
                n = min(left, nd)
                hd[:n].copy_(dd[:n], non_blocking=True)
                left -= n
        s1.synchronize()
        s2.synchronize()

    once()
    barrier(ws)
    t = time.perf_counter()
    for _ in range(reps):
        once()
    barrier(ws)
    el = max_over_ranks((time.perf_counter() - t) / reps, ws)
    del hs, hd, ds, dd
    return el


def run_e2e(args, w, w_full, shards, ws, rank, dev):
    """Round trip through the public host-batch API (torch_ans_b200.host_pipeline.HostStreamCoder)
    from pinned host memory, with the job-wide concatenated bitstream assembled from the per-stream
    length all-gather (host wall clock, max over ranks)."""
    from torch_ans_b200 import _C
    from torch_ans_b200.host_pipeline import HostStreamCoder
    from torch_ans_b200.sharding import JobBitstream, gather_stream_lengths, record_offsets_from_lengths
    B_all, N = w.symbols.shape
    # pinned host buffers per rank: symbols, indexes, decoded symbols (4 B each) and the bitstream;
    # every rank of this host gets an equal share of 40 % of the available host memory, and when
    # a rank's whole batch does not fit, the round trip runs on its first streams (same workload)
    try:
        import psutil
        avail = psutil.virtual_memory().available
    except Exception:
        avail = 64 << 30
    local_ws = int(os.environ.get("LOCAL_WORLD_SIZE", ws))
    per_stream = N * (3 * 4 + 2)
    B = int(max(1, min(B_all, (0.4 * avail / max(local_ws, 1)) // per_stream)))
    if ws > 1:  # every rank codes the same number of streams
        t = torch.tensor([B], dtype=torch.int64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        B = int(t.item())
    e2e_shards = [(r * B, (r + 1) * B) for r in range(ws)]  # this rank's records in the job bitstream
    h_sym = torch.empty((B, N), dtype=torch.int32, pin_memory=True)
    h_idx = torch.empty((B, N), dtype=torch.int32, pin_memory=True)
    h_out = torch.empty((B, N), dtype=torch.int32, pin_memory=True)
    h_sym.copy_(w.symbols[:B])
    h_idx.copy_(w.indexes[:B])
    torch.cuda.synchronize()
    coder = HostStreamCoder(w.variant, w.tables_for_push(), w.tables_for_pop(), w.cdfs_sizes, w.offsets,
                            freq_precision=w.fp, bypass_coding=w.bypass, bypass_precision=w.bp,
                            alias=w.push_cdfs is not None, lookup=w.lookup, device=dev, chunk_symbols=args.e2e_chunk)
    job = None
    h_in = None
    h2d = d2h = 0
    state = {}

    def once():
        nonlocal job, h_in, h2d, d2h
        stream = coder.encode_to_device(h_sym, h_idx)
        if ws > 1:
            lens = gather_stream_lengths(stream[:, 0].contiguous(), e2e_shards)  # NCCL, one int32 per stream
            offs, total = record_offsets_from_lengths(lens)
            lo, hi = e2e_shards[rank]
            start = int(offs[lo])
            end = int(offs[hi]) if hi < len(lens) else total
            if job is None:  # first round: rank 0 makes the job file with the job's total size
                name = [JobBitstream.default_path(f"{os.getpid()}", total) if rank == 0 else None]
                dist.broadcast_object_list(name, src=0)
                job = JobBitstream(name[0])
                if rank == 0:
                    job.create(total)
                dist.barrier()
                job.open()
                # this rank's byte range of the job file, page-locked: the records go straight in
                h_in = job.map_range(start, end - start)
                state.update(total=total, lens=lens, offs=offs, start=start, end=end, registered=job.registered)
            elif total != state["total"] or start != state["start"]:
                raise RuntimeError("job bitstream layout changed between identical steps")
            data = coder.container_to_host(stream, out=h_in)  # raises unless it matches the lengths
            del stream
        else:
            data = coder.container_to_host(stream)
            del stream
        coder.decode(data, h_idx, out=h_out)
        h2d = 2 * B * N * 4 + B * N * 4 + data.numel()
        d2h = data.numel() + B * N * 4
        return data.numel()

    once()  # warm-up (pinned buffer allocation, table prep, job file)
    ok = bool(torch.equal(h_out, h_sym))
    barrier(ws)
    t = time.perf_counter()
    for _ in range(args.e2e_steps):
        once()
    barrier(ws)
    el = (time.perf_counter() - t) / args.e2e_steps
    ok = ok and bool(torch.equal(h_out, h_sym)) and coder.device_status() == 0
    el = max_over_ranks(el, ws)
    res = {"value": B * N * ws / el / 1e9, "unit": UNIT, "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
           "ms_per_step": el * 1e3, "streams_per_gpu": B, "of_streams_per_gpu": B_all}
    if ws > 1:
        # the job bitstream against single-process records: rank 0 pushes the first and the last
        # stream of every rank's range on its own and compares their records byte for byte
        checked = 0
        if rank == 0:
            lens, offs = state["lens"], state["offs"]
            pick = sorted({(r, j) for r in range(ws) for j in (0, B - 1)})
            rows = [shards[r][0] + j for r, j in pick]  # stream of the configuration each record codes
            ws_ = w_full.symbols[rows].contiguous()
            wi_ = w_full.indexes[rows].contiguous()
            st = getattr(_C, f"{w.variant}_init_stream")(len(rows), device=str(dev))
            getattr(_C, w.push_op)(st, ws_, wi_, w.tables_for_push(), w.cdfs_sizes, w.offsets, freq_precision=w.fp,
                                   bypass_coding=w.bypass, bypass_precision=w.bp)
            alone = _C.rans_stream_to_byte_strings(st)
            for (r, j), rec in zip(pick, alone):
                g = e2e_shards[r][0] + j
                got = job.read(int(offs[g]), torch.empty(4 + len(rec), dtype=torch.uint8)).numpy().tobytes()
                ok = ok and got == struct.pack("<I", len(rec)) + rec and int(lens[g]) == len(rec)
                checked += 1
        dist.barrier()
        h_in = None  # the last view of this rank's mapped range goes before the mapping closes
        job.close(unlink=(rank == 0))
        res["job_bitstream"] = {"bytes": int(state["total"]), "records": int(B * ws), "records_checked": checked,
                                "against": "records of the same streams pushed alone on one GPU",
                                "collective": "all_gather of one int32 length per stream (NCCL)",
                                "host_file": "shared file mapped by every rank, each rank's range page-locked"
                                if state["registered"] else "shared file mapped by every rank (not page-locked)"}
    res["ok"] = max_over_ranks(0.0 if ok else 1.0, ws) == 0.0
    del h_sym, h_idx, h_out, coder, h_in
    ceil_s = host_link_ceiling(int(h2d), int(d2h), ws, dev)
    res["host_link"] = {"copy_only_ms": ceil_s * 1e3, "h2d_gbs": h2d * ws / ceil_s / 1e9 if ceil_s else None,
                        "d2h_gbs": d2h * ws / ceil_s / 1e9 if ceil_s else None,
                        "e2e_frac_of_copy_ceiling": ceil_s / el if el else None,
                        "how": "plain pinned H2D and D2H copies of the step's bytes, both directions at once, "
                               "all ranks at once, max over ranks"}
    res["path"] = ("pinned host -> HostStreamCoder.encode_to_device (column chunks: H2D || push) -> per-stream length "
                   "all-gather -> device assembly of this rank's records -> D2H into the job bitstream at the scanned "
                   "offset -> this rank's byte range -> HostStreamCoder.decode (H2D || pop || D2H) -> pinned host")
    return res


# ----------------------------------------------------------------------------- ragged workload
def run_ours_ragged(args, ws, rank, local):
    """ragged_adaptive: streams of different lengths, one cdf row per symbol (ragged ops)."""
    from torch_ans_b200 import _C
    from torch_ans_b200.workloads import ragged_adaptive
    dev = torch.device("cuda", local)
    w = ragged_adaptive(dev, scale=args.scale, length_scale=args.length_scale, seed=4 + 1000 * rank)
    B, T = w.num_streams, w.num_symbols
    push = getattr(_C, f"{w.variant}_push_ragged")
    pop = getattr(_C, f"{w.variant}_pop_ragged")
    kw = dict(freq_precision=w.fp, bypass_coding=w.bypass, bypass_precision=w.bp)
    init = getattr(_C, f"{w.variant}_init_stream")
    lengths = (w.row_starts[1:] - w.row_starts[:-1]).cpu()

    def step(ev=None):
        st = init(B, device=str(dev))
        if ev:
            ev[0].record()
        push(st, w.symbols, w.row_starts, w.cdfs, w.cdfs_sizes, offsets=w.offsets, **kw)
        if ev:
            ev[1].record()
        comp = st[:, 0].clone()
        dec = pop(st, w.row_starts, w.cdfs, w.cdfs_sizes, offsets=w.offsets, **kw)
        if ev:
            ev[2].record()
        return dec, comp

    for _ in range(args.warmup):
        dec, comp = step()
    torch.cuda.synchronize()
    ok = bool(torch.equal(dec, w.symbols))
    comp_bytes = float((comp.to(torch.int64) - 4).sum().item())
    del dec
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local, args.clocks_dir) as clk:
        barrier(ws)
        n_launch0 = _C.launch_count()
        t0.record()
        for k in range(args.steps):
            dec, comp = step(evs[k])
        t1.record()
        n_launch = _C.launch_count() - n_launch0
        barrier(ws)
    ok = ok and bool(torch.equal(dec, w.symbols)) and _C.device_status() == 0
    del dec
    ms = t0.elapsed_time(t1) / args.steps
    push_ms = sum(e[0].elapsed_time(e[1]) for e in evs) / args.steps
    pop_ms = sum(e[1].elapsed_time(e[2]) for e in evs) / args.steps
    ms_max = max_over_ranks(ms, ws)
    push_ms_max, pop_ms_max = max_over_ranks(push_ms, ws), max_over_ranks(pop_ms, ws)
    all_ok = max_over_ranks(0.0 if ok else 1.0, ws) == 0.0
    total = T * ws
    c = comp_bytes / T
    # algorithmic bytes: encode reads symbol + the two cdf entries bracketing it and writes c;
    # decode reads the whole 33-entry row (the symbol is unknown before the lookup), reads c and
    # writes the symbol
    A1 = w.cdfs.shape[1]
    alg = {"push": T * (4 + 8 + c), "pop": T * (4 * A1 + c + 4)}
    dom = "pop" if pop_ms >= push_ms else "push"
    dom_ms = pop_ms if dom == "pop" else push_ms
    peak, peak_kind = measured_peak_hbm()
    achieved = alg[dom] / (dom_ms / 1e3) / 1e9
    res = dict(value=total / (ms_max / 1e3) / 1e9, ms=ms_max, gpu_launches=int(n_launch), push_ms=push_ms_max,
               pop_ms=pop_ms_max, ok=all_ok, nsym=T, B=B, N=int(lengths.max()), job_streams=B * ws,
               comp_bytes_per_symbol=c, clocks=clk.summary(),
               roofline={"bound": "hbm", "kernel": f"{w.variant}_{dom}_ragged", "achieved": achieved, "peak": peak,
                         "unit": "GB/s", "frac": achieved / peak, "peak_kind": peak_kind, "traffic": None,
                         "algorithmic_bytes_per_launch": alg[dom], "launch_ms": dom_ms},
               encode_gsym_s=total / (push_ms_max / 1e3) / 1e9, decode_gsym_s=total / (pop_ms_max / 1e3) / 1e9,
               lengths={"total_symbols": T, "max": int(lengths.max()), "mean": float(lengths.double().mean())})
    del w
    torch.cuda.empty_cache()
    return res


_RAGGED_REF = None


def _ragged_ref_init():
    global _RAGGED_REF
    torch.set_num_threads(1)
    _RAGGED_REF = reference_lib()


def _ragged_ref_worker(task):
    """One worker's share of the ragged sample: build its streams (same generator recipe), then
    run the reference op per stream (B = 1), as the reference must for ragged streams."""
    lengths, seed = task
    from torch_ans_b200.workloads import quantize_pmf
    ref = _RAGGED_REF
    g = torch.Generator().manual_seed(seed)
    streams = []
    for n in lengths:
        p = torch.softmax(torch.randn((n, 32), generator=g, dtype=torch.float64) * 2.0, -1)
        cdf = quantize_pmf(p, 16)
        u = torch.randint(0, 1 << 16, (n, 1), generator=g, dtype=torch.int64)
        sym = (torch.searchsorted(cdf, u, right=True) - 1).reshape(1, n).to(torch.int32)
        streams.append((sym, cdf.to(torch.int32).contiguous(), torch.full((n,), 33, dtype=torch.int32),
                        torch.zeros(n, dtype=torch.int32), torch.arange(n, dtype=torch.int32).reshape(1, n)))
    kw = dict(freq_precision=16, bypass_coding=False, bypass_precision=4)
    ok = True
    t0 = time.perf_counter()
    tp = 0.0
    for sym, cdf, sizes, offs, idx in streams:
        st = ref.rans32_init_stream(1)
        a = time.perf_counter()
        ref.rans32_push(st, sym, idx, cdf, sizes, offs, **kw)
        tp += time.perf_counter() - a
        dec = ref.rans32_pop(st, idx, cdf, sizes, offs, **kw)
        ok = ok and bool(torch.equal(dec, sym))
    return sum(lengths), time.perf_counter() - t0, tp, ok


def cpu_reference_ragged(seconds, scale, length_scale):
    """Reference CPU on a bounded sample of the ragged workload: the first streams of the length
    list (same distribution) up to about `seconds` of work, spread over all host cores as
    separate processes (the reference op on B = 1 runs on one thread), timed as the slowest
    worker's push + pop loop."""
    import multiprocessing as mp
    from torch_ans_b200.workloads import ragged_lengths
    if reference_lib() is None:
        return None
    threads = len(os.sched_getaffinity(0))
    lengths = ragged_lengths(max(1, int(4096 * scale)), length_scale, 4).tolist()
    budget = int(seconds * threads * 4e6)  # symbols: ~4 M per core-second of push + pop
    picked, tot = [], 0
    for n in lengths:
        if tot + n > budget and picked:
            break
        picked.append(int(n))
        tot += n
    shares = [[] for _ in range(threads)]
    loads = [0] * threads
    for n in sorted(picked, reverse=True):  # longest first onto the least loaded worker
        j = loads.index(min(loads))
        shares[j].append(n)
        loads[j] += n
    tasks = [(s, 100 + j) for j, s in enumerate(shares) if s]
    with mp.get_context("spawn").Pool(len(tasks), initializer=_ragged_ref_init) as pool:
        out = pool.map(_ragged_ref_worker, tasks)
    nsym = sum(o[0] for o in out)
    wall = max(o[1] for o in out)
    tp = max(o[2] for o in out)
    assert all(o[3] for o in out), "reference CPU round trip failed"
    return {"value": nsym / wall / 1e9, "unit": UNIT, "cores": len(tasks), "kind": "reference",
            "sample": f"{len(picked)} of {len(lengths)} streams ({nsym} symbols) of ragged_adaptive, per-stream "
                      f"B=1 reference calls in {len(tasks)} processes, push + pop",
            "encode_gsym_s": nsym / tp / 1e9, "decode_gsym_s": nsym / max(wall - tp, 1e-9) / 1e9,
            "ms_per_step": wall * 1e3}


# ----------------------------------------------------------------------------- reference CPU
def cpu_reference(workload_name, seconds, scale, length_scale, steps=1, warmup=0, keep_sample=False,
                  max_streams=None):
    """Time the reference CPU implementation (oracle/_ref, else the oracle's C port) on a
    bounded sample of the workload: S streams of the configuration (same tables, same stream
    length), S chosen so one push + pop takes about `seconds` on all host threads.  Every table,
    alias tables included, is made by the reference's own code.  With `keep_sample` the sample and
    the reference's pushed stream come back too (for the byte-parity check)."""
    ref = reference_lib()
    kind = "reference" if ref is not None else "port"
    alias_builder = ref.rans_alias_build_table if ref is not None else port_alias_builder()
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    # the stream count of the full configuration, from a probe with one-symbol streams
    probe = build_workload(workload_name, "cpu", scale=scale, length_scale=1e-9, alias_builder=alias_builder)
    b_full = probe.symbols.shape[0]
    del probe

    def make(nstreams):
        return build_workload(workload_name, "cpu", scale=scale * nstreams / b_full, length_scale=length_scale,
                              alias_builder=alias_builder)

    pushed = {}

    def run(w):
        B = w.symbols.shape[0]
        push_t, pop_t = w.tables_for_push().contiguous(), w.tables_for_pop().contiguous()
        kw = dict(freq_precision=w.fp, bypass_coding=w.bypass, bypass_precision=w.bp)
        if kind == "reference":
            st = getattr(ref, f"{w.variant}_init_stream")(B)
            t0 = time.perf_counter()
            getattr(ref, w.push_op)(st, w.symbols, w.indexes, push_t, w.cdfs_sizes, w.offsets, **kw)
            t1 = time.perf_counter()
            if keep_sample:
                pushed["stream"] = st.clone()
            dec = getattr(ref, w.pop_op)(st, w.indexes, pop_t, w.cdfs_sizes, w.offsets, **kw)
            t2 = time.perf_counter()
        else:
            from oracle import oracle as O
            st = O.init_stream(w.variant, B)
            t0 = time.perf_counter()
            st, _ = O.push(w.variant, st, w.symbols.numpy(), w.indexes.numpy(), push_t.numpy(), w.cdfs_sizes.numpy(),
                           w.offsets.numpy(), w.fp, w.bypass, w.bp, alias=w.lookup == "alias", threads=threads)
            t1 = time.perf_counter()
            if keep_sample:
                pushed["stream"] = torch.from_numpy(st.copy())
            dec, _ = O.pop(w.variant, st, w.indexes.numpy(), pop_t.numpy(), w.cdfs_sizes.numpy(), w.offsets.numpy(),
                           w.fp, w.bypass, w.bp, lookup=w.lookup, threads=threads)
            dec = torch.from_numpy(dec)
            t2 = time.perf_counter()
        assert torch.equal(dec, w.symbols), "reference CPU round trip failed"
        return t1 - t0, t2 - t1

    n = min(b_full, max(threads, 1))
    if max_streams is not None:
        n = min(b_full, max_streams) if seconds <= 0 else min(n, max_streams)
    w = make(n)
    tp, tq = run(w)
    per_stream = (tp + tq) / n
    n2 = int(min(b_full, max(n, seconds / max(per_stream, 1e-9))))
    # at most 2^28 symbols (2 GiB of host symbols + indexes) per sample, so the sample's build and
    # the whole reference run stay within a few minutes on any host
    N_full = w.symbols.shape[1]
    n2 = max(n, min(n2, (1 << 28) // max(N_full, 1)))
    if max_streams is not None:
        n2 = min(n2, max_streams)
    if n2 >= threads:
        n2 = n2 // threads * threads
    if n2 > n:
        del w
        n = n2
        w = make(n)
    for _ in range(warmup):
        run(w)
    tps, tqs = [], []
    for _ in range(max(1, steps)):
        tp, tq = run(w)
        tps.append(tp)
        tqs.append(tq)
    tp, tq = sum(tps) / len(tps), sum(tqs) / len(tqs)
    N = w.symbols.shape[1]
    nsym = n * N
    out = {"value": nsym / (tp + tq) / 1e9, "unit": UNIT, "cores": threads, "kind": kind,
           "sample": f"{n} of {b_full} streams x {N} symbols ({nsym} symbols) of {workload_name}, push + pop, "
                     f"{max(1, steps)} timed step(s) after {warmup} warm-up",
           "encode_gsym_s": nsym / tp / 1e9, "decode_gsym_s": nsym / tq / 1e9, "ms_per_step": (tp + tq) * 1e3}
    if keep_sample:
        return out, w, pushed["stream"]
    return out


def check_parity(w, ref_stream, kind, dev):
    """Push and pop the reference's sample on the GPU through `_C` and compare row lengths,
    payload bytes and decoded symbols with the reference's."""
    from torch_ans_b200 import _C
    B = w.symbols.shape[0]
    kw = dict(freq_precision=w.fp, bypass_coding=w.bypass, bypass_precision=w.bp)
    sym, idx = w.symbols.to(dev), w.indexes.to(dev)
    st = getattr(_C, f"{w.variant}_init_stream")(B, device=str(dev))
    getattr(_C, w.push_op)(st, sym, idx, w.tables_for_push().to(dev), w.cdfs_sizes.to(dev), w.offsets.to(dev), **kw)
    lens_equal = bool(torch.equal(st[:, 0].cpu(), ref_stream[:, 0]))
    ours = _C.rans_stream_to_byte_strings(st)
    theirs = [ref_stream[b, 1:].numpy().tobytes()[: int(ref_stream[b, 0])] for b in range(B)]
    bytes_equal = lens_equal and ours == theirs
    width_equal = st.shape[1] == ref_stream.shape[1]
    dec = getattr(_C, w.pop_op)(st, idx, w.tables_for_pop().to(dev), w.cdfs_sizes.to(dev), w.offsets.to(dev), **kw)
    decode_equal = bool(torch.equal(dec.cpu(), w.symbols))
    status = _C.device_status()
    del st, dec, sym, idx
    return {"streams_checked": B, "symbols_checked": int(w.symbols.numel()), "bytes_equal": bytes_equal,
            "lengths_equal": lens_equal, "row_width_equal": width_equal, "decode_equal": decode_equal,
            "device_status": status, "against": "oracle/_ref (the reference CPU path)" if kind == "reference"
            else "the oracle's C port"}


OTHER_CONFIGS = ("laplace64", "gaussian_latent", "zipf_alias", "ragged_adaptive")


def other_configs(args, dev):
    """The metric's other configurations on this GPU, one short run each: device round trips timed
    as the headline is (CUDA events, warm-up first, clocks sampled), a byte-parity sample against
    the reference CPU (oracle/_ref) and the reference CPU's rate on that sample (not for the ragged
    configuration, whose per-stream reference calls are timed by --workload ragged_adaptive)."""
    import copy
    out = {}
    for name in OTHER_CONFIGS:
        if name == args.workload:
            continue
        a = copy.copy(args)
        a.workload, a.no_e2e, a.scale, a.length_scale = name, True, 1.0, 1.0
        a.steps, a.warmup = max(1, min(args.steps, 5)), max(3, min(args.warmup, 3))
        torch.cuda.empty_cache()
        if name == "ragged_adaptive":
            r = run_ours_ragged(a, 1, 0, dev.index or 0)
            base = par = None
        else:
            r = run_ours(a, 1, 0, dev.index or 0)
            base = par = None
            if not args.no_cpu:
                base, sample, ref_stream = cpu_reference(name, 2.0, 1.0, 1.0, steps=1, warmup=0, keep_sample=True)
                par = check_parity(sample, ref_stream, base["kind"], dev)
                del sample, ref_stream
        out[name] = {"value": r["value"], "unit": UNIT, "ms_per_step": r["ms"], "steps": a.steps, "warmup": a.warmup,
                     "push_ms": r["push_ms"], "pop_ms": r["pop_ms"], "streams": r["B"], "symbols": r["nsym"],
                     "bit_exact_roundtrip": r["ok"], "gpu_launches": r["gpu_launches"], "clocks": r["clocks"],
                     "roofline_frac": r["roofline"]["frac"], "roofline_kernel": r["roofline"]["kernel"],
                     "cpu_baseline": base, "parity": par}
        torch.cuda.empty_cache()
    return out


def reference_arm(args, ws, rank, cfg):
    """--impl reference: the reference's own CPU implementation only (rank 0)."""
    if rank == 0:
        per_step = reference_steps(args.steps, args.warmup)
        if args.workload == "ragged_adaptive":
            base = cpu_reference_ragged(per_step * 4, args.scale, args.length_scale)
        else:
            base = cpu_reference(args.workload, per_step, args.scale, args.length_scale, steps=args.steps,
                                 warmup=args.warmup)
        if base is None:
            print(json.dumps({"impl": "reference", "unavailable": "the reference CPU library (oracle/_ref) is "
                              "not built on this machine"}), flush=True)
        else:
            line = {"metric": METRIC, "value": base["value"], "unit": UNIT, "n_gpus": ws, "steps": args.steps,
                    "warmup": args.warmup, "ms_per_step": base["ms_per_step"], "higher_is_better": True,
                    "scaling": args.scaling, "vs_baseline": None, "dtype": "int64", "data": "synthetic", "config": cfg,
                    "impl": "reference", "cpu_baseline": base,
                    "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
            print(json.dumps(line), flush=True)


def run_probes():
    """The latency probes behind the kernel design: cycles of one dependent step (clock64 on the
    device), printed as one JSON line."""
    from torch_ans_b200 import capi
    steps = {"smem_chase": 1 << 20, "l2_chase": 1 << 18, "l2_chase_busy": 1 << 15}
    out = {k: capi.probe(k, steps.get(k, 1 << 20)) for k in capi.PROBES}
    mhz = None
    try:
        r = subprocess.run(["nvidia-smi", "--id=0", "--query-gpu=clocks.sm", "--format=csv,noheader,nounits"],
                           capture_output=True, text=True, timeout=20)
        mhz = float(r.stdout.strip().splitlines()[0])
    except Exception:
        pass
    print(json.dumps({"probe": "cycles per dependent step", "gpu": torch.cuda.get_device_name(0), "sm_mhz_after": mhz,
                      "cycles": {k: round(v, 1) for k, v in out.items()}}), flush=True)


def main():
    args = parse()
    if args.probe:
        run_probes()
        return
    ws, rank, local = dist_setup()
    ragged = args.workload == "ragged_adaptive"
    cfg = {"workload": args.workload, "scale": args.scale, "length_scale": args.length_scale,
           "l2": "inputs larger than L2 (no flush)",
           "parallelism": (f"stream shards x{ws} ({args.scaling} scaling)" if ws > 1 else "single GPU")}
    if args.impl == "reference":
        reference_arm(args, ws, rank, cfg)
        if ws > 1:
            dist.destroy_process_group()
        return

    if ragged and args.scaling == "strong" and ws > 1:
        args.scaling = "weak"  # the ragged workload runs one batch per rank
    res = run_ours_ragged(args, ws, rank, local) if ragged else run_ours(args, ws, rank, local)
    base = parity = None
    dev = torch.device("cuda", local)
    if rank == 0 and not ragged:
        per_step = reference_steps(args.steps, args.warmup)
        if ws == 1 and not args.no_cpu:
            base, sample, ref_stream = cpu_reference(args.workload, per_step, args.scale, args.length_scale,
                                                     steps=args.steps, warmup=args.warmup, keep_sample=True)
        else:
            _, sample, ref_stream = cpu_reference(args.workload, 0.0, args.scale, args.length_scale, steps=1,
                                                  warmup=0, keep_sample=True, max_streams=args.parity_streams)
        parity = check_parity(sample, ref_stream, (base or {"kind": "reference" if reference_lib() else "port"})["kind"],
                              dev)
        del sample, ref_stream
    elif rank == 0 and ws == 1 and not args.no_cpu:
        base = cpu_reference_ragged(reference_steps(args.steps, args.warmup) * 4, args.scale, args.length_scale)
    if ws > 1:
        dist.barrier()
    if rank == 0:
        if "lengths" in res:
            cfg["ragged_lengths"] = res["lengths"]
        cfg.update({"streams_per_gpu": res["B"], "symbols_per_stream": res["N"], "global_batch_streams": res["job_streams"],
                    "compressed_bytes_per_symbol": round(res["comp_bytes_per_symbol"], 4)})
        line = {"metric": METRIC, "value": res["value"], "unit": UNIT, "n_gpus": ws, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": res["ms"], "higher_is_better": True, "scaling": args.scaling,
                "vs_baseline": None, "dtype": "int64", "data": "synthetic", "config": cfg,
                "encode_gsym_s": res["encode_gsym_s"], "decode_gsym_s": res["decode_gsym_s"],
                "push_ms": res["push_ms"], "pop_ms": res["pop_ms"], "bit_exact_roundtrip": res["ok"],
                "roofline": res["roofline"], "clocks": res["clocks"],
                "gpu_launches": res["gpu_launches"], "cpu_baseline": base, "parity": parity}
        for k in ("e2e", "weak_scaling"):
            if k in res:
                line[k] = res[k]
        if ws == 1 and args.workload == "mixture_invcdf" and args.scale == 1.0 and args.length_scale == 1.0 \
                and not args.no_other_configs:
            del res
            line["other_configs"] = other_configs(args, dev)
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
