"""Coding of batches that live in host memory, streamed through the GPU.

The reference's coders take CPU tensors and code them on the host.  A B200 codes a batch far
faster than PCIe can move it (about 15 GB/s of int32 symbols and indexes per direction through
the coding kernels versus roughly 50 GB/s over PCIe for the whole batch), so for host-resident
data the cost is the transfer.  ``HostStreamCoder`` hides the kernels under it:

* encode: the symbol axis is cut into column chunks (last chunk first, the order rANS pushes in);
  chunk j's symbols and indexes are copied host -> device on one CUDA stream (a single pitched
  copy per matrix, straight out of the pinned host buffer) while chunk j-1 is pushed on another;
  every stream row keeps its state between chunks, so the rows are exactly those of one push of
  the whole batch (rans_push over a concatenation equals consecutive pushes, last part first).
  At the end the concatenated bitstream is assembled on the device and copied to pinned host
  memory.
* decode: the bitstream is copied over and scattered into stream rows; then chunk j's indexes
  are copied in while chunk j-1 is popped and chunk j-2's decoded symbols are copied out on a
  third stream.

Outputs are bit-identical to the whole-batch path: ``encode`` returns the bytes of
``stream_to_merged_tensor(push(...))`` (merge_bytes of rans_stream_to_byte_strings,
torch_ans/utils.py:47-72, torch_ans/rans.cpp:5-21) and ``decode`` returns what ``pop`` returns.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _C, capi

_STATE_BYTES = {"rans64": 8, "rans32": 4, "rans32_16": 4}


class HostStreamCoder:
    """Encoder/decoder for pinned host batches (``symbols``/``indexes`` of shape (B, N), int32).

    ``variant``: "rans64", "rans32" or "rans32_16"; ``push_cdfs`` are the tables the push reads
    (alias remap rows when ``alias``), ``pop_cdfs`` those the pop reads (``lookup`` "search",
    "invcdf" or "alias"), with ``cdf_sizes`` and ``offsets`` as in the reference's ops.
    ``chunk_symbols`` sets the column chunk (a multiple of 4 keeps the fast kernels in use).
    """

    def __init__(self, variant: str, push_cdfs: torch.Tensor, pop_cdfs: torch.Tensor, cdf_sizes: torch.Tensor,
                 offsets: Optional[torch.Tensor] = None, *, freq_precision: int = 16, bypass_coding: bool = False,
                 bypass_precision: int = 4, alias: bool = False, lookup: str = "search",
                 device: Optional[torch.device] = None, chunk_symbols: int = 16384, num_bytes_length: int = 4):
        if variant not in capi.VARIANT:
            raise ValueError(f"unknown variant {variant}")
        if lookup not in capi.LOOKUP:
            raise ValueError(f"unknown lookup {lookup}")
        if num_bytes_length not in (1, 2, 4):
            raise ValueError("num_bytes_length must be 1, 2 or 4")
        if chunk_symbols < 1:
            raise ValueError("chunk_symbols must be >= 1")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        dev = self.device

        def i32(t):
            return t.to(device=dev, dtype=torch.int32).contiguous()

        self.variant, self.v = variant, capi.VARIANT[variant]
        self.alias, self.lookup = bool(alias), capi.LOOKUP[lookup]
        self.push_cdfs, self.pop_cdfs, self.sizes = i32(push_cdfs), i32(pop_cdfs), i32(cdf_sizes)
        self.offsets = i32(offsets) if offsets is not None else torch.zeros_like(self.sizes)
        self.fp, self.bypass, self.bp = int(freq_precision), bool(bypass_coding), int(bypass_precision)
        self.chunk = int(chunk_symbols)
        self.prefix = int(num_bytes_length)
        self.lib = capi.load()
        with torch.cuda.device(dev):
            self.s_h2d, self.s_comp, self.s_d2h = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
            self.status = torch.zeros(1, dtype=torch.int32, device=dev)
            K, Wc = self.push_cdfs.shape
            self.push_ws = torch.empty(self.lib.tans_push_workspace_size(self.v, K, Wc) + 256, dtype=torch.uint8,
                                       device=dev)
            K2, Wc2 = self.pop_cdfs.shape
            self.pop_ws = torch.empty(self.lib.tans_pop_workspace_size(self.v, self.lookup, K2, Wc2, self.fp) + 256,
                                      dtype=torch.uint8, device=dev)
        self._host_out = torch.empty(0, dtype=torch.uint8)

    # ------------------------------------------------------------------ helpers
    def _check(self, rc, what):
        if rc != 0:
            raise RuntimeError(f"torch_ans_b200: {what}: {self.lib.tans_status_string(rc).decode()}")

    def _chunks(self, n):
        return [(c0, min(self.chunk, n - c0)) for c0 in range(0, n, self.chunk)]

    def device_status(self) -> int:
        """TANS_DEV_* bits reported by this coder's kernels since the last call (synchronises)."""
        torch.cuda.synchronize(self.device)
        bits = int(self.status.item())
        self.status.zero_()
        return bits

    # ------------------------------------------------------------------ encode
    def encode(self, symbols: torch.Tensor, indexes: torch.Tensor) -> torch.Tensor:
        """Push every row of (B, N) pinned host ``symbols`` with ``indexes`` onto a fresh stream and
        return the concatenated bitstream (uint8 pinned host tensor; a view into a buffer that the
        next ``encode`` call reuses)."""
        return self.container_to_host(self.encode_to_device(symbols, indexes))

    def container_to_host(self, stream: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Assemble the concatenated bitstream of the device stream rows ``stream`` (merge_bytes of
        rans_stream_to_byte_strings) on the device and copy it to host memory: into ``out`` (a
        uint8 host tensor of exactly the container's size, page-locked for an asynchronous copy)
        when given, else into a pinned buffer that the next call reuses (the returned view)."""
        dev = self.device
        with torch.cuda.device(dev):
            comp = self.s_comp
            with torch.cuda.stream(comp):
                packed = _C.stream_to_merged_tensor(stream, self.prefix, None)
                done = torch.cuda.Event()
                done.record(comp)
            total = packed.numel()
            if out is not None:
                if out.numel() != total or out.dtype != torch.uint8 or out.is_cuda:
                    raise ValueError(f"out must be a uint8 host tensor of {total} bytes")
            else:
                if self._host_out.numel() < total:
                    self._host_out = torch.empty(int(total * 1.1) + 4096, dtype=torch.uint8, pin_memory=True)
                out = self._host_out[:total]
            self.s_d2h.wait_event(done)
            with torch.cuda.stream(self.s_d2h):
                out.copy_(packed, non_blocking=True)
            self.s_d2h.synchronize()
            del packed
        return out

    def encode_to_device(self, symbols: torch.Tensor, indexes: torch.Tensor) -> torch.Tensor:
        """The push half of ``encode``: returns the (B, W) device stream rows, ready on this coder's
        compute stream (``container_to_host`` orders itself after it)."""
        if symbols.shape != indexes.shape or symbols.dim() != 2:
            raise ValueError("symbols and indexes must be 2-D with the same shape")
        for t in (symbols, indexes):
            if t.is_cuda or not t.is_pinned() or t.dtype != torch.int32 or not t.is_contiguous():
                raise ValueError("symbols and indexes must be contiguous pinned int32 host tensors")
        B, N = symbols.shape
        dev, lib = self.device, self.lib
        chunks = self._chunks(N)[::-1]  # pushes run last symbol first
        C = max((c for _, c in chunks), default=0)
        # worst-case row width for the whole batch (the resize rule of rans.hpp:105-124 over N symbols,
        # plus a few bytes per chunk for the per-call rounding)
        safe = _STATE_BYTES[self.variant] + (N * self.fp + 7) // 8 + len(chunks) * 8
        if self.bypass:
            safe += N * 4
        W = safe // 4 + 2
        with torch.cuda.device(dev):
            comp = self.s_comp
            # the caller's earlier work on its stream (tables, freed buffers) comes first
            comp.wait_stream(torch.cuda.current_stream(dev))
            self.s_h2d.wait_stream(torch.cuda.current_stream(dev))
            stream = torch.empty((B, W), dtype=torch.int32, device=dev)
            with torch.cuda.stream(comp):
                self._check(lib.tans_init_stream(self.v, 1, stream.data_ptr(), B, W, comp.cuda_stream), "init")
            # two chunk buffers in turn; the one short chunk (if any) gets buffers of its own width
            # so that every chunk the kernels read is a dense (B, cn) matrix
            bufs = {}

            def chunk_bufs(sl, cn):
                key = (sl if cn == C else "short", cn)
                if key not in bufs:
                    bufs[key] = (torch.empty((B, cn), dtype=torch.int32, device=dev),
                                 torch.empty((B, cn), dtype=torch.int32, device=dev))
                return bufs[key]

            ev_in = [torch.cuda.Event() for _ in range(2)]
            ev_free = [torch.cuda.Event() for _ in range(2)]
            K, Wc = self.push_cdfs.shape
            for j, (c0, cn) in enumerate(chunks):
                sl = j % 2
                sd, idd = chunk_bufs(sl, cn)
                if j >= 2:
                    self.s_h2d.wait_event(ev_free[sl])
                _C.copy_columns(sd, 0, symbols, c0, cn, self.s_h2d.cuda_stream)
                _C.copy_columns(idd, 0, indexes, c0, cn, self.s_h2d.cuda_stream)
                ev_in[sl].record(self.s_h2d)
                comp.wait_event(ev_in[sl])
                sp, ip = sd.data_ptr(), idd.data_ptr()
                rc = lib.tans_push(self.v, int(self.alias), 1, stream.data_ptr(), B, W, sp, ip, cn,
                                   self.push_cdfs.data_ptr(), K, Wc, self.sizes.data_ptr(), self.offsets.data_ptr(),
                                   self.fp, int(self.bypass), self.bp, self.push_ws.data_ptr(), self.push_ws.numel(),
                                   self.status.data_ptr(), comp.cuda_stream)
                self._check(rc, "push")
                ev_free[sl].record(comp)
            # the chunk buffers are freed on the caller's stream: order that after the last push
            torch.cuda.current_stream(dev).wait_stream(comp)
            del bufs
        return stream

    # ------------------------------------------------------------------ decode
    def decode(self, data: torch.Tensor, indexes: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Pop N symbols from each of the B records of the concatenated bitstream ``data`` (uint8
        host tensor, pinned for an asynchronous copy) with (B, N) pinned host ``indexes``; returns
        the (B, N) int32 symbols in pinned host memory (``out`` if given)."""
        if indexes.dim() != 2 or indexes.is_cuda or not indexes.is_pinned() or indexes.dtype != torch.int32 \
                or not indexes.is_contiguous():
            raise ValueError("indexes must be a contiguous pinned (B, N) int32 host tensor")
        B, N = indexes.shape
        if out is None:
            out = torch.empty((B, N), dtype=torch.int32, pin_memory=True)
        elif out.shape != (B, N) or out.dtype != torch.int32 or not out.is_pinned() or not out.is_contiguous():
            raise ValueError("out must be a contiguous pinned (B, N) int32 host tensor")
        dev, lib = self.device, self.lib
        offs, lens = _C.parse_merged(data, self.prefix, B)
        width = (int(lens.max().item()) + 3) // 4 + 1 if B else 1
        chunks = self._chunks(N)
        C = max((c for _, c in chunks), default=0)
        with torch.cuda.device(dev):
            comp = self.s_comp
            comp.wait_stream(torch.cuda.current_stream(dev))
            self.s_h2d.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(self.s_h2d):
                d_data = data.to(dev, non_blocking=True)
                d_off = offs.to(dev, non_blocking=True)
                d_len = lens.to(dev, non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(self.s_h2d)
            stream = torch.empty((B, width), dtype=torch.int32, device=dev)
            comp.wait_event(ready)
            if B:
                self._check(lib.tans_scatter_payloads(d_data.data_ptr(), d_off.data_ptr(), d_len.data_ptr(),
                                                      stream.data_ptr(), B, width, comp.cuda_stream), "parse")
            bufs = {}

            def chunk_bufs(sl, cn):  # (indexes, decoded symbols) as dense (B, cn) matrices
                key = (sl if cn == C else "short", cn)
                if key not in bufs:
                    bufs[key] = (torch.empty((B, cn), dtype=torch.int32, device=dev),
                                 torch.empty((B, cn), dtype=torch.int32, device=dev))
                return bufs[key]

            ev_in = [torch.cuda.Event() for _ in range(2)]
            ev_idx_free = [torch.cuda.Event() for _ in range(2)]
            ev_popped = [torch.cuda.Event() for _ in range(2)]
            ev_out_free = [torch.cuda.Event() for _ in range(2)]
            K, Wc = self.pop_cdfs.shape
            for j, (c0, cn) in enumerate(chunks):
                sl = j % 2
                ib, ob = chunk_bufs(sl, cn)
                if j >= 2:
                    self.s_h2d.wait_event(ev_idx_free[sl])
                _C.copy_columns(ib, 0, indexes, c0, cn, self.s_h2d.cuda_stream)
                ev_in[sl].record(self.s_h2d)
                comp.wait_event(ev_in[sl])
                if j >= 2:
                    comp.wait_event(ev_out_free[sl])
                ip, op = ib.data_ptr(), ob.data_ptr()
                rc = lib.tans_pop(self.v, self.lookup, 1, stream.data_ptr(), B, width, op, ip, cn,
                                  self.pop_cdfs.data_ptr(), K, Wc, self.sizes.data_ptr(), self.offsets.data_ptr(),
                                  self.fp, int(self.bypass), self.bp, self.pop_ws.data_ptr(), self.pop_ws.numel(),
                                  self.status.data_ptr(), comp.cuda_stream)
                self._check(rc, "pop")
                ev_idx_free[sl].record(comp)
                ev_popped[sl].record(comp)
                self.s_d2h.wait_event(ev_popped[sl])
                _C.copy_columns(out, c0, ob, 0, cn, self.s_d2h.cuda_stream)
                ev_out_free[sl].record(self.s_d2h)
            self.s_d2h.synchronize()
            del stream, d_data, bufs
        return out
