"""High-level coder API of torch_ans_b200: a drop-in for torch_ans.utils (torch_ans/utils.py).

Same names, arguments, defaults and byte formats as the reference:
  * ``merge_bytes`` / ``split_merged_bytes``: the container of the concatenated bitstream, a
    little-endian length prefix per segment then its bytes, the last segment unprefixed when
    ``num_segments`` is given (utils.py:47-101);
  * ``pmf_to_quantized_cdf_batched``, ``inverse_quantized_cdf`` (utils.py:103-184);
  * ``TorchEntropyCoderBaseInterface`` / ``TorchANSInterface`` (utils.py:187-966): encode /
    decode with per-symbol table indexes or per-element frequencies, LIFO caching
    (``encode(..., cache=True)`` then ``encode_flush``), the CompressAI-like byte API.

Differences, all because coding runs on the GPU here:
  * ``device=None`` means the current CUDA device (the reference leaves tensors on the CPU);
  * ``flush`` / ``encode_with_*`` assemble the container on the device
    (``_C.stream_to_merged_bytes``), producing the same bytes as
    ``merge_bytes(rans_stream_to_byte_strings(stream))``;
  * the inverse-cdf and alias-table decoders the reference hard-wires off (utils.py:612-613) can
    be switched on with ``use_inverse_cdf=True`` / ``use_alias_table=True``.
"""
from __future__ import annotations

import io
import struct
from typing import List, Optional

import torch

from . import _C
from ._C import (rans_alias_build_table, rans_byte_strings_to_stream, rans_pmf_to_quantized_cdf,
                 rans_stream_to_byte_strings)

__all__ = ["merge_bytes", "split_merged_bytes", "pmf_to_quantized_cdf_batched", "inverse_quantized_cdf",
           "TorchEntropyCoderBaseInterface", "TorchANSInterface"]


def _get_bytes_format(num_bytes=4):
    """struct format of a segment-length prefix of ``num_bytes`` bytes (utils.py:21-44)."""
    formats = {1: "B", 2: "<H", 4: "<I", 8: "<L"}
    if num_bytes not in formats:
        raise ValueError("")
    return formats[num_bytes]


def merge_bytes(data: List[bytes], num_bytes_length=4, num_segments=None) -> bytes:
    """Concatenate byte strings, each preceded by its length (utils.py:47-72).  With
    ``num_segments`` the last of the ``num_segments`` segments carries no length prefix."""
    fmt = _get_bytes_format(num_bytes_length)
    out = io.BytesIO()
    for i, segment in enumerate(data):
        if num_segments is not None:
            assert i < num_segments, "Number of segments exceed predefined {}".format(num_segments)
            if i < num_segments - 1:
                out.write(struct.pack(fmt, len(segment)))
        else:
            out.write(struct.pack(fmt, len(segment)))
        out.write(segment)
    return out.getvalue()


def split_merged_bytes(data: bytes, num_bytes_length=4, num_segments=None) -> List[bytes]:
    """Inverse of merge_bytes (utils.py:74-101); pads with empty segments up to num_segments."""
    fmt = _get_bytes_format(num_bytes_length)
    pos, segments = 0, []
    while pos < len(data):
        if num_segments is not None and len(segments) >= num_segments - 1:
            segments.append(data[pos:])
            pos = len(data)
            continue
        (length,) = struct.unpack(fmt, data[pos:pos + num_bytes_length])
        pos += num_bytes_length
        segments.append(data[pos:pos + length])
        pos += length
    if num_segments is not None:
        segments.extend(b"" for _ in range(num_segments - len(segments)))
    return segments


def pmf_to_quantized_cdf_batched(pmf: torch.Tensor, precision=16, add_tail=True, tail_mass=1e-10, normalize=True):
    """Batched pmf -> quantised cdf without the borrow repair (utils.py:103-167): every symbol
    gets +1 before scaling, rows whose total exceeds 2^precision are rescaled until they fit."""
    top = 1 << precision
    assert pmf.shape[-1] * 2 < top
    if add_tail:
        pmf = torch.cat([pmf.clone(), torch.zeros(pmf.shape[0], 1).type_as(pmf) + tail_mass], dim=1)
    if normalize:
        pmf = pmf / pmf.sum(1, keepdim=True)
    lifted = pmf * top + 1.0
    step = pmf.shape[-1] // 2
    counts = (lifted * top / (lifted.sum(1, keepdim=True) + step)).round()
    row_total = counts.sum(dim=1, keepdim=True)
    scale = row_total.clone()
    while (row_total > top).any():
        scale[row_total > top] += step
        counts = (counts * top / scale).round()
        row_total = counts.sum(dim=1, keepdim=True)
    cum = counts.cumsum(dim=1)
    cdf = torch.cat([torch.zeros(pmf.shape[0], 1).type_as(cum), cum[:, :-1],
                     torch.zeros(pmf.shape[0], 1).type_as(cum) + top], dim=1)
    return cdf.int()


def inverse_quantized_cdf(quantized_cdf, freq_precision=16):
    """inv[..., r] = #{j : cdf[..., j] <= r} - 1 for r < 2^freq_precision (utils.py:170-184),
    computed by sorting each row and a right-sided searchsorted, so it needs O(2^fp) memory per
    row instead of O(2^fp * row length)."""
    rows = quantized_cdf.reshape(-1, quantized_cdf.shape[-1])
    r = torch.arange(1 << freq_precision, device=rows.device, dtype=torch.int64)
    srt = rows.to(torch.int64).sort(dim=-1).values
    inv = torch.searchsorted(srt, r.unsqueeze(0).expand(srt.shape[0], -1).contiguous(), right=True) - 1
    return inv.to(quantized_cdf.dtype).reshape(quantized_cdf.shape[:-1] + (1 << freq_precision,))


class TorchEntropyCoderBaseInterface(object):
    """Entropy-coder base (utils.py:187-580): caching, tensor placement, encode/decode patterns."""

    def __init__(self, symbol_precision: int = 8, freq_precision: int = 16, mode="encdec", dtype=torch.int32,
                 device=None, **kwargs) -> None:
        self.symbol_precision = symbol_precision
        self.freq_precision = freq_precision
        self.mode = mode
        if self.mode in ("encoder", "encdec"):
            self._init_encoder(**kwargs)
        if self.mode in ("decoder", "encdec"):
            self._init_decoder(**kwargs)
        self._set_dtype(dtype)
        self._set_device(device)

    def _init_encoder(self, **kwargs):
        self._encode_queue = []

    def _init_decoder(self, **kwargs):
        self._encoded_stream = None

    def _init_tensor(self, tensor: torch.Tensor) -> torch.Tensor:
        return tensor.to(dtype=self.dtype, device=self.device)

    def _init_stream(self, **kwargs) -> torch.Tensor:
        return torch.zeros(1, dtype=self.dtype, device=self.device)

    def _set_dtype(self, dtype: torch.dtype) -> None:
        self.dtype = dtype

    def _set_device(self, device) -> None:
        # coding runs on CUDA only: "no device" means the current CUDA device
        self.device = torch.device(device) if device is not None else torch.device("cuda")

    def init_params(self, freqs: torch.Tensor, num_freqs: torch.Tensor, offsets: torch.Tensor) -> None:
        self.freqs = self._init_tensor(freqs)
        self.num_freqs = self._init_tensor(num_freqs)
        self.offsets = self._init_tensor(offsets)

    def _encode_func(self, symbols, stream, **kwargs) -> torch.Tensor:
        raise NotImplementedError()

    def _decode_func(self, stream, **kwargs) -> torch.Tensor:
        raise NotImplementedError()

    def _cache_concat(self, prev: torch.Tensor, new: torch.Tensor):
        return torch.stack([prev, new], dim=0)

    def reset_cache(self) -> None:
        self._encode_queue = []

    def encode(self, symbols: torch.Tensor, dist_indexes: Optional[torch.Tensor] = None,
               dist_freqs: Optional[torch.Tensor] = None, dist_num_freqs: Optional[torch.Tensor] = None,
               dist_min: Optional[torch.Tensor] = None, cache=False, **kwargs) -> Optional[torch.Tensor]:
        """Encode with per-symbol table indexes or per-element frequencies (utils.py:328-376);
        with cache=True the call is queued for encode_flush."""
        if dist_indexes is not None:
            assert symbols.shape == dist_indexes.shape, \
                "For encode_with_indexes pattern, symbols and dist_indexes should have the same shape"
            dist_indexes = self._init_tensor(dist_indexes)
        elif dist_freqs is not None:
            assert symbols.shape == dist_freqs.shape[:-1], \
                "For encode_with_freqs pattern, symbols.shape should match dist_freqs.shape[:-1]"
            dist_freqs = self._init_tensor(dist_freqs)
            dist_num_freqs = self._init_tensor(dist_num_freqs if dist_num_freqs is not None
                                               else torch.zeros_like(symbols) + dist_freqs.shape[-1])
            dist_min = self._init_tensor(dist_min if dist_min is not None else torch.zeros_like(symbols))
        else:
            raise NotImplementedError("Unsupported encoding pattern. Please provide either dist_indexes or dist_freqs.")
        symbols = self._init_tensor(symbols)
        item = dict(symbols=symbols, dist_indexes=dist_indexes, dist_freqs=dist_freqs,
                    dist_num_freqs=dist_num_freqs, dist_min=dist_min, **kwargs)
        if cache:
            self._encode_queue.append(item)
            return None
        return self._encode_func(stream=self._init_stream(), **item)

    def encode_flush(self, **kwargs) -> Optional[torch.Tensor]:
        """Encode the queued items last-first (rANS is LIFO) onto one stream (utils.py:378-393)."""
        stream = None
        for item in reversed(self._encode_queue):
            stream = self._encode_func(stream=stream, **item, **kwargs)
        return stream

    def decode(self, stream: Optional[torch.Tensor], dist_indexes: Optional[torch.Tensor] = None,
               dist_freqs: Optional[torch.Tensor] = None, dist_num_freqs: Optional[torch.Tensor] = None,
               dist_min: Optional[torch.Tensor] = None, **kwargs) -> torch.Tensor:
        """Decode (utils.py:403-439); the stream tensor is consumed in place, so consecutive
        calls decode consecutive items."""
        if stream is None:
            stream = self._encoded_stream
        if dist_indexes is not None:
            dist_indexes = self._init_tensor(dist_indexes)
        elif dist_freqs is not None:
            dist_freqs = self._init_tensor(dist_freqs)
            dist_num_freqs = self._init_tensor(dist_num_freqs if dist_num_freqs is not None
                                               else torch.zeros_like(dist_freqs[..., 0]) + dist_freqs.shape[-1])
            dist_min = self._init_tensor(dist_min if dist_min is not None else torch.zeros_like(dist_freqs[..., 0]))
        else:
            raise NotImplementedError("Unsupported decoding pattern. Please provide either dist_indexes or dist_freqs.")
        return self._decode_func(stream, dist_indexes=dist_indexes, dist_freqs=dist_freqs,
                                 dist_num_freqs=dist_num_freqs, dist_min=dist_min, **kwargs)

    def encode_with_indexes(self, symbols, indexes, cache=False, **kwargs):
        raise NotImplementedError()

    def decode_with_indexes(self, encoded, indexes, **kwargs):
        raise NotImplementedError()

    def flush(self, **kwargs) -> bytes:
        stream = self.encode_flush(**kwargs)
        if stream is None:
            return b""
        return self._stream_to_bytes(stream)

    def _stream_to_bytes(self, stream: torch.Tensor) -> bytes:
        return merge_bytes(rans_stream_to_byte_strings(stream), num_bytes_length=self.num_bytes_code_length,
                           num_segments=self.num_parallel_states)

    def set_stream(self, encoded) -> None:
        self.encoded = encoded

    def decode_stream(self, indexes, **kwargs):
        raise NotImplementedError()

    def encode_with_freqs(self, symbols, freqs, num_freqs, offsets, cache=False, **kwargs):
        raise NotImplementedError()

    def decode_with_freqs(self, encoded, freqs, num_freqs, offsets, **kwargs):
        raise NotImplementedError()

    def decode_stream_with_freqs(self, freqs, num_freqs, offsets, **kwargs):
        raise NotImplementedError()


class TorchANSInterface(TorchEntropyCoderBaseInterface):
    """rANS coder (utils.py:583-966).  ``impl`` picks the variant by prefix exactly as the
    reference does: "rans64*" -> rans64 (freq precision <= 31), "rans32*" / "rans_byte*" -> rans32
    with byte words (<= 23; this includes "rans32_16", as in the reference)."""

    def __init__(self, impl="rans64", bypass_coding: bool = True, bypass_precision: int = 4,
                 num_parallel_states=None, num_bytes_code_length=4, use_inverse_cdf: bool = False,
                 use_alias_table: bool = False, **kwargs) -> None:
        self.impl = impl
        self.bypass_coding = bypass_coding
        self.bypass_precision = bypass_precision
        self.num_parallel_states = num_parallel_states
        self.num_bytes_code_length = num_bytes_code_length
        super().__init__(**kwargs)
        self.impl_use_inverse_cdf = use_inverse_cdf
        self.impl_use_alias_table = use_alias_table
        if self.impl.startswith("rans64"):
            prefix, cap = "rans64", 31
        elif self.impl.startswith("rans32") or self.impl.startswith("rans_byte"):
            prefix, cap = "rans32", 23
        else:
            raise NotImplementedError(f"Unknown impl {self.impl}")
        self.freq_precision = min(self.freq_precision, cap)
        self.ans_init_func = getattr(_C, f"{prefix}_init_stream")
        self.ans_encode_func = getattr(_C, f"{prefix}_alias_push" if use_alias_table else f"{prefix}_push")
        if use_alias_table:
            self.ans_decode_func = getattr(_C, f"{prefix}_alias_pop")
        elif use_inverse_cdf:
            self.ans_decode_func = getattr(_C, f"{prefix}_invcdf_pop")
        else:
            self.ans_decode_func = getattr(_C, f"{prefix}_pop")

    def _init_stream(self, num_parallel_states=None, **kwargs) -> torch.Tensor:
        n = num_parallel_states if num_parallel_states is not None else self.num_parallel_states
        n = int(n) if n is not None else 1
        if self.device.type == "cuda":  # made on the device: the first push needs no device read
            return self.ans_init_func(n, device=str(self.device))
        return self._init_tensor(self.ans_init_func(n))

    def init_params(self, freqs, num_freqs, offsets) -> None:
        """Quantise frequency rows into cdf tables (utils.py:641-673): with escape coding an extra
        symbol of mass 1e-10 is appended and each table's cdf_size is num_freqs + 2, else + 1."""
        if self.bypass_coding:
            freqs = torch.cat([freqs.clone(), torch.zeros_like(freqs[..., :1]) + 1e-10], dim=-1)
        pmf = freqs.float() / freqs.sum(-1, keepdim=True)
        cdfs = rans_pmf_to_quantized_cdf(pmf.to(device=self.device), self.freq_precision)
        cdfs_sizes = num_freqs + (2 if self.bypass_coding else 1)
        self._set_tables(cdfs, cdfs_sizes, offsets)

    def _set_tables(self, cdfs, cdfs_sizes, offsets):
        if self.impl_use_alias_table:
            remap, table = rans_alias_build_table(cdfs, cdfs_sizes, symbol_precision=self.symbol_precision,
                                                  freq_precision=self.freq_precision)
            cdfs = remap
            self.cdfs_with_alias_table = self._init_tensor(table).contiguous()
        elif self.impl_use_inverse_cdf:
            cdfs = torch.cat([cdfs, inverse_quantized_cdf(cdfs, freq_precision=self.freq_precision)], dim=-1)
        self.cdfs = self._init_tensor(cdfs).contiguous()
        self.cdfs_sizes = self._init_tensor(cdfs_sizes).contiguous()
        self.offsets = self._init_tensor(offsets).contiguous()

    def set_cdfs(self, cdfs: torch.Tensor, cdfs_sizes: torch.Tensor, offsets: torch.Tensor) -> None:
        self.cdfs = self._init_tensor(cdfs).contiguous()
        self.cdfs_sizes = self._init_tensor(cdfs_sizes).contiguous()
        self.offsets = self._init_tensor(offsets).contiguous()

    def _coding_kwargs(self):
        return dict(freq_precision=self.freq_precision, bypass_coding=self.bypass_coding,
                    bypass_precision=self.bypass_precision)

    def _encode_func(self, symbols, stream: Optional[torch.Tensor] = None, dist_indexes=None, dist_freqs=None,
                     dist_num_freqs=None, dist_min=None, **kwargs) -> torch.Tensor:
        if stream is None:
            n = symbols.size(0) if self.num_parallel_states is None else self.num_parallel_states
            stream = self._init_stream(num_parallel_states=n)
        else:
            n = stream.size(0)
        if dist_indexes is None and dist_freqs is not None:
            self.init_params(dist_freqs.reshape(-1, dist_freqs.shape[-1]), dist_num_freqs.reshape(-1),
                             dist_min.reshape(-1))
            dist_indexes = torch.arange(symbols.numel(), dtype=self.dtype, device=stream.device).reshape_as(symbols)
        elif dist_indexes is None:
            raise NotImplementedError("Unsupported encoding pattern. Please provide either dist_indexes or dist_freqs.")
        self.ans_encode_func(stream, symbols.reshape(n, -1).contiguous(), dist_indexes.reshape(n, -1).contiguous(),
                             self.cdfs, self.cdfs_sizes, self.offsets, **self._coding_kwargs())
        return stream

    def _decode_func(self, stream, dist_indexes=None, dist_freqs=None, dist_num_freqs=None, dist_min=None,
                     **kwargs) -> torch.Tensor:
        n = stream.size(0) if self.num_parallel_states is None else self.num_parallel_states
        if dist_indexes is not None:
            shape_like = dist_indexes
        elif dist_freqs is not None:
            self.init_params(dist_freqs.reshape(-1, dist_freqs.shape[-1]), dist_num_freqs.reshape(-1),
                             dist_min.reshape(-1))
            dist_indexes = torch.arange(dist_num_freqs.numel(), dtype=self.dtype,
                                        device=stream.device).reshape_as(dist_num_freqs)
            shape_like = dist_num_freqs
        else:
            raise NotImplementedError("Unsupported decoding pattern. Please provide either dist_indexes or dist_freqs.")
        cdfs = self.cdfs_with_alias_table if self.impl_use_alias_table else self.cdfs
        decoded = self.ans_decode_func(stream, dist_indexes.reshape(n, -1).contiguous(), cdfs, self.cdfs_sizes,
                                       self.offsets, **self._coding_kwargs())
        return decoded.reshape_as(shape_like).to(device=stream.device)

    def _stream_to_bytes(self, stream: torch.Tensor) -> bytes:
        if stream.is_cuda:
            return _C.stream_to_merged_bytes(stream, self.num_bytes_code_length, self.num_parallel_states)
        return super()._stream_to_bytes(stream)

    def _bytes_to_stream(self, encoded) -> torch.Tensor:
        segments = split_merged_bytes(encoded, num_bytes_length=self.num_bytes_code_length,
                                      num_segments=self.num_parallel_states)
        return self._init_tensor(rans_byte_strings_to_stream(segments))

    def encode_with_indexes(self, symbols: torch.Tensor, indexes: torch.Tensor, cache=False, **kwargs):
        stream = self.encode(symbols, dist_indexes=indexes, cache=cache, **kwargs)
        return None if cache else self._stream_to_bytes(stream)

    def decode_with_indexes(self, encoded, indexes: torch.Tensor, **kwargs) -> torch.Tensor:
        return self.decode(stream=self._bytes_to_stream(encoded), dist_indexes=indexes, **kwargs)

    def set_stream(self, encoded) -> None:
        self._encoded_stream = self._bytes_to_stream(encoded)

    def decode_stream(self, indexes: torch.Tensor, **kwargs) -> torch.Tensor:
        return self.decode(stream=self._encoded_stream, dist_indexes=indexes, **kwargs)

    def encode_with_freqs(self, symbols, freqs, num_freqs, offsets, cache=False, **kwargs):
        stream = self.encode(symbols, dist_freqs=freqs, dist_num_freqs=num_freqs, dist_min=offsets, cache=cache,
                             **kwargs)
        return None if cache else self._stream_to_bytes(stream)

    def decode_with_freqs(self, encoded, freqs, num_freqs, offsets, **kwargs) -> torch.Tensor:
        return self.decode(stream=self._bytes_to_stream(encoded), dist_freqs=freqs, dist_num_freqs=num_freqs,
                           dist_min=offsets, **kwargs)

    def decode_stream_with_freqs(self, freqs, num_freqs, offsets, **kwargs) -> torch.Tensor:
        return self.decode(stream=self._encoded_stream, dist_freqs=freqs, dist_num_freqs=num_freqs,
                           dist_min=offsets, **kwargs)
