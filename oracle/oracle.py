"""Python face of the oracle: the CPU restatement of torch_ans's rANS path (TEST INFRASTRUCTURE).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference leg use this
module, and only as the oracle the results are compared with (or as the timed CPU reference); the product package
``torch_ans_b200`` never imports it.

* The coding loops live in ``oracle/rans_oracle.c`` (plain C, compiled here with gcc into
  ``oracle/_build/librans_oracle.so``) and are called through ctypes on numpy arrays.
* The op-level glue is restated here in numpy:
    - worst-case stream resize before a push      torch_ans/rans.hpp:105-124
    - default offsets                               torch_ans/rans.hpp:131-135, 242-246
    - stream <-> list-of-bytes conversion           torch_ans/rans.cpp:5-53
    - pmf -> quantised cdf (float32 arithmetic)     torch_ans/rans_cpu.cpp:326-385
    - inverse quantised cdf                         torch_ans/utils.py:170-184
    - container format merge / split               torch_ans/utils.py:47-101

Pinning: every function here is checked against golden vectors written by the compiled reference
(``tests/golden/make_golden.py`` -> ``tests/golden/*.npz``) and against the reference's own known
answers (``tests/torch_ans_test.py:54-67``, ``tests/test_utils.py:23-130`` of the reference).
"""
from __future__ import annotations

import ctypes
import io
import os
import struct
import subprocess
from typing import List, Optional, Sequence, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "rans_oracle.c")
LIB = os.path.join(HERE, "_build", "librans_oracle.so")

VARIANTS = {"rans64": 0, "rans32": 1, "rans32_16": 2}
STATE_BYTES = {"rans64": 8, "rans32": 4, "rans32_16": 4}
WORD_BYTES = {"rans64": 4, "rans32": 1, "rans32_16": 2}
LOOKUPS = {"search": 0, "invcdf": 1, "alias": 2}

ERR_BAD_INDEX = 1
ERR_BAD_VALUE = 2
ERR_OVERFLOW = 4
ERR_UNDERFLOW = 8
ERR_BAD_FREQ = 16
ERR_BAD_ESCAPE = 32

_lib = None


def build(force: bool = False) -> str:
    """Compile rans_oracle.c (gcc, OpenMP) unless the shared object is newer than the source."""
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        os.makedirs(os.path.dirname(LIB), exist_ok=True)
        tmp = LIB + f".tmp{os.getpid()}"
        subprocess.run(["gcc", "-O2", "-fPIC", "-shared", "-fopenmp", "-std=c11", "-o", tmp, SRC],
                       check=True)
        os.replace(tmp, LIB)
    return LIB


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB)
        P = ctypes.c_void_p
        i64, i32 = ctypes.c_int64, ctypes.c_int
        L.orc_init_stream.argtypes = [i32, P, i64, i64, i32]
        L.orc_init_stream.restype = None
        L.orc_push.argtypes = [i32, i32, i32, P, i64, i64, P, P, i64, P, i64, i64, P, P, i32, i32, i32, i32]
        L.orc_push.restype = ctypes.c_uint32
        L.orc_pop.argtypes = [i32, i32, i32, P, i64, i64, P, P, i64, P, i64, i64, P, P, i32, i32, i32, i32]
        L.orc_pop.restype = ctypes.c_uint32
        L.orc_alias_build.argtypes = [P, P, i64, i64, i32, i32, P, P]
        L.orc_alias_build.restype = ctypes.c_int64
        _lib = L
    return _lib


def _i32(a) -> np.ndarray:
    a = np.asarray(a)
    if a.dtype != np.int32:
        a = a.astype(np.int32)
    return np.ascontiguousarray(a)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def init_stream(variant: str, size: int, num_interleaves: int = 1, preallocate_size: int = 0) -> np.ndarray:
    """rans_init_stream, torch_ans/rans_cpu.cpp:22-41."""
    sb = STATE_BYTES[variant]
    width = 1 + preallocate_size // 4 + num_interleaves * ((sb + 3) // 4)
    s = np.zeros((size, width), dtype=np.int32)
    lib().orc_init_stream(VARIANTS[variant], _ptr(s), size, width, num_interleaves)
    return s


def resized_width(stream: np.ndarray, num_symbols: int, freq_precision: int, bypass_coding: bool) -> int:
    """Row width after the worst-case resize of rans_push, torch_ans/rans.hpp:105-124."""
    max_len = int(stream[:, 0].max()) if stream.shape[0] else 0
    safe = max_len + (num_symbols * freq_precision + 7) // 8
    if bypass_coding:
        safe += num_symbols * 4
    if safe < max_len:
        raise ValueError("Overflow!")
    return max(stream.shape[1], safe // 4 + 1)


def push(variant: str, stream: np.ndarray, symbols, indexes, cdfs, cdfs_sizes, offsets=None,
         freq_precision: int = 16, bypass_coding: bool = True, bypass_precision: int = 4,
         alias: bool = False, interleave: int = 1, threads: int = 1) -> Tuple[np.ndarray, int]:
    """rans_push (torch_ans/rans.hpp:84-217) on the CPU path; returns (new stream, error bits)."""
    symbols, indexes, cdfs, sizes = _i32(symbols), _i32(indexes), _i32(cdfs), _i32(cdfs_sizes)
    if symbols.ndim == 1:
        symbols = symbols.reshape(stream.shape[0], -1)
    if symbols.shape[0] != stream.shape[0]:
        raise ValueError("Symbols batch size mismatch!")
    if indexes.shape != symbols.shape:
        raise RuntimeError("indexes / symbols shape mismatch")
    offsets = np.zeros(cdfs.shape[0], np.int32) if offsets is None else _i32(offsets)
    B, N = symbols.shape
    W = resized_width(stream, N, freq_precision, bypass_coding)
    out = np.zeros((B, W), dtype=np.int32)
    out[:, : stream.shape[1]] = stream
    err = lib().orc_push(VARIANTS[variant], int(alias), interleave, _ptr(out), B, W, _ptr(symbols),
                         _ptr(indexes), N, _ptr(cdfs), cdfs.shape[0], cdfs.shape[1], _ptr(sizes),
                         _ptr(offsets), freq_precision, int(bypass_coding), bypass_precision, threads)
    return out, int(err)


def pop(variant: str, stream: np.ndarray, indexes, cdfs, cdfs_sizes, offsets=None,
        freq_precision: int = 16, bypass_coding: bool = True, bypass_precision: int = 4,
        lookup: str = "search", interleave: int = 1, threads: int = 1) -> Tuple[np.ndarray, int]:
    """rans_pop (torch_ans/rans.hpp:220-276) on the CPU path; mutates ``stream`` in place and
    returns (decoded int32 symbols shaped like indexes, error bits)."""
    assert stream.dtype == np.int32 and stream.flags.c_contiguous
    indexes, cdfs, sizes = _i32(indexes), _i32(cdfs), _i32(cdfs_sizes)
    shape = indexes.shape
    indexes = indexes.reshape(stream.shape[0], -1)
    offsets = np.zeros(cdfs.shape[0], np.int32) if offsets is None else _i32(offsets)
    B, N = indexes.shape
    out = np.zeros((B, N), dtype=np.int32)
    err = lib().orc_pop(VARIANTS[variant], LOOKUPS[lookup], interleave, _ptr(stream), B,
                        stream.shape[1], _ptr(out), _ptr(indexes), N, _ptr(cdfs), cdfs.shape[0],
                        cdfs.shape[1], _ptr(sizes), _ptr(offsets), freq_precision,
                        int(bypass_coding), bypass_precision, threads)
    return out.reshape(shape), int(err)


def alias_build_table(cdfs, cdfs_sizes, symbol_precision: int = 8, freq_precision: int = 16):
    """rans_alias_build_table (torch_ans/rans.cpp:56-95): returns (remap rows, table rows, ok rows)."""
    cdfs, sizes = _i32(cdfs), _i32(cdfs_sizes)
    K, Wc = cdfs.shape
    remap = np.zeros((K, Wc + (1 << freq_precision)), np.int32)
    table = np.zeros((K, Wc * 5), np.int32)
    ok = lib().orc_alias_build(_ptr(cdfs), _ptr(sizes), K, Wc, symbol_precision, freq_precision,
                               _ptr(remap), _ptr(table))
    return remap, table, int(ok)


def stream_to_byte_strings(stream: np.ndarray) -> List[bytes]:
    """rans_stream_to_byte_strings, torch_ans/rans.cpp:5-21."""
    s = np.ascontiguousarray(stream, dtype=np.int32)
    return [s[b, 1:].tobytes()[: int(s[b, 0])] for b in range(s.shape[0])]


def byte_strings_to_stream(byte_strings: Sequence[bytes]) -> np.ndarray:
    """rans_byte_strings_to_stream, torch_ans/rans.cpp:23-53."""
    max_len = max((len(b) for b in byte_strings), default=0)
    width = (max_len + 3) // 4 + 1
    s = np.zeros((len(byte_strings), width), np.int32)
    for b, bs in enumerate(byte_strings):
        s[b, 0] = len(bs)
        s[b, 1:].view(np.uint8)[: len(bs)] = np.frombuffer(bs, np.uint8)
    return s


def _len_format(num_bytes: int) -> str:
    """_get_bytes_format, torch_ans/utils.py:21-44."""
    return {1: "B", 2: "<H", 4: "<I", 8: "<L"}[num_bytes]


def merge_bytes(data: Sequence[bytes], num_bytes_length: int = 4, num_segments: Optional[int] = None) -> bytes:
    """merge_bytes, torch_ans/utils.py:47-72."""
    fmt = _len_format(num_bytes_length)
    out = io.BytesIO()
    for i, bs in enumerate(data):
        if num_segments is None or i < num_segments - 1:
            out.write(struct.pack(fmt, len(bs)))
        out.write(bs)
    return out.getvalue()


def split_merged_bytes(data: bytes, num_bytes_length: int = 4, num_segments: Optional[int] = None) -> List[bytes]:
    """split_merged_bytes, torch_ans/utils.py:74-101."""
    fmt = _len_format(num_bytes_length)
    pos, out = 0, []
    while pos < len(data):
        if num_segments is not None and len(out) >= num_segments - 1:
            out.append(data[pos:])
            pos = len(data)
        else:
            (n,) = struct.unpack(fmt, data[pos:pos + num_bytes_length])
            pos += num_bytes_length
            out.append(data[pos:pos + n])
            pos += n
    if num_segments is not None:
        out += [b""] * (num_segments - len(out))
    return out


def pmf_to_quantized_cdf(pmf, precision: int = 16) -> np.ndarray:
    """rans_pmf_to_quantized_cdf_cpu, torch_ans/rans_cpu.cpp:326-385, in float32/int32 arithmetic:
    round-half-even of pmf*2^p, int32 (wrapping) rescale by 2^p, float32 true division by the row
    total, truncation, cumsum, last entry forced to 2^p, then the zero-frequency repair that
    borrows one count from the smallest frequency > 1 (first such, scanning up)."""
    pmf = np.asarray(pmf, dtype=np.float32)
    one_d = pmf.ndim == 1
    p2 = pmf[None, :] if one_d else pmf
    B, N = p2.shape
    freq = np.rint(p2 * np.float32(1 << precision)).astype(np.int32)
    cdf = np.zeros((B, N + 1), np.int32)
    cdf[:, 1:] = freq
    total = cdf.astype(np.int64).sum(1, keepdims=True).astype(np.int32)
    total = np.where(total == 0, np.int32(1), total)
    scaled = (cdf.astype(np.int64) * (1 << precision)).astype(np.int32)
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        cdf = (scaled.astype(np.float32) / total.astype(np.float32)).astype(np.int32)
    cdf = np.cumsum(cdf.astype(np.int64), axis=1).astype(np.int32)
    cdf[:, N] = 1 << precision
    for b in range(B):
        row = cdf[b]
        for i in range(N):
            if row[i] == row[i + 1]:
                f = row[1:] - row[:-1]
                cand = np.nonzero(f > 1)[0]
                if cand.size == 0:
                    raise RuntimeError("No symbol to steal frequency from")
                best = int(cand[np.argmin(f[cand])])
                if best < i:
                    row[best + 1:i + 1] -= 1
                else:
                    row[i + 1:best + 1] += 1
    return cdf[0] if one_d else cdf


def inverse_quantized_cdf(quantized_cdf, freq_precision: int = 16) -> np.ndarray:
    """inverse_quantized_cdf, torch_ans/utils.py:170-184: inv[r] = #{j : cdf[j] <= r} - 1."""
    cdf = np.asarray(quantized_cdf)
    two = cdf.reshape(-1, cdf.shape[-1])
    r = np.arange(1 << freq_precision)
    out = np.stack([np.searchsorted(np.sort(row), r, side="right") - 1 for row in two]).astype(cdf.dtype)
    return out.reshape(cdf.shape[:-1] + (1 << freq_precision,))
