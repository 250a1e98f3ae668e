"""Seeded synthetic inputs with the shapes of the benchmark configurations.

Five configurations of the rANS coding path (tables, per-symbol table indexes, symbols):

1. ``laplace64``  -- rans64, 64 streams x 65,536 symbols, 64 discretised zero-mean Laplace tables
   (alphabet 256, support -128..127 shifted to 0..255, scale log-uniform in [0.1, 20]),
   fp 16, no escape coding, search decode.  Seed 0.
2. ``gaussian_latent`` -- rans32 (byte words), a CompressAI GaussianConditional-style latent
   16x192x16x16: y ~ N(mu, sigma), mu ~ U(-5, 5), sigma log-uniform in [0.11, 64]; 64 scale
   tables log-spaced in [0.11, 256], index = first table scale >= sigma; table k covers
   [-t_k, t_k], t_k = ceil(scale_k * Phi^-1(1 - 1e-9/2)), plus the escape slot; offsets -t_k;
   symbols round(y - mu) clamped to the table (``clamp=False`` exercises escape coding); one
   stream per batch item (16 x 49,152); fp 16, escape precision 4.  Seed 1.
3. ``zipf_alias`` -- rans32_16, 1,024 streams x 1,048,576 symbols over one Zipf(1.1) table of
   4,096 symbols quantised to 2^15, alias tables (symbol precision 12); no escape coding.  Seed 2.
4. ``mixture_invcdf`` -- rans64 push + inverse-cdf pop, 8,192 streams x 262,144 symbols (2^31),
   256 tables of a 2-Gaussian mixture over 0..1023 (means U(0,1023), sigma log-uniform [1,200],
   weight U(0.1, 0.9)), rows [cdf | inverse cdf (2^16)], fp 16, no escape coding.  Seed 3.
5. ``ragged_adaptive`` -- rans32 with a 33-entry cdf row per symbol (softmax of N(0, 2^2) logits
   over 32 symbols), 4,096 streams with lognormal lengths (mu = ln 32768, sigma = 1) clamped to
   [1024, 524288].  Seed 4.

Tables are quantised with an exact integer rule: every symbol gets 1, the remaining 2^fp - A
counts are split by largest remainder of p * (2^fp - A) (float64, ties by index).  Symbols are
drawn from the quantised pmf itself (inverse-cdf sampling of a uniform 2^fp draw), so every
symbol is codable.  Large arrays are sampled on the target device; ``scale`` < 1 shrinks the
stream count (and ``length_scale`` the stream length) for tests.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, Optional

import torch


@dataclass
class Workload:
    name: str
    variant: str
    fp: int
    bypass: bool
    bp: int
    push_op: str                # _C op name used to encode
    pop_op: str                 # _C op name used to decode
    symbols: torch.Tensor       # (B, N) int32
    indexes: torch.Tensor       # (B, N) int32
    cdfs: torch.Tensor          # (K, W) int32 plain cdf rows
    cdfs_sizes: torch.Tensor    # (K,) int32
    offsets: torch.Tensor       # (K,) int32
    push_cdfs: Optional[torch.Tensor] = None  # rows the push reads (alias remap) if not cdfs
    pop_cdfs: Optional[torch.Tensor] = None   # rows the pop reads (alias / inverse) if not cdfs
    lookup: str = "search"
    extra: Dict[str, object] = field(default_factory=dict)

    @property
    def num_symbols(self) -> int:
        return self.symbols.numel()

    def tables_for_push(self):
        return self.push_cdfs if self.push_cdfs is not None else self.cdfs

    def tables_for_pop(self):
        return self.pop_cdfs if self.pop_cdfs is not None else self.cdfs


def quantize_pmf(p: torch.Tensor, fp: int) -> torch.Tensor:
    """Exact integer quantiser: rows of p (float64, >= 0) -> cdf rows (int64) summing to 2^fp
    with every frequency >= 1."""
    p = p.to(torch.float64)
    p = p / p.sum(-1, keepdim=True)
    A = p.shape[-1]
    extra = (1 << fp) - A
    assert extra >= 0, "alphabet larger than 2^fp"
    want = p * extra
    base = torch.floor(want).to(torch.int64)
    rem = extra - base.sum(-1)
    frac = want - base
    order = torch.argsort(frac, dim=-1, descending=True, stable=True)
    ranks = torch.empty_like(order)
    ranks.scatter_(-1, order, torch.arange(A, device=p.device).expand_as(order))
    base = base + (ranks < rem.unsqueeze(-1)).to(torch.int64)
    freq = base + 1
    cdf = torch.zeros(p.shape[:-1] + (A + 1,), dtype=torch.int64, device=p.device)
    cdf[..., 1:] = torch.cumsum(freq, -1)
    assert bool((cdf[..., -1] == (1 << fp)).all())
    return cdf


def inverse_rows(cdf: torch.Tensor, fp: int) -> torch.Tensor:
    """inv[r] = largest s with cdf[s] <= r, r < 2^fp (cdf rows sorted)."""
    r = torch.arange(1 << fp, device=cdf.device, dtype=torch.int64)
    c = cdf.to(torch.int64)
    return (torch.searchsorted(c, r.unsqueeze(0).expand(c.shape[0], -1).contiguous(), right=True) - 1).to(torch.int32)


def _sample(cdf_rows: torch.Tensor, inv: torch.Tensor, indexes: torch.Tensor, fp: int, gen) -> torch.Tensor:
    """symbol = inv[index, u], u uniform on [0, 2^fp): an exact draw from the quantised pmf."""
    u = torch.randint(0, 1 << fp, indexes.shape, generator=gen, device=indexes.device, dtype=torch.int64)
    flat = inv.reshape(-1)
    return flat[indexes.to(torch.int64) * (1 << fp) + u].to(torch.int32)


def _gen(device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def laplace64(device="cuda", scale: float = 1.0, length_scale: float = 1.0, seed: int = 0) -> Workload:
    fp, K, A = 16, 64, 256
    B, N = max(1, int(64 * scale)), max(1, int(65536 * length_scale))
    g = _gen("cpu", seed)
    s = torch.exp(torch.empty(K, dtype=torch.float64).uniform_(math.log(0.1), math.log(20.0), generator=g))
    x = torch.arange(-128, 128, dtype=torch.float64)
    # discretised Laplace: F(x + 1/2) - F(x - 1/2), tails folded into the end symbols
    def F(t):
        return torch.where(t < 0, 0.5 * torch.exp(t / s[:, None]), 1 - 0.5 * torch.exp(-t / s[:, None]))
    p = F(x + 0.5) - F(x - 0.5)
    p[:, :1] += F(torch.full((1,), -128.5, dtype=torch.float64))
    p[:, -1:] += 1 - F(torch.full((1,), 127.5, dtype=torch.float64))
    cdf = quantize_pmf(p, fp).to(torch.int32)
    inv = inverse_rows(cdf, fp)
    gd = _gen(device, seed)
    idx = torch.randint(0, K, (B, N), generator=gd, device=device, dtype=torch.int32)
    sym = _sample(cdf.to(device), inv.to(device), idx, fp, gd)
    return Workload("laplace64", "rans64", fp, False, 4, "rans64_push", "rans64_pop", sym, idx, cdf.to(device),
                    torch.full((K,), A + 1, dtype=torch.int32, device=device),
                    torch.zeros(K, dtype=torch.int32, device=device))


def gaussian_latent(device="cuda", scale: float = 1.0, clamp: bool = True, seed: int = 1,
                    outliers: float = 0.0) -> Workload:
    """``outliers``: fraction of symbols replaced by values 1..3,000 beyond their table's tail (either
    side), so that escape coding runs on these tables (without it a value past the 1e-9 tail is
    all but absent)."""
    fp, K = 16, 64
    nb = max(1, int(16 * scale))
    g = _gen("cpu", seed)
    shape = (nb, 192, 16, 16)
    mu = torch.empty(shape, dtype=torch.float64).uniform_(-5, 5, generator=g)
    sigma = torch.exp(torch.empty(shape, dtype=torch.float64).uniform_(math.log(0.11), math.log(64.0), generator=g))
    y = mu + sigma * torch.randn(shape, dtype=torch.float64, generator=g)
    scales = torch.exp(torch.linspace(math.log(0.11), math.log(256.0), K, dtype=torch.float64))
    idx = torch.searchsorted(scales, sigma.reshape(-1), right=False).clamp(max=K - 1).reshape(shape)
    z = math.sqrt(2.0) * torch.special.erfinv(torch.tensor(1 - 1e-9, dtype=torch.float64)).item()  # Phi^-1(1 - 1e-9/2)
    tails = torch.ceil(scales * z).to(torch.int64)
    width = int(2 * tails.max().item() + 3)
    cdfs = torch.zeros(K, width, dtype=torch.int32)
    normal = torch.distributions.Normal(torch.tensor(0.0, dtype=torch.float64), torch.tensor(1.0, dtype=torch.float64))
    for k in range(K):
        t = int(tails[k])
        v = torch.arange(-t, t + 1, dtype=torch.float64)
        p = normal.cdf((v + 0.5) / scales[k]) - normal.cdf((v - 0.5) / scales[k])
        p = torch.cat([p, torch.tensor([1e-9], dtype=torch.float64)])  # escape slot
        row = quantize_pmf(p[None], fp)[0]
        cdfs[k, : row.numel()] = row.to(torch.int32)
    sizes = (2 * tails + 3).to(torch.int32)
    offsets = (-tails).to(torch.int32)
    sym = torch.round(y - mu).to(torch.int64)
    if clamp:
        t_of = tails[idx]
        sym = torch.maximum(torch.minimum(sym, t_of), -t_of)
    if outliers > 0:
        pick = torch.rand(shape, dtype=torch.float64, generator=g) < outliers
        beyond = torch.randint(1, 3001, shape, generator=g, dtype=torch.int64)
        side = torch.where(torch.rand(shape, dtype=torch.float64, generator=g) < 0.5, -1, 1)
        sym = torch.where(pick, side * (tails[idx] + beyond), sym)
    B = nb
    sym = sym.reshape(B, -1).to(torch.int32)
    idx = idx.reshape(B, -1).to(torch.int32)
    return Workload("gaussian_latent", "rans32", fp, True, 4, "rans32_push", "rans32_pop", sym.to(device),
                    idx.to(device), cdfs.to(device), sizes.to(device), offsets.to(device),
                    extra={"clamp": clamp})


def zipf_alias(device="cuda", scale: float = 1.0, length_scale: float = 1.0, seed: int = 2, alias: bool = True,
               alias_builder=None) -> Workload:
    """``alias_builder``: the ``rans_alias_build_table(cdfs, cdfs_sizes, symbol_precision,
    freq_precision)`` that makes the alias tables (CPU tensors in, CPU tensors out); by default
    this library's.  The reference CPU leg of the benchmark passes the reference's own."""
    fp, A = 15, 4096
    B, N = max(1, int(1024 * scale)), max(1, int(1048576 * length_scale))
    p = 1.0 / torch.arange(1, A + 1, dtype=torch.float64) ** 1.1
    cdf = quantize_pmf(p[None], fp).to(torch.int32)
    sizes = torch.tensor([A + 1], dtype=torch.int32)
    inv = inverse_rows(cdf, fp)
    gd = _gen(device, seed)
    idx = torch.zeros((B, N), dtype=torch.int32, device=device)
    sym = _sample(cdf.to(device), inv.to(device), idx, fp, gd)
    if alias_builder is None:
        from torch_ans_b200 import _C
        alias_builder = _C.rans_alias_build_table
    remap, table = alias_builder(cdf, sizes, symbol_precision=12, freq_precision=fp)
    w = Workload("zipf_alias", "rans32_16", fp, False, 4,
                 "rans32_16_alias_push" if alias else "rans32_16_push",
                 "rans32_16_alias_pop" if alias else "rans32_16_pop", sym, idx, cdf.to(device),
                 sizes.to(device), torch.zeros(1, dtype=torch.int32, device=device),
                 push_cdfs=remap.to(device) if alias else None, pop_cdfs=table.to(device) if alias else None,
                 lookup="alias" if alias else "search")
    return w


def mixture_invcdf(device="cuda", scale: float = 1.0, length_scale: float = 1.0, seed: int = 3) -> Workload:
    fp, K, A = 16, 256, 1024
    B, N = max(1, int(8192 * scale)), max(1, int(262144 * length_scale))
    g = _gen("cpu", seed)
    means = torch.empty(K, 2, dtype=torch.float64).uniform_(0, A - 1, generator=g)
    sig = torch.exp(torch.empty(K, 2, dtype=torch.float64).uniform_(0.0, math.log(200.0), generator=g))
    wgt = torch.empty(K, dtype=torch.float64).uniform_(0.1, 0.9, generator=g)
    x = torch.arange(A, dtype=torch.float64)
    normal = torch.distributions.Normal(torch.tensor(0.0, dtype=torch.float64), torch.tensor(1.0, dtype=torch.float64))

    def comp(j):
        return normal.cdf((x[None] + 0.5 - means[:, j:j + 1]) / sig[:, j:j + 1]) - \
            normal.cdf((x[None] - 0.5 - means[:, j:j + 1]) / sig[:, j:j + 1])
    p = wgt[:, None] * comp(0) + (1 - wgt[:, None]) * comp(1) + 1e-300
    cdf = quantize_pmf(p, fp).to(torch.int32)
    inv = inverse_rows(cdf, fp)
    rows = torch.cat([cdf, inv], dim=1)
    gd = _gen(device, seed)
    idx = torch.randint(0, K, (B, N), generator=gd, device=device, dtype=torch.int32)
    sym = _sample(cdf.to(device), inv.to(device), idx, fp, gd)
    return Workload("mixture_invcdf", "rans64", fp, False, 4, "rans64_push", "rans64_invcdf_pop", sym, idx,
                    cdf.to(device), torch.full((K,), A + 1, dtype=torch.int32, device=device),
                    torch.zeros(K, dtype=torch.int32, device=device), pop_cdfs=rows.to(device), lookup="invcdf")


@dataclass
class RaggedWorkload:
    """Streams of different lengths over flat arrays, one cdf row per symbol."""
    name: str
    variant: str
    fp: int
    bypass: bool
    bp: int
    symbols: torch.Tensor     # (T,) int32
    row_starts: torch.Tensor  # (B + 1,) int64
    cdfs: torch.Tensor        # (T, A + 1) int32, row i for symbol i
    cdfs_sizes: torch.Tensor  # (T,) int32
    offsets: torch.Tensor     # (T,) int32
    lookup: str = "search"

    @property
    def num_symbols(self) -> int:
        return self.symbols.numel()

    @property
    def num_streams(self) -> int:
        return self.row_starts.numel() - 1


def ragged_lengths(streams: int, length_scale: float, seed: int) -> torch.Tensor:
    """Stream lengths clamp(round(exp(N(ln 32768, 1))), 1024, 524288), scaled by length_scale."""
    g = _gen("cpu", seed)
    ln = torch.empty(streams, dtype=torch.float64).normal_(math.log(32768.0), 1.0, generator=g)
    lo, hi = max(1, round(1024 * length_scale)), max(1, round(524288 * length_scale))
    return torch.clamp(torch.round(torch.exp(ln) * length_scale), lo, hi).to(torch.int64)


def ragged_adaptive(device="cuda", scale: float = 1.0, length_scale: float = 1.0, seed: int = 4,
                    chunk_rows: int = 1 << 22) -> RaggedWorkload:
    """rans32, 4,096 streams of lognormal lengths, each symbol with its own 33-entry cdf row
    (softmax of N(0, 2^2) logits over 32 symbols, exact integer quantisation to 2^16), symbols
    drawn from their rows.  Rows are generated on `device` in chunks of `chunk_rows`."""
    fp, A = 16, 32
    B = max(1, int(4096 * scale))
    lengths = ragged_lengths(B, length_scale, seed)
    rows = torch.zeros(B + 1, dtype=torch.int64)
    rows[1:] = torch.cumsum(lengths, 0)
    T = int(rows[-1])
    cdfs = torch.empty((T, A + 1), dtype=torch.int32, device=device)
    syms = torch.empty(T, dtype=torch.int32, device=device)
    g = _gen(device, seed + 1)
    for c0 in range(0, T, chunk_rows):
        n = min(chunk_rows, T - c0)
        logits = torch.randn((n, A), generator=g, device=device, dtype=torch.float64) * 2.0
        cdf = quantize_pmf(torch.softmax(logits, -1), fp)
        cdfs[c0:c0 + n] = cdf.to(torch.int32)
        u = torch.randint(0, 1 << fp, (n, 1), generator=g, device=device, dtype=torch.int64)
        syms[c0:c0 + n] = (torch.searchsorted(cdf, u, right=True) - 1).squeeze(1).to(torch.int32)
        del logits, cdf, u
    return RaggedWorkload("ragged_adaptive", "rans32", fp, False, 4, syms, rows.to(device), cdfs,
                          torch.full((T,), A + 1, dtype=torch.int32, device=device),
                          torch.zeros(T, dtype=torch.int32, device=device))


BUILDERS = {
    "laplace64": laplace64,
    "gaussian_latent": gaussian_latent,
    "zipf_alias": zipf_alias,
    "mixture_invcdf": mixture_invcdf,
    "ragged_adaptive": ragged_adaptive,
}
