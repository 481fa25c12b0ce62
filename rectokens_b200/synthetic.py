"""Seeded synthetic workloads for the constrained decoding step.

Nothing here runs on the decoding hot path: these functions build the inputs
(item catalogs, LM-head rows, per-level hidden states) that the benchmark and
the tests feed to the CUDA kernels.

Token layout follows the reference's item tokenizer: the token id of code ``c``
at level ``l`` is ``l * K + c`` (rectokens/integrations/hf/tokenizer.py:90-92
with ``original_vocab_size = 0``), so an ``L``-level catalog over ``K`` codes
has ``N = L * K`` item tokens.

Value generator (identical on host and device, integer-only so it is
bit-reproducible):

* ``mix64`` is the SplitMix64 output function (Steele, Lea & Flood, 2014).
* element ``e`` of stream ``s`` under seed ``seed`` draws
  ``z = mix64(mix64((seed << 20) ^ s) ^ e)`` and maps the top 16 bits to a
  65,536-entry table of bf16 standard-normal quantiles
  ``bf16(fp32(PhiInv((i + 0.5) / 65536)))``.
* hidden state of global row ``r`` at level ``l`` uses stream ``l`` and
  ``e = r * H + h``; the LM head uses stream ``HEAD_STREAM`` and
  ``e = n * H + h`` and is scaled by 0.02 (fp32 multiply, bf16 round-to-even).

The CUDA generator (``vtnk_synth_hidden``) implements the same function.
"""

from __future__ import annotations

import statistics
from dataclasses import dataclass
from functools import lru_cache
from typing import Callable

import numpy as np

HEAD_STREAM = 0xFFFFF
M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


# --------------------------------------------------------------------------- bits
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16, returned as uint16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(
        np.float32
    )


@lru_cache(maxsize=1)
def normal_table_f32() -> np.ndarray:
    """65,536 fp32 standard-normal quantiles at (i+0.5)/65536."""
    nd = statistics.NormalDist()
    q = np.array([nd.inv_cdf((i + 0.5) / 65536.0) for i in range(65536)])
    return q.astype(np.float32)


@lru_cache(maxsize=1)
def normal_table_bf16() -> np.ndarray:
    """The fp32 quantile table rounded to bf16 (bit patterns)."""
    return f32_to_bf16_bits(normal_table_f32())


def mix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = (np.asarray(x, dtype=np.uint64) + np.uint64(0x9E3779B97F4A7C15)) & M64
        z = ((z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)) & M64
        z = ((z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)) & M64
        return z ^ (z >> np.uint64(31))


def stream_key(seed: int, stream: int) -> np.uint64:
    return mix64(np.array([((seed << 20) ^ stream) & 0xFFFFFFFFFFFFFFFF], dtype=np.uint64))[0]


def table_index(seed: int, stream: int, start: int, count: int) -> np.ndarray:
    """Quantile-table index of elements ``start .. start+count-1`` of a stream."""
    key = stream_key(seed, stream)
    e = np.arange(start, start + count, dtype=np.uint64)
    return (mix64(e ^ key) >> np.uint64(48)).astype(np.int64)


def normal_bits(seed: int, stream: int, start: int, count: int) -> np.ndarray:
    """bf16 bits of elements ``start .. start+count-1`` of one stream."""
    return normal_table_bf16()[table_index(seed, stream, start, count)]


def hidden_bits(seed: int, level: int, row0: int, rows: int, H: int) -> np.ndarray:
    """Host copy of the per-level hidden states, ``(rows, H)`` bf16 bits."""
    return normal_bits(seed, level, row0 * H, rows * H).reshape(rows, H)


def hidden_f32(seed: int, level: int, row0: int, rows: int, H: int) -> np.ndarray:
    """fp32 variant (fp32 quantile table) for fp32 workloads, ``(rows, H)``."""
    idx = table_index(seed, level, row0 * H, rows * H)
    return normal_table_f32()[idx].reshape(rows, H)


def head_bits(seed: int, N: int, H: int, std: float = 0.02) -> np.ndarray:
    """LM-head item-token rows ``W`` ``(N, H)`` as bf16 bits, N(0, std)."""
    z = bf16_bits_to_f32(normal_bits(seed, HEAD_STREAM, 0, N * H))
    return f32_to_bf16_bits(z * np.float32(std)).reshape(N, H)


def head_f32(seed: int, N: int, H: int, std: float = 0.02) -> np.ndarray:
    """fp32 LM-head rows for fp32 workloads, ``(N, H)``."""
    idx = table_index(seed, HEAD_STREAM, 0, N * H)
    return (normal_table_f32()[idx] * np.float32(std)).reshape(N, H)


# ------------------------------------------------------------------- catalogs
def _digits(flat: np.ndarray, L: int, K: int) -> np.ndarray:
    out = np.empty((flat.size, L), dtype=np.int64)
    v = flat.astype(np.int64)
    for d in range(L - 1, -1, -1):
        out[:, d] = v % K
        v //= K
    return out


def to_tokens(codes: np.ndarray, K: int) -> np.ndarray:
    """Codes ``(n, L)`` -> token ids ``code + level * K`` (still sorted)."""
    return codes + (np.arange(codes.shape[1], dtype=np.int64) * K)[None, :]


def catalog_uniform_unique(n: int, L: int, K: int, seed: int) -> np.ndarray:
    """``n`` i.i.d. uniform codes, duplicates removed, lexicographically sorted."""
    rng = np.random.default_rng(seed)
    return np.unique(rng.integers(0, K, size=(n, L), dtype=np.int64), axis=0)


def catalog_dedup_counter(n: int, L: int, K: int, seed: int) -> np.ndarray:
    """Levels 1..L-1 uniform, last level = occurrence index within the shared
    prefix (so every item is distinct)."""
    rng = np.random.default_rng(seed)
    pre = rng.integers(0, K, size=(n, L - 1), dtype=np.int64)
    pre = pre[np.lexsort(pre.T[::-1])]
    new = np.ones(n, dtype=bool)
    new[1:] = (pre[1:] != pre[:-1]).any(axis=1)
    grp = np.cumsum(new) - 1
    first = np.flatnonzero(new)
    last = np.arange(n) - first[grp]
    if last.max(initial=0) >= K:
        raise ValueError("dedup counter overflows the codebook")
    return np.concatenate([pre, last[:, None]], axis=1)


def catalog_zipf_unique(n: int, L: int, K: int, s: float, seed: int) -> np.ndarray:
    """Level-1 codes Zipf(s) over K, deeper levels uniform, duplicates removed."""
    rng = np.random.default_rng(seed)
    p = 1.0 / np.arange(1, K + 1, dtype=np.float64) ** s
    p /= p.sum()
    first = rng.choice(K, size=n, p=p)
    rest = rng.integers(0, K, size=(n, L - 1), dtype=np.int64)
    return np.unique(np.concatenate([first[:, None], rest], axis=1), axis=0)


def catalog_sample_space(n: int, L: int, K: int, seed: int) -> np.ndarray:
    """``n`` distinct codes drawn without replacement from all ``K**L``."""
    rng = np.random.default_rng(seed)
    flat = np.sort(rng.choice(K**L, size=n, replace=False))
    return _digits(flat, L, K)


def catalog_density(p: float, L: int, K: int, seed: int) -> np.ndarray:
    """Every one of the ``K**L`` codes kept independently with probability p."""
    rng = np.random.default_rng(seed)
    flat = np.flatnonzero(rng.random(K**L) < p)
    return _digits(flat, L, K)


# -------------------------------------------------------------------- configs
@dataclass(frozen=True)
class Workload:
    name: str
    levels: int           # L
    codes: int            # K
    hidden: int           # H
    dtype: str            # "f32" | "bf16"
    batch: int
    beams: int            # k (beams kept per query)
    topk: int             # beam_size (candidates per beam and level)
    make_catalog: Callable[[], np.ndarray]
    sampling: bool = False
    temperature: float = 1.0
    seed: int = 0

    @property
    def vocab(self) -> int:
        return self.levels * self.codes

    def rows(self, level: int) -> int:
        return self.batch if level == 0 else self.batch * self.beams


WORKLOADS: dict[str, Workload] = {
    "cfg1": Workload(
        "cfg1", 3, 256, 64, "f32", 4, 5, 5,
        lambda: catalog_uniform_unique(10_000, 3, 256, seed=0),
    ),
    "cfg2": Workload(
        "cfg2", 4, 256, 896, "bf16", 256, 10, 10,
        lambda: catalog_dedup_counter(12_000, 4, 256, seed=0),
    ),
    "cfg3": Workload(
        "cfg3", 4, 256, 1536, "bf16", 1024, 20, 20,
        lambda: catalog_zipf_unique(1_000_000, 4, 256, 1.1, seed=0),
    ),
    "cfg4": Workload(
        "cfg4", 3, 256, 3584, "bf16", 4096, 1, 1,
        lambda: catalog_sample_space(4_000_000, 3, 256, seed=0),
        sampling=True, temperature=0.7,
    ),
    # the SparseLinear route's fixture: every depth has at least beam_size
    # branches (its top-k op, like torch.topk, needs k <= max_branches)
    "route_b": Workload(
        "route_b", 3, 64, 256, "bf16", 64, 5, 5,
        lambda: catalog_uniform_unique(20_000, 3, 64, seed=1),
    ),
    "cfg5": Workload(
        "cfg5", 3, 256, 3584, "bf16", 65_536, 10, 10,
        lambda: catalog_density(0.95, 3, 256, seed=0),
    ),
}


def search_rows(w: Workload) -> int:
    """Rows processed by one full search: sum over levels of rows(level)."""
    return sum(w.rows(level) for level in range(w.levels))


def ceil_div(a: int, b: int) -> int:
    return -(-a // b)


__all__ = [
    "WORKLOADS",
    "Workload",
    "bf16_bits_to_f32",
    "f32_to_bf16_bits",
    "head_bits",
    "hidden_bits",
    "normal_table_bf16",
    "search_rows",
    "to_tokens",
]
