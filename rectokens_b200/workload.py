"""Device-side construction of the benchmark workloads (catalog trie, LM-head
item rows, per-level hidden states) from ``rectokens_b200.synthetic``.

Input preparation only: the trie is built once (``from_sorted_batch`` on the
GPU), the head rows on the host (they are small), and the hidden states by the
``vtnk_synth_normal`` kernel so that large levels never cross PCIe.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from rectokens_b200 import _lib as L
from rectokens_b200 import synthetic as S
from rectokens_b200.schemas.compact_csr_trie import CompactCSRTrie

_TABLES: dict = {}


def quantile_table(dtype: torch.dtype, device) -> torch.Tensor:
    key = (dtype, str(device))
    t = _TABLES.get(key)
    if t is None:
        if dtype == torch.bfloat16:
            t = torch.from_numpy(S.normal_table_bf16().view(np.int16).copy()).to(device)
        else:
            t = torch.from_numpy(S.normal_table_f32().copy()).to(device)
        _TABLES[key] = t
    return t


def synth_hidden(seed: int, level: int, row0: int, rows: int, H: int, dtype: torch.dtype,
                 device, out: torch.Tensor | None = None) -> torch.Tensor:
    """Rows ``row0 .. row0+rows-1`` of level ``level``'s hidden states, on device."""
    if out is None:
        out = torch.empty((rows, H), dtype=dtype, device=device)
    code = L.BF16 if dtype == torch.bfloat16 else L.F32
    tab = quantile_table(dtype, device)
    L.check(L.lib().vtnk_synth_normal(seed, level, row0, rows, H, tab.data_ptr(), code,
                                      out.data_ptr(), L.stream_of(out.device)))
    return out


def head_weight(w: S.Workload, device) -> torch.Tensor:
    if w.dtype == "f32":
        return torch.from_numpy(S.head_f32(w.seed, w.vocab, w.hidden)).to(device)
    bits = S.head_bits(w.seed, w.vocab, w.hidden)
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).to(device)


def build_trie(w: S.Workload, device, codes: np.ndarray | None = None) -> CompactCSRTrie:
    if codes is None:
        codes = w.make_catalog()
    tok = torch.from_numpy(S.to_tokens(codes, w.codes)).to(device)
    return CompactCSRTrie.from_sorted_batch(tok, vocab_size=w.vocab, dense_lookup_layers=1)


@dataclass
class DeviceWorkload:
    spec: S.Workload
    trie: CompactCSRTrie
    weight: torch.Tensor
    hidden: list            # per level, rows of this shard
    row_offset: list        # global first row per level
    batch: int              # queries in this shard


def make_device_workload(w: S.Workload, device, shard: int = 0, n_shards: int = 1,
                         trie: CompactCSRTrie | None = None) -> DeviceWorkload:
    """Shard ``shard`` of ``n_shards`` (contiguous query ranges) of workload ``w``."""
    from rectokens_b200.distributed import level_rows, shard_queries

    q0, bq = shard_queries(w.batch, shard, n_shards)
    dtype = torch.float32 if w.dtype == "f32" else torch.bfloat16
    if trie is None:
        trie = build_trie(w, device)
    weight = head_weight(w, device)
    hidden, offs = [], []
    for level in range(w.levels):
        r0, rows = level_rows(q0, bq, level, w.beams)
        hidden.append(synth_hidden(w.seed, level, r0, rows, w.hidden, dtype, device))
        offs.append(r0)
    return DeviceWorkload(w, trie, weight, hidden, offs, bq)
