"""CSR-encoded item trie: the data layout the constrained decoding step reads.

Same fields, dtypes and semantics as the reference's ``CompactCSRTrie``
(rectokens/schemas/compact_csr_trie.py:14-35):

* ``row_ptrs``          int64 ``[n_nodes]`` -- start of each node's child list.
  There is no trailing ``nnz`` entry: every leaf (and every node after the
  last node with children) points at ``nnz``.  Reading ``row_ptrs[cur + 1]``
  for the very last node is therefore out of range in the reference; the
  CUDA kernels clamp it to ``nnz``.
* ``stacked_cols_vals`` int64 ``[2, nnz + 1]`` -- row 0 is the child token id,
  row 1 the child's BFS node id (= edge index + 1), followed by a ``(-1, -1)``
  sentinel column.
* ``layer_max_branches`` -- largest child count of any node at each depth.
* ``dense_mask_by_layer`` / ``dense_states`` -- dense lookup tables for the
  first ``dense_lookup_layers`` levels.

The builders are written from the reference's documented behaviour
(``from_trie`` :37-95 BFS numbering, ``from_sorted_batch`` :97-177 vectorised
construction over lexicographically sorted codes) and produce bit-identical
tensors; ``tests/test_trie.py`` pins them against the reference's own
known-answer arrays and against fixtures generated from the reference.
"""

from __future__ import annotations

from collections import deque
from typing import TYPE_CHECKING, NamedTuple

import torch
from torch import Tensor

if TYPE_CHECKING:  # pragma: no cover
    from rectokens_b200.decoding.trie import Trie


class CompactCSRTrie(NamedTuple):
    row_ptrs: Tensor
    stacked_cols_vals: Tensor
    layer_max_branches: list[int]
    dense_mask_by_layer: list[Tensor]
    dense_states: Tensor
    vocab_size: int

    # ------------------------------------------------------------------ builders
    @classmethod
    def from_trie(
        cls, trie: "Trie", vocab_size: int, dense_lookup_layers: int = 2
    ) -> "CompactCSRTrie":
        """BFS walk of a pointer trie (reference compact_csr_trie.py:37-95).

        Children are emitted in the node's insertion order; node ids are BFS
        order with the root as node 0.
        """
        starts: list[int] = []
        cols: list[int] = []
        widest: dict[int, int] = {}
        shape = [vocab_size] * dense_lookup_layers
        dense_mask = torch.zeros(shape, dtype=torch.bool)
        dense_states = torch.zeros(shape, dtype=torch.long)

        next_id = 1
        queue: deque = deque([(trie.root, 0, ())])
        while queue:
            node, depth, path = queue.popleft()
            starts.append(len(cols))
            widest[depth] = max(widest.get(depth, 0), len(node.children))
            for token, child in node.children.items():
                cols.append(token)
                child_path = path + (token,)
                if len(child_path) == dense_lookup_layers:
                    dense_mask[child_path] = True
                    dense_states[child_path] = next_id
                queue.append((child, depth + 1, child_path))
                next_id += 1

        n_edges = len(cols)
        cols.append(-1)
        vals = list(range(1, n_edges + 1)) + [-1]
        depth_count = (max(widest) + 1) if widest else 0
        layer_max_branches = [widest.get(d, 0) for d in range(depth_count)]

        return cls(
            row_ptrs=torch.tensor(starts, dtype=torch.long),
            stacked_cols_vals=torch.tensor([cols, vals], dtype=torch.long),
            layer_max_branches=layer_max_branches,
            dense_mask_by_layer=_dense_masks(dense_mask, dense_lookup_layers),
            dense_states=dense_states,
            vocab_size=vocab_size,
        )

    @classmethod
    def from_sorted_batch(
        cls, sem_ids: Tensor, vocab_size: int, dense_lookup_layers: int = 2
    ) -> "CompactCSRTrie":
        """Vectorised build from lexicographically sorted codes ``(n_items, L)``.

        Follows reference compact_csr_trie.py:97-177.  On a CUDA device the
        build runs in the library's trie kernels (scan / segment; two host
        synchronisations, for the output sizes and the branch maxima); on the
        CPU it runs as tensor operations.

        Node numbering: a (depth, item) pair opens a new node when the item's
        prefix up to that depth differs from the previous item's.  New nodes are
        numbered depth-major, item-minor, starting at 1 (root = 0), which is
        exactly BFS order for a sorted catalog.
        """
        if sem_ids.is_cuda and _device_buildable(sem_ids, vocab_size, dense_lookup_layers):
            return _build_on_device(sem_ids, vocab_size, dense_lookup_layers, assume_sorted=True)
        n_items, L = sem_ids.shape
        dense_lookup_layers = min(dense_lookup_layers, L)
        dev = sem_ids.device
        sem_ids = sem_ids.to(torch.long)

        prev = torch.cat([torch.full_like(sem_ids[:1], -1), sem_ids[:-1]], dim=0)
        # prefix differs from the previous item's at some depth <= d
        opens = (sem_ids != prev).to(torch.int32).cumsum(dim=1) > 0  # (n, L)
        opens_t = opens.T.contiguous()  # (L, n) depth-major
        node_of = opens_t.reshape(-1).to(torch.long).cumsum(0).view(L, n_items)

        cols = torch.cat(
            [sem_ids.T[opens_t], torch.full((1,), -1, dtype=torch.long, device=dev)]
        )
        n_edges = cols.numel() - 1

        parent_chunks = [
            torch.zeros(int(opens[:, 0].sum()), dtype=torch.long, device=dev)
        ]
        layer_max_branches = [parent_chunks[0].numel()]
        for d in range(1, L):
            par = node_of[d - 1][opens[:, d]]
            parent_chunks.append(par)
            layer_max_branches.append(
                int(torch.bincount(par).max()) if par.numel() else 0
            )
        parents = torch.cat(parent_chunks)

        if parents.numel() > 1:
            boundaries = torch.nonzero(parents[1:] != parents[:-1]).flatten() + 1
        else:
            boundaries = torch.zeros(0, dtype=torch.long, device=dev)
        row_ptrs = torch.cat(
            [
                torch.zeros(1, dtype=torch.long, device=dev),
                boundaries,
                torch.full(
                    (n_edges - boundaries.numel(),), n_edges, dtype=torch.long, device=dev
                ),
            ]
        )
        vals = torch.arange(1, n_edges + 2, dtype=torch.long, device=dev)
        vals[-1] = -1

        shape = [vocab_size] * dense_lookup_layers
        head = sem_ids[:, :dense_lookup_layers].unbind(-1)
        dense_mask = torch.zeros(shape, dtype=torch.bool, device=dev)
        dense_mask[head] = True
        dense_states = torch.zeros(shape, dtype=torch.long, device=dev)
        dense_states[head] = node_of[dense_lookup_layers - 1]

        return cls(
            row_ptrs=row_ptrs,
            stacked_cols_vals=torch.stack([cols, vals]),
            layer_max_branches=layer_max_branches,
            dense_mask_by_layer=_dense_masks(dense_mask, dense_lookup_layers),
            dense_states=dense_states,
            vocab_size=vocab_size,
        )

    @classmethod
    def from_codes(
        cls, sem_ids: Tensor, vocab_size: int, dense_lookup_layers: int = 2
    ) -> "CompactCSRTrie":
        """Build from item token rows in any order (duplicates allowed): the
        lexicographic sort of ``ItemAwareTokenizer.build_item_trie``
        (rectokens/integrations/hf/tokenizer.py:214-229) followed by
        ``from_sorted_batch``.  On a CUDA device the sort is the library's
        radix sort of packed keys."""
        if sem_ids.is_cuda and _device_buildable(sem_ids, vocab_size, dense_lookup_layers):
            return _build_on_device(sem_ids, vocab_size, dense_lookup_layers, assume_sorted=False)
        rows = sem_ids.to(torch.long)
        order = torch.arange(rows.shape[0], device=rows.device)
        for d in range(rows.shape[1] - 1, -1, -1):  # stable passes, last level first
            order = order[torch.sort(rows[order, d], stable=True).indices]
        return cls.from_sorted_batch(rows[order], vocab_size, dense_lookup_layers)

    # ------------------------------------------------------------------ helpers
    def to(self, device) -> "CompactCSRTrie":
        """Copy every tensor field to ``device``."""
        return self._replace(
            row_ptrs=self.row_ptrs.to(device),
            stacked_cols_vals=self.stacked_cols_vals.to(device),
            dense_mask_by_layer=[m.to(device) for m in self.dense_mask_by_layer],
            dense_states=self.dense_states.to(device),
        )


def _dense_masks(full_mask: Tensor, layers: int) -> list[Tensor]:
    """Masks for depths 0..layers-1: depth d is ``full_mask`` reduced over the
    trailing ``layers-1-d`` axes (reference compact_csr_trie.py:79-84)."""
    out = []
    m = full_mask
    for _ in range(layers):
        out.append(m)
        m = m.any(dim=-1)
    out.reverse()
    return out


def _device_buildable(sem_ids: Tensor, vocab_size: int, dense_lookup_layers: int) -> bool:
    """Whether the library's trie kernels take this catalog: every item's
    tokens pack into one 64-bit key and node ids fit in 32 bits."""
    n, L = sem_ids.shape
    bits = max(1, (max(vocab_size, 2) - 1).bit_length())
    return (1 <= L <= 16 and bits * L <= 64 and bits <= 62 and n * L < 2**31 - 2
            and min(dense_lookup_layers, L) <= 4)


def _build_on_device(sem_ids: Tensor, vocab_size: int, dense_lookup_layers: int,
                     assume_sorted: bool) -> "CompactCSRTrie":
    """The trie kernels of libvtnk_b200 (``vtnk_trie_count`` + ``vtnk_trie_fill``)."""
    import ctypes

    from rectokens_b200 import _lib as L

    lib = L.lib()
    dev = sem_ids.device
    n, levels = sem_ids.shape
    dl = min(dense_lookup_layers, levels)
    sem = sem_ids.to(torch.long).contiguous()
    ws = torch.empty((lib.vtnk_trie_workspace_bytes(n, levels),), dtype=torch.uint8, device=dev)
    counts = torch.empty((levels + 2,), dtype=torch.long, device=dev)
    stream = L.stream_of(dev)
    L.check(lib.vtnk_trie_count(sem.data_ptr() if n else None, n, levels, vocab_size,
                                int(assume_sorted), ws.data_ptr(), ws.numel(),
                                counts.data_ptr(), stream))
    c = counts.tolist()  # output sizes
    if c[0] < 0:
        raise ValueError(f"token ids must lie in [0, vocab_size={vocab_size})")
    n_nodes, nnz = c[0], c[1]
    row_ptrs = torch.empty((n_nodes,), dtype=torch.long, device=dev)
    cols_vals = torch.empty((2, nnz + 1), dtype=torch.long, device=dev)
    lmb = torch.empty((levels,), dtype=torch.long, device=dev)
    masks = [torch.empty((vocab_size,) * (d + 1), dtype=torch.bool, device=dev)
             for d in range(dl)]
    states = torch.empty((vocab_size,) * dl, dtype=torch.long, device=dev)
    mp = (ctypes.c_void_p * max(1, dl))(*[m.data_ptr() for m in masks])
    L.check(lib.vtnk_trie_fill(n, levels, vocab_size, dl, ws.data_ptr(), ws.numel(), n_nodes,
                               nnz, row_ptrs.data_ptr(), cols_vals.data_ptr(), lmb.data_ptr(),
                               mp, states.data_ptr() if dl else None, stream))
    if dl == 0:
        states.zero_()
    return CompactCSRTrie(
        row_ptrs=row_ptrs,
        stacked_cols_vals=cols_vals,
        layer_max_branches=lmb.tolist(),
        dense_mask_by_layer=masks,
        dense_states=states,
        vocab_size=vocab_size,
    )
