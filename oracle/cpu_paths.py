"""The reference's two CPU paths for a full constrained beam search --
TEST / BASELINE INFRASTRUCTURE ONLY.

``bench.py`` times these on the GPU box's host cores as the CPU baseline
(``cpu_baseline`` leg and ``--impl reference``); ``tests/test_cpu_paths.py``
pins both to the oracle's ``beam_search`` (itself pinned to the reference's own
``decode_one_step`` runs).  Nothing in the product path imports this module.

* Sparse-PyTorch path: the reference's ``sparse_linear_pytorch``
  (rectokens/decoding/vntk.py:4-38) in eager torch on the CPU, fp32 (the
  reference function needs fp32 on the CPU), rows processed in chunks so the
  ``(rows, max_branches, H)`` weight gather stays bounded; then route A of
  ``decode_one_step`` (rectokens/decoding/constrained_decoding.py:294-349,
  next node :368-383): ``topk(beam_size)`` and ``log_softmax`` over the
  ``-inf``-masked full-vocabulary logits, beam merge by ``topk(k)``.
* CPU trie path: the reference's pointer ``Trie`` (rectokens/decoding/trie.py:
  5-33) walked row by row as in examples/scripts/benchmark/benchmark_vtnk.py:
  54-80 (``node.children`` gives each row's allowed tokens), the allowed
  tokens scored by fp32 dot products, then the same merge.
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import vtnk_oracle as O


# ------------------------------------------------------------------ sparse path
def sparse_linear(a, weight, cur_node, row_ptrs, cols_vals, mb, chunk=16):
    """``sparse_linear_pytorch(a, weight, cur_node, trie, step)`` with
    ``layer_max_branches[step] = mb``: ``(next_node, valid_idxs,
    corrected_logits (B, N) fp32)``.  The last node's end is ``nnz`` (the
    reference reads one past ``row_ptrs`` there)."""
    B = a.shape[0]
    N = weight.shape[0]
    n_nodes = row_ptrs.shape[0]
    nnz = cols_vals.shape[1] - 1
    idx_start = row_ptrs[cur_node]
    nxt = torch.where(cur_node + 1 < n_nodes, row_ptrs[(cur_node + 1).clamp(max=n_nodes - 1)],
                      torch.full_like(cur_node, nnz))
    n_children = nxt - idx_start
    ar = torch.arange(mb)
    slice_idxs = (idx_start.unsqueeze(-1) + ar).clamp(max=nnz)
    cols, vals = cols_vals[:, slice_idxs].unbind()
    valid_range = ar < n_children.unsqueeze(-1)
    valid_idxs = torch.where(valid_range, cols, -1)
    next_node = torch.where(valid_range, vals, -1)
    clamped = valid_idxs.clamp(min=0)
    logits_valid = torch.empty((B, mb), dtype=torch.float32)
    for r0 in range(0, B, chunk):
        w = weight[clamped[r0:r0 + chunk]]                      # (c, mb, H)
        logits_valid[r0:r0 + chunk] = (a[r0:r0 + chunk].unsqueeze(1) * w).sum(dim=-1)
    corrected = torch.full((B, N), float("-inf"), dtype=torch.float32)
    b_idx = torch.arange(B).unsqueeze(-1).expand_as(valid_idxs)
    valid = valid_idxs >= 0
    corrected[b_idx[valid], valid_idxs[valid]] = logits_valid[valid]
    return next_node, valid_idxs, corrected


def merge_route_a(level, logits, next_nodes, valid_idxs, prev_logp, prev_ids, B, k, beam_size):
    """Route A of ``decode_one_step`` at temperature 0 on masked logits."""
    _, samples = logits.topk(beam_size, dim=-1)
    lp = torch.log_softmax(logits, dim=-1).gather(1, samples)
    if level == 0:
        top_lp, top_i = lp.topk(k, dim=1)
        ids = torch.gather(samples, 1, top_i).reshape(B * k, 1)
        parent = torch.arange(B).repeat_interleave(k)
    else:
        total = prev_logp.reshape(B, k).repeat_interleave(beam_size, dim=1) + lp.reshape(
            B, k * beam_size)
        top_lp, top_i = total.topk(k, dim=1)
        parent = (torch.arange(B).unsqueeze(1) * k + top_i // beam_size).reshape(B * k)
        tok = torch.gather(samples.reshape(B, k * beam_size), 1, top_i).reshape(B * k, 1)
        ids = torch.cat([prev_ids[parent], tok], dim=-1)
    match = valid_idxs[parent] == ids[:, -1:]
    node = torch.where(match, next_nodes[parent], 0).sum(dim=1)
    return ids, top_lp.reshape(B * k), node


def sparse_path_search(hidden_levels, W, row_ptrs, cols_vals, lmb, B, k, beam_size, chunk=16):
    """Full search through the sparse-PyTorch path.  ``hidden_levels``: fp32
    torch tensors; ``W``: fp32 ``(N, H)``; trie arrays int64 torch tensors.
    Returns ``(ids (B, k, L), logp (B*k,), node (B*k,))`` as numpy."""
    cur = torch.zeros(B, dtype=torch.int64)
    ids = logp = None
    for level, a in enumerate(hidden_levels):
        nn, vi, logits = sparse_linear(a, W, cur, row_ptrs, cols_vals, lmb[level], chunk)
        ids, logp, cur = merge_route_a(level, logits, nn, vi, logp, ids, B, k, beam_size)
    return ids.reshape(B, k, -1).numpy(), logp.numpy(), cur.numpy()


# ------------------------------------------------------------------ CPU trie path
class TrieNode:
    """The reference's pointer-trie node (rectokens/decoding/trie.py:5-12),
    plus the BFS id that ``cur_node`` indexes by."""

    __slots__ = ("children", "node_id")

    def __init__(self, node_id):
        self.children = {}
        self.node_id = node_id


class PointerTrie:
    """A pointer trie holding the nodes a search visits, materialised from
    the CSR arrays (set-up, not timed); ``nodes[id]`` is the BFS-id lookup the
    reference's benchmark builds with its node list (benchmark_vtnk.py:54-67)."""

    def __init__(self, row_ptrs, cols_vals):
        self.rp = np.asarray(row_ptrs)
        self.cv = np.asarray(cols_vals)
        self.nodes: dict = {}

    def add(self, node_id):
        if node_id in self.nodes:
            return self.nodes[node_id]
        n = TrieNode(node_id)
        s = int(self.rp[node_id])
        e = int(self.rp[node_id + 1]) if node_id + 1 < self.rp.size else self.cv.shape[1] - 1
        for j in range(s, e):
            n.children[int(self.cv[0, j])] = TrieNode(int(self.cv[1, j]))
        self.nodes[node_id] = n
        return n


def trie_path_search(hidden_levels, W, trie: PointerTrie, lmb, B, k, beam_size):
    """Full search through the CPU trie path: per row, the allowed tokens are
    ``nodes[cur].children`` (benchmark_vtnk.py:70-80), scored by fp32 dot
    products, then log-softmax over the allowed tokens (equal to the masked
    full-vocabulary log-softmax), top-``beam_size`` and the beam merge.
    ``hidden_levels`` / ``W``: fp32 numpy.  Returns numpy like
    ``sparse_path_search``."""
    cur = np.zeros(B, dtype=np.int64)
    ids = logp = None
    for level, a in enumerate(hidden_levels):
        R = a.shape[0]
        mb = max(lmb[level], beam_size)
        tok = np.full((R, mb), -1, np.int64)
        node = np.full((R, mb), -1, np.int64)
        logit = np.full((R, mb), -np.inf, np.float32)
        for r in range(R):
            tn = trie.nodes.get(int(cur[r])) or trie.add(int(cur[r]))
            toks = list(tn.children.keys())
            if not toks:
                continue
            n = len(toks)
            tok[r, :n] = toks
            node[r, :n] = [c.node_id for c in tn.children.values()]
            logit[r, :n] = W[toks] @ a[r]
        lp_all, _ = O.log_softmax_valid(logit)
        sel = O.topk_desc(logit, beam_size)
        ok = np.take_along_axis(logit, sel, 1) > -np.inf
        ctok = np.where(ok, np.take_along_axis(tok, sel, 1), -1)
        cnode = np.where(ok, np.take_along_axis(node, sel, 1), -1)
        clp = np.where(ok, np.take_along_axis(lp_all, sel, 1), -np.inf)
        ids, logp, cur, _ = O.beam_merge(level, B, k, beam_size, ctok, cnode, clp, logp, ids)
    return ids.reshape(B, k, -1), logp.astype(np.float32), cur
