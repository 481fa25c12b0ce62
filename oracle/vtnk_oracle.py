"""CPU oracle for the trie-constrained decoding step -- TEST INFRASTRUCTURE ONLY.

This module restates the reference's algorithm (EdoardoBotta/RecTokens) in
numpy so that the CUDA path can be checked against it.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it, and only as the checker or the timed CPU
baseline -- never as the product path.

Parity pinning: ``tests/test_oracle.py`` checks every function here against
golden vectors produced by the reference's own Python code
(``tests/golden/make_golden.py`` imports the reference and records
``from_sorted_batch``, ``vtnk_pytorch``, ``sparse_linear_pytorch`` + ``torch.topk``
and full ``decode_one_step`` beam searches) and against the reference's
hand-written known answers (tests/test_trie.py:168-190, :307-347,
tests/test_kernel.py:179-189).  The Gumbel-max sampling op has no reference
test; its oracle is pinned to the reference's formula and to Triton's Philox
(third-party dependency ``triton`` 3.6.0, ``triton/language/random.py``).

Conventions that the reference leaves open and this oracle fixes (the CUDA
kernels follow the same ones):
* ``row_ptrs[cur + 1]`` for the last node reads past the array in the
  reference; here it is ``nnz``.  ``cur < 0`` or ``cur >= n_nodes`` has no
  children.
* ``torch.topk`` tie order is unspecified; here ties go to the lower branch
  slot (top-k op) / lower flat candidate index (beam merge).
"""

from __future__ import annotations

import numpy as np

NEG_INF = np.float32(-np.inf)


# ============================================================== CSR primitives
def csr_children(row_ptrs, cols_vals, cur_node, max_branches):
    """Branch table of each row: ``(next_node, valid_idxs, n_valid)``.

    Restates rectokens/decoding/vntk.py:57-67 (and the kernels' ``_load_csr_state``,
    rectokens/kernels/constrained_node_transition.py:195-203): slot ``j`` of row
    ``b`` holds edge ``row_ptrs[cur] + j`` when ``j < n_children``; other slots
    are ``-1``.
    """
    row_ptrs = np.asarray(row_ptrs, dtype=np.int64)
    cols_vals = np.asarray(cols_vals, dtype=np.int64)
    cur = np.asarray(cur_node, dtype=np.int64)
    n_nodes = row_ptrs.shape[0]
    nnz = cols_vals.shape[1] - 1
    ok = (cur >= 0) & (cur < n_nodes)
    c = np.where(ok, cur, 0)
    start = np.where(ok, row_ptrs[c], 0)
    nxt = np.where(c + 1 < n_nodes, row_ptrs[np.minimum(c + 1, n_nodes - 1)], nnz)
    end = np.where(ok, nxt, 0)
    n_children = np.maximum(end - start, 0)
    slot = np.arange(max_branches, dtype=np.int64)[None, :]
    valid = slot < n_children[:, None]
    edge = np.clip(start[:, None] + slot, 0, nnz)
    valid_idxs = np.where(valid, cols_vals[0][edge], -1)
    next_node = np.where(valid, cols_vals[1][edge], -1)
    return next_node, valid_idxs, np.minimum(n_children, max_branches)


def mask_logits(logits, valid_idxs):
    """``logits`` kept where the column is a valid child, ``-inf`` elsewhere
    (rectokens/decoding/vntk.py:68-76)."""
    logits = np.asarray(logits)
    B, N = logits.shape
    keep = np.zeros((B, N), dtype=bool)
    r, s = np.nonzero(valid_idxs >= 0)
    keep[r, valid_idxs[r, s]] = True
    return np.where(keep, logits, np.array(-np.inf, dtype=logits.dtype))


def constrained_node_transition(logits, row_ptrs, cols_vals, cur_node, max_branches):
    """Mask-only op (reference kernels:14-176 == vntk.py:41-69)."""
    nn, vi, _ = csr_children(row_ptrs, cols_vals, cur_node, max_branches)
    return nn, vi, mask_logits(logits, vi)


# ============================================================== fused linear
def branch_logits(a, b, bias, valid_idxs, acc=np.float64):
    """Per (row, slot) logit ``sum_k a[row,k] * b[k,col]`` (+ ``bias[col]``),
    ``-inf`` on padded slots.  ``b`` is ``W.T`` with shape ``(H, N)``.

    Restates the contraction of kernels:273-356 / vntk.py:36-39 with the
    inputs' exact values accumulated in ``acc`` precision.
    """
    a = np.asarray(a)
    bt = np.asarray(b).T  # (N, H), weight rows
    B, mb = valid_idxs.shape
    out = np.full((B, mb), -np.inf, dtype=np.float64)
    N, H = bt.shape
    if N * H <= (1 << 24) and B * mb >= 4 * N:
        # many rows over a small head: one GEMM against every head row, then
        # the valid columns (the same dot products, summed by BLAS)
        wt = bt.astype(acc, copy=False)
        rchunk = max(1, (1 << 24) // N)
        for r0 in range(0, B, rchunk):
            vi = valid_idxs[r0:r0 + rchunk]
            full = a[r0:r0 + rchunk].astype(acc, copy=False) @ wt.T        # (r, N)
            vals = np.take_along_axis(full, np.maximum(vi, 0), axis=1)
            if bias is not None:
                vals = vals + np.asarray(bias, dtype=acc)[np.maximum(vi, 0)]
            out[r0:r0 + rchunk] = np.where(vi >= 0, vals, -np.inf)
        return out.astype(np.float32)
    chunk = max(1, (1 << 25) // max(1, mb * a.shape[1]))  # bound the gathered block
    for r0 in range(0, B, chunk):
        vi = valid_idxs[r0:r0 + chunk]
        wg = bt[np.maximum(vi, 0)].astype(acc, copy=False)          # (r, mb, H)
        ar = a[r0:r0 + chunk].astype(acc, copy=False)[:, :, None]   # (r, H, 1)
        vals = np.matmul(wg, ar)[:, :, 0]
        if bias is not None:
            vals = vals + np.asarray(bias, dtype=acc)[np.maximum(vi, 0)]
        out[r0:r0 + chunk] = np.where(vi >= 0, vals, -np.inf)
    return out.astype(np.float32)


def fused_linear(a, b, bias, row_ptrs, cols_vals, cur_node, max_branches, acc=np.float64):
    """``fused_linear_constrained_node_transition`` (reference ops:12-43,
    kernels:388-554): ``(next_node, valid_idxs, corrected_logits (B, N) fp32)``."""
    nn, vi, _ = csr_children(row_ptrs, cols_vals, cur_node, max_branches)
    bl = branch_logits(a, b, bias, vi, acc)
    N = np.asarray(b).shape[1]
    full = np.full((vi.shape[0], N), -np.inf, dtype=np.float32)
    r, s = np.nonzero(vi >= 0)
    full[r, vi[r, s]] = bl[r, s]
    return nn, vi, full


def topk_desc(values, k):
    """Indices of the ``k`` largest entries per row, descending, ties to the
    lower index (stable).  ``-inf`` entries rank last, by index."""
    order = np.argsort(-values, axis=1, kind="stable")
    return order[:, :k]


def fused_topk(a, b, bias, row_ptrs, cols_vals, cur_node, max_branches, k, acc=np.float64):
    """``fused_linear_constrained_node_transition_topk`` (ops:79-112,
    kernels:791-853): per-branch logits into a ``-inf`` padded ``(B, mb)``
    buffer, ``topk(k)``, then ``valid_idxs.gather``."""
    if k > max_branches:
        raise ValueError("k must not exceed max_branches")
    nn, vi, _ = csr_children(row_ptrs, cols_vals, cur_node, max_branches)
    bl = branch_logits(a, b, bias, vi, acc)
    sel = topk_desc(bl, k)
    tl = np.take_along_axis(bl, sel, axis=1)
    ti = np.take_along_axis(vi, sel, axis=1)
    ti = np.where(tl > -np.inf, ti, -1)
    return nn, vi, tl, ti


# ============================================================== Gumbel sampling
_PHILOX_KEY_A = np.uint64(0x9E3779B9)
_PHILOX_KEY_B = np.uint64(0xBB67AE85)
_PHILOX_ROUND_A = np.uint64(0xD2511F53)
_PHILOX_ROUND_B = np.uint64(0xCD9E8D57)
_M32 = np.uint64(0xFFFFFFFF)


def philox4x32_10(c0, c1, c2, c3, k0, k1):
    """Philox4x32-10 (Salmon et al., SC'11) with Triton's round/key constants
    and lane order (triton/language/random.py ``philox_impl``)."""
    c0, c1, c2, c3 = (np.asarray(x, dtype=np.uint64) & _M32 for x in (c0, c1, c2, c3))
    k0 = np.uint64(k0) & _M32
    k1 = np.uint64(k1) & _M32
    for _ in range(10):
        p0 = _PHILOX_ROUND_B * c2
        p2 = _PHILOX_ROUND_A * c0
        n0 = (p0 >> np.uint64(32)) ^ c1 ^ k0
        n2 = (p2 >> np.uint64(32)) ^ c3 ^ k1
        c1 = p0 & _M32
        c3 = p2 & _M32
        c0, c2 = n0 & _M32, n2 & _M32
        k0 = (k0 + _PHILOX_KEY_A) & _M32
        k1 = (k1 + _PHILOX_KEY_B) & _M32
    return c0, c1, c2, c3


def rand_uniform(seed, offsets):
    """``tl.rand(seed, offset)`` for int32 offsets: Philox of counter
    ``(offset, 0, 0, 0)`` keyed by the 64-bit seed, first lane mapped to
    ``[0, 1)`` by Triton's ``uint_to_uniform_float``."""
    off = np.asarray(offsets, dtype=np.int64) & 0xFFFFFFFF
    zero = np.zeros_like(off, dtype=np.uint64)
    r0, _, _, _ = philox4x32_10(off.astype(np.uint64), zero, zero, zero,
                               seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF)
    x = r0.astype(np.uint32).view(np.int32).astype(np.int64)
    x = np.where(x < 0, -x - 1, x)
    return x.astype(np.float32) * np.float32(4.6566127342e-10)


def gumbel_noise(seed, B, max_branches, row0=0):
    """Noise the sampling kernel adds to ``logit / T`` at (row, slot):
    ``-log(-log(u + 1e-10) + 1e-10)``, ``u = rand(seed, row * mb + slot)``
    (kernels:359-380).  fp32 arithmetic; the log is numpy's, so the last ulp
    may differ from a GPU ``logf`` -- parity tests feed the kernel's own noise."""
    off = (np.arange(row0, row0 + B, dtype=np.int64)[:, None] * max_branches
           + np.arange(max_branches, dtype=np.int64)[None, :])
    off = ((off + 2**31) % 2**32) - 2**31  # int32 wrap, as in the Triton kernel
    u = rand_uniform(seed, off)
    eps = np.float32(1e-10)
    with np.errstate(divide="ignore"):
        return -np.log(-np.log(u + eps) + eps)


def fused_sampling(a, b, bias, row_ptrs, cols_vals, cur_node, max_branches,
                   noise, temperature, acc=np.float64):
    """``fused_linear_constrained_node_transition_sampling`` (ops:46-76,
    kernels:562-783): ``argmax_j (logit_j / T + g_j)`` over valid slots with a
    strict ``>`` scan in slot order (first maximum wins); ``sample`` is the
    token id as float32, ``-1.0`` when no child scores above ``-inf``."""
    nn, vi, _ = csr_children(row_ptrs, cols_vals, cur_node, max_branches)
    bl = branch_logits(a, b, bias, vi, acc)
    t = np.float32(temperature)
    score = np.where(vi >= 0, bl / t + np.asarray(noise, dtype=np.float32), -np.inf)
    best = np.argmax(score, axis=1)  # first maximum
    top = score[np.arange(score.shape[0]), best]
    tok = vi[np.arange(vi.shape[0]), best]
    sample = np.where(top > -np.inf, tok.astype(np.float32), np.float32(-1.0))
    return nn, vi, sample.astype(np.float32), score


# ============================================================== beam search
def log_softmax_valid(bl):
    """Row-wise ``log_softmax`` where padded slots are ``-inf``: equal to the
    reference's ``F.log_softmax`` over the masked full-vocabulary logits
    (rectokens/decoding/constrained_decoding.py:294-297)."""
    bl = np.asarray(bl, dtype=np.float64)
    m = np.max(bl, axis=1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    with np.errstate(divide="ignore"):
        lse = m + np.log(np.sum(np.exp(bl - m), axis=1, keepdims=True))
    return bl - lse, lse[:, 0]


def beam_step(hidden, W, row_ptrs, cols_vals, cur_node, max_branches, n_cand,
              bias=None, acc=np.float64):
    """Per-row candidates for one level: the ``n_cand`` best children by logit
    (ties to the lower slot), their log-probabilities under the row's
    constrained softmax, tokens and child node ids.

    The reference obtains the same from ``logits.topk(beam_size)`` and
    ``log_softmax(...).gather`` (constrained_decoding.py:294-297) on the
    ``-inf``-masked logits; masked logits equal ``branch_logits`` scattered.
    Missing candidates (fewer children than ``n_cand``) are ``(-inf, -1, -1)``.
    """
    nn, vi, _ = csr_children(row_ptrs, cols_vals, cur_node, max_branches)
    bl = branch_logits(hidden, np.asarray(W).T, bias, vi, acc)
    logp, lse = log_softmax_valid(bl)
    pad = max(0, n_cand - bl.shape[1])
    if pad:
        bl = np.pad(bl, ((0, 0), (0, pad)), constant_values=-np.inf)
        logp = np.pad(logp, ((0, 0), (0, pad)), constant_values=-np.inf)
        vi = np.pad(vi, ((0, 0), (0, pad)), constant_values=-1)
        nn = np.pad(nn, ((0, 0), (0, pad)), constant_values=-1)
    sel = topk_desc(bl, n_cand)
    logit = np.take_along_axis(bl, sel, axis=1)
    ok = logit > -np.inf
    tok = np.where(ok, np.take_along_axis(vi, sel, axis=1), -1)
    node = np.where(ok, np.take_along_axis(nn, sel, axis=1), -1)
    lp = np.where(ok, np.take_along_axis(logp, sel, axis=1), -np.inf)
    return tok, logit, node, lp, lse


def beam_merge(level, B, k, n_cand, cand_tok, cand_node, cand_logp, prev_logp, prev_ids):
    """Beam merge of constrained_decoding.py:305-349 (+ next node :368-383).

    Level 0: each query keeps its ``k`` best of ``n_cand`` candidates.
    Later levels: ``total = prev_logp[parent] + cand_logp`` over the
    ``k * n_cand`` candidates of a query, best ``k`` kept, ``parent = idx //
    n_cand``.  Returns ``(ids (B*k, level+1), logp (B*k,), node (B*k,),
    parent_row (B*k,))``.
    """
    if level == 0:
        if k > n_cand:
            raise ValueError("k must not exceed the number of candidates")
        total = cand_logp.reshape(B, n_cand)
        toks = cand_tok.reshape(B, n_cand)
        nodes = cand_node.reshape(B, n_cand)
        sel = topk_desc(total, k)
        parent = np.repeat(np.arange(B), k)
        ids = np.take_along_axis(toks, sel, 1).reshape(B * k, 1)
    else:
        total = (np.repeat(np.asarray(prev_logp, np.float64).reshape(B, k), n_cand, axis=1)
                 + cand_logp.reshape(B, k * n_cand))
        toks = cand_tok.reshape(B, k * n_cand)
        nodes = cand_node.reshape(B, k * n_cand)
        sel = topk_desc(total, k)
        parent = (np.arange(B)[:, None] * k + sel // n_cand).reshape(B * k)
        ids = np.concatenate(
            [prev_ids[parent], np.take_along_axis(toks, sel, 1).reshape(B * k, 1)], axis=1)
    logp = np.take_along_axis(total, sel, 1).reshape(B * k)
    node = np.take_along_axis(nodes, sel, 1).reshape(B * k)
    return ids, logp, node, parent


def beam_search(hidden_levels, W, row_ptrs, cols_vals, layer_max_branches, B, k,
                n_cand, bias=None, acc=np.float64, trace=None):
    """Full constrained beam search, route A of ``decode_one_step``
    (temperature 0): level ``l`` reads ``hidden_levels[l]`` (rows = ``B`` at
    level 0, ``B*k`` after) -- the stand-in LM whose output depends on the
    beam slot.  Level 0 starts every query at the root (node 0); this equals
    the reference's dense-mask first level (constrained_decoding.py:261-268,
    368-371) because the root's CSR children are exactly the level-0 tokens.

    Returns ``(generated_ids (B, k, L), log_probas (B*k,), cur_node (B*k,))``.
    ``trace`` (a list) receives per-level candidate tables when given.
    """
    L = len(hidden_levels)
    cur = np.zeros(B, dtype=np.int64)
    ids = None
    logp = None
    for level in range(L):
        tok, logit, node, lp, lse = beam_step(
            hidden_levels[level], W, row_ptrs, cols_vals, cur,
            layer_max_branches[level], n_cand, bias, acc)
        if trace is not None:
            trace.append(dict(cur=cur, tok=tok, logit=logit, node=node, logp=lp, lse=lse))
        ids, logp, cur, _ = beam_merge(level, B, k, n_cand, tok, node, lp, logp, ids)
    return ids.reshape(B, k, L), logp.astype(np.float32), cur


# ============================================================== trie builder
def build_sorted_csr(sem_ids, vocab_size, dense_lookup_layers=2):
    """numpy restatement of ``CompactCSRTrie.from_sorted_batch``
    (rectokens/schemas/compact_csr_trie.py:97-177).  Returns
    ``(row_ptrs, cols_vals, layer_max_branches, dense_mask_by_layer, dense_states)``."""
    sem = np.asarray(sem_ids, dtype=np.int64)
    n, L = sem.shape
    dl = min(dense_lookup_layers, L)
    prev = np.concatenate([np.full((1, L), -1, np.int64), sem[:-1]], axis=0)
    opens = np.cumsum(sem != prev, axis=1) > 0
    node_of = np.cumsum(opens.T.reshape(-1)).reshape(L, n)
    cols = np.concatenate([sem.T[opens.T], [-1]])
    parents = [np.zeros(int(opens[:, 0].sum()), np.int64)]
    lmb = [parents[0].size]
    for d in range(1, L):
        p = node_of[d - 1][opens[:, d]]
        parents.append(p)
        lmb.append(int(np.bincount(p).max()) if p.size else 0)
    par = np.concatenate(parents)
    n_edges = cols.size - 1
    ch = np.flatnonzero(np.diff(par) != 0) + 1 if par.size > 1 else np.zeros(0, np.int64)
    row_ptrs = np.concatenate([[0], ch, np.full(n_edges - ch.size, n_edges)]).astype(np.int64)
    vals = np.arange(1, n_edges + 2, dtype=np.int64)
    vals[-1] = -1
    shape = (vocab_size,) * dl
    mask = np.zeros(shape, dtype=bool)
    head = tuple(sem[:, d] for d in range(dl))
    mask[head] = True
    states = np.zeros(shape, dtype=np.int64)
    states[head] = node_of[dl - 1]
    masks = []
    m = mask
    for _ in range(dl):
        masks.append(m)
        m = m.any(axis=-1)
    masks.reverse()
    return row_ptrs, np.stack([cols, vals]), lmb, masks, states
