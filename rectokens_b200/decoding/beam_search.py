"""Device-resident constrained beam search over item tokens.

Equivalent to the reference's ``autoregressive_generate`` with
``GenerationConfig(steps=L, k=beams, beam_size=n_cand, temperature=0.0)``
(rectokens/decoding/constrained_decoding.py:140-179, route A of
``decode_one_step`` :194-398) for a language model whose item-token logits at
level ``l`` are ``hidden[l] @ W.T (+ bias)``: each level is one fused
step kernel (contraction + CSR mask + per-beam top-``n_cand`` + log-sum-exp)
and one beam-merge kernel; full logits never reach HBM and there is no host
synchronisation inside the search.

Level 0 starts every query at the root: the reference's dense first-level
mask (constrained_decoding.py:261-268) admits exactly the root's CSR
children, and ``dense_states`` maps them to the same node ids
(:368-371), so the outputs are identical.
"""

from __future__ import annotations

import ctypes
from typing import NamedTuple, Sequence

import torch
from torch import Tensor

from rectokens_b200 import _lib as L
from rectokens_b200.schemas.compact_csr_trie import CompactCSRTrie
from rectokens_b200.schemas.config import GenerationConfig


class BeamSearchResult(NamedTuple):
    generated_ids: Tensor   # (B, k, L) int64 token ids
    log_probas: Tensor      # (B * k,) float32 cumulative log-probabilities
    cur_node: Tensor        # (B * k,) int64 trie node reached


# ------------------------------------------------------------------ level windows
_WINDOW_CACHE: dict = {}


def level_windows(trie: CompactCSRTrie) -> list[tuple[int, int]]:
    """Token range ``(lo, n)`` holding every child of every node at each depth.

    Nodes are numbered in BFS order, so the nodes of one depth -- and the edges
    leaving them -- are contiguous; the window of depth ``d`` is the min/max
    child token over that edge range.  Computed once per trie storage (a few
    host synchronisations) and cached.
    """
    rp, cv = trie.row_ptrs, trie.stacked_cols_vals
    key = (rp.data_ptr(), cv.data_ptr(), rp.numel(), cv.shape[1], str(rp.device))
    hit = _WINDOW_CACHE.get(key)
    if hit is not None:
        return hit
    n_nodes, nnz = rp.numel(), cv.shape[1] - 1
    out = []
    n0, n1 = 0, 1
    for _ in range(len(trie.layer_max_branches)):
        e0 = int(rp[n0]) if n0 < n_nodes else nnz
        e1 = int(rp[n1]) if n1 < n_nodes else nnz
        if e1 <= e0:
            out.append((0, 0))
            n0, n1 = n1, n1
            continue
        seg = cv[0, e0:e1]
        lo, hi = int(seg.min()), int(seg.max())
        out.append((lo, hi - lo + 1))
        n0, n1 = e0 + 1, e1 + 1
    if len(_WINDOW_CACHE) > 64:
        _WINDOW_CACHE.clear()
    _WINDOW_CACHE[key] = out
    return out


# ------------------------------------------------------------------ workspace
_WS: dict = {}


def _workspace(device: torch.device, nbytes: int) -> Tensor:
    buf = _WS.get(device)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
        _WS[device] = buf
    return buf


def _search_struct(hidden: Sequence[Tensor], weight: Tensor, bias, trie: CompactCSRTrie,
                   beams: int, n_cand: int, windows, keep: list):
    levels = len(hidden)
    if levels < 1:
        raise ValueError("need at least one level")
    if levels > len(trie.layer_max_branches):
        raise ValueError("more levels than the trie has depths")
    B = hidden[0].shape[0]
    H = weight.shape[1]
    dt = weight.dtype
    for l, h in enumerate(hidden):
        rows = B if l == 0 else B * beams
        if h.shape != (rows, H) or h.dtype != dt or h.stride(1) != 1 or h.stride(0) != H:
            raise ValueError(f"hidden[{l}] must be contiguous {(rows, H)} {dt}")
    if not weight.is_contiguous():
        raise ValueError("weight must be a contiguous (N, H) tensor")
    hp = (ctypes.c_void_p * levels)(*[h.data_ptr() for h in hidden])
    mb = (ctypes.c_int64 * levels)(*trie.layer_max_branches[:levels])
    wlo = (ctypes.c_int64 * levels)(*[w[0] for w in windows[:levels]])
    wn = (ctypes.c_int64 * levels)(*[w[1] for w in windows[:levels]])
    keep += [hp, mb, wlo, wn]
    csr = L.csr_struct(trie.row_ptrs, trie.stacked_cols_vals)
    return L.Search(ctypes.cast(hp, ctypes.POINTER(ctypes.c_void_p)), H, weight.data_ptr(),
                    weight.shape[0], H, L.ptr(bias), L.DTYPE_CODE[dt], csr,
                    ctypes.cast(mb, ctypes.POINTER(ctypes.c_int64)),
                    ctypes.cast(wlo, ctypes.POINTER(ctypes.c_int64)),
                    ctypes.cast(wn, ctypes.POINTER(ctypes.c_int64)),
                    levels, B, beams, n_cand)


def constrained_beam_search(
    hidden: Sequence[Tensor],
    weight: Tensor,
    trie: CompactCSRTrie,
    config: GenerationConfig,
    bias: Tensor | None = None,
    use_windows: bool = True,
) -> BeamSearchResult:
    """Run an ``L = len(hidden)``-level beam search on the GPU in one call.

    ``hidden[l]``: CUDA tensor ``(B, H)`` at level 0 and ``(B*k, H)`` after
    (row ``b*k + i`` is beam ``i`` of query ``b``); ``weight``: the item-token
    rows of the LM head ``(N, H)``; ``config.k`` beams kept, ``config.beam_size``
    candidates per beam and level.  Only ``temperature == 0`` (greedy beam
    search) is a beam search; use the sampling op for sampling.
    """
    if config.temperature != 0.0:
        raise ValueError("constrained_beam_search implements temperature == 0.0")
    dev = weight.device
    if dev.type != "cuda":
        raise RuntimeError("constrained_beam_search runs on CUDA tensors only")
    windows = level_windows(trie) if use_windows else [(0, 0)] * len(hidden)
    keep: list = []
    s = _search_struct(hidden, weight, bias, trie, config.k, config.beam_size, windows, keep)
    B, k, Lv = s.batch, s.beams, s.levels
    lib = L.lib()
    nbytes = lib.vtnk_beam_search_workspace_bytes(s)
    ws = _workspace(dev, nbytes)
    ids = torch.empty((B * k, Lv), dtype=torch.int64, device=dev)
    logp = torch.empty((B * k,), dtype=torch.float32, device=dev)
    node = torch.empty((B * k,), dtype=torch.int64, device=dev)
    L.check(lib.vtnk_beam_search(s, ws.data_ptr(), ws.numel(), ids.data_ptr(), logp.data_ptr(),
                                 node.data_ptr(), L.stream_of(dev)))
    return BeamSearchResult(ids.view(B, k, Lv), logp, node)


def beam_step(a: Tensor, weight: Tensor, trie: CompactCSRTrie, step: int, cur_node: Tensor | None,
              n_cand: int, bias: Tensor | None = None, window: tuple[int, int] | None = None):
    """One fused level: ``(cand_tok, cand_logit, cand_node, row_lse)`` for the
    rows of ``a`` at trie depth ``step`` (``cur_node=None``: the root)."""
    dev = a.device
    R = a.shape[0]
    mb = trie.layer_max_branches[step]
    if window is None:
        window = level_windows(trie)[step]
    tok = torch.empty((R, n_cand), dtype=torch.int64, device=dev)
    logit = torch.empty((R, n_cand), dtype=torch.float32, device=dev)
    node = torch.empty((R, n_cand), dtype=torch.int64, device=dev)
    lse = torch.empty((R,), dtype=torch.float32, device=dev)
    lin = L.linear_struct(a, weight.T, bias)
    csr = L.csr_struct(trie.row_ptrs, trie.stacked_cols_vals)
    L.check(L.lib().vtnk_beam_step(lin, L.ptr(cur_node), csr, mb, n_cand, window[0], window[1],
                                   tok.data_ptr(), logit.data_ptr(), node.data_ptr(),
                                   lse.data_ptr(), L.stream_of(dev)))
    return tok, logit, node, lse


def beam_merge(level: int, B: int, k: int, cand, prev_logp: Tensor | None,
               prev_ids: Tensor | None):
    """Beam merge of one level: ``(ids, logp, node, parent)``."""
    tok, logit, node, lse = cand
    n_cand = tok.shape[1]
    dev = tok.device
    ids = torch.empty((B * k, level + 1), dtype=torch.int64, device=dev)
    logp = torch.empty((B * k,), dtype=torch.float32, device=dev)
    nxt = torch.empty((B * k,), dtype=torch.int64, device=dev)
    parent = torch.empty((B * k,), dtype=torch.int64, device=dev)
    L.check(L.lib().vtnk_beam_merge(
        level, B, k, n_cand, tok.data_ptr(), logit.data_ptr(), node.data_ptr(), lse.data_ptr(),
        L.ptr(prev_logp), L.ptr(prev_ids), ids.data_ptr(), logp.data_ptr(), nxt.data_ptr(),
        parent.data_ptr(), L.stream_of(dev)))
    return ids, logp, nxt, parent


def constrained_beam_search_from_host(
    hidden_host: Sequence[Tensor],
    weight: Tensor,
    trie: CompactCSRTrie,
    config: GenerationConfig,
    bias: Tensor | None = None,
    out: tuple[Tensor, Tensor, Tensor] | None = None,
) -> BeamSearchResult:
    """Beam search whose per-level hidden states start in (pinned) host memory.

    Level ``l + 1``'s host-to-device copy runs on a side stream while level
    ``l`` computes; the results are copied back into ``out`` (pinned host
    tensors ``(ids (B,k,L), logp (B*k,), node (B*k,))``) when given.  Returns
    host tensors after synchronising the device.
    """
    dev = weight.device
    main = torch.cuda.current_stream(dev)
    copy = torch.cuda.Stream(dev)
    Lv = len(hidden_host)
    B, k = hidden_host[0].shape[0], config.k
    windows = level_windows(trie)
    dev_h: list = [None] * Lv
    ready: list = [None] * Lv

    def issue(l):
        with torch.cuda.stream(copy):
            dev_h[l] = hidden_host[l].to(dev, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(copy)
            ready[l] = ev

    issue(0)
    prev_logp = prev_ids = cur = None
    for l in range(Lv):
        if l + 1 < Lv:
            issue(l + 1)
        main.wait_event(ready[l])
        dev_h[l].record_stream(main)
        cand = beam_step(dev_h[l], weight, trie, l, cur, config.beam_size, bias, windows[l])
        prev_ids, prev_logp, cur, _ = beam_merge(l, B, k, cand, prev_logp, prev_ids)
        dev_h[l] = None
    if out is None:
        out = (torch.empty((B, k, Lv), dtype=torch.int64, pin_memory=True),
               torch.empty((B * k,), dtype=torch.float32, pin_memory=True),
               torch.empty((B * k,), dtype=torch.int64, pin_memory=True))
    out[0].view(B * k, Lv).copy_(prev_ids, non_blocking=True)
    out[1].copy_(prev_logp, non_blocking=True)
    out[2].copy_(cur, non_blocking=True)
    main.synchronize()
    return BeamSearchResult(*out)
