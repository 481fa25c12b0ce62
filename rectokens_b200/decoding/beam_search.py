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
import weakref
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


# ------------------------------------------------------------------ per-depth layout
class DepthLayout(NamedTuple):
    node_lo: int    # nodes of this depth are [node_lo, node_hi) (BFS order)
    node_hi: int
    window_lo: int  # every child token of those nodes lies in [window_lo, window_lo + window_n)
    window_n: int


_LAYOUT_CACHE: dict = {}  # id(row_ptrs) -> (weakref to row_ptrs, {version key: slot})


def _cache_slot(trie: CompactCSRTrie) -> dict:
    """Per-trie cache, dropped when the trie's row_ptrs tensor is freed and
    keyed by both arrays' identity and version counters (an in-place edit or
    a new array invalidates it; the entry keeps the arrays it was built from
    alive, so their memory cannot be reused under it)."""
    rp = trie.row_ptrs
    ent = _LAYOUT_CACHE.get(id(rp))
    if ent is None or ent[0]() is not rp:
        ent = (weakref.ref(rp), {})
        _LAYOUT_CACHE[id(rp)] = ent
        weakref.finalize(rp, _LAYOUT_CACHE.pop, id(rp), None)
    per = ent[1]
    key = (id(trie.stacked_cols_vals), trie.stacked_cols_vals._version, rp._version)
    slot = per.get(key)
    if slot is None:
        per.clear()
        slot = per[key] = {"cols_vals": trie.stacked_cols_vals}
    return slot


def depth_layout(trie: CompactCSRTrie) -> list[DepthLayout]:
    """Node range and child-token window of every depth.

    Nodes are numbered in BFS order, so the nodes of one depth -- and the edges
    leaving them -- are contiguous; the window of depth ``d`` is the min/max
    child token over that edge range.  Computed once per trie (a few host
    synchronisations) and cached.
    """
    slot = _cache_slot(trie)
    if "layout" in slot:
        return slot["layout"]
    rp, cv = trie.row_ptrs, trie.stacked_cols_vals
    n_nodes, nnz = rp.numel(), cv.shape[1] - 1
    out = []
    n0, n1 = 0, 1
    for _ in range(len(trie.layer_max_branches)):
        e0 = int(rp[n0]) if n0 < n_nodes else nnz
        e1 = int(rp[n1]) if n1 < n_nodes else nnz
        if e1 <= e0:
            out.append(DepthLayout(n0, n1, 0, 0))
            n0 = n1
            continue
        seg = cv[0, e0:e1]
        lo, hi = int(seg.min()), int(seg.max())
        out.append(DepthLayout(n0, n1, lo, hi - lo + 1))
        n0, n1 = e0 + 1, e1 + 1
    slot["layout"] = out
    return out


def level_windows(trie: CompactCSRTrie) -> list[tuple[int, int]]:
    """``(window_lo, window_n)`` of every depth (see ``depth_layout``)."""
    return [(d.window_lo, d.window_n) for d in depth_layout(trie)]


def child_index(trie: CompactCSRTrie, depth: int):
    """The depth's child-bitmask index (``_lib.ChildIndex``, or ``None`` when
    the depth's window is wider than one 256-column tile).  Built on the
    trie's device on first use and cached with the trie."""
    slot = _cache_slot(trie)
    idx = slot.setdefault("index", {})
    if depth in idx:
        return idx[depth][0]
    d = depth_layout(trie)[depth]
    if not 1 <= d.window_n <= 256 or trie.row_ptrs.device.type != "cuda":
        idx[depth] = (None, None)
        return None
    # one allocation: the masks, then one row whose first word is the flag word
    # (bit 0: the depth's children are BFS-numbered, node id = edge index + 1)
    n = max(1, d.node_hi - d.node_lo)
    buf = torch.empty((n + 1, 8), dtype=torch.int32, device=trie.row_ptrs.device)
    masks = buf[:n]
    ci = L.ChildIndex(buf.data_ptr(), d.node_lo, d.node_hi, d.window_lo, d.window_n,
                      buf[n].data_ptr())
    csr = L.csr_struct(trie.row_ptrs, trie.stacked_cols_vals)
    L.check(L.lib().vtnk_build_child_index(csr, ci, L.stream_of(masks.device)))
    idx[depth] = (ci, masks, buf)
    return ci


def child_index_masks(trie: CompactCSRTrie, depth: int):
    """The mask tensor ``(nodes, 8)`` int32 behind ``child_index`` (or None)."""
    child_index(trie, depth)
    return _cache_slot(trie)["index"][depth][1]


# ------------------------------------------------------------------ workspace
_WS: dict = {}


def _workspace(device: torch.device, nbytes: int) -> Tensor:
    buf = _WS.get(device)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
        _WS[device] = buf
    return buf


def _search_struct(hidden: Sequence[Tensor], weight: Tensor, bias, trie: CompactCSRTrie,
                   beams: int, n_cand: int, use_index: bool, keep: list):
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
    idx = (L.ChildIndex * levels)()
    for l in range(levels):
        ci = child_index(trie, l) if use_index else None
        if ci is not None:
            idx[l] = ci
    keep += [hp, mb, idx]
    csr = L.csr_struct(trie.row_ptrs, trie.stacked_cols_vals)
    return L.Search(ctypes.cast(hp, ctypes.POINTER(ctypes.c_void_p)), H, weight.data_ptr(),
                    weight.shape[0], H, L.ptr(bias), L.DTYPE_CODE[dt], csr,
                    ctypes.cast(mb, ctypes.POINTER(ctypes.c_int64)),
                    ctypes.cast(idx, ctypes.POINTER(L.ChildIndex)),
                    levels, B, beams, n_cand)


def constrained_beam_search(
    hidden: Sequence[Tensor],
    weight: Tensor,
    trie: CompactCSRTrie,
    config: GenerationConfig,
    bias: Tensor | None = None,
    use_index: bool = True,
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
    keep: list = []
    s = _search_struct(hidden, weight, bias, trie, config.k, config.beam_size, use_index, keep)
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
              n_cand: int, bias: Tensor | None = None, index="auto"):
    """One fused level: ``(cand_tok, cand_logit, cand_node, row_lse)`` for the
    rows of ``a`` at trie depth ``step`` (``cur_node=None``: the root).
    ``index``: ``"auto"`` (the depth's cached child index), ``None`` (CUDA-core
    row kernel) or an explicit ``_lib.ChildIndex``."""
    dev = a.device
    R = a.shape[0]
    mb = trie.layer_max_branches[step]
    if isinstance(index, str):
        index = child_index(trie, step)
    tok = torch.empty((R, n_cand), dtype=torch.int64, device=dev)
    logit = torch.empty((R, n_cand), dtype=torch.float32, device=dev)
    node = torch.empty((R, n_cand), dtype=torch.int64, device=dev)
    lse = torch.empty((R,), dtype=torch.float32, device=dev)
    lin = L.linear_struct(a, weight.T, bias)
    csr = L.csr_struct(trie.row_ptrs, trie.stacked_cols_vals)
    L.check(L.lib().vtnk_beam_step(lin, L.ptr(cur_node), csr, mb, n_cand, index,
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
    device_out: bool = False,
) -> BeamSearchResult:
    """Beam search whose per-level hidden states start in (pinned) host memory.

    Level ``l + 1``'s host-to-device copy runs on a side stream while level
    ``l`` computes; the results are copied back into ``out`` (pinned host
    tensors ``(ids (B,k,L), logp (B*k,), node (B*k,))``) when given.  Returns
    host tensors after synchronising the device, or -- ``device_out`` -- the
    device tensors, without synchronising (for a caller that gathers them
    across ranks first).
    """
    dev = weight.device
    main = torch.cuda.current_stream(dev)
    copy = torch.cuda.Stream(dev)
    Lv = len(hidden_host)
    B, k = hidden_host[0].shape[0], config.k
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
        cand = beam_step(dev_h[l], weight, trie, l, cur, config.beam_size, bias)
        prev_ids, prev_logp, cur, _ = beam_merge(l, B, k, cand, prev_logp, prev_ids)
        dev_h[l] = None
    if device_out:
        return BeamSearchResult(prev_ids.view(B, k, Lv), prev_logp, cur)
    if out is None:
        out = (torch.empty((B, k, Lv), dtype=torch.int64, pin_memory=True),
               torch.empty((B * k,), dtype=torch.float32, pin_memory=True),
               torch.empty((B * k,), dtype=torch.int64, pin_memory=True))
    out[0].view(B * k, Lv).copy_(prev_ids, non_blocking=True)
    out[1].copy_(prev_logp, non_blocking=True)
    out[2].copy_(cur, non_blocking=True)
    main.synchronize()
    return BeamSearchResult(*out)


# ------------------------------------------------------------------ sampled search
def sample_step(a: Tensor, weight: Tensor, trie: CompactCSRTrie, step: int,
                cur_node: Tensor | None, seed: int, temperature: Tensor,
                bias: Tensor | None = None, index="auto", out=None):
    """One Gumbel-max sampling level (the reference's ``_sampling`` op,
    kernels:562-783, without its ``[rows, mb]`` tables): ``(sample, node)``
    with ``sample`` the sampled token id as float32 (-1.0 when a row has no
    child) and ``node`` the sampled child's node id (the next level's
    ``cur_node``).  ``temperature``: CUDA fp32 scalar tensor."""
    dev = a.device
    R = a.shape[0]
    mb = trie.layer_max_branches[step]
    if isinstance(index, str):
        index = child_index(trie, step)
    if out is None:
        out = (torch.empty((R,), dtype=torch.float32, device=dev),
               torch.empty((R,), dtype=torch.int64, device=dev))
    lin = L.linear_struct(a, weight.T, bias)
    csr = L.csr_struct(trie.row_ptrs, trie.stacked_cols_vals)
    L.check(L.lib().vtnk_fused_linear_constrained_node_transition_sampling_ix(
        lin, L.ptr(cur_node), csr, mb, seed & 0xFFFFFFFFFFFFFFFF, temperature.data_ptr(), index,
        None, None, out[0].data_ptr(), out[1].data_ptr(), L.stream_of(dev)))
    return out


def constrained_sampling_search(hidden: Sequence[Tensor], weight: Tensor, trie: CompactCSRTrie,
                                seed: int, temperature: float | Tensor,
                                bias: Tensor | None = None):
    """``L = len(hidden)`` levels of trie-constrained Gumbel-max sampling, one
    sample per row (``hidden[l]``: ``(B, H)`` CUDA tensors, row ``b`` of every
    level is sequence ``b``).  Every level draws with ``seed`` at the
    reference's offsets ``row * mb + slot``.  Returns ``(tokens (B, L) int64,
    node (B,) int64)``; a row that reaches a node without children gets -1."""
    dev = weight.device
    if not isinstance(temperature, Tensor):
        temperature = torch.tensor([float(temperature)], dtype=torch.float32, device=dev)
    B = hidden[0].shape[0]
    samples = torch.empty((len(hidden), B), dtype=torch.float32, device=dev)
    node = torch.empty((B,), dtype=torch.int64, device=dev)
    nodes = [torch.empty((B,), dtype=torch.int64, device=dev) for _ in range(2)]
    cur = None
    for l, h in enumerate(hidden):
        nxt = nodes[l & 1]
        sample_step(h, weight, trie, l, cur, seed, temperature, bias, out=(samples[l], nxt))
        cur = nxt
    node.copy_(cur)
    return samples.t().to(torch.int64), node
