"""Public entry points of the constrained decoding step.

Drop-in for the reference's ``rectokens.ops.constrained_node_transition``
(rectokens/ops/constrained_node_transition.py:12-135): same names, same
arguments, same return tuples.  ``b`` is ``weight.T`` (``[hidden, N]``, any
strides; the transposed view of an ``nn.Linear`` weight is the fast layout).
The work runs in the CUDA kernels of libvtnk_b200 (sm_100a); there is no CPU
path.
"""

from __future__ import annotations

import torch

from rectokens_b200.ops._vtnk_ops import (
    _constrained_node_transition_op,
    _fused_linear_constrained_node_transition_op,
    _fused_linear_constrained_node_transition_sampling_ix_op,
    _fused_linear_constrained_node_transition_sampling_op,
    _fused_linear_constrained_node_transition_topk_ix_op,
    _fused_linear_constrained_node_transition_topk_op,
    default_seed,
)
from rectokens_b200.schemas.state import ConstraintState


def _tile_index(a: torch.Tensor, constraint_state: ConstraintState):
    """``(masks, node_lo, node_hi, window_lo, window_n)`` of the step's depth
    when the tile kernel can serve the call (bf16 CUDA operands, a child
    index for the depth), else None."""
    if a.dtype != torch.bfloat16 or a.device.type != "cuda" or a.shape[0] < 128:
        return None
    from rectokens_b200.decoding.beam_search import child_index, child_index_masks

    trie, step = constraint_state.trie, constraint_state.step
    ci = child_index(trie, step)
    if ci is None:
        return None
    return (child_index_masks(trie, step), ci.node_lo, ci.node_hi, ci.window_lo, ci.window_n)


def fused_linear_constrained_node_transition(
    a: torch.Tensor,
    b: torch.Tensor,
    constraint_state: ConstraintState,
    bias: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Fused linear projection + constrained node transition.

    Returns ``(next_node, valid_idxs, corrected_logits)``:
      next_node        (B, max_branches) int64 -- child BFS ids, -1 padding
      valid_idxs       (B, max_branches) int64 -- child token ids, -1 padding
      corrected_logits (B, N) float32          -- a @ b (+ bias) on child columns, -inf elsewhere
    """
    bias_val = bias if bias is not None else a.new_empty(0)
    max_branches = constraint_state.trie.layer_max_branches[constraint_state.step]
    return _fused_linear_constrained_node_transition_op(
        a, b, bias_val, constraint_state.cur_node, constraint_state.trie.row_ptrs,
        constraint_state.trie.stacked_cols_vals, max_branches, bias is not None)


def fused_linear_constrained_node_transition_sampling(
    a: torch.Tensor,
    b: torch.Tensor,
    constraint_state: ConstraintState,
    bias: torch.Tensor | None = None,
    rng_seed: int | None = None,
    temperature: float | torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Fused linear projection + constrained node transition + Gumbel-max sampling.

    Returns ``(next_node, valid_idxs, sample)``; ``sample`` (B,) float32 holds
    the sampled token id per row (-1.0 when a row has no child).  With
    ``rng_seed=None`` the seed is drawn from the clock, as in the reference.
    """
    bias_val = bias if bias is not None else a.new_empty(0)
    max_branches = constraint_state.trie.layer_max_branches[constraint_state.step]
    if rng_seed is None:
        rng_seed = default_seed()
    if temperature is None:
        temperature = 1.0
    if not isinstance(temperature, torch.Tensor):
        temperature = torch.tensor([float(temperature)], dtype=torch.float32, device=a.device)
    ix = _tile_index(a, constraint_state)
    if ix is not None:
        return _fused_linear_constrained_node_transition_sampling_ix_op(
            a, b, bias_val, constraint_state.cur_node, constraint_state.trie.row_ptrs,
            constraint_state.trie.stacked_cols_vals, *ix, max_branches, bias is not None,
            int(rng_seed), temperature)
    return _fused_linear_constrained_node_transition_sampling_op(
        a, b, bias_val, constraint_state.cur_node, constraint_state.trie.row_ptrs,
        constraint_state.trie.stacked_cols_vals, max_branches, bias is not None,
        int(rng_seed), temperature)


def fused_linear_constrained_node_transition_topk(
    a: torch.Tensor,
    b: torch.Tensor,
    constraint_state: ConstraintState,
    k: int,
    bias: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Fused linear projection + constrained node transition + top-k.

    Returns ``(next_node, valid_idxs, topk_logits, topk_idxs)``:
      topk_logits (B, k) float32 -- descending
      topk_idxs   (B, k) int64   -- token ids, -1 where a row has fewer than k children
    """
    bias_val = bias if bias is not None else a.new_empty(0)
    max_branches = constraint_state.trie.layer_max_branches[constraint_state.step]
    ix = _tile_index(a, constraint_state)
    if ix is not None:
        return _fused_linear_constrained_node_transition_topk_ix_op(
            a, b, bias_val, constraint_state.cur_node, constraint_state.trie.row_ptrs,
            constraint_state.trie.stacked_cols_vals, *ix, max_branches, bias is not None, k)
    return _fused_linear_constrained_node_transition_topk_op(
        a, b, bias_val, constraint_state.cur_node, constraint_state.trie.row_ptrs,
        constraint_state.trie.stacked_cols_vals, max_branches, bias is not None, k)


def constrained_node_transition(
    logits: torch.Tensor,
    constraint_state: ConstraintState,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Mask precomputed ``logits`` (B, N) to the children of ``cur_node``.

    Returns ``(next_node, valid_idxs, corrected_logits)`` with
    ``corrected_logits`` of ``logits``' dtype, -inf off the child columns.
    """
    trie = constraint_state.trie
    max_branches = trie.layer_max_branches[constraint_state.step]
    return _constrained_node_transition_op(
        logits, constraint_state.cur_node, trie.row_ptrs, trie.stacked_cols_vals, max_branches)
