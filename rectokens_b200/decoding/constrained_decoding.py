"""Drop-in beam-search driver for language models that return full logits.

Same entry points and semantics as the reference's
``rectokens.decoding.constrained_decoding`` (``autoregressive_generate``
:140-179, ``decode_one_step`` :194-398, route A: the model computes logits over
the whole vocabulary and the CSR trie masks them).  Per level:

* dense levels (``step < len(trie.dense_mask_by_layer)``): the dense mask, as
  in the reference (:261-268);
* CSR levels at temperature 0: one CUDA kernel
  (``vtnk_beam_candidates_from_logits``) gathers each row's children's
  logits, forms the row's log-sum-exp and its ``beam_size`` best children
  with their node ids -- the mask op, ``log_softmax``, ``topk(beam_size)`` and
  the next-node lookup of :271-303 and :372-383, with no host
  synchronisation; other levels (dense, sampling) use the CUDA mask op and
  tensor operations as the reference does (:294-303);
* beam merge: the CUDA merge kernel (``vtnk_beam_merge``), which also returns
  the parent row of every new beam;
* KV cache and attention mask are reordered by the parent rows (:305-366).

Route B, the ``SparseLinear`` output projection (``attr_path``; reference
:219-237, :281-293): on CSR levels the model's projection runs the fused op
of ``GenerationConfig.csr_kernel`` -- ``"default"`` (full masked logits, then
as above), ``"topk"`` (the op's ``beam_size`` best children, scored by the
log-softmax over those top-k logits only, as the reference does) or
``"sample"`` (one Gumbel-max sample per row, log-probability 0) -- and its
``next_nodes`` / ``valid_idxs`` tables give the child nodes.
"""

from __future__ import annotations

import contextlib
from typing import Optional

import torch
import torch.nn.functional as F
from torch import nn

from rectokens_b200 import _lib as L
from rectokens_b200.modules.constraint_enforcer import SparseTrieConstraintEnforcer
from rectokens_b200.modules.sparse_linear import SparseLinear
from rectokens_b200.ops.constrained_node_transition import constrained_node_transition
from rectokens_b200.schemas.compact_csr_trie import CompactCSRTrie
from rectokens_b200.schemas.config import GenerationConfig
from rectokens_b200.schemas.state import (
    ConstrainedGenerationState,
    ConstraintState,
    GenerationState,
)


def _reindex_past_key_values(past_key_values, indices: torch.Tensor):
    """Reorder a KV cache along the batch axis (reference :182-191)."""
    if past_key_values is None:
        return None
    if hasattr(past_key_values, "reorder_cache"):
        past_key_values.reorder_cache(indices)
        return past_key_values
    return tuple((k.index_select(0, indices), v.index_select(0, indices))
                 for k, v in past_key_values)


def _merge(level, B, k, tok, logit, node, lse, prev_logp, prev_ids):
    n = tok.shape[1]
    dev = tok.device
    ids = torch.empty((B * k, level + 1), dtype=torch.int64, device=dev)
    logp = torch.empty((B * k,), dtype=torch.float32, device=dev)
    nxt = torch.empty((B * k,), dtype=torch.int64, device=dev)
    parent = torch.empty((B * k,), dtype=torch.int64, device=dev)
    tok, logit, node, lse = (t.contiguous() for t in (tok, logit, node, lse))
    L.check(L.lib().vtnk_beam_merge(
        level, B, k, n, tok.data_ptr(), logit.data_ptr(), node.data_ptr(), lse.data_ptr(),
        L.ptr(prev_logp), L.ptr(prev_ids), ids.data_ptr(), logp.data_ptr(), nxt.data_ptr(),
        parent.data_ptr(), L.stream_of(dev)))
    return ids, logp, nxt, parent


def _candidates(logits, cs, beam_size):
    """``vtnk_beam_candidates_from_logits``: ``(tok, logit, node, lse)``."""
    trie = cs.trie
    R, N = logits.shape
    logits = logits if logits.stride(1) == 1 else logits.contiguous()
    dev = logits.device
    tok = torch.empty((R, beam_size), dtype=torch.int64, device=dev)
    logit = torch.empty((R, beam_size), dtype=torch.float32, device=dev)
    node = torch.empty((R, beam_size), dtype=torch.int64, device=dev)
    lse = torch.empty((R,), dtype=torch.float32, device=dev)
    cur = cs.cur_node.contiguous()
    csr = L.csr_struct(trie.row_ptrs, trie.stacked_cols_vals)
    L.check(L.lib().vtnk_beam_candidates_from_logits(
        logits.data_ptr(), L.DTYPE_CODE[logits.dtype], R, N, max(logits.stride(0), N),
        cur.data_ptr(), csr, trie.layer_max_branches[cs.step], beam_size, tok.data_ptr(),
        logit.data_ptr(), node.data_ptr(), lse.data_ptr(), L.stream_of(dev)))
    return tok, logit, node, lse


def _candidates_torch(logits, cs, config, step, n_dense, first, prev_ids, R, beam_size, sparse):
    """Candidates of dense levels, of sampling (temperature > 0) and of the
    routed SparseLinear strategies: ``(tok, logit, node, lse)``."""
    trie = cs.trie
    next_nodes = valid_idxs = None
    if step < n_dense:
        layer_mask = trie.dense_mask_by_layer[step]
        if first:
            layer_mask = layer_mask.unsqueeze(0).expand(R, -1)
        else:
            layer_mask = layer_mask[prev_ids.unbind(-1)]
        masked = logits.float().masked_fill(~layer_mask, float("-inf"))
    elif sparse is not None:
        next_nodes, valid_idxs = sparse.next_nodes, sparse.valid_idxs
        masked = logits.float()
    else:
        next_nodes, valid_idxs, masked = constrained_node_transition(logits, cs)
        masked = masked.float()

    routed = sparse is not None and (sparse.sample is not None or sparse.topk_idxs is not None)
    if sparse is not None and sparse.sample is not None:
        # one Gumbel-max sample per row, scored 0 (reference :281-286)
        cand_tok = sparse.sample.long().unsqueeze(1)
        cand_logit = torch.where(cand_tok >= 0, 0.0, float("-inf")).float()
        lse = torch.zeros((R,), dtype=torch.float32, device=logits.device)
    elif sparse is not None and sparse.topk_idxs is not None:
        # the op's top beam_size children, scored by the log-softmax over
        # those logits only (reference :287-293)
        cand_tok = sparse.topk_idxs
        cand_logit = masked
        lse = torch.logsumexp(masked, dim=-1)
    else:
        lse = torch.logsumexp(masked, dim=-1)
    if routed:
        pass  # candidates come from the fused op
    elif config.temperature == 0.0:
        cand_logit, cand_tok = masked.topk(beam_size, dim=-1)
    else:
        probs = F.softmax(masked / config.temperature, dim=-1)
        cand_tok = torch.multinomial(probs, num_samples=beam_size)
        cand_logit = masked.gather(1, cand_tok)
        # sampled candidates are unsorted; the merge takes its exact path for them
    cand_tok = torch.where(cand_logit > float("-inf"), cand_tok, torch.full_like(cand_tok, -1))

    if next_nodes is not None:
        # child node of each candidate: the branch slot whose token matches
        # (per-row sort + binary search; padding sorts last)
        vi = torch.where(valid_idxs >= 0, valid_idxs, torch.iinfo(torch.int64).max)
        vs, perm = torch.sort(vi, dim=1)
        pos = torch.searchsorted(vs, cand_tok).clamp(max=vs.shape[1] - 1)
        hit = vs.gather(1, pos) == cand_tok
        slot = perm.gather(1, pos)
        cand_node = torch.where(hit & (cand_tok >= 0), next_nodes.gather(1, slot), -1)
    else:
        cand_node = torch.full_like(cand_tok, -1)

    if config.temperature != 0.0 and not routed:
        # the reference scores sampled candidates by log(p_T) (:298-303)
        cand_logit = torch.where(cand_tok >= 0, cand_logit / config.temperature, cand_logit)
        lse = torch.logsumexp(masked / config.temperature, dim=-1)
    return cand_tok, cand_logit, cand_node, lse


@torch.inference_mode()
def decode_one_step(
    constrained_generation_state: ConstrainedGenerationState,
    model_fwd: nn.Module,
    input_ids: torch.Tensor,
    attention_mask: Optional[torch.Tensor] = None,
) -> ConstrainedGenerationState:
    """One constrained beam-search level (reference constrained_decoding.py:194-398)."""
    assert input_ids.ndim == 2
    cs = constrained_generation_state.constraint_state
    trie, step = cs.trie, cs.step
    gen = constrained_generation_state.generation_state
    config = constrained_generation_state.generation_config
    k, beam_size = config.k, config.beam_size
    first = gen is None
    if first:
        past_key_values, log_probas = None, None
    else:
        past_key_values, log_probas = gen.past_key_values, gen.log_probas
        attention_mask = gen.attention_mask

    n_dense = len(trie.dense_mask_by_layer)
    # route B: a SparseLinear output projection runs the fused op on CSR levels
    sparse = (next((m for m in model_fwd.modules() if isinstance(m, SparseLinear)), None)
              if isinstance(model_fwd, nn.Module) else None)
    use_sparse = sparse is not None and step >= n_dense
    ctx = (sparse.constrained(cs, strategy=config.csr_kernel, temperature=config.temperature,
                              k=beam_size) if use_sparse else contextlib.nullcontext())
    with ctx:
        out = model_fwd(input_ids, past_key_values=past_key_values,
                        attention_mask=attention_mask, use_cache=True)
    logits = out.logits[:, -1, :]
    new_past = out.past_key_values
    R = logits.shape[0]
    B = R if first else R // k
    prev_ids = None if first else gen.generated_ids.reshape(B * k, -1)

    routed = use_sparse and (sparse.sample is not None or sparse.topk_idxs is not None)
    if step >= n_dense and config.temperature == 0.0 and not routed:
        # CSR level, greedy: one kernel gathers the children's logits, forms
        # the row log-sum-exp and the beam_size best children with their
        # nodes (the mask op + log_softmax + topk + node lookup, :271-303)
        cand_tok, cand_logit, cand_node, lse = _candidates(logits, cs, beam_size)
    else:
        cand_tok, cand_logit, cand_node, lse = _candidates_torch(
            logits, cs, config, step, n_dense, first, prev_ids, R, beam_size,
            sparse if use_sparse else None)

    ids, new_logp, nxt, parent = _merge(step, B, k, cand_tok, cand_logit.float(), cand_node,
                                        lse.float(), log_probas, prev_ids)
    new_past = _reindex_past_key_values(new_past, parent)
    if attention_mask is not None:
        attention_mask = torch.cat(
            [attention_mask.index_select(0, parent),
             torch.ones(B * k, 1, dtype=attention_mask.dtype, device=attention_mask.device)],
            dim=1)
    if step == n_dense - 1:
        nxt = trie.dense_states[ids.unbind(-1)]
    elif step < n_dense - 1:
        nxt = None
    return ConstrainedGenerationState(
        generation_config=config,
        generation_state=GenerationState(generated_ids=ids.reshape(B, k, -1),
                                         past_key_values=new_past, log_probas=new_logp,
                                         attention_mask=attention_mask),
        constraint_state=ConstraintState(step=step + 1, trie=trie, cur_node=nxt),
    )


@torch.inference_mode()
def autoregressive_generate(
    model: nn.Module,
    trie: CompactCSRTrie,
    input_ids: torch.Tensor,
    generation_config: GenerationConfig,
    attr_path: Optional[str] = None,
    attention_mask: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Constrained generation for ``generation_config.steps`` levels; returns
    ``generated_ids`` ``(B, k, steps)`` (reference :140-179)."""
    if attr_path is not None:
        SparseTrieConstraintEnforcer(attr_path).prepare(model)
    state = ConstrainedGenerationState(
        generation_config=generation_config, generation_state=None,
        constraint_state=ConstraintState(step=0, trie=trie, cur_node=None))
    for _ in range(generation_config.steps):
        state = decode_one_step(state, model, input_ids, attention_mask)
        g = state.generation_state.generated_ids
        input_ids = g.reshape(-1, g.shape[-1])[:, -1:]
        attention_mask = None
    return state.generation_state.generated_ids
