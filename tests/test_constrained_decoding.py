"""The drop-in ``decode_one_step`` / ``autoregressive_generate`` (GPU) against
the reference's own runs (golden) and its test properties
(reference tests/test_constrained_decoding.py)."""

import types

import numpy as np
import pytest
import torch
from torch import nn

from conftest import load_golden
from rectokens_b200 import synthetic as S
from rectokens_b200 import workload as WL
from rectokens_b200.decoding.constrained_decoding import autoregressive_generate, decode_one_step
from rectokens_b200.schemas import (CompactCSRTrie, ConstrainedGenerationState, ConstraintState,
                                    GenerationConfig)

pytestmark = pytest.mark.gpu
DEV = "cuda"


class _StubLM:
    """Logits at level l = hidden[l] @ W.T in fp32 (the golden fixtures' model)."""

    def __init__(self, hidden, W):
        self.h = [h.float() for h in hidden]
        self.W = W.float()
        self.calls = 0

    def __call__(self, input_ids, past_key_values=None, attention_mask=None, use_cache=True):
        h = self.h[self.calls]
        self.calls += 1
        return types.SimpleNamespace(logits=(h @ self.W.T).unsqueeze(1), past_key_values=None)


@pytest.mark.parametrize("name", ["cfg1", "cfg2"])
def test_generate_matches_reference_golden(name, cuda_ok):
    g = load_golden(f"search_{name}.npz")
    w = S.WORKLOADS[name]
    dw = WL.make_device_workload(w, DEV)
    model = _StubLM(dw.hidden, dw.weight)
    cfg = GenerationConfig(steps=w.levels, k=w.beams, beam_size=w.topk, temperature=0.0)
    state = ConstrainedGenerationState(generation_config=cfg,
                                       constraint_state=ConstraintState(0, dw.trie, None))
    ids = torch.zeros(w.batch, 1, dtype=torch.long, device=DEV)
    for _ in range(w.levels):
        state = decode_one_step(state, model, ids)
        gen = state.generation_state.generated_ids
        ids = gen.reshape(-1, gen.shape[-1])[:, -1:]
    np.testing.assert_array_equal(state.generation_state.generated_ids.cpu().numpy(),
                                  g["generated_ids"])
    np.testing.assert_array_equal(state.constraint_state.cur_node.cpu().numpy(), g["cur_node"])
    np.testing.assert_allclose(state.generation_state.log_probas.cpu().numpy(), g["log_probas"],
                               atol=1e-4, rtol=0)


SEQS_5 = [[1, 2, 3, 4, 5], [1, 2, 7, 3, 6], [3, 1, 2, 5, 4], [2, 5, 1, 3, 7], [4, 6, 2, 1, 3]]
SEQS_3 = [[1, 2, 3], [1, 2, 7], [3, 1, 2], [2, 5, 1], [4, 6, 2]]


class _RandomModel(nn.Module):
    """Embedding + linear LM with a KV cache, as in the reference's tests."""

    def __init__(self, vocab, hidden, cache_dim=4):
        super().__init__()
        self.embedding = nn.Embedding(vocab, hidden)
        self.linear = nn.Linear(hidden, vocab)
        self.cache_dim = cache_dim

    def forward(self, input_ids, past_key_values=None, use_cache=False, attention_mask=None):
        logits = self.linear(self.embedding(input_ids))
        B = input_ids.shape[0]
        kv = ((torch.arange(B, device=input_ids.device, dtype=torch.float).view(B, 1, 1, 1)
               .expand(B, 1, 1, self.cache_dim).clone(),) * 2,)
        return types.SimpleNamespace(logits=logits, past_key_values=kv)


def _trie(seqs, vocab=8, dense=2):
    return CompactCSRTrie.from_sorted_batch(torch.tensor(sorted(seqs), device=DEV), vocab, dense)


@pytest.mark.parametrize("seqs,dense", [(SEQS_5, 2), (SEQS_3, 3), (SEQS_3, 1)])
def test_every_beam_is_a_catalog_item(seqs, dense, cuda_ok):
    torch.manual_seed(0)
    trie = _trie(seqs, dense=dense)
    model = _RandomModel(8, 16).to(DEV)
    B, k, beam = 2, 4, 8
    ids = autoregressive_generate(model, trie, torch.randint(0, 8, (B, 4), device=DEV),
                                  GenerationConfig(steps=len(seqs[0]), k=k, beam_size=beam,
                                                   temperature=0.0))
    assert ids.shape == (B, k, len(seqs[0]))
    idx = torch.tensor(seqs, device=DEV)
    assert (ids.reshape(-1, len(seqs[0])).unsqueeze(1) == idx.unsqueeze(0)).all(-1).any(-1).all()


def test_log_probas_and_cache_reordering(cuda_ok):
    torch.manual_seed(1)
    trie = _trie(SEQS_5)
    model = _RandomModel(8, 16).to(DEV)
    B, k, beam = 2, 3, 6
    state = ConstrainedGenerationState(
        generation_config=GenerationConfig(steps=5, k=k, beam_size=beam, temperature=0.0),
        constraint_state=ConstraintState(0, trie, None))
    ids = torch.randint(0, 8, (B, 4), device=DEV)
    mask = torch.ones(B, 4, dtype=torch.long, device=DEV)
    prev_max = 0.0
    for step in range(5):
        state = decode_one_step(state, model, ids, attention_mask=mask if step == 0 else None)
        gs = state.generation_state
        assert gs.generated_ids.shape == (B, k, step + 1)
        assert gs.log_probas.shape == (B * k,)
        assert (gs.log_probas <= 1e-6).all()
        assert gs.log_probas.max().item() <= prev_max + 1e-6
        prev_max = gs.log_probas.max().item()
        assert gs.attention_mask.shape == (B * k, 4 + step + 1)
        assert gs.past_key_values[0][0].shape[0] == B * k
        ids = gs.generated_ids.reshape(-1, step + 1)[:, -1:]


class _LMHeadModel(nn.Module):
    """A model whose output projection is ``lm_head`` (an ``nn.Linear``); level
    ``l`` feeds ``hidden[l]`` through it (the golden fixture's model)."""

    def __init__(self, hidden, W):
        super().__init__()
        self.lm_head = nn.Linear(W.shape[1], W.shape[0], bias=False).to(W.device, W.dtype)
        with torch.no_grad():
            self.lm_head.weight.copy_(W)
        self.h = hidden
        self.calls = 0

    def forward(self, input_ids, past_key_values=None, attention_mask=None, use_cache=True):
        h = self.h[self.calls]
        self.calls += 1
        return types.SimpleNamespace(logits=self.lm_head(h).unsqueeze(1), past_key_values=None)


@pytest.mark.parametrize("kern", ["topk", "default"])
def test_route_b_matches_reference_golden(kern, cuda_ok):
    """The SparseLinear route (``attr_path="lm_head"``): CSR levels run the
    fused op of ``csr_kernel`` inside the model's projection; ``topk`` scores
    candidates by the log-softmax over the op's top-k logits only.  Pinned to
    the reference's own ``autoregressive_generate`` on the same model."""
    g = load_golden("search_routeb_route_b.npz")
    w = S.WORKLOADS["route_b"]
    dw = WL.make_device_workload(w, DEV)
    model = _LMHeadModel([h.float() for h in dw.hidden], dw.weight.float())
    cfg = GenerationConfig(steps=w.levels, k=w.beams, beam_size=w.topk, temperature=0.0,
                           csr_kernel=kern)
    ids = autoregressive_generate(model, dw.trie, torch.zeros(w.batch, 1, dtype=torch.long,
                                                              device=DEV),
                                  cfg, attr_path="lm_head")
    np.testing.assert_array_equal(ids.cpu().numpy(), g[f"{kern}/generated_ids"])
    from rectokens_b200.modules import SparseLinear

    assert isinstance(model.lm_head, SparseLinear)


def test_route_b_sampling_paths_are_catalog_items(cuda_ok):
    """``csr_kernel="sample"`` (k = beam_size = 1): every CSR level draws one
    Gumbel-max child in the projection; each generated path is an item."""
    w = S.WORKLOADS["route_b"]
    codes = w.make_catalog()
    dw = WL.make_device_workload(w, DEV, trie=WL.build_trie(w, DEV, codes))
    hidden = [dw.hidden[0]] + [h[::w.beams].contiguous() for h in dw.hidden[1:]]
    model = _LMHeadModel([h.float() for h in hidden], dw.weight.float())
    cfg = GenerationConfig(steps=w.levels, k=1, beam_size=1, temperature=0.7, csr_kernel="sample")
    ids = autoregressive_generate(model, dw.trie, torch.zeros(w.batch, 1, dtype=torch.long,
                                                              device=DEV),
                                  cfg, attr_path="lm_head").cpu().numpy().reshape(-1, w.levels)
    items = {tuple(t) for t in S.to_tokens(codes, w.codes).tolist()}
    assert all(tuple(r) in items for r in ids.tolist())


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_candidates_kernel_matches_mask_topk_path(dtype, cuda_ok):
    """``vtnk_beam_candidates_from_logits`` (one pass over the children's
    columns) against the mask op + log-sum-exp + topk + node lookup it
    replaces in ``decode_one_step``, on random full-vocabulary logits at
    every CSR depth of the cfg2 catalog (ties are absent in random data)."""
    from rectokens_b200.decoding.constrained_decoding import _candidates, _candidates_torch

    w = S.WORKLOADS["cfg2"]
    trie = WL.build_trie(w, DEV)
    g = torch.Generator(device=DEV).manual_seed(3)
    cfg = GenerationConfig(steps=w.levels, k=w.beams, beam_size=w.topk, temperature=0.0)
    from rectokens_b200.decoding.beam_search import depth_layout

    for step in range(1, w.levels):
        R = 777
        logits = torch.randn(R, w.vocab, generator=g, device=DEV).to(dtype)
        d = depth_layout(trie)[step]  # node ids of this depth: [node_lo, node_hi)
        cur = torch.randint(d.node_lo, d.node_hi, (R,), generator=g, device=DEV)
        cs = ConstraintState(step, trie, cur)
        a = _candidates(logits, cs, w.topk)
        b = _candidates_torch(logits, cs, cfg, step, 1, False, None, R, w.topk, None)
        torch.testing.assert_close(a[3], b[3].float(), atol=1e-5, rtol=0)
        assert torch.equal(a[1], b[1].float())          # the same logits, in order
        # tokens equal except among equal logits (bf16 has exact ties, whose
        # order torch.topk leaves open; the kernel takes the lower slot)
        diff = a[0] != b[0]
        assert bool((a[1][diff] == b[1].float()[diff]).all())
        assert torch.equal(a[2][~diff], b[2][~diff])
        if dtype == torch.float32:
            assert not bool(diff.any())
