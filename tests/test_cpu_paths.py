"""The two CPU baselines ``bench.py`` times (the reference's sparse-PyTorch
path and its CPU trie path, oracle/cpu_paths.py) reproduce the reference's own
``decode_one_step`` searches (golden, configs 1-2) -- so the CPU numbers in the
bench line time the same search the GPU runs."""

import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import cpu_paths as C
from oracle import vtnk_oracle as O
from rectokens_b200 import synthetic as S


def _inputs(w):
    tok = S.to_tokens(w.make_catalog(), w.codes)
    rp, cv, lmb, _, _ = O.build_sorted_csr(tok, w.vocab, 1)
    if w.dtype == "f32":
        W = S.head_f32(w.seed, w.vocab, w.hidden)
        hid = [S.hidden_f32(w.seed, l, 0, w.rows(l), w.hidden) for l in range(w.levels)]
    else:
        W = S.bf16_bits_to_f32(S.head_bits(w.seed, w.vocab, w.hidden))
        hid = [S.bf16_bits_to_f32(S.hidden_bits(w.seed, l, 0, w.rows(l), w.hidden))
               for l in range(w.levels)]
    return rp, cv, lmb, W, hid


@pytest.mark.parametrize("name", ["cfg1", "cfg2"])
def test_sparse_path_matches_reference(name):
    g = load_golden(f"search_{name}.npz")
    w = S.WORKLOADS[name]
    rp, cv, lmb, W, hid = _inputs(w)
    ids, logp, node = C.sparse_path_search(
        [torch.from_numpy(h) for h in hid], torch.from_numpy(W), torch.from_numpy(rp),
        torch.from_numpy(cv), lmb, w.batch, w.beams, w.topk)
    np.testing.assert_array_equal(ids, g["generated_ids"])
    np.testing.assert_array_equal(node, g["cur_node"])
    np.testing.assert_allclose(logp, g["log_probas"], atol=1e-3, rtol=0)


@pytest.mark.parametrize("name", ["cfg1", "cfg2"])
def test_trie_path_matches_reference(name):
    g = load_golden(f"search_{name}.npz")
    w = S.WORKLOADS[name]
    rp, cv, lmb, W, hid = _inputs(w)
    ids, logp, node = C.trie_path_search(hid, W, C.PointerTrie(rp, cv), lmb, w.batch, w.beams,
                                         w.topk)
    np.testing.assert_array_equal(ids, g["generated_ids"])
    np.testing.assert_array_equal(node, g["cur_node"])
    np.testing.assert_allclose(logp, g["log_probas"], atol=1e-3, rtol=0)
