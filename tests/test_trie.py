"""CompactCSRTrie builders against the reference's own outputs and known
answers (CPU).  Mirrors the reference's tests/test_trie.py."""

import numpy as np
import pytest
import torch

from conftest import case_names, group, load_golden
from rectokens_b200 import synthetic as S
from rectokens_b200.decoding.trie import Trie
from rectokens_b200.schemas import CompactCSRTrie

TRIE = load_golden("trie_small.npz")


def _check(csr, d):
    np.testing.assert_array_equal(csr.row_ptrs.numpy(), d["row_ptrs"])
    np.testing.assert_array_equal(csr.stacked_cols_vals.numpy(), d["cols_vals"])
    assert csr.layer_max_branches == d["lmb"].tolist()
    np.testing.assert_array_equal(csr.dense_states.numpy(), d["dense_states"])
    for i, m in enumerate(csr.dense_mask_by_layer):
        np.testing.assert_array_equal(m.numpy(), d[f"dense_mask_{i}"])
    assert csr.row_ptrs.dtype == torch.int64 and csr.stacked_cols_vals.dtype == torch.int64


@pytest.mark.parametrize("name", case_names(TRIE))
def test_from_sorted_batch_matches_reference(name):
    d = group(TRIE, name + "/")
    csr = CompactCSRTrie.from_sorted_batch(torch.from_numpy(d["sem_ids"]), int(d["vocab"]),
                                           int(d["dl"]))
    _check(csr, group(d, "sorted/"))


@pytest.mark.parametrize("name", case_names(TRIE))
def test_from_trie_matches_reference(name):
    d = group(TRIE, name + "/")
    t = Trie()
    seqs = d["sem_ids"].tolist()
    if name == "rand12":  # the fixture inserted the unsorted draw order
        g = torch.Generator()
        g.manual_seed(0)
        seqs = torch.randint(0, 8, (12, 3), generator=g).tolist()
    for s in seqs:
        t.insert(s)
    csr = CompactCSRTrie.from_trie(t, int(d["vocab"]), int(d["dl"]))
    _check(csr, group(d, "trie/"))


@pytest.mark.parametrize("name", ["cfg1", "cfg2"])
def test_catalog_builder_matches_reference(name):
    g = load_golden("trie_catalog.npz")
    w = S.WORKLOADS[name]
    tok = torch.from_numpy(S.to_tokens(w.make_catalog(), w.codes))
    csr = CompactCSRTrie.from_sorted_batch(tok, vocab_size=w.vocab, dense_lookup_layers=1)
    np.testing.assert_array_equal(csr.row_ptrs.numpy(), g[f"{name}/row_ptrs"])
    np.testing.assert_array_equal(csr.stacked_cols_vals.numpy(), g[f"{name}/cols_vals"])
    assert csr.layer_max_branches == g[f"{name}/lmb"].tolist()
    np.testing.assert_array_equal(csr.dense_states.numpy(), g[f"{name}/dense_states"])


def test_known_answers_multi_branch():
    # reference tests/test_trie.py:159-190
    t = Trie()
    for s in ([1, 2, 1], [3, 1, 2], [3, 1, 3]):
        t.insert(s)
    csr = CompactCSRTrie.from_trie(t, vocab_size=8)
    assert csr.row_ptrs.tolist() == [0, 2, 3, 4, 5, 7, 7, 7]
    assert csr.stacked_cols_vals[0].tolist() == [1, 3, 2, 1, 1, 2, 3, -1]
    assert csr.stacked_cols_vals[1].tolist() == [1, 2, 3, 4, 5, 6, 7, -1]


def test_trie_prefix_queries():
    t = Trie()
    t.insert([1, 2, 3])
    t.insert([1, 2, 7])
    assert sorted(t.find_prefix([1, 2]).children) == [3, 7]
    assert t.find_prefix([9]) is None
    assert t.find_prefix([1, 2, 3]).is_end_of_token


def test_level_windows_cover_children():
    from rectokens_b200 import level_windows

    w = S.WORKLOADS["cfg2"]
    csr = CompactCSRTrie.from_sorted_batch(torch.from_numpy(S.to_tokens(w.make_catalog(), w.codes)),
                                           vocab_size=w.vocab, dense_lookup_layers=1)
    wins = level_windows(csr)
    assert wins == [(l * 256, 256) if l < 3 else wins[3] for l in range(4)]
    lo, n = wins[3]
    assert 768 <= lo and lo + n <= 1024


def test_depth_layout_cache_follows_the_trie():
    import gc

    from rectokens_b200.decoding import beam_search as B

    w = S.WORKLOADS["cfg1"]
    tok = torch.from_numpy(S.to_tokens(w.make_catalog(), w.codes))
    csr = CompactCSRTrie.from_sorted_batch(tok, vocab_size=w.vocab, dense_lookup_layers=1)
    first = B.depth_layout(csr)
    assert B.depth_layout(csr) is first                     # cached
    csr.stacked_cols_vals[0, 0] += 0                         # in-place edit bumps the version
    assert B.depth_layout(csr) is not first
    n = len(B._LAYOUT_CACHE)
    del csr
    gc.collect()
    assert len(B._LAYOUT_CACHE) == n - 1                     # dropped with the trie


@pytest.mark.parametrize("name", case_names(TRIE))
def test_from_codes_sorts_like_the_tokenizer(name):
    """``from_codes`` (any row order, duplicates allowed) equals the sorted
    build, as ``ItemAwareTokenizer.build_item_trie`` sorts before building."""
    d = group(TRIE, name + "/")
    rows = np.concatenate([d["sem_ids"], d["sem_ids"][::2]])
    rows = rows[np.random.default_rng(2).permutation(rows.shape[0])]
    csr = CompactCSRTrie.from_codes(torch.from_numpy(rows), int(d["vocab"]), int(d["dl"]))
    _check(csr, group(d, "sorted/"))
