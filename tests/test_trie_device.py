"""The device trie builder (sort / scan / segment kernels, vtnk_trie_count +
vtnk_trie_fill) against the reference's own builder outputs (golden) and the
CPU builder at catalog scale, up to the 16M-item target catalog (GPU)."""

import time

import numpy as np
import pytest
import torch

from conftest import case_names, group, load_golden
from oracle import vtnk_oracle as O
from rectokens_b200 import synthetic as S
from rectokens_b200.schemas import CompactCSRTrie

pytestmark = pytest.mark.gpu
TRIE = load_golden("trie_small.npz")


def _check(csr, d):
    np.testing.assert_array_equal(csr.row_ptrs.cpu().numpy(), d["row_ptrs"])
    np.testing.assert_array_equal(csr.stacked_cols_vals.cpu().numpy(), d["cols_vals"])
    assert csr.layer_max_branches == d["lmb"].tolist()
    np.testing.assert_array_equal(csr.dense_states.cpu().numpy(), d["dense_states"])
    assert len(csr.dense_mask_by_layer) == sum(1 for k in d if k.startswith("dense_mask_"))
    for i, m in enumerate(csr.dense_mask_by_layer):
        np.testing.assert_array_equal(m.cpu().numpy(), d[f"dense_mask_{i}"])
    assert csr.row_ptrs.is_cuda and csr.row_ptrs.dtype == torch.int64


@pytest.mark.parametrize("name", case_names(TRIE))
def test_device_builder_matches_reference(name, cuda_ok):
    d = group(TRIE, name + "/")
    sem = torch.from_numpy(d["sem_ids"]).cuda()
    csr = CompactCSRTrie.from_sorted_batch(sem, int(d["vocab"]), int(d["dl"]))
    _check(csr, group(d, "sorted/"))


@pytest.mark.parametrize("name", case_names(TRIE))
def test_device_sort_matches_reference(name, cuda_ok):
    """Shuffled rows with duplicates: the radix sort restores the order the
    reference's builder needs, duplicates open no nodes."""
    d = group(TRIE, name + "/")
    rows = np.concatenate([d["sem_ids"], d["sem_ids"][::2]])
    rows = rows[np.random.default_rng(1).permutation(rows.shape[0])]
    csr = CompactCSRTrie.from_codes(torch.from_numpy(rows).cuda(), int(d["vocab"]), int(d["dl"]))
    _check(csr, group(d, "sorted/"))


@pytest.mark.parametrize("name", ["cfg1", "cfg2"])
def test_device_catalog_matches_reference(name, cuda_ok):
    g = load_golden("trie_catalog.npz")
    w = S.WORKLOADS[name]
    tok = torch.from_numpy(S.to_tokens(w.make_catalog(), w.codes)).cuda()
    csr = CompactCSRTrie.from_sorted_batch(tok, vocab_size=w.vocab, dense_lookup_layers=1)
    np.testing.assert_array_equal(csr.row_ptrs.cpu().numpy(), g[f"{name}/row_ptrs"])
    np.testing.assert_array_equal(csr.stacked_cols_vals.cpu().numpy(), g[f"{name}/cols_vals"])
    assert csr.layer_max_branches == g[f"{name}/lmb"].tolist()
    np.testing.assert_array_equal(csr.dense_states.cpu().numpy(), g[f"{name}/dense_states"])
    np.testing.assert_array_equal(csr.dense_mask_by_layer[0].cpu().numpy(),
                                  g[f"{name}/dense_mask_0"])


@pytest.mark.parametrize("name", ["cfg3", "cfg5"])
def test_device_builder_at_catalog_scale(name, cuda_ok):
    """Config 3 (1M items) and the 16M-item target catalog: the device build
    (sorted input, and shuffled input through the radix sort) equals the CPU
    restatement of the reference's builder; build times are printed."""
    w = S.WORKLOADS[name]
    tok_np = S.to_tokens(w.make_catalog(), w.codes)
    rp, cv, lmb, masks, states = O.build_sorted_csr(tok_np, w.vocab, 1)
    tok = torch.from_numpy(tok_np).cuda()
    shuf = tok[torch.randperm(tok.shape[0], device="cuda", generator=torch.Generator(
        device="cuda").manual_seed(0))]
    for label, build in (("sorted", lambda: CompactCSRTrie.from_sorted_batch(tok, w.vocab, 1)),
                         ("shuffled", lambda: CompactCSRTrie.from_codes(shuf, w.vocab, 1))):
        build()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        csr = build()
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        print(f"\n{name} device trie build ({label}, {tok.shape[0]} items): {dt * 1e3:.1f} ms")
        assert torch.equal(csr.row_ptrs.cpu(), torch.from_numpy(rp))
        assert torch.equal(csr.stacked_cols_vals.cpu(), torch.from_numpy(cv))
        assert csr.layer_max_branches == list(lmb)
        assert torch.equal(csr.dense_states.cpu(), torch.from_numpy(states))
        assert torch.equal(csr.dense_mask_by_layer[0].cpu(), torch.from_numpy(masks[0]))


def test_device_builder_edge_cases(cuda_ok):
    # empty catalog: the root alone (reference layout: row_ptrs [0], one sentinel)
    csr = CompactCSRTrie.from_sorted_batch(torch.zeros((0, 3), dtype=torch.long, device="cuda"),
                                           8, 1)
    assert csr.row_ptrs.tolist() == [0]
    assert csr.stacked_cols_vals.tolist() == [[-1], [-1]]
    assert csr.layer_max_branches == [0, 0, 0]
    # a token outside [0, vocab_size) is rejected
    with pytest.raises(ValueError):
        CompactCSRTrie.from_sorted_batch(torch.tensor([[1, 9]], device="cuda"), 8, 1)
    # one level only
    one = CompactCSRTrie.from_codes(torch.tensor([[5], [2], [5]], device="cuda"), 8, 1)
    ref = CompactCSRTrie.from_sorted_batch(torch.tensor([[2], [5], [5]]), 8, 1)
    assert one.row_ptrs.tolist() == ref.row_ptrs.tolist()
    assert one.stacked_cols_vals.tolist() == ref.stacked_cols_vals.tolist()
    assert one.layer_max_branches == ref.layer_max_branches
