"""The CPU oracle against the reference's golden vectors and known answers
(CPU only).  Fixtures: tests/golden/make_golden.py."""

import numpy as np
import pytest

from conftest import case_names, group, load_golden
from oracle import vtnk_oracle as O
from rectokens_b200 import synthetic as S

TRIE = load_golden("trie_small.npz")
OPS = load_golden("ops_small.npz")


@pytest.mark.parametrize("name", case_names(TRIE))
def test_oracle_builder_matches_reference(name):
    d = group(TRIE, name + "/")
    rp, cv, lmb, masks, states = O.build_sorted_csr(d["sem_ids"], int(d["vocab"]), int(d["dl"]))
    np.testing.assert_array_equal(rp, d["sorted/row_ptrs"])
    np.testing.assert_array_equal(cv, d["sorted/cols_vals"])
    np.testing.assert_array_equal(lmb, d["sorted/lmb"])
    np.testing.assert_array_equal(states, d["sorted/dense_states"])
    for i, m in enumerate(masks):
        np.testing.assert_array_equal(m, d[f"sorted/dense_mask_{i}"])


def test_oracle_builder_catalogs():
    cat = load_golden("trie_catalog.npz")
    for name in ("cfg1", "cfg2"):
        w = S.WORKLOADS[name]
        tok = S.to_tokens(w.make_catalog(), w.codes)
        rp, cv, lmb, masks, states = O.build_sorted_csr(tok, w.vocab, 1)
        np.testing.assert_array_equal(rp, cat[f"{name}/row_ptrs"])
        np.testing.assert_array_equal(cv, cat[f"{name}/cols_vals"])
        np.testing.assert_array_equal(lmb, cat[f"{name}/lmb"])
        np.testing.assert_array_equal(states, cat[f"{name}/dense_states"])
        np.testing.assert_array_equal(masks[0], cat[f"{name}/dense_mask_0"])


def test_known_answer_three_sequences():
    # reference tests/test_trie.py:168-190
    rp, cv, lmb, _, _ = O.build_sorted_csr(np.array([[1, 2, 1], [3, 1, 2], [3, 1, 3]]), 8)
    assert rp.tolist() == [0, 2, 3, 4, 5, 7, 7, 7]
    assert cv[0].tolist() == [1, 3, 2, 1, 1, 2, 3, -1]
    assert cv[1].tolist() == [1, 2, 3, 4, 5, 6, 7, -1]
    # reference tests/test_kernel.py:179-189 (valid_idxs known answers)
    for cur, step, expect in [([0], 0, [[1, 3]]), ([1, 2], 1, [[2], [1]]),
                              ([4], 2, [[2, 3]]), ([3, 4], 2, [[1], [2, 3]])]:
        _, vi, _ = O.csr_children(rp, cv, np.array(cur), lmb[step])
        for row, exp in zip(vi, expect):
            assert sorted(row[row >= 0].tolist()) == exp
            assert (row[row < 0] == -1).all()


@pytest.mark.parametrize("name", case_names(OPS))
def test_oracle_ops_match_reference(name):
    d = group(OPS, name + "/")
    mb = int(d["mb"])
    nn, vi, cl = O.constrained_node_transition(d["logits"], d["row_ptrs"], d["cols_vals"], d["cur"], mb)
    np.testing.assert_array_equal(nn, d["mask_nn"])
    np.testing.assert_array_equal(vi, d["mask_vi"])
    np.testing.assert_array_equal(cl, d["mask_cl"])
    nn, vi, cl = O.fused_linear(d["a"], d["b"], None, d["row_ptrs"], d["cols_vals"], d["cur"], mb)
    np.testing.assert_array_equal(nn, d["sparse_nn"])
    np.testing.assert_array_equal(vi, d["sparse_vi"])
    np.testing.assert_allclose(cl, d["sparse_cl"], atol=1e-4, rtol=0)
    k = int(d["topk_k"])
    _, _, tl, ti = O.fused_topk(d["a"], d["b"], None, d["row_ptrs"], d["cols_vals"], d["cur"], mb, k)
    np.testing.assert_allclose(np.sort(tl, 1), np.sort(d["topk_vals"], 1), atol=1e-4)
    np.testing.assert_array_equal(np.sort(ti, 1), np.sort(d["topk_idxs"], 1))


def test_philox_matches_triton():
    z = load_golden("philox.npz")
    for key in z:
        if not key.startswith("u_"):
            continue
        seed = int(key[2:])
        u = O.rand_uniform(seed, np.arange(z[key].size))
        np.testing.assert_array_equal(u, z[key])
        g = O.gumbel_noise(seed, 1, z[key].size)[0]
        np.testing.assert_allclose(g, z["g_" + key[2:]], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("name", ["cfg1", "cfg2"])
def test_oracle_beam_search_matches_reference(name):
    g = load_golden(f"search_{name}.npz")
    w = S.WORKLOADS[name]
    tok = S.to_tokens(w.make_catalog(), w.codes)
    rp, cv, lmb, _, _ = O.build_sorted_csr(tok, w.vocab, 1)
    if w.dtype == "f32":
        W = S.head_f32(w.seed, w.vocab, w.hidden)
        hid = [S.hidden_f32(w.seed, l, 0, w.rows(l), w.hidden) for l in range(w.levels)]
    else:
        W = S.bf16_bits_to_f32(S.head_bits(w.seed, w.vocab, w.hidden))
        hid = [S.bf16_bits_to_f32(S.hidden_bits(w.seed, l, 0, w.rows(l), w.hidden))
               for l in range(w.levels)]
    ids, logp, node = O.beam_search(hid, W, rp, cv, lmb, w.batch, w.beams, w.topk)
    np.testing.assert_array_equal(ids, g["generated_ids"])
    np.testing.assert_allclose(logp, g["log_probas"], atol=1e-4, rtol=0)
    np.testing.assert_array_equal(node, g["cur_node"])
