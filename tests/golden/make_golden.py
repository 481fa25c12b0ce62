"""Generate the golden fixtures in this folder from the reference implementation.

Run in a container where the reference (EdoardoBotta/RecTokens) is checked out:

    python tests/golden/make_golden.py --reference /path/to/RecTokens

It imports the reference's own Python code and records its outputs:

* ``trie_*.npz``    -- ``CompactCSRTrie.from_sorted_batch`` / ``from_trie``
  (rectokens/schemas/compact_csr_trie.py) on hand-written and seeded catalogs.
* ``ops_small.npz`` -- ``vtnk_pytorch`` (mask op), ``sparse_linear_pytorch``
  (fused op) and the top-k recipe of the reference's kernel test
  (``vtnk_pytorch(a @ b)`` + ``torch.topk``, tests/test_kernel.py:211-245).
* ``search_cfg1.npz`` / ``search_cfg2.npz`` -- full beam searches through the
  reference's unmodified ``decode_one_step``
  (rectokens/decoding/constrained_decoding.py:194-398).  The reference's
  Triton kernel module asserts a GPU at import, so a stand-in module that
  routes ``_constrained_node_transition_op`` to the reference's own
  ``vtnk_pytorch`` is placed in ``sys.modules`` first (the reference's kernel
  test pins the Triton op to ``vtnk_pytorch`` exactly, tests/test_kernel.py:73-75).
  The model is a stub whose logits at level ``l`` are ``hidden_l @ W.T`` in
  fp32, with the seeded synthetic hidden states / head of
  ``rectokens_b200.synthetic``.
* ``search_routeb_route_b.npz`` -- the same search through the reference's
  ``SparseLinear`` route (``autoregressive_generate(..., attr_path="lm_head")``,
  ``GenerationConfig.csr_kernel`` "topk" and "default"), whose CSR levels call
  the fused ops from ``SparseLinear.forward`` (rectokens/modules/
  sparse_linear.py:47-98) and score candidates as route B of
  ``decode_one_step`` does (constrained_decoding.py:281-293: for "topk" the
  log-softmax over the returned top-k logits only).  The stand-in module
  computes the fused ops with the reference's ``sparse_linear_pytorch``
  (+ ``torch.topk`` as kernels:816-852).  ``SparseLinear`` passes the weight
  untransposed where the ops expect ``W.T``; the stand-in takes the operand
  for what it is (the ``(N, H)`` weight), i.e. the search the route is meant
  to run.
* ``philox.npz``    -- ``tl.rand`` and the Gumbel transform of the reference's
  sampling kernel (kernels:359-380) evaluated by Triton's CPU interpreter.

Nothing at test time reads the reference; the tests read these files only.
"""

from __future__ import annotations

import argparse
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def _install_kernel_stub():
    import torch
    from rectokens.decoding.vntk import vtnk_pytorch

    class _TrieView:
        def __init__(self, row_ptrs, cols_vals, mb):
            self.row_ptrs = row_ptrs
            self.stacked_cols_vals = cols_vals
            self.layer_max_branches = [mb]

    def _mask_op(logits, cur_node, row_ptrs, cols_vals, max_branches):
        return vtnk_pytorch(logits, cur_node, _TrieView(row_ptrs, cols_vals, max_branches), 0)

    from rectokens.decoding.vntk import sparse_linear_pytorch

    def _weight(a, b):
        # SparseLinear hands over the (N, H) weight itself (see the module docstring)
        return b if b.shape[1] == a.shape[1] else b.T

    def _fused_op(a, b, bias_val, cur_node, row_ptrs, cols_vals, max_branches, has_bias):
        W = _weight(a, b).float()
        nn_, vi, cl = sparse_linear_pytorch(a.float(), W, cur_node,
                                            _TrieView(row_ptrs, cols_vals, max_branches), 0)
        if has_bias:
            cl = torch.where(cl > float("-inf"), cl + bias_val.float(), cl)
        return nn_, vi, cl

    def _topk_op(a, b, bias_val, cur_node, row_ptrs, cols_vals, max_branches, has_bias, k):
        # kernels:816-852: per-branch logits in a -inf padded [B, mb] buffer,
        # torch.topk, then valid_idxs.gather
        nn_, vi, cl = _fused_op(a, b, bias_val, cur_node, row_ptrs, cols_vals, max_branches,
                                has_bias)
        branch = torch.where(vi >= 0, cl.gather(1, vi.clamp(min=0)), float("-inf"))
        tl_, ti = torch.topk(branch, k, dim=-1)
        return nn_, vi, tl_, vi.gather(1, ti)

    stub = types.ModuleType("rectokens.kernels.constrained_node_transition")
    stub._constrained_node_transition_op = _mask_op
    stub._fused_linear_constrained_node_transition_op = _fused_op
    stub._fused_linear_constrained_node_transition_topk_op = _topk_op
    stub._fused_linear_constrained_node_transition_sampling_op = None
    sys.modules["rectokens.kernels.constrained_node_transition"] = stub


def trie_fixtures(out: Path):
    import torch
    from rectokens.decoding.trie import Trie
    from rectokens.schemas.compact_csr_trie import CompactCSRTrie

    def pack(prefix, csr, d):
        d[prefix + "row_ptrs"] = csr.row_ptrs.numpy()
        d[prefix + "cols_vals"] = csr.stacked_cols_vals.numpy()
        d[prefix + "lmb"] = np.array(csr.layer_max_branches, dtype=np.int64)
        d[prefix + "dense_states"] = csr.dense_states.numpy()
        for i, m in enumerate(csr.dense_mask_by_layer):
            d[prefix + f"dense_mask_{i}"] = m.numpy()

    cases = {
        "three": ([[1, 2, 1], [3, 1, 2], [3, 1, 3]], 8, 2),
        "chain": ([[1, 2, 3]], 8, 2),
        "branch": ([[1, 2, 3], [1, 2, 7]], 8, 2),
        "zero": ([[0, 1, 2], [0, 3, 0], [2, 0, 1]], 4, 2),
        "single": ([[42]], 50, 1),
    }
    g = torch.Generator()
    g.manual_seed(0)
    rand12 = torch.randint(0, 8, (12, 3), generator=g).tolist()
    cases["rand12"] = (rand12, 8, 2)
    d = {}
    for name, (seqs, vocab, dl) in cases.items():
        s = sorted(seqs)
        d[f"{name}/sem_ids"] = np.array(s, dtype=np.int64)
        d[f"{name}/vocab"] = np.array(vocab)
        d[f"{name}/dl"] = np.array(dl)
        pack(f"{name}/sorted/", CompactCSRTrie.from_sorted_batch(
            torch.tensor(s, dtype=torch.long), vocab_size=vocab, dense_lookup_layers=dl), d)
        t = Trie()
        for row in seqs:  # insertion order as given
            t.insert(row)
        pack(f"{name}/trie/", CompactCSRTrie.from_trie(t, vocab_size=vocab, dense_lookup_layers=dl), d)
    np.savez_compressed(out / "trie_small.npz", **d)

    # catalog-scale builder output (cfg1, cfg2): store a digest-sized subset
    from rectokens_b200 import synthetic as S
    d = {}
    for name in ("cfg1", "cfg2"):
        w = S.WORKLOADS[name]
        tok = S.to_tokens(w.make_catalog(), w.codes)
        csr = CompactCSRTrie.from_sorted_batch(torch.from_numpy(tok), vocab_size=w.vocab,
                                               dense_lookup_layers=1)
        d[f"{name}/row_ptrs"] = csr.row_ptrs.numpy()
        d[f"{name}/cols_vals"] = csr.stacked_cols_vals.numpy()
        d[f"{name}/lmb"] = np.array(csr.layer_max_branches, dtype=np.int64)
        d[f"{name}/dense_states"] = csr.dense_states.numpy()
        d[f"{name}/dense_mask_0"] = csr.dense_mask_by_layer[0].numpy()
    np.savez_compressed(out / "trie_catalog.npz", **d)


def ops_fixtures(out: Path):
    import torch
    from rectokens.decoding.vntk import sparse_linear_pytorch, vtnk_pytorch
    from rectokens.schemas.compact_csr_trie import CompactCSRTrie

    d = {}
    csr = CompactCSRTrie.from_sorted_batch(
        torch.tensor(sorted([[1, 2, 1], [3, 1, 2], [3, 1, 3]])), vocab_size=8)
    dense = CompactCSRTrie.from_sorted_batch(
        torch.tensor(sorted([[i, j, k] for i in range(4) for j in range(4) for k in range(4)])),
        vocab_size=16)
    cases = [
        # (name, trie, B, K, step, cur_node)  -- the reference's own test cases
        ("b1s0", csr, 1, 16, 0, [0]),
        ("b2s0", csr, 2, 16, 0, [0, 0]),
        ("b2s1", csr, 2, 16, 1, [1, 2]),
        ("b3s2", csr, 3, 16, 2, [3, 4, 3]),
        ("b4s1", csr, 4, 16, 1, [1, 2, 1, 2]),
        ("b8bigk", csr, 8, 128, 0, [0] * 8),
        ("b256s0", csr, 256, 16, 0, [0] * 256),
        ("dense_s0", dense, 32, 24, 0, [0] * 32),
        ("dense_s1", dense, 32, 24, 1, [1, 2, 3, 4] * 8),
        ("dense_s2", dense, 32, 24, 2, list(range(5, 21)) * 2),
    ]
    for name, trie, B, K, step, cur in cases:
        torch.manual_seed(1000 + B + K + step)
        N = trie.vocab_size
        a = torch.randn(B, K)
        b = torch.randn(K, N)
        bias = torch.randn(N)
        cur_t = torch.tensor(cur, dtype=torch.long)
        logits = a @ b
        nn, vi, cl = vtnk_pytorch(logits, cur_t, trie, step)
        snn, svi, scl = sparse_linear_pytorch(a, b.T.contiguous(), cur_t, trie, step)
        k = min(2, trie.layer_max_branches[step])
        tv, ti_raw = torch.topk(cl, k, dim=-1)
        ti = torch.where(tv > float("-inf"), ti_raw, torch.full_like(ti_raw, -1))
        p = f"{name}/"
        d[p + "row_ptrs"] = trie.row_ptrs.numpy()
        d[p + "cols_vals"] = trie.stacked_cols_vals.numpy()
        d[p + "mb"] = np.array(trie.layer_max_branches[step])
        d[p + "a"] = a.numpy()
        d[p + "b"] = b.numpy()
        d[p + "bias"] = bias.numpy()
        d[p + "cur"] = cur_t.numpy()
        d[p + "logits"] = logits.numpy()
        d[p + "mask_nn"] = nn.numpy()
        d[p + "mask_vi"] = vi.numpy()
        d[p + "mask_cl"] = cl.numpy()
        d[p + "sparse_nn"] = snn.numpy()
        d[p + "sparse_vi"] = svi.numpy()
        d[p + "sparse_cl"] = scl.numpy()
        d[p + "topk_k"] = np.array(k)
        d[p + "topk_vals"] = tv.numpy()
        d[p + "topk_idxs"] = ti.numpy()
    np.savez_compressed(out / "ops_small.npz", **d)


class _StubLM:
    """Logits at level ``l`` = ``hidden[l] @ W.T`` (fp32), one call per level."""

    def __init__(self, hidden_levels, W):
        import torch

        self.h = [torch.from_numpy(np.asarray(h, dtype=np.float32)) for h in hidden_levels]
        self.W = torch.from_numpy(np.asarray(W, dtype=np.float32))
        self.calls = 0

    def __call__(self, input_ids, past_key_values=None, attention_mask=None, use_cache=True):
        h = self.h[self.calls]
        assert h.shape[0] == input_ids.shape[0], (h.shape, input_ids.shape)
        self.calls += 1
        logits = (h @ self.W.T).unsqueeze(1)
        return types.SimpleNamespace(logits=logits, past_key_values=None)


def search_fixture(out: Path, name: str):
    import torch
    from rectokens.decoding.constrained_decoding import decode_one_step
    from rectokens.schemas.compact_csr_trie import CompactCSRTrie
    from rectokens.schemas.config import GenerationConfig
    from rectokens.schemas.state import ConstrainedGenerationState, ConstraintState

    from rectokens_b200 import synthetic as S

    w = S.WORKLOADS[name]
    tok = S.to_tokens(w.make_catalog(), w.codes)
    trie = CompactCSRTrie.from_sorted_batch(torch.from_numpy(tok), vocab_size=w.vocab,
                                            dense_lookup_layers=1)
    if w.dtype == "f32":
        W = S.head_f32(w.seed, w.vocab, w.hidden)
        hidden = [S.hidden_f32(w.seed, l, 0, w.rows(l), w.hidden) for l in range(w.levels)]
    else:
        W = S.bf16_bits_to_f32(S.head_bits(w.seed, w.vocab, w.hidden))
        hidden = [S.bf16_bits_to_f32(S.hidden_bits(w.seed, l, 0, w.rows(l), w.hidden))
                  for l in range(w.levels)]
    model = _StubLM(hidden, W)
    state = ConstrainedGenerationState(
        generation_config=GenerationConfig(steps=w.levels, k=w.beams, beam_size=w.topk,
                                           temperature=0.0),
        constraint_state=ConstraintState(step=0, trie=trie, cur_node=None),
    )
    input_ids = torch.zeros(w.batch, 1, dtype=torch.long)
    for _ in range(w.levels):
        state = decode_one_step(constrained_generation_state=state, model_fwd=model,
                                input_ids=input_ids)
        gen = state.generation_state.generated_ids
        input_ids = gen.reshape(-1, gen.shape[-1])[:, -1:]
    gs = state.generation_state
    np.savez_compressed(
        out / f"search_{name}.npz",
        generated_ids=gs.generated_ids.numpy(),
        log_probas=gs.log_probas.numpy(),
        cur_node=state.constraint_state.cur_node.numpy(),
        lmb=np.array(trie.layer_max_branches, dtype=np.int64),
        n_nodes=np.array(trie.row_ptrs.numel()),
    )


class _StubLMHead:
    """A model whose output projection is an ``nn.Linear`` named ``lm_head``
    (the SparseLinear route replaces it): level ``l`` feeds ``hidden[l]``
    through it, one call per level."""

    def __new__(cls, hidden_levels, W):
        import torch
        from torch import nn

        class M(nn.Module):
            def __init__(self):
                super().__init__()
                self.lm_head = nn.Linear(W.shape[1], W.shape[0], bias=False)
                with torch.no_grad():
                    self.lm_head.weight.copy_(torch.from_numpy(np.asarray(W, np.float32)))
                self.h = [torch.from_numpy(np.asarray(h, dtype=np.float32))
                          for h in hidden_levels]
                self.calls = 0

            def forward(self, input_ids, past_key_values=None, attention_mask=None,
                        use_cache=True):
                h = self.h[self.calls]
                self.calls += 1
                return types.SimpleNamespace(logits=self.lm_head(h).unsqueeze(1),
                                             past_key_values=None)

        return M()


def routeb_fixture(out: Path, name: str):
    import torch
    from rectokens.decoding.constrained_decoding import autoregressive_generate
    from rectokens.schemas.compact_csr_trie import CompactCSRTrie
    from rectokens.schemas.config import GenerationConfig

    from rectokens_b200 import synthetic as S

    w = S.WORKLOADS[name]
    tok = S.to_tokens(w.make_catalog(), w.codes)
    trie = CompactCSRTrie.from_sorted_batch(torch.from_numpy(tok), vocab_size=w.vocab,
                                            dense_lookup_layers=1)
    W = S.bf16_bits_to_f32(S.head_bits(w.seed, w.vocab, w.hidden))
    hidden = [S.bf16_bits_to_f32(S.hidden_bits(w.seed, l, 0, w.rows(l), w.hidden))
              for l in range(w.levels)]
    d = {}
    for kern in ("topk", "default"):
        model = _StubLMHead(hidden, W)
        cfg = GenerationConfig(steps=w.levels, k=w.beams, beam_size=w.topk, temperature=0.0,
                               csr_kernel=kern)
        ids = autoregressive_generate(model, trie, torch.zeros(w.batch, 1, dtype=torch.long),
                                      cfg, attr_path="lm_head")
        d[f"{kern}/generated_ids"] = ids.numpy()
    np.savez_compressed(out / f"search_routeb_{name}.npz", **d)


def philox_fixture(out: Path):
    code = r'''
import os, sys
os.environ["TRITON_INTERPRET"] = "1"
import numpy as np, torch, triton, triton.language as tl

@triton.jit
def k(out, seed, n, BLOCK: tl.constexpr):
    offs = tl.program_id(0) * BLOCK + tl.arange(0, BLOCK)
    u = tl.rand(seed, offs)
    g = -tl.log(-tl.log(u + 1e-10) + 1e-10)
    tl.store(out + offs, u, mask=offs < n)
    tl.store(out + n + offs, g, mask=offs < n)

n = 4096
res = {}
for seed in (0, 7, 12345, 2**31 - 1, 2**33 + 5):
    o = torch.empty(2 * n)
    k[(n // 256,)](o, seed, n, BLOCK=256)
    res[f"u_{seed}"] = o[:n].numpy().copy()
    res[f"g_{seed}"] = o[n:].numpy().copy()
np.savez_compressed(sys.argv[1], **res)
'''
    import subprocess

    subprocess.run([sys.executable, "-c", code, str(out / "philox.npz")], check=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("RECTOKENS_REFERENCE", ""))
    args = ap.parse_args()
    if args.reference:
        sys.path.insert(0, args.reference)
    sys.path.insert(0, str(REPO))
    _install_kernel_stub()
    trie_fixtures(HERE)
    ops_fixtures(HERE)
    for name in ("cfg1", "cfg2"):
        search_fixture(HERE, name)
    routeb_fixture(HERE, "route_b")
    philox_fixture(HERE)
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
