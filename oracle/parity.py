"""Parity checks of whole searches against the CPU oracle -- TEST
INFRASTRUCTURE ONLY (used by ``tests/`` and by ``bench.py``'s parity report,
never by the product path).

The oracle (``oracle/vtnk_oracle.py``) is pinned to the reference's own
``decode_one_step`` runs; these helpers run it on a strided sample of a large
search's queries, regenerating the sample's hidden states from the seeded
generator, and count exact matches and documented near-ties.
"""

from __future__ import annotations

import numpy as np


def hidden_rows(w, level, rows) -> np.ndarray:
    """fp64 copies of the given global hidden-state rows of ``level``."""
    from rectokens_b200 import synthetic as S

    if w.dtype == "f32":
        return np.concatenate([S.hidden_f32(w.seed, level, int(r), 1, w.hidden)
                               for r in rows]).astype(np.float64)
    return np.concatenate([S.bf16_bits_to_f32(S.hidden_bits(w.seed, level, int(r), 1, w.hidden))
                           for r in rows]).astype(np.float64)


def parity_sample(batch: int, n: int = 512) -> np.ndarray:
    """Strided query sample: first and last queries, both ends of every
    region, ``n`` queries in all (all of them for small batches)."""
    if batch <= n:
        return np.arange(batch)
    q = np.unique(np.linspace(0, batch - 1, n).round().astype(np.int64))
    return np.unique(np.concatenate([q, [0, 1, batch // 2, batch - 2, batch - 1]]))


def check_search(w, rp, cv, lmb, W64, queries, ids, logp, node, rel=1e-3):
    """The GPU search results of ``queries`` (``ids (q, k, L)``, ``logp (q*k,)``,
    ``node (q*k,)``) against the oracle's search of the same queries."""
    from oracle import vtnk_oracle as O

    k = w.beams
    hid = []
    for level in range(w.levels):
        per = 1 if level == 0 else k
        rows = (queries[:, None] * per + np.arange(per)[None, :]).reshape(-1)
        hid.append(hidden_rows(w, level, rows))
    oids, ologp, onode = O.beam_search(hid, W64, rp, cv, lmb, len(queries), k, w.topk)
    q_ok = (ids.reshape(len(queries), -1) == oids.reshape(len(queries), -1)).all(1) & (
        node.reshape(len(queries), k) == onode.reshape(len(queries), k)).all(1)
    d = np.abs(logp.reshape(len(queries), k) - ologp.reshape(len(queries), k))
    # a query that differs must do so through a near-tie: its sorted scores
    # still agree with the oracle's within the tie tolerance
    scale = np.maximum(1.0, np.abs(ologp.reshape(len(queries), k)))
    near = (d <= rel * scale).all(1)
    return {"queries": int(len(queries)), "exact": int(q_ok.sum()),
            "near_tie": int((~q_ok & near).sum()), "mismatch": int((~q_ok & ~near).sum()),
            "max_abs_logp_diff_exact": float(d[q_ok].max()) if q_ok.any() else None,
            "tolerance": f"ids/nodes bit-exact except near-ties within {rel} relative; "
                         f"logp within {rel}"}


def check_sampling(w, rp, cv, lmb, W64, queries, tok, node, noise_fn, q0=0):
    """Sampled search of ``queries`` against the oracle's Gumbel-max given the
    kernel's own noise (``noise_fn(level, rows)``), level by level on the
    GPU's samples; returns exact / near-tie counts.  ``queries`` are rows of
    this rank's shard (the kernel's noise offsets), ``q0`` its first global
    query (the hidden-state generator's row index)."""
    from oracle import vtnk_oracle as O

    exact = near = bad = 0
    cur = np.zeros(len(queries), dtype=np.int64)
    for level in range(w.levels):
        mb = lmb[level]
        a = hidden_rows(w, level, np.asarray(queries) + q0)
        noise = noise_fn(level, queries, mb)
        nn, vi, osmp, score = O.fused_sampling(a, W64.T, None, rp, cv, cur, mb, noise,
                                               w.temperature)
        got = tok[:, level]
        for r in range(len(queries)):
            if got[r] == int(osmp[r]):
                exact += 1
                continue
            slot = np.nonzero(vi[r] == got[r])[0]
            if slot.size == 1 and score[r, slot[0]] >= np.max(score[r]) - 1e-3 * max(
                    1.0, abs(np.max(score[r]))):
                near += 1
            else:
                bad += 1
        # follow the GPU's samples (teacher-forced) to the next level
        nxt = np.full_like(cur, -1)
        for r in range(len(queries)):
            j = np.nonzero(vi[r] == got[r])[0]
            nxt[r] = nn[r, j[0]] if j.size else -1
        cur = nxt
    ok_nodes = bool((cur == node).all())
    return {"samples": int(len(queries) * w.levels), "exact": exact, "near_tie": near,
            "mismatch": bad, "final_node_walk_ok": ok_nodes,
            "tolerance": "sampled tokens bit-exact given the kernel's noise, except score "
                         "near-ties within 1e-3 relative"}
