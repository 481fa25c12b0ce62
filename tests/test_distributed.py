"""Batch sharding + all-gather of the beam search (CPU, two gloo ranks).

Each rank searches its contiguous query shard with the CPU oracle, using the
hidden states of its global rows; the gathered result must equal the
single-process search of the whole batch (the GPU bench does the same with the
CUDA search and NCCL)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rectokens_b200 import distributed as D
from rectokens_b200 import synthetic as S


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _inputs(w, q0, nq):
    hid = []
    for level in range(w.levels):
        r0, rows = D.level_rows(q0, nq, level, w.beams)
        hid.append(S.hidden_f32(w.seed, level, r0, rows, w.hidden))
    return hid


def _worker(rank, world, port, q):
    from oracle import vtnk_oracle as O

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = S.WORKLOADS["cfg1"]
        w = type(w)(**{**w.__dict__, "batch": 8})
        tok = S.to_tokens(w.make_catalog(), w.codes)
        rp, cv, lmb, _, _ = O.build_sorted_csr(tok, w.vocab, 1)
        W = S.head_f32(w.seed, w.vocab, w.hidden)
        q0, nq = D.shard_queries(w.batch, rank, world)
        ids, logp, node = O.beam_search(_inputs(w, q0, nq), W, rp, cv, lmb, nq, w.beams, w.topk)
        out = D.gather_results(torch.from_numpy(ids.reshape(nq * w.beams, -1)),
                               torch.from_numpy(logp), torch.from_numpy(node))
        # the packed single-collective path (fp32 log-probs)
        lp32 = torch.from_numpy(logp).float()
        out32 = D.gather_results(torch.from_numpy(ids.reshape(nq * w.beams, -1)), lp32,
                                 torch.from_numpy(node))
        rec = D.ResultRecord(nq * w.beams, w.levels, "cpu")
        rec.ids.copy_(torch.from_numpy(ids.reshape(nq * w.beams, -1)))
        rec.logp.copy_(lp32)
        rec.node.copy_(torch.from_numpy(node))
        r_ids, r_logp, r_node = rec.gather()
        assert torch.equal(r_ids.reshape(-1, w.levels), out32[0])
        assert torch.equal(r_logp.reshape(-1), out32[1])
        assert torch.equal(r_node.reshape(-1), out32[2])
        assert torch.equal(out32[0], out[0]) and torch.equal(out32[2], out[2])
        assert torch.equal(out32[1], out[1].float())
        if rank == 0:
            full = O.beam_search(_inputs(w, 0, w.batch), W, rp, cv, lmb, w.batch, w.beams, w.topk)
            q.put((out[0].numpy(), out[1].numpy(), out[2].numpy(),
                   full[0].reshape(w.batch * w.beams, -1), full[1], full[2]))
    finally:
        dist.destroy_process_group()


def test_sharded_search_equals_single_process():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    g_ids, g_logp, g_node, f_ids, f_logp, f_node = res
    np.testing.assert_array_equal(g_ids, f_ids)
    np.testing.assert_array_equal(g_node, f_node)
    np.testing.assert_allclose(g_logp, f_logp, rtol=0, atol=1e-6)


def _fault_worker(rank, world, port, mode, q):
    """One rank of a two-rank search with an injected host-side failure:
    ``before``  rank 1 raises inside its local search (before the gather);
    ``after``   rank 1 raises after a successful gather;
    ``absent``  rank 1 never joins the gather (exits), so rank 0's collective
                must end by the process group's timeout, not hang."""
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    out = "ok"
    try:
        n, levels = 4, 3

        def search():
            if mode == "before" and rank == 1:
                raise ValueError("injected failure in the local search")
            return (torch.full((n, levels), rank, dtype=torch.int64),
                    torch.full((n,), -1.0 * rank), torch.full((n,), 10 + rank, dtype=torch.int64))

        if mode == "absent" and rank == 1:
            q.put((rank, "left"))
            q.close()
            q.join_thread()  # flush before leaving without any teardown
            os._exit(0)
        try:
            ids, logp, node = D.sharded_search(search, n, levels, "cpu")
            assert ids.shape == (world, n, levels)
            assert torch.equal(node[:, 0], torch.tensor([10, 11]))
            if mode == "after" and rank == 1:
                raise ValueError("injected failure after the gather")
        except D.ShardFailure as e:
            out = f"ShardFailure: {e}"
        except ValueError as e:
            out = f"ValueError: {e}"
        except RuntimeError as e:  # the process group's timeout
            out = f"RuntimeError: {type(e).__name__}"
        q.put((rank, out))
    finally:
        if mode != "absent":
            dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["before", "after", "absent"])
def test_rank_failures_end_the_search(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fault_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=90) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            raise AssertionError("a rank hung")
    if mode == "before":
        assert got[0].startswith("ShardFailure: rank 1 failed"), got
        assert got[1].startswith("ShardFailure: rank 1 failed"), got
    elif mode == "after":
        assert got[0] == "ok" and got[1].startswith("ValueError"), got
    else:
        assert got[1] == "left"
        assert got[0].startswith("RuntimeError"), got


def test_shard_arithmetic():
    assert D.shard_queries(65536, 3, 8) == (24576, 8192)
    assert D.level_rows(24576, 8192, 0, 10) == (24576, 8192)
    assert D.level_rows(24576, 8192, 2, 10) == (245760, 81920)
    with pytest.raises(ValueError):
        D.shard_queries(10, 0, 3)
