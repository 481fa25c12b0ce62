"""Batch-parallel beam search across GPUs (one process per GPU).

Queries are independent, so the batch shards into contiguous query ranges:
every rank holds the full trie and head rows, generates (or receives) the
hidden states of its own queries -- global row ``q`` at level 0 and rows
``q*k .. q*k+k-1`` after -- runs the search locally, and the per-rank results
are concatenated with one all-gather (NCCL over NVLink on GPUs; gloo works
the same way on CPU tensors).  There is no other exchange.

The three result tensors of a rank travel as one packed record
``[ids int64 (b*k*L) | node int64 (b*k) | logp fp32 (b*k), padded to 16 B]``
so that the gather is a single collective: ``ResultRecord`` allocates a
rank's tensors as views of its record (the search writes them in place, no
packing copy) and the gathered buffer is read through rank-strided views.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_queries(batch: int, rank: int, world: int) -> tuple[int, int]:
    """``(first_query, n_queries)`` of ``rank``'s contiguous shard."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world")
    if batch % world:
        raise ValueError(f"batch {batch} does not divide evenly across {world} ranks")
    per = batch // world
    return rank * per, per


def level_rows(first_query: int, n_queries: int, level: int, beams: int) -> tuple[int, int]:
    """Global ``(first_row, rows)`` of a shard's hidden states at ``level``."""
    per_q = 1 if level == 0 else beams
    return first_query * per_q, n_queries * per_q


class ResultRecord:
    """One rank's search results ``(ids (n, L) int64, logp (n,) fp32, node (n,)
    int64)`` as views of a single byte buffer, ``n = b*k`` rows."""

    def __init__(self, n: int, levels: int, device):
        self.n, self.levels = n, levels
        self.ids_bytes = n * levels * 8
        self.node_bytes = n * 8
        self.logp_bytes = n * 4
        used = self.ids_bytes + self.node_bytes + self.logp_bytes
        self.nbytes = (used + 15) // 16 * 16
        self.buf = torch.zeros((self.nbytes,), dtype=torch.uint8, device=device)
        self.ids, self.node, self.logp = self.views(self.buf.view(1, -1))
        self.ids, self.node, self.logp = self.ids[0], self.node[0], self.logp[0]

    def views(self, rec: torch.Tensor):
        """``(ids (R, n, L), node (R, n), logp (R, n))`` views of ``R`` records
        laid out back to back (``rec``: ``(R, nbytes)`` uint8)."""
        a, b = self.ids_bytes, self.ids_bytes + self.node_bytes
        ids = rec[:, :a].view(torch.int64).view(rec.shape[0], self.n, self.levels)
        node = rec[:, a:b].view(torch.int64)
        logp = rec[:, b:b + self.logp_bytes].view(torch.float32)
        return ids, node, logp

    def gather(self, group=None, out: torch.Tensor | None = None):
        """All-gather the records of every rank (one collective).  Returns
        ``(ids (world, n, L), logp (world, n), node (world, n))`` views of the
        gathered buffer; rank r's rows are queries of shard r, in order."""
        world = dist.get_world_size(group)
        if out is None:
            out = self.buf.new_empty((world * self.nbytes,))
        dist.all_gather_into_tensor(out, self.buf, group=group)
        ids, node, logp = self.views(out.view(world, self.nbytes))
        return ids, logp, node


def gather_results(ids: torch.Tensor, logp: torch.Tensor, node: torch.Tensor, group=None,
                   out=None):
    """All-gather each rank's ``(ids (b*k, L), logp (b*k,), node (b*k,))`` into the
    full-batch tensors in rank order (pre-allocated ``out`` may be passed).
    The three tensors are packed into one record and gathered with a single
    collective."""
    world = dist.get_world_size(group)
    if (ids.dtype, logp.dtype, node.dtype) != (torch.int64, torch.float32, torch.int64):
        if out is None:  # other dtypes: one collective per tensor
            out = (ids.new_empty((ids.shape[0] * world,) + tuple(ids.shape[1:])),
                   logp.new_empty((logp.shape[0] * world,)),
                   node.new_empty((node.shape[0] * world,)))
        for dst, src in zip(out, (ids, logp, node)):
            dist.all_gather_into_tensor(dst, src.contiguous(), group=group)
        return out
    rec = ResultRecord(ids.shape[0], ids.shape[1], ids.device)
    rec.ids.copy_(ids)
    rec.logp.copy_(logp)
    rec.node.copy_(node)
    g_ids, g_logp, g_node = rec.gather(group)
    if out is None:
        out = (ids.new_empty((ids.shape[0] * world,) + tuple(ids.shape[1:])),
               logp.new_empty((logp.shape[0] * world,)),
               node.new_empty((node.shape[0] * world,)))
    out[0].view(world, ids.shape[0], -1).copy_(g_ids)
    out[1].view(world, -1).copy_(g_logp)
    out[2].view(world, -1).copy_(g_node)
    return out


class ShardFailure(RuntimeError):
    """A rank's local search failed; raised on every rank of the group."""


def checked_gather(rec: ResultRecord, local_error: BaseException | None = None, group=None,
                   out: torch.Tensor | None = None):
    """``rec.gather`` preceded by one agreement step, so that a failure on one
    rank ends the search on every rank instead of leaving the others blocked
    in the gather: each rank contributes ``rank + 1`` if its local search
    raised (``local_error``) and 0 otherwise; after a MAX all-reduce every
    rank raises ``ShardFailure`` naming the highest failing rank, or all
    proceed to the gather.  A rank that never arrives (it died or hangs) is
    caught by the process group's timeout, which makes the collective raise
    on the others.  Costs one small collective; the benchmark's timed search
    uses the plain gather."""
    rank = dist.get_rank(group)
    dev = rec.buf.device
    flag = torch.tensor([rank + 1 if local_error is not None else 0], dtype=torch.int32,
                        device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=group)
    failed = int(flag.item())
    if failed:
        msg = f"rank {failed - 1} failed before the result gather"
        if local_error is not None:
            raise ShardFailure(msg) from local_error
        raise ShardFailure(msg)
    return rec.gather(group=group, out=out)


def sharded_search(search_fn, n_rows: int, levels: int, device, group=None):
    """Run ``search_fn() -> (ids (n, L), logp (n,), node (n,))`` on this rank's
    shard and all-gather every rank's results with ``checked_gather``.
    Returns the gathered ``(ids (world, n, L), logp (world, n), node (world, n))``."""
    rec = ResultRecord(n_rows, levels, device)
    err = None
    try:
        ids, logp, node = search_fn()
        rec.ids.copy_(ids.reshape(n_rows, levels))
        rec.logp.copy_(logp)
        rec.node.copy_(node)
    except Exception as e:  # noqa: BLE001 -- reported to every rank, then re-raised
        err = e
    return checked_gather(rec, err, group=group)


class PeerGather:
    """All-gather of the ranks' search results over peer memory (NVLink):
    ``vtnk_peer_gather`` pushes this rank's packed record (int32 ids and
    nodes, fp32 log-probs: 20 bytes per beam at 3 levels, against 36 in the
    NCCL record) into every rank's buffer with plain 16-byte stores, then the
    ranks meet at a flag barrier -- one kernel, no NCCL call.  Buffers are
    exchanged once through CUDA IPC (one process per GPU, world <= 8)."""

    def __init__(self, n: int, levels: int, device, group=None, wait_ns: int = 0):
        import ctypes

        from rectokens_b200 import _lib as L

        self.L = L
        lib = L.lib()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("peer gather supports up to 8 ranks")
        self.n, self.levels = n, levels
        self.rb = lib.vtnk_peer_record_bytes(n, levels)
        dev = torch.device(device)
        self.buf = torch.zeros((2 * self.world * self.rb,), dtype=torch.uint8, device=dev)
        self.flags = torch.zeros((8,), dtype=torch.int32, device=dev)
        self.ctl = torch.zeros((4,), dtype=torch.int32, device=dev)  # epoch, ticket, status
        torch.cuda.synchronize(dev)
        hb = lib.vtnk_ipc_handle_bytes()

        def handle(t):
            h = (ctypes.c_uint8 * hb)()
            off = ctypes.c_int64()
            L.check(lib.vtnk_ipc_get_handle(t.data_ptr(), h, ctypes.byref(off)))
            return bytes(h), off.value

        mine = (handle(self.buf), handle(self.flags))
        allh = [None] * self.world
        dist.all_gather_object(allh, mine, group=group)
        self._opened = []
        g = L.PeerGroup()
        g.world, g.rank, g.record_bytes = self.world, self.rank, self.rb
        for r, ((hbuf, obuf), (hfl, ofl)) in enumerate(allh):
            if r == self.rank:
                g.records[r] = self.buf.data_ptr()
                g.flags[r] = self.flags.data_ptr()
                continue
            ptrs = []
            for h, off in ((hbuf, obuf), (hfl, ofl)):
                p = ctypes.c_void_p()
                L.check(lib.vtnk_ipc_open_handle((ctypes.c_uint8 * hb).from_buffer_copy(h),
                                                 ctypes.byref(p)))
                self._opened.append(p.value)
                ptrs.append(p.value + off)
            g.records[r], g.flags[r] = ptrs
        g.epoch = self.ctl.data_ptr()
        g.status = self.ctl[2:].data_ptr()
        g.wait_ns = wait_ns
        self.group = g
        self.calls = 0
        dist.barrier(group=group)

    def push(self, ids: torch.Tensor, logp: torch.Tensor, node: torch.Tensor, stream=None):
        """Launch the push + barrier kernel on ``stream`` (current stream by default)."""
        s = self.L.stream_of(self.buf.device) if stream is None else stream
        self.L.check(self.L.lib().vtnk_peer_gather(self.group, ids.data_ptr(), logp.data_ptr(),
                                                  node.data_ptr(), self.n, self.levels, s))
        self.calls += 1

    def result(self):
        """``(ids (world, n, L) int32, logp (world, n) fp32, node (world, n) int32)``
        views of the latest completed gather (reads the device epoch), and the
        status word (0 ok, 1 a wait ran out, 2 an id did not fit int32)."""
        ctl = self.ctl.cpu().tolist()
        half = ctl[0] & 1
        w, n, Lv, rb = self.world, self.n, self.levels, self.rb
        rec = self.buf.view(2, w, rb)[half]
        off_node = (n * Lv * 4 + 15) // 16 * 16
        off_logp = off_node + (n * 4 + 15) // 16 * 16
        ids = rec[:, :n * Lv * 4].contiguous().view(torch.int32).view(w, n, Lv)
        node = rec[:, off_node:off_node + n * 4].contiguous().view(torch.int32)
        logp = rec[:, off_logp:off_logp + n * 4].contiguous().view(torch.float32)
        return ids, logp, node, ctl[2]

    def close(self):
        lib = self.L.lib()
        for p in self._opened:
            lib.vtnk_ipc_close_handle(p)
        self._opened = []
