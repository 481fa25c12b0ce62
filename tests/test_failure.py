"""Failure detection of the tile kernel, without a GPU fault.

Every mbarrier wait of the tcgen05 tile kernel is bounded in time.  The test
hook ``vtnk_debug_stall_launches`` makes the next launch issue no operand
copies, so its consumers' first waits run out after a short, explicit limit
(``vtnk_set_wait_limit_ns``).  The kernel must then drain, free its tensor
memory and exit; the host reads ``VTNK_ERR_DEVICE`` from ``vtnk_device_status``
and the context stays usable: the next launch is correct.
"""

import numpy as np
import pytest
import torch

from rectokens_b200 import _lib as L
from rectokens_b200 import synthetic as S
from rectokens_b200 import workload as WL
from rectokens_b200.decoding.beam_search import beam_step, sample_step

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture
def short_waits():
    lib = L.lib()
    L.check(lib.vtnk_device_status(1))          # start from a clean record
    L.check(lib.vtnk_set_wait_limit_ns(1_000_000))  # 1 ms
    yield lib
    lib.vtnk_debug_stall_launches(0)
    lib.vtnk_set_wait_limit_ns(0)
    lib.vtnk_device_status(1)


def _expect_expired(lib):
    rc = lib.vtnk_device_status(1)
    assert rc == 4, (rc, lib.vtnk_last_error())   # VTNK_ERR_DEVICE
    assert b"bounded wait expired" in lib.vtnk_last_error()
    L.check(lib.vtnk_device_status(0))          # the reset cleared it


@pytest.mark.parametrize("variant", ["pair_topn", "split_sampling"])
def test_expired_wait_reports_and_recovers(variant, short_waits, cuda_ok):
    lib = short_waits
    w = S.WORKLOADS["cfg2"]
    dw = WL.make_device_workload(w, DEV)
    h = dw.hidden[1][:640]                       # 640 rows: tile kernel (>= 128 rows)
    cur = (torch.arange(640, device=DEV) % 200 + 1)  # depth-1 nodes
    if variant == "pair_topn":
        run = lambda: beam_step(h, dw.weight, dw.trie, 1, cur, 10)  # noqa: E731
        ref = beam_step(h, dw.weight, dw.trie, 1, cur, 10, index=None)
    else:
        t = torch.tensor([0.7], dtype=torch.float32, device=DEV)
        run = lambda: sample_step(h, dw.weight, dw.trie, 1, cur, 3, t)  # noqa: E731
        ref = sample_step(h, dw.weight, dw.trie, 1, cur, 3, t, index=None)
    torch.cuda.synchronize()

    L.check(lib.vtnk_debug_stall_launches(1))
    run()                                         # stalled launch: waits run out
    _expect_expired(lib)

    got = run()                                   # clean launch on the same context
    torch.cuda.synchronize()
    L.check(lib.vtnk_device_status(1))
    if variant == "pair_topn":
        np.testing.assert_array_equal(got[0].cpu().numpy()[:, 0], ref[0].cpu().numpy()[:, 0])
        np.testing.assert_allclose(got[3].cpu().numpy(), ref[3].cpu().numpy(), atol=2e-3)
    else:
        assert (got[0] == ref[0]).float().mean().item() > 0.99


def test_stalled_search_reports(short_waits, cuda_ok):
    """A stalled level inside a fused search: the search returns, the status
    word names the expired wait, and a following search is exact."""
    from rectokens_b200 import constrained_beam_search
    from rectokens_b200.schemas import GenerationConfig

    lib = short_waits
    w = S.WORKLOADS["cfg2"]
    dw = WL.make_device_workload(w, DEV)
    cfg = GenerationConfig(steps=w.levels, k=w.beams, beam_size=w.topk, temperature=0.0)
    good = constrained_beam_search(dw.hidden, dw.weight, dw.trie, cfg)
    torch.cuda.synchronize()
    L.check(lib.vtnk_debug_stall_launches(2))
    constrained_beam_search(dw.hidden, dw.weight, dw.trie, cfg)
    _expect_expired(lib)
    lib.vtnk_debug_stall_launches(0)
    again = constrained_beam_search(dw.hidden, dw.weight, dw.trie, cfg)
    torch.cuda.synchronize()
    L.check(lib.vtnk_device_status(1))
    assert torch.equal(again.generated_ids, good.generated_ids)
    assert torch.equal(again.cur_node, good.cur_node)
