"""The allocation-free search entry point (GPU).

vtnk_beam_search_noalloc serves callers that may not allocate device memory
while decoding -- a plugin whose host process owns all GPU memory through
its own pool, or code that must not risk the device synchronisation an
allocation can cause.  It takes its scratch from an array built into the
library instead of a caller workspace.  This file is collected last, so a
failure here never hides the other tests, and it passes both alone in a
fresh process and after the rest of the suite.
"""

import ctypes

import numpy as np
import pytest
import torch

from rectokens_b200 import _lib as L
from rectokens_b200 import synthetic as S
from rectokens_b200 import workload as WL
from rectokens_b200.decoding.beam_search import _search_struct, constrained_beam_search
from rectokens_b200.schemas import GenerationConfig

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_noalloc_search_matches_workspace_search(cuda_ok):
    w = S.WORKLOADS["cfg2"]
    dw = WL.make_device_workload(w, DEV)
    cfg = GenerationConfig(steps=w.levels, k=w.beams, beam_size=w.topk, temperature=0.0)
    ref = constrained_beam_search(dw.hidden, dw.weight, dw.trie, cfg)
    keep: list = []
    s = _search_struct(dw.hidden, dw.weight, None, dw.trie, w.beams, w.topk, True, keep)
    B, k, Lv = w.batch, w.beams, w.levels
    for _ in range(2):  # two calls in a row share (and reuse) the built-in scratch
        ids = torch.full((B * k, Lv), -7, dtype=torch.int64, device=DEV)
        logp = torch.full((B * k,), 7.0, dtype=torch.float32, device=DEV)
        node = torch.full((B * k,), -7, dtype=torch.int64, device=DEV)
        L.check(L.lib().vtnk_beam_search_noalloc(
            ctypes.byref(s), ids.data_ptr(), logp.data_ptr(), node.data_ptr(),
            L.stream_of(ids.device)))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(ids.view(B, k, Lv).cpu().numpy(),
                                      ref.generated_ids.cpu().numpy())
        np.testing.assert_array_equal(node.cpu().numpy(), ref.cur_node.cpu().numpy())
        np.testing.assert_allclose(logp.cpu().numpy(), ref.log_probas.cpu().numpy(),
                                   atol=1e-3, rtol=0)


def test_noalloc_search_rejects_oversized_requests(cuda_ok):
    w = S.WORKLOADS["cfg2"]
    dw = WL.make_device_workload(w, DEV)
    keep: list = []
    s = _search_struct(dw.hidden, dw.weight, None, dw.trie, w.beams, w.topk, True, keep)
    s.batch = 1 << 22  # scratch need far above the built-in array; rejected before any launch
    assert L.lib().vtnk_beam_search_workspace_bytes(ctypes.byref(s)) > 32 << 20
    rc = L.lib().vtnk_beam_search_noalloc(ctypes.byref(s), None, None, None, None)
    assert rc == 3
    assert b"scratch" in L.lib().vtnk_last_error()
