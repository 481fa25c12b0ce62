"""``vtnk::`` custom ops backed by libvtnk_b200 (CUDA, sm_100a).

Same op names and positional arguments as the reference's
``torch.library.triton_op`` registrations
(rectokens/kernels/constrained_node_transition.py:14-61, 388-447, 562-635,
791-853): functional ops that allocate their outputs and never mutate inputs.
Each op launches exactly one kernel on the current CUDA stream and does not
synchronise the host.
"""

from __future__ import annotations

import time
from typing import Optional

import torch
from torch import Tensor

from rectokens_b200 import _lib as L


def _require_cuda(*ts: Tensor) -> torch.device:
    dev = ts[0].device
    if dev.type != "cuda":
        raise RuntimeError("vtnk ops run on CUDA tensors only (no CPU fallback)")
    for t in ts[1:]:
        if t.device != dev:
            raise RuntimeError(f"all tensors must be on {dev}, got {t.device}")
    return dev


def _bias_arg(a: Tensor, bias_val: Tensor, has_bias: bool) -> Optional[Tensor]:
    if not has_bias:
        return None
    return bias_val.to(a.dtype).contiguous()


@torch.library.custom_op("vtnk::_constrained_node_transition_op", mutates_args=())
def _constrained_node_transition_op(
    logits: Tensor,
    cur_node: Tensor,
    csr_row_ptrs: Tensor,
    csr_cols_vals: Tensor,
    max_branches: int,
) -> tuple[Tensor, Tensor, Tensor]:
    B, N = logits.shape
    assert cur_node.shape == (B,), f"Expected cur_node shape ({B},), got {cur_node.shape}"
    dev = _require_cuda(logits, cur_node, csr_row_ptrs, csr_cols_vals)
    logits = logits if logits.stride(1) == 1 else logits.contiguous()
    cur_node = cur_node.contiguous()
    csr_cols_vals = csr_cols_vals.contiguous()
    corrected = torch.empty((B, N), dtype=logits.dtype, device=dev)
    next_node = torch.empty((B, max_branches), dtype=torch.int64, device=dev)
    valid_idxs = torch.empty((B, max_branches), dtype=torch.int64, device=dev)
    csr = L.csr_struct(csr_row_ptrs.contiguous(), csr_cols_vals)
    L.check(L.lib().vtnk_constrained_node_transition(
        logits.data_ptr(), L.DTYPE_CODE[logits.dtype], B, N, max(logits.stride(0), N),
        cur_node.data_ptr(), csr, max_branches, corrected.data_ptr(), next_node.data_ptr(),
        valid_idxs.data_ptr(), L.stream_of(dev)))
    return next_node, valid_idxs, corrected


@_constrained_node_transition_op.register_fake
def _(logits, cur_node, csr_row_ptrs, csr_cols_vals, max_branches):
    B, N = logits.shape
    return (cur_node.new_empty(B, max_branches), cur_node.new_empty(B, max_branches),
            torch.empty_like(logits))


@torch.library.custom_op("vtnk::_fused_linear_constrained_node_transition_op", mutates_args=())
def _fused_linear_constrained_node_transition_op(
    a: Tensor,
    b: Tensor,
    bias_val: Tensor,
    cur_node: Tensor,
    csr_row_ptrs: Tensor,
    csr_cols_vals: Tensor,
    max_branches: int,
    has_bias: bool,
) -> tuple[Tensor, Tensor, Tensor]:
    B = a.shape[0]
    N = b.shape[1]
    assert cur_node.shape == (B,), f"Expected cur_node shape (B,), got {cur_node.shape}"
    dev = _require_cuda(a, b, cur_node, csr_row_ptrs, csr_cols_vals)
    a = a.contiguous()
    cur_node = cur_node.contiguous()
    bias = _bias_arg(a, bias_val, has_bias)
    corrected = torch.empty((B, N), dtype=torch.float32, device=dev)
    next_node = torch.empty((B, max_branches), dtype=torch.int64, device=dev)
    valid_idxs = torch.empty((B, max_branches), dtype=torch.int64, device=dev)
    lin = L.linear_struct(a, b, bias)
    csr = L.csr_struct(csr_row_ptrs.contiguous(), csr_cols_vals.contiguous())
    L.check(L.lib().vtnk_fused_linear_constrained_node_transition(
        lin, cur_node.data_ptr(), csr, max_branches, corrected.data_ptr(), next_node.data_ptr(),
        valid_idxs.data_ptr(), L.stream_of(dev)))
    return next_node, valid_idxs, corrected


@_fused_linear_constrained_node_transition_op.register_fake
def _(a, b, bias_val, cur_node, csr_row_ptrs, csr_cols_vals, max_branches, has_bias):
    B, N = a.shape[0], b.shape[1]
    return (cur_node.new_empty(B, max_branches), cur_node.new_empty(B, max_branches),
            a.new_empty((B, N), dtype=torch.float32))


@torch.library.custom_op("vtnk::_fused_linear_constrained_node_transition_topk_op",
                         mutates_args=())
def _fused_linear_constrained_node_transition_topk_op(
    a: Tensor,
    b: Tensor,
    bias_val: Tensor,
    cur_node: Tensor,
    csr_row_ptrs: Tensor,
    csr_cols_vals: Tensor,
    max_branches: int,
    has_bias: bool,
    k: int,
) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    B = a.shape[0]
    assert cur_node.shape == (B,), f"Expected cur_node shape ({B},), got {cur_node.shape}"
    if not 1 <= k <= max_branches:
        raise RuntimeError(f"selected index k out of range (k={k}, max_branches={max_branches})")
    dev = _require_cuda(a, b, cur_node, csr_row_ptrs, csr_cols_vals)
    a = a.contiguous()
    cur_node = cur_node.contiguous()
    bias = _bias_arg(a, bias_val, has_bias)
    next_node = torch.empty((B, max_branches), dtype=torch.int64, device=dev)
    valid_idxs = torch.empty((B, max_branches), dtype=torch.int64, device=dev)
    topk_logits = torch.empty((B, k), dtype=torch.float32, device=dev)
    topk_idxs = torch.empty((B, k), dtype=torch.int64, device=dev)
    lin = L.linear_struct(a, b, bias)
    csr = L.csr_struct(csr_row_ptrs.contiguous(), csr_cols_vals.contiguous())
    L.check(L.lib().vtnk_fused_linear_constrained_node_transition_topk(
        lin, cur_node.data_ptr(), csr, max_branches, k, next_node.data_ptr(),
        valid_idxs.data_ptr(), topk_logits.data_ptr(), topk_idxs.data_ptr(), L.stream_of(dev)))
    return next_node, valid_idxs, topk_logits, topk_idxs


@_fused_linear_constrained_node_transition_topk_op.register_fake
def _(a, b, bias_val, cur_node, csr_row_ptrs, csr_cols_vals, max_branches, has_bias, k):
    B = a.shape[0]
    return (cur_node.new_empty(B, max_branches), cur_node.new_empty(B, max_branches),
            a.new_empty((B, k), dtype=torch.float32), cur_node.new_empty(B, k))


@torch.library.custom_op("vtnk::_fused_linear_constrained_node_transition_sampling_op",
                         mutates_args=())
def _fused_linear_constrained_node_transition_sampling_op(
    a: Tensor,
    b: Tensor,
    bias_val: Tensor,
    cur_node: Tensor,
    csr_row_ptrs: Tensor,
    csr_cols_vals: Tensor,
    max_branches: int,
    has_bias: bool,
    rng_seed: int,
    temperature: Tensor,
) -> tuple[Tensor, Tensor, Tensor]:
    B = a.shape[0]
    assert cur_node.shape == (B,), f"Expected cur_node shape ({B},), got {cur_node.shape}"
    dev = _require_cuda(a, b, cur_node, csr_row_ptrs, csr_cols_vals, temperature)
    a = a.contiguous()
    cur_node = cur_node.contiguous()
    bias = _bias_arg(a, bias_val, has_bias)
    temperature = temperature.to(torch.float32).reshape(-1)[:1].contiguous()
    next_node = torch.empty((B, max_branches), dtype=torch.int64, device=dev)
    valid_idxs = torch.empty((B, max_branches), dtype=torch.int64, device=dev)
    sample = torch.empty((B,), dtype=torch.float32, device=dev)
    lin = L.linear_struct(a, b, bias)
    csr = L.csr_struct(csr_row_ptrs.contiguous(), csr_cols_vals.contiguous())
    L.check(L.lib().vtnk_fused_linear_constrained_node_transition_sampling(
        lin, cur_node.data_ptr(), csr, max_branches, rng_seed & 0xFFFFFFFFFFFFFFFF,
        temperature.data_ptr(), next_node.data_ptr(), valid_idxs.data_ptr(), sample.data_ptr(),
        L.stream_of(dev)))
    return next_node, valid_idxs, sample


@_fused_linear_constrained_node_transition_sampling_op.register_fake
def _(a, b, bias_val, cur_node, csr_row_ptrs, csr_cols_vals, max_branches, has_bias, rng_seed,
      temperature):
    B = a.shape[0]
    return (cur_node.new_empty(B, max_branches), cur_node.new_empty(B, max_branches),
            a.new_empty((B,), dtype=torch.float32))


def default_seed() -> int:
    """The reference's default sampling seed (kernels:577-578)."""
    return time.time_ns() & 0x7FFFFFFF


def gumbel_noise(rng_seed: int, rows: int, max_branches: int, device) -> Tensor:
    """The noise ``g[row, slot]`` the sampling op adds for this seed (for
    replaying a sampling call in a checker)."""
    out = torch.empty((rows, max_branches), dtype=torch.float32, device=device)
    L.check(L.lib().vtnk_gumbel_noise(rng_seed & 0xFFFFFFFFFFFFFFFF, rows, max_branches,
                                      out.data_ptr(), L.stream_of(out.device)))
    return out


# ---------------------------------------------------------------- tile-kernel variants
# The same ops with the trie depth's child-bitmask index as extra arguments:
# the logits of the depth's 256-token window are computed by the tcgen05 tile
# kernel and reduced in its epilogue (top-k, or Gumbel-max sampling).  The
# ops layer calls these when the depth has an index; the library falls back
# to the warp-per-row kernel when the shape is not tile-able.


def _index_struct(masks: Tensor, node_lo: int, node_hi: int, window_lo: int, window_n: int):
    return L.ChildIndex(masks.data_ptr(), node_lo, node_hi, window_lo, window_n)


@torch.library.custom_op("vtnk::_fused_linear_constrained_node_transition_topk_ix_op",
                         mutates_args=())
def _fused_linear_constrained_node_transition_topk_ix_op(
    a: Tensor,
    b: Tensor,
    bias_val: Tensor,
    cur_node: Tensor,
    csr_row_ptrs: Tensor,
    csr_cols_vals: Tensor,
    index_masks: Tensor,
    node_lo: int,
    node_hi: int,
    window_lo: int,
    window_n: int,
    max_branches: int,
    has_bias: bool,
    k: int,
) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    B = a.shape[0]
    assert cur_node.shape == (B,), f"Expected cur_node shape ({B},), got {cur_node.shape}"
    if not 1 <= k <= max_branches:
        raise RuntimeError(f"selected index k out of range (k={k}, max_branches={max_branches})")
    dev = _require_cuda(a, b, cur_node, csr_row_ptrs, csr_cols_vals, index_masks)
    a = a.contiguous()
    cur_node = cur_node.contiguous()
    bias = _bias_arg(a, bias_val, has_bias)
    next_node = torch.empty((B, max_branches), dtype=torch.int64, device=dev)
    valid_idxs = torch.empty((B, max_branches), dtype=torch.int64, device=dev)
    topk_logits = torch.empty((B, k), dtype=torch.float32, device=dev)
    topk_idxs = torch.empty((B, k), dtype=torch.int64, device=dev)
    lin = L.linear_struct(a, b, bias)
    csr = L.csr_struct(csr_row_ptrs.contiguous(), csr_cols_vals.contiguous())
    ci = _index_struct(index_masks, node_lo, node_hi, window_lo, window_n)
    L.check(L.lib().vtnk_fused_linear_constrained_node_transition_topk_ix(
        lin, cur_node.data_ptr(), csr, max_branches, k, ci, next_node.data_ptr(),
        valid_idxs.data_ptr(), topk_logits.data_ptr(), topk_idxs.data_ptr(), L.stream_of(dev)))
    return next_node, valid_idxs, topk_logits, topk_idxs


@_fused_linear_constrained_node_transition_topk_ix_op.register_fake
def _(a, b, bias_val, cur_node, csr_row_ptrs, csr_cols_vals, index_masks, node_lo, node_hi,
      window_lo, window_n, max_branches, has_bias, k):
    B = a.shape[0]
    return (cur_node.new_empty(B, max_branches), cur_node.new_empty(B, max_branches),
            a.new_empty((B, k), dtype=torch.float32), cur_node.new_empty(B, k))


@torch.library.custom_op("vtnk::_fused_linear_constrained_node_transition_sampling_ix_op",
                         mutates_args=())
def _fused_linear_constrained_node_transition_sampling_ix_op(
    a: Tensor,
    b: Tensor,
    bias_val: Tensor,
    cur_node: Tensor,
    csr_row_ptrs: Tensor,
    csr_cols_vals: Tensor,
    index_masks: Tensor,
    node_lo: int,
    node_hi: int,
    window_lo: int,
    window_n: int,
    max_branches: int,
    has_bias: bool,
    rng_seed: int,
    temperature: Tensor,
) -> tuple[Tensor, Tensor, Tensor]:
    B = a.shape[0]
    assert cur_node.shape == (B,), f"Expected cur_node shape (B,), got {cur_node.shape}"
    dev = _require_cuda(a, b, cur_node, csr_row_ptrs, csr_cols_vals, temperature, index_masks)
    a = a.contiguous()
    cur_node = cur_node.contiguous()
    bias = _bias_arg(a, bias_val, has_bias)
    temperature = temperature.to(torch.float32).reshape(-1)[:1].contiguous()
    next_node = torch.empty((B, max_branches), dtype=torch.int64, device=dev)
    valid_idxs = torch.empty((B, max_branches), dtype=torch.int64, device=dev)
    sample = torch.empty((B,), dtype=torch.float32, device=dev)
    lin = L.linear_struct(a, b, bias)
    csr = L.csr_struct(csr_row_ptrs.contiguous(), csr_cols_vals.contiguous())
    ci = _index_struct(index_masks, node_lo, node_hi, window_lo, window_n)
    L.check(L.lib().vtnk_fused_linear_constrained_node_transition_sampling_ix(
        lin, cur_node.data_ptr(), csr, max_branches, rng_seed & 0xFFFFFFFFFFFFFFFF,
        temperature.data_ptr(), ci, next_node.data_ptr(), valid_idxs.data_ptr(),
        sample.data_ptr(), None, L.stream_of(dev)))
    return next_node, valid_idxs, sample


@_fused_linear_constrained_node_transition_sampling_ix_op.register_fake
def _(a, b, bias_val, cur_node, csr_row_ptrs, csr_cols_vals, index_masks, node_lo, node_hi,
      window_lo, window_n, max_branches, has_bias, rng_seed, temperature):
    B = a.shape[0]
    return (cur_node.new_empty(B, max_branches), cur_node.new_empty(B, max_branches),
            a.new_empty((B,), dtype=torch.float32))
