"""ctypes binding of libvtnk_b200.so (the C ABI declared in include/vtnk_b200.h).

There is no fallback: if the library is missing or was built without the
CUDA kernels, every op raises.  Build it with ``python -m rectokens_b200.csrc.build``.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_uint64, c_void_p
from pathlib import Path

import torch

import os

# VTNK_LIB_PATH: load another build of the library (tuning builds)
LIB_PATH = Path(os.environ.get("VTNK_LIB_PATH") or
                Path(__file__).resolve().with_name("libvtnk_b200.so"))

F32, BF16, F16 = 0, 1, 2
DTYPE_CODE = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}

EXPORTS = (
    "vtnk_constrained_node_transition",
    "vtnk_fused_linear_constrained_node_transition",
    "vtnk_fused_linear_constrained_node_transition_topk",
    "vtnk_fused_linear_constrained_node_transition_sampling",
    "vtnk_fused_linear_constrained_node_transition_topk_ix",
    "vtnk_fused_linear_constrained_node_transition_sampling_ix",
    "vtnk_gumbel_noise",
    "vtnk_build_child_index",
    "vtnk_beam_step",
    "vtnk_beam_merge",
    "vtnk_beam_candidates_from_logits",
    "vtnk_beam_search_workspace_bytes",
    "vtnk_beam_search",
    "vtnk_beam_search_noalloc",
    "vtnk_synth_normal",
    "vtnk_trie_workspace_bytes",
    "vtnk_trie_count",
    "vtnk_trie_fill",
    "vtnk_peer_record_bytes",
    "vtnk_peer_gather",
    "vtnk_ipc_handle_bytes",
    "vtnk_ipc_get_handle",
    "vtnk_ipc_open_handle",
    "vtnk_ipc_close_handle",
    "vtnk_device_status",
    "vtnk_set_wait_limit_ns",
    "vtnk_debug_stall_launches",
    "vtnk_last_error",
    "vtnk_version",
)


class Csr(ctypes.Structure):
    _fields_ = [("row_ptrs", c_void_p), ("cols", c_void_p), ("vals", c_void_p),
                ("n_nodes", c_int64), ("nnz", c_int64)]


class Linear(ctypes.Structure):
    _fields_ = [("a", c_void_p), ("rows", c_int64), ("hidden", c_int64), ("a_stride", c_int64),
                ("b", c_void_p), ("n_vocab", c_int64), ("b_stride_k", c_int64),
                ("b_stride_n", c_int64), ("bias", c_void_p), ("dtype", c_int32)]


class ChildIndex(ctypes.Structure):
    _fields_ = [("masks", c_void_p), ("node_lo", c_int64), ("node_hi", c_int64),
                ("window_lo", c_int64), ("window_n", c_int64), ("flags", c_void_p)]


class Search(ctypes.Structure):
    _fields_ = [("hidden", POINTER(c_void_p)), ("hidden_stride", c_int64), ("weight", c_void_p),
                ("n_vocab", c_int64), ("hidden_dim", c_int64), ("bias", c_void_p),
                ("dtype", c_int32), ("csr", Csr), ("layer_max_branches", POINTER(c_int64)),
                ("index", POINTER(ChildIndex)),
                ("levels", c_int64), ("batch", c_int64), ("beams", c_int64), ("n_cand", c_int64)]


class PeerGroup(ctypes.Structure):
    _fields_ = [("world", c_int32), ("rank", c_int32), ("record_bytes", c_int64),
                ("records", c_void_p * 8), ("flags", c_void_p * 8), ("epoch", c_void_p),
                ("status", c_void_p), ("wait_ns", c_uint64)]


_lib = None


def lib() -> ctypes.CDLL:
    """Load the library once; raise if it is absent."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built; run `python -m rectokens_b200.csrc.build` "
                "(the CUDA kernels are required -- there is no CPU fallback)")
        L = ctypes.CDLL(str(LIB_PATH))
        P, I64, V = c_void_p, c_int64, c_void_p
        sig = {
            "vtnk_constrained_node_transition":
                [P, c_int32, I64, I64, I64, P, POINTER(Csr), I64, P, P, P, V],
            "vtnk_fused_linear_constrained_node_transition":
                [POINTER(Linear), P, POINTER(Csr), I64, P, P, P, V],
            "vtnk_fused_linear_constrained_node_transition_topk":
                [POINTER(Linear), P, POINTER(Csr), I64, I64, P, P, P, P, V],
            "vtnk_fused_linear_constrained_node_transition_sampling":
                [POINTER(Linear), P, POINTER(Csr), I64, c_uint64, P, P, P, P, V],
            "vtnk_fused_linear_constrained_node_transition_topk_ix":
                [POINTER(Linear), P, POINTER(Csr), I64, I64, POINTER(ChildIndex), P, P, P, P, V],
            "vtnk_fused_linear_constrained_node_transition_sampling_ix":
                [POINTER(Linear), P, POINTER(Csr), I64, c_uint64, P, POINTER(ChildIndex), P, P,
                 P, P, V],
            "vtnk_gumbel_noise": [c_uint64, I64, I64, P, V],
            "vtnk_build_child_index": [POINTER(Csr), POINTER(ChildIndex), V],
            "vtnk_beam_step": [POINTER(Linear), P, POINTER(Csr), I64, I64, POINTER(ChildIndex),
                               P, P, P, P, V],
            "vtnk_beam_merge": [I64, I64, I64, I64, P, P, P, P, P, P, P, P, P, P, V],
            "vtnk_beam_candidates_from_logits": [P, c_int32, I64, I64, I64, P, POINTER(Csr), I64,
                                                 I64, P, P, P, P, V],
            "vtnk_beam_search": [POINTER(Search), P, c_size_t, P, P, P, V],
            "vtnk_beam_search_noalloc": [POINTER(Search), P, P, P, V],
            "vtnk_synth_normal": [c_uint64, c_uint64, I64, I64, I64, P, c_int32, P, V],
            "vtnk_trie_count": [P, I64, I64, I64, c_int, P, c_size_t, P, V],
            "vtnk_trie_fill": [I64, I64, I64, I64, P, c_size_t, I64, I64, P, P, P,
                               POINTER(c_void_p), P, V],
        }
        for name, args in sig.items():
            fn = getattr(L, name, None)
            if fn is None:  # an older tuning build (VTNK_LIB_PATH) lacks newer entry points
                continue
            fn.argtypes = args
            fn.restype = c_int
        other = {  # name: (argtypes, restype)
            "vtnk_peer_record_bytes": ([I64, I64], c_int64),
            "vtnk_peer_gather": ([POINTER(PeerGroup), P, P, P, I64, I64, V], c_int),
            "vtnk_ipc_handle_bytes": ([], c_int),
            "vtnk_ipc_get_handle": ([P, P, POINTER(c_int64)], c_int),
            "vtnk_ipc_open_handle": ([P, POINTER(c_void_p)], c_int),
            "vtnk_ipc_close_handle": ([P], c_int),
            "vtnk_trie_workspace_bytes": ([I64, I64], c_size_t),
            "vtnk_beam_search_workspace_bytes": ([POINTER(Search)], c_size_t),
            "vtnk_set_wait_limit_ns": ([c_uint64], c_int),
            "vtnk_debug_stall_launches": ([c_int], c_int),
            "vtnk_device_status": ([c_int], c_int),
            "vtnk_last_error": ([], c_char_p),
            "vtnk_version": ([], c_int),
        }
        for name, (args, res) in other.items():
            fn = getattr(L, name, None)
            if fn is not None:
                fn.argtypes = args
                fn.restype = res
        _lib = L
    return _lib


class VtnkError(RuntimeError):
    pass


def check(rc: int) -> None:
    if rc != 0:
        msg = lib().vtnk_last_error().decode(errors="replace")
        if rc == 1:
            raise ValueError(f"vtnk: {msg}")
        raise VtnkError(f"vtnk error {rc}: {msg}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def csr_struct(row_ptrs: torch.Tensor, cols_vals: torch.Tensor) -> Csr:
    """C view of a CompactCSRTrie's arrays (both int64 on the launch device)."""
    if row_ptrs.dtype != torch.int64 or cols_vals.dtype != torch.int64:
        raise TypeError("trie row_ptrs / stacked_cols_vals must be int64")
    if cols_vals.dim() != 2 or cols_vals.shape[0] != 2:
        raise ValueError("stacked_cols_vals must have shape [2, nnz + 1]")
    if not row_ptrs.is_contiguous() or cols_vals.stride(1) != 1:
        raise ValueError("trie arrays must be contiguous")
    return Csr(row_ptrs.data_ptr(), cols_vals[0].data_ptr(), cols_vals[1].data_ptr(),
               row_ptrs.numel(), cols_vals.shape[1] - 1)


def linear_struct(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor | None) -> Linear:
    """``a`` [rows, hidden] (unit column stride), ``b`` = W.T [hidden, n_vocab] any strides."""
    if a.dtype not in DTYPE_CODE:
        raise TypeError(f"unsupported dtype {a.dtype}")
    if b.dtype != a.dtype:
        raise TypeError(f"a and b must share a dtype (got {a.dtype} and {b.dtype})")
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[0]:
        raise ValueError(f"shape mismatch: a {tuple(a.shape)}, b {tuple(b.shape)}")
    if a.stride(1) != 1:
        raise ValueError("a must have unit column stride")
    return Linear(a.data_ptr(), a.shape[0], a.shape[1], max(a.stride(0), a.shape[1]),
                  b.data_ptr(), b.shape[1], b.stride(0), b.stride(1),
                  ptr(bias), DTYPE_CODE[a.dtype])
