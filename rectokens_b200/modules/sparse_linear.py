"""``SparseLinear``: an output projection that runs the fused constrained ops.

Same interface as the reference's module (rectokens/modules/sparse_linear.py:
13-98): wrap an ``nn.Linear``; inside ``constrained(constraint_state,
strategy, temperature, k, rng_seed)`` a forward pass runs the fused op of the
chosen strategy on this step's CSR level and keeps its side outputs
(``next_nodes``, ``valid_idxs`` and ``sample`` or ``topk_logits`` /
``topk_idxs``) for ``decode_one_step``; outside it the module is the plain
linear layer.

One deliberate difference: the fused ops take ``b = W.T`` (``[hidden, N]``);
the reference's module hands them the untransposed ``(N, hidden)`` weight
(:56-94), which the ops read with the wrong strides.  Here the transposed
view is passed, so the route computes ``x @ W.T`` as intended.
"""

from __future__ import annotations

from contextlib import contextmanager
from typing import Literal, Optional

import torch
from torch import nn

from rectokens_b200.ops.constrained_node_transition import (
    fused_linear_constrained_node_transition,
    fused_linear_constrained_node_transition_sampling,
    fused_linear_constrained_node_transition_topk,
)
from rectokens_b200.schemas.state import ConstraintState


class SparseLinear(nn.Module):
    def __init__(self, base_linear: nn.Linear):
        super().__init__()
        self.base_linear = base_linear
        self._ctx: Optional[ConstraintState] = None
        self._strategy: Literal["default", "sample", "topk"] = "default"
        self._temperature: Optional[float] = None
        self._k: int = 1
        self._rng_seed: Optional[int] = None
        self.next_nodes: Optional[torch.Tensor] = None
        self.valid_idxs: Optional[torch.Tensor] = None
        self.sample: Optional[torch.Tensor] = None
        self.topk_logits: Optional[torch.Tensor] = None
        self.topk_idxs: Optional[torch.Tensor] = None

    @contextmanager
    def constrained(
        self,
        constraint_state: ConstraintState,
        strategy: Literal["default", "sample", "topk"] = "default",
        temperature: Optional[float] = None,
        k: int = 1,
        rng_seed: Optional[int] = None,
    ):
        """Scope the constrained forward to one step's ``constraint_state``."""
        self._ctx = constraint_state
        self._strategy = strategy
        self._temperature = temperature
        self._k = k
        self._rng_seed = rng_seed
        try:
            yield
        finally:
            self._ctx = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        assert x.ndim == 2, "the fused ops take 2-D inputs (rows, hidden)"
        self.next_nodes = self.valid_idxs = None
        self.sample = self.topk_logits = self.topk_idxs = None
        if self._ctx is None:
            return self.base_linear(x)
        w, bias = self.base_linear.weight, self.base_linear.bias
        b = w.T  # the ops' operand layout: [hidden, N]
        if self._strategy == "sample":
            self.next_nodes, self.valid_idxs, self.sample = (
                fused_linear_constrained_node_transition_sampling(
                    x, b, self._ctx, bias=bias, temperature=self._temperature,
                    rng_seed=self._rng_seed))
            # decode_one_step reads self.sample; the logits are not formed
            return x.new_zeros(x.shape[0], w.shape[0])
        if self._strategy == "topk":
            (self.next_nodes, self.valid_idxs, self.topk_logits,
             self.topk_idxs) = fused_linear_constrained_node_transition_topk(
                x, b, self._ctx, self._k, bias=bias)
            return self.topk_logits
        self.next_nodes, self.valid_idxs, logits = fused_linear_constrained_node_transition(
            x, b, self._ctx, bias=bias)
        return logits
