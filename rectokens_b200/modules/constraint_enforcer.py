"""Installs a ``SparseLinear`` in place of a model's output projection
(the reference's rectokens/modules/constraint_enforcer.py:9-120, same
interface: ``prepare(model)`` swaps the ``nn.Linear`` at a dotted attribute
path, ``constrained(...)`` scopes one constrained forward pass)."""

from __future__ import annotations

from abc import ABC, abstractmethod
from contextlib import AbstractContextManager, contextmanager
from typing import Literal, Optional

from torch import nn

from rectokens_b200.modules.sparse_linear import SparseLinear
from rectokens_b200.schemas.state import ConstraintState


class ConstraintEnforcer(ABC, nn.Module):
    @abstractmethod
    def prepare(self, model: nn.Module) -> nn.Module:
        """Modify ``model`` in place to enable constraint enforcement."""

    @abstractmethod
    def constrained(self, constraint_state: ConstraintState, **kwargs) -> AbstractContextManager:
        """Scope constraint enforcement to one forward pass."""

    def forward(self, *args, **kwargs):
        raise NotImplementedError(
            "a ConstraintEnforcer is not a model: call .prepare(model) and pass the model "
            "to autoregressive_generate")


class SparseTrieConstraintEnforcer(ConstraintEnforcer):
    """Replaces the output projection at ``attr_path`` (e.g. ``"lm_head"``)
    with a ``SparseLinear``."""

    def __init__(self, attr_path: str):
        super().__init__()
        self.attr_path = attr_path
        self.constrained_linear: Optional[SparseLinear] = None

    @classmethod
    def convert_to_sparse_linear(cls, model: nn.Module, attr_path: str) -> SparseLinear:
        """Swap the ``nn.Linear`` at ``attr_path`` for a ``SparseLinear`` in
        place and return it.  ``AttributeError`` for a missing path component,
        ``TypeError`` when the target is not an ``nn.Linear``."""
        *path, name = attr_path.split(".")
        parent = model
        for part in path:
            parent = getattr(parent, part)
        linear = getattr(parent, name)
        if isinstance(linear, SparseLinear):
            return linear
        if not isinstance(linear, nn.Linear):
            raise TypeError(f"Expected nn.Linear at '{attr_path}', got {type(linear).__name__}")
        sparse = SparseLinear(linear)
        setattr(parent, name, sparse)
        return sparse

    def prepare(self, model: nn.Module) -> nn.Module:
        self.constrained_linear = self.convert_to_sparse_linear(model, self.attr_path)
        return model

    @contextmanager
    def constrained(
        self,
        constraint_state: ConstraintState,
        strategy: Literal["default", "sample", "topk"] = "default",
        temperature: Optional[float] = None,
        k: int = 1,
        rng_seed: Optional[int] = None,
    ):
        if self.constrained_linear is None:
            raise RuntimeError("Call .prepare(model) before using .constrained()")
        with self.constrained_linear.constrained(constraint_state, strategy=strategy,
                                                 temperature=temperature, k=k,
                                                 rng_seed=rng_seed):
            yield
