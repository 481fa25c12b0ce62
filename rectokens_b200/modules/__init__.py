from rectokens_b200.modules.constraint_enforcer import (
    ConstraintEnforcer,
    SparseTrieConstraintEnforcer,
)
from rectokens_b200.modules.sparse_linear import SparseLinear

__all__ = ["ConstraintEnforcer", "SparseLinear", "SparseTrieConstraintEnforcer"]
