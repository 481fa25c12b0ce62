from rectokens_b200.schemas.compact_csr_trie import CompactCSRTrie
from rectokens_b200.schemas.config import GenerationConfig
from rectokens_b200.schemas.state import (
    ConstrainedGenerationState,
    ConstraintState,
    GenerationState,
)

__all__ = [
    "CompactCSRTrie",
    "GenerationConfig",
    "ConstraintState",
    "GenerationState",
    "ConstrainedGenerationState",
]
