"""B200-native (sm_100a) trie-constrained decoding step.

Drop-in for the constrained-decoding hot path of RecTokens
(``rectokens.ops.constrained_node_transition`` and the beam search of
``rectokens.decoding.constrained_decoding``), backed by the CUDA kernels of
``libvtnk_b200.so``.  There is no CPU fallback: the library is loaded on the
first call of an op (a missing build raises there), so importing the package
alone maps no native code.
"""

from rectokens_b200.decoding.beam_search import (
    BeamSearchResult,
    constrained_beam_search,
    constrained_beam_search_from_host,
    level_windows,
)
from rectokens_b200.ops.constrained_node_transition import (
    constrained_node_transition,
    fused_linear_constrained_node_transition,
    fused_linear_constrained_node_transition_sampling,
    fused_linear_constrained_node_transition_topk,
)
from rectokens_b200.schemas import (
    CompactCSRTrie,
    ConstrainedGenerationState,
    ConstraintState,
    GenerationConfig,
    GenerationState,
)

__all__ = [
    "BeamSearchResult",
    "CompactCSRTrie",
    "ConstrainedGenerationState",
    "ConstraintState",
    "GenerationConfig",
    "GenerationState",
    "constrained_beam_search",
    "constrained_beam_search_from_host",
    "constrained_node_transition",
    "fused_linear_constrained_node_transition",
    "fused_linear_constrained_node_transition_sampling",
    "fused_linear_constrained_node_transition_topk",
    "level_windows",
]
