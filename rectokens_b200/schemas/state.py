"""Decoding state records, field-for-field the reference's
(rectokens/schemas/state.py:7-25)."""

from __future__ import annotations

from typing import NamedTuple, Optional

from torch import Tensor

from rectokens_b200.schemas.compact_csr_trie import CompactCSRTrie
from rectokens_b200.schemas.config import GenerationConfig


class GenerationState(NamedTuple):
    generated_ids: Tensor
    past_key_values: Optional[tuple]
    log_probas: Optional[Tensor]
    attention_mask: Optional[Tensor] = None


class ConstraintState(NamedTuple):
    """``step`` = trie depth of every node in ``cur_node``; ``cur_node`` = BFS
    node id per row (int64 ``[B]``)."""

    step: int
    trie: CompactCSRTrie
    cur_node: Optional[Tensor]


class ConstrainedGenerationState(NamedTuple):
    generation_config: GenerationConfig
    constraint_state: ConstraintState
    generation_state: Optional[GenerationState] = None
