"""Pointer-based prefix tree, the input of ``CompactCSRTrie.from_trie``
(same interface as the reference's rectokens/decoding/trie.py:6-33)."""

from __future__ import annotations

from typing import Optional


class TrieNode:
    __slots__ = ("children", "is_end_of_token")

    def __init__(self) -> None:
        self.children: dict[int, TrieNode] = {}
        self.is_end_of_token = False

    def take_step(self, idx: int) -> Optional["TrieNode"]:
        return self.children.get(idx)


class Trie:
    def __init__(self) -> None:
        self.root = TrieNode()

    def insert(self, token: list[int]) -> None:
        node = self.root
        for idx in token:
            nxt = node.children.get(idx)
            if nxt is None:
                nxt = node.children[idx] = TrieNode()
            node = nxt
        node.is_end_of_token = True

    def find_prefix(self, token: list[int]) -> Optional[TrieNode]:
        node = self.root
        for idx in token:
            node = node.children.get(idx)
            if node is None:
                return None
        return node
