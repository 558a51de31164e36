"""Prefix-cache index on the host (no GPU): the reference's radix unit test
(tests/e2e/test_prefix_caching.py:14-31) plus insertion, partial matches, token verification and
least-recently-used eviction of the trie behind the scheduler's prefix cache
(runtime/src/radix_tree.cpp:7-220)."""

from __future__ import annotations

import numpy as np


def _tree(t):
    from ggmlc_b200 import _runtime as R

    return R.PagedRadixTree(t)


def test_radix_tree_unit():
    tree = _tree(128)
    assert tree.tokens_per_page == 128
    assert tree.total_cached_pages == 0
    assert tree.total_nodes == 1  # the root
    m = tree.match_prefix(list(range(10, 50)))  # shorter than one page
    assert m.matched_pages == 0 and m.matched_tokens == 0
    m = tree.match_prefix(list(range(100, 228)) + [999])  # empty tree
    assert m.matched_pages == 0 and m.matched_tokens == 0


def test_radix_insert_and_match_whole_pages():
    tree = _tree(4)
    prompt = list(range(1, 11))  # two whole pages and a 2-token tail
    assert tree.insert_prefix(prompt) == 2
    assert tree.total_cached_pages == 2 and tree.total_nodes == 3
    assert tree.insert_prefix(prompt) == 0  # already indexed
    m = tree.match_prefix(prompt)
    assert (m.matched_pages, m.matched_tokens) == (2, 8)
    m = tree.match_prefix(prompt[:4] + [0, 0, 0, 0])  # diverges in page 2
    assert (m.matched_pages, m.matched_tokens) == (1, 4)
    m = tree.match_prefix([0] + prompt[1:])  # diverges in page 1
    assert m.matched_pages == 0
    # a second branch below the shared first page
    assert tree.insert_prefix(prompt[:4] + [7, 7, 7, 7]) == 1
    assert tree.total_cached_pages == 3
    tree.reset()
    assert tree.total_cached_pages == 0 and tree.total_nodes == 1
    assert tree.match_prefix(prompt).matched_pages == 0


def test_radix_lru_evicts_leaves_only():
    tree = _tree(2)
    a = [1, 2, 3, 4, 5, 6]
    b = [1, 2, 9, 9]
    assert tree.insert_prefix(a) == 3  # pages 0, 1, 2
    assert tree.insert_prefix(b) == 1  # page 3 under page 0
    tree.match_prefix(a)  # a's path is now the most recent
    assert tree.evict_lru() == 3  # b's leaf is the oldest leaf
    assert tree.evict_lru() == 2  # then a's deepest page; page 0 and 1 are inner nodes
    assert tree.evict_lru() == 1
    assert tree.evict_lru() == 0
    assert tree.evict_lru() == -1
    assert tree.total_cached_pages == 0


def test_radix_chunk_hash_is_checked_against_tokens():
    rng = np.random.default_rng(3)
    tree = _tree(8)
    base = rng.integers(0, 1 << 30, size=64).astype(np.int32)
    assert tree.insert_prefix(base) == 8
    for i in range(0, 64, 8):
        other = base.copy()
        other[i] ^= 1  # one token of page i // 8 differs
        assert tree.match_prefix(other).matched_tokens == i
