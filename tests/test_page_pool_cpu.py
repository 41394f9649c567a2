"""Native page pool: tail-page copy-on-write, reference counts, commit/promotion, trie dedup.

Behaviours of the reference's tail-COW and tree-dedup suites, stated for this
framework's RoutePool (routes share the committed prefix's full pages and own
short tail page lists; N writers of one partial page cost N-1 copies).
"""

from __future__ import annotations

import pytest
import torch

from conftest import mod

PS = 4


def pool(num_pages=64):
    host = mod("ops._native").host()
    pp = host.PagePool(num_pages, PS)
    return host, pp, host.RoutePool(pp)


def pages_of(slots):
    return sorted({int(s) // PS for s in slots.tolist()})


def test_two_writers_of_shared_partial_tail_copy_once():
    _, pp, rp = pool()
    rp.append_prefix(6)  # one full page + a partial page holding 2 tokens
    for r in (1, 2):
        rp.fork_from_prefix(r)
    slots, copies = rp.prepare_append([1, 2])
    assert copies.shape[0] == 1 and rp.cow_pages_copied == 1
    assert int(copies[0, 2]) == 2  # the two valid tokens of the page are copied
    assert len(set(pages_of(slots))) == 2
    rp.validate()


@pytest.mark.parametrize("n", [2, 3, 5, 8])
def test_n_writers_copy_n_minus_one_pages(n):
    _, pp, rp = pool()
    rp.append_prefix(5)
    for r in range(n):
        rp.fork_from_prefix(r)
    _, copies = rp.prepare_append(list(range(n)))
    assert copies.shape[0] == n - 1
    rp.validate()


def test_same_partial_page_with_different_valid_lengths_is_copied():
    _, pp, rp = pool()
    rp.append_prefix(5)
    rp.fork_from_prefix(1)
    rp.prepare_append([1])  # route 1 advances inside the shared page (in place: sole writer)
    rp.fork_from_prefix(2)  # route 2 sees the page at the prefix length (1 valid token)
    _, copies = rp.prepare_append([2])
    assert copies.shape[0] == 1 and int(copies[0, 2]) == 1
    rp.validate()


def test_distinct_partial_tail_pages_are_not_copied():
    _, pp, rp = pool()
    rp.append_prefix(4)  # full page only: routes start without tail pages
    rp.fork_from_prefix(1)
    rp.fork_from_prefix(2)
    rp.prepare_append([1, 2])  # each allocates its own page
    _, copies = rp.prepare_append([1, 2])
    assert copies.shape[0] == 0 and rp.cow_pages_copied == 0


def test_private_cow_tail_appends_without_another_copy():
    _, pp, rp = pool()
    rp.append_prefix(5)
    rp.fork_from_prefix(1)
    rp.fork_from_prefix(2)
    rp.prepare_append([1, 2])
    copied = rp.cow_pages_copied
    _, copies = rp.prepare_append([1, 2])
    assert copies.shape[0] == 0 and rp.cow_pages_copied == copied


def test_branches_write_disjoint_slots():
    _, pp, rp = pool()
    rp.append_prefix(5)
    for r in (1, 2, 3):
        rp.fork_from_prefix(r)
    written = []
    for _ in range(6):
        s, _ = rp.prepare_append([1, 2, 3])
        written += s.tolist()
    assert len(written) == len(set(written)), "two routes were given the same KV slot"
    rp.validate()


def test_full_pages_are_never_copied():
    _, pp, rp = pool()
    rp.append_prefix(8)
    for r in range(4):
        rp.fork_from_prefix(r)
    for _ in range(PS * 2):
        _, copies = rp.prepare_append(list(range(4)))
        assert copies.shape[0] == 0


def test_batch_one_decode_does_not_copy():
    _, pp, rp = pool()
    rp.append_prefix(7)
    rp.fork_from_prefix(1)
    for _ in range(10):
        _, copies = rp.prepare_append([1])
        assert copies.shape[0] == 0


def test_refcounts_commit_promotion_and_release():
    _, pp, rp = pool()
    rp.append_prefix(6)
    for r in (1, 2):
        rp.fork_from_prefix(r)
    for _ in range(3):
        rp.prepare_append([1, 2])
    rp.fork(3, 1)  # route 3 extends route 1
    rp.prepare_append([3])
    rc = rp.recomputed_refcounts()
    for page, cnt in rc.items():
        assert pp.refcount(page) == cnt
    used_before = pp.used_pages
    released, freed = rp.retain([1, 3])  # route 2 diverged: it goes before the commit
    assert released == 1 and freed >= 1
    rp.commit(1)  # route 1 becomes the prefix (zero copy); route 3 is rebased onto it
    assert rp.prefix_len == 9
    assert not rp.has_route(1) and rp.has_route(3) and rp.route_len(3) == 10
    assert pp.used_pages < used_before
    rp.validate()
    rp.clear()
    assert pp.free_pages == pp.num_pages


def test_commit_rejects_routes_that_do_not_extend_it():
    _, pp, rp = pool()
    rp.append_prefix(4)
    rp.fork_from_prefix(1)
    rp.fork_from_prefix(2)
    for _ in range(5):
        rp.prepare_append([1, 2])
    with pytest.raises(RuntimeError, match="share the committed full pages"):
        rp.commit(1)


def test_target_scratch_and_compaction_region():
    _, pp, rp = pool()
    slots, _ = rp.append_prefix(6)
    scratch = rp.reserve_scratch(6 + 5)
    assert scratch.numel() == 5 and rp.prefix_len == 6
    assert rp.slots_for_positions(6, 5).tolist() == scratch.tolist()
    rp.set_prefix_len(8)  # commit two scratch positions, free pages past them
    assert rp.prefix_len == 8 and rp.prefix_pages().numel() == 2
    with pytest.raises(IndexError):
        rp.slots_for_positions(8, 5)


def test_prefix_page_table_covers_full_partial_and_empty_paths():
    _, pp, rp = pool()
    assert rp.prefix_pages().numel() == 0
    rp.append_prefix(4)
    assert rp.prefix_pages().numel() == 1 and rp.prefix_full_pages == 1
    rp.append_prefix(3)
    assert rp.prefix_pages().numel() == 2 and rp.prefix_full_pages == 1
    rp.fork_from_prefix(9)
    tails, lens = rp.row_tables([9], 4)
    assert lens.tolist() == [7] and int(tails[0, 0]) == int(rp.prefix_pages()[1])


def test_pool_exhaustion_raises_instead_of_corrupting():
    host = mod("ops._native").host()
    pp = host.PagePool(2, PS)
    rp = host.RoutePool(pp)
    rp.append_prefix(8)
    with pytest.raises(RuntimeError):
        rp.append_prefix(1)


# ------------------------------------------------------------------ trie
def test_trie_reuses_shared_prefixes_and_builds_ancestor_masks():
    host = mod("ops._native").host()
    paths = torch.tensor([[5, 6, 7], [5, 6, 8], [9, 6, 7]], dtype=torch.int64)
    tokens, parents, depths, node_paths, masks = host.build_tree(paths)
    assert tokens.tolist() == [5, 6, 7, 8, 9, 6, 7]
    assert parents.tolist() == [-1, 0, 1, 1, -1, 4, 5]
    assert depths.tolist() == [0, 1, 2, 2, 0, 1, 2]
    assert node_paths.tolist() == [[0, 1, 2], [0, 1, 3], [4, 5, 6]]
    bits = masks[:, 0].tolist()
    assert bits[3] == (1 << 0) | (1 << 1) | (1 << 3)
    assert bits[6] == (1 << 4) | (1 << 5) | (1 << 6)


def test_trie_keeps_identical_routes_logically_distinct():
    host = mod("ops._native").host()
    paths = torch.tensor([[1, 2], [1, 2], [1, 3]], dtype=torch.int64)
    tokens, _, _, node_paths, _ = host.build_tree(paths)
    assert tokens.numel() == 3
    assert node_paths.tolist() == [[0, 1], [0, 1], [0, 2]]


def test_trie_masks_span_multiple_words():
    host = mod("ops._native").host()
    paths = torch.arange(70 * 2, dtype=torch.int64).reshape(70, 2)  # 140 unique nodes
    tokens, parents, _, node_paths, masks = host.build_tree(paths)
    assert masks.shape == (140, 3)
    last = int(node_paths[69, 1])
    w = masks[last].tolist()
    assert (w[last // 64] >> (last % 64)) & 1 and (w[(last - 1) // 64] >> ((last - 1) % 64)) & 1
