"""PrefixPool bookkeeping on the CPU (the reference's engine/prefix_pool.py:55-322 and the behaviours its
runtime/python/tests/test_prefix_pool.py holds it to): page geometry, the empty prefix in slot 0, lookups and keys,
least-recently-used eviction, counted pins, the errors that name the pool-size settings, forgetting an adapter's
prefixes, block tables, and a prefix written through its pages reading back exactly.

A tiny geometry keeps the pools small: 256-byte pages hold 4 recurrent states of 4 x 4 floats (4 layers x 4 heads:
4 state pages) and 2 layers of convolution tails (2 pages), so every prefix takes 6 fixed pages plus one per 32
tokens."""

from __future__ import annotations

import pytest
import torch

from jeff_b200.prefix_pool import (FAST_PATH_SHAPES, EngineError, PrefixPool, PrefixShapes, check_pool_holds,
                                   check_pool_size, pool_pages, prefix_pool_mb_for, prefixes_held)

SMALL = PrefixShapes(gdn_layers=4, conv=(3, 16), state=(4, 4, 4), attn_layers=1, kv=(1, 2))
FIXED = 6


def small_pool(pages: int) -> PrefixPool:
    return PrefixPool(pages, "cpu", shapes=SMALL)


def test_geometry_of_the_small_and_the_fast_path_layouts() -> None:
    assert SMALL.page_bytes == 256
    assert (SMALL.state_pages, SMALL.heads_per_page, SMALL.conv_pages, SMALL.fixed_pages) == (4, 4, 2, FIXED)
    fp = FAST_PATH_SHAPES
    assert fp.page_bytes == 393216
    assert (fp.state_pages, fp.heads_per_page, fp.conv_pages, fp.layers_per_conv_page) == (48, 6, 2, 9)
    assert fp.pages_per_prefix(1000) == 82 and fp.pages_per_prefix(8192) == 306
    assert pool_pages(8192) == 21845 and prefixes_held(8192, 1000) == 266


@pytest.mark.parametrize(("tokens", "kv_pages"), [(0, 0), (1, 1), (31, 1), (32, 1), (33, 2), (2000, 63)])
def test_a_prefix_takes_its_fixed_pages_and_one_per_32_tokens(tokens: int, kv_pages: int) -> None:
    assert SMALL.pages_per_prefix(tokens) == FIXED + kv_pages
    assert FAST_PATH_SHAPES.pages_per_prefix(tokens) == 50 + kv_pages
    pool = small_pool(2 + FIXED + 64)
    slot = pool.reserve(1, "p", tokens)
    assert len(pool.block_table(slot)) == FIXED + kv_pages and pool.length(slot) == tokens


def test_slot_zero_is_empty_and_the_reserved_pages_are_never_handed_out() -> None:
    pool = small_pool(2 + 2 * (FIXED + 2))
    assert pool.length(0) == 0 and pool.block_table(0) == [1] * FIXED
    a, b = pool.reserve(1, "a", 64), pool.reserve(1, "b", 64)
    assert {a, b} == {1, 2}
    handed = sorted(pool.block_table(a) + pool.block_table(b))
    assert handed == list(range(2, 2 + 2 * (FIXED + 2)))   # every page but the sink (0) and the zero page (1)
    conv, state, kv = pool.gather(0)
    assert not conv.any() and not state.any() and kv.shape[2] == 0


def test_lookup_and_key_by_adapter_row_and_prefix_text() -> None:
    pool = small_pool(40)
    slot = pool.reserve(3, "text", 40)
    assert pool.lookup(3, "text") == slot
    assert pool.lookup(2, "text") is None and pool.lookup(3, "other") is None
    assert pool.key(slot) == (3, "text")
    with pytest.raises(ValueError, match="already in the pool"):
        pool.reserve(3, "text", 40)
    with pytest.raises(ValueError, match="holds no prefix"):
        pool.key(0)
    pool.release(slot)
    with pytest.raises(ValueError, match="holds no prefix"):
        pool.key(slot)


def test_eviction_takes_the_least_recently_used_prefix() -> None:
    pool = small_pool(2 + 3 * (FIXED + 1))   # three prefixes of up to 32 tokens
    a, b, c = (pool.reserve(1, name, 10) for name in "abc")
    pool.lookup(1, "a")                        # use order now b, c, a
    assert pool.reserve(1, "d", 10) == b and pool.lookup(1, "b") is None
    assert [pool.lookup(1, name) for name in "acd"] == [a, c, b]   # order now a, c, d
    assert pool.reserve(1, "e", 10) == a and pool.lookup(1, "a") is None


def test_eviction_frees_as_many_old_prefixes_as_a_long_one_needs() -> None:
    pool = small_pool(2 + 4 * (FIXED + 2))   # full with four 64-token prefixes
    for name in "abcd":
        pool.reserve(1, name, 64)
    pool.lookup(1, "a")                        # order b, c, d, a
    slot = pool.reserve(1, "long", 128)        # FIXED + 4 pages: b and c must go
    assert len(pool.block_table(slot)) == FIXED + 4
    assert pool.lookup(1, "b") is None and pool.lookup(1, "c") is None
    assert pool.lookup(1, "d") is not None and pool.lookup(1, "a") is not None


def test_pinned_prefixes_are_not_evicted_and_pins_are_counted() -> None:
    pool = small_pool(2 + 3 * (FIXED + 1))
    a, b, _ = (pool.reserve(1, name, 10) for name in "abc")
    pool.pin([a, a, b])                        # two rows of one pass on a, one on b
    pool.reserve(1, "d", 10)                   # a and b are older but pinned: c goes
    assert pool.lookup(1, "c") is None and pool.lookup(1, "a") == a and pool.lookup(1, "b") == b
    pool.unpin([a, b])                         # a still pinned once
    pool.lookup(1, "d")
    pool.reserve(1, "e", 10)                   # b is now the oldest unpinned
    assert pool.lookup(1, "b") is None and pool.lookup(1, "a") == a
    pool.unpin([a])
    with pytest.raises(ValueError, match="not pinned"):
        pool.unpin([a])
    with pytest.raises(ValueError, match="slot 5"):
        pool.pin([5])


def test_no_room_is_an_engine_error_that_evicts_nothing() -> None:
    pool = small_pool(2 + 2 * (FIXED + 1))
    a, b = pool.reserve(1, "a", 10), pool.reserve(1, "b", 10)
    pool.pin([a, b])
    with pytest.raises(EngineError, match="pinned"):
        pool.reserve(1, "c", 10)
    assert pool.lookup(1, "a") == a and pool.lookup(1, "b") == b
    pool.unpin([a, b])
    roomy = small_pool(2 + 2 * (FIXED + 2) + 4)   # two 64-token prefixes and 4 free pages
    held = roomy.reserve(1, "a", 64)
    roomy.reserve(1, "b", 64)
    roomy.pin([held])
    with pytest.raises(EngineError, match="pinned"):
        roomy.reserve(1, "long", 7 * 32)        # needs FIXED + 7 = 13 pages: 8 (b) + 4 free are 12
    assert roomy.lookup(1, "b") is not None
    with pytest.raises(EngineError, match="--prefix-pool-mb"):
        small_pool(2 + FIXED + 2).reserve(1, "long", 3 * 32)   # more pages than the whole pool
    with pytest.raises(ValueError, match="longest prefix"):
        small_pool(40).reserve(1, "huge", 8193)


def test_release_returns_a_reservation_that_was_never_written() -> None:
    pool = small_pool(40)
    free = pool.free_page_count()
    slot = pool.reserve(1, "a", 40)
    pool.release(slot)
    assert pool.lookup(1, "a") is None and len(pool) == 0 and pool.free_page_count() == free
    with pytest.raises(ValueError, match="holds no prefix"):
        pool.release(slot)
    pinned = pool.reserve(1, "b", 40)
    pool.pin([pinned])
    with pytest.raises(ValueError, match="pinned"):
        pool.release(pinned)


def test_forget_adapter_frees_that_adapters_prefixes_only() -> None:
    pool = small_pool(80)
    kept = {name: pool.reserve(1, name, 40) for name in ("a", "b")}
    for name in ("a", "c"):
        pool.reserve(2, name, 70)
    tables = {slot: pool.block_table(slot) for slot in kept.values()}
    slots, pages = pool.free_slot_count(), pool.free_page_count()
    pool.forget_adapter(2)
    assert pool.lookup(2, "a") is None and pool.lookup(2, "c") is None
    assert {name: pool.lookup(1, name) for name in kept} == kept
    assert {slot: pool.block_table(slot) for slot in kept.values()} == tables
    assert pool.free_slot_count() == slots + 2 and pool.free_page_count() == pages + 2 * (FIXED + 3)
    pool.forget_adapter(9)
    assert pool.free_slot_count() == slots + 2
    pool.pin([kept["a"]])
    with pytest.raises(ValueError, match="pinned"):
        pool.forget_adapter(1)


def test_block_tables_mirror_the_page_lists() -> None:
    pool = small_pool(60)
    pool.reserve(1, "a", 64)
    slot = pool.reserve(1, "b", 100)
    assert pool.tables.shape == (pool.slots, FIXED + 256)
    assert pool.tables[slot, :FIXED + 4].tolist() == pool.block_table(slot)
    assert pool.tables[0, :FIXED].tolist() == [1] * FIXED


def test_a_prefix_written_into_its_pages_reads_back_exactly() -> None:
    pool = small_pool(40)
    other = pool.reserve(1, "other", 10)
    slot = pool.reserve(1, "p", 70)
    g = torch.Generator().manual_seed(0)
    conv = torch.randn(4, 3, 16, generator=g).to(torch.bfloat16)
    state = torch.randn(4, 4, 4, 4, generator=g)
    kv = torch.randn(1, 2, 70, 1, 2, generator=g).to(torch.bfloat16)
    pool.write(slot, conv, state, kv)
    got_conv, got_state, got_kv = pool.gather(slot)
    assert torch.equal(got_conv, conv) and torch.equal(got_state, state) and torch.equal(got_kv, kv)
    assert not pool.data[1].any()                              # the zero page
    assert not pool.gather(other)[1].any()                     # another prefix's pages are untouched


def test_pool_sizes_and_their_refusals() -> None:
    assert prefix_pool_mb_for(1) == 116 and prefix_pool_mb_for(64) == 7345
    assert pool_pages(7345) - 2 >= 64 * 306 > pool_pages(7344) - 2
    check_pool_holds(8192, 64)
    with pytest.raises(EngineError) as error:
        check_pool_holds(4096, 64)
    assert "--prefix-pool-mb 4096" in str(error.value) and "--max-batch-rows 64" in str(error.value)
    for bad in (None, 115, 0, -3, 1.5, "2048", True):
        with pytest.raises(EngineError, match="at least 116"):
            check_pool_size(bad)
    assert check_pool_size(116) == 116
