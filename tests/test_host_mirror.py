"""Host-side mirror of the reference interface (no GPU): ports of the allocator / block table
tests (src/models/common/paged.rs:343-411) and the batch metadata builder."""

import numpy as np
import pytest

from flour_b200.paged import BlockAllocator, BlockTable, build_batch
from flour_b200.workloads import (QWEN7B, c5_contexts, c5_plan, lpt_partition, make_c3,
                                  mixed_partition, prefill_units)


def test_allocator_hands_out_distinct_blocks_then_exhausts():  # paged.rs:343-353
    alloc = BlockAllocator(2)
    assert alloc.num_free() == 2
    a, b = alloc.allocate(), alloc.allocate()
    assert a != b
    assert alloc.allocate() is None
    assert alloc.decref(a)
    assert alloc.num_free() == 1
    assert alloc.allocate() == a


def test_allocator_refcounts_govern_when_a_block_is_freed():  # paged.rs:355-375
    alloc = BlockAllocator(2)
    a = alloc.allocate()
    assert a == 0 and alloc.ref_count(a) == 1  # first allocation is block 0 (paged.rs:14)
    alloc.incref(a)
    assert alloc.ref_count(a) == 2
    assert not alloc.decref(a)
    assert alloc.num_free() == 1
    assert alloc.decref(a)
    assert alloc.ref_count(a) == 0 and alloc.num_free() == 2
    assert alloc.allocate() == a


def test_block_table_maps_logical_positions_to_physical_slots():  # paged.rs:377-394
    t = BlockTable(2)
    assert t.is_empty()
    t.push_block(5)
    t.push_block(3)
    assert t.capacity() == 4
    assert [t.slot(p) for p in range(4)] == [10, 11, 6, 7]
    t.advance(3)
    assert t.len() == 3
    assert t.slots(0, 3) == [10, 11, 6]
    # Past the last block or before the first: out of range (a panic in the reference).
    with pytest.raises(IndexError):
        t.slot(4)
    with pytest.raises(IndexError):
        t.slot(-1)


def test_block_table_exposes_blocks_and_clears():  # paged.rs:396-411
    t = BlockTable(2)
    t.push_block(5)
    t.push_block(3)
    t.advance(4)
    assert t.blocks() == [5, 3] and t.block_at(0) == 5 and t.block_at(1) == 3
    t.clear()
    assert t.is_empty() and t.len() == 0 and t.blocks() == [] and t.block_size() == 2


def test_build_batch_matches_per_sequence_slots():
    tables = []
    for blocks, n in (([4, 9], 20), ([1], 3), ([7, 2, 5], 40)):
        t = BlockTable(16)
        for b in blocks:
            t.push_block(b)
        t.advance(n)
        tables.append(t)
    meta = build_batch(tables, [1, 3, 8], "cpu")
    assert meta.block_tables.tolist() == [[4, 9, 0], [1, 0, 0], [7, 2, 5]]
    assert meta.context_lens.tolist() == [20, 3, 40]
    assert meta.cu_seqlens_q.tolist() == [0, 1, 4, 12]
    want = tables[0].slots(19, 20) + tables[1].slots(0, 3) + tables[2].slots(32, 40)
    assert meta.slot_mapping.tolist() == want
    assert meta.max_context_len == 40 and meta.max_seqlen_q == 8


def test_build_batch_edge_cases():
    """Empty batch, a sequence with no new tokens, and the C++ host's two errors."""
    empty = build_batch([], [], "cpu")
    assert empty.block_tables.shape == (0, 1) and empty.context_lens.tolist() == []
    assert empty.cu_seqlens_q.tolist() == [0] and empty.slot_mapping.tolist() == []
    assert empty.max_context_len == 0 and empty.max_seqlen_q == 0
    a, b = BlockTable(16), BlockTable(16)
    a.push_block(3)
    a.advance(10)
    b.push_block(5)
    b.push_block(6)
    b.advance(17)
    meta = build_batch([a, b], [0, 2], "cpu")
    assert meta.cu_seqlens_q.tolist() == [0, 0, 2]
    assert meta.slot_mapping.tolist() == [5 * 16 + 15, 6 * 16 + 0]
    assert meta.block_tables.tolist() == [[3, 0], [5, 6]] and meta.max_seqlen_q == 2
    with pytest.raises(ValueError, match="differ in length"):
        build_batch([a, b], [1], "cpu")
    with pytest.raises(ValueError, match="q_len exceeds the sequence length"):
        build_batch([a], [11], "cpu")
    with pytest.raises(ValueError, match="q_len exceeds the sequence length"):
        build_batch([a], [-1], "cpu")


def test_lpt_partition_balances_lognormal_contexts():
    ctx = c5_contexts(5)
    parts = lpt_partition(ctx, 8)
    assert sorted(i for p in parts for i in p) == list(range(len(ctx)))
    loads = [ctx[p].sum() for p in parts]
    assert max(loads) / min(loads) < 1.02


def test_mixed_partition_balances_two_stream_steps():
    ctx, is_pf, _, cost = c5_plan(1000)

    def step(b, overlap=0.5):
        p = cost[[i for i in b if is_pf[i]]].sum()
        d = cost[[i for i in b if not is_pf[i]]].sum()
        return max(p, d) + overlap * min(p, d)

    for world in (1, 2, 4, 8):
        parts = mixed_partition(cost, is_pf, world)
        assert sorted(i for p in parts for i in p) == list(range(len(ctx)))
        new = max(step(b) for b in parts)
        old = max(step(b) for b in lpt_partition(cost, world))
        assert new <= old * 1.0001
        assert new <= min(step(b) for b in parts) * 1.01  # within 1 % across ranks


def test_prefill_units_count_tiles_and_items():
    # Qwen2-7B: n_rep 7 -> 18-token Q tiles, 36-token chunks; 4 KV heads.
    assert prefill_units(36, QWEN7B) == (1 + 3) * 4
    assert prefill_units(37, QWEN7B) == (1 + 3 + 1 + 3) * 4
    # a cached prefix adds KV tiles to every chunk
    assert prefill_units(36, QWEN7B, prefix=128) == (2 + 3) * 4


def test_c3_generator_shares_prefix_blocks():
    b = make_c3("cpu", seed=3)
    bt = b.block_tables.numpy()
    for g0 in range(0, 16, 4):
        p = int(b.prefix[g0]) // 16
        for i in range(g0 + 1, g0 + 4):
            assert (bt[i, :p] == bt[g0, :p]).all()
        assert b.prefix[g0] % 16 == 0 and b.prefix[g0] <= 0.5 * b.lens[g0:g0 + 4].min()
    # every suffix slot is unique and lies outside the shared prefixes
    s = b.slot_mapping.numpy()
    assert len(np.unique(s)) == len(s)
    assert b.flops() > 0
