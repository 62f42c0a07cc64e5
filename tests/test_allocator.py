"""Native page allocator vs the reference's semantics (no GPU: allocator-only
caches).  Mirrors tests/paged_kvcache_test.cu of the reference: LIFO order,
fragmentation {8,2,5} -> table {5,2,8}, boundary lengths, reuse order,
exhaustion without partial mutation, double free."""
import random

import pytest

from oracle import allocator as OA
from vllm_b200 import _native as N
from vllm_b200 import cache as C


def host_cache(num_blocks, max_seq_len=1024):
    return C.allocatePagedKVCache(num_blocks, max_seq_len=max_seq_len, device_storage=False)


def test_initial_allocation_order_is_ascending():
    cache = host_cache(9)
    assert [C.allocatePhysicalBlock(cache) for _ in range(9)] == list(range(9))


@pytest.mark.parametrize("prompt_length", [1, 15, 16, 17, 31, 32, 33])
def test_fragmented_translation_matches_reference(prompt_length):
    """tests/paged_kvcache_test.cu:36-66 (allocation/table part, all 3 passes)."""
    cache = host_cache(9)
    for b in range(9):
        assert C.allocatePhysicalBlock(cache) == b
    for b in (8, 2, 5):
        C.freePhysicalBlock(cache, b)
    seq = C.SequenceKVState()
    for p in range(3):
        count = prompt_length if p == 0 else 1
        start = seq.current_seq_len
        before = seq.block_table
        C.reserveSequenceBlocks(cache, seq, start + count)
        assert seq.current_seq_len == start
        assert len(seq.block_table) == (start + count + 15) // 16
        assert seq.block_table[:len(before)] == before
        seq.current_seq_len = start + count
        assert seq.block_table == [5, 2, 8][:len(seq.block_table)]
        assert len(cache.free_blocks) == 3 - len(seq.block_table)
    released = seq.block_table
    C.freeSequenceBlocks(cache, seq)
    assert seq.current_seq_len == 0 and seq.block_table == []
    assert len(cache.free_blocks) == 3
    for b in reversed(released):
        assert C.allocatePhysicalBlock(cache) == b


def test_exhaustion_does_not_mutate_and_double_free_is_rejected():
    """tests/paged_kvcache_test.cu:99-133."""
    cache = host_cache(2)
    seq = C.SequenceKVState()
    with pytest.raises(RuntimeError):
        C.reserveSequenceBlocks(cache, seq, 33)
    assert seq.block_table == [] and len(cache.free_blocks) == 2
    first = C.allocatePhysicalBlock(cache)
    C.allocatePhysicalBlock(cache)
    with pytest.raises(N.TvpNoFreeBlocks):
        C.allocatePhysicalBlock(cache)
    C.freePhysicalBlock(cache, first)
    with pytest.raises(ValueError):
        C.freePhysicalBlock(cache, first)
    assert len(cache.free_blocks) == 1
    with pytest.raises(ValueError):
        C.freePhysicalBlock(cache, 2)
    with pytest.raises(ValueError):
        C.freePhysicalBlock(cache, -1)


def test_context_cap_and_invalid_lengths():
    cache = host_cache(80)
    seq = C.SequenceKVState()
    with pytest.raises(ValueError):
        C.reserveSequenceBlocks(cache, seq, 1025)  # reference cap
    C.reserveSequenceBlocks(cache, seq, 1024)
    assert len(seq.block_table) == 64
    seq2 = C.SequenceKVState()
    seq2.current_seq_len = 20  # claims tokens without pages
    with pytest.raises(ValueError):
        C.reserveSequenceBlocks(cache, seq2, 21)
    seq3 = C.SequenceKVState()
    C.reserveSequenceBlocks(cache, seq3, 5)
    seq3.current_seq_len = 5
    with pytest.raises(ValueError):
        C.reserveSequenceBlocks(cache, seq3, 4)  # shrinking


def test_long_context_cap_is_a_parameter():
    cache = host_cache(2048, max_seq_len=32768)
    seq = C.SequenceKVState()
    C.reserveSequenceBlocks(cache, seq, 32768)
    assert len(seq.block_table) == 2048
    assert seq.block_table[:3] == [0, 1, 2]


def test_freeing_a_table_with_a_free_block_is_rejected():
    cache = host_cache(4)
    seq = C.SequenceKVState()
    C.reserveSequenceBlocks(cache, seq, 20)
    C.freePhysicalBlock(cache, seq.block_table[0])  # corrupt: table names a free block
    with pytest.raises(ValueError):
        C.freeSequenceBlocks(cache, seq)


def test_shuffled_free_list_hands_out_from_the_top():
    cache = host_cache(6)
    cache.free_blocks = [3, 0, 5, 1, 4, 2]
    seq = C.SequenceKVState()
    C.reserveSequenceBlocks(cache, seq, 40)
    assert seq.block_table == [2, 4, 1]
    with pytest.raises(ValueError):
        cache.free_blocks = [0, 0]


@pytest.mark.parametrize("seed", [0, 1, 2, 3])
def test_random_operation_sequences_match_oracle_id_for_id(seed):
    rng = random.Random(seed)
    nb = 24
    cache = host_cache(nb, max_seq_len=160)
    ocache = OA.OracleCache(nb, max_seq_len=160)
    seqs = [(C.SequenceKVState(), OA.OracleSequence()) for _ in range(4)]
    for step in range(300):
        i = rng.randrange(len(seqs))
        s, o = seqs[i]
        op = rng.random()
        if op < 0.55:
            total = o.current_seq_len + rng.randint(0, 40)
            err_native = err_oracle = None
            try:
                C.reserveSequenceBlocks(cache, s, total)
            except (ValueError, RuntimeError) as e:
                err_native = type(e)
            try:
                OA.reserve_sequence_blocks(ocache, o, total)
            except (ValueError, RuntimeError) as e:
                err_oracle = type(e)
            assert (err_native is None) == (err_oracle is None)
            if err_native is not None:
                assert issubclass(err_native, ValueError) == issubclass(err_oracle, ValueError)
            elif total <= 16 * len(o.block_table):
                s.current_seq_len = total
                o.current_seq_len = total
        elif op < 0.75:
            C.freeSequenceBlocks(cache, s)
            OA.free_sequence_blocks(ocache, o)
        else:
            if ocache.free_blocks:
                b = C.allocatePhysicalBlock(cache)
                ob = ocache.allocate()
                assert b == ob
                C.freePhysicalBlock(cache, b)
                ocache.free(ob)
        assert s.block_table == o.block_table
        assert cache.free_blocks == ocache.free_blocks

