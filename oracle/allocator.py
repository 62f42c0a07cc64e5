"""TEST INFRASTRUCTURE ONLY — restatement of the reference page allocator.

Pure Python (small, integer-only).  Follows src/model/paged_kvcache.cu:
  allocatePagedKVCache  :65-90   free list seeded descending, so block 0 is handed out first
  allocatePhysicalBlock :100-108 LIFO pop from the back; empty -> runtime_error
  freePhysicalBlock     :110-117 range / double-free check -> invalid_argument; push back
  freeSequenceBlocks    :119-126 frees in table order, clears the table, length 0
  reserveSequenceBlocks :128-145 validation, lazy ceil(L/16) pages, exhaustion checked first
Used to check the native allocator id-for-id.
"""
from __future__ import annotations


class OracleCache:
    def __init__(self, num_blocks: int, max_seq_len: int = 1024):
        if num_blocks <= 0:
            raise ValueError("Invalid paged cache capacity")
        self.num_blocks = num_blocks
        self.max_seq_len = max_seq_len
        self.free_blocks = list(range(num_blocks - 1, -1, -1))

    def allocate(self) -> int:
        if not self.free_blocks:
            raise RuntimeError("Paged KV cache has no free blocks")
        return self.free_blocks.pop()

    def free(self, block: int) -> None:
        if block < 0 or block >= self.num_blocks or block in self.free_blocks:
            raise ValueError("Invalid block or double free")
        self.free_blocks.append(block)


class OracleSequence:
    def __init__(self):
        self.block_table: list[int] = []
        self.current_seq_len = 0


def _validate(cache: OracleCache, seq: OracleSequence) -> None:
    for i, block in enumerate(seq.block_table):
        if (block < 0 or block >= cache.num_blocks or block in cache.free_blocks
                or block in seq.block_table[:i]):
            raise ValueError("Invalid or duplicate sequence block")


def free_sequence_blocks(cache: OracleCache, seq: OracleSequence) -> None:
    _validate(cache, seq)
    for block in seq.block_table:
        cache.free(block)
    seq.block_table = []
    seq.current_seq_len = 0


def reserve_sequence_blocks(cache: OracleCache, seq: OracleSequence, total_seq_len: int) -> None:
    _validate(cache, seq)
    if (seq.current_seq_len < 0 or total_seq_len < seq.current_seq_len
            or total_seq_len > cache.max_seq_len
            or (seq.current_seq_len + 15) // 16 > len(seq.block_table)):
        raise ValueError("Invalid sequence length or incomplete block table")
    needed = (total_seq_len + 15) // 16
    if needed <= len(seq.block_table):
        return
    if needed - len(seq.block_table) > len(cache.free_blocks):
        raise RuntimeError("Insufficient free paged KV blocks")
    while len(seq.block_table) < needed:
        seq.block_table.append(cache.allocate())
