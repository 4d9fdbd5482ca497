"""Paged KV-cache blocks and recurrent-state slots.

Block 0 and state slot 0 are reserved as scratch targets for padding rows of a captured CUDA graph,
so padded rows never touch a live sequence's memory.

The allocator is the native C++ one when the host library is built (``engine/csrc/block_alloc.cpp``),
otherwise the Python implementation below; both hand out blocks in the same order.
"""
from __future__ import annotations


class BlockAllocator:
    def __init__(self, num_blocks: int, reserved: int = 1):
        if num_blocks <= reserved:
            raise ValueError("need more blocks than reserved")
        self.num_blocks = num_blocks
        self.reserved = reserved
        self._free = list(range(num_blocks - 1, reserved - 1, -1))  # pop() yields ascending ids

    @property
    def num_free(self) -> int:
        return len(self._free)

    def can_allocate(self, n: int) -> bool:
        return n <= len(self._free)

    def allocate(self, n: int) -> list[int]:
        if n > len(self._free):
            raise MemoryError(f"out of KV blocks: need {n}, free {len(self._free)}")
        return [self._free.pop() for _ in range(n)]

    def free(self, blocks: list[int]) -> None:
        for b in reversed(blocks):
            if b < self.reserved or b >= self.num_blocks:
                raise ValueError(f"bad block id {b}")
            self._free.append(b)


class SlotAllocator(BlockAllocator):
    """Recurrent-state slots (one per running sequence)."""

    def allocate_one(self) -> int:
        return self.allocate(1)[0]

    def free_one(self, s: int) -> None:
        self.free([s])
