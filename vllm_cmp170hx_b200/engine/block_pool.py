"""KV block and recurrent-state slot pools.

The allocator itself is native (``csrc/block_pool.cpp``, exposed as
``_C.BlockPool``): a free list with reference counts and a prefix-hash table
for prefix caching (the role of upstream vLLM's KVCacheManager that the
reference plugs its KV planning into, vllm_sm80/kv_planning.py:48).  When the
extension is not built (a CPU-only checkout), :class:`PyBlockPool` -- the same
interface in Python -- stands in; tests run both against each other.

Block 0 is reserved: padded CUDA-graph entries point at it.  Slot 0 of the KDA
state pool is reserved the same way.
"""

from __future__ import annotations

import collections


class PyBlockPool:
    def __init__(self, num_blocks: int, reserved: int = 1):
        self.num_blocks = num_blocks
        self._free = collections.deque(range(reserved, num_blocks))
        self._ref = [0] * num_blocks
        self._hash_to_block: dict[int, int] = {}
        self._block_hash: dict[int, int] = {}

    def num_free(self) -> int:
        return len(self._free)

    def allocate(self, n: int) -> list[int]:
        if n > len(self._free):
            raise RuntimeError(f"out of KV blocks: want {n}, have {len(self._free)}")
        out = []
        for _ in range(n):
            b = self._free.popleft()
            h = self._block_hash.pop(b, None)
            if h is not None and self._hash_to_block.get(h) == b:
                del self._hash_to_block[h]
            self._ref[b] = 1
            out.append(b)
        return out

    def free(self, blocks: list[int]) -> None:
        for b in blocks:
            self._ref[b] -= 1
            if self._ref[b] == 0:
                # cached blocks go to the tail so they are reused last (LRU)
                self._free.append(b)

    def cache_block(self, block: int, h: int) -> None:
        self._hash_to_block[h] = block
        self._block_hash[block] = h

    def lookup(self, h: int) -> int:
        return self._hash_to_block.get(h, -1)

    def touch(self, block: int) -> None:
        """Take a reference on a cached block (prefix hit)."""
        if self._ref[block] == 0:
            self._free.remove(block)
        self._ref[block] += 1

    def ref(self, block: int) -> int:
        return self._ref[block]


def make_block_pool(num_blocks: int, reserved: int = 1):
    try:
        from .. import _C

        return _C.BlockPool(num_blocks, reserved)
    except ImportError:
        return PyBlockPool(num_blocks, reserved)


class SlotPool:
    """Fixed pool of recurrent-state slots (one per running sequence)."""

    def __init__(self, num_slots: int, reserved: int = 1):
        self._free = list(range(num_slots - 1, reserved - 1, -1))

    def num_free(self) -> int:
        return len(self._free)

    def allocate(self) -> int:
        if not self._free:
            raise RuntimeError("out of recurrent-state slots")
        return self._free.pop()

    def free(self, s: int) -> None:
        if s > 0:
            self._free.append(s)
