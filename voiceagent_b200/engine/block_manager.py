"""Paged KV block allocation with audio-aware prefix caching.

Semantics of the reference's BlockManager (engine/block_manager.py:94-151): blocks of
``block_size`` tokens; only the purely textual blocks before the audio span take part
in prefix caching (keys chained with xxh64 over the int64 token ids, 8-byte
little-endian prefix); a new block is claimed only when a token opens one; free
blocks are handed out oldest-freed first. The block ids it assigns are the input of
the on-GPU packer.
"""

from __future__ import annotations

import numpy as np
import xxhash

from voiceagent_b200.engine.request import AsrRequest

NO_HASH = -1


class _Block:
    __slots__ = ("block_id", "ref_count", "hash", "token_ids")

    def __init__(self, block_id: int):
        self.block_id = block_id
        self.ref_count = 0
        self.hash = NO_HASH
        self.token_ids: list[int] = []


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int, enable_prefix_cache: bool = True):
        if num_blocks <= 0:
            raise ValueError(f"num_blocks must be positive, got {num_blocks}")
        self.block_size = block_size
        self.enable_prefix_cache = enable_prefix_cache
        self.blocks = [_Block(i) for i in range(num_blocks)]
        self.hash_to_block_id: dict[int, int] = {}
        # dict keeps insertion order: O(1) pop of the oldest free block and O(1)
        # removal of a specific block on a prefix-cache hit.
        self.free_block_ids: dict[int, None] = dict.fromkeys(range(num_blocks))
        self.num_cache_hit_blocks = 0

    @property
    def num_free_blocks(self) -> int:
        return len(self.free_block_ids)

    @staticmethod
    def compute_hash(token_ids: list[int], prefix: int = NO_HASH) -> int:
        h = xxhash.xxh64()
        if prefix != NO_HASH:
            h.update(prefix.to_bytes(8, "little"))
        h.update(np.asarray(token_ids, dtype=np.int64).tobytes())
        return h.intdigest()

    def _take(self, block_id: int) -> _Block:
        block = self.blocks[block_id]
        if block.ref_count != 0:
            raise RuntimeError(f"block {block_id} is still referenced")
        block.ref_count = 1
        block.hash = NO_HASH
        block.token_ids = []
        del self.free_block_ids[block_id]
        return block

    def _take_any(self) -> _Block:
        return self._take(next(iter(self.free_block_ids)))

    def can_allocate(self, request: AsrRequest) -> bool:
        return self.num_free_blocks >= request.num_blocks

    def can_ever_allocate(self, request: AsrRequest) -> bool:
        return len(self.blocks) >= request.num_blocks

    def allocate(self, request: AsrRequest) -> None:
        if request.block_table:
            raise RuntimeError("request already holds blocks")
        cacheable = request.num_cacheable_blocks if self.enable_prefix_cache else 0
        prefix = NO_HASH
        missed = False
        for index in range(request.num_blocks):
            ids = request.block(index)
            full_text_block = index < cacheable and len(ids) == self.block_size
            key = self.compute_hash(ids, prefix) if full_text_block else NO_HASH
            hit_id = self.hash_to_block_id.get(key, -1) if key != NO_HASH else -1
            if hit_id == -1 or self.blocks[hit_id].token_ids != ids:
                missed = True
            if missed:
                block = self._take_any()
            else:
                request.num_cached_tokens += self.block_size
                self.num_cache_hit_blocks += 1
                block = self.blocks[hit_id]
                if block.ref_count:
                    block.ref_count += 1
                else:
                    block = self._take(hit_id)
            if key != NO_HASH:
                block.hash, block.token_ids = key, ids
                self.hash_to_block_id[key] = block.block_id
                prefix = key
            request.block_table.append(block.block_id)
        request.num_computed_tokens = request.num_cached_tokens

    def deallocate(self, request: AsrRequest) -> None:
        for block_id in reversed(request.block_table):
            block = self.blocks[block_id]
            block.ref_count -= 1
            if block.ref_count == 0:
                self.free_block_ids[block_id] = None
        request.block_table.clear()
        request.num_cached_tokens = 0

    def can_append(self, request: AsrRequest) -> bool:
        return self.num_free_blocks >= (1 if len(request) % self.block_size == 1 else 0)

    def may_append(self, request: AsrRequest) -> None:
        """Cover the position the next decode step writes (len - 1). Equivalent to the
        reference's ``len % block_size == 1`` test, and a no-op when the block was
        already taken ahead (multi-step decode)."""
        if len(request.block_table) * self.block_size < len(request.token_ids):  # < num_blocks
            request.block_table.append(self._take_any().block_id)

    def blocks_ahead(self, request: AsrRequest, steps: int) -> int:
        """New blocks the positions written by ``steps`` decode steps need beyond those
        already held (the step at length L writes position L - 1)."""
        needed = -(-(len(request) + steps - 1) // self.block_size)
        return max(0, needed - len(request.block_table))

    def append_ahead(self, request: AsrRequest, steps: int) -> None:
        for _ in range(self.blocks_ahead(request, steps)):
            request.block_table.append(self._take_any().block_id)
