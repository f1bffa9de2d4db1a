"""Minimal per-sequence state and block allocation for driving the model
runner: the fields of the reference's ``Sequence`` that batch preparation reads
(``qslab/runtime/state/sequence.py``; ``model_runner.py:262-283``) and a
free-list block pool.  Scheduling, prefix caching and preemption stay with the
reference's engine and are not rebuilt here."""
from __future__ import annotations

import random


class Sequence:
    def __init__(self, token_ids: list[int], block_size: int = 256):
        self.token_ids = list(token_ids)
        self.block_size = block_size
        self.block_table: list[int] = []
        self.num_cached_tokens = 0           # tokens whose KV is already in the pool
        self.num_prompt_tokens = len(token_ids)

    def __len__(self):
        return len(self.token_ids)

    @property
    def last_token(self):
        return self.token_ids[-1]

    @property
    def num_blocks(self):
        return (len(self.token_ids) + self.block_size - 1) // self.block_size

    @property
    def last_block_num_tokens(self):
        return len(self.token_ids) - (self.num_blocks - 1) * self.block_size

    def slot(self, position: int) -> int:
        return self.block_table[position // self.block_size] * self.block_size + position % self.block_size

    def append(self, token: int):
        self.token_ids.append(token)


class BlockPool:
    """Hands out physical block ids; ``shuffle`` permutes the free list so that
    logical and physical order differ, as they do in a live server."""

    def __init__(self, num_blocks: int, shuffle_seed: int | None = None):
        self.free = list(range(num_blocks))
        if shuffle_seed is not None:
            random.Random(shuffle_seed).shuffle(self.free)

    def ensure(self, seq: Sequence, tokens: int) -> None:
        need = (tokens + seq.block_size - 1) // seq.block_size
        while len(seq.block_table) < need:
            if not self.free:
                raise RuntimeError("KV pool exhausted")
            seq.block_table.append(self.free.pop())

    def release(self, seq: Sequence) -> None:
        self.free.extend(seq.block_table)
        seq.block_table.clear()
