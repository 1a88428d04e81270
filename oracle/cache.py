"""Restatement of the reference's paged KV-cache manager (engine/cache_manager.py).

The allocator semantics are integer work and must be bit-exact: a FIFO free list that pops
from the front on allocation (cache_manager.py:44,91) and appends freed blocks at the back in
logical order (cache_manager.py:110-117).
"""
from __future__ import annotations

import numpy as np


class OracleKVCache:
    """numpy mirror of ``KVCacheManager`` (engine/cache_manager.py:4-120)."""

    def __init__(self, max_batch_size: int, max_seq_len: int, num_layers: int, num_kv_heads: int,
                 head_dim: int, block_size: int = 16, dtype=np.float32, allocate_pool: bool = True,
                 num_blocks: int | None = None) -> None:
        self.max_batch_size = max_batch_size
        self.max_seq_len = max_seq_len
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.block_size = block_size
        # cache_manager.py:25-26
        self.max_blocks_per_seq = (max_seq_len + block_size - 1) // block_size
        self.total_physical_blocks = (max_batch_size * self.max_blocks_per_seq
                                      if num_blocks is None else num_blocks)
        shape = (num_layers, self.total_physical_blocks, num_kv_heads, block_size, head_dim)
        if allocate_pool:
            self.key_cache = np.zeros(shape, dtype=dtype)      # cache_manager.py:32
            self.value_cache = np.zeros(shape, dtype=dtype)    # cache_manager.py:34
        else:
            self.key_cache = self.value_cache = None
        self.seq_len = np.zeros(max_batch_size, dtype=np.int32)                          # :38
        self.block_tables = np.full((max_batch_size, self.max_blocks_per_seq), -1, np.int32)  # :41
        self.free_blocks = list(range(self.total_physical_blocks))                      # :44

    # cache_manager.py:51-101
    def allocate_and_insert(self, layer_idx: int, batch_indices, new_keys, new_values):
        batch_indices = np.asarray(batch_indices).reshape(-1)
        if batch_indices.size == 0:
            raise ValueError("batch_indices cannot be empty.")
        if np.any(self.seq_len[batch_indices] > self.max_seq_len):
            raise ValueError("Sequence length exceeds maximum allowed length.")
        if new_keys is not None and new_keys.ndim == 3:
            new_keys = new_keys[:, :, None, :]
            new_values = new_values[:, :, None, :]
        incoming = new_keys.shape[2]
        for i, b in enumerate(batch_indices.tolist()):
            start = int(self.seq_len[b])
            for t in range(incoming):
                pos = start + t
                if pos >= self.max_seq_len:
                    raise ValueError(
                        f"Sequence length exceeds maximum allowed length for batch index {b}.")
                lb, off = pos // self.block_size, pos % self.block_size
                if self.block_tables[b, lb] == -1:
                    if not self.free_blocks:
                        raise RuntimeError("OOM : No free physical blocks available for allocation.")
                    self.block_tables[b, lb] = self.free_blocks.pop(0)
                phys = int(self.block_tables[b, lb])
                if self.key_cache is not None:
                    self.key_cache[layer_idx, phys, :, off, :] = new_keys[i, :, t, :]
                    self.value_cache[layer_idx, phys, :, off, :] = new_values[i, :, t, :]
        return self.block_tables, self.seq_len

    # cache_manager.py:104-120
    def free_batch_slot(self, batch_idx: int) -> None:
        if batch_idx < 0 or batch_idx >= self.max_batch_size:
            raise IndexError(f"batch_idx {batch_idx} is out of range.")
        for lb in range(self.max_blocks_per_seq):
            phys = int(self.block_tables[batch_idx, lb])
            if phys != -1:
                self.free_blocks.append(phys)
                self.block_tables[batch_idx, lb] = -1
        self.seq_len[batch_idx] = 0

    def slot_mapping(self, batch_indices, num_tokens: int) -> np.ndarray:
        """Flat pool slot (physical_block * block_size + offset) of each new token, for the
        positions ``seq_len[b] .. seq_len[b] + num_tokens - 1`` (after allocation)."""
        out = np.empty((len(batch_indices), num_tokens), dtype=np.int64)
        for i, b in enumerate(np.asarray(batch_indices).tolist()):
            for t in range(num_tokens):
                pos = int(self.seq_len[b]) + t
                out[i, t] = int(self.block_tables[b, pos // self.block_size]) * self.block_size \
                    + pos % self.block_size
        return out
