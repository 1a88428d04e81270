"""Paged KV-cache manager: drop-in for the reference's ``KVCacheManager``
(engine/cache_manager.py:4-120).

Public surface kept: the constructor arguments, the attributes other code reads
(``key_cache``/``value_cache`` [L, num_blocks, KVH, block_size, D] on the device, ``seq_len``
int32 [max_batch], ``block_tables`` int32 [max_batch, max_blocks_per_seq] with -1 = unassigned,
``free_blocks``, ``max_blocks_per_seq``, ``block_size`` ...), and ``allocate_and_insert`` /
``free_batch_slot`` with the reference's exception types and messages.

Allocation is host-authoritative and bit-exact with the reference: a FIFO free list popped from
the front when a token needs a new block (cache_manager.py:86-92) and appended to in logical
order when a slot is freed (:110-117).  The reference walks tokens in Python with a device sync
per token per layer; here the engine plans a whole step's allocations on host mirrors of
``seq_len`` / ``block_tables`` once (not once per layer) and the device tables are updated by
the step's own kernels.

Differences, by design: the pool lives on a CUDA device only; ``num_blocks`` may be given to
size the pool independently of max_batch * max_blocks_per_seq (the reference's formula is the
default); the free list is a deque (``pop(0)`` is O(1)).
"""
from __future__ import annotations

import collections

import numpy as np
import torch

from . import _native as N


class FreeBlockList(collections.deque):
    """FIFO free list with the list API the reference uses (``pop(0)``, ``append``)."""

    def pop(self, index: int = -1):   # noqa: D401 - list-compatible signature
        if index == 0:
            return self.popleft()
        if index == -1:
            return super().pop()
        raise IndexError("FreeBlockList supports pop(0) and pop(-1)")

    def __eq__(self, other):
        return list(self) == list(other)


class BlockAllocator:
    """Host side of the paged pool: the FIFO free list, per-slot lengths and block tables, and
    the reference's allocation order (engine/cache_manager.py:51-120) -- no device state, so
    schedulers and tests can plan on it anywhere.  ``KVCacheManager`` owns one and mirrors its
    tables to the device."""

    def __init__(self, max_batch_size: int, max_seq_len: int, block_size: int = 16,
                 num_blocks: int | None = None) -> None:
        self.max_batch_size = max_batch_size
        self.max_seq_len = max_seq_len
        self.block_size = block_size
        self.max_blocks_per_seq = (max_seq_len + block_size - 1) // block_size      # :25
        self.total_physical_blocks = (max_batch_size * self.max_blocks_per_seq        # :26
                                      if num_blocks is None else int(num_blocks))
        self.free_blocks = FreeBlockList(range(self.total_physical_blocks))
        self.seq_len = np.zeros(max_batch_size, np.int32)
        self.block_tables = np.full((max_batch_size, self.max_blocks_per_seq), -1, np.int32)

    def plan_tokens(self, slots, counts, *, strict_len: bool = True):
        """Allocate blocks for ``counts[i]`` new tokens of each slot, in the reference's order
        (slot by slot, token by token, cache_manager.py:73-92).

        Returns (slot_mapping int64 [sum(counts)], updates list of (slot, logical, phys)).
        Raises ValueError / RuntimeError like the reference; on error the blocks allocated
        before the failing token stay assigned (``updates`` then lists them in the exception's
        ``updates`` attribute), as in the reference.
        """
        bs = self.block_size
        out = np.empty(int(sum(counts)), np.int64)
        updates = []
        k = 0
        try:
            for b, n in zip(slots, counts):
                b, n = int(b), int(n)
                start = int(self.seq_len[b])
                if strict_len and start > self.max_seq_len:                        # :60-61
                    raise ValueError("Sequence length exceeds maximum allowed length.")
                # tokens before the first position >= max_seq_len (:79-80); a slot's blocks are
                # taken in ascending logical order, as token-by-token allocation does
                n_ok = max(0, min(n, self.max_seq_len - start))
                if n_ok:
                    lbs = np.arange(start // bs, (start + n_ok - 1) // bs + 1)
                    need = lbs[self.block_tables[b, lbs] == -1]
                    take = min(len(need), len(self.free_blocks))
                    if take:
                        fb = self.free_blocks
                        phys = np.array([fb.popleft() for _ in range(take)], np.int32)
                        self.block_tables[b, need[:take]] = phys
                        updates.extend(zip([b] * take, need[:take].tolist(), phys.tolist()))
                    if take < len(need):                                            # :87-88
                        raise RuntimeError("OOM : No free physical blocks available for allocation.")
                    pos = np.arange(start, start + n_ok, dtype=np.int64)
                    out[k:k + n_ok] = self.block_tables[b, pos // bs].astype(np.int64) * bs + pos % bs
                    k += n_ok
                if n_ok < n:
                    raise ValueError(f"Sequence length exceeds maximum allowed length for batch index {b}.")
        except (ValueError, RuntimeError) as e:
            e.updates = updates
            raise
        return out, updates

    def plan_decode(self, slots) -> np.ndarray:
        """One new token per slot: the block each slot takes from the free list, or -1.  Same
        order and error points as allocating slot by slot: blocks go to the slots that need one
        in slot order; a slot at max_seq_len raises ValueError after the slots before it got
        theirs, an empty free list RuntimeError after the ones that could be served."""
        bs = self.block_size
        sl = np.asarray(slots, np.int64)
        new_block = np.full(len(sl), -1, np.int32)
        if len(sl) == 0:
            return new_block
        pos = self.seq_len[sl]
        stop = len(sl)
        if pos.max() >= self.max_seq_len:
            stop = int(np.argmax(pos >= self.max_seq_len))
        # table entries of the slots' current logical blocks, by flat index (one gather)
        flat = sl[:stop] * self.block_tables.shape[1] + pos[:stop] // bs
        need = np.flatnonzero(np.take(self.block_tables, flat) == -1)
        take = min(len(need), len(self.free_blocks))
        if take:
            phys = np.fromiter((self.free_blocks.popleft() for _ in range(take)), np.int32, take)
            idx = need[:take]
            np.put(self.block_tables, flat[idx], phys)
            new_block[idx] = phys
        if take < len(need):
            raise RuntimeError("OOM : No free physical blocks available for allocation.")
        if stop < len(sl):
            raise ValueError(f"Sequence length exceeds maximum allowed length for batch index "
                             f"{int(sl[stop])}.")
        return new_block

    def advance(self, slots, n) -> None:
        """seq_len[slots] += n."""
        self.seq_len[np.asarray(slots, np.int64)] += np.asarray(n, np.int32)

    def free_slot(self, batch_idx: int) -> None:
        """engine/cache_manager.py:104-120: return the slot's blocks to the back of the free
        list in logical order, reset its table row and its length."""
        if batch_idx < 0 or batch_idx >= self.max_batch_size:
            raise IndexError(f"batch_idx {batch_idx} is out of range.")
        row = self.block_tables[batch_idx]
        for lb in range(self.max_blocks_per_seq):
            phys = int(row[lb])
            if phys != -1:
                self.free_blocks.append(phys)
                row[lb] = -1
        self.seq_len[batch_idx] = 0


class KVCacheManager:
    def __init__(self, max_batch_size: int, max_seq_len: int, num_layers: int, num_kv_heads: int,
                 head_dim: int, block_size: int = 16,
                 device: torch.device | str = "cuda", dtype: torch.dtype = torch.bfloat16,
                 num_blocks: int | None = None) -> None:
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("tiny_infra_b200 keeps the KV pool on a CUDA device")
        if dtype not in (torch.bfloat16, torch.float16):
            raise RuntimeError("KV pool dtype must be bfloat16 or float16")
        self.max_batch_size = max_batch_size
        self.max_seq_len = max_seq_len
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.block_size = block_size
        self.device = device
        self.dtype = dtype
        self.alloc = BlockAllocator(max_batch_size, max_seq_len, block_size, num_blocks)
        self.max_blocks_per_seq = self.alloc.max_blocks_per_seq
        self.total_physical_blocks = self.alloc.total_physical_blocks
        shape = (num_layers, self.total_physical_blocks, num_kv_heads, block_size, head_dim)
        self.key_cache = torch.zeros(shape, device=device, dtype=dtype)
        self.value_cache = torch.zeros(shape, device=device, dtype=dtype)
        self.seq_len = torch.zeros(max_batch_size, device=device, dtype=torch.int32)
        self.block_tables = torch.full((max_batch_size, self.max_blocks_per_seq), -1,
                                       dtype=torch.int32, device=device)
        # host mirrors (the allocator's arrays), authoritative for the engine's step planning
        self._seq_host = self.alloc.seq_len
        self._bt_host = self.alloc.block_tables

    @property
    def free_blocks(self) -> FreeBlockList:
        return self.alloc.free_blocks

    # ---- mirrors ------------------------------------------------------------------------
    def sync_from_device(self) -> None:
        """Refresh the host mirrors from the device tensors (one device sync).  Needed only when
        code outside this class wrote ``seq_len`` / ``block_tables`` directly, as the reference
        scheduler does with ``kv_cache.seq_len[idx] += n``."""
        self._seq_host[:] = self.seq_len.cpu().numpy()
        self._bt_host[:] = self.block_tables.cpu().numpy()

    def seq_len_host(self, slot: int) -> int:
        return int(self._seq_host[slot])

    def plan_tokens(self, slots, counts, *, strict_len: bool = True):
        """``BlockAllocator.plan_tokens`` on the host mirror; the new block-table entries are
        pushed to the device table (also those made before an allocation error)."""
        try:
            out, updates = self.alloc.plan_tokens(slots, counts, strict_len=strict_len)
        except (ValueError, RuntimeError) as e:
            self._push_updates(getattr(e, "updates", []))
            raise
        self._push_updates(updates)
        return out, updates

    def plan_decode(self, slots) -> np.ndarray:
        """One new token per slot: the block each slot must take from the free list this step,
        or -1.  Same order and checks as :meth:`plan_tokens`; the device block table is written
        by the step's prepare kernel (``ti_decode_prepare``), not here."""
        return self.alloc.plan_decode(slots)

    def _push_updates(self, updates) -> None:
        if not updates:
            return
        u = torch.tensor(updates, dtype=torch.int64)
        self.block_tables[u[:, 0].to(self.device), u[:, 1].to(self.device)] = \
            u[:, 2].to(torch.int32).to(self.device)

    def advance(self, slots, n) -> None:
        """seq_len[slots] += n on the host mirror (the device copy is advanced by the step, or
        by :meth:`advance_device`)."""
        self.alloc.advance(slots, n)

    def advance_device(self, slots, n) -> None:
        idx = torch.as_tensor(np.asarray(slots, np.int64), device=self.device)
        self.seq_len[idx] += torch.as_tensor(np.asarray(n, np.int32), device=self.device)
        self.advance(slots, n)

    # ---- reference API --------------------------------------------------------------------
    def allocate_and_insert(self, layer_idx: int, batch_indices: torch.Tensor,
                            new_keys: torch.Tensor, new_values: torch.Tensor):
        """engine/cache_manager.py:51-101: allocate blocks for the new tokens and write their
        K/V ([B, KVH, S, D], or [B, KVH, D]) into layer ``layer_idx``.  ``seq_len`` is not
        advanced.  Returns the full (block_tables, seq_len) tensors."""
        if batch_indices.numel() == 0:
            raise ValueError("batch_indices cannot be empty.")
        self.sync_from_device()
        slots = [int(x) for x in batch_indices.reshape(-1).tolist()]
        if np.any(self._seq_host[slots] > self.max_seq_len):
            raise ValueError("Sequence length exceeds maximum allowed length.")
        if new_keys.ndim == 3:
            new_keys = new_keys.unsqueeze(2)
            new_values = new_values.unsqueeze(2)
        S = new_keys.size(2)
        err = None
        try:
            mapping, _ = self.plan_tokens(slots, [S] * len(slots))
        except (ValueError, RuntimeError) as e:
            err = e
            mapping = self._mapping_so_far(slots, S)
        k = new_keys.to(device=self.device, dtype=self.dtype).permute(0, 2, 1, 3).reshape(-1, self.num_kv_heads, self.head_dim).contiguous()
        v = new_values.to(device=self.device, dtype=self.dtype).permute(0, 2, 1, 3).reshape(-1, self.num_kv_heads, self.head_dim).contiguous()
        n = len(mapping)
        if n:
            m = torch.from_numpy(mapping).to(self.device)
            N.check(N.lib().ti_kv_scatter(
                self.key_cache[layer_idx].data_ptr(), self.value_cache[layer_idx].data_ptr(),
                k.data_ptr(), k.stride(0), k.stride(1), v.data_ptr(), v.stride(0), v.stride(1),
                m.data_ptr(), n, self.total_physical_blocks, self.num_kv_heads, self.head_dim,
                self.block_size, N.dtype_code(self.dtype), N.stream_of(k)))
            torch.cuda.current_stream(self.device).synchronize()
        if err is not None:
            raise err
        return self.block_tables, self.seq_len

    def _mapping_so_far(self, slots, S) -> np.ndarray:
        """Pool slots of the tokens that were placed before an allocation error (the reference
        writes those before raising)."""
        bs = self.block_size
        out = []
        for b in slots:
            start = int(self._seq_host[b])
            for t in range(S):
                pos = start + t
                if pos >= self.max_seq_len:
                    return np.array(out, np.int64)
                phys = int(self._bt_host[b, pos // bs])
                if phys < 0:
                    return np.array(out, np.int64)
                out.append(phys * bs + pos % bs)
        return np.array(out, np.int64)

    def free_batch_slot(self, batch_idx: int) -> None:
        """engine/cache_manager.py:104-120: return the slot's blocks to the back of the free
        list in logical order, reset its table row and its length."""
        self.alloc.free_slot(batch_idx)
        self.block_tables[batch_idx].fill_(-1)
        self.seq_len[batch_idx] = 0
