"""BlockAllocator.plan_decode (vectorized) against slot-by-slot allocation in the reference's
order (engine/cache_manager.py:73-92): random decode steps with frees, running out of blocks
(RuntimeError after the slots that could be served) and reaching max_seq_len (ValueError after
the slots before the failing one) -- tables, free list and returned blocks identical."""
import numpy as np

from tiny_infra_b200.cache_manager import BlockAllocator


def _slot_by_slot(a, slots):
    out = np.full(len(slots), -1, np.int32)
    for i, b in enumerate(slots):
        pos = int(a.seq_len[b])
        if pos >= a.max_seq_len:
            raise ValueError("Sequence length exceeds maximum allowed length")
        lb = pos // a.block_size
        if a.block_tables[b, lb] == -1:
            if not a.free_blocks:
                raise RuntimeError("OOM : No free physical blocks available for allocation.")
            p = a.free_blocks.popleft()
            a.block_tables[b, lb] = p
            out[i] = p
    return out


def _outcome(fn, a, slots):
    try:
        return fn(a, slots), None
    except (ValueError, RuntimeError) as e:
        return None, type(e)


def test_plan_decode_matches_slot_by_slot():
    rng = np.random.default_rng(0)
    for _ in range(200):
        B, S, bs = 8, 64, 16
        nb = int(rng.integers(1, 40))
        a1, a2 = BlockAllocator(B, S, bs, nb), BlockAllocator(B, S, bs, nb)
        for _ in range(40):
            slots = [int(x) for x in rng.permutation(B)[:rng.integers(1, B + 1)]]
            r1, e1 = _outcome(lambda a, s: a.plan_decode(s), a1, slots)
            r2, e2 = _outcome(_slot_by_slot, a2, slots)
            assert e1 == e2
            np.testing.assert_array_equal(a1.block_tables, a2.block_tables)
            assert list(a1.free_blocks) == list(a2.free_blocks)
            if e1 is None:
                np.testing.assert_array_equal(r1, r2)
                a1.advance(slots, 1)
                a2.advance(slots, 1)
            if rng.random() < 0.2:
                f = int(rng.integers(0, B))
                a1.free_slot(f)
                a2.free_slot(f)
