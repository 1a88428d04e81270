"""BlockAllocator.plan_decode and plan_tokens (vectorized) against token-by-token allocation in
the reference's order (engine/cache_manager.py:73-92): random steps with frees, running out of
blocks (RuntimeError after the tokens that could be served) and reaching max_seq_len (ValueError
after the tokens before the failing one) -- tables, free list, updates and returned slots
identical."""
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


def _token_by_token(a, slots, counts, strict_len=True):
    bs = a.block_size
    out = np.empty(int(sum(counts)), np.int64)
    updates = []
    k = 0
    try:
        for b, n in zip(slots, counts):
            start = int(a.seq_len[b])
            if strict_len and start > a.max_seq_len:
                raise ValueError("Sequence length exceeds maximum allowed length.")
            for t in range(n):
                pos = start + t
                if pos >= a.max_seq_len:
                    raise ValueError("Sequence length exceeds maximum allowed length")
                lb = pos // bs
                if a.block_tables[b, lb] == -1:
                    if not a.free_blocks:
                        raise RuntimeError("OOM : No free physical blocks available for allocation.")
                    phys = a.free_blocks.popleft()
                    a.block_tables[b, lb] = phys
                    updates.append((b, lb, phys))
                out[k] = int(a.block_tables[b, lb]) * bs + pos % bs
                k += 1
    except (ValueError, RuntimeError) as e:
        e.updates = updates
        raise
    return out, updates


def test_plan_tokens_matches_token_by_token():
    rng = np.random.default_rng(1)
    for _ in range(150):
        B, S, bs = 6, 80, 16
        nb = int(rng.integers(1, 36))
        a1, a2 = BlockAllocator(B, S, bs, nb), BlockAllocator(B, S, bs, nb)
        for _ in range(25):
            slots = [int(x) for x in rng.permutation(B)[:rng.integers(1, B + 1)]]
            counts = [int(rng.integers(0, 30)) for _ in slots]
            res = []
            for a, fn in ((a1, lambda a: a.plan_tokens(slots, counts)),
                          (a2, lambda a: _token_by_token(a, slots, counts))):
                try:
                    res.append((fn(a), None, None))
                except (ValueError, RuntimeError) as e:
                    res.append((None, type(e), e.updates))
            (r1, e1, u1), (r2, e2, u2) = res
            assert e1 == e2
            np.testing.assert_array_equal(a1.block_tables, a2.block_tables)
            assert list(a1.free_blocks) == list(a2.free_blocks)
            if e1 is None:
                np.testing.assert_array_equal(r1[0], r2[0])
                assert [tuple(map(int, u)) for u in r1[1]] == [tuple(map(int, u)) for u in r2[1]]
                a1.advance(slots, counts)
                a2.advance(slots, counts)
            else:
                assert [tuple(map(int, u)) for u in u1] == [tuple(map(int, u)) for u in u2]
            if rng.random() < 0.3:
                f = int(rng.integers(0, B))
                a1.free_slot(f)
                a2.free_slot(f)
