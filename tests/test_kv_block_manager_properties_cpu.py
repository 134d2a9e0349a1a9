"""Random allocate / extend / free sequences through the KV block manager
(host tensors): pages are conserved, never shared between live sequences,
the block table mirrors every chain, and failed operations change nothing."""
import pytest
from hypothesis import given, settings
from hypothesis import strategies as st

from scirs_b200.inference.kv_cache import BlockManager, BlockManagerConfig, InferenceError, KvPageConfig, KvPagePool

OPS = st.lists(st.tuples(st.sampled_from(["alloc", "extend", "free"]), st.integers(0, 9)), max_size=80)


@settings(max_examples=60, deadline=None)
@given(st.integers(1, 24), st.integers(1, 6), st.integers(1, 5), OPS)
def test_block_manager_invariants(num_pages, max_seqs, max_pages_per_seq, ops):
    cfg = KvPageConfig(block_size=4, num_heads=1, head_dim=8)
    pool = KvPagePool(num_pages, cfg, device="cpu")
    bm = BlockManager(pool, BlockManagerConfig(max_sequences=max_seqs, max_pages_per_seq=max_pages_per_seq))
    for op, sid in ops:
        before = (pool.free_count(), bm.active_sequences(),
                  {s: bm.sequence_page_chain(s) for s in list(bm._pages)})
        try:
            if op == "alloc":
                bm.allocate_sequence(sid)
            elif op == "extend":
                if sid not in bm._pages:
                    continue
                bm.extend_sequence(sid)
            elif sid in bm._pages:
                bm.free_sequence(sid)
        except InferenceError:
            after = (pool.free_count(), bm.active_sequences(),
                     {s: bm.sequence_page_chain(s) for s in list(bm._pages)})
            assert after == before  # a refused operation leaves everything as it was
        chains = {s: bm.sequence_page_chain(s) for s in bm._pages}
        used = [p for c in chains.values() for p in c]
        assert len(used) == len(set(used))  # no page in two chains
        assert pool.free_count() + len(used) == num_pages
        assert all(1 <= len(c) <= max_pages_per_seq for c in chains.values())
        rows = {bm.row_of(s) for s in chains}
        assert len(rows) == len(chains) and all(0 <= r < max_seqs for r in rows)
        for s, c in chains.items():
            assert bm._bt_host[bm.row_of(s), : len(c)].tolist() == c


def test_failed_allocation_releases_the_row():
    pool = KvPagePool(1, KvPageConfig(block_size=4, num_heads=1, head_dim=8), device="cpu")
    bm = BlockManager(pool, BlockManagerConfig(max_sequences=2, max_pages_per_seq=2))
    bm.allocate_sequence(0)
    with pytest.raises(InferenceError):
        bm.allocate_sequence(1)  # no page left
    assert bm.active_sequences() == 1 and len(bm._free_rows) == 1
    bm.free_sequence(0)
    bm.allocate_sequence(1)
    assert bm.active_sequences() == 1


def test_reserve_is_all_or_nothing():
    import torch

    pool = KvPagePool(3, KvPageConfig(block_size=4, num_heads=1, head_dim=8), device="cpu")
    bm = BlockManager(pool, BlockManagerConfig(max_sequences=2, max_pages_per_seq=4))
    bm.allocate_sequence(0)
    bm.allocate_sequence(1)
    k = torch.ones(16, 1, 8, dtype=torch.bfloat16)
    with pytest.raises(InferenceError):
        bm.append([0, 1], [8, 8], k, k)  # needs 2 more pages, 1 is free
    assert bm.seq_len(0) == 0 and bm.seq_len(1) == 0 and pool.free_count() == 1
    bm.append([0, 1], [4, 4], k[:8], k[:8])
    assert bm.seq_len(0) == 4 and bm.seq_len(1) == 4 and pool.free_count() == 1
