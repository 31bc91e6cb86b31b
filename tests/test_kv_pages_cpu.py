"""The paged-KV page allocator (K5) without a GPU: the oracle's batch
restatement against the host PagedKVCacheManager mirror (the reference's
src/cuda/paged_kv_cache.cu semantics, pinned by the reference's own
tests/test_paged_kv_cache.cpp scenarios in test_host_cpu.py), the reference's
scenarios replayed through the oracle, and the all-or-nothing error cases."""
import numpy as np
import pytest

import oracle
from a11spec.kv_pages import KVCacheConfig, PagedKVCacheManager

OK, EBOUNDS, ENOSPACE = 0, 2, 6


def host_mgr(num_pages, max_sequences):
    cfg = KVCacheConfig(num_layers=1, head_dim=16, num_kv_heads=1, max_sequences=max_sequences,
                        vram_cap_gb=num_pages * 2 * 16 * 16 * 2 / (1 << 30))
    m = PagedKVCacheManager(cfg, allocate_pool=False)
    assert m.num_pages == num_pages
    return m


def host_table(m, B, max_pages):
    pt = np.full((B, max_pages), -1, np.int32)
    for b in range(B):
        if m._seqs[b].active:
            bt = m.get_block_table(b)
            pt[b, : len(bt)] = bt
    return pt


def test_oracle_matches_host_manager_on_random_batches():
    rng = np.random.default_rng(7)
    P, B, MP = 200, 12, 24
    m = host_mgr(P, B)
    stack, top = list(range(P)), P
    pt = np.full((B, MP), -1, np.int32)
    sl = np.zeros(B, np.int32)
    for step in range(60):
        op = rng.integers(0, 3)
        if op < 2:  # reserve: allocate_sequence + append_token loops, batch order
            n_new = rng.integers(0, 40, B).astype(np.int32) * (rng.random(B) < 0.6)
            r = oracle.kv_reserve(stack, top, P, pt, sl, n_new)
            need = sum(max(1, -(-(int(sl[b]) + int(n_new[b])) // 16)) - (max(1, -(-int(sl[b]) // 16)) if pt[b, 0] >= 0 else 0)
                       for b in range(B))
            if need > top or any(max(1, -(-(int(sl[b]) + int(n_new[b])) // 16)) > MP for b in range(B)):
                assert r["status"] != OK and r["top"] == top  # nothing changed
                continue
            assert r["status"] == OK, (step, r["status"], r["detail"])
            for b in range(B):
                if not m._seqs[b].active:
                    m.allocate_sequence(b)
                m.append_tokens(b, int(n_new[b]))
            stack, top, pt, sl = list(r["stack"]), r["top"], r["page_table"], r["seq_lens"]
        else:  # free a random subset (free_sequence in batch order)
            mask = (rng.random(B) < 0.3).astype(np.int32)
            r = oracle.kv_free_sequences(stack, top, P, pt, sl, mask)
            assert r["status"] == OK
            for b in range(B):
                if mask[b]:
                    m.free_sequence(b)
            stack, top, pt, sl = list(r["stack"]), r["top"], r["page_table"], r["seq_lens"]
        assert stack == m.free_stack(), step
        np.testing.assert_array_equal(pt, host_table(m, B, MP))
        assert [int(x) for x in sl] == [m.num_tokens(b) if m._seqs[b].active else 0 for b in range(B)]


def test_reference_scenarios_through_oracle():  # tests/test_paged_kv_cache.cpp:5-38, 88-117
    P = 64
    pt = np.full((3, 8), -1, np.int32)
    r = oracle.kv_reserve(list(range(P)), P, P, pt, np.zeros(3, np.int32), [0, 0, 0])
    assert r["status"] == OK and P - r["top"] == 3  # allocate_sequence: one block each
    r1 = oracle.kv_reserve(r["stack"], r["top"], P, r["page_table"], r["seq_lens"], [16, 0, 0])
    assert P - r1["top"] == 3  # 16 tokens still fit the first block
    r2 = oracle.kv_reserve(r1["stack"], r1["top"], P, r1["page_table"], r1["seq_lens"], [1, 0, 0])
    assert P - r2["top"] == 4 and (r2["page_table"][0] >= 0).sum() == 2  # the 17th token opens a block
    r3 = oracle.kv_reserve(r2["stack"], r2["top"], P, r2["page_table"], r2["seq_lens"], [31, 48, 48])
    assert P - r3["top"] == 9 and list(r3["seq_lens"]) == [48, 48, 48]  # 3 x 48 tokens = 9 blocks
    r4 = oracle.kv_free_sequences(r3["stack"], r3["top"], P, r3["page_table"], r3["seq_lens"], [0, 1, 0])
    assert P - r4["top"] == 6 and (r4["page_table"][1] < 0).all() and r4["seq_lens"][1] == 0
    # freed blocks go back in table order, so the next sequence reuses them last-freed first
    assert list(r4["stack"][-3:]) == list(r3["page_table"][1, :3])


def test_out_of_pages_changes_nothing():
    P = 5
    pt = np.full((2, 8), -1, np.int32)
    r = oracle.kv_reserve(list(range(P)), P, P, pt, np.zeros(2, np.int32), [40, 40])  # 3 + 3 pages > 5
    assert r["status"] == ENOSPACE and r["detail"] == 6 and r["top"] == P
    assert (r["page_table"] == -1).all() and (r["seq_lens"] == 0).all()


def test_bounds_errors_report_lowest_sequence():
    P = 100
    pt = np.full((4, 2), -1, np.int32)
    r = oracle.kv_reserve(list(range(P)), P, P, pt, np.zeros(4, np.int32), [0, 33, -1, 50])
    assert r["status"] == EBOUNDS and r["detail"] == 1 and r["top"] == P  # 33 tokens need 3 > 2 pages
    lists = np.array([[1, 2], [3, 200]], np.int32)
    r = oracle.kv_release([], 0, P, lists, [2, 2])
    assert r["status"] == EBOUNDS and r["detail"] == 1 and r["top"] == 0  # page 200 outside the pool
    r = oracle.kv_release(list(range(P)), P, P, lists[:1], [1])
    assert r["status"] == EBOUNDS and r["detail"] == -1  # the stack would overflow: a double free


@pytest.mark.parametrize("seed", [1, 2])
def test_release_pushes_lists_in_batch_order(seed):
    rng = np.random.default_rng(seed)
    P = 50
    lists = np.full((5, 4), -1, np.int32)
    n = rng.integers(0, 5, 5).astype(np.int32)
    ids = iter(rng.permutation(P))
    for b in range(5):
        for j in range(n[b]):
            lists[b, j] = next(ids)
    r = oracle.kv_release([], 0, P, lists, n)
    assert r["status"] == OK
    assert list(r["stack"]) == [int(lists[b, j]) for b in range(5) for j in range(n[b])]
