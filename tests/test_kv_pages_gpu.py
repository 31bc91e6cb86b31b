"""The paged-KV page allocator (K5) on the GPU against the oracle, bit-exact:
free stack, stack top, page tables, lengths and status, through whole
decode-step lifecycles (reserve tree slots -> a11s_kv_compact -> release the
freed pages -> free finished sequences), a batch larger than one block of
threads, and the all-or-nothing error cases."""
import numpy as np
import pytest
import torch

import a11spec
import oracle
from a11spec.ops import KVPagePool

pytestmark = pytest.mark.gpu

OK, EBOUNDS, ENOSPACE = 0, 2, 6


def _state(pool, pt, sl):
    torch.cuda.synchronize()
    return (pool.free_pages().cpu().numpy(), int(pool.free_top.item()), pt.cpu().numpy(), sl.cpu().numpy(),
            [int(x) for x in pool.status.tolist()])


def _same(dev, ref, what):
    stack, top, pt, sl, st = dev
    assert st[0] == ref["status"] and st[1] == ref["detail"], (what, st, ref["status"], ref["detail"])
    assert top == ref["top"], what
    np.testing.assert_array_equal(stack, ref["stack"], err_msg=what)
    if "page_table" in ref:
        np.testing.assert_array_equal(pt, ref["page_table"], err_msg=what)
        np.testing.assert_array_equal(sl, ref["seq_lens"], err_msg=what)


def test_decode_step_lifecycle_matches_oracle(dev):
    rng = np.random.default_rng(11)
    B, N, MP, P, Hkv, D = 6, 24, 32, 120, 2, 16
    pool = KVPagePool(P, dev)
    pt = torch.full((B, MP), -1, dtype=torch.int32, device=dev)
    sl = torch.zeros(B, dtype=torch.int32, device=dev)
    k_pool = torch.randn(P, 16, Hkv, D, device=dev).to(torch.bfloat16)
    v_pool = torch.randn(P, 16, Hkv, D, device=dev).to(torch.bfloat16)
    o_stack, o_top = list(range(P)), P
    o_pt, o_sl = pt.cpu().numpy(), sl.cpu().numpy()
    o_k, o_v = k_pool.cpu().view(torch.int16).numpy(), v_pool.cpu().view(torch.int16).numpy()
    # prompts of random length
    prompt = rng.integers(1, 60, B).astype(np.int32)
    pool.reserve(pt, sl, torch.from_numpy(prompt).to(dev))
    ref = oracle.kv_reserve(o_stack, o_top, P, o_pt, o_sl, prompt)
    _same(_state(pool, pt, sl), ref, "prompt")
    o_stack, o_top, o_pt, o_sl = list(ref["stack"]), ref["top"], ref["page_table"], ref["seq_lens"]
    for step in range(8):
        n_nodes = rng.integers(1, N + 1, B).astype(np.int32)
        ctx = o_sl.copy()
        pool.reserve(pt, sl, torch.from_numpy(n_nodes).to(dev))  # tree slots
        ref = oracle.kv_reserve(o_stack, o_top, P, o_pt, o_sl, n_nodes)
        _same(_state(pool, pt, sl), ref, f"tree slots {step}")
        o_stack, o_top, o_pt = list(ref["stack"]), ref["top"], ref["page_table"]
        # accepted path: a chain of distinct increasing nodes, shorter than the tree
        alen = np.array([rng.integers(0, n) for n in n_nodes], np.int32)
        acc = np.full((B, N), -1, np.int32)
        for b in range(B):
            acc[b, : alen[b]] = np.sort(rng.choice(np.arange(1, n_nodes[b]), alen[b], replace=False))
        sl.copy_(torch.from_numpy(ctx))  # kv_compact takes the length before the tree
        freed, nfreed = a11spec.kv_compact(k_pool, v_pool, pt, sl, torch.from_numpy(alen).to(dev),
                                           torch.from_numpy(acc).to(dev), torch.from_numpy(n_nodes).to(dev),
                                           check_status=True)
        rc = oracle.kv_compact(o_k, o_v, o_pt, ctx, alen, acc, n_nodes)
        o_k, o_v, o_pt, o_sl = rc["k_pool"], rc["v_pool"], rc["page_table"], rc["seq_lens"]
        np.testing.assert_array_equal(freed.cpu().numpy(), rc["freed_pages"])
        pool.release(freed, nfreed)
        ref = oracle.kv_release(o_stack, o_top, P, rc["freed_pages"], rc["n_freed"])
        _same(_state(pool, pt, sl), ref, f"release {step}")
        o_stack, o_top = list(ref["stack"]), ref["top"]
        np.testing.assert_array_equal(pt.cpu().numpy(), o_pt)
        np.testing.assert_array_equal(sl.cpu().numpy(), o_sl)
        if step % 3 == 2:  # a finished request leaves and a new one arrives
            mask = np.zeros(B, np.int32)
            mask[rng.integers(0, B)] = 1
            pool.free_sequences(pt, sl, torch.from_numpy(mask).to(dev))
            ref = oracle.kv_free_sequences(o_stack, o_top, P, o_pt, o_sl, mask)
            _same(_state(pool, pt, sl), ref, f"free {step}")
            o_stack, o_top, o_pt, o_sl = list(ref["stack"]), ref["top"], ref["page_table"], ref["seq_lens"]
            new = (mask * rng.integers(1, 40)).astype(np.int32)
            pool.reserve(pt, sl, torch.from_numpy(new).to(dev))
            ref = oracle.kv_reserve(o_stack, o_top, P, o_pt, o_sl, new)
            _same(_state(pool, pt, sl), ref, f"new request {step}")
            o_stack, o_top, o_pt, o_sl = list(ref["stack"]), ref["top"], ref["page_table"], ref["seq_lens"]
    torch.cuda.synchronize()
    np.testing.assert_array_equal(k_pool.cpu().view(torch.int16).numpy(), o_k)


def test_large_batch_multi_tile(dev):
    rng = np.random.default_rng(3)
    B, MP, P = 3000, 8, 30000
    pool = KVPagePool(P, dev)
    pt = torch.full((B, MP), -1, dtype=torch.int32, device=dev)
    sl = torch.zeros(B, dtype=torch.int32, device=dev)
    o = dict(stack=list(range(P)), top=P, page_table=pt.cpu().numpy(), seq_lens=sl.cpu().numpy())
    for r in range(3):
        n_new = rng.integers(0, 40, B).astype(np.int32)
        pool.reserve(pt, sl, torch.from_numpy(n_new).to(dev))
        ref = oracle.kv_reserve(o["stack"], o["top"], P, o["page_table"], o["seq_lens"], n_new)
        _same(_state(pool, pt, sl), ref, f"reserve {r}")
        o = ref
        mask = (rng.random(B) < 0.25).astype(np.int32)
        pool.free_sequences(pt, sl, torch.from_numpy(mask).to(dev))
        ref = oracle.kv_free_sequences(o["stack"], o["top"], P, o["page_table"], o["seq_lens"], mask)
        _same(_state(pool, pt, sl), ref, f"free {r}")
        o = ref


def test_errors_change_nothing_and_match_oracle(dev):
    P = 10
    pool = KVPagePool(P, dev)
    pt = torch.full((3, 8), -1, dtype=torch.int32, device=dev)
    sl = torch.zeros(3, dtype=torch.int32, device=dev)
    n_new = np.array([40, 40, 40], np.int32)  # 9 pages of 10: fits
    pool.reserve(pt, sl, torch.from_numpy(n_new).to(dev), check_status=True)
    before = _state(pool, pt, sl)
    more = np.array([40, 0, 0], np.int32)  # sequence 0 needs 2 more pages, 1 is left
    with pytest.raises(a11spec.A11Error):
        pool.reserve(pt, sl, torch.from_numpy(more).to(dev), check_status=True)
    after = _state(pool, pt, sl)
    ref = oracle.kv_reserve(before[0], before[1], P, before[2], before[3], more)
    assert ref["status"] == ENOSPACE
    _same(after, ref, "enospace")
    for a, b in zip(before[:4], after[:4]):
        np.testing.assert_array_equal(np.asarray(a), np.asarray(b))
    big = np.array([0, 100, 0], np.int32)  # 140 tokens need 9 > 8 pages: EBOUNDS at sequence 1
    pool.reserve(pt, sl, torch.from_numpy(big).to(dev))
    ref = oracle.kv_reserve(before[0], before[1], P, before[2], before[3], big)
    assert ref["status"] == EBOUNDS and ref["detail"] == 1
    _same(_state(pool, pt, sl), ref, "ebounds")
    lists = torch.tensor([[3, 99]], dtype=torch.int32, device=dev)  # page 99 outside the pool
    pool.release(lists, torch.tensor([2], dtype=torch.int32, device=dev))
    st = _state(pool, pt, sl)
    assert st[4] == [EBOUNDS, 0] and st[1] == before[1]


def test_decoder_steps_keep_pages_on_device(dev):
    """SpeculativeDecoder.step with a KVPagePool: tree slots reserved after
    drafting, detached pages returned after compaction; after each step every
    table holds exactly max(1, ceil(len/16)) pages and the stack the rest."""
    from a11spec.decoder import SpeculativeDecoder
    from a11spec import workloads as W
    V, B, N, Hkv, Hq, D, MP, P = 4096, 3, 16, 2, 16, 128, 16, 64
    table = W.make_ngram_table(log2_buckets=10, vocab=V, seed=2)
    dec = SpeculativeDecoder(table=torch.from_numpy(table), log2_buckets=10, max_depth=3, max_nodes=N,
                             temperature=0.7)
    pool = KVPagePool(P, dev)
    kpool = torch.randn(P, 16, Hkv, D, device=dev).to(torch.bfloat16)
    vpool = torch.randn(P, 16, Hkv, D, device=dev).to(torch.bfloat16)
    pt = torch.full((B, MP), -1, dtype=torch.int32, device=dev)
    lens = torch.zeros(B, dtype=torch.int32, device=dev)
    pool.reserve(pt, lens, torch.tensor([40, 77, 5], dtype=torch.int32, device=dev), check_status=True)
    last = torch.tensor([[5, 9], [1, 2], [7, 7]], dtype=torch.int32, device=dev)
    for step in range(4):
        before = lens.cpu().clone()
        q = torch.randn(B, N, Hq, D, device=dev).to(torch.bfloat16)
        tree, res = dec.step(last, q, kpool, vpool, pt, lens,
                             lambda attn, tr: torch.randn(B, N, V, device=dev).to(torch.bfloat16), pages=pool)
        torch.cuda.synchronize()
        assert int(pool.status[0]) == OK, pool.status.tolist()
        assert torch.equal(lens.cpu(), before + 1 + res.accept_len.cpu())
        held = (pt >= 0).sum(dim=1).cpu()
        want = torch.clamp((lens.cpu() + 15) // 16, min=1)
        assert torch.equal(held, want.to(held.dtype)), (step, held, want)
        assert int(pool.free_top.item()) == P - int(want.sum())
        used = set(pt[pt >= 0].cpu().tolist())
        assert used.isdisjoint(set(pool.free_pages().cpu().tolist())) and len(used) == int(want.sum())
        last = torch.stack([last[:, 1], res.bonus.clamp_min(0)], dim=1).contiguous()


def test_matches_the_reference_manager_itself(dev):
    """The device allocator against the reference's own PagedKVCacheManager
    (src/cuda/paged_kv_cache.cu, built from the reference tree into
    oracle/_ref/libref_kv.so with a C shim; it cudaMallocs its 256 blocks). The
    same random batches go to both: a batch reserve is the reference's
    allocate_sequence / append_token loop in batch order, a masked free its
    free_sequence loop (a sequence of the batch without pages is started with
    allocate_sequence, which takes its first block even for 0 tokens, as the
    device reserve documents). Block tables must be identical after every batch."""
    import ctypes
    import os
    path = os.path.join(os.path.dirname(oracle.__file__), "_ref", "libref_kv.so")
    if not os.path.exists(path):
        pytest.skip("oracle/_ref/libref_kv.so not built (needs the reference tree at build time)")
    L = ctypes.CDLL(path)
    L.ref_kv_create.restype = ctypes.c_void_p
    L.ref_kv_create.argtypes = [ctypes.c_uint32]
    L.ref_kv_destroy.argtypes = [ctypes.c_void_p]
    for f in (L.ref_kv_allocate, L.ref_kv_free):
        f.argtypes = [ctypes.c_void_p, ctypes.c_uint32]
    L.ref_kv_append.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32]
    L.ref_kv_table.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_int]
    L.ref_kv_used_blocks.restype = ctypes.c_size_t
    L.ref_kv_used_blocks.argtypes = [ctypes.c_void_p]
    B, MP, P = 10, 40, 256
    ref = L.ref_kv_create(B)
    assert ref, "reference manager construction failed"
    try:
        pool = KVPagePool(P, dev)
        pt = torch.full((B, MP), -1, dtype=torch.int32, device=dev)
        sl = torch.zeros(B, dtype=torch.int32, device=dev)
        active = np.zeros(B, bool)
        lens = np.zeros(B, np.int64)
        rng = np.random.default_rng(23)
        buf = (ctypes.c_int32 * MP)()
        for step in range(40):
            if step % 5 == 4 and active.any():  # free a random set of active sequences
                mask = active & (rng.random(B) < 0.5)
                pool.free_sequences(pt, sl, torch.from_numpy(mask.astype(np.int32)).to(dev), check_status=True)
                for b in np.nonzero(mask)[0]:
                    assert L.ref_kv_free(ref, int(b)) == 0
                active &= ~mask
                lens[mask] = 0
            else:  # every sequence adds 0..40 tokens, without running out of pages
                add = rng.integers(0, 41, B)
                add[(lens + add + 15) // 16 > MP] = 0
                if int(np.maximum(1, (lens + add + 15) // 16).sum()) > P:
                    continue
                pool.reserve(pt, sl, torch.from_numpy(add.astype(np.int32)).to(dev), check_status=True)
                for b in range(B):
                    if not active[b]:
                        assert L.ref_kv_allocate(ref, b) == 0
                        active[b] = True
                    if add[b]:
                        assert L.ref_kv_append(ref, b, int(add[b])) == 0
                lens += add
            got = pt.cpu().numpy()
            for b in range(B):
                n = L.ref_kv_table(ref, b, buf, MP)
                want = list(buf[:n]) if n >= 0 else []
                assert got[b, :len(want)].tolist() == want and (got[b, len(want):] == -1).all(), (step, b)
            assert P - int(pool.free_top.item()) == L.ref_kv_used_blocks(ref), step
    finally:
        L.ref_kv_destroy(ref)
