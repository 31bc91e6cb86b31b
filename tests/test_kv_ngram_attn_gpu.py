"""K1 n-gram expansion, K2 tree attention and K4 compaction on the GPU,
through the C ABI, against the oracle (bit-exact for K1/K4, 2e-2 for K2)."""
import numpy as np
import pytest
import torch

import attn_tolerance as AT
import oracle
import a11spec
from a11spec import workloads as W

pytestmark = pytest.mark.gpu


# ----------------------------------------------------------------------------- K1
@pytest.mark.parametrize("widths", [(4, 2, 5, 64), (3, 1, 4, 64), (8, 8, 3, 200), (0, 2, 5, 64), (4, 2, 5, 1)])
def test_ngram_expand_vs_oracle(dev, widths):
    wr, wi, depth, max_nodes = widths
    table = W.make_ngram_table(log2_buckets=12, vocab=5000, seed=3)
    rng = np.random.default_rng(2)
    empty = rng.random(table.shape[:2]) < 0.3  # ragged buckets
    table[..., 1][empty] = 0
    table[7, :, 1] = 5  # all-tie bucket
    last = rng.integers(0, 5000, (37, 2)).astype(np.int32)
    g = a11spec.ngram_expand(torch.from_numpy(table).to(dev), torch.from_numpy(last).to(dev),
                             wr, wi, depth, max_nodes)
    o = oracle.ngram_expand(table, 12, last, wr, wi, depth, max_nodes)
    for got, key in zip(g, ("tokens", "parents", "depths", "n_nodes")):
        np.testing.assert_array_equal(got.cpu().numpy(), o[key], err_msg=key)



@pytest.mark.parametrize("slots", [1, 3, 4, 5, 16, 27, 32])
def test_ngram_expand_slot_counts(dev, slots):
    """Every compiled slot bound (4, 8, 16, 32), odd counts (the 4-byte bucket
    reads) and ties of count across a whole bucket, against the oracle."""
    rng = np.random.default_rng(10 + slots)
    table = W.make_ngram_table(log2_buckets=10, slots=slots, vocab=3000, seed=slots)
    table[..., 1][rng.random(table.shape[:2]) < 0.25] = 0
    table[3, :, 1] = 2
    last = rng.integers(0, 3000, (19, 2)).astype(np.int32)
    wr, wi = min(slots, 4), min(slots, 3)
    g = a11spec.ngram_expand(torch.from_numpy(table).to(dev), torch.from_numpy(last).to(dev), wr, wi, 4, 64)
    o = oracle.ngram_expand(table, 10, last, wr, wi, 4, 64)
    for got, key in zip(g, ("tokens", "parents", "depths", "n_nodes")):
        np.testing.assert_array_equal(got.cpu().numpy(), o[key], err_msg=key)

def test_ngram_bucket_host_device_agree():
    for a, b in [(0, 0), (3, 4), (151935, 12), (-7, 2**31 - 1)]:
        assert a11spec.ngram_bucket(a, b, 20) == oracle.ngram_bucket(a, b, 20)


# ----------------------------------------------------------------------------- K4
def _compact_case(rng, B, N, ctx_lo, ctx_hi, P, Hkv=4, D=128, dtype=torch.bfloat16):
    ctx = rng.integers(ctx_lo, ctx_hi, B).astype(np.int32)
    per = (ctx.max() + N + 15) // 16 + 2
    perm = rng.permutation(P)[: B * per].reshape(B, per).astype(np.int32)
    pt = perm.copy()
    for b in range(B):  # pages beyond the tree are not owned
        pt[b, (ctx[b] + N + 15) // 16:] = -1
    parents = np.stack([W.random_parents(N, rng) for _ in range(B)])
    nodes = np.full((B, N), -1, np.int32)
    alen = np.zeros(B, np.int32)
    for b in range(B):  # a random root-to-node path
        leaf = int(rng.integers(0, N))
        path = []
        a = leaf
        while a > 0:
            path.append(a)
            a = int(parents[b, a])
        path = path[::-1]
        alen[b] = len(path)
        nodes[b, : len(path)] = path
    k = torch.randn(P, 16, Hkv, D).to(dtype)
    v = torch.randn(P, 16, Hkv, D).to(dtype)
    return ctx, pt, nodes, alen, k, v


def test_kv_compact_vs_oracle_bit_exact(dev):
    rng = np.random.default_rng(4)
    B, N, P = 16, 64, 4096
    ctx, pt, nodes, alen, k, v = _compact_case(rng, B, N, 1, 500, P)
    nn = np.full(B, N, np.int32)
    o = oracle.kv_compact(k.view(torch.int16).numpy(), v.view(torch.int16).numpy(), pt, ctx, alen,
                          nodes, nn)
    kd, vd = k.to(dev), v.to(dev)
    ptd, sld = torch.from_numpy(pt).to(dev), torch.from_numpy(ctx).to(dev)
    freed, nf = a11spec.kv_compact(kd, vd, ptd, sld, torch.from_numpy(alen).to(dev),
                                   torch.from_numpy(nodes).to(dev), torch.from_numpy(nn).to(dev),
                                   check_status=True)
    assert o["status"] == 0
    assert torch.equal(kd.view(torch.int16).cpu(), torch.from_numpy(o["k_pool"]))
    assert torch.equal(vd.view(torch.int16).cpu(), torch.from_numpy(o["v_pool"]))
    np.testing.assert_array_equal(ptd.cpu().numpy(), o["page_table"])
    np.testing.assert_array_equal(sld.cpu().numpy(), o["seq_lens"])
    np.testing.assert_array_equal(nf.cpu().numpy(), o["n_freed"])
    fr = freed.cpu().numpy()
    for b in range(B):
        np.testing.assert_array_equal(fr[b, : o["n_freed"][b]], o["freed_pages"][b, : o["n_freed"][b]])


def test_kv_compact_overlapping_path_in_place(dev):
    """Path 2 -> 5: slot len+2 is a source (j=0) and a destination (j=1)."""
    P, Hkv, D = 8, 1, 8
    k = torch.arange(P * 16 * Hkv * D, dtype=torch.float32).view(P, 16, Hkv, D)
    v = -k
    pt = np.array([[3, 5, 6, 1]], np.int32)
    nodes = np.full((1, 20), -1, np.int32)
    nodes[0, :2] = [2, 5]
    o = oracle.kv_compact(k.numpy(), v.numpy(), pt, np.array([14], np.int32), np.array([2], np.int32),
                          nodes, np.array([20], np.int32))
    kd, vd = k.to(dev), v.to(dev)
    a11spec.kv_compact(kd, vd, torch.from_numpy(pt).to(dev), torch.tensor([14], dtype=torch.int32, device=dev),
                       torch.tensor([2], dtype=torch.int32, device=dev), torch.from_numpy(nodes).to(dev),
                       torch.tensor([20], dtype=torch.int32, device=dev), check_status=True)
    assert torch.equal(kd.cpu(), torch.from_numpy(o["k_pool"]))
    assert torch.equal(vd.cpu(), torch.from_numpy(o["v_pool"]))


def test_kv_compact_multilayer_and_bad_page(dev):
    rng = np.random.default_rng(8)
    B, N, P, Lyr = 4, 16, 256, 3
    ctx, pt, nodes, alen, _, _ = _compact_case(rng, B, N, 20, 60, P, Hkv=2, D=64)
    k = torch.randn(Lyr, P, 16, 2, 64).to(torch.bfloat16)
    v = torch.randn(Lyr, P, 16, 2, 64).to(torch.bfloat16)
    nn = np.full(B, N, np.int32)
    o = oracle.kv_compact(k.view(torch.int16).numpy(), v.view(torch.int16).numpy(), pt, ctx, alen,
                          nodes, nn, num_layers=Lyr, layer_stride=P * 16 * 128)
    kd, vd = k.to(dev), v.to(dev)
    a11spec.kv_compact(kd, vd, torch.from_numpy(pt).to(dev), torch.from_numpy(ctx).to(dev),
                       torch.from_numpy(alen).to(dev), torch.from_numpy(nodes).to(dev),
                       torch.from_numpy(nn).to(dev), num_layers=Lyr, check_status=True)
    assert torch.equal(kd.view(torch.int16).cpu(), torch.from_numpy(o["k_pool"]))
    # a page id outside the pool is reported, not dereferenced
    pt2 = pt.copy()
    pt2[0, ctx[0] // 16:(ctx[0] + N + 15) // 16] = P + 5
    al2, nd2 = alen.copy(), nodes.copy()
    al2[0], nd2[0, 0] = 1, 1
    ws = a11spec.ops.workspace(256, dev)
    a11spec.kv_compact(kd, vd, torch.from_numpy(pt2).to(dev), torch.from_numpy(ctx).to(dev),
                       torch.from_numpy(al2).to(dev), torch.from_numpy(nd2).to(dev),
                       torch.from_numpy(nn).to(dev), num_layers=Lyr, ws=ws)
    assert a11spec.read_status(ws)[0] == a11spec.ops._lib.EBOUNDS


# ----------------------------------------------------------------------------- K2
def _attn_case(seed, B, N, Hq, Hkv, ctx, dev, ragged=True):
    rng = np.random.default_rng(seed)
    parents = np.stack([W.random_parents(N, rng) for _ in range(B)])
    P = B * ((ctx + N + 15) // 16) + 7
    kv = W.paged_kv(B, ctx, N, Hkv, 128, P, seed=seed, device=dev)
    if ragged:  # different context lengths per sequence
        kv["ctx_lens"] = torch.as_tensor(rng.integers(max(1, ctx - 40), ctx + 1, B), dtype=torch.int32, device=dev)
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(B, N, Hq, 128, device=dev, generator=g).to(torch.bfloat16)
    nn = np.array([N if b % 2 == 0 else max(1, N - 3 * b) for b in range(B)], np.int32)
    return q, kv, parents, nn


@pytest.mark.parametrize("ctx,N,B", [(37, 12, 3), (300, 64, 3), (1, 5, 3), (5000, 16, 1), (1000, 40, 2)])
def test_tree_attention_vs_oracle(dev, ctx, N, B):
    """(5000, 16, 1) and (1000, 40, 2) run with split-KV partials and the combine
    kernel. Element-wise bound: |got - ref| <= 2e-2 |ref| + a per-row floor from
    the bf16 rounding of the probabilities (tests/attn_tolerance.py)."""
    Hq, Hkv = 16, 2
    q, kv, parents, nn = _attn_case(7, B, N, Hq, Hkv, ctx, dev)
    par, nnt = torch.from_numpy(parents).to(dev), torch.from_numpy(nn).to(dev)
    out, lse, _ = a11spec.tree_attention(q, kv["k_pool"], kv["v_pool"], kv["page_table"], kv["ctx_lens"],
                                         par, nnt, want_lse=True, check_status=True)
    ref, ref_lse, rc = oracle.tree_attention(q.float().cpu().numpy(), kv["k_pool"].float().cpu().numpy(),
                                             kv["v_pool"].float().cpu().numpy(), kv["page_table"].cpu().numpy(),
                                             kv["ctx_lens"].cpu().numpy(), parents, nn, 1 / np.sqrt(128))
    assert rc == 0
    _, floor = AT.reference(q, kv["k_pool"], kv["v_pool"], kv["page_table"], kv["ctx_lens"], par, nnt)
    AT.assert_close(out.float().cpu(), ref, floor.cpu(), f"ctx {ctx}, {N} nodes")
    np.testing.assert_allclose(lse.cpu().numpy(), ref_lse, rtol=1e-3, atol=1e-3)
    got = out.float().cpu().numpy()
    for b in range(B):
        assert np.all(got[b, nn[b]:] == 0)


def _full_check(d, what):
    """Every sequence and head of a full-size launch against the torch fp32
    restatement on the GPU, element by element."""
    out, _, _ = a11spec.tree_attention(d["q"], d["k_pool"], d["v_pool"], d["page_table"], d["ctx_lens"],
                                       d["parents"], d["n_nodes"], check_status=True)
    ref, floor = AT.reference(d["q"], d["k_pool"], d["v_pool"], d["page_table"], d["ctx_lens"], d["parents"],
                              d["n_nodes"])
    AT.assert_close(out.float(), ref, floor, what)
    return out, floor


def test_tree_attention_c4_full_size(dev):
    """C4 (B=32, ctx 4096, 64-node random trees, GQA 32/4): all 32 sequences
    against the torch restatement, and two of them against the oracle."""
    d = W.make_c4(seed=4, batch=32, device=dev)
    out, floor = _full_check(d, "C4")
    for b in (0, 31):
        ref, _, rc = oracle.tree_attention(
            d["q"][b:b + 1].float().cpu().numpy(), d["k_pool"].float().cpu().numpy(),
            d["v_pool"].float().cpu().numpy(), d["page_table"][b:b + 1].cpu().numpy(),
            d["ctx_lens"][b:b + 1].cpu().numpy(), d["parents"][b:b + 1].cpu().numpy(),
            d["n_nodes"][b:b + 1].cpu().numpy(), 1 / np.sqrt(128))
        assert rc == 0
        AT.assert_close(out[b:b + 1].float().cpu(), ref, floor[b:b + 1].cpu(), f"C4 sequence {b} vs oracle")


def test_tree_attention_c5_full_size(dev):
    """C5 shapes (B=32, ctx 32768, 64 nodes, GQA 32/4): the launch runs
    unsplit, 257 blocks of 128 keys per CTA. All 32 sequences against the torch
    restatement; one sequence's first KV head (its 8 query heads) against the
    oracle, which keeps the CPU side to a few seconds."""
    d = W.make_c4(seed=5, batch=32, ctx=32768, pool_pages=32 * 2053 + 64, device=dev)
    out, floor = _full_check(d, "C5")
    b = 7
    pages = d["page_table"][b].long()  # this sequence's pages, gathered into a pool of their own
    ref, _, rc = oracle.tree_attention(
        d["q"][b:b + 1, :, 0:8].float().cpu().numpy(), d["k_pool"][pages, :, 0:1].float().cpu().numpy(),
        d["v_pool"][pages, :, 0:1].float().cpu().numpy(),
        np.arange(len(pages), dtype=np.int32)[None, :], d["ctx_lens"][b:b + 1].cpu().numpy(),
        d["parents"][b:b + 1].cpu().numpy(), d["n_nodes"][b:b + 1].cpu().numpy(), 1 / np.sqrt(128))
    assert rc == 0
    AT.assert_close(out[b:b + 1, :, 0:8].float().cpu(), ref, floor[b:b + 1, :, 0:8].cpu(), "C5 vs oracle")
