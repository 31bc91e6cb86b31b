"""Edge cases across the entry points, on the GPU against the oracle: empty
batches, a vocab whose last 2048-token chunk is ragged, the largest vocab and
tree the acceptance kernel takes (and the limit errors just past them),
attention with no context (the tree only) and root-only trees, compaction
with nothing accepted."""
import numpy as np
import pytest
import torch

import a11spec
import attn_tolerance as AT
import oracle
from a11spec import workloads as W

pytestmark = pytest.mark.gpu


def _accept(mode, x, tokens, parents, nn=None, T=1.0, uni=None):
    dev = "cuda"
    r = a11spec.accept(mode, torch.as_tensor(x, device=dev), torch.as_tensor(tokens, device=dev),
                       torch.as_tensor(parents, device=dev), None if nn is None else torch.as_tensor(nn, device=dev),
                       temperature=T, uniforms=None if uni is None else torch.as_tensor(uni, device=dev),
                       check_status=True)
    o = oracle.accept(mode, np.asarray(x), np.asarray(tokens), np.asarray(parents),
                      None if nn is None else np.asarray(nn), temperature=T,
                      uniforms=None if uni is None else np.asarray(uni))
    for k in ("accept_len", "accepted_nodes", "accepted_tokens", "bonus"):
        np.testing.assert_array_equal(getattr(r, k).cpu().numpy(), o[k], err_msg=k)
    return r


def _tree(rng, B, N, V, x, p_force=0.7):
    parents = np.stack([W.random_parents(N, rng) for _ in range(B)]).astype(np.int32)
    tokens = rng.integers(0, V, (B, N)).astype(np.int32)
    for b in range(B):
        for i in range(1, N):
            if rng.random() < p_force:
                x[b, parents[b, i], tokens[b, i]] += 40.0
    return tokens, parents


def test_empty_batches(dev):
    V, N = 4096, 8
    ws = torch.full((256,), 255, dtype=torch.uint8, device=dev)  # a stale status word must be cleared
    r = a11spec.accept(0, torch.zeros(0, N, V, device=dev), torch.zeros(0, N, dtype=torch.int32, device=dev),
                       torch.zeros(0, N, dtype=torch.int32, device=dev), ws=ws, check_status=True)
    assert r.accept_len.numel() == 0
    ws.fill_(255)
    q = torch.zeros(0, N, 16, 128, dtype=torch.bfloat16, device=dev)
    pool = torch.zeros(4, 16, 2, 128, dtype=torch.bfloat16, device=dev)
    a11spec.tree_attention(q, pool, pool, torch.zeros(0, 4, dtype=torch.int32, device=dev),
                           torch.zeros(0, dtype=torch.int32, device=dev), torch.zeros(0, N, dtype=torch.int32, device=dev),
                           ws=ws, check_status=True)
    table = torch.zeros(1 << 6, 4, 2, dtype=torch.int32, device=dev)
    tk, pa, de, nn = a11spec.ngram_expand(table, torch.zeros(0, 2, dtype=torch.int32, device=dev), 2, 1, 3, 8)
    assert tk.numel() == 0
    pool = a11spec.KVPagePool(8, dev)
    pool.reserve(torch.zeros(0, 4, dtype=torch.int32, device=dev), torch.zeros(0, dtype=torch.int32, device=dev),
                 torch.zeros(0, dtype=torch.int32, device=dev), check_status=True)
    assert int(pool.free_top.item()) == 8


@pytest.mark.parametrize("mode", [0, 1])
def test_ragged_last_chunk(dev, mode):
    rng = np.random.default_rng(3)
    B, N, V = 4, 24, 2048 * 3 + 136  # 3 full chunks and one of 136 tokens
    x = rng.normal(0, 2, (B, N, V)).astype(np.float32)
    tokens, parents = _tree(rng, B, N, V, x)
    tokens[:, 1:4] = V - 1 - np.arange(3)  # children in the ragged chunk
    for b in range(B):
        x[b, 0, V - 1] += 60.0
    _accept(mode, x, tokens, parents, T=0.8, uni=rng.random((B, N)).astype(np.float32) if mode else None)


def test_largest_vocab_and_tree(dev):
    rng = np.random.default_rng(4)
    B, N, V = 2, 16, 1 << 18  # the largest vocab
    x = rng.normal(0, 2, (B, N, V)).astype(np.float32)
    tokens, parents = _tree(rng, B, N, V, x)
    _accept(0, x, tokens, parents)
    _accept(1, x, tokens, parents, T=0.7, uni=rng.random((B, N)).astype(np.float32))
    B, N, V = 2, 256, 4096  # the largest tree
    x = rng.normal(0, 2, (B, N, V)).astype(np.float32)
    tokens, parents = _tree(rng, B, N, V, x, p_force=0.9)
    _accept(0, x, tokens, parents, nn=np.array([256, 200], np.int32))


def test_limits_just_past_the_maximum(dev):
    tok = torch.zeros(1, 257, dtype=torch.int32, device=dev)
    par = torch.full((1, 257), 0, dtype=torch.int32, device=dev)
    par[0, 0] = -1
    with pytest.raises(a11spec.A11Error) as e:
        a11spec.accept(0, torch.zeros(1, 257, 64, device=dev), tok, par)
    assert e.value.code == a11spec.EUNSUPPORTED
    with pytest.raises(a11spec.A11Error) as e:
        a11spec.accept(0, torch.zeros(1, 2, (1 << 18) + 4, device=dev), tok[:, :2], par[:, :2])
    assert e.value.code == a11spec.EUNSUPPORTED


@pytest.mark.parametrize("ctx,N", [(0, 20), (0, 1), (33, 1)])
def test_attention_tree_only_and_root_only(dev, ctx, N):
    B, Hkv = 2, 2
    kv = W.paged_kv(B, ctx, N, Hkv, 128, B * ((ctx + N + 15) // 16), seed=7, device=dev)
    g = torch.Generator(device=dev).manual_seed(8)
    q = torch.randn(B, N, Hkv * 8, 128, device=dev, generator=g).to(torch.bfloat16)
    par = torch.from_numpy(np.stack([W.random_parents(N, np.random.default_rng(b)) for b in range(B)])).to(dev)
    nn = torch.full((B,), N, dtype=torch.int32, device=dev)
    out, _, _ = a11spec.tree_attention(q, kv["k_pool"], kv["v_pool"], kv["page_table"], kv["ctx_lens"], par, nn,
                                       check_status=True)
    ref, _, rc = oracle.tree_attention(q.float().cpu().numpy(), kv["k_pool"].float().cpu().numpy(),
                                       kv["v_pool"].float().cpu().numpy(), kv["page_table"].cpu().numpy(),
                                       kv["ctx_lens"].cpu().numpy(), par.cpu().numpy(), nn.cpu().numpy(),
                                       1 / np.sqrt(128))
    assert rc == 0
    _, floor = AT.reference(q, kv["k_pool"], kv["v_pool"], kv["page_table"], kv["ctx_lens"], par, nn)
    AT.assert_close(out.float().cpu(), ref, floor.cpu(), f"ctx {ctx}, {N} nodes")


def test_compaction_with_nothing_accepted(dev):
    B, N, ctx, Hkv = 3, 20, 50, 2
    kv = W.paged_kv(B, ctx, N, Hkv, 128, B * ((ctx + N + 15) // 16), seed=9, device=dev)
    alen = torch.zeros(B, dtype=torch.int32, device=dev)
    nodes = torch.full((B, N), -1, dtype=torch.int32, device=dev)
    nn = torch.full((B,), N, dtype=torch.int32, device=dev)
    o = oracle.kv_compact(kv["k_pool"].cpu().view(torch.int16).numpy(), kv["v_pool"].cpu().view(torch.int16).numpy(),
                          kv["page_table"].cpu().numpy(), kv["ctx_lens"].cpu().numpy(), alen.cpu().numpy(),
                          nodes.cpu().numpy(), nn.cpu().numpy())
    freed, nf = a11spec.kv_compact(kv["k_pool"], kv["v_pool"], kv["page_table"], kv["ctx_lens"], alen, nodes, nn,
                                   check_status=True)
    torch.cuda.synchronize()
    assert kv["ctx_lens"].cpu().tolist() == [ctx + 1] * B  # the root stays
    np.testing.assert_array_equal(kv["page_table"].cpu().numpy(), o["page_table"])
    np.testing.assert_array_equal(nf.cpu().numpy(), o["n_freed"])
    np.testing.assert_array_equal(kv["k_pool"].cpu().view(torch.int16).numpy(), o["k_pool"])
