"""The benchmark configurations at their full sizes, every sequence against the
oracle, through the C ABI:

* C4: greedy acceptance on the bf16 [32, 64, 151936] logits with 50 % forced
  matches, then compaction of the accepted nodes' K/V (whole pools compared bit
  for bit, page tables, lengths and detached pages) and the page allocator
  taking the detached pages back;
* C5: one-hot sampling acceptance at T = 0.7 on [32, 64, 151936] bf16 logits
  from the C5 LM head, over trees drafted from the C5 trigram table, with
  forced matches so that walks leave the root.

Decisions (accepted lengths, nodes, tokens, bonus), compacted K/V and page
tables are bit-exact; the reference's rule is src/engine/speculative_verifier.cpp:84-135.
"""
import numpy as np
import pytest
import torch

import a11spec
import oracle
from a11spec import workloads as W

pytestmark = pytest.mark.gpu
VOCAB = 151936


def _same_decisions(r, o, B):
    for name in ("accept_len", "accepted_nodes", "accepted_tokens", "bonus"):
        got = getattr(r, name).cpu().numpy()
        np.testing.assert_array_equal(got, o[name], err_msg=name)
    assert o["status"] == 0


def test_c4_accept_compact_release_full_size(dev):
    d = W.make_c4(seed=4, batch=32, device=dev)
    B, N = 32, 64
    P = d["k_pool"].shape[0]
    # the step's attention runs first (its numerics: test_kv_ngram_attn_gpu.py)
    a11spec.tree_attention(d["q"], d["k_pool"], d["v_pool"], d["page_table"], d["ctx_lens"], d["parents"],
                           d["n_nodes"], check_status=True)
    # K3: greedy acceptance, all 32 sequences
    r = a11spec.accept(a11spec.GREEDY, d["logits"], d["tokens"], d["parents"], d["n_nodes"], check_status=True)
    tokens, parents, nn = (d[k].cpu().numpy() for k in ("tokens", "parents", "n_nodes"))
    o = oracle.accept(0, d["logits"].float().cpu().numpy(), tokens, parents, nn)
    _same_decisions(r, o, B)
    alen = r.accept_len.cpu().numpy()
    assert alen.max() >= 2 and (alen > 0).sum() >= 8, alen  # forced matches: walks leave the root
    # K5 state: the allocator owns every pool page that no table holds
    pool = a11spec.KVPagePool(P, dev)
    pool.adopt(d["page_table"])
    stack0, top0 = pool.free_pages().cpu().numpy(), int(pool.free_top.item())
    # K4: compaction of the accepted paths, against the oracle on the whole pools
    k0 = d["k_pool"].cpu().view(torch.int16).numpy()
    v0 = d["v_pool"].cpu().view(torch.int16).numpy()
    pt0, len0 = d["page_table"].cpu().numpy(), d["ctx_lens"].cpu().numpy()
    o4 = oracle.kv_compact(k0, v0, pt0, len0, o["accept_len"], o["accepted_nodes"], nn)
    assert o4["status"] == 0
    freed, n_freed = a11spec.kv_compact(d["k_pool"], d["v_pool"], d["page_table"], d["ctx_lens"], r.accept_len,
                                        r.accepted_nodes, d["n_nodes"], check_status=True)
    torch.cuda.synchronize()
    assert torch.equal(d["k_pool"].view(torch.int16), torch.from_numpy(o4["k_pool"]).to(dev))
    assert torch.equal(d["v_pool"].view(torch.int16), torch.from_numpy(o4["v_pool"]).to(dev))
    np.testing.assert_array_equal(d["page_table"].cpu().numpy(), o4["page_table"])
    np.testing.assert_array_equal(d["ctx_lens"].cpu().numpy(), o4["seq_lens"])
    np.testing.assert_array_equal(n_freed.cpu().numpy(), o4["n_freed"])
    np.testing.assert_array_equal(freed.cpu().numpy(), o4["freed_pages"])
    assert np.array_equal(o4["seq_lens"], len0 + 1 + alen)
    # K5: the detached pages go back on the free stack
    pool.release(freed, n_freed, check_status=True)
    o5 = oracle.kv_release(stack0, top0, P, o4["freed_pages"], o4["n_freed"])
    assert int(pool.free_top.item()) == int(o5["top"]) == top0 + int(o4["n_freed"].sum())
    np.testing.assert_array_equal(pool.free_pages().cpu().numpy(), o5["stack"])


def test_c5_onehot_sampling_full_shape(dev):
    """C5 acceptance: trees from the C5 trigram table (K1), logits from the C5
    LM head (hidden [2048, 2048] x W [2048, 151936], bf16); half of the drafted
    nodes are made likely (their token gets +12 in the parent's row) so the
    walks go deep and the rejections exercise the residual renormalisation."""
    B, N, T = 32, 64, 0.7
    table = torch.from_numpy(W.make_ngram_table(20, 8, VOCAB, 1.2, seed=5)).to(dev)
    rng = np.random.default_rng(55)
    last = torch.from_numpy(rng.integers(0, VOCAB, (B, 2)).astype(np.int32)).to(dev)
    tk, pa, _, nn = a11spec.ngram_expand(table, last, 4, 2, 5, N)
    g = torch.Generator(device=dev).manual_seed(8)
    hidden = torch.randn(B * N, 2048, generator=g, device=dev).to(torch.bfloat16)
    w = (0.02 * torch.randn(2048, VOCAB, generator=g, device=dev)).to(torch.bfloat16)
    logits = (hidden @ w).view(B, N, VOCAB)
    tok, par, n = tk.cpu().numpy(), pa.cpu().numpy(), nn.cpu().numpy()
    force = rng.random((B, N)) < 0.5
    for b in range(B):
        for i in range(1, int(n[b])):
            if force[b, i]:
                logits[b, par[b, i], tok[b, i]] += 12.0
    uni = torch.rand(B, N, generator=g, device=dev)
    stats = torch.zeros(6, dtype=torch.int64, device=dev)
    r = a11spec.accept(a11spec.STOCH_ONEHOT, logits, tk, pa, nn, temperature=T, uniforms=uni, stats=stats,
                       want_node_probs=True, check_status=True)
    o = oracle.accept(1, logits.float().cpu().numpy(), tok, par, n, temperature=T, uniforms=uni.cpu().numpy())
    _same_decisions(r, o, B)
    np.testing.assert_array_equal(r.node_probs.cpu().numpy(), o["node_probs"])  # bit-identical softmax
    alen = r.accept_len.cpu().numpy()
    assert alen.max() >= 3 and (alen > 0).sum() >= 16, alen
    s = stats.cpu().numpy()
    assert s[4] == B and s[5] == int(alen.sum()) + B and s[3] == int((n - 1).sum())
