"""CPU tests: the oracle against golden vectors, the reference verifier (when
built here), numpy/torch restatements, and the C-ABI library's symbol table."""
import ctypes
import json
import math
import os
import re

import numpy as np
import pytest
import torch

import oracle
from a11spec import workloads as W

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")


def load_golden(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


# ----------------------------------------------------------------------------- numerics
def test_exp2_poly_accuracy():
    L = oracle.lib()
    fs = np.linspace(-0.5, 0.5, 20001, dtype=np.float32)
    got = np.array([L.or_exp2_poly(float(f)) for f in fs], dtype=np.float64)
    rel = np.abs(got / np.exp2(fs.astype(np.float64)) - 1)
    assert rel.max() < 3e-7


def test_weight_matches_exact_power():
    k = oracle.temperature_k(0.7)
    rng = np.random.default_rng(0)
    for l in rng.normal(0, 4, 200).astype(np.float32):
        c = int(math.ceil(np.float32(12.0) * np.float32(k)))
        w = oracle.weight(float(l), k, c)
        exact = 2.0 ** (float(np.float32(l)) * k - c) * 2.0 ** 40
        # t = l*k - c is rounded to fp32 (|t| < 64: error <= 2^-18 in the
        # exponent), the polynomial adds 2.2e-7, truncation one unit
        assert abs(w - exact) <= exact * 5e-6 + 1
    assert oracle.weight(float("-inf"), k, 0) == 0


@pytest.mark.parametrize("temp", [0.7, 1.0, 0.05])
def test_fixed_point_softmax_close_to_float64(temp):
    rng = np.random.default_rng(1)
    V = 10000
    row = rng.normal(0, 3, V).astype(np.float32)
    row[17] = -np.inf
    tgt = np.zeros((1, 2, V), np.float32)
    tgt[0, 0] = row
    tokens = np.array([[0, 5]], np.int32)
    parents = np.array([[-1, 0]], np.int32)
    toks = rng.integers(0, V, 64)
    z = row.astype(np.float64) / temp
    ref = np.exp(z - z.max())
    ref /= ref.sum()
    for x in toks:
        tokens[0, 1] = x
        r = oracle.accept(1, tgt, tokens, parents, temperature=temp,
                          uniforms=np.array([[0.999, 0.999]], np.float32))
        assert r["status"] == 0
        p = r["node_probs"][0, 1]
        assert abs(p - ref[x]) <= 1e-5 * ref[x] + 1e-9


# ----------------------------------------------------------------------------- golden vectors
def test_golden_c1_greedy_chain():
    g = load_golden("c1_greedy_chain.json")
    d = W.make_c1(seed=g["seed"])
    assert int(d["tokens"].sum()) == g["token_sum"]
    r = oracle.accept(0, d["logits"], d["tokens"], d["parents"], d["n_nodes"])
    assert r["status"] == 0
    assert int(r["accept_len"][0]) == g["accept_len"]
    assert r["accepted_tokens"][0, : g["accept_len"]].tolist() == g["accepted_tokens"]
    assert int(r["bonus"][0]) == g["bonus"]


def test_golden_reference_chains():
    """Stochastic chains whose decisions came from the reference's own verifier."""
    g = load_golden("ref_chains.json")
    for case in g["cases"]:
        n = len(case["p"])
        V = 8
        # build a target row per node whose softmax-free probability is given:
        # the oracle's linear-space rule is exercised through or_accept with
        # one-hot drafts on crafted logits; here we check the rule directly.
        acc = 0
        for i in range(n):
            lt = min(max(case["p"][i], 0.0), 1.0 + 1e-6)
            ld = min(max(case["q"][i], 1e-10), 1.0)
            a = np.float32(np.float32(lt) / np.float32(ld))
            a = min(a, np.float32(1.0))
            if np.float32(case["u"][i]) < a:
                acc += 1
            else:
                break
        assert acc == case["ref_accepted_len"], case


def test_reference_kats_against_shim():
    R = oracle.ref()
    if R is None:
        pytest.skip("reference verifier not built on this machine")
    # tests/test_speculative_verifier.cpp:77-85 and :96-107 of the reference
    lp = [-0.1, -0.2, -0.15, -0.3, -0.1, -0.25, -0.2, -0.18]
    assert oracle.ref_verify(list(range(1, 9)), lp, lp) == (8, 7)
    a, last = oracle.ref_verify([10, 20, 30, 40, 50, 60, 70, 80], [-0.5] * 8,
                                [-0.1, -0.1, -0.1, -5.0, -0.1, -0.1, -0.1, -0.1])
    assert 0 < a <= 8 and last < 7
    assert R.ref_verify_mismatch(3, 2, 3) == 1


def test_oracle_chain_matches_reference_verifier_live():
    """Greedy bridge: linear-space {0,1} probabilities make the reference's
    decisions RNG-independent; both must agree on C1-style chains."""
    if oracle.ref() is None:
        pytest.skip("reference verifier not built on this machine")
    for seed in range(20):
        d = W.make_c1(seed=seed, vocab=4000)
        r = oracle.accept(0, d["logits"], d["tokens"], d["parents"], d["n_nodes"])
        am = d["logits"][0].argmax(axis=-1)
        lt = [1.0 if d["tokens"][0, i + 1] == am[i] else 0.0 for i in range(5)]
        ref_len, _ = oracle.ref_verify(d["tokens"][0, 1:], [1.0] * 5, lt)
        assert ref_len == int(r["accept_len"][0])


def test_oracle_stochastic_chain_matches_reference_verifier_live():
    """Sampling bridge: hand the reference the oracle's p(x) (linear space) with
    its own mt19937(42) uniforms; accepted lengths must be identical."""
    if oracle.ref() is None:
        pytest.skip("reference verifier not built on this machine")
    u = oracle.ref_uniform_stream(8)
    rng = np.random.default_rng(3)
    V, n = 2048, 6
    for trial in range(30):
        tgt = rng.normal(0, 1, (1, n, V)).astype(np.float32)
        tokens = np.zeros((1, n), np.int32)
        parents = W.chain_parents(n)[None]
        for i in range(1, n):  # favour likely tokens so chains get long
            tokens[0, i] = int(np.argsort(tgt[0, i - 1])[-1 - rng.integers(0, 3)])
        T = 0.05
        uni = np.zeros((1, n), np.float32)
        uni[0, 1:] = u[: n - 1]
        r = oracle.accept(1, tgt, tokens, parents, temperature=T, uniforms=uni)
        assert r["status"] == 0
        p = r["node_probs"][0, 1:]
        ref_len, _ = oracle.ref_verify(tokens[0, 1:], np.ones(n - 1, np.float32), p)
        assert ref_len == int(r["accept_len"][0]), (trial, p, u[: n - 1])


# ----------------------------------------------------------------------------- acceptance semantics
def test_oracle_greedy_tree_walk_rules():
    V = 64
    tgt = np.full((1, 5, V), -1.0, np.float32)
    parents = np.array([[-1, 0, 0, 1, 2]], np.int32)
    tokens = np.array([[7, 3, 9, 11, 12]], np.int32)
    tgt[0, 0, 9] = 5.0   # root argmax 9 -> child 2
    tgt[0, 2, 12] = 5.0  # node 2 argmax 12 -> child 4
    tgt[0, 4, 40] = 5.0  # bonus 40
    r = oracle.accept(0, tgt, tokens, parents)
    assert r["accept_len"][0] == 2
    assert r["accepted_nodes"][0, :3].tolist() == [2, 4, -1]
    assert r["accepted_tokens"][0, :2].tolist() == [9, 12]
    assert r["bonus"][0] == 40
    # ties: lowest index wins
    tgt2 = np.zeros((1, 2, V), np.float32)
    r2 = oracle.accept(0, tgt2, np.array([[0, 0]], np.int32), np.array([[-1, 0]], np.int32))
    assert r2["accept_len"][0] == 1 and r2["bonus"][0] == 0


def test_oracle_status_codes():
    V = 64
    tgt = np.zeros((1, 3, V), np.float32)
    par = np.array([[-1, 0, 1]], np.int32)
    assert oracle.accept(0, tgt, np.array([[0, 1, V]], np.int32), par)["status"] == 2
    assert oracle.accept(0, tgt, np.array([[0, 1, 2]], np.int32), np.array([[-1, 0, 2]], np.int32))["status"] == 2
    bad = tgt.copy()
    bad[0, 1, 5] = np.nan
    assert oracle.accept(0, bad, np.array([[0, 1, 2]], np.int32), par)["status"] == 5
    assert oracle.accept(0, tgt, np.array([[0, 1, 2]], np.int32), par,
                         n_nodes=np.array([4], np.int32))["status"] == 2


def test_oracle_onehot_residual_excludes_rejected_tokens():
    """After rejecting sibling x, p'(x) is 0 so a duplicate sibling is rejected."""
    V = 32
    tgt = np.zeros((1, 3, V), np.float32)
    tgt[0, 0, 5] = 3.0
    toks = np.array([[1, 5, 5]], np.int32)
    par = np.array([[-1, 0, 0]], np.int32)
    uni = np.array([[0.5, 0.999999, 0.0]], np.float32)  # reject first 5, second has p'=0
    r = oracle.accept(1, tgt, toks, par, temperature=1.0, uniforms=uni)
    assert r["accept_len"][0] == 0
    assert r["bonus"][0] != 5


# ----------------------------------------------------------------------------- attention
def torch_tree_attention(q, k_pool, v_pool, page_table, ctx_lens, parents, n_nodes, scale):
    """engine/pipeline.py:391-402 restated for a tree (fp32 scores, bf16 probs)."""
    B, N, Hq, D = q.shape
    Hkv = k_pool.shape[2]
    rep = Hq // Hkv
    out = torch.zeros(B, N, Hq, D)
    for b in range(B):
        L = int(ctx_lens[b])
        for i in range(int(n_nodes[b])):
            anc = set()
            a = i
            while a >= 0:
                anc.add(a)
                a = int(parents[b, a])
            pos = list(range(L)) + [L + j for j in sorted(anc)]
            pg = page_table[b, torch.tensor(pos) // 16].long()
            sl = torch.tensor(pos) % 16
            kk = k_pool[pg, sl].float().repeat_interleave(rep, dim=1)  # [S, Hq, D]
            vv = v_pool[pg, sl].float().repeat_interleave(rep, dim=1)
            s = torch.einsum("hd,shd->hs", q[b, i].float(), kk) * scale
            p = torch.softmax(s, dim=-1).to(torch.bfloat16).float()
            out[b, i] = torch.einsum("hs,shd->hd", p, vv)
    return out


def test_oracle_attention_matches_torch_restatement():
    rng = np.random.default_rng(5)
    B, N, Hq, Hkv, D, ctx = 2, 7, 4, 2, 16, 37
    parents = np.stack([W.random_parents(N, rng) for _ in range(B)])
    P = 40
    kv = W.paged_kv(B, ctx, N, Hkv, D, P, seed=9, device="cpu")
    q = torch.randn(B, N, Hq, D).to(torch.bfloat16)
    nn = np.array([N, N - 2], np.int32)
    ref = torch_tree_attention(q, kv["k_pool"], kv["v_pool"], kv["page_table"], kv["ctx_lens"],
                               torch.from_numpy(parents), nn, 0.25)
    out, lse, rc = oracle.tree_attention(q.float().numpy(), kv["k_pool"].float().numpy(),
                                         kv["v_pool"].float().numpy(), kv["page_table"].numpy(),
                                         kv["ctx_lens"].numpy(), parents, nn, 0.25)
    assert rc == 0
    np.testing.assert_allclose(out, ref.numpy(), rtol=1e-4, atol=1e-4)
    assert np.all(out[1, N - 2:] == 0)


# ----------------------------------------------------------------------------- compaction
def test_oracle_compaction_semantics():
    P, Hkv, D = 8, 1, 8
    k = np.arange(P * 16 * Hkv * D, dtype=np.float32).reshape(P, 16, Hkv, D)
    v = -k
    pt = np.array([[3, 5, 6, 1]], np.int32)  # ctx 14 + 20 nodes -> pages 0..2 used
    L, n = 14, 20
    nodes = np.full((1, n), -1, np.int32)
    nodes[0, :3] = [2, 5, 9]
    res = oracle.kv_compact(k, v, pt, np.array([L], np.int32), np.array([3], np.int32), nodes,
                            np.array([n], np.int32))
    assert res["status"] == 0
    assert res["seq_lens"][0] == L + 4

    def row(pool, pos, tab):
        return pool[tab[pos // 16], pos % 16]

    for j, node in enumerate([2, 5, 9]):
        np.testing.assert_array_equal(row(res["k_pool"], L + 1 + j, pt[0]), row(k, L + node, pt[0]))
        np.testing.assert_array_equal(row(res["v_pool"], L + 1 + j, pt[0]), row(v, L + node, pt[0]))
    # new length 18 -> pages 0,1 kept; page 2 (slots 32..47) held tree slots -> freed
    assert res["page_table"][0].tolist() == [3, 5, -1, 1]
    assert res["n_freed"][0] == 1 and res["freed_pages"][0, 0] == 6


# ----------------------------------------------------------------------------- n-gram
def splitmix_bucket(a, b, log2b):
    z = ((a & 0xFFFFFFFF) << 32) | (b & 0xFFFFFFFF)
    m = (1 << 64) - 1
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & m
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & m
    z ^= z >> 31
    return z >> (64 - log2b)


def test_oracle_ngram_bucket_and_tree_shape():
    for a, b in [(0, 0), (1, 2), (151935, 7), (-1, 5)]:
        assert oracle.ngram_bucket(a, b, 20) == splitmix_bucket(a, b, 20)
    table = W.make_ngram_table(log2_buckets=10, vocab=1000, seed=1)
    table[5, :, 1] = 0  # an empty bucket
    last = np.array([[1, 2], [3, 4]], np.int32)
    r = oracle.ngram_expand(table, 10, last, 4, 2, 5, 64)
    assert r["status"] == 0
    for b in range(2):
        n = r["n_nodes"][b]
        assert n == 64  # full buckets -> 1+4+8+16+32 = 61, plus 3 at depth 5
        par, dep = r["parents"][b, :n], r["depths"][b, :n]
        assert par[0] == -1 and all(0 <= par[i] < i for i in range(1, n))
        assert dep.max() == 5 and np.sum(dep == 1) == 4
        assert r["tokens"][b, 0] == last[b, 1]


def test_library_loads_and_exports_every_declared_symbol():
    from a11spec import _lib
    hdr = open(os.path.join(ROOT, "include", "a11spec.h")).read()
    declared = set(re.findall(r"\b(a11s_\w+)\s*\(", hdr))
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [s for s in sorted(declared) if not hasattr(lib, s)]
    assert not missing, missing
    assert declared == set(_lib.symbols())
    assert lib.a11s_abi_version() == 1


def test_every_entry_point_with_parameters_has_ctypes_argtypes():
    """Undeclared argtypes make ctypes pass 64-bit pointers as 32-bit ints."""
    from a11spec import _lib
    hdr = open(os.path.join(ROOT, "include", "a11spec.h")).read()
    for name, params in re.findall(r"\b(a11s_\w+)\s*\(([^)]*)\)", hdr):
        f = getattr(_lib.lib, name)
        if params.strip() in ("", "void"):
            continue
        assert f.argtypes is not None, name
        assert len(f.argtypes) == len(params.split(",")), name
