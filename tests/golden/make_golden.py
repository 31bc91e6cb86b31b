"""Regenerate the golden fixtures of this directory.

Runs where the reference tree is mounted: it builds the reference's own
verifier (oracle/_ref, from src/engine/speculative_verifier.cpp) and records
its decisions, so the committed JSON pins the oracle and the kernels to the
reference on machines without it.

attn_chains.npz comes from the reference's decode attention itself: its paged
KV cache class (engine/kv_cache.py, KVCacheManager.append / get_kv) holds the
keys and values, and the attention statements of A11Pipeline.forward_layer
(engine/pipeline.py, from the "Grouped Query Attention" comment to attn_out)
are read from that file at generation time and executed on the tensors. A
chain-shaped draft tree is exactly the reference's token-by-token decode: node
i attends to the context and nodes 0..i.

    A11_REFERENCE_ROOT=<reference tree> python tests/golden/make_golden.py
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [ROOT, os.path.join(ROOT, "a11-llm-optimizer_b200")]

import oracle  # noqa: E402
from a11spec import workloads as W  # noqa: E402


def c1():
    seed = 1
    d = W.make_c1(seed=seed)
    r = oracle.accept(0, d["logits"], d["tokens"], d["parents"], d["n_nodes"])
    assert r["status"] == 0
    alen = int(r["accept_len"][0])
    # bridge to the reference verifier: greedy decisions as {0,1} linear probabilities
    am = d["logits"][0].argmax(axis=-1)
    lt = [1.0 if d["tokens"][0, i + 1] == am[i] else 0.0 for i in range(5)]
    ref_len, ref_last = oracle.ref_verify(d["tokens"][0, 1:], [1.0] * 5, lt)
    assert ref_len == alen, (ref_len, alen)
    return dict(seed=seed, token_sum=int(d["tokens"].sum()), accept_len=alen,
                accepted_tokens=r["accepted_tokens"][0, :alen].tolist(), bonus=int(r["bonus"][0]),
                ref_accepted_len=ref_len, ref_last_idx=ref_last,
                note="C1 greedy chain; decisions equal the reference verifier's via {0,1} linear probabilities")


def ref_chains():
    rng = np.random.default_rng(7)
    u = oracle.ref_uniform_stream(8)
    cases = []
    for _ in range(64):
        k = int(rng.integers(1, 9))
        q = rng.uniform(0.05, 1.0, k).astype(np.float32)
        p = np.clip(q * rng.uniform(0.2, 1.6, k), 0, 1).astype(np.float32)
        ref_len, ref_last = oracle.ref_verify(np.arange(1, k + 1), q, p)
        cases.append(dict(p=[float(x) for x in p], q=[float(x) for x in q],
                          u=[float(x) for x in u[:k]], ref_accepted_len=ref_len,
                          ref_last_idx=ref_last))
    # the reference's own test vectors (tests/test_speculative_verifier.cpp:77-85, :96-107), log space
    kats = [dict(draft=[-0.1, -0.2, -0.15, -0.3, -0.1, -0.25, -0.2, -0.18],
                 target=[-0.1, -0.2, -0.15, -0.3, -0.1, -0.25, -0.2, -0.18]),
            dict(draft=[-0.5] * 8, target=[-0.1, -0.1, -0.1, -5.0, -0.1, -0.1, -0.1, -0.1]),
            dict(draft=[-0.5, -0.6, -0.7, -0.8], target=[-0.5, -0.6, -0.7, -0.8]),
            dict(draft=[-0.5] * 4, target=[-0.6, -0.6, -10.0, -0.6])]
    for kat in kats:
        n = len(kat["draft"])
        kat["u"] = [float(x) for x in u[:n]]
        kat["ref_accepted_len"], kat["ref_last_idx"] = oracle.ref_verify(
            np.arange(n), kat["draft"], kat["target"])
    return dict(uniform_stream=[float(x) for x in u], cases=cases, log_space_kats=kats,
                note="linear-space chains judged by the reference's verify_draft_tokens with its "
                     "thread_local mt19937(42) stream (u)")


# The reference tree's location; no default. Only the generation below reads it.
REF = os.environ.get("A11_REFERENCE_ROOT", "")


def _reference_attention_statements():
    """The decode-attention statements of the reference's forward_layer, as
    source text read from its file (executed below, not copied here)."""
    lines = open(os.path.join(REF, "engine", "pipeline.py")).read().splitlines()
    i0 = next(i for i, l in enumerate(lines) if "Grouped Query Attention" in l)
    i1 = next(i for i in range(i0, len(lines)) if lines[i].strip().startswith("attn_out ="))
    block = lines[i0:i1 + 1]
    indent = min(len(l) - len(l.lstrip()) for l in block if l.strip())
    return "\n".join(l[indent:] for l in block)


def attn_chains():
    import math
    import types
    import torch
    import torch.nn.functional as F
    sys.path.insert(0, REF)
    from engine.kv_cache import KVCacheManager  # the reference's paged KV cache
    code = compile(_reference_attention_statements(), "engine/pipeline.py (decode attention)", "exec")
    out = {}
    for ci, (ctx, n, hkv, seed) in enumerate(((37, 6, 2, 11), (130, 4, 1, 12), (0, 5, 4, 13))):
        hq, d = 8 * hkv, 128
        g = torch.Generator().manual_seed(seed)
        k = torch.randn(ctx + n, hkv, d, generator=g).to(torch.bfloat16)
        v = torch.randn(ctx + n, hkv, d, generator=g).to(torch.bfloat16)
        q = torch.randn(n, hq, d, generator=g).to(torch.bfloat16)
        cache = KVCacheManager(n_layers=1, n_head_kv=hkv, head_dim=d, page_size=16)
        if ctx:
            cache.append(0, k[:ctx], v[:ctx])  # the prompt
        res = []
        for i in range(n):  # decode the chain token by token, as stream_inference does
            cache.append(0, k[ctx + i:ctx + i + 1], v[ctx + i:ctx + i + 1])
            k_cat, v_cat = cache.get_kv(0, 0, ctx + i + 1)
            ns = dict(torch=torch, math=math, F=F, k_cat=k_cat, v_cat=v_cat, q=q[i:i + 1],
                      cfg=types.SimpleNamespace(n_head=hq, n_head_kv=hkv, head_dim=d),
                      self=types.SimpleNamespace(compute_dtype=torch.bfloat16))
            exec(code, ns)
            res.append(ns["attn_out"].reshape(hq, d))
        bits = lambda t: t.contiguous().view(torch.int16).numpy()
        out[f"c{ci}_meta"] = np.array([ctx, n, hkv], np.int32)
        out[f"c{ci}_q"], out[f"c{ci}_k"], out[f"c{ci}_v"] = bits(q), bits(k), bits(v)
        out[f"c{ci}_out"] = bits(torch.stack(res).to(torch.bfloat16))
    return out


def sampler_probs():
    """Probabilities of the reference's TokenSampler (engine/sampler.py) with
    top-k and top-p off, i.e. softmax(logits / max(T, 1e-5)): the sampler
    runs unchanged, and the probabilities it hands to torch.multinomial are
    recorded. Logits come from a seeded numpy generator the tests rerun."""
    import torch
    sys.path.insert(0, REF)
    from engine.sampler import TokenSampler  # the reference's sampler
    cases = []
    for seed, vocab, temperature in ((21, 32000, 0.7), (22, 151936, 1.3), (23, 4096, 0.05)):
        x = sampler_logits(seed, vocab)
        seen = {}
        multinomial = torch.multinomial
        def record(probs, num_samples=1, **kw):
            seen["p"] = probs.detach().clone()
            return multinomial(probs, num_samples, **kw)
        torch.multinomial = record
        try:
            TokenSampler(temperature=temperature, top_k=0, top_p=1.0).sample_next_token(torch.from_numpy(x.copy()))
        finally:
            torch.multinomial = multinomial
        p = seen["p"].double().numpy()
        rng = np.random.default_rng(seed + 100)
        idx = [int(i) for i in np.argsort(-x)[:8]] + [int(i) for i in rng.choice(vocab, 55, replace=False)]
        cases.append(dict(seed=seed, vocab=vocab, temperature=temperature, tokens=idx,
                          probs=[float(p[i]) for i in idx]))
    return dict(cases=cases, note="p(token) of engine/sampler.py TokenSampler(T, top_k=0, top_p=1.0); logits from "
                                  "sampler_logits(seed, vocab) in make_golden.py")


def sampler_logits(seed, vocab):
    """The logits of a sampler_probs case (also rebuilt by the tests)."""
    x = np.random.default_rng(seed).normal(0.0, 3.0, vocab).astype(np.float32)
    x[seed % vocab] += 10.0
    return x


if __name__ == "__main__":
    if not REF or not os.path.isdir(os.path.join(REF, "engine")):
        sys.exit("make_golden.py: set A11_REFERENCE_ROOT to the reference tree (its engine/ and src/ are read)")
    oracle.build()
    if not oracle.build_ref(REF):
        sys.exit("reference tree not found: golden fixtures need the reference verifier")
    with open(os.path.join(HERE, "c1_greedy_chain.json"), "w") as f:
        json.dump(c1(), f, indent=1)
    with open(os.path.join(HERE, "ref_chains.json"), "w") as f:
        json.dump(ref_chains(), f, indent=1)
    np.savez_compressed(os.path.join(HERE, "attn_chains.npz"), **attn_chains())
    with open(os.path.join(HERE, "sampler_probs.json"), "w") as f:
        json.dump(sampler_probs(), f, indent=1)
    print("golden fixtures written")
