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


TREE_DECODER = dict(n_layers=2, n_embd=256, n_head=8, n_head_kv=1, head_dim=128, n_ff=512, vocab=512)
TREE_DECODER_SEED = 7
TREE_DECODER_STEPS = 40


def tree_decoder_decode():
    """Greedy decode of a small synthetic decoder by the reference's own
    A11Pipeline.forward_token / forward_layer (engine/pipeline.py:350-473, its
    dense SwiGLU branch, bf16 compute, its KVCacheManager holding the keys and
    values), on the seeded weights of a11spec.tree_model.synthetic_tensors.
    The prompt is the first of a seeded series whose first 20 greedy steps all
    have a top-2 logit gap of at least 0.1 (bf16 logits tie often; a gap that
    wide cannot be closed by rounding differences between machines), and 40
    steps are recorded with their logits and gaps."""
    import types
    import torch
    sys.path.insert(0, REF)
    from engine.kv_cache import KVCacheManager  # the reference's KV cache
    from engine.pipeline import A11Pipeline  # the reference's decoder (its methods run unchanged)
    from a11spec.tree_model import DecoderConfig, synthetic_tensors
    cfg = DecoderConfig(**TREE_DECODER)
    tensors = synthetic_tensors(cfg, TREE_DECODER_SEED)

    def reference_pipeline():
        pipe = A11Pipeline.__new__(A11Pipeline)  # no model files: the decoder state only
        pipe.config = types.SimpleNamespace(n_head=cfg.n_head, n_head_kv=cfg.n_head_kv, head_dim=cfg.head_dim,
                                            rms_eps=cfg.rms_eps, rope_base=cfg.rope_base)
        pipe.weights = types.SimpleNamespace(get_torch=lambda name: tensors[name])
        pipe.loader = types.SimpleNamespace(tensors=dict.fromkeys(tensors))
        pipe.kv_cache_manager = KVCacheManager(n_layers=cfg.n_layers, n_head_kv=cfg.n_head_kv,
                                               head_dim=cfg.head_dim, page_size=16)
        pipe.device = torch.device("cpu")
        pipe.compute_dtype = torch.bfloat16
        pipe.num_layers = cfg.n_layers
        return pipe

    for prompt_seed in range(100):
        prompt = np.random.default_rng(prompt_seed).integers(0, cfg.vocab, 6).astype(np.int32)
        pipe = reference_pipeline()
        for pos, tok in enumerate(prompt[:-1]):
            pipe.forward_token(int(tok), pos)
        tok, pos = int(prompt[-1]), len(prompt) - 1
        out, rows, gaps = [], [], []
        for _ in range(TREE_DECODER_STEPS):
            logits = pipe.forward_token(tok, pos).float()
            top = torch.topk(logits, 2).values
            gaps.append(float(top[0] - top[1]))
            rows.append(logits.numpy())
            tok = int(torch.argmax(logits))
            out.append(tok)
            pos += 1
        if min(gaps[:20]) >= 0.1:
            return dict(prompt=prompt, tokens=np.array(out, np.int32), logits=np.stack(rows).astype(np.float32),
                        gaps=np.array(gaps, np.float32), prompt_seed=np.int32(prompt_seed),
                        weight_seed=np.int32(TREE_DECODER_SEED))
    raise RuntimeError("no prompt with 20 well-separated greedy steps")


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
    np.savez_compressed(os.path.join(HERE, "tree_decoder_decode.npz"), **tree_decoder_decode())
    print("golden fixtures written")
