"""Regenerate the golden fixtures of this directory.

Runs where the reference tree is mounted: it builds the reference's own
verifier (oracle/_ref, from src/engine/speculative_verifier.cpp) and records
its decisions, so the committed JSON pins the oracle and the kernels to the
reference on machines without it.

    python tests/golden/make_golden.py
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


if __name__ == "__main__":
    oracle.build()
    if not oracle.build_ref():
        sys.exit("reference tree not found: golden fixtures need the reference verifier")
    with open(os.path.join(HERE, "c1_greedy_chain.json"), "w") as f:
        json.dump(c1(), f, indent=1)
    with open(os.path.join(HERE, "ref_chains.json"), "w") as f:
        json.dump(ref_chains(), f, indent=1)
    print("golden fixtures written")
