"""Seeded single-kernel cases for timing and profiling.

    python bench_cases.py attention --batch 16 --ctx 4096 --iters 2
    python bench_cases.py accept --mode onehot --batch 32 --iters 2
    python bench_cases.py compact --batch 32 --ctx 4096 --iters 2
    python bench_cases.py ngram --batch 32 --iters 2
    python bench_cases.py pages --batch 32 --ctx 32768 --iters 20
    python bench_cases.py lm_head --batch 32 --nodes 64 --vocab 32768 --iters 2

Each case builds its inputs on cuda:0 (seeded), runs the kernel `--warmup`
times, then `--iters` times between CUDA events, and prints one JSON line
with the mean device time per launch and the algorithmic bytes or FLOPs of
one launch. A profiler wrapped around the command sees warmup + iters
launches of the kernel, nothing else of this library.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "a11-llm-optimizer_b200"))

import numpy as np
import torch

import a11spec
from a11spec import workloads as W

VOCAB = 151936


def _time(fn, warmup: int, iters: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) * 1e3 / max(iters, 1)


def _random_trees(batch: int, nodes: int, dev: str) -> torch.Tensor:
    return torch.from_numpy(np.stack([W.random_parents(nodes, np.random.default_rng(b)) for b in range(batch)])).to(dev)


def case_attention(a) -> dict:
    """Tree attention, GQA 32/4, head_dim 128, random 64-node trees (C4/C5 shapes)."""
    dev = "cuda"
    B, N, HQ, HKV, D, ctx = a.batch, a.nodes, 32, 4, 128, a.ctx
    kv = W.paged_kv(B, ctx, N, HKV, D, B * ((ctx + N + 15) // 16), seed=3, device=dev)
    g = torch.Generator(device=dev).manual_seed(4)
    q = torch.randn(B, N, HQ, D, device=dev, generator=g).to(torch.bfloat16)
    par = _random_trees(B, N, dev)
    nn = torch.full((B,), N, dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    ws = a11spec.ops.workspace(a11spec.ops.tree_attention_workspace_bytes(B, N, HQ, HKV, D, ctx + N), dev)

    def run():
        a11spec.tree_attention(q, kv["k_pool"], kv["v_pool"], kv["page_table"], kv["ctx_lens"], par, nn,
                               max_kv_len=ctx + N, out=out, ws=ws)

    us = _time(run, a.warmup, a.iters)
    flops = 4.0 * B * N * HQ * D * (ctx + (N + 1) / 2)  # QK^T and PV over the visible keys
    kv_bytes = 2.0 * B * (ctx + N) * HKV * D * 2
    return {"case": "attention", "batch": B, "ctx": ctx, "nodes": N, "us": us, "flops": flops,
            "tflops": flops / us / 1e6, "kv_bytes": kv_bytes}


def case_accept(a) -> dict:
    """Acceptance over bf16 logits [batch, 64, 151936] (greedy / one-hot, random
    drafts: walks stop at the root), the C4 greedy case (make_c4: random trees,
    50 % of the drafts forced to their parent's argmax, so walks go deep) or
    fp32 p and q [batch, 63, 151936] (draft mode, C3 shape)."""
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(5)
    if a.mode == "c4greedy":
        d = W.make_c4(seed=4, batch=a.batch, device=dev)
        args = (a11spec.GREEDY, d["logits"], d["tokens"], d["parents"], d["n_nodes"])
        kw = {}
        nbytes = d["logits"].numel() * 2.0
    elif a.mode == "draft":
        d = W.make_c3(seed=3, batch=a.batch, device=dev)
        args = (2, d["p"], d["tokens"], d["parents"], d["n_nodes"])
        kw = dict(draft_logits=d["q"], temperature=0.8, uniforms=d["uniforms"])
        nbytes = 2.0 * d["p"].numel() * 4
    else:
        B, N = a.batch, a.nodes
        logits = (2 * torch.randn(B, N, VOCAB, device=dev, generator=g)).to(torch.bfloat16)
        tok = torch.randint(0, VOCAB, (B, N), device=dev, dtype=torch.int32, generator=g)
        par = _random_trees(B, N, dev)
        uni = torch.rand(B, N, device=dev, generator=g)
        mode = a11spec.GREEDY if a.mode == "greedy" else a11spec.STOCH_ONEHOT
        args = (mode, logits, tok, par)
        kw = dict(temperature=0.7, uniforms=uni)
        nbytes = logits.numel() * 2.0
    r = a11spec.accept(*args, **kw)
    us = _time(lambda: a11spec.accept(*args, **kw, out=r), a.warmup, a.iters)
    return {"case": "accept", "mode": a.mode, "batch": a.batch, "us": us, "bytes": nbytes,
            "gbps": nbytes / us / 1e3}


def case_compact(a) -> dict:
    """KV compaction of accepted paths (5 accepted nodes per sequence)."""
    dev = "cuda"
    B, N, HKV, D, ctx = a.batch, a.nodes, 4, 128, a.ctx
    kv = W.paged_kv(B, ctx, N, HKV, D, B * ((ctx + N + 15) // 16), seed=3, device=dev)
    nn = torch.full((B,), N, dtype=torch.int32, device=dev)
    alen = torch.full((B,), 5, dtype=torch.int32, device=dev)
    nodes = torch.full((B, N), -1, dtype=torch.int32, device=dev)
    nodes[:, :5] = torch.tensor([3, 9, 17, 30, 41], dtype=torch.int32, device=dev)
    pt0, cl0 = kv["page_table"].clone(), kv["ctx_lens"].clone()

    def run():
        kv["page_table"].copy_(pt0)
        kv["ctx_lens"].copy_(cl0)
        a11spec.kv_compact(kv["k_pool"], kv["v_pool"], kv["page_table"], kv["ctx_lens"], alen, nodes, nn)

    us = _time(run, a.warmup, a.iters)
    return {"case": "compact", "batch": B, "us": us, "bytes": 2.0 * 2 * B * 5 * HKV * D * 2}


def case_ngram(a) -> dict:
    """Trigram tree expansion from a 2^20-bucket table (C5 shape: top-4 / top-2, depth 5, 64 nodes)."""
    dev = "cuda"
    table = torch.from_numpy(W.make_ngram_table(log2_buckets=20, vocab=VOCAB, seed=1)).to(dev)
    g = torch.Generator(device=dev).manual_seed(6)
    last = torch.randint(0, VOCAB, (a.batch, 2), device=dev, dtype=torch.int32, generator=g)
    us = _time(lambda: a11spec.ngram_expand(table, last, 4, 2, 5, a.nodes), a.warmup, a.iters)
    return {"case": "ngram", "batch": a.batch, "us": us}


def case_pages(a) -> dict:
    """Page allocator per decode step: reserve the tree slots of every sequence
    (a11s_kv_reserve), then hand the tree's pages back (a11s_kv_release), as
    after a compaction that kept nothing. Each launch is timed with its own
    CUDA events; the torch ops that rebuild the freed lists sit between them."""
    dev = "cuda"
    B, MP = a.batch, (a.ctx + a.nodes + 15) // 16 + 1
    pool = a11spec.ops.KVPagePool(B * MP, dev)
    pt = torch.full((B, MP), -1, dtype=torch.int32, device=dev)
    sl = torch.zeros(B, dtype=torch.int32, device=dev)
    pool.reserve(pt, sl, torch.full((B,), a.ctx, dtype=torch.int32, device=dev), check_status=True)
    n_new = torch.full((B,), a.nodes, dtype=torch.int32, device=dev)
    freed = torch.full((B, MP), -1, dtype=torch.int32, device=dev)
    nfreed = torch.zeros(B, dtype=torch.int32, device=dev)
    p0 = (a.ctx + 15) // 16
    span = (a.ctx + a.nodes + 15) // 16 - p0
    ev = []

    def run(timed):
        e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        e[0].record()
        pool.reserve(pt, sl, n_new)  # tree slots
        e[1].record()
        sl.sub_(n_new)
        freed[:, :span] = pt[:, p0:p0 + span]
        pt[:, p0:p0 + span] = -1
        nfreed.fill_(span)
        e[2].record()
        pool.release(freed, nfreed)
        e[3].record()
        if timed:
            ev.append(e)

    for _ in range(a.warmup):
        run(False)
    for _ in range(a.iters):
        run(True)
    torch.cuda.synchronize()
    res = sum(x[0].elapsed_time(x[1]) for x in ev) * 1e3 / len(ev)
    rel = sum(x[2].elapsed_time(x[3]) for x in ev) * 1e3 / len(ev)
    return {"case": "pages", "batch": B, "ctx": a.ctx, "nodes": a.nodes, "reserve_us": res, "release_us": rel,
            "pages_per_step": B * span, "status": [int(x) for x in pool.status.tolist()]}


def case_ngram_update(a) -> dict:
    """n-gram learning after one step: the committed tokens of `batch`
    sequences (5 accepted + bonus each) into the C5 table (2^20 buckets)."""
    dev = "cuda"
    table = torch.from_numpy(W.make_ngram_table(log2_buckets=20, vocab=VOCAB, seed=1)).to(dev)
    g = torch.Generator(device=dev).manual_seed(7)
    B, N = a.batch, a.nodes
    last = torch.randint(0, VOCAB, (B, 2), device=dev, dtype=torch.int32, generator=g)
    acc = torch.randint(0, VOCAB, (B, N), device=dev, dtype=torch.int32, generator=g)
    alen = torch.full((B,), 5, dtype=torch.int32, device=dev)
    bonus = torch.randint(0, VOCAB, (B,), device=dev, dtype=torch.int32, generator=g)
    hist, lens = a11spec.history_from_accept(last, acc, alen, bonus)
    status = torch.zeros(2, dtype=torch.int32, device=dev)
    us = _time(lambda: a11spec.ngram_update(table, hist, lens, 20, status=status), a.warmup, a.iters)
    return {"case": "ngram_update", "batch": B, "us": us, "trigrams": int(status[1])}


def case_lm_head(a) -> dict:
    """The tree nodes' LM head: `batch` x `nodes` rows of hidden size `hidden`
    against a [vocab, hidden] output projection, with the chunk keys."""
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(6)
    R, H, V = a.batch * a.nodes, a.hidden, a.vocab
    h = torch.randn(R, H, device=dev, generator=g).to(torch.bfloat16)
    w = (torch.randn(V, H, device=dev, generator=g) / H ** 0.5).to(torch.bfloat16)
    out = torch.empty(R, V, dtype=torch.bfloat16, device=dev)
    keys = torch.empty(R, (V + 2047) // 2048, dtype=torch.int64, device=dev)
    ws = a11spec.ops.workspace(256, dev)
    us = _time(lambda: a11spec.lm_head(h, w, out=out, keys=keys, ws=ws), a.warmup, a.iters)
    flops = 2.0 * R * H * V
    return {"case": "lm_head", "rows": R, "hidden": H, "vocab": V, "us": us, "flops": flops,
            "tflops": flops / us / 1e6, "bytes": 2 * (R * H + V * H + R * V)}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("case", choices=["attention", "accept", "compact", "ngram", "pages", "ngram_update", "lm_head"])
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--nodes", type=int, default=64)
    ap.add_argument("--mode", choices=["greedy", "onehot", "draft", "c4greedy"], default="greedy")
    ap.add_argument("--hidden", type=int, default=2048)
    ap.add_argument("--vocab", type=int, default=VOCAB)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--iters", type=int, default=2)
    a = ap.parse_args(argv)
    torch.cuda.set_device(0)
    fn = {"attention": case_attention, "accept": case_accept, "compact": case_compact, "ngram": case_ngram,
          "pages": case_pages, "ngram_update": case_ngram_update, "lm_head": case_lm_head}[a.case]
    print(json.dumps(fn(a)), flush=True)


if __name__ == "__main__":
    main()
