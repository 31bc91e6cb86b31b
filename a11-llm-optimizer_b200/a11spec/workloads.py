"""Seeded synthetic workloads with the shapes and distributions of the five
benchmark configurations of the speculative path (no dataset exists for it).

C1  greedy chain, B=1, 5 drafts, fp32 logits [6, 32000] ~ N(0, 3^2)
C2  greedy complete binary tree (31 nodes), B=8, bf16 logits ~ N(0, 2^2), V=151936
C3  sampling acceptance T=0.8, B=64, 63-node tree (branching 4/3/2/2/1, BFS),
    draft q ~ N(0,1), target p = q + N(0, 0.5^2), fp32, V=151936, Philox uniforms
C4  tree attention (ctx 4096, 64-node random tree, GQA 32/4, d=128, 16-token
    pages from a permuted 16384-page pool) + greedy acceptance + compaction, B=32
C5  end to end per GPU: hashed trigram table (2^20 x 8, Zipf(1.2) counts) ->
    tree (4 at depth 1, 2 below, depth <= 5, <= 64 nodes) -> attention over
    ctx 32768 -> LM head [nodes, 2048] x [2048, 151936] -> sampling T=0.7 ->
    compaction, B=32 per GPU

Every size can be shrunk for tests. Small configurations use numpy (platform
independent PCG64 / Philox streams); large ones are drawn on the target device
with a seeded torch generator.
"""
from __future__ import annotations

import math
from typing import Dict, Optional, Sequence

import numpy as np
import torch

VOCAB = 151936


# ----------------------------------------------------------------------------- trees
def chain_parents(n: int) -> np.ndarray:
    return np.arange(-1, n - 1, dtype=np.int32)


def binary_parents(n: int) -> np.ndarray:
    p = (np.arange(n, dtype=np.int32) - 1) // 2
    p[0] = -1
    return p


def schedule_parents(branching: Sequence[int], n: int) -> np.ndarray:
    """Breadth-first tree where every node at depth d gets branching[d] children,
    truncated at n nodes (root included)."""
    parents = [-1]
    depth = [0]
    i = 0
    while len(parents) < n and i < len(parents):
        d = depth[i]
        if d < len(branching):
            for _ in range(branching[d]):
                if len(parents) >= n:
                    break
                parents.append(i)
                depth.append(d + 1)
        i += 1
    return np.asarray(parents, dtype=np.int32)


def random_parents(n: int, rng: np.random.Generator) -> np.ndarray:
    p = np.full(n, -1, dtype=np.int32)
    for i in range(1, n):
        p[i] = rng.integers(0, i)
    return p


# ----------------------------------------------------------------------------- C1
def make_c1(seed: int = 1, vocab: int = 32000, n_draft: int = 5, p_match: float = 0.7) -> Dict:
    """Greedy chain: row i-1 argmax equals draft token i with probability p_match."""
    rng = np.random.Generator(np.random.PCG64(seed))
    n = n_draft + 1
    logits = rng.normal(0.0, 3.0, size=(1, n, vocab)).astype(np.float32)
    tokens = np.zeros((1, n), np.int32)
    tokens[0, 0] = rng.integers(0, vocab)
    for i in range(1, n):
        row = logits[0, i - 1]
        if rng.random() < p_match:
            x = int(rng.integers(0, vocab))
            row[x] += 10.0
            if int(np.argmax(row)) != x:
                row[x] = row.max() + 1.0
        else:
            am = int(np.argmax(row))
            x = int(rng.integers(0, vocab - 1))
            x = x + 1 if x >= am else x
        tokens[0, i] = x
    return dict(logits=logits, tokens=tokens, parents=chain_parents(n)[None, :].copy(),
                n_nodes=np.array([n], np.int32))


# ----------------------------------------------------------------------------- C2
def make_c2(seed: int = 2, batch: int = 8, vocab: int = VOCAB, n_nodes: int = 31,
            p_force: float = 0.6) -> Dict:
    rng = np.random.Generator(np.random.PCG64(seed))
    logits = rng.normal(0.0, 2.0, size=(batch, n_nodes, vocab)).astype(np.float32)
    tokens = rng.integers(0, vocab, size=(batch, n_nodes)).astype(np.int32)
    parents = np.tile(binary_parents(n_nodes), (batch, 1))
    for b in range(batch):
        for i in range(1, n_nodes):
            if rng.random() < p_force:
                row = logits[b, parents[b, i]]
                row[tokens[b, i]] = row.max() + 8.0
    bf = torch.from_numpy(logits).to(torch.bfloat16)
    return dict(logits_bf16=bf, logits=bf.float().numpy(), tokens=tokens, parents=parents,
                n_nodes=np.full(batch, n_nodes, np.int32))


# ----------------------------------------------------------------------------- C3
C3_BRANCHING = (4, 3, 2, 2, 1)


def make_c3(seed: int = 3, batch: int = 64, vocab: int = VOCAB, n_nodes: int = 64,
            temperature: float = 0.8, device: Optional[str] = None) -> Dict:
    """Sampling acceptance. Returns torch tensors on `device` (numpy on host when
    device is None)."""
    parents = schedule_parents(C3_BRANCHING, n_nodes)
    n = len(parents)
    if device is None:
        rng = np.random.Generator(np.random.PCG64(seed))
        q = rng.normal(0.0, 1.0, size=(batch, n, vocab)).astype(np.float32)
        p = (q + rng.normal(0.0, 0.5, size=q.shape)).astype(np.float32)
        tokens = np.zeros((batch, n), np.int32)
        tokens[:, 0] = rng.integers(0, vocab, size=batch)
        for b in range(batch):
            for i in range(1, n):
                z = q[b, parents[i]].astype(np.float64) / temperature
                pr = np.exp(z - z.max())
                pr /= pr.sum()
                tokens[b, i] = rng.choice(vocab, p=pr)
        uni = np.random.Generator(np.random.Philox(seed)).random((batch, n), dtype=np.float32)
        return dict(p=p, q=q, tokens=tokens, parents=np.tile(parents, (batch, 1)),
                    n_nodes=np.full(batch, n, np.int32), uniforms=uni, temperature=temperature)
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(batch, n, vocab, generator=g, device=device)
    p = q + 0.5 * torch.randn(batch, n, vocab, generator=g, device=device)
    par_t = torch.as_tensor(parents, device=device).long()
    tokens = torch.empty(batch, n, dtype=torch.int32, device=device)
    tokens[:, 0] = torch.randint(0, vocab, (batch,), generator=g, device=device, dtype=torch.int32)
    probs = torch.softmax(q[:, par_t[1:]] / temperature, dim=-1)  # [B, n-1, V]
    tokens[:, 1:] = torch.multinomial(probs.reshape(-1, vocab), 1, generator=g).view(batch, n - 1).int()
    del probs
    uni = torch.rand(batch, n, generator=g, device=device)
    return dict(p=p, q=q, tokens=tokens, parents=par_t.int().repeat(batch, 1).contiguous(),
                n_nodes=torch.full((batch,), n, dtype=torch.int32, device=device), uniforms=uni,
                temperature=temperature)


# ----------------------------------------------------------------------------- paged KV
def paged_kv(batch: int, ctx: int, n_nodes: int, num_kv_heads: int, head_dim: int,
             pool_pages: int, seed: int, device: str, dtype=torch.bfloat16,
             spare_pages: int = 0) -> Dict:
    """KV pool [pool_pages, 16, Hkv, D] ~ N(0,1) and page tables drawn from a
    seeded permutation of the pool (each sequence owns ceil((ctx + n)/16) pages,
    plus `spare_pages` extra logical entries)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    per = (ctx + n_nodes + 15) // 16
    need = batch * per
    if need > pool_pages:
        raise ValueError(f"pool of {pool_pages} pages cannot hold {need}")
    perm = torch.randperm(pool_pages, generator=g)[:need].view(batch, per).int()
    table = torch.full((batch, per + spare_pages), -1, dtype=torch.int32)
    table[:, :per] = perm
    gd = torch.Generator(device=device).manual_seed(seed + 1)
    shape = (pool_pages, 16, num_kv_heads, head_dim)
    k = torch.randn(shape, generator=gd, device=device, dtype=torch.float32).to(dtype)
    v = torch.randn(shape, generator=gd, device=device, dtype=torch.float32).to(dtype)
    return dict(k_pool=k, v_pool=v, page_table=table.to(device),
                ctx_lens=torch.full((batch,), ctx, dtype=torch.int32, device=device))


# ----------------------------------------------------------------------------- C4
def make_c4(seed: int = 4, batch: int = 32, ctx: int = 4096, n_nodes: int = 64,
            num_q_heads: int = 32, num_kv_heads: int = 4, head_dim: int = 128,
            pool_pages: int = 16384, vocab: int = VOCAB, device: str = "cuda",
            p_force: float = 0.5) -> Dict:
    rng = np.random.Generator(np.random.PCG64(seed))
    parents = np.stack([random_parents(n_nodes, rng) for _ in range(batch)])
    tokens = rng.integers(0, vocab, size=(batch, n_nodes)).astype(np.int32)
    kv = paged_kv(batch, ctx, n_nodes, num_kv_heads, head_dim, pool_pages, seed, device)
    g = torch.Generator(device=device).manual_seed(seed + 2)
    q = torch.randn(batch, n_nodes, num_q_heads, head_dim, generator=g, device=device).to(torch.bfloat16)
    logits = 2.0 * torch.randn(batch, n_nodes, vocab, generator=g, device=device)
    force = rng.random((batch, n_nodes)) < p_force
    bi, ii = np.nonzero(force[:, 1:])
    ii = ii + 1
    if len(bi):
        rows_b = torch.as_tensor(bi, device=device).long()
        rows_n = torch.as_tensor(parents[bi, ii], device=device).long()
        toks = torch.as_tensor(tokens[bi, ii], device=device).long()
        rmax = logits[rows_b, rows_n].amax(dim=-1)
        logits[rows_b, rows_n, toks] = rmax + 8.0
    return dict(q=q, **kv, parents=torch.as_tensor(parents, device=device),
                tokens=torch.as_tensor(tokens, device=device),
                n_nodes=torch.full((batch,), n_nodes, dtype=torch.int32, device=device),
                logits=logits.to(torch.bfloat16))


# ----------------------------------------------------------------------------- C5
def make_ngram_table(log2_buckets: int = 20, slots: int = 8, vocab: int = VOCAB, zipf_a: float = 1.2,
                     seed: int = 5) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed))
    nb = 1 << log2_buckets
    table = np.empty((nb, slots, 2), np.int32)
    table[:, :, 0] = rng.integers(0, vocab, size=(nb, slots))
    table[:, :, 1] = np.minimum(rng.zipf(zipf_a, size=(nb, slots)), 2**31 - 1)
    return table


def make_c5(seed: int = 5, batch: int = 32, ctx: int = 32768, max_nodes: int = 64,
            num_q_heads: int = 32, num_kv_heads: int = 4, head_dim: int = 128,
            hidden: int = 2048, vocab: int = VOCAB, log2_buckets: int = 20,
            device: str = "cuda", temperature: float = 0.7, spare_pages: int = 0) -> Dict:
    """spare_pages: extra logical table entries per sequence and as many extra
    physical pages per sequence in the pool (room for a growing context)."""
    table = torch.from_numpy(make_ngram_table(log2_buckets, 8, vocab, 1.2, seed)).to(device)
    pool_pages = batch * ((ctx + max_nodes + 15) // 16 + spare_pages)
    kv = paged_kv(batch, ctx, max_nodes, num_kv_heads, head_dim, pool_pages, seed, device,
                  spare_pages=spare_pages)
    g = torch.Generator(device=device).manual_seed(seed + 3)
    q = torch.randn(batch, max_nodes, num_q_heads, head_dim, generator=g, device=device).to(torch.bfloat16)
    h = torch.randn(batch * max_nodes, hidden, generator=g, device=device).to(torch.bfloat16)
    w = (0.02 * torch.randn(hidden, vocab, generator=g, device=device)).to(torch.bfloat16)
    rng = np.random.Generator(np.random.PCG64(seed + 4))
    last = torch.from_numpy(rng.integers(0, vocab, size=(batch, 2)).astype(np.int32)).to(device)
    return dict(table=table, log2_buckets=log2_buckets, q=q, hidden=h, w=w, last_tokens=last,
                temperature=temperature, vocab=vocab, **kv)
