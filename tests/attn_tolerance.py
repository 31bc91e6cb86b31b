"""Element-wise tolerance of the tree-attention checks (test helper).

Bar: |got - ref| <= 2e-2 * |ref| + floor_row for every output element, where
ref is the checker's output (the oracle, the reference's own decode attention,
or the torch fp32 restatement below) and floor_row is an absolute term of the
row (sequence b, node i, query head h) derived from the one rounding both
sides make on purpose: the attention probabilities are cast to bf16 before the
PV product (engine/pipeline.py:401 of the reference; the kernel rounds its
unnormalised probabilities the same way). Each cast has relative error at most
2^-9, independently on the two sides, so the outputs differ by
sum_s p_s (d_s - d'_s) v_s, whose standard deviation is at most
2^-9 * sqrt(2/3) * ||p_row||_2 * rms(v) (uniform rounding errors, independent
terms). floor_row is 8 * 2^-9 * ||p_row||_2 * rms(v), about 10 standard
deviations, with rms(v) taken over the sequence's keys of the row's KV head.
The relative 2e-2 term covers the bf16 rounding of the outputs themselves
(2^-9) with room to spare. A row whose softmax concentrates on one key has
||p||_2 near 1 and a floor near 1.6e-2 * rms(v); a row spread over 32k keys has
||p||_2 near 1/sqrt(32k) and a floor about 180 times smaller, so errors that a
bound relative to the largest output would hide stay visible.
"""
from __future__ import annotations

import math

import numpy as np
import torch

REL = 2e-2
FLOOR_SIGMAS = 8.0


def _ancestors(parents_row, n):
    allowed = torch.zeros(n, n, dtype=torch.bool)
    for i in range(n):
        a = i
        while a >= 0:
            allowed[i, a] = True
            a = int(parents_row[a]) if a > 0 else -1
    return allowed


def reference(q, k_pool, v_pool, page_table, ctx_lens, parents, n_nodes=None, scale=None, device=None):
    """torch fp32 restatement of the reference's decode attention over a token
    tree: scores q.k * scale in fp32 (query head h reads KV head h // (Hq/Hkv)),
    softmax over the context and the node's ancestors (itself included),
    probabilities cast to bf16, then PV in fp32. Returns (out [B,N,Hq,D] fp32,
    floor [B,N,Hq] fp32); rows of dead nodes are zero with a zero floor."""
    dev = device or q.device
    q, k_pool, v_pool = (torch.as_tensor(x).to(dev) for x in (q, k_pool, v_pool))
    page_table, ctx_lens, parents = (torch.as_tensor(np.asarray(x.cpu() if torch.is_tensor(x) else x))
                                     for x in (page_table, ctx_lens, parents))
    B, N, Hq, D = q.shape
    Hkv = k_pool.shape[2]
    rep = Hq // Hkv
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    nn = [N] * B if n_nodes is None else [int(x) for x in torch.as_tensor(np.asarray(
        n_nodes.cpu() if torch.is_tensor(n_nodes) else n_nodes))]
    out = torch.zeros(B, N, Hq, D, dtype=torch.float32, device=dev)
    floor = torch.zeros(B, N, Hq, dtype=torch.float32, device=dev)
    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for b in range(B):
            n, L = nn[b], int(ctx_lens[b])
            if n == 0:
                continue
            pos = torch.arange(L + n)
            pages = page_table[b, pos // 16].long()
            k = k_pool[pages.to(dev), (pos % 16).to(dev)].float()  # [S, Hkv, D]
            v = v_pool[pages.to(dev), (pos % 16).to(dev)].float()
            allowed = torch.ones(n, L + n, dtype=torch.bool)
            allowed[:, L:] = _ancestors(parents[b], n)
            allowed = allowed.to(dev)
            for h in range(Hkv):
                qh = q[b, :n, h * rep:(h + 1) * rep].float().reshape(n * rep, D)
                s = (qh @ k[:, h].T).mul_(scale).view(n, rep, L + n)
                s.masked_fill_(~allowed[:, None, :], float("-inf"))
                p = torch.softmax(s, dim=-1)
                rms_v = v[:, h].square().mean().sqrt()
                floor[b, :n, h * rep:(h + 1) * rep] = FLOOR_SIGMAS * 2.0 ** -9 * p.square().sum(-1).sqrt() * rms_v
                pb = p.to(torch.bfloat16).float().view(n * rep, L + n)
                out[b, :n, h * rep:(h + 1) * rep] = (pb @ v[:, h]).view(n, rep, D)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = tf32
    return out, floor


def worst(got, ref, floor):
    """(worst ratio |got-ref| / (REL*|ref| + floor) over all elements, index of
    its row (b, i, h)). A check passes when the ratio is <= 1."""
    got = torch.as_tensor(got).float()
    ref = torch.as_tensor(ref).float().to(got.device)
    floor = torch.as_tensor(floor).float().to(got.device)
    bound = REL * ref.abs() + floor[..., None]
    ratio = ((got - ref).abs() / bound.clamp_min(1e-30)).amax(dim=-1)  # per row
    idx = int(torch.argmax(ratio))
    return float(ratio.flatten()[idx]), tuple(int(x) for x in np.unravel_index(idx, tuple(ratio.shape)))


def assert_close(got, ref, floor, what=""):
    r, row = worst(got, ref, floor)
    assert r <= 1.0, f"{what}: worst row {row} at {r:.3f} of the bound (2e-2 |ref| + floor)"
    return r
