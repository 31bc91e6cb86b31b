"""Speculative generation: the decode loop around the kernels.

The reference streams one token per target forward
(A11Pipeline.stream_inference, engine/pipeline.py:475-503: prefill, then
sample -> yield -> forward_token). ``speculative_stream`` is the same stream
with a drafted token tree per target forward:

    K1 draft a tree from the n-gram table (root = the last committed token)
    K5 reserve pages for the tree's slots          (positions ctx_len + i)
       model.forward_tree: the target writes the tree's K/V there, runs
       a11s_tree_attention and returns logits [B, N, V]
    K3 accept (greedy or one-hot sampling) -> accepted path + bonus token
    K4 compact the accepted path's K/V; K5 release the detached pages
    K6 the n-gram table learns the committed tokens
       yield the committed tokens (accepted path + bonus) of every sequence

Greedy acceptance commits exactly the target's own greedy tokens, so the
stream equals non-speculative greedy decoding, only with more tokens per
target forward.

The target model is any object with:

* ``vocab`` (int), ``k_pool`` / ``v_pool`` (bf16 [pages, 16, Hkv, D], or
  [num_layers, pages, 16, Hkv, D] with a ``num_layers`` attribute: the paged KV
  cache the model's attention reads, one slab per layer);
* ``prefill(tokens, page_table, ctx_lens)``: write the K/V of tokens
  [B, T] at positions 0 .. T-1 (ctx_lens is 0 on entry; the caller sets it);
* ``forward_tree(tokens, parents, n_nodes, page_table, ctx_lens)`` ->
  logits [B, N, V] (bf16 or fp32): node i's row judges its children.
"""
from __future__ import annotations

from typing import Iterator, List, Optional

import torch

from . import _lib, ops
from .decoder import SpeculativeDecoder


def speculative_stream(model, prompts: torch.Tensor, max_new_tokens: int, decoder: SpeculativeDecoder,
                       pages: ops.KVPagePool, max_pages: int, learn: bool = True,
                       uniforms_fn=None) -> Iterator[List[List[int]]]:
    """Yield, per target forward, the committed tokens of every sequence
    (a list per sequence, empty once it has max_new_tokens). prompts: int32
    [B, T], T >= 2, on the model's device. Page tables and lengths live on
    the device; the loop reads
    back only the committed tokens it yields. The decoder's temperature
    decides the rule: None = greedy, else one-hot sampling at that temperature
    (uniforms from `uniforms_fn(B, N)` or the decoder's own generator)."""
    dev = prompts.device
    B, T = prompts.shape
    if T < 2:
        raise ValueError("prompts need at least two tokens (the n-gram key of the first tree)")
    N = decoder.max_nodes
    page_table = torch.full((B, max_pages), -1, dtype=torch.int32, device=dev)
    ctx_lens = torch.zeros(B, dtype=torch.int32, device=dev)
    # the prompt's last token is the first tree's root: prefill the others
    pages.reserve(page_table, ctx_lens, torch.full((B,), T - 1, dtype=torch.int32, device=dev), check_status=True)
    model.prefill(prompts[:, :T - 1].contiguous(), page_table, ctx_lens)
    last = prompts[:, T - 2:].contiguous().to(torch.int32)
    grown = torch.empty_like(ctx_lens)
    hist_buf = (torch.empty(B, N + 3, dtype=torch.int32, device=dev), torch.empty(B, dtype=torch.int32, device=dev))
    status = torch.zeros(2, dtype=torch.int32, device=dev)
    produced = [0] * B
    while min(produced) < max_new_tokens:
        tree = decoder.draft(last)
        grown.copy_(ctx_lens)
        pages.reserve(page_table, grown, tree.n_nodes)
        logits = model.forward_tree(tree.tokens, tree.parents, tree.n_nodes, page_table, ctx_lens)
        uni = uniforms_fn(B, N) if (uniforms_fn is not None and decoder.temperature is not None) else None
        # draws its own uniforms when sampling without them; takes its records from
        # the LM head's chunk keys when the model's head left them
        res = decoder.verify(tree, logits, uniforms=uni, keys=getattr(model, "last_chunk_keys", None))
        freed, n_freed = ops.kv_compact(model.k_pool, model.v_pool, page_table, ctx_lens, res.accept_len,
                                        res.accepted_nodes, tree.n_nodes,
                                        num_layers=getattr(model, "num_layers", 1))
        pages.release(freed, n_freed)
        # next root pair (last accepted token, or the old root; bonus) and, when
        # learning, the committed-token rows built from the old pair: one launch
        ops.next_roots(tree.tokens, res.accepted_tokens, res.accept_len, res.bonus, last,
                       history=hist_buf if learn else None)
        if learn:
            ops.ngram_update(decoder.table, hist_buf[0], hist_buf[1], decoder.log2_buckets, status=status)
        alen = res.accept_len.cpu().tolist()
        toks = res.accepted_tokens.cpu().tolist()
        bonus = res.bonus.cpu().tolist()
        out: List[List[int]] = []
        for b in range(B):
            new = toks[b][:alen[b]] + ([bonus[b]] if bonus[b] >= 0 else [])
            new = new[: max(0, max_new_tokens - produced[b])]
            produced[b] += len(new)
            out.append(new)
        code = int(pages.status[0])
        if code != _lib.OK:
            raise _lib.A11Error(code, f"page allocator status {code} (detail {int(pages.status[1])})")
        yield out
