"""SpeculativeDecoder with the interface of the reference's engine/speculative.py:4-34,
plus the batched tree step the B200 kernels implement.

List-based methods (``generate_draft_tokens``, ``verify_candidates``) keep the
reference signatures: they build one-sequence device tensors, run the kernels
and synchronise to return Python lists. The batched API (``draft``,
``verify``, ``step``) stays on the device and never synchronises.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List, Optional

import numpy as np
import torch

from . import _lib, ops


@dataclass
class DraftTree:
    tokens: torch.Tensor   # int32 [B, N]
    parents: torch.Tensor  # int32 [B, N]
    depths: torch.Tensor   # int32 [B, N]
    n_nodes: torch.Tensor  # int32 [B]


class SpeculativeDecoder:
    """Draft-and-verify engine over a hashed trigram table.

    draft_k      drafts returned by generate_draft_tokens (reference default 3)
    table        int32 [2^k, slots, 2] (token, count) continuation table; an
                 empty table drafts nothing
    width_root / width_inner / max_depth / max_nodes
                 tree shape of draft() (top-4 at depth 1, top-2 below, depth <= 5,
                 <= 64 nodes by default)
    temperature  None = greedy verification; otherwise sampling acceptance at T
    """

    def __init__(self, draft_k: int = 3, table: Optional[torch.Tensor] = None, log2_buckets: int = 20,
                 width_root: int = 4, width_inner: int = 2, max_depth: int = 5, max_nodes: int = 64,
                 temperature: Optional[float] = None, device: str = "cuda", seed: int = 0):
        self.draft_k = draft_k
        self.device = torch.device(device)
        if table is None:
            table = torch.zeros((1 << log2_buckets, 8, 2), dtype=torch.int32)
        self.table = table.to(self.device, torch.int32).contiguous()
        self.log2_buckets = log2_buckets
        self.width_root, self.width_inner = width_root, width_inner
        self.max_depth, self.max_nodes = max_depth, max_nodes
        self.temperature = temperature
        self.stats = torch.zeros(_lib.STATS_LEN, dtype=torch.int64, device=self.device)
        self._gen = torch.Generator(device=self.device).manual_seed(seed)

    # -- reference interface (engine/speculative.py) --------------------------
    def generate_draft_tokens(self, context_tokens: List[int]) -> List[int]:
        """Greedy chain of up to draft_k drafts: at every depth the most frequent
        continuation of the last two tokens (engine/speculative.py:21 key)."""
        ctx = list(context_tokens)
        if not ctx:
            ctx = [0]
        if len(ctx) < 2:
            ctx = [0] + ctx  # a missing older token hashes as token 0
        last = torch.tensor([[ctx[-2], ctx[-1]]], dtype=torch.int32, device=self.device)
        tk, _, _, nn = ops.ngram_expand(self.table, last, 1, 1, self.draft_k, self.draft_k + 1)
        n = int(nn.item())
        return tk[0, 1:n].cpu().tolist()

    def verify_candidates(self, target_logits: torch.Tensor, draft_tokens: List[int]) -> List[int]:
        """Accepted prefix of draft_tokens. target_logits [k or k+1, V]: row i is
        the target distribution that judges draft i (row k, when present, the
        bonus distribution)."""
        k = len(draft_tokens)
        if k == 0:
            return []
        V = target_logits.shape[-1]
        rows = target_logits.reshape(-1, V).to(self.device)
        if rows.shape[0] not in (k, k + 1):
            raise ValueError("target_logits must have len(draft_tokens) or len+1 rows")
        if rows.shape[0] == k:
            rows = torch.cat([rows, rows[-1:]], dim=0)
        if rows.dtype not in (torch.float32, torch.bfloat16):
            rows = rows.float()
        if V % 8:
            pad = 8 - V % 8
            rows = torch.nn.functional.pad(rows, (0, pad), value=float("-inf"))
        tree = self._chain(draft_tokens)
        res = self.verify(tree, rows.unsqueeze(0).contiguous())
        n = int(res.accept_len.item())
        return res.accepted_tokens[0, :n].cpu().tolist()

    # -- batched device API ---------------------------------------------------
    def _chain(self, draft_tokens: List[int]) -> DraftTree:
        k = len(draft_tokens)
        toks = torch.tensor([[0] + list(draft_tokens)], dtype=torch.int32, device=self.device)
        par = torch.arange(-1, k, dtype=torch.int32, device=self.device).unsqueeze(0)
        dep = torch.arange(0, k + 1, dtype=torch.int32, device=self.device).unsqueeze(0)
        nn = torch.tensor([k + 1], dtype=torch.int32, device=self.device)
        return DraftTree(toks, par, dep, nn)

    def draft(self, last_tokens: torch.Tensor, out: Optional[DraftTree] = None) -> DraftTree:
        """K1: trees from the two newest tokens of each sequence ([B, 2] int32)."""
        o = None if out is None else (out.tokens, out.parents, out.depths, out.n_nodes)
        tk, pa, de, nn = ops.ngram_expand(self.table, last_tokens, self.width_root, self.width_inner,
                                          self.max_depth, self.max_nodes, out=o)
        return DraftTree(tk, pa, de, nn)

    def verify(self, tree: DraftTree, target_logits: torch.Tensor, uniforms: Optional[torch.Tensor] = None,
               draft_logits: Optional[torch.Tensor] = None, out: Optional[ops.AcceptResult] = None,
               keys: Optional[torch.Tensor] = None):
        """K3 on [B, N, V] logits (row i judges node i's children). keys: the
        chunk keys a11s_lm_head wrote with these bf16 logits; the acceptance
        then takes its records from them (not with draft logits)."""
        if self.temperature is None:
            mode = _lib.GREEDY
        else:
            mode = _lib.STOCH_DRAFT if draft_logits is not None else _lib.STOCH_ONEHOT
            if uniforms is None:
                B, N = tree.tokens.shape
                uniforms = torch.rand(B, N, generator=self._gen, device=self.device)
        if draft_logits is not None or target_logits.dtype != torch.bfloat16:
            keys = None
        return ops.accept(mode, target_logits, tree.tokens, tree.parents, tree.n_nodes,
                          draft_logits=draft_logits, temperature=self.temperature or 1.0,
                          uniforms=uniforms, stats=self.stats, out=out, keys=keys)

    def step(self, last_tokens: torch.Tensor, q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
             page_table: torch.Tensor, seq_lens: torch.Tensor,
             logits_fn: Callable[[torch.Tensor, DraftTree], torch.Tensor],
             uniforms: Optional[torch.Tensor] = None, pages: Optional["ops.KVPagePool"] = None,
             kv_fn: Optional[Callable[[DraftTree, torch.Tensor, torch.Tensor], None]] = None):
        """One speculative step on the device: draft (K1), tree attention (K2),
        logits_fn(attention_out, tree) -> [B, N, V] (the target model's
        remaining layers and LM head), acceptance (K3), compaction (K4).

        Without `pages` the caller has already given the tree slots (positions
        seq_lens + i) their pages. With a KVPagePool the step reserves exactly
        the drafted tree's slots after drafting (K5) and returns the pages
        compaction detaches, so page tables, lengths and the free stack stay
        on the device. `kv_fn(tree, page_table, seq_lens)`, when given, runs
        between the reservation and the attention: the target model writes the
        tree's K/V there. Returns (tree, acceptance result); seq_lens and
        page_table are updated."""
        tree = self.draft(last_tokens)
        if pages is not None:
            grown = seq_lens.clone()
            pages.reserve(page_table, grown, tree.n_nodes)
        if kv_fn is not None:
            kv_fn(tree, page_table, seq_lens)
        attn, _, _ = ops.tree_attention(q, k_pool, v_pool, page_table, seq_lens, tree.parents, tree.n_nodes)
        logits = logits_fn(attn, tree)
        res = self.verify(tree, logits, uniforms=uniforms)
        freed, n_freed = ops.kv_compact(k_pool, v_pool, page_table, seq_lens, res.accept_len, res.accepted_nodes,
                                        tree.n_nodes)
        if pages is not None:
            pages.release(freed, n_freed)
        return tree, res

    def diagnostics(self) -> dict:
        return dict(zip(_lib.STAT_NAMES, self.stats.cpu().tolist()))
