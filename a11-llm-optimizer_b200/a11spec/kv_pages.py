"""Paged KV cache on the device with the block-table semantics of the
reference's PagedKVCacheManager (include/cuda/paged_kv_cache.hpp:20-67,
src/cuda/paged_kv_cache.cu:85-162): 16-token blocks, a free stack of physical
pages (LIFO), a block table per sequence, a new block when the token count
exceeds blocks * 16, blocks returned to the stack on free.

Unlike the reference (one cudaMalloc per block of num_layers*head_dim*16 fp32),
the pool is one tensor per K and V, [num_layers][pages][16][Hkv][D], so a
page id indexes every layer and the kernels see a page table of int32 ids.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch

from ._lib import PAGE_TOKENS

KV_CACHE_VRAM_GB = 8


@dataclass
class KVCacheConfig:
    """PagedKVCacheManager::Config (paged_kv_cache.hpp:22-27) plus the KV head count."""
    num_layers: int = 80
    head_dim: int = 128
    max_sequences: int = 64
    vram_cap_gb: float = KV_CACHE_VRAM_GB
    num_kv_heads: int = 1
    dtype: torch.dtype = torch.bfloat16


@dataclass
class _Seq:
    active: bool = False
    num_tokens: int = 0
    block_table: List[int] = field(default_factory=list)


class PagedKVCacheManager:
    def __init__(self, cfg: KVCacheConfig, device: str = "cuda", allocate_pool: bool = True):
        self.cfg = cfg
        esize = torch.tensor([], dtype=cfg.dtype).element_size()
        self._block_bytes = cfg.num_layers * cfg.num_kv_heads * cfg.head_dim * PAGE_TOKENS * esize
        cap = int(cfg.vram_cap_gb * (1 << 30))
        self.num_pages = max(0, cap // max(1, 2 * self._block_bytes))
        self._free: List[int] = list(range(self.num_pages))  # pop() takes the highest id first
        self._seqs: List[_Seq] = [_Seq() for _ in range(cfg.max_sequences)]
        self._used = 0
        self._tokens = 0
        self.k_pool = self.v_pool = None
        if allocate_pool and self.num_pages:
            shape = (cfg.num_layers, self.num_pages, PAGE_TOKENS, cfg.num_kv_heads, cfg.head_dim)
            self.k_pool = torch.zeros(shape, dtype=cfg.dtype, device=device)
            self.v_pool = torch.zeros(shape, dtype=cfg.dtype, device=device)

    # -- reference API -------------------------------------------------------
    def _alloc_block(self) -> int:
        if not self._free:
            raise RuntimeError("PagedKVCache: out of physical blocks")
        self._used += 1
        return self._free.pop()

    def _dealloc_block(self, idx: int) -> None:
        if 0 <= idx < self.num_pages:
            self._free.append(idx)
            self._used -= 1

    def allocate_sequence(self, seq_id: int) -> List[int]:
        if not 0 <= seq_id < len(self._seqs):
            raise RuntimeError("PagedKVCache: seq_id out of range")
        s = self._seqs[seq_id]
        if s.active:
            raise RuntimeError("PagedKVCache: sequence already allocated")
        blk = self._alloc_block()
        s.active, s.num_tokens, s.block_table = True, 0, [blk]
        return list(s.block_table)

    def append_token(self, seq_id: int) -> None:
        self.append_tokens(seq_id, 1)

    def append_tokens(self, seq_id: int, count: int) -> None:
        s = self._seqs[seq_id]
        if not s.active:
            raise RuntimeError("PagedKVCache: sequence not active")
        for _ in range(count):
            s.num_tokens += 1
            self._tokens += 1
            if s.num_tokens > len(s.block_table) * PAGE_TOKENS:
                s.block_table.append(self._alloc_block())

    def free_sequence(self, seq_id: int) -> None:
        if not 0 <= seq_id < len(self._seqs) or not self._seqs[seq_id].active:
            return
        s = self._seqs[seq_id]
        for blk in s.block_table:
            self._dealloc_block(blk)
        self._tokens -= s.num_tokens
        s.active, s.num_tokens, s.block_table = False, 0, []

    def get_block_table(self, seq_id: int) -> List[int]:
        s = self._seqs[seq_id]
        if not s.active:
            raise RuntimeError("PagedKVCache: sequence not active")
        return list(s.block_table)

    def free_stack(self) -> List[int]:
        """The free page ids, bottom of the stack first (the next pop is the last)."""
        return list(self._free)

    def used_blocks(self) -> int:
        return self._used

    def total_tokens(self) -> int:
        return self._tokens

    def vram_usage_bytes(self) -> int:
        return self._used * self._block_bytes * 2

    # -- speculative-step support -------------------------------------------
    def num_tokens(self, seq_id: int) -> int:
        return self._seqs[seq_id].num_tokens

    def reserve_tree(self, seq_id: int, n_nodes: int) -> int:
        """Grow the sequence by the tree slots (node i at position len + i);
        returns the context length before the tree."""
        L = self._seqs[seq_id].num_tokens
        self.append_tokens(seq_id, n_nodes)
        return L

    def page_table(self, seq_ids: List[int], max_pages: int, device) -> torch.Tensor:
        pt = torch.full((len(seq_ids), max_pages), -1, dtype=torch.int32)
        for r, sid in enumerate(seq_ids):
            bt = self._seqs[sid].block_table[:max_pages]
            pt[r, :len(bt)] = torch.tensor(bt, dtype=torch.int32)
        return pt.to(device)

    def commit_compaction(self, seq_ids: List[int], new_lens, freed_pages, n_freed) -> None:
        """Apply a11s_kv_compact's results: shorter sequences, pages back on the
        free stack in the order kv_compact lists them (the device allocator's
        a11s_kv_release order)."""
        new_lens = torch.as_tensor(new_lens).cpu().tolist()
        n_freed = torch.as_tensor(n_freed).cpu().tolist()
        freed_pages = torch.as_tensor(freed_pages).cpu()
        for r, sid in enumerate(seq_ids):
            s = self._seqs[sid]
            drop = freed_pages[r, : n_freed[r]].tolist()  # a11s_kv_compact lists them in table order
            if drop:
                gone = set(drop)
                s.block_table = [p for p in s.block_table if p not in gone]
                for p in drop:  # pushed in that order, like free_sequence's dealloc loop
                    self._dealloc_block(p)
            self._tokens += int(new_lens[r]) - s.num_tokens
            s.num_tokens = int(new_lens[r])
