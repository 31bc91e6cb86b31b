"""A target model whose forward pass runs over a draft tree: the decoder of the
reference's A11Pipeline (forward_token and forward_layer, engine/pipeline.py:
350-473, dense SwiGLU FFN branch) restated for token trees on the paged KV
pools, so that ``generate.speculative_stream`` can drive a real decoder stack.

Per layer, for every tree node at once, the same statements as forward_layer
in the reference's compute dtype (bf16):
  h_norm = rms_norm(h, attn_norm)                  pipeline.py:356-360, 322-324
  q, k, v = h_norm W_q^T, h_norm W_k^T, h_norm W_v^T (+ biases)   :364-373
  optional q/k head norms                          :375-381
  q, k = rotary(q, k, position)                    :384, 332-341
  K/V of the nodes -> the layer's page pool        (the reference appends to its
                                                    KV cache, :388)
  attn = tree attention (a11s_tree_attention)      :391-402 (GQA, fp32 scores,
                                                    softmax, bf16 probabilities)
  h += attn W_o^T                                  :403-405
  h += down(silu(gate(rms_norm(h))) * up(...))     :407-447
and logits = rms_norm(h, output_norm) W_out^T (:469-473).

What changes for a tree: node i of a tree whose root sits at position ctx
(the last committed token) has rotary position ctx + depth(i), the position
it takes in the sequence if accepted; its K/V go to the tree slot ctx + i of
the page table (where a11s_kv_compact expects them); its attention sees the
context and its own ancestors. A one-node tree is the reference's single-token
decode step; the prompt is prefilled as chain trees of up to 64 tokens.

Weights use the reference's GGUF tensor names (token_embd.weight,
blk.{i}.attn_q.weight, ..., output.weight), as its WeightStore serves them.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional

import torch
import torch.nn.functional as F

from . import ops

PAGE_TOKENS = 16


@dataclass
class DecoderConfig:
    """The fields of the reference's ModelConfig that forward_layer reads."""
    n_layers: int
    n_embd: int
    n_head: int
    n_head_kv: int
    head_dim: int
    n_ff: int
    vocab: int
    rms_eps: float = 1e-6
    rope_base: float = 10000.0


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """A11Pipeline._rms_norm (engine/pipeline.py:322-324), in x's dtype."""
    variance = x.pow(2).mean(-1, keepdim=True)
    return x * torch.rsqrt(variance + eps) * w


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def rotary(q: torch.Tensor, k: torch.Tensor, pos: torch.Tensor, base: float):
    """A11Pipeline._apply_rotary_emb (engine/pipeline.py:332-341) at a position
    per token: pos int [..., T], q/k [..., T, heads, D]. The angles are fp32,
    so the results are fp32 (bf16 x fp32 promotes), as in the reference."""
    dim = q.shape[-1]
    inv_freq = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float32, device=q.device) / dim))
    freqs = pos.to(torch.float32).unsqueeze(-1) * inv_freq  # [..., T, D/2]
    emb = torch.cat((freqs, freqs), dim=-1)
    cos, sin = emb.cos().unsqueeze(-2), emb.sin().unsqueeze(-2)
    return q * cos + rotate_half(q) * sin, k * cos + rotate_half(k) * sin


def tree_depths(parents: torch.Tensor, n_nodes: torch.Tensor) -> torch.Tensor:
    """Depth of every node (root 0) of trees [B, N] with parents[i] < i."""
    B, N = parents.shape
    depth = torch.zeros(B, N, dtype=torch.int64, device=parents.device)
    par = parents.long().clamp_min(0)
    for i in range(1, N):  # parents[i] < i: one pass in index order
        depth[:, i] = depth.gather(1, par[:, i:i + 1]).squeeze(1) + 1
    live = torch.arange(N, device=parents.device).unsqueeze(0) < n_nodes.unsqueeze(1)
    return torch.where(live, depth, torch.zeros_like(depth))


class TreeDecoder:
    """Decoder stack over token trees (see the module docstring).

    tensors: name -> tensor with the reference's GGUF names; converted to the
    compute dtype on `device`. The K/V pools are [n_layers, num_pages, 16,
    n_head_kv, head_dim] bf16, the layout a11s_kv_compact moves (num_layers
    slabs) and a11s_tree_attention reads one layer of."""

    def __init__(self, tensors: Dict[str, torch.Tensor], cfg: DecoderConfig, num_pages: int, device="cuda",
                 compute_dtype: torch.dtype = torch.bfloat16):
        if cfg.n_head % cfg.n_head_kv:
            raise ValueError("n_head must be a multiple of n_head_kv")
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = compute_dtype
        self.w = {k: v.to(self.device, compute_dtype).contiguous() for k, v in tensors.items()}
        self.num_layers = cfg.n_layers
        self.vocab = cfg.vocab
        shape = (cfg.n_layers, num_pages, PAGE_TOKENS, cfg.n_head_kv, cfg.head_dim)
        self.k_pool = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        self.v_pool = torch.zeros_like(self.k_pool)
        self.forwards = 0
        self.last_chunk_keys = None  # chunk keys of the last forward's logits (K7), or None

    def _proj(self, x: torch.Tensor, name: str) -> torch.Tensor:
        y = torch.matmul(x, self.w[name + ".weight"].t())
        b = self.w.get(name + ".bias")
        return y + b if b is not None else y

    def _write_kv(self, layer: int, k, v, slots, page_table, live):
        """K/V of the live tokens into the layer's pool at logical slots [B, N]."""
        b, i = torch.nonzero(live, as_tuple=True)
        s = slots[b, i]
        page = page_table[b, s // PAGE_TOKENS].long()
        off = s % PAGE_TOKENS
        self.k_pool[layer, page, off] = k[b, i].to(torch.bfloat16)
        self.v_pool[layer, page, off] = v[b, i].to(torch.bfloat16)

    def _forward(self, tokens, parents, n_nodes, page_table, ctx_lens, positions):
        cfg = self.cfg
        B, N = tokens.shape
        ar = torch.arange(N, device=tokens.device)
        live = ar.unsqueeze(0) < n_nodes.unsqueeze(1)
        slots = ctx_lens.long().unsqueeze(1) + ar.unsqueeze(0)
        h = self.w["token_embd.weight"][tokens.clamp_min(0).long()]  # [B, N, n_embd]
        for l in range(cfg.n_layers):
            blk = f"blk.{l}."
            hn = rms_norm(h, self.w[blk + "attn_norm.weight"], cfg.rms_eps)
            q = self._proj(hn, blk + "attn_q").view(B, N, cfg.n_head, cfg.head_dim)
            k = self._proj(hn, blk + "attn_k").view(B, N, cfg.n_head_kv, cfg.head_dim)
            v = self._proj(hn, blk + "attn_v").view(B, N, cfg.n_head_kv, cfg.head_dim)
            if blk + "attn_q_norm.weight" in self.w:
                q = rms_norm(q, self.w[blk + "attn_q_norm.weight"], cfg.rms_eps)
            if blk + "attn_k_norm.weight" in self.w:
                k = rms_norm(k, self.w[blk + "attn_k_norm.weight"], cfg.rms_eps)
            q, k = rotary(q, k, positions, cfg.rope_base)
            self._write_kv(l, k, v, slots, page_table, live)
            attn, _, _ = ops.tree_attention(q.to(torch.bfloat16).contiguous(), self.k_pool[l], self.v_pool[l],
                                            page_table, ctx_lens, parents, n_nodes)
            h = h + self._proj(attn.to(self.dtype).reshape(B, N, cfg.n_head * cfg.head_dim), blk + "attn_output")
            hf = rms_norm(h, self.w[blk + "ffn_norm.weight"], cfg.rms_eps)
            act = F.silu(self._proj(hf, blk + "ffn_gate")) * self._proj(hf, blk + "ffn_up")
            h = h + self._proj(act, blk + "ffn_down")
        hn = rms_norm(h, self.w["output_norm.weight"], cfg.rms_eps)
        self.forwards += 1
        return self._head(hn)

    def _head(self, hn: torch.Tensor) -> torch.Tensor:
        """logits = hn output_w^T (engine/pipeline.py:469-472). A bf16 model
        whose sizes K7 takes (multiples of 8) runs a11s_lm_head, which also
        leaves the acceptance's chunk keys in last_chunk_keys; otherwise torch."""
        w = self.w["output.weight"]
        V, H = w.shape
        self.last_chunk_keys = None
        if w.dtype != torch.bfloat16 or H % 8 or V % 8 or "output.bias" in self.w:
            return self._proj(hn, "output")
        lead = hn.shape[:-1]
        logits, keys, _ = ops.lm_head(hn.reshape(-1, H).to(torch.bfloat16).contiguous(), w, want_keys=True)
        self.last_chunk_keys = keys
        return logits.view(*lead, V)

    # -- the target-model interface of generate.speculative_stream -----------
    def forward_tree(self, tokens, parents, n_nodes, page_table, ctx_lens) -> torch.Tensor:
        """Logits [B, N, V] of every node; node i's K/V land at slot ctx + i."""
        pos = ctx_lens.long().unsqueeze(1) + tree_depths(parents, n_nodes)
        return self._forward(tokens, parents, n_nodes, page_table, ctx_lens, pos).contiguous()

    def prefill(self, tokens, page_table, ctx_lens=None, chunk: int = 64) -> Optional[torch.Tensor]:
        """K/V of the prompt tokens [B, T] at positions 0 .. T-1, as chain trees
        of up to `chunk` tokens (each attends to the earlier chunks and to its
        own prefix). Returns the logits of the last chunk."""
        B, T = tokens.shape
        logits = None
        for c0 in range(0, T, chunk):
            n = min(chunk, T - c0)
            par = (torch.arange(n, device=tokens.device, dtype=torch.int32) - 1).unsqueeze(0).expand(B, n).contiguous()
            nn = torch.full((B,), n, dtype=torch.int32, device=tokens.device)
            ctx = torch.full((B,), c0, dtype=torch.int32, device=tokens.device)
            pos = c0 + torch.arange(n, device=tokens.device).unsqueeze(0).expand(B, n)
            logits = self._forward(tokens[:, c0:c0 + n].contiguous(), par, nn, page_table, ctx, pos)
        return logits


def synthetic_tensors(cfg: DecoderConfig, seed: int) -> Dict[str, torch.Tensor]:
    """Seeded fp32 weights with the reference's tensor names (CPU generator,
    so every machine draws the same values): embeddings N(0, 1), projections
    N(0, 1/fan_in), norms 1 + N(0, 0.1^2)."""
    g = torch.Generator().manual_seed(seed)

    def rnd(*shape, std=1.0):
        return torch.randn(*shape, generator=g) * std

    H, D = cfg.n_embd, cfg.head_dim
    t = {"token_embd.weight": rnd(cfg.vocab, H)}
    for l in range(cfg.n_layers):
        p = f"blk.{l}."
        t[p + "attn_norm.weight"] = 1.0 + rnd(H, std=0.1)
        t[p + "attn_q.weight"] = rnd(cfg.n_head * D, H, std=H ** -0.5)
        t[p + "attn_k.weight"] = rnd(cfg.n_head_kv * D, H, std=H ** -0.5)
        t[p + "attn_v.weight"] = rnd(cfg.n_head_kv * D, H, std=H ** -0.5)
        t[p + "attn_output.weight"] = rnd(H, cfg.n_head * D, std=(cfg.n_head * D) ** -0.5)
        t[p + "ffn_norm.weight"] = 1.0 + rnd(H, std=0.1)
        t[p + "ffn_gate.weight"] = rnd(cfg.n_ff, H, std=H ** -0.5)
        t[p + "ffn_up.weight"] = rnd(cfg.n_ff, H, std=H ** -0.5)
        t[p + "ffn_down.weight"] = rnd(H, cfg.n_ff, std=cfg.n_ff ** -0.5)
    t["output_norm.weight"] = 1.0 + rnd(H, std=0.1)
    t["output.weight"] = rnd(cfg.vocab, H, std=2.0 * H ** -0.5)
    return t
