"""speculative_stream end to end on the GPU with a toy target model: greedy
speculative output equals plain greedy decoding of the same model token for
token, the n-gram table's learning raises the tokens committed per target
forward, and one-hot sampling runs the same loop.

The toy model writes K/V from token embeddings into the paged pools at the
tree's positions, runs the tree-attention kernel, and returns logits with a
margin of 20 on perm[token] plus a small attention-dependent term (|.| < 1),
so its greedy next token is perm[token] whatever the attention returns."""
import numpy as np
import pytest
import torch

import a11spec
from a11spec.decoder import SpeculativeDecoder
from a11spec.generate import speculative_stream
from a11spec.ops import KVPagePool

pytestmark = pytest.mark.gpu

V, HQ, HKV, D = 512, 16, 2, 128


class ToyTarget:
    def __init__(self, num_pages, seed, dev):
        g = torch.Generator(device="cpu").manual_seed(seed)
        cycles = torch.randperm(V, generator=g)  # permutation made of cycles of 7 tokens
        self.perm = torch.empty(V, dtype=torch.long)
        for c0 in range(0, V - V % 7, 7):
            cyc = cycles[c0:c0 + 7]
            self.perm[cyc] = torch.roll(cyc, -1)
        for t in cycles[V - V % 7:]:
            self.perm[t] = t
        self.perm_dev = self.perm.to(dev)
        self.emb_k = (torch.randn(V, HKV, D, generator=g) * 0.5).to(dev)
        self.emb_v = torch.randn(V, HKV, D, generator=g).to(dev)
        self.emb_q = (torch.randn(V, HQ, D, generator=g) * 0.5).to(dev)
        self.proj = (torch.randn(D, V, generator=g) * 0.02).to(dev)
        self.k_pool = torch.zeros(num_pages, 16, HKV, D, dtype=torch.bfloat16, device=dev)
        self.v_pool = torch.zeros_like(self.k_pool)
        self.vocab = V

    def _write(self, tokens, pos, page_table, valid):
        b, i = torch.nonzero(valid, as_tuple=True)
        p = pos[b, i]
        page = page_table[b, p // 16].long()
        slot = (p % 16).long()
        t = tokens[b, i].long()
        self.k_pool[page, slot] = self.emb_k[t].to(torch.bfloat16)
        self.v_pool[page, slot] = self.emb_v[t].to(torch.bfloat16)

    def prefill(self, tokens, page_table, ctx_lens):
        B, T = tokens.shape
        pos = torch.arange(T, device=tokens.device).expand(B, T)
        self._write(tokens, pos, page_table, torch.ones(B, T, dtype=torch.bool, device=tokens.device))

    def forward_tree(self, tokens, parents, n_nodes, page_table, ctx_lens):
        B, N = tokens.shape
        ar = torch.arange(N, device=tokens.device)
        valid = ar.unsqueeze(0) < n_nodes.unsqueeze(1)
        self._write(tokens, ctx_lens.unsqueeze(1).long() + ar.unsqueeze(0), page_table, valid)
        q = self.emb_q[tokens.clamp_min(0).long()].to(torch.bfloat16).contiguous()
        attn, _, _ = a11spec.tree_attention(q, self.k_pool, self.v_pool, page_table, ctx_lens, parents, n_nodes)
        small = torch.tanh(attn.float().mean(dim=2) @ self.proj)  # [B, N, V], |.| < 1
        logits = small + 20.0 * torch.nn.functional.one_hot(self.perm_dev[tokens.clamp_min(0).long()], V)
        return logits.to(torch.bfloat16).contiguous()


def _run(dev, temperature, learn=True, steps_out=None):
    B, T, NEW = 3, 5, 60
    model = ToyTarget(num_pages=96, seed=3, dev=dev)
    prompts = torch.randint(0, V, (B, T), generator=torch.Generator().manual_seed(1), dtype=torch.int32).to(dev)
    dec = SpeculativeDecoder(table=torch.zeros((1 << 10, 4, 2), dtype=torch.int32), log2_buckets=10, width_root=2,
                             width_inner=1, max_depth=5, max_nodes=16, temperature=temperature, device=dev)
    pages = KVPagePool(96, dev)
    outs = [[] for _ in range(B)]
    steps = 0
    for new in speculative_stream(model, prompts, NEW, dec, pages, max_pages=16, learn=learn):
        steps += 1
        for b in range(B):
            outs[b] += new[b]
    if steps_out is not None:
        steps_out.append(steps)
    return model, prompts.cpu(), outs


def test_greedy_speculative_equals_greedy_decoding(dev):
    steps = []
    model, prompts, outs = _run(dev, None, steps_out=steps)
    for b in range(prompts.shape[0]):
        want, t = [], int(prompts[b, -1])
        for _ in range(60):
            t = int(model.perm[t])
            want.append(t)
        assert outs[b] == want, b
    # the table learns the 7-token cycles: far fewer target forwards than tokens
    assert steps[0] < 30, steps


def test_learning_raises_tokens_per_forward(dev):
    with_learning, without = [], []
    _run(dev, None, learn=True, steps_out=with_learning)
    _run(dev, None, learn=False, steps_out=without)
    assert without[0] == 60  # an empty table drafts nothing: one token (the bonus) per forward
    assert with_learning[0] < without[0] // 2


def test_sampling_mode_runs_the_same_loop(dev):
    model, prompts, outs = _run(dev, 0.7)
    for b in range(prompts.shape[0]):
        assert len(outs[b]) == 60 and all(0 <= t < V for t in outs[b])
        # a margin of 20 at temperature 0.7 leaves other tokens ~e^-28: the chain is followed
        t = int(prompts[b, -1])
        for x in outs[b][:10]:
            t = int(model.perm[t])
            assert x == t
