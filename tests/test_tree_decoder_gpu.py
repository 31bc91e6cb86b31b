"""Speculative generation driven by a decoder stack shaped like the
reference's (a11spec.tree_model.TreeDecoder: forward_layer of
engine/pipeline.py:350-447 over token trees, tree attention where the
reference computes its decode attention, K/V through the page table).

tests/golden/tree_decoder_decode.npz holds a greedy decode by the reference's
own A11Pipeline.forward_token / forward_layer (bf16, its KVCacheManager) on the
same seeded weights (make_golden.py). On the GPU:

* teacher-forced one-token decode through TreeDecoder (one-node trees, paged
  KV, a11s_tree_attention) reproduces the reference's logits at every step;
* free-running greedy decoding through speculative_stream with an empty n-gram
  table (one token per target forward) reproduces the reference's tokens over
  the steps whose top-2 gap the rounding cannot close;
* speculative greedy decoding with an n-gram table that knows the sequence
  commits exactly the same tokens, with several tokens per target forward:
  accepted drafts, their compaction and the rotary positions of tree nodes are
  all on that path.
"""
import os

import numpy as np
import pytest
import torch

import a11spec
from a11spec.decoder import SpeculativeDecoder
from a11spec.generate import speculative_stream
from a11spec.ops import KVPagePool
from a11spec.tree_model import DecoderConfig, TreeDecoder, synthetic_tensors

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = np.load(os.path.join(HERE, "golden", "tree_decoder_decode.npz"))
CFG = DecoderConfig(n_layers=2, n_embd=256, n_head=8, n_head_kv=1, head_dim=128, n_ff=512, vocab=512)
PAGES = 64
# bf16 logits of magnitude <= 8 from two bf16 pipelines (the reference's on the
# host, this one on the GPU): every bf16 rounding of an intermediate may land
# one unit (2^-8 relative) apart; the bound is 4 % of the row's largest logit.
TOL_REL = 4e-2


def _model(dev):
    return TreeDecoder(synthetic_tensors(CFG, int(GOLD["weight_seed"])), CFG, PAGES, dev)


def test_teacher_forced_decode_matches_reference(dev):
    model = _model(dev)
    prompt = torch.from_numpy(GOLD["prompt"]).to(dev).view(1, -1)
    T = prompt.shape[1]
    pool = KVPagePool(PAGES, dev)
    page_table = torch.full((1, 16), -1, dtype=torch.int32, device=dev)
    ctx = torch.zeros(1, dtype=torch.int32, device=dev)
    pool.reserve(page_table, ctx, torch.full((1,), T - 1, dtype=torch.int32, device=dev), check_status=True)
    model.prefill(prompt[:, :T - 1], page_table)
    one = torch.ones(1, dtype=torch.int32, device=dev)
    par = torch.full((1, 1), -1, dtype=torch.int32, device=dev)
    tok = int(GOLD["prompt"][-1])
    worst = 0.0
    for k in range(len(GOLD["tokens"])):
        grown = ctx.clone()
        pool.reserve(page_table, grown, one, check_status=True)  # the slot of this token
        logits = model.forward_tree(torch.tensor([[tok]], dtype=torch.int32, device=dev), par, one, page_table, ctx)
        got = logits[0, 0].float().cpu().numpy()
        want = GOLD["logits"][k]
        err = float(np.abs(got - want).max() / np.abs(want).max())
        worst = max(worst, err)
        assert err <= TOL_REL, (k, err)
        if GOLD["gaps"][k] >= 2 * TOL_REL * np.abs(want).max():
            assert int(np.argmax(got)) == int(GOLD["tokens"][k]), k
        ctx.copy_(grown)
        tok = int(GOLD["tokens"][k])  # teacher forcing: the reference's token
    print(f"worst logit deviation {worst:.4f} of the row maximum")


def _stream(dev, table=None, learn=False):
    model = _model(dev)
    prompt = torch.from_numpy(GOLD["prompt"]).to(dev).view(1, -1).contiguous()
    dec = SpeculativeDecoder(table=table if table is not None else torch.zeros((1 << 10, 4, 2), dtype=torch.int32),
                             log2_buckets=10, width_root=2, width_inner=1, max_depth=5, max_nodes=16,
                             temperature=None, device=dev)
    out, forwards = [], 0
    for new in speculative_stream(model, prompt, len(GOLD["tokens"]), dec, KVPagePool(PAGES, dev), max_pages=16,
                                  learn=learn):
        out += new[0]
        forwards += 1
    return out, forwards


def test_greedy_decoding_reproduces_reference_tokens(dev):
    out, forwards = _stream(dev)
    assert forwards == len(GOLD["tokens"])  # an empty table drafts nothing: one token per forward
    want = GOLD["tokens"].tolist()
    first_close = int(np.argmax(GOLD["gaps"] < 0.1)) if (GOLD["gaps"] < 0.1).any() else len(want)
    assert first_close >= 20
    assert out[:first_close] == want[:first_close]


def test_speculative_greedy_equals_token_by_token(dev):
    plain, _ = _stream(dev)
    # a table that knows this sequence: every trigram of prompt + output
    seq = GOLD["prompt"].tolist() + plain
    hist = torch.tensor([seq], dtype=torch.int32, device=dev)
    table = torch.zeros((1 << 10, 4, 2), dtype=torch.int32, device=dev)
    a11spec.ngram_update(table, hist, torch.tensor([len(seq)], dtype=torch.int32, device=dev), 10,
                         check_status=True)
    spec, forwards = _stream(dev, table=table, learn=True)
    assert spec == plain
    assert forwards <= len(plain) // 2, forwards  # drafts accepted: several tokens per target forward
