"""The acceptance softmax against the reference's sampler.

tests/golden/sampler_probs.json holds p(token) from the reference's
TokenSampler (engine/sampler.py) with top-k and top-p off, i.e.
softmax(logits / max(T, 1e-5)), for three logits rows (vocab 32000 / 151936 /
4096, T = 0.7 / 1.3 / 0.05). The acceptance kernel's node_probs report
p(tokens[i]) in the parent's row, so a root with one child per recorded token
reads them out. Oracle (CPU) and kernel (GPU) must match within the fp32
probability tolerance: 1e-5 relative (1e-9 absolute for vanishing p)."""
import json
import os
import sys

import numpy as np
import pytest

import oracle

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
from make_golden import sampler_logits  # noqa: E402

GOLDEN = json.load(open(os.path.join(HERE, "golden", "sampler_probs.json")))["cases"]


def _tree(case):
    """One sequence: row 0 = the case's logits, children of the root carry
    the recorded tokens (the other rows are never read for node_probs)."""
    toks = case["tokens"]
    n = 1 + len(toks)
    x = np.zeros((1, n, case["vocab"]), np.float32)
    x[0, 0] = sampler_logits(case["seed"], case["vocab"])
    tokens = np.array([[0] + toks], np.int32)
    parents = np.array([[-1] + [0] * len(toks)], np.int32)
    uni = np.full((1, n), 0.5, np.float32)
    return x, tokens, parents, uni


def _check(node_probs, case):
    got = np.asarray(node_probs, np.float64)[0, 1:]
    want = np.asarray(case["probs"], np.float64)
    assert np.all(np.abs(got - want) <= 1e-5 * want + 1e-9), np.abs(got - want).max()


@pytest.mark.parametrize("ci", range(len(GOLDEN)))
def test_oracle_matches_reference_sampler(ci):
    case = GOLDEN[ci]
    x, tokens, parents, uni = _tree(case)
    o = oracle.accept(1, x, tokens, parents, temperature=case["temperature"], uniforms=uni)
    _check(o["node_probs"], case)


@pytest.mark.gpu
@pytest.mark.parametrize("ci", range(len(GOLDEN)))
def test_kernel_matches_reference_sampler(dev, ci):
    import torch
    import a11spec
    case = GOLDEN[ci]
    x, tokens, parents, uni = _tree(case)
    r = a11spec.accept(a11spec.STOCH_ONEHOT, torch.from_numpy(x).to(dev), torch.from_numpy(tokens).to(dev),
                       torch.from_numpy(parents).to(dev), temperature=case["temperature"],
                       uniforms=torch.from_numpy(uni).to(dev), want_node_probs=True, check_status=True)
    _check(r.node_probs.cpu().numpy(), case)
