"""Tree attention against the reference's own decode attention.

tests/golden/attn_chains.npz was produced by the reference's code (its paged
KV cache, engine/kv_cache.py, and the attention statements of
A11Pipeline.forward_layer, engine/pipeline.py; see make_golden.py): a prompt
of `ctx` tokens, then a chain of `n` tokens decoded one by one. A chain-shaped
draft tree (parents[i] = i - 1) asks exactly that: node i attends to the
context and nodes 0..i. The oracle (CPU) and the kernel (GPU) must match the
reference's outputs element by element: |got - ref| <= 2e-2 |ref| + a floor
per row from the bf16 rounding of the probabilities (tests/attn_tolerance.py);
the reference rounds its probabilities to bf16 before PV, as the kernel does."""
import os

import numpy as np
import pytest
import torch

import attn_tolerance as AT
import oracle

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = np.load(os.path.join(HERE, "golden", "attn_chains.npz"))
CASES = sorted({k.split("_")[0] for k in GOLDEN.files})


def _bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.int16)).view(torch.bfloat16)


def _case(name: str):
    ctx, n, hkv = (int(x) for x in GOLDEN[f"{name}_meta"])
    q = _bf16(GOLDEN[f"{name}_q"])          # [n, Hq, D]
    k = _bf16(GOLDEN[f"{name}_k"])          # [ctx + n, Hkv, D]
    v = _bf16(GOLDEN[f"{name}_v"])
    want = _bf16(GOLDEN[f"{name}_out"]).float().numpy()  # [n, Hq, D]
    # the sequence's tokens on 16-token pages in a shuffled page order
    s = ctx + n
    pages = (s + 15) // 16
    perm = np.random.default_rng(len(name) + ctx).permutation(pages + 3)[:pages].astype(np.int32)
    k_pool = torch.zeros(pages + 3, 16, hkv, 128, dtype=torch.bfloat16)
    v_pool = torch.zeros_like(k_pool)
    for t in range(s):
        k_pool[perm[t // 16], t % 16] = k[t]
        v_pool[perm[t // 16], t % 16] = v[t]
    page_table = torch.from_numpy(perm).view(1, pages)
    parents = torch.tensor([[-1] + list(range(n - 1))], dtype=torch.int32)
    return dict(q=q.unsqueeze(0), k_pool=k_pool, v_pool=v_pool, page_table=page_table,
                ctx_lens=torch.tensor([ctx], dtype=torch.int32), parents=parents,
                n_nodes=torch.tensor([n], dtype=torch.int32), want=want)


def _check(got: np.ndarray, c: dict, what: str) -> None:
    _, floor = AT.reference(c["q"], c["k_pool"], c["v_pool"], c["page_table"], c["ctx_lens"], c["parents"],
                            c["n_nodes"])
    AT.assert_close(torch.as_tensor(got)[None], torch.as_tensor(c["want"])[None], floor, what)


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_decode(name):
    c = _case(name)
    out, _, rc = oracle.tree_attention(c["q"].float().numpy(), c["k_pool"].float().numpy(), c["v_pool"].float().numpy(),
                                       c["page_table"].numpy(), c["ctx_lens"].numpy(), c["parents"].numpy(),
                                       c["n_nodes"].numpy(), 1 / np.sqrt(128))
    assert rc == 0
    _check(out[0], c, f"oracle, {name}")


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_kernel_matches_reference_decode(dev, name):
    import a11spec
    c = _case(name)
    d = {k: v.to(dev) for k, v in c.items() if k != "want"}
    out, _, _ = a11spec.tree_attention(d["q"], d["k_pool"], d["v_pool"], d["page_table"], d["ctx_lens"],
                                       d["parents"], d["n_nodes"], check_status=True)
    _check(out[0].float().cpu().numpy(), c, f"kernel, {name}")
