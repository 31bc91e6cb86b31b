"""K3 acceptance on the GPU, through the C ABI, against the oracle and the
golden vectors. Decisions (lengths, nodes, tokens, bonus) are bit-exact;
probabilities are compared with fp32 torch softmax at rtol 1e-5."""
import json
import os

import numpy as np
import pytest
import torch

import oracle
import a11spec
from a11spec import workloads as W

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_gpu(mode, target, tokens, parents, n_nodes=None, draft=None, T=1.0, uniforms=None,
            dtype=torch.float32, stats=None):
    dev = "cuda"
    t = torch.as_tensor(target).to(dev, dtype).contiguous()
    d = None if draft is None else torch.as_tensor(draft).to(dev, dtype).contiguous()
    r = a11spec.accept(mode, t, torch.as_tensor(tokens, dtype=torch.int32, device=dev),
                       torch.as_tensor(parents, dtype=torch.int32, device=dev),
                       None if n_nodes is None else torch.as_tensor(n_nodes, dtype=torch.int32, device=dev),
                       draft_logits=d, temperature=T,
                       uniforms=None if uniforms is None else torch.as_tensor(uniforms, dtype=torch.float32, device=dev),
                       stats=stats, want_node_probs=mode != a11spec.GREEDY)
    code, _ = a11spec.read_status(r.workspace)
    out = dict(accept_len=r.accept_len.cpu().numpy(), accepted_nodes=r.accepted_nodes.cpu().numpy(),
               accepted_tokens=r.accepted_tokens.cpu().numpy(), bonus=r.bonus.cpu().numpy(),
               status=code)
    if r.node_probs is not None:
        out["node_probs"] = r.node_probs.cpu().numpy()
    return out


def widen(x, dtype):
    """Values the kernel sees: bf16 inputs widened exactly to fp32."""
    t = torch.as_tensor(x)
    return t.to(dtype).float().numpy() if dtype == torch.bfloat16 else t.float().numpy()


def assert_same_decisions(g, o):
    assert g["status"] == o["status"] == 0
    np.testing.assert_array_equal(g["accept_len"], o["accept_len"])
    np.testing.assert_array_equal(g["accepted_nodes"], o["accepted_nodes"])
    np.testing.assert_array_equal(g["accepted_tokens"], o["accepted_tokens"])
    np.testing.assert_array_equal(g["bonus"], o["bonus"])


def test_c1_greedy_chain_golden():
    g = json.load(open(os.path.join(ROOT, "tests", "golden", "c1_greedy_chain.json")))
    d = W.make_c1(seed=g["seed"])
    r = run_gpu(a11spec.GREEDY, d["logits"], d["tokens"], d["parents"], d["n_nodes"])
    assert r["status"] == 0
    assert int(r["accept_len"][0]) == g["accept_len"] == g["ref_accepted_len"]
    assert r["accepted_tokens"][0, : g["accept_len"]].tolist() == g["accepted_tokens"]
    assert int(r["bonus"][0]) == g["bonus"]


@pytest.mark.parametrize("seed", range(6))
def test_c1_greedy_chain_vs_oracle(seed):
    d = W.make_c1(seed=seed)
    r = run_gpu(a11spec.GREEDY, d["logits"], d["tokens"], d["parents"], d["n_nodes"])
    o = oracle.accept(0, d["logits"], d["tokens"], d["parents"], d["n_nodes"])
    assert_same_decisions(r, o)


def test_c2_greedy_binary_tree_full_size():
    d = W.make_c2(seed=2)
    r = run_gpu(a11spec.GREEDY, d["logits_bf16"], d["tokens"], d["parents"], d["n_nodes"],
                dtype=torch.bfloat16)
    o = oracle.accept(0, d["logits"], d["tokens"], d["parents"], d["n_nodes"])
    assert_same_decisions(r, o)
    assert r["accept_len"].max() >= 1  # 60% forced matches make some paths


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_greedy_random_trees_ragged(dtype):
    rng = np.random.default_rng(11)
    B, N, V = 6, 40, 20000
    x = rng.normal(0, 2, (B, N, V)).astype(np.float32)
    parents = np.stack([W.random_parents(N, rng) for _ in range(B)])
    tokens = rng.integers(0, V, (B, N)).astype(np.int32)
    for b in range(B):
        for i in range(1, N):
            if rng.random() < 0.6:
                x[b, parents[b, i], tokens[b, i]] = 50.0 + i  # later siblings win ties of force
    nn = np.array([N, 1, 2, 17, N - 1, 30], np.int32)
    r = run_gpu(0, x, tokens, parents, nn, dtype=dtype)
    o = oracle.accept(0, widen(x, dtype), tokens, parents, nn)
    assert_same_decisions(r, o)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("T", [0.7, 1.0])
def test_stochastic_onehot_vs_oracle(dtype, T):
    rng = np.random.default_rng(21)
    B, N, V = 8, 33, 151936
    x = rng.normal(0, 2, (B, N, V)).astype(np.float32)
    parents = np.tile(W.schedule_parents((4, 2, 2, 2), N), (B, 1))
    tokens = np.zeros((B, N), np.int32)
    xw = widen(x, dtype)
    for b in range(B):
        for i in range(1, N):  # propose likely tokens so some get accepted
            row = xw[b, parents[b, i]]
            tokens[b, i] = int(np.argsort(row)[-1 - rng.integers(0, 4)])
    uni = rng.random((B, N), dtype=np.float32)
    r = run_gpu(1, x, tokens, parents, T=T, uniforms=uni, dtype=dtype)
    o = oracle.accept(1, xw, tokens, parents, temperature=T, uniforms=uni)
    assert_same_decisions(r, o)
    np.testing.assert_array_equal(r["node_probs"], o["node_probs"])  # bit-identical softmax
    # and against torch fp32 softmax (tolerance for fp32 probabilities)
    sm = torch.softmax(torch.from_numpy(xw[:, :, :]).double() / T, dim=-1).numpy()
    for b in range(B):
        for i in range(1, N):
            ref = sm[b, parents[b, i], tokens[b, i]]
            assert abs(r["node_probs"][b, i] - ref) <= 1e-5 * ref + 1e-9


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_walk_with_and_without_waiting_for_records(mode):
    """Up to one sequence per SM, the walk waits for the rows that other blocks
    record; above that it takes a visited row's statistics from the row itself.
    Both give the oracle's decisions, on deep walks (forced matches) and a
    ragged last chunk."""
    n_sms = torch.cuda.get_device_properties(0).multi_processor_count
    N, V = 12, 2 * 2048 + 136
    for B in (3, n_sms + 52):
        rng = np.random.default_rng(31 + mode + B)
        x = rng.normal(0, 2, (B, N, V)).astype(np.float32)
        parents = np.stack([W.random_parents(N, rng) for _ in range(B)]).astype(np.int32)
        tokens = rng.integers(0, V, (B, N)).astype(np.int32)
        for b in range(B):
            for i in range(1, N):
                if rng.random() < 0.7:
                    x[b, parents[b, i], tokens[b, i]] += 40.0
        q = (x + rng.normal(0, 0.5, x.shape)).astype(np.float32) if mode == 2 else None
        uni = rng.random((B, N), dtype=np.float32) if mode else None
        r = run_gpu(mode, x, tokens, parents, draft=q, T=0.8, uniforms=uni)
        o = oracle.accept(mode, x, tokens, parents, draft=q, temperature=0.8, uniforms=uni)
        assert_same_decisions(r, o)
        assert r["accept_len"].mean() > 1.0, B  # the walks leave the root


def test_c3_draft_logits_reduced_vs_oracle():
    d = W.make_c3(seed=3, batch=3, n_nodes=64, vocab=151936)
    r = run_gpu(2, d["p"], d["tokens"], d["parents"], d["n_nodes"], draft=d["q"],
                T=d["temperature"], uniforms=d["uniforms"])
    o = oracle.accept(2, d["p"], d["tokens"], d["parents"], d["n_nodes"], draft=d["q"],
                      temperature=d["temperature"], uniforms=d["uniforms"])
    assert_same_decisions(r, o)
    np.testing.assert_array_equal(r["node_probs"], o["node_probs"])


def test_c3_full_size_properties(dev):
    """Full C3 (B=64, 63 drafts, fp32 p and q over 151936 tokens, 4.98 GB):
    deterministic, invariants hold, and every one of the 64 sequences matches
    the oracle bit for bit (decisions, bonus and node probabilities)."""
    d = W.make_c3(seed=3, batch=64, device=dev)
    args = (d["p"], d["tokens"], d["parents"], d["n_nodes"])
    kw = dict(draft_logits=d["q"], temperature=d["temperature"], uniforms=d["uniforms"])
    stats = torch.zeros(6, dtype=torch.int64, device=dev)
    r1 = a11spec.accept(2, *args, stats=stats, want_node_probs=True, **kw)
    r2 = a11spec.accept(2, *args, **kw)
    assert a11spec.read_status(r1.workspace)[0] == 0
    assert torch.equal(r1.accept_len, r2.accept_len) and torch.equal(r1.bonus, r2.bonus)
    al = r1.accept_len.cpu()
    assert al.min() >= 0 and al.max() <= 5  # depth of the 63-node tree
    assert int(stats[4]) == 64 and int(stats[5]) == int(al.sum()) + 64
    got = dict(accept_len=al.numpy(), accepted_nodes=r1.accepted_nodes.cpu().numpy(),
               accepted_tokens=r1.accepted_tokens.cpu().numpy(), bonus=r1.bonus.cpu().numpy(),
               node_probs=r1.node_probs.cpu().numpy())
    tokens, parents, uni = d["tokens"].cpu().numpy(), d["parents"].cpu().numpy(), d["uniforms"].cpu().numpy()
    for b0 in range(0, 64, 8):  # eight sequences per oracle call (about 2.5 GB of host copies at a time)
        sl = slice(b0, b0 + 8)
        o = oracle.accept(2, d["p"][sl].cpu().numpy(), tokens[sl], parents[sl], None, draft=d["q"][sl].cpu().numpy(),
                          temperature=d["temperature"], uniforms=uni[sl])
        assert o["status"] == 0
        for name in ("accept_len", "accepted_nodes", "accepted_tokens", "bonus", "node_probs"):
            np.testing.assert_array_equal(got[name][sl], o[name], err_msg=f"{name}, sequences {b0}..{b0 + 7}")


def test_stats_counters(dev):
    d = W.make_c1(seed=4)
    st = torch.zeros(6, dtype=torch.int64, device=dev)
    for _ in range(3):
        run_gpu(0, d["logits"], d["tokens"], d["parents"], d["n_nodes"], stats=st)
    o = oracle.accept(0, d["logits"], d["tokens"], d["parents"], d["n_nodes"])
    s = st.cpu().numpy()
    assert s[4] == 3 and s[3] == 15
    assert s[5] == 3 * (int(o["accept_len"][0]) + 1)
    assert s[0] + s[1] == s[4]


def test_status_words(dev):
    V = 64
    x = np.zeros((1, 3, V), np.float32)
    par = np.array([[-1, 0, 1]], np.int32)
    assert run_gpu(0, x, np.array([[0, 1, V]], np.int32), par)["status"] == a11spec.ops._lib.EBOUNDS
    bad = x.copy()
    bad[0, 1, 5] = np.nan
    assert run_gpu(0, bad, np.array([[0, 1, 2]], np.int32), par)["status"] == a11spec.ops._lib.ENONFINITE
    bad[0, 1, 5] = np.inf
    assert run_gpu(1, bad, np.array([[0, 1, 2]], np.int32), par, T=1.0,
                   uniforms=np.zeros((1, 3), np.float32))["status"] == a11spec.ops._lib.ENONFINITE
    # a clean call afterwards reports OK again (the word is cleared per call)
    assert run_gpu(0, x, np.array([[0, 1, 2]], np.int32), par)["status"] == 0


def test_host_validation_errors(dev):
    t = torch.zeros(1, 2, 12, device=dev)  # vocab 12 not a multiple of 8 for bf16
    tok = torch.zeros(1, 2, dtype=torch.int32, device=dev)
    par = torch.tensor([[-1, 0]], dtype=torch.int32, device=dev)
    with pytest.raises(a11spec.A11Error):
        a11spec.accept(0, t.to(torch.bfloat16), tok, par)
    with pytest.raises(a11spec.A11Error):
        a11spec.accept(1, t, tok, par)  # sampling without uniforms
    with pytest.raises(a11spec.A11Error):
        a11spec.accept(2, t, tok, par, uniforms=torch.zeros(1, 2, device=dev))  # no draft logits
