"""The drop-in host layer on the GPU: a11s_verify_chain against the reference
verifier's recorded decisions, the reference's verifier test expectations
(tests/test_speculative_verifier.cpp, tests/test_python_bindings.py:166-275)
run against the a11spec verifier, the SpeculativeDecoder list API, and one
end-to-end step through the paged KV manager."""
import json
import os
import subprocess

import numpy as np
import pytest
import torch

import oracle
import a11spec
from a11spec import workloads as W
from a11spec.decoder import SpeculativeDecoder
from a11spec.kv_pages import KVCacheConfig, PagedKVCacheManager
from a11spec.verifier import SpecConfig, SpeculativeTreeVerifier, verify_chains, SPEC_K

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = json.load(open(os.path.join(ROOT, "tests", "golden", "ref_chains.json")))


def _cuda(a):
    return torch.tensor(np.asarray(a, np.float32)).cuda()


def test_verify_chain_matches_reference_decisions(dev):
    cases = GOLD["cases"]
    n = max(len(c["p"]) for c in cases)
    d = np.ones((len(cases), n), np.float32)
    t = np.zeros((len(cases), n), np.float32)
    u = np.ones((len(cases), n), np.float32)  # padding positions are never reached past a rejection...
    lens = []
    for i, c in enumerate(cases):
        k = len(c["p"])
        d[i, :k], t[i, :k], u[i, :k] = c["q"], c["p"], c["u"]
        lens.append(k)
    # ...except when the whole chain is accepted: pad with a rejecting uniform (u=1)
    al, li, _ = verify_chains(_cuda(d), _cuda(t), _cuda(u))
    for i, c in enumerate(cases):
        assert int(al[i]) == c["ref_accepted_len"], (i, c)
        assert int(li[i]) == c["ref_last_idx"], (i, c)


def test_verify_chain_log_space_kats_and_oracle(dev):
    for kat in GOLD["log_space_kats"]:
        al, li, _ = verify_chains(_cuda([kat["draft"]]), _cuda([kat["target"]]), _cuda([kat["u"]]))
        assert (int(al[0]), int(li[0])) == (kat["ref_accepted_len"], kat["ref_last_idx"])
    rng = np.random.default_rng(9)
    d = -rng.uniform(0.01, 3.0, (500, 8)).astype(np.float32)
    t = (d + rng.normal(0, 0.8, d.shape)).astype(np.float32)
    t[::7] = np.abs(t[::7])  # some rows in linear space
    u = rng.random(d.shape, dtype=np.float32)
    al, li, _ = verify_chains(_cuda(d), _cuda(t), _cuda(u))
    oal, oli, rc = oracle.verify_chain(d, t, u)
    assert rc == 0
    np.testing.assert_array_equal(al.cpu().numpy(), oal)
    np.testing.assert_array_equal(li.cpu().numpy(), oli)


def test_verify_chain_nonfinite_reports(dev):
    ws = torch.zeros(256, dtype=torch.uint8, device="cuda")
    al, _, ws = verify_chains(_cuda([[0.5, 0.5]]), _cuda([[0.5, np.nan]]), _cuda([[0.1, 0.1]]), ws)
    assert int(al[0]) == -1 and a11spec.read_status(ws)[0] == a11spec.ENONFINITE


# ----------------------------------------------------------------------------- reference test expectations
def _verifier(**kw):
    cfg = SpecConfig()
    cfg.log_diagnostics = False
    for k, v in kw.items():
        setattr(cfg, k, v)
    return SpeculativeTreeVerifier(cfg)


def test_reference_verifier_cases(dev):
    v = _verifier()
    lp = [-0.1, -0.2, -0.15, -0.3, -0.1, -0.25, -0.2, -0.18]
    assert v.verify_draft_tokens(list(range(1, 9)), lp, lp) == (SPEC_K, SPEC_K - 1)
    a, last = v.verify_draft_tokens([10, 20, 30, 40, 50, 60, 70, 80], [-0.5] * 8,
                                    [-0.1, -0.1, -0.1, -5.0, -0.1, -0.1, -0.1, -0.1])
    assert 0 < a <= SPEC_K and last < SPEC_K - 1
    with pytest.raises(RuntimeError):
        v.verify_draft_tokens([1, 2, 3], [-0.5, -0.5], [0.9, 0.9, 0.9])
    root = v.build_draft_tree(42)
    assert root.token_id == 42 and root.parent_idx == 0xFFFFFFFF and root.depth == 0 and not root.children
    v100 = _verifier(vocab_size=100)
    tree = [a11spec.verifier.TreeNode(token_id=10 + 10 * i, parent_idx=i - 1 if i else 0xFFFFFFFF, depth=i)
            for i in range(SPEC_K)]
    mask = np.asarray(v100.construct_tree_mask(tree)).reshape(SPEC_K, 100)
    assert mask.sum() == SPEC_K and all(mask[i, 10 + 10 * i] == 1.0 for i in range(SPEC_K))


def test_reference_binding_cases(dev):  # tests/test_python_bindings.py:198-275 of the reference
    v = _verifier()
    assert v.verify_draft_tokens([10, 20, 30, 40], [-0.5, -0.6, -0.7, -0.8], [-0.5, -0.6, -0.7, -0.8]) == (4, 3)
    a, last = v.verify_draft_tokens([10, 20, 30, 40], [-0.5] * 4, [-0.6, -0.6, -10.0, -0.6])
    assert 0 <= a < 4 and (last < 3 or a == 0)
    out, full = v.speculate_step([1, 2, 3], 100)
    assert isinstance(out, list) and len(out) >= 1 and isinstance(full, bool)
    for i in range(5):
        v.speculate_step([1], 42 + i)
    d = v.diagnostics()
    assert d.total_steps == 6 and d.steps_accepted + d.steps_rejected == d.total_steps
    assert d.total_draft_tokens == 6 * SPEC_K
    v.reset_diagnostics()
    assert v.diagnostics().total_steps == 0 and v.diagnostics().fallback_count == 0


def test_stream_continuity_matches_reference_verifier(dev):
    """Successive calls on one thread continue the uniform stream exactly where
    the reference's thread_local generator would be."""
    if oracle.ref() is None:
        pytest.skip("reference verifier not built on this machine")
    import threading
    rng = np.random.default_rng(4)
    calls = []
    for _ in range(12):
        k = int(rng.integers(1, 9))
        q = rng.uniform(0.05, 1, k).astype(np.float32)
        p = np.clip(q * rng.uniform(0.3, 1.5, k), 0, 1).astype(np.float32)
        calls.append((q, p))
    ours, theirs = [], []

    def run_ours():
        v = _verifier()
        for q, p in calls:
            ours.append(v.verify_draft_tokens(list(range(len(q))), q.tolist(), p.tolist()))

    th = threading.Thread(target=run_ours)  # a fresh thread starts a fresh stream
    th.start()
    th.join()
    # replay: call i consumed min(n, accepted + 1) draws of the reference stream
    u = oracle.ref_uniform_stream(200)
    pos = 0
    for (q, p), (a, last) in zip(calls, ours):
        al, li, _ = oracle.verify_chain(q[None], p[None], u[pos:pos + len(q)][None])
        assert (int(al[0]), int(li[0])) == (a, last)
        pos += min(len(q), a + 1)


def test_reference_catch2_suite_against_cpp_adapter(dev):
    """The reference's tests/test_speculative_verifier.cpp, unchanged, linked
    against A11::Engine::SpeculativeTreeVerifier of this repository (built
    from the reference tree by `make -C oracle adapter`)."""
    exe = os.path.join(ROOT, "oracle", "_ref", "ref_tests_on_a11spec")
    if not os.path.exists(exe):
        pytest.skip("adapter test binary not built (needs the reference tree at build time)")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert "All tests passed" in r.stdout


def test_reference_python_binding_tests_against_a11_optimizer(dev):
    """The reference's tests/test_python_bindings.py, unchanged (compiled to
    bytecode from the reference tree at build time), against the module
    a11_optimizer of this repository: its module constants, PagedKVCacheManager,
    SpeculativeTreeVerifier (:166-275) and cross-class cases. The NvmeAsyncLoader
    cases belong to weight streaming, which this library does not provide."""
    import importlib.machinery
    import importlib.util

    import a11_optimizer
    pyc = os.path.join(ROOT, "oracle", "_ref", "test_python_bindings.bytecode")
    if not os.path.exists(pyc):
        pytest.skip("reference binding tests not compiled (needs the reference tree at build time)")
    loader = importlib.machinery.SourcelessFileLoader("ref_test_python_bindings", pyc)
    mod = importlib.util.module_from_spec(importlib.util.spec_from_loader(loader.name, loader))
    loader.exec_module(mod)
    ran = []
    for cls_name in ("TestModuleConstants", "TestPagedKVCacheManager", "TestSpeculativeTreeVerifier",
                     "TestCrossClassIntegration"):
        cls = getattr(mod, cls_name)
        for name in sorted(n for n in dir(cls) if n.startswith("test_")):
            getattr(cls(), name)(a11_optimizer)
            ran.append(f"{cls_name}.{name}")
    assert len(ran) == 3 + 7 + 9 + 1, ran


# ----------------------------------------------------------------------------- SpeculativeDecoder
def test_decoder_list_api_and_step(dev):
    V = 4096
    table = W.make_ngram_table(log2_buckets=10, vocab=V, seed=2)
    dec = SpeculativeDecoder(draft_k=3, table=torch.from_numpy(table), log2_buckets=10, max_depth=3,
                             max_nodes=16)
    drafts = dec.generate_draft_tokens([5, 9])
    o = oracle.ngram_expand(table, 10, np.array([[5, 9]], np.int32), 1, 1, 3, 4)
    assert drafts == o["tokens"][0, 1:o["n_nodes"][0]].tolist() and len(drafts) == 3
    logits = torch.randn(4, V, device="cuda")
    logits[0, drafts[0]] = 50.0
    logits[1, drafts[1]] = 50.0
    assert dec.verify_candidates(logits, drafts) == drafts[:2]
    assert dec.verify_candidates(logits[:3], drafts) == drafts[:2]

    # one batched step through the paged KV manager
    B, N, Hkv, Hq, D = 2, 16, 2, 16, 128
    kv = PagedKVCacheManager(KVCacheConfig(num_layers=1, head_dim=D, num_kv_heads=Hkv, max_sequences=B,
                                           vram_cap_gb=0.01), device="cuda")
    ctx = [40, 77]
    for s in range(B):
        kv.allocate_sequence(s)
        kv.append_tokens(s, ctx[s])
        kv.reserve_tree(s, N)
    kpool, vpool = kv.k_pool[0], kv.v_pool[0]
    kpool.normal_()
    vpool.normal_()
    pt = kv.page_table([0, 1], 8, "cuda")
    seq_lens = torch.tensor(ctx, dtype=torch.int32, device="cuda")
    q = torch.randn(B, N, Hq, D, device="cuda").to(torch.bfloat16)
    last = torch.tensor([[5, 9], [1, 2]], dtype=torch.int32, device="cuda")
    dec2 = SpeculativeDecoder(table=torch.from_numpy(table), log2_buckets=10, max_depth=3, max_nodes=N,
                              temperature=0.7)
    tree, res = dec2.step(last, q, kpool, vpool, pt, seq_lens,
                          lambda attn, tr: torch.randn(B, N, V, device="cuda").to(torch.bfloat16))
    torch.cuda.synchronize()
    assert torch.equal(seq_lens.cpu(), torch.tensor(ctx, dtype=torch.int32) + 1 + res.accept_len.cpu())
    st = dec2.diagnostics()
    assert st["total_steps"] == B and st["emitted_tokens"] == int(res.accept_len.sum()) + B
