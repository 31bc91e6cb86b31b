"""K6 on the GPU against the oracle, bit-exact: many rows hitting few
buckets (the kernel sorts the updates so each bucket sees them in row and
position order), calls in a row on the same table, batches split over
several launches, the error path, and the draft -> accept -> learn loop."""
import numpy as np
import pytest
import torch

import a11spec
import oracle
from a11spec import ngram_table
from a11spec.ops import history_from_accept, ngram_update

pytestmark = pytest.mark.gpu
OK, EBOUNDS = 0, 2


@pytest.mark.parametrize("log2_buckets,slots,B,stride,vocab", [(4, 4, 64, 20, 12), (8, 8, 200, 40, 500),
                                                               (12, 3, 30, 70, 50)])
def test_update_matches_oracle_under_contention(dev, log2_buckets, slots, B, stride, vocab):
    rng = np.random.default_rng(log2_buckets)
    t = ngram_table.empty(log2_buckets, slots)
    dt = torch.from_numpy(t).to(dev)
    for call in range(3):
        h = rng.integers(0, vocab, (B, stride)).astype(np.int32)
        h[rng.random((B, stride)) < 0.1] = -1  # skipped trigrams
        lens = rng.integers(0, stride + 1, B).astype(np.int32)
        st = ngram_update(dt, torch.from_numpy(h).to(dev), torch.from_numpy(lens).to(dev), log2_buckets)
        r = oracle.ngram_update(t, log2_buckets, h, lens)
        torch.cuda.synchronize()
        t = r["table"]
        assert st.tolist()[0] == OK
        np.testing.assert_array_equal(dt.cpu().numpy(), t, err_msg=f"call {call}")


def test_large_batch_is_split_and_matches(dev):
    rng = np.random.default_rng(5)
    K, B, stride = 6, 600, 40  # 600 * 38 trigrams > 8192: three launches
    t = ngram_table.empty(K, 4)
    dt = torch.from_numpy(t).to(dev)
    h = rng.integers(0, 30, (B, stride)).astype(np.int32)
    lens = np.full(B, stride, np.int32)
    ngram_update(dt, torch.from_numpy(h).to(dev), torch.from_numpy(lens).to(dev), K, check_status=True)
    np.testing.assert_array_equal(dt.cpu().numpy(), oracle.ngram_update(t, K, h, lens)["table"])


def test_bad_length_reports_and_changes_nothing(dev):
    t = ngram_table.empty(5)
    dt = torch.from_numpy(t).to(dev)
    h = torch.zeros(3, 6, dtype=torch.int32, device=dev)
    with pytest.raises(a11spec.A11Error):
        ngram_update(dt, h, torch.tensor([6, 7, 2], dtype=torch.int32, device=dev), 5, check_status=True)
    assert torch.equal(dt.cpu(), torch.from_numpy(t))


def test_accept_then_learn_then_draft(dev):
    """Committed tokens become drafts: after learning the accepted paths, the
    drafter proposes them from the same context."""
    K, V, B, N = 10, 4096, 4, 16
    t = ngram_table.empty(K, 4)
    dt = torch.from_numpy(t).to(dev)
    last = torch.tensor([[1, 2], [3, 4], [5, 6], [7, 8]], dtype=torch.int32, device=dev)
    acc = torch.full((B, N), -1, dtype=torch.int32, device=dev)
    acc[:, :3] = torch.tensor([[100, 101, 102], [200, 201, 202], [300, 301, 302], [400, 401, 402]],
                              dtype=torch.int32, device=dev)
    alen = torch.tensor([3, 2, 1, 0], dtype=torch.int32, device=dev)
    bonus = torch.tensor([900, 901, 902, 903], dtype=torch.int32, device=dev)
    hist, lens = history_from_accept(last, acc, alen, bonus)
    ngram_update(dt, hist, lens, K, check_status=True)
    r = oracle.ngram_update(t, K, hist.cpu().numpy(), lens.cpu().numpy())
    np.testing.assert_array_equal(dt.cpu().numpy(), r["table"])
    tk, pa, de, nn = a11spec.ngram_expand(dt, last, 1, 1, 4, N)
    torch.cuda.synchronize()
    want = [[100, 101, 102, 900], [200, 201, 901], [300, 902], [903]]
    for b in range(B):
        assert tk[b, 1:1 + len(want[b])].tolist() == want[b], (b, tk[b].tolist())


@pytest.mark.parametrize("with_history", [True, False])
def test_next_roots_matches_host_ops(dev, with_history):
    """a11s_next_roots gives the same next root pair and committed-token rows as
    the torch composition it replaces (history_from_accept, gather/where), for
    accept lengths 0..N, and bonus -1 (nothing drawn) included."""
    g = torch.Generator().manual_seed(5)
    B, N, V = 37, 16, 5000
    alen = torch.randint(0, N + 1, (B,), generator=g, dtype=torch.int32)
    alen[:3] = torch.tensor([0, N, 1], dtype=torch.int32)
    acc = torch.randint(0, V, (B, N), generator=g, dtype=torch.int32)
    acc[torch.arange(N).unsqueeze(0) >= alen.unsqueeze(1)] = -1  # a11s_accept's layout: -1 past accept_len
    bonus = torch.randint(-1, V, (B,), generator=g, dtype=torch.int32)
    tree = torch.randint(0, V, (B, N), generator=g, dtype=torch.int32)
    last = torch.randint(0, V, (B, 2), generator=g, dtype=torch.int32)
    acc, alen, bonus, tree, last_d = (t.to(dev) for t in (acc, alen, bonus, tree, last))
    want_hist, want_len = history_from_accept(last_d, acc, alen, bonus)
    idx = (alen.long() - 1).clamp_min(0).unsqueeze(1)
    want_last = torch.stack([torch.where(alen > 0, acc.gather(1, idx).squeeze(1), tree[:, 0]),
                             bonus.clamp_min(0)], dim=1)
    hist = (torch.full((B, N + 3), 7, dtype=torch.int32, device=dev), torch.zeros(B, dtype=torch.int32, device=dev))
    a11spec.next_roots(tree, acc, alen, bonus, last_d, history=hist if with_history else None)
    torch.cuda.synchronize()
    assert torch.equal(last_d, want_last)
    if with_history:
        assert torch.equal(hist[0], want_hist)
        assert torch.equal(hist[1], want_len)
