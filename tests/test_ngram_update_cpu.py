"""K6 without a GPU: the table-update rule in the oracle on crafted buckets,
learning a repeated phrase until the n-gram drafter (K1's oracle) proposes it,
the on-disk table format, and the host helper that turns acceptance results
into history rows."""
import numpy as np
import pytest
import torch

import oracle
from a11spec import ngram_table
from a11spec.ops import history_from_accept

OK, EBOUNDS = 0, 2
K = 6


def _bucket_rows(table, x, y):
    return table[oracle.ngram_bucket(x, y, K)]


def test_update_rule_increment_fill_evict():
    t = ngram_table.empty(K, slots=3)
    h = np.array([[5, 6, 7, 5, 6, 7, 5, 6, 8, 5, 6, 9, 5, 6, 10]], np.int32)
    r = oracle.ngram_update(t, K, h, [15])
    assert r["status"] == OK
    b = _bucket_rows(r["table"], 5, 6)
    # (5,6)->7 twice, ->8 once, ->9 once fill the three slots in order; ->10 evicts the lowest count
    # among (7:2, 8:1, 9:1): slot 1 (8) is the lowest index with the smallest count
    assert b.tolist() == [[7, 2], [10, 1], [9, 1]]


def test_update_saturates_and_skips_negative_tokens():
    t = ngram_table.empty(K, slots=2)
    bk = oracle.ngram_bucket(1, 2, K)
    t[bk, 0] = [3, 2**31 - 1]
    r = oracle.ngram_update(t, K, np.array([[1, 2, 3, -1, 2, 3]], np.int32), [6])
    assert r["table"][bk].tolist() == [[3, 2**31 - 1], [-1, 0]] and r["detail"] == 1


def test_update_bad_length_changes_nothing():
    t = ngram_table.empty(K)
    r = oracle.ngram_update(t, K, np.array([[1, 2, 3], [4, 5, 6]], np.int32), [3, 4])
    assert r["status"] == EBOUNDS and r["detail"] == 1 and np.array_equal(r["table"], t)


def test_learned_phrase_is_drafted():
    t = ngram_table.empty(10, slots=4)
    phrase = [11, 22, 33, 44, 55]
    h = np.array([phrase * 6], np.int32)
    t = oracle.ngram_update(t, 10, h, [h.shape[1]])["table"]
    d = oracle.ngram_expand(t, 10, np.array([[11, 22]], np.int32), 2, 2, 3, 8)
    # the chain 33 -> 44 -> 55 is the top continuation at every level
    assert d["tokens"][0, 1] == 33
    kids = {int(d["tokens"][0, i]) for i in range(d["n_nodes"][0]) if d["parents"][0, i] == 1}
    assert 44 in kids


def test_table_file_round_trip(tmp_path):
    rng = np.random.default_rng(1)
    t = rng.integers(-1, 1000, (1 << 7, 5, 2)).astype(np.int32)
    p = str(tmp_path / "t.a11ng")
    ngram_table.save(p, t, 7)
    back, k = ngram_table.load(p)
    assert k == 7 and np.array_equal(back, t)
    raw = open(p, "rb").read()
    open(p, "wb").write(b"NOTATABL" + raw[8:])
    with pytest.raises(ValueError):
        ngram_table.load(p)
    open(p, "wb").write(raw[:100])
    with pytest.raises(ValueError):
        ngram_table.load(p)


def test_history_from_accept_rows():
    last = torch.tensor([[1, 2], [3, 4]], dtype=torch.int32)
    acc = torch.tensor([[7, 8, -1], [-1, -1, -1]], dtype=torch.int32)
    hist, lens = history_from_accept(last, acc, torch.tensor([2, 0], dtype=torch.int32),
                                     torch.tensor([9, 6], dtype=torch.int32))
    assert lens.tolist() == [5, 3]
    assert hist[0, :5].tolist() == [1, 2, 7, 8, 9] and hist[1, :3].tolist() == [3, 4, 6]
