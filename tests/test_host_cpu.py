"""Host-side logic without a GPU: the paged-KV block tables (the reference's
tests/test_paged_kv_cache.cpp scenarios), the reference-compatible uniform
stream, batch sharding."""
import json
import os

import numpy as np
import pytest

from a11spec import distributed as D
from a11spec.kv_pages import KVCacheConfig, PagedKVCacheManager
from a11spec.verifier import SpecConfig, TreeNode, reference_uniforms, SPEC_K, BLOCK_TOKENS

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def mgr(**kw):
    cfg = KVCacheConfig(**kw)
    return PagedKVCacheManager(cfg, allocate_pool=False)


def test_block_rollover_16_17():  # reference test_paged_kv_cache.cpp:5-38
    m = mgr(num_layers=8, head_dim=64, max_sequences=16, vram_cap_gb=1)
    assert len(m.allocate_sequence(0)) == 1 and m.used_blocks() == 1 and m.total_tokens() == 0
    for _ in range(15):
        m.append_token(0)
    assert m.used_blocks() == 1 and m.total_tokens() == 15
    m.append_token(0)
    assert m.used_blocks() == 1 and m.total_tokens() == 16 and len(m.get_block_table(0)) == 1
    m.append_token(0)
    assert m.used_blocks() == 2 and len(m.get_block_table(0)) == 2


def test_free_and_reallocate():  # :41-61
    m = mgr(num_layers=4, head_dim=32, max_sequences=8, vram_cap_gb=1)
    m.allocate_sequence(0)
    m.free_sequence(0)
    assert m.used_blocks() == 0
    assert len(m.allocate_sequence(0)) == 1 and m.used_blocks() == 1


def test_cap_enforcement():  # :63-86
    m = mgr(num_layers=2, head_dim=32, max_sequences=64, vram_cap_gb=1e-4)
    n = 0
    with pytest.raises(RuntimeError):
        while True:
            m.allocate_sequence(n)
            n += 1
    assert n > 0 and m.used_blocks() == n


def test_fragmentation_and_reuse():  # :88-117
    m = mgr(num_layers=4, head_dim=64, max_sequences=16, vram_cap_gb=1)
    for s in range(3):
        m.allocate_sequence(s)
        for _ in range(48):
            m.append_token(s)
    assert m.used_blocks() == 9 and m.total_tokens() == 144
    m.free_sequence(1)
    assert m.used_blocks() == 6 and m.total_tokens() == 96
    assert len(m.allocate_sequence(3)) == 1 and m.used_blocks() == 7


def test_usage_bytes():  # :119-136, bf16 pool with one KV head
    m = mgr(num_layers=2, head_dim=32, max_sequences=8, vram_cap_gb=1)
    assert m.vram_usage_bytes() == 0
    m.allocate_sequence(0)
    assert m.vram_usage_bytes() == 2 * 32 * BLOCK_TOKENS * 2 * 2


def test_tree_reservation_and_compaction_commit():
    m = mgr(num_layers=1, head_dim=8, max_sequences=2, vram_cap_gb=1e-3)
    m.allocate_sequence(0)
    m.append_tokens(0, 30)
    L = m.reserve_tree(0, 20)  # tree slots 30..49 -> 4 pages
    assert L == 30 and len(m.get_block_table(0)) == 4
    bt = m.get_block_table(0)
    freed = np.full((1, 8), -1, np.int32)
    freed[0, 0] = bt[3]
    used = m.used_blocks()
    m.commit_compaction([0], [33], freed, [1])  # 2 drafts accepted + root
    assert m.num_tokens(0) == 33 and m.get_block_table(0) == bt[:3] and m.used_blocks() == used - 1


def test_reference_uniform_stream_golden():
    g = json.load(open(os.path.join(ROOT, "tests", "golden", "ref_chains.json")))
    u = np.asarray(g["uniform_stream"], np.float32)
    import threading
    out = {}
    t = threading.Thread(target=lambda: out.setdefault("u", reference_uniforms(len(u))))
    t.start()
    t.join()  # a fresh thread starts the stream at its beginning, as the reference's thread_local
    np.testing.assert_array_equal(out["u"], u)


def test_interface_defaults():  # python_bindings.cpp constants, test_python_bindings.py:177-195
    cfg = SpecConfig()
    assert (cfg.max_draft_depth, cfg.vocab_size, cfg.acceptance_threshold, cfg.log_diagnostics) == (8, 32000, 1.0, True)
    assert TreeNode().parent_idx == 0xFFFFFFFF and SPEC_K == 8 and BLOCK_TOKENS == 16


@pytest.mark.parametrize("gb,world", [(256, 8), (10, 3), (3, 4)])
def test_shard_partition(gb, world):
    spans = [D.shard(gb, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == gb
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    assert max(s[1] - s[0] for s in spans) - min(s[1] - s[0] for s in spans) <= 1


def test_attention_split_planner_picks():
    """The split planner (waves x (blocks per split + 12)) as seen through the
    workspace size, on the 148-SM count it assumes without a device: the C5
    and C4 batches run unsplit (header only), one long sequence splits 18 ways
    and eight split 2 ways (partials of B x N x Hq x (D + 2) floats per split)."""
    import a11spec
    f = a11spec.ops.tree_attention_workspace_bytes
    per_split = lambda B: B * 64 * 32 * (128 + 2) * 4
    assert f(32, 64, 32, 4, 128, 32768 + 128) == 256
    assert f(16, 64, 32, 4, 128, 4096 + 64) == 256
    assert f(1, 64, 32, 4, 128, 32832) == 256 + 18 * per_split(1)
    assert f(8, 64, 32, 4, 128, 32832) == 256 + 2 * per_split(8)
