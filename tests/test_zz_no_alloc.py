"""a11s_accept_static: the acceptance entry point for callers that cannot
allocate device memory (their HBM belongs to another allocator, or they bind
the library from a language without a device allocator), so its scratch is a
fixed array inside the library instead of a caller workspace.

Checked through the C ABI against a11s_accept on the same inputs, on two calls
in a row (the array keeps the previous call's contents, which must not leak
into the next result). Decisions are bit-exact, like every acceptance test.
This file is collected last so a stop-at-first-failure run has already run
every other test; it also passes alone in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import a11spec
from a11spec import _lib

pytestmark = pytest.mark.gpu


def _bind():
    f = _lib.lib.a11s_accept_static
    vp, i32, i64, f32 = C.c_void_p, C.c_int32, C.c_int64, C.c_float
    f.argtypes = [i32, i32, vp, vp, i64, f32, vp, vp, vp, vp, i32, i32, i32, vp, vp, vp, vp, vp,
                  vp, vp, vp]
    f.restype = C.c_int
    return f


def _case(seed, B, N, V, dtype):
    g = torch.Generator(device="cuda").manual_seed(seed)
    logits = (2 * torch.randn(B, N, V, generator=g, device="cuda")).to(dtype)
    parents = torch.empty(B, N, dtype=torch.int32, device="cuda")
    parents[:, 0] = -1
    for i in range(1, N):  # breadth-first 4/2 tree
        parents[:, i] = (i - 1) // 4 if i <= 4 else 1 + (i - 5) // 2
    # likely tokens so that some drafts get accepted
    top = logits.float().topk(3, dim=-1).indices
    pick = torch.randint(0, 3, (B, N), generator=g, device="cuda")
    rows = top.gather(2, pick.unsqueeze(-1)).squeeze(-1)
    tokens = rows.gather(1, parents.clamp_min(0).long()).int()
    n_nodes = torch.full((B,), N, dtype=torch.int32, device="cuda")
    n_nodes[1] = N // 2
    uni = torch.rand(B, N, generator=g, device="cuda")
    return logits, tokens.contiguous(), parents, n_nodes, uni


def _static(f, mode, logits, tokens, parents, n_nodes, uni, T, stats):
    B, N, V = logits.shape
    out = a11spec.ops.alloc_accept(mode, B, N, V, "cuda", want_node_probs=True)
    status = torch.full((2,), -7, dtype=torch.int32, device="cuda")
    rc = f(mode, _lib.BF16 if logits.dtype == torch.bfloat16 else _lib.F32, logits.data_ptr(), None, V,
           T, uni.data_ptr(), tokens.data_ptr(), parents.data_ptr(), n_nodes.data_ptr(), B, N, V,
           out.accept_len.data_ptr(), out.accepted_nodes.data_ptr(), out.accepted_tokens.data_ptr(),
           out.bonus.data_ptr(), out.node_probs.data_ptr(), stats.data_ptr(), status.data_ptr(),
           torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.lib.a11s_last_error()
    return out, status


@pytest.mark.parametrize("mode,dtype", [(_lib.STOCH_ONEHOT, torch.bfloat16), (_lib.GREEDY, torch.float32)])
def test_static_scratch_matches_workspace_entry_point(dev, mode, dtype):
    f = _bind()
    for call, seed in enumerate((11, 12)):  # two calls in a row on the same array
        logits, tokens, parents, n_nodes, uni = _case(seed, 8, 64, 151936, dtype)
        st_ref = torch.zeros(6, dtype=torch.int64, device="cuda")
        st_fix = torch.zeros(6, dtype=torch.int64, device="cuda")
        ref = a11spec.accept(mode, logits, tokens, parents, n_nodes, temperature=0.7, uniforms=uni,
                             stats=st_ref, want_node_probs=True, check_status=True)
        got, status = _static(f, mode, logits, tokens, parents, n_nodes, uni, 0.7, st_fix)
        torch.cuda.synchronize()
        assert status.tolist() == [0, 0], (call, status.tolist())
        assert torch.equal(got.accept_len, ref.accept_len), call
        assert torch.equal(got.accepted_nodes, ref.accepted_nodes), call
        assert torch.equal(got.accepted_tokens, ref.accepted_tokens), call
        assert torch.equal(got.bonus, ref.bonus), call
        if mode != _lib.GREEDY:
            assert torch.equal(got.node_probs, ref.node_probs), call
        assert torch.equal(st_fix, st_ref), call


def _compare_at(f, mode, B, N, V, seed):
    """One call of each entry point on the same inputs; bit-exact results."""
    logits, tokens, parents, n_nodes, uni = _case(seed, B, N, V, torch.bfloat16)
    draft = None
    if mode == _lib.STOCH_DRAFT:
        g = torch.Generator(device="cuda").manual_seed(seed + 100)
        draft = (logits.float() + 0.5 * torch.randn(logits.shape, generator=g, device="cuda")).to(torch.bfloat16)
    st_ref = torch.zeros(6, dtype=torch.int64, device="cuda")
    st_fix = torch.zeros(6, dtype=torch.int64, device="cuda")
    ref = a11spec.accept(mode, logits, tokens, parents, n_nodes, draft_logits=draft, temperature=0.8,
                         uniforms=uni, stats=st_ref, want_node_probs=True, check_status=True)
    out = a11spec.ops.alloc_accept(mode, B, N, V, "cuda", want_node_probs=True)
    status = torch.full((2,), -7, dtype=torch.int32, device="cuda")
    rc = f(mode, _lib.BF16, logits.data_ptr(), None if draft is None else draft.data_ptr(), V, 0.8,
           uni.data_ptr(), tokens.data_ptr(), parents.data_ptr(), n_nodes.data_ptr(), B, N, V,
           out.accept_len.data_ptr(), out.accepted_nodes.data_ptr(), out.accepted_tokens.data_ptr(),
           out.bonus.data_ptr(), out.node_probs.data_ptr(), st_fix.data_ptr(), status.data_ptr(),
           torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.lib.a11s_last_error()
    torch.cuda.synchronize()
    assert status.tolist() == [0, 0], status.tolist()
    for name in ("accept_len", "accepted_nodes", "accepted_tokens", "bonus"):
        assert torch.equal(getattr(out, name), getattr(ref, name)), name
    if mode != _lib.GREEDY:
        assert torch.equal(out.node_probs, ref.node_probs)
    assert torch.equal(st_fix, st_ref)
    return ref


def _largest_batch(mode, N, V):
    limit = 4 << 20
    B = 1
    while a11spec.ops.accept_workspace_bytes(mode, B + 1, N, V) <= limit:
        B += 1
    return B


def test_static_scratch_draft_logits_two_calls(dev):
    """Sampling against draft logits uses two row sets and both roots' sums."""
    f = _bind()
    for seed in (21, 22):
        _compare_at(f, _lib.STOCH_DRAFT, 6, 64, 151936, seed)


@pytest.mark.parametrize("mode", [_lib.GREEDY, _lib.STOCH_ONEHOT, _lib.STOCH_DRAFT])
def test_static_scratch_full_array_and_one_more(dev, mode):
    """The largest batch whose workspace fits the 4 MiB array uses its top end
    and still matches a11s_accept; one sequence more is refused with ENOSPACE
    and names the largest batch."""
    f = _bind()
    N, V = 64, 151936
    B = _largest_batch(mode, N, V)
    assert a11spec.ops.accept_workspace_bytes(mode, B, N, V) > 0.95 * (4 << 20)  # the top end of the array
    _compare_at(f, mode, B, N, V, seed=31 + mode)
    z = torch.zeros(1, dtype=torch.int32, device="cuda")
    logits = torch.zeros(8, dtype=torch.bfloat16, device="cuda")  # never read
    rc = f(mode, _lib.BF16, logits.data_ptr(), logits.data_ptr(), V, 1.0, z.data_ptr(), z.data_ptr(),
           z.data_ptr(), None, B + 1, N, V, z.data_ptr(), z.data_ptr(), z.data_ptr(), z.data_ptr(), None,
           None, None, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.ENOSPACE
    assert f"at most {B} sequences".encode() in _lib.lib.a11s_last_error()


def test_static_scratch_empty_batch_writes_status(dev):
    f = _bind()
    status = torch.full((2,), -7, dtype=torch.int32, device="cuda")
    z = torch.zeros(1, dtype=torch.int32, device="cuda")
    logits = torch.zeros(8, dtype=torch.float32, device="cuda")
    rc = f(_lib.GREEDY, _lib.F32, logits.data_ptr(), None, 8, 1.0, None, z.data_ptr(), z.data_ptr(), None,
           0, 4, 8, z.data_ptr(), z.data_ptr(), z.data_ptr(), z.data_ptr(), None, None, status.data_ptr(),
           torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.lib.a11s_last_error()
    torch.cuda.synchronize()
    assert status.tolist() == [0, 0]


def test_static_scratch_rejects_oversize_without_launching(dev):
    f = _bind()
    B, N, V = 65536, 64, 151936  # 65536 sequences x 75 root-row chunk records of 4 B > 4 MiB
    need = a11spec.ops.accept_workspace_bytes(_lib.GREEDY, B, N, V)
    assert need > (4 << 20)
    logits = torch.zeros(1, dtype=torch.float32, device="cuda")  # never read
    z = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = f(_lib.GREEDY, _lib.F32, logits.data_ptr(), None, V, 1.0, None, z.data_ptr(), z.data_ptr(),
           None, B, N, V, z.data_ptr(), z.data_ptr(), z.data_ptr(), z.data_ptr(), None, None, None,
           torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.ENOSPACE
    assert b"fixed array" in _lib.lib.a11s_last_error()
