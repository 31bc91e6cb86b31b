"""K7, the tree-node LM head (a11s_lm_head), and the acceptance that takes its
chunk records from the head's chunk keys (a11s_accept_recorded).

The head restates `logits = torch.matmul(h_norm, output_w.t())` of
engine/pipeline.py:471 for every tree node at once (and, with a scale, the
1/sqrt(hidden_dim) form of tree_forward_pass_kernel, src/cuda/tree_verification.cu:34-68).
Its logits are checked element by element against the fp32 product:
|got - ref| <= 2^-8 |ref| + 1e-3 max|ref row| (one bf16 rounding, 2^-9 relative,
plus fp32 summation-order differences). Its chunk keys must equal, bit for bit,
the maximum and first position recomputed from the logits it wrote; and the
recorded acceptance must reproduce a11s_accept on the same logits exactly
(decisions, tokens, bonus, node probabilities, counters)."""
import ctypes as C

import numpy as np
import pytest
import torch

import a11spec
from a11spec import _lib, ops
from a11spec import workloads as W

pytestmark = pytest.mark.gpu
V5, H5 = 151936, 2048  # the C5 LM head: vocabulary and hidden size


def _bound_ok(got, h, w, scale):
    ref = (h.float() @ w.float().t()) * scale
    err = (got.float() - ref).abs()
    tol = 2.0 ** -8 * ref.abs() + 1e-3 * ref.abs().amax(-1, keepdim=True)
    worst = float((err / tol.clamp_min(1e-30)).max())
    return worst <= 1.0, worst


def _keys_from_logits(lg):
    """(maximum, first position) per 2048-token chunk of bf16 logits [R, V]: -0 as +0."""
    R, V = lg.shape
    nch = (V + 2047) // 2048
    x = lg.float()
    pad = nch * 2048 - V
    if pad:
        x = torch.cat([x, torch.full((R, pad), float("-inf"), device=x.device)], 1)
    x = x.view(R, nch, 2048)
    x = torch.where(x == 0, torch.zeros_like(x), x)
    mx = x.amax(-1)
    first = (x == mx[..., None]).to(torch.int8).argmax(-1)
    return mx, first


def _decode(keys):
    o = (keys >> 32) & 0xFFFF
    h = torch.where(o >= 0x8000, o & 0x7FFF, (~o) & 0xFFFF).to(torch.int32)
    val = (h << 16).view(torch.float32)
    pos = 0xFFFFFFFF - (keys & 0xFFFFFFFF)
    return val, pos


def _check_keys(lg, keys):
    mx, first = _keys_from_logits(lg)
    val, pos = _decode(keys)
    assert torch.equal(val, mx)
    assert torch.equal(pos, first)


@pytest.mark.parametrize("rows,H,V,scale,stride", [
    (5, 64, 256, 1.0, None),          # one tile
    (130, 136, 2056, 1.0, None),      # ragged rows, K not a multiple of 64, a chunk of 8 columns
    (300, 256, 4104, 0.125, 4120),    # scaled, padded rows (the padding stays untouched)
    (257, H5, V5, 1.0, None),         # the C5 vocabulary
])
def test_lm_head_numerics_and_keys(dev, rows, H, V, scale, stride):
    g = torch.Generator(device="cuda").manual_seed(rows + V)
    h = (0.5 * torch.randn(rows, H, device="cuda", generator=g)).to(torch.bfloat16)
    w = (0.05 * torch.randn(V, H, device="cuda", generator=g)).to(torch.bfloat16)
    full = None
    out = None
    if stride is not None:
        full = torch.full((rows, stride), 7.0, dtype=torch.bfloat16, device="cuda")
        out = full[:, :V]
    lg, keys, ws = ops.lm_head(h, w, out=out, want_keys=True, scale=scale)
    assert ops.read_status(ws)[0] == _lib.OK
    ok, worst = _bound_ok(lg, h, w, scale)
    assert ok, worst
    _check_keys(lg, keys)
    if full is not None:
        assert bool((full[:, V:] == 7.0).all())


def test_lm_head_signed_zero_and_negative_rows(dev):
    """Zero rows under a negative scale give -0 everywhere: the key's maximum
    is zero at position 0. Rows whose logits are all negative keep their
    least negative value and its first position."""
    g = torch.Generator(device="cuda").manual_seed(11)
    rows, H, V = 64, 128, 4096
    h = (0.5 * torch.randn(rows, H, device="cuda", generator=g)).abs().to(torch.bfloat16)
    h[:8] = 0
    w = (0.05 * torch.randn(V, H, device="cuda", generator=g)).abs().to(torch.bfloat16)
    lg, keys, _ = ops.lm_head(h, w, want_keys=True, scale=-1.0)
    torch.cuda.synchronize()
    assert bool((lg[:8].view(torch.int16) == -32768).all())  # -0 bit patterns
    assert bool((lg[8:].float() <= 0).all())
    _check_keys(lg, keys)
    val, pos = _decode(keys[:8])
    assert bool((val == 0).all()) and bool((pos == 0).all())


def _peaked_rows(w, tok, gen, strength=16.0):
    """Hidden rows whose logits peak at the given tokens (row r ~ strength * w[tok[r]] + noise): a logit
    of about 16 against about 0 for the rest, so p(token) is close to 1 at T = 0.7."""
    wt = w[tok].float()
    wt = wt / wt.norm(dim=-1, keepdim=True)
    noise = 0.02 * torch.randn(wt.shape, device="cuda", generator=gen)
    return (strength * wt + noise).to(torch.bfloat16)


@pytest.fixture(scope="module")
def head_weight():
    g = torch.Generator(device="cuda").manual_seed(5)
    return (torch.randn(V5, H5, device="cuda", generator=g) / H5 ** 0.5).to(torch.bfloat16)


def _tree_batch(w, B, N, seed, p_force=0.5):
    """Random trees; a forced node's token is drawn first and its parent row made
    to peak at it, so greedy walks and likely samples go deep."""
    rng = np.random.default_rng(seed)
    parents = np.stack([W.random_parents(N, rng) for _ in range(B)])
    tokens = rng.integers(0, V5, size=(B, N)).astype(np.int32)
    gen = torch.Generator(device="cuda").manual_seed(seed)
    h = (torch.randn(B * N, H5, device="cuda", generator=gen) / 4).to(torch.bfloat16)
    force = rng.random((B, N)) < p_force
    force[:, 0] = False
    rows, toks = [], []
    for b in range(B):
        for i in range(1, N):
            if force[b, i]:
                rows.append(b * N + int(parents[b, i]))
                toks.append(int(tokens[b, i]))
    if rows:
        # several forced children of one parent: the last one wins the peak
        h[torch.tensor(rows, device="cuda")] = _peaked_rows(w, torch.tensor(toks, device="cuda"), gen)
    return (h, torch.as_tensor(parents, device="cuda"), torch.as_tensor(tokens, device="cuda"),
            torch.full((B,), N, dtype=torch.int32, device="cuda"))


def _accept_both(mode, lg3, keys, tokens, parents, n_nodes, temperature=1.0, seed=0):
    B, N, _ = lg3.shape
    uni = None
    if mode != _lib.GREEDY:
        uni = torch.rand(B, N, generator=torch.Generator(device="cuda").manual_seed(seed), device="cuda")
    s0 = torch.zeros(_lib.STATS_LEN, dtype=torch.int64, device="cuda")
    s1 = torch.zeros_like(s0)
    r0 = ops.accept(mode, lg3, tokens, parents, n_nodes, temperature=temperature, uniforms=uni, stats=s0,
                    want_node_probs=mode != _lib.GREEDY)
    r1 = ops.accept(mode, lg3, tokens, parents, n_nodes, temperature=temperature, uniforms=uni, stats=s1,
                    want_node_probs=mode != _lib.GREEDY, keys=keys)
    assert ops.read_status(r0.workspace) == ops.read_status(r1.workspace)
    assert torch.equal(r0.accept_len, r1.accept_len)
    for a, b in ((r0.accepted_nodes, r1.accepted_nodes), (r0.accepted_tokens, r1.accepted_tokens),
                 (r0.bonus, r1.bonus), (s0, s1)):
        assert torch.equal(a, b)
    if mode != _lib.GREEDY:
        assert torch.equal(r0.node_probs.view(torch.int32), r1.node_probs.view(torch.int32))
    return r0


@pytest.mark.parametrize("mode", [_lib.GREEDY, _lib.STOCH_ONEHOT])
def test_recorded_accept_matches_accept(dev, head_weight, mode):
    B, N = 8, 32
    h, parents, tokens, n_nodes = _tree_batch(head_weight, B, N, seed=21 + mode)
    lg, keys, ws = ops.lm_head(h, head_weight, want_keys=True)
    assert ops.read_status(ws)[0] == _lib.OK
    r = _accept_both(mode, lg.view(B, N, V5), keys, tokens, parents, n_nodes, temperature=0.7, seed=3)
    assert int(r.accept_len.max()) >= 2  # the walks leave the root


@pytest.mark.parametrize("mode", [_lib.GREEDY, _lib.STOCH_ONEHOT])
def test_recorded_accept_ragged_trees(dev, head_weight, mode):
    """Sequences with fewer live nodes than max_nodes: the dead rows' keys (of
    whatever the head computed for them) take no part, as their logits do not
    in a11s_accept."""
    B, N = 12, 24
    h, parents, tokens, _ = _tree_batch(head_weight, B, N, seed=31 + mode)
    n_nodes = torch.tensor([N if b % 3 == 0 else 1 + (7 * b) % N for b in range(B)], dtype=torch.int32,
                           device="cuda")
    lg, keys, _ = ops.lm_head(h, head_weight, want_keys=True)
    _accept_both(mode, lg.view(B, N, V5), keys, tokens, parents, n_nodes, temperature=0.7, seed=5)


def test_recorded_accept_c5_shape(dev, head_weight):
    """The bench's acceptance: one-hot drafts at T = 0.7 on [32, 64, 151936] bf16 logits."""
    B, N = 32, 64
    h, parents, tokens, n_nodes = _tree_batch(head_weight, B, N, seed=55)
    lg, keys, _ = ops.lm_head(h, head_weight, want_keys=True)
    _check_keys(lg, keys)
    r = _accept_both(_lib.STOCH_ONEHOT, lg.view(B, N, V5), keys, tokens, parents, n_nodes, temperature=0.7, seed=9)
    assert int(r.accept_len.max()) >= 2
    r = _accept_both(_lib.GREEDY, lg.view(B, N, V5), keys, tokens, parents, n_nodes)
    assert int(r.accept_len.max()) >= 2


def test_recorded_accept_reports_nonfinite(dev, head_weight):
    """A NaN in one node's hidden state makes that row's logits NaN: both paths report ENONFINITE for it."""
    B, N = 2, 8
    h, parents, tokens, n_nodes = _tree_batch(head_weight, B, N, seed=77)
    h[N + 3, 5] = float("nan")
    lg, keys, _ = ops.lm_head(h, head_weight, want_keys=True)
    for mode in (_lib.GREEDY, _lib.STOCH_ONEHOT):
        uni = torch.rand(B, N, device="cuda") if mode else None
        r0 = ops.accept(mode, lg.view(B, N, V5), tokens, parents, n_nodes, temperature=0.7, uniforms=uni)
        r1 = ops.accept(mode, lg.view(B, N, V5), tokens, parents, n_nodes, temperature=0.7, uniforms=uni, keys=keys)
        assert ops.read_status(r0.workspace) == (_lib.ENONFINITE, 1)
        assert ops.read_status(r1.workspace) == (_lib.ENONFINITE, 1)


def test_recorded_accept_argument_checks(dev):
    lib = _lib.lib
    B, N, V = 1, 2, 4096
    lg = torch.zeros(B, N, V, dtype=torch.bfloat16, device="cuda")
    i32 = torch.zeros(B, N, dtype=torch.int32, device="cuda")
    ws = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    keys = torch.zeros(B * N, 2, dtype=torch.int64, device="cuda")
    args = lambda mode, k: (mode, lg.data_ptr(), V, C.c_float(1.0), i32.data_ptr(), i32.data_ptr(), i32.data_ptr(),
                            None, B, N, V, k, i32.data_ptr(), i32.data_ptr(), i32.data_ptr(), i32.data_ptr(), None,
                            None, ws.data_ptr(), ws.numel(), None)
    assert lib.a11s_accept_recorded(*args(_lib.STOCH_DRAFT, keys.data_ptr())) == _lib.EUNSUPPORTED
    assert lib.a11s_accept_recorded(*args(_lib.GREEDY, None)) == _lib.EINVAL
    assert lib.a11s_lm_head(lg.data_ptr(), lg.data_ptr(), 2, 12, V, C.c_float(1.0), lg.data_ptr(), V, None,
                            ws.data_ptr(), ws.numel(), None) == _lib.EINVAL  # hidden_dim not a multiple of 8
