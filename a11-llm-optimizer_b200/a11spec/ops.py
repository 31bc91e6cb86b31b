"""Torch-facing wrappers of the C-ABI entry points.

Every function takes CUDA tensors, launches on the current torch stream and
returns without synchronising (unless ``check_status=True``, which reads the
device status word and raises on a device-side error). Workspaces come from
torch's caching allocator unless the caller passes one.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from ._lib import A11Error, check, lib


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _need(t: torch.Tensor, name: str, dtype=None, device=None):
    if not t.is_cuda:
        raise A11Error(_lib.EINVAL, f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise A11Error(_lib.EINVAL, f"{name} must be contiguous")
    if dtype is not None and t.dtype != dtype:
        raise A11Error(_lib.EINVAL, f"{name} must be {dtype}, got {t.dtype}")


def read_status(workspace: torch.Tensor):
    """(code, detail) of the device status word; synchronises the stream."""
    st, de = _lib.C.c_int32(0), _lib.C.c_int32(0)
    check(lib.a11s_read_status(workspace.data_ptr(), _lib.C.byref(st), _lib.C.byref(de), _stream()))
    return int(st.value), int(de.value)


def raise_on_status(workspace: torch.Tensor) -> None:
    code, detail = read_status(workspace)
    if code != _lib.OK:
        raise A11Error(code, f"device status (detail {detail})")


def workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


# --------------------------------------------------------------------------- K3
@dataclass
class AcceptResult:
    accept_len: torch.Tensor       # int32 [B]
    accepted_nodes: torch.Tensor   # int32 [B, N]
    accepted_tokens: torch.Tensor  # int32 [B, N]
    bonus: torch.Tensor            # int32 [B]
    node_probs: Optional[torch.Tensor]
    workspace: torch.Tensor


def accept_workspace_bytes(mode: int, batch: int, max_nodes: int, vocab: int) -> int:
    return int(lib.a11s_accept_workspace_bytes(mode, batch, max_nodes, vocab))


def alloc_accept(mode: int, batch: int, max_nodes: int, vocab: int, device,
                 want_node_probs: bool = False) -> AcceptResult:
    """Output buffers and workspace for repeated a11s_accept calls (pass as `out`)."""
    i32 = dict(dtype=torch.int32, device=device)
    return AcceptResult(
        accept_len=torch.empty(batch, **i32), accepted_nodes=torch.empty(batch, max_nodes, **i32),
        accepted_tokens=torch.empty(batch, max_nodes, **i32), bonus=torch.empty(batch, **i32),
        node_probs=torch.empty(batch, max_nodes, dtype=torch.float32, device=device) if want_node_probs else None,
        workspace=workspace(accept_workspace_bytes(mode, batch, max_nodes, vocab), device))


def accept(mode: int, target_logits: torch.Tensor, tokens: torch.Tensor, parents: torch.Tensor,
           n_nodes: Optional[torch.Tensor] = None, draft_logits: Optional[torch.Tensor] = None,
           temperature: float = 1.0, uniforms: Optional[torch.Tensor] = None,
           stats: Optional[torch.Tensor] = None, want_node_probs: bool = False,
           ws: Optional[torch.Tensor] = None, out: Optional[AcceptResult] = None,
           check_status: bool = False, keys: Optional[torch.Tensor] = None) -> AcceptResult:
    """K3. target_logits [B, N, V] (fp32 or bf16, rows contiguous).

    keys: the chunk keys of lm_head for these rows ([B * N, ceil(V / 2048)]
    int64): the records come from them instead of a pass over the logits
    (a11s_accept_recorded; GREEDY or STOCH_ONEHOT on bf16 logits)."""
    B, N, V = target_logits.shape
    dt = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16}.get(target_logits.dtype)
    if dt is None:
        raise A11Error(_lib.EINVAL, "logits must be float32 or bfloat16")
    _need(target_logits, "target_logits")
    _need(tokens, "tokens", torch.int32)
    _need(parents, "parents", torch.int32)
    if n_nodes is not None:
        _need(n_nodes, "n_nodes", torch.int32)
    if draft_logits is not None:
        _need(draft_logits, "draft_logits", target_logits.dtype)
        if draft_logits.shape != target_logits.shape:
            raise A11Error(_lib.EINVAL, "draft_logits shape differs from target_logits")
    if uniforms is not None:
        _need(uniforms, "uniforms", torch.float32)
    dev = target_logits.device
    if out is None:
        out = AcceptResult(
            accept_len=torch.empty(B, dtype=torch.int32, device=dev),
            accepted_nodes=torch.empty(B, N, dtype=torch.int32, device=dev),
            accepted_tokens=torch.empty(B, N, dtype=torch.int32, device=dev),
            bonus=torch.empty(B, dtype=torch.int32, device=dev),
            node_probs=torch.empty(B, N, dtype=torch.float32, device=dev) if want_node_probs else None,
            workspace=ws if ws is not None else workspace(accept_workspace_bytes(mode, B, N, V), dev))
    if keys is not None:
        _need(keys, "keys", torch.int64)
        if draft_logits is not None:
            raise A11Error(_lib.EUNSUPPORTED, "chunk keys cover the target rows only")
        rc = lib.a11s_accept_recorded(mode, target_logits.data_ptr(), V, float(temperature), _ptr(uniforms),
                                      tokens.data_ptr(), parents.data_ptr(), _ptr(n_nodes), B, N, V,
                                      keys.data_ptr(), out.accept_len.data_ptr(), out.accepted_nodes.data_ptr(),
                                      out.accepted_tokens.data_ptr(), out.bonus.data_ptr(),
                                      _ptr(out.node_probs), _ptr(stats), out.workspace.data_ptr(),
                                      out.workspace.numel(), _stream())
    else:
        rc = lib.a11s_accept(mode, dt, target_logits.data_ptr(), _ptr(draft_logits), V,
                             float(temperature), _ptr(uniforms), tokens.data_ptr(), parents.data_ptr(),
                             _ptr(n_nodes), B, N, V, out.accept_len.data_ptr(),
                             out.accepted_nodes.data_ptr(), out.accepted_tokens.data_ptr(),
                             out.bonus.data_ptr(), _ptr(out.node_probs), _ptr(stats),
                             out.workspace.data_ptr(), out.workspace.numel(), _stream())
    check(rc)
    if check_status:
        raise_on_status(out.workspace)
    return out


# --------------------------------------------------------------------------- K2
def tree_attention_workspace_bytes(batch, max_nodes, num_q_heads, num_kv_heads, head_dim, max_kv_len):
    return int(lib.a11s_tree_attention_workspace_bytes(batch, max_nodes, num_q_heads, num_kv_heads,
                                                       head_dim, max_kv_len))


def tree_attention(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                   page_table: torch.Tensor, ctx_lens: torch.Tensor, parents: torch.Tensor,
                   n_nodes: Optional[torch.Tensor] = None, scale: Optional[float] = None,
                   max_kv_len: Optional[int] = None, want_lse: bool = False,
                   out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None,
                   ws: Optional[torch.Tensor] = None, check_status: bool = False):
    """K2. q [B, N, Hq, D] bf16; pools [P, 16, Hkv, D] bf16; page_table [B, maxpages] int32."""
    B, N, Hq, D = q.shape
    P, pg, Hkv, D2 = k_pool.shape
    if pg != _lib.PAGE_TOKENS or D2 != D or v_pool.shape != k_pool.shape:
        raise A11Error(_lib.EINVAL, "pool shape must be [P, 16, Hkv, D] for K and V")
    for t, nm in ((q, "q"), (k_pool, "k_pool"), (v_pool, "v_pool")):
        _need(t, nm, torch.bfloat16)
    _need(page_table, "page_table", torch.int32)
    _need(ctx_lens, "ctx_lens", torch.int32)
    _need(parents, "parents", torch.int32)
    if max_kv_len is None:
        max_kv_len = page_table.shape[1] * _lib.PAGE_TOKENS
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    dev = q.device
    if out is None:
        out = torch.empty_like(q)
    if want_lse and lse is None:
        lse = torch.empty(B, N, Hq, dtype=torch.float32, device=dev)
    if ws is None:
        ws = workspace(tree_attention_workspace_bytes(B, N, Hq, Hkv, D, max_kv_len), dev)
    rc = lib.a11s_tree_attention(q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), P,
                                 page_table.data_ptr(), page_table.shape[1], ctx_lens.data_ptr(),
                                 parents.data_ptr(), _ptr(n_nodes), B, N, Hq, Hkv, D, int(max_kv_len),
                                 float(scale), out.data_ptr(), _ptr(lse), ws.data_ptr(), ws.numel(),
                                 _stream())
    check(rc)
    if check_status:
        raise_on_status(ws)
    return out, lse, ws


# --------------------------------------------------------------------------- K7
def lm_head_keys_bytes(rows: int, vocab: int) -> int:
    return int(lib.a11s_lm_head_keys_bytes(rows, vocab))


def lm_head(hidden: torch.Tensor, weight: torch.Tensor, out: Optional[torch.Tensor] = None,
            keys: Optional[torch.Tensor] = None, want_keys: bool = False, scale: float = 1.0,
            ws: Optional[torch.Tensor] = None, check_status: bool = False):
    """K7. hidden [..., H] bf16, weight [V, H] bf16 -> logits [..., V] bf16
    (out may be a view with a row stride >= V), and the chunk keys
    [rows, ceil(V / 2048)] int64 when want_keys (or keys) is given."""
    H = hidden.shape[-1]
    V, H2 = weight.shape
    if H2 != H:
        raise A11Error(_lib.EINVAL, "weight must be [vocab, hidden_dim]")
    _need(hidden, "hidden", torch.bfloat16)
    _need(weight, "weight", torch.bfloat16)
    rows = hidden.numel() // H
    dev = hidden.device
    if out is None:
        out = torch.empty(*hidden.shape[:-1], V, dtype=torch.bfloat16, device=dev)
    if out.dtype != torch.bfloat16 or out.device != dev or out.shape[-1] != V or out.stride(-1) != 1:
        raise A11Error(_lib.EINVAL, "out must be bf16 [..., vocab] with unit column stride on the device")
    row_stride = out.stride(-2) if out.dim() >= 2 else V
    if out.numel() and any(out.stride(d) != out.stride(d + 1) * out.shape[d + 1] for d in range(out.dim() - 2)):
        raise A11Error(_lib.EINVAL, "out rows must be evenly spaced")
    if keys is None and want_keys:
        keys = torch.empty(rows, (V + 2047) // 2048, dtype=torch.int64, device=dev)
    if keys is not None:
        _need(keys, "keys", torch.int64)
    if ws is None:
        ws = workspace(256, dev)
    rc = lib.a11s_lm_head(hidden.data_ptr(), weight.data_ptr(), rows, H, V, float(scale), out.data_ptr(),
                          int(row_stride), _ptr(keys), ws.data_ptr(), ws.numel(), _stream())
    check(rc)
    if check_status:
        raise_on_status(ws)
    return out, keys, ws


# --------------------------------------------------------------------------- K4
def kv_compact(k_pool: torch.Tensor, v_pool: torch.Tensor, page_table: torch.Tensor,
               seq_lens: torch.Tensor, accept_len: torch.Tensor, accepted_nodes: torch.Tensor,
               n_nodes: Optional[torch.Tensor] = None, num_layers: int = 1,
               freed_pages: Optional[torch.Tensor] = None, n_freed: Optional[torch.Tensor] = None,
               ws: Optional[torch.Tensor] = None, check_status: bool = False):
    """K4, in place on the pools, page_table and seq_lens.

    Pools are [P, 16, Hkv, D] (or [layers, P, 16, Hkv, D] with num_layers > 1).
    """
    for t, nm in ((page_table, "page_table"), (seq_lens, "seq_lens"), (accept_len, "accept_len"),
                  (accepted_nodes, "accepted_nodes")):
        _need(t, nm, torch.int32)
    _need(k_pool, "k_pool")
    _need(v_pool, "v_pool")
    B, N = accepted_nodes.shape
    shape = k_pool.shape[1:] if num_layers > 1 else k_pool.shape
    P, row_elems = shape[0], shape[2] * shape[3]
    layer_stride = P * _lib.PAGE_TOKENS * row_elems if num_layers > 1 else 0
    dev = k_pool.device
    if freed_pages is None:
        freed_pages = torch.full_like(page_table, -1)
    if n_freed is None:
        n_freed = torch.zeros(B, dtype=torch.int32, device=dev)
    if ws is None:
        ws = workspace(256, dev)
    rc = lib.a11s_kv_compact(k_pool.data_ptr(), v_pool.data_ptr(), num_layers, layer_stride, P,
                             row_elems, k_pool.element_size(), page_table.data_ptr(),
                             page_table.shape[1], seq_lens.data_ptr(), accept_len.data_ptr(),
                             accepted_nodes.data_ptr(), _ptr(n_nodes), B, N, freed_pages.data_ptr(),
                             n_freed.data_ptr(), ws.data_ptr(), ws.numel(), _stream())
    check(rc)
    if check_status:
        raise_on_status(ws)
    return freed_pages, n_freed


# --------------------------------------------------------------------------- K5
class KVPagePool:
    """The paged KV cache's page allocator in device memory (K5): a LIFO free
    stack of page ids with the reference PagedKVCacheManager's order
    (src/cuda/paged_kv_cache.cu:61-149). Page tables [B][max_pages] (-1 = no
    page) and seq_lens [B] are the caller's int32 CUDA tensors, shared with
    tree_attention and kv_compact. Every call is asynchronous on the current
    stream; with check_status=True it synchronises and raises A11Error for a
    device-side error (nothing changes on an error)."""

    def __init__(self, num_pages: int, device):
        self.num_pages = int(num_pages)
        self.free_stack = torch.empty(max(1, self.num_pages), dtype=torch.int32, device=device)
        self.free_top = torch.zeros(1, dtype=torch.int32, device=device)
        self.status = torch.zeros(2, dtype=torch.int32, device=device)
        check(lib.a11s_kv_pool_init(self.free_stack.data_ptr(), self.free_top.data_ptr(), self.num_pages,
                                    _stream()))

    def _done(self, rc: int, check_status: bool) -> None:
        check(rc)
        if check_status:
            code, detail = (int(x) for x in self.status.tolist())
            if code != _lib.OK:
                raise A11Error(code, f"device status {_lib.ERROR_NAMES.get(code, code)} (detail {detail})")

    def reserve(self, page_table: torch.Tensor, seq_lens: torch.Tensor, n_new: torch.Tensor,
                check_status: bool = False) -> None:
        """seq_lens += n_new; tables grow to max(1, ceil(len/16)) pages (append_token / allocate_sequence)."""
        for t, nm in ((page_table, "page_table"), (seq_lens, "seq_lens"), (n_new, "n_new")):
            _need(t, nm, torch.int32)
        rc = lib.a11s_kv_reserve(self.free_stack.data_ptr(), self.free_top.data_ptr(), self.num_pages,
                                 page_table.data_ptr(), page_table.shape[1], seq_lens.data_ptr(),
                                 n_new.data_ptr(), page_table.shape[0], self.status.data_ptr(), _stream())
        self._done(rc, check_status)

    def release(self, freed_pages: torch.Tensor, n_freed: torch.Tensor, check_status: bool = False) -> None:
        """Push the freed lists of kv_compact back on the stack (dealloc_block)."""
        _need(freed_pages, "freed_pages", torch.int32)
        _need(n_freed, "n_freed", torch.int32)
        rc = lib.a11s_kv_release(self.free_stack.data_ptr(), self.free_top.data_ptr(), self.num_pages,
                                 freed_pages.data_ptr(), freed_pages.shape[1], n_freed.data_ptr(),
                                 freed_pages.shape[0], self.status.data_ptr(), _stream())
        self._done(rc, check_status)

    def free_sequences(self, page_table: torch.Tensor, seq_lens: torch.Tensor, mask: torch.Tensor,
                       check_status: bool = False) -> None:
        """Return every page of the masked sequences in table order (free_sequence)."""
        for t, nm in ((page_table, "page_table"), (seq_lens, "seq_lens"), (mask, "mask")):
            _need(t, nm, torch.int32)
        rc = lib.a11s_kv_free_sequences(self.free_stack.data_ptr(), self.free_top.data_ptr(), self.num_pages,
                                        page_table.data_ptr(), page_table.shape[1], seq_lens.data_ptr(),
                                        mask.data_ptr(), page_table.shape[0], self.status.data_ptr(), _stream())
        self._done(rc, check_status)

    def adopt(self, page_table: torch.Tensor) -> None:
        """Set-up for tables built elsewhere: the free stack becomes every
        pool page that no table entry holds, in ascending order (so, like the
        reference's initial stack, the highest free id is taken first).
        Synchronises; not for the decode loop."""
        used = torch.zeros(self.num_pages, dtype=torch.bool, device=page_table.device)
        ids = page_table[page_table >= 0].long()
        if ids.numel() and (int(ids.min()) < 0 or int(ids.max()) >= self.num_pages):
            raise A11Error(_lib.EBOUNDS, "page table holds ids outside the pool")
        used[ids] = True
        free = torch.nonzero(~used).flatten().to(torch.int32)
        self.free_stack[: free.numel()] = free
        self.free_top.fill_(free.numel())
        torch.cuda.synchronize(page_table.device)

    def free_pages(self) -> torch.Tensor:
        """The stack's live entries, bottom first (a synchronising copy)."""
        return self.free_stack[: int(self.free_top.item())].clone()


# --------------------------------------------------------------------------- K6
def history_from_accept(last_tokens: torch.Tensor, accepted_tokens: torch.Tensor, accept_len: torch.Tensor,
                        bonus: torch.Tensor, out=None):
    """History rows of one acceptance step for ngram_update: (last_tokens[b][0],
    last_tokens[b][1], accepted_tokens[b][0 .. accept_len[b]), bonus[b]) and
    their lengths, built with device ops (no host synchronisation). `out`:
    preallocated (history int32 [B, N + 3], lens int32 [B]) to fill."""
    B, N = accepted_tokens.shape
    if out is None:
        hist = torch.empty((B, N + 3), dtype=torch.int32, device=accepted_tokens.device)
        lens_out = None
    else:
        hist, lens_out = out
    hist.fill_(-1)
    hist[:, :2] = last_tokens
    hist[:, 2:2 + N] = accepted_tokens
    alen = accept_len.long().clamp(0, N)
    hist.scatter_(1, (2 + alen).unsqueeze(1), bonus.to(torch.int32).unsqueeze(1))
    if lens_out is None:
        return hist, (alen + 3).to(torch.int32)
    torch.add(accept_len.clamp(0, N), 3, out=lens_out)
    return hist, lens_out


def next_roots(tree_tokens: torch.Tensor, accepted_tokens: torch.Tensor, accept_len: torch.Tensor,
               bonus: torch.Tensor, last_tokens: torch.Tensor, history=None):
    """One launch after an acceptance step (a11s_next_roots): last_tokens int32
    [B, 2] becomes the next tree's root pair (last accepted token, or the old
    root; the bonus, 0 if none), in place. With `history` = (rows int32
    [B, >= N + 3], lens int32 [B]) it also writes the committed-token rows for
    ngram_update from the old pair, as history_from_accept does. Returns
    `history` (or None)."""
    B, N = accepted_tokens.shape
    for t, name in ((tree_tokens, "tree_tokens"), (accepted_tokens, "accepted_tokens"), (accept_len, "accept_len"),
                    (bonus, "bonus"), (last_tokens, "last_tokens")):
        _need(t, name, torch.int32)
    if tuple(tree_tokens.shape) != (B, N) or tuple(last_tokens.shape) != (B, 2):
        raise ValueError("next_roots: tree_tokens [B, N] and last_tokens [B, 2] expected")
    rows = lens = None
    if history is not None:
        rows, lens = history
        _need(rows, "history", torch.int32)
        _need(lens, "history lens", torch.int32)
        if rows.shape[0] != B or rows.shape[1] < N + 3 or lens.numel() != B:
            raise ValueError("next_roots: history rows [B, >= N + 3] and lens [B] expected")
    check(lib.a11s_next_roots(_ptr(tree_tokens), _ptr(accepted_tokens), _ptr(accept_len), _ptr(bonus), B, N,
                              _ptr(last_tokens), _ptr(rows) if rows is not None else None,
                              rows.shape[1] if rows is not None else 0, _ptr(lens) if lens is not None else None,
                              _stream()))
    return history


def ngram_update(table: torch.Tensor, history: torch.Tensor, lens: torch.Tensor, log2_buckets: int,
                 status: Optional[torch.Tensor] = None, check_status: bool = False) -> torch.Tensor:
    """K6, in place on table int32 [2^k, slots, 2]: adds the trigrams of each
    history row (rows split into calls of at most NGRAM_MAX_UPDATES trigrams).
    Returns the device status int32[2] of the last call."""
    _need(table, "table", torch.int32)
    _need(history, "history", torch.int32)
    _need(lens, "lens", torch.int32)
    if status is None:
        status = torch.zeros(2, dtype=torch.int32, device=table.device)
    B, stride = history.shape
    per = max(1, _lib.NGRAM_MAX_UPDATES // max(1, stride - 2))
    for b0 in range(0, max(B, 1), per):
        rows = history[b0:b0 + per]
        rc = lib.a11s_ngram_update(table.data_ptr(), log2_buckets, table.shape[1], _ptr(rows) if B else None,
                                   stride, _ptr(lens[b0:b0 + per]) if B else None, rows.shape[0],
                                   status.data_ptr(), _stream())
        check(rc)
        if check_status:
            code, detail = (int(x) for x in status.tolist())
            if code != _lib.OK:
                raise A11Error(code, f"device status {_lib.ERROR_NAMES.get(code, code)} (row {b0 + detail})")
    return status


# --------------------------------------------------------------------------- K1
def ngram_bucket(a: int, b: int, log2_buckets: int) -> int:
    return int(lib.a11s_ngram_bucket(a, b, log2_buckets))


def ngram_expand(table: torch.Tensor, last_tokens: torch.Tensor, width_root: int = 4,
                 width_inner: int = 2, max_depth: int = 5, max_nodes: int = 64, out=None):
    """K1. table int32 [2^k, slots, 2]; last_tokens int32 [B, 2]. Returns
    (tokens, parents, depths, n_nodes)."""
    _need(table, "table", torch.int32)
    _need(last_tokens, "last_tokens", torch.int32)
    nb, slots, two = table.shape
    log2b = nb.bit_length() - 1
    if two != 2 or (1 << log2b) != nb:
        raise A11Error(_lib.EINVAL, "table must be [2^k, slots, 2]")
    B = last_tokens.shape[0]
    dev = table.device
    if out is None:
        out = (torch.empty(B, max_nodes, dtype=torch.int32, device=dev),
               torch.empty(B, max_nodes, dtype=torch.int32, device=dev),
               torch.empty(B, max_nodes, dtype=torch.int32, device=dev),
               torch.empty(B, dtype=torch.int32, device=dev))
    tk, pa, de, nn = out
    rc = lib.a11s_ngram_expand(table.data_ptr(), log2b, slots, last_tokens.data_ptr(), B,
                               width_root, width_inner, max_depth, max_nodes, tk.data_ptr(),
                               pa.data_ptr(), de.data_ptr(), nn.data_ptr(), _stream())
    check(rc)
    return out
