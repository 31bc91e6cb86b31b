"""CPU oracle for the speculative-decoding hot path (TEST INFRASTRUCTURE ONLY).

This package is the checker of the CUDA kernels. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s ``cpu_baseline`` /
``--impl reference`` legs may import it; the product path (the ``a11spec``
package and ``liba11spec.so``) never does.

* ``liba11oracle.so`` (built from ``a11oracle.c`` by ``Makefile``) restates the
  path in plain C: acceptance (rule of the reference's
  src/engine/speculative_verifier.cpp:102-132), the chunked fixed-point
  softmax, tree attention (engine/pipeline.py:386-402), compaction, the
  paged-KV page allocator (src/cuda/paged_kv_cache.cu:85-149), n-gram
  expansion and the n-gram table update.
* ``_ref/libref_verifier.so`` (``make ref``, only where the reference tree is
  mounted) is the reference's own ``SpeculativeTreeVerifier`` behind the
  ``ref_harness.cpp`` shim; absent on machines without the reference.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liba11oracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libref_verifier.so")

_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
_u64p = np.ctypeslib.ndpointer(dtype=np.uint64, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")

_lib = None
_ref = None


def build(force: bool = False) -> str:
    """Compile liba11oracle.so (and _ref/ when the reference tree exists)."""
    if force or not os.path.exists(LIB_PATH):
        subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    return LIB_PATH


def build_ref(ref_root: str | None = None) -> bool:
    """Compile the reference verifier into _ref/ from the reference tree at
    `ref_root` (default: the A11_REFERENCE_ROOT environment variable). Returns
    False, building nothing, when no tree is given or its sources are absent."""
    ref_root = ref_root or os.environ.get("A11_REFERENCE_ROOT")
    if not ref_root or not os.path.isdir(os.path.join(ref_root, "src", "engine")):
        return False
    subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={ref_root}"], check=True)
    # The reference's binding tests, compiled unchanged to bytecode, so a GPU
    # machine without the reference tree can run them against a11_optimizer.
    import py_compile
    py_compile.compile(os.path.join(ref_root, "tests", "test_python_bindings.py"),
                       cfile=os.path.join(HERE, "_ref", "test_python_bindings.bytecode"), doraise=True)
    return True


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(LIB_PATH)
        L.or_weight.restype = C.c_uint64
        L.or_weight.argtypes = [C.c_float, C.c_float, C.c_int32]
        L.or_exp2_poly.restype = C.c_float
        L.or_exp2_poly.argtypes = [C.c_float]
        L.or_temperature_k.restype = C.c_float
        L.or_temperature_k.argtypes = [C.c_float]
        L.or_chunk_records.argtypes = [_f32p, C.c_int32, C.c_float, _f32p, _i32p, _u64p]
        L.or_accept.argtypes = [C.c_int32, _f32p, C.c_void_p, C.c_int64, C.c_float, C.c_void_p,
                                _i32p, _i32p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32,
                                _i32p, _i32p, _i32p, _i32p, C.c_void_p, C.c_void_p]
        L.or_exp_neg.restype = C.c_float
        L.or_exp_neg.argtypes = [C.c_float]
        L.or_verify_chain.argtypes = [_f32p, _f32p, _f32p, C.c_int32, C.c_int32, _i32p, _i32p]
        L.or_tree_attention.argtypes = [_f32p, _f32p, _f32p, C.c_int32, _i32p, C.c_int32, _i32p,
                                        _i32p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32,
                                        C.c_int32, C.c_int32, C.c_float, _f32p, C.c_void_p]
        L.or_kv_compact.argtypes = [_u8p, _u8p, C.c_int32, C.c_int64, C.c_int32, C.c_int32,
                                    C.c_int32, _i32p, C.c_int32, _i32p, _i32p, _i32p, C.c_void_p,
                                    C.c_int32, C.c_int32, _i32p, _i32p]
        L.or_kv_reserve.argtypes = [_i32p, _i32p, C.c_int32, _i32p, C.c_int32, _i32p, _i32p, C.c_int32,
                                    _i32p]
        L.or_kv_release.argtypes = [_i32p, _i32p, C.c_int32, _i32p, C.c_int32, _i32p, C.c_int32, _i32p]
        L.or_kv_free_sequences.argtypes = [_i32p, _i32p, C.c_int32, _i32p, C.c_int32, _i32p, _i32p,
                                           C.c_int32, _i32p]
        L.or_ngram_update.argtypes = [_i32p, C.c_int32, C.c_int32, _i32p, C.c_int32, _i32p, C.c_int32, _i32p]
        L.or_ngram_bucket.restype = C.c_uint32
        L.or_ngram_bucket.argtypes = [C.c_int32, C.c_int32, C.c_int32]
        L.or_ngram_expand.argtypes = [_i32p, C.c_int32, C.c_int32, _i32p, C.c_int32, C.c_int32,
                                      C.c_int32, C.c_int32, C.c_int32, _i32p, _i32p, _i32p, _i32p]
        _lib = L
    return _lib


def ref():
    """The reference's own verifier (oracle/_ref), or None where it was not built."""
    global _ref
    if _ref is None:
        if not os.path.exists(REF_PATH):
            return None
        R = C.CDLL(REF_PATH)
        R.ref_verify.argtypes = [C.c_int, _i32p, _f32p, _f32p, C.POINTER(C.c_uint32),
                                 C.POINTER(C.c_uint32)]
        R.ref_uniform_stream.argtypes = [C.c_int, _f32p]
        R.ref_verify_batch.argtypes = [C.c_int, C.c_int, _i32p, _f32p, _f32p, _u32p, C.c_int]
        R.ref_tree_mask.argtypes = [C.c_int, _i32p, C.c_int, _f32p]
        R.ref_tree_mask.restype = C.c_int
        R.ref_verify_mismatch.argtypes = [C.c_int, C.c_int, C.c_int]
        _ref = R
    return _ref


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


# ----------------------------------------------------------------------------- acceptance
def temperature_k(t: float) -> float:
    return float(lib().or_temperature_k(t))


def weight(l: float, k: float, c: int) -> int:
    return int(lib().or_weight(l, k, c))


def chunk_records(row: np.ndarray, k: float):
    row = np.ascontiguousarray(row, dtype=np.float32)
    nch = (row.shape[0] + 2047) // 2048
    cm = np.zeros(nch, np.float32)
    fr = np.zeros(nch, np.int32)
    sm = np.zeros(nch, np.uint64)
    lib().or_chunk_records(row, row.shape[0], k, cm, fr, sm)
    return cm, fr, sm


def accept(mode, target, tokens, parents, n_nodes=None, draft=None, temperature=1.0,
           uniforms=None, stats=None):
    """Run the oracle acceptance. target/draft: float32 [B, N, V] (bf16 widened)."""
    target = np.ascontiguousarray(target, dtype=np.float32)
    B, N, V = target.shape
    tokens = np.ascontiguousarray(tokens, dtype=np.int32)
    parents = np.ascontiguousarray(parents, dtype=np.int32)
    nn = None if n_nodes is None else np.ascontiguousarray(n_nodes, dtype=np.int32)
    dr = None if draft is None else np.ascontiguousarray(draft, dtype=np.float32)
    un = None if uniforms is None else np.ascontiguousarray(uniforms, dtype=np.float32)
    out = dict(accept_len=np.zeros(B, np.int32), accepted_nodes=np.zeros((B, N), np.int32),
               accepted_tokens=np.zeros((B, N), np.int32), bonus=np.zeros(B, np.int32),
               node_probs=np.zeros((B, N), np.float32))
    st = np.zeros(6, np.int64) if stats is None else stats
    rc = lib().or_accept(int(mode), target, _ptr(dr), V, float(temperature), _ptr(un), tokens,
                         parents, _ptr(nn), B, N, V, out["accept_len"], out["accepted_nodes"],
                         out["accepted_tokens"], out["bonus"], _ptr(out["node_probs"]), _ptr(st))
    out["status"] = rc
    out["stats"] = st
    return out


def verify_chain(draft, target, uniforms):
    """Chain rule of the reference verifier on [batch, n] per-token probabilities."""
    d = np.ascontiguousarray(draft, dtype=np.float32)
    t = np.ascontiguousarray(target, dtype=np.float32)
    u = np.ascontiguousarray(uniforms, dtype=np.float32)
    B, n = d.shape
    al = np.zeros(B, np.int32)
    li = np.zeros(B, np.int32)
    rc = lib().or_verify_chain(d, t, u, B, n, al, li)
    return al, li, rc


# ----------------------------------------------------------------------------- attention
def tree_attention(q, k_pool, v_pool, page_table, ctx_lens, parents, n_nodes, scale):
    q = np.ascontiguousarray(q, dtype=np.float32)
    B, N, Hq, D = q.shape
    k_pool = np.ascontiguousarray(k_pool, dtype=np.float32)
    v_pool = np.ascontiguousarray(v_pool, dtype=np.float32)
    P, _, Hkv, _ = k_pool.shape
    pt = np.ascontiguousarray(page_table, dtype=np.int32)
    out = np.zeros((B, N, Hq, D), np.float32)
    lse = np.zeros((B, N, Hq), np.float32)
    nn = None if n_nodes is None else np.ascontiguousarray(n_nodes, dtype=np.int32)
    rc = lib().or_tree_attention(q, k_pool, v_pool, P, pt, pt.shape[1],
                                 np.ascontiguousarray(ctx_lens, dtype=np.int32),
                                 np.ascontiguousarray(parents, dtype=np.int32), _ptr(nn), B, N,
                                 Hq, Hkv, D, float(scale), out, _ptr(lse))
    return out, lse, rc


# ----------------------------------------------------------------------------- compaction
def kv_compact(k_pool: np.ndarray, v_pool: np.ndarray, page_table, seq_lens, accept_len,
               accepted_nodes, n_nodes, num_layers=1, layer_stride=0):
    """In-place on copies; pools are any-dtype arrays [L?][P][16][Hkv][D]."""
    kb = np.ascontiguousarray(k_pool).copy()
    vb = np.ascontiguousarray(v_pool).copy()
    es = kb.dtype.itemsize
    row_elems = kb.shape[-1] * kb.shape[-2]
    P = kb.shape[-4]
    pt = np.ascontiguousarray(page_table, dtype=np.int32).copy()
    sl = np.ascontiguousarray(seq_lens, dtype=np.int32).copy()
    B, N = accepted_nodes.shape
    freed = np.full(pt.shape, -1, np.int32)
    nfreed = np.zeros(B, np.int32)
    nn = None if n_nodes is None else np.ascontiguousarray(n_nodes, dtype=np.int32)
    rc = lib().or_kv_compact(kb.view(np.uint8).reshape(-1), vb.view(np.uint8).reshape(-1),
                             num_layers, layer_stride, P, row_elems, es, pt, pt.shape[1], sl,
                             np.ascontiguousarray(accept_len, dtype=np.int32),
                             np.ascontiguousarray(accepted_nodes, dtype=np.int32), _ptr(nn), B,
                             N, freed, nfreed)
    return dict(k_pool=kb, v_pool=vb, page_table=pt, seq_lens=sl, freed_pages=freed,
                n_freed=nfreed, status=rc)


# ----------------------------------------------------------------------------- page allocator
def _pool_state(stack, top, num_pages):
    st = np.zeros(max(1, num_pages), np.int32)
    st[: len(stack)] = np.asarray(stack, dtype=np.int32)
    return st, np.array([top], np.int32)


def kv_reserve(stack, top, num_pages, page_table, seq_lens, n_new):
    """PagedKVCacheManager allocate_sequence / append_token over a batch, on copies.
    stack: the live entries (bottom first); returns the new state and (status, detail)."""
    st, tp = _pool_state(stack, top, num_pages)
    pt = np.ascontiguousarray(page_table, dtype=np.int32).copy()
    sl = np.ascontiguousarray(seq_lens, dtype=np.int32).copy()
    det = np.zeros(1, np.int32)
    rc = lib().or_kv_reserve(st, tp, num_pages, pt, pt.shape[1], sl, np.ascontiguousarray(n_new, dtype=np.int32),
                             pt.shape[0], det)
    return dict(stack=st[: tp[0]].copy(), top=int(tp[0]), page_table=pt, seq_lens=sl, status=rc, detail=int(det[0]))


def kv_release(stack, top, num_pages, freed_pages, n_freed):
    """dealloc_block of each freed list, batch order, on copies."""
    st, tp = _pool_state(stack, top, num_pages)
    fp = np.ascontiguousarray(freed_pages, dtype=np.int32)
    det = np.zeros(1, np.int32)
    rc = lib().or_kv_release(st, tp, num_pages, fp, fp.shape[1], np.ascontiguousarray(n_freed, dtype=np.int32),
                             fp.shape[0], det)
    return dict(stack=st[: tp[0]].copy(), top=int(tp[0]), status=rc, detail=int(det[0]))


def kv_free_sequences(stack, top, num_pages, page_table, seq_lens, mask):
    """free_sequence of every masked sequence, batch order, on copies."""
    st, tp = _pool_state(stack, top, num_pages)
    pt = np.ascontiguousarray(page_table, dtype=np.int32).copy()
    sl = np.ascontiguousarray(seq_lens, dtype=np.int32).copy()
    det = np.zeros(1, np.int32)
    rc = lib().or_kv_free_sequences(st, tp, num_pages, pt, pt.shape[1], sl, np.ascontiguousarray(mask, dtype=np.int32),
                                    pt.shape[0], det)
    return dict(stack=st[: tp[0]].copy(), top=int(tp[0]), page_table=pt, seq_lens=sl, status=rc, detail=int(det[0]))


# ----------------------------------------------------------------------------- n-gram
def ngram_bucket(a: int, b: int, log2_buckets: int) -> int:
    return int(lib().or_ngram_bucket(a, b, log2_buckets))


def ngram_update(table, log2_buckets, history, lens):
    """Serial restatement of a11s_ngram_update on a copy of the table."""
    t = np.ascontiguousarray(table, dtype=np.int32).copy()
    h = np.ascontiguousarray(history, dtype=np.int32)
    det = np.zeros(1, np.int32)
    rc = lib().or_ngram_update(t, log2_buckets, t.shape[1], h.reshape(-1) if h.size else np.zeros(1, np.int32),
                               h.shape[1] if h.ndim == 2 else 0, np.ascontiguousarray(lens, dtype=np.int32),
                               h.shape[0] if h.ndim == 2 else 0, det)
    return dict(table=t, status=rc, detail=int(det[0]))


def ngram_expand(table, log2_buckets, last_tokens, width_root, width_inner, max_depth, max_nodes):
    table = np.ascontiguousarray(table, dtype=np.int32)
    slots = table.shape[1]
    last = np.ascontiguousarray(last_tokens, dtype=np.int32)
    B = last.shape[0]
    tk = np.zeros((B, max_nodes), np.int32)
    pa = np.zeros((B, max_nodes), np.int32)
    de = np.zeros((B, max_nodes), np.int32)
    nn = np.zeros(B, np.int32)
    rc = lib().or_ngram_expand(table, log2_buckets, slots, last, B, width_root, width_inner,
                               max_depth, max_nodes, tk, pa, de, nn)
    return dict(tokens=tk, parents=pa, depths=de, n_nodes=nn, status=rc)


# ----------------------------------------------------------------------------- reference shim
def ref_uniform_stream(n: int) -> np.ndarray:
    r = ref()
    out = np.zeros(n, np.float32)
    r.ref_uniform_stream(n, out)
    return out


def ref_verify(tokens, draft, target):
    r = ref()
    tk = np.ascontiguousarray(tokens, dtype=np.int32)
    d = np.ascontiguousarray(draft, dtype=np.float32)
    t = np.ascontiguousarray(target, dtype=np.float32)
    a, l = C.c_uint32(0), C.c_uint32(0)
    rc = r.ref_verify(len(tk), tk, d, t, C.byref(a), C.byref(l))
    return (int(a.value), int(l.value)) if rc == 0 else None
