"""ctypes binding of liba11spec.so (the C ABI in include/a11spec.h).

The library is the product: there is no fallback. Importing this module loads
the in-tree ``liba11spec.so`` (building it with nvcc first when it is missing
and nvcc exists); if that fails the import raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liba11spec.so")

OK, EINVAL, EBOUNDS, ECUDA, ETIMEOUT, ENONFINITE, ENOSPACE, EUNSUPPORTED = range(8)
F32, BF16 = 0, 1
GREEDY, STOCH_ONEHOT, STOCH_DRAFT = 0, 1, 2
PAGE_TOKENS = 16
NGRAM_MAX_UPDATES = 8192
STATS_LEN = 6
STAT_NAMES = ("steps_accepted", "steps_rejected", "fallback_count", "total_draft_tokens",
              "total_steps", "emitted_tokens")
ERROR_NAMES = {OK: "OK", EINVAL: "EINVAL", EBOUNDS: "EBOUNDS", ECUDA: "ECUDA",
               ETIMEOUT: "ETIMEOUT", ENONFINITE: "ENONFINITE", ENOSPACE: "ENOSPACE",
               EUNSUPPORTED: "EUNSUPPORTED"}


class A11Error(RuntimeError):
    """A C-ABI call returned an error code (host-side or device status)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{ERROR_NAMES.get(code, code)}: {message}")
        self.code = code


def _load() -> C.CDLL:
    if not os.path.exists(LIB_PATH):
        import importlib.util
        spec = importlib.util.spec_from_file_location(
            "_a11spec_build", os.path.join(os.path.dirname(HERE), "build.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()
    lib = C.CDLL(LIB_PATH)
    vp, i32, i64, f32, sz = C.c_void_p, C.c_int32, C.c_int64, C.c_float, C.c_size_t
    lib.a11s_abi_version.restype = C.c_int
    lib.a11s_last_error.restype = C.c_char_p
    lib.a11s_read_status.argtypes = [vp, C.POINTER(i32), C.POINTER(i32), vp]
    lib.a11s_accept_workspace_bytes.restype = sz
    lib.a11s_accept_workspace_bytes.argtypes = [i32, i32, i32, i32]
    lib.a11s_accept.argtypes = [i32, i32, vp, vp, i64, f32, vp, vp, vp, vp, i32, i32, i32,
                                vp, vp, vp, vp, vp, vp, vp, sz, vp]
    lib.a11s_tree_attention_workspace_bytes.restype = sz
    lib.a11s_tree_attention_workspace_bytes.argtypes = [i32, i32, i32, i32, i32, i32]
    lib.a11s_tree_attention.argtypes = [vp, vp, vp, i32, vp, i32, vp, vp, vp, i32, i32, i32, i32,
                                        i32, i32, f32, vp, vp, vp, sz, vp]
    lib.a11s_kv_compact.argtypes = [vp, vp, i32, i64, i32, i32, i32, vp, i32, vp, vp, vp, vp, i32,
                                    i32, vp, vp, vp, sz, vp]
    lib.a11s_ngram_expand.argtypes = [vp, i32, i32, vp, i32, i32, i32, i32, i32, vp, vp, vp, vp, vp]
    lib.a11s_ngram_bucket.restype = C.c_uint32
    lib.a11s_ngram_bucket.argtypes = [i32, i32, i32]
    lib.a11s_verify_chain.argtypes = [vp, vp, vp, i32, i32, vp, vp, vp, sz, vp]
    lib.a11s_accept_static.argtypes = [i32, i32, vp, vp, i64, f32, vp, vp, vp, vp, i32, i32, i32,
                                       vp, vp, vp, vp, vp, vp, vp, vp]
    lib.a11s_ngram_update.argtypes = [vp, i32, i32, vp, i32, vp, i32, vp, vp]
    lib.a11s_next_roots.argtypes = [vp, vp, vp, vp, i32, i32, vp, vp, i32, vp, vp]
    lib.a11s_kv_pool_init.argtypes = [vp, vp, i32, vp]
    lib.a11s_kv_reserve.argtypes = [vp, vp, i32, vp, i32, vp, vp, i32, vp, vp]
    lib.a11s_kv_release.argtypes = [vp, vp, i32, vp, i32, vp, i32, vp, vp]
    lib.a11s_kv_free_sequences.argtypes = [vp, vp, i32, vp, i32, vp, vp, i32, vp, vp]
    lib.a11s_lm_head_keys_bytes.restype = sz
    lib.a11s_lm_head_keys_bytes.argtypes = [i32, i32]
    lib.a11s_lm_head.argtypes = [vp, vp, i32, i32, i32, f32, vp, i64, vp, vp, sz, vp]
    lib.a11s_accept_recorded.argtypes = [i32, vp, i64, f32, vp, vp, vp, vp, i32, i32, i32, vp, vp, vp, vp, vp,
                                         vp, vp, vp, sz, vp]
    for name in ("a11s_read_status", "a11s_accept", "a11s_tree_attention", "a11s_kv_compact",
                 "a11s_ngram_expand", "a11s_verify_chain", "a11s_accept_static", "a11s_kv_pool_init",
                 "a11s_kv_reserve", "a11s_kv_release", "a11s_kv_free_sequences", "a11s_ngram_update",
                 "a11s_next_roots", "a11s_lm_head", "a11s_accept_recorded"):
        getattr(lib, name).restype = C.c_int
    if lib.a11s_abi_version() != 1:
        raise ImportError("liba11spec.so ABI version mismatch")
    return lib


lib = _load()


def check(rc: int) -> None:
    if rc != OK:
        raise A11Error(rc, lib.a11s_last_error().decode())


def symbols():
    """Names of every entry point declared in include/a11spec.h."""
    return ["a11s_abi_version", "a11s_last_error", "a11s_read_status",
            "a11s_accept_workspace_bytes", "a11s_accept", "a11s_accept_static",
            "a11s_tree_attention_workspace_bytes", "a11s_tree_attention", "a11s_kv_compact",
            "a11s_ngram_expand", "a11s_ngram_bucket", "a11s_verify_chain", "a11s_kv_pool_init",
            "a11s_kv_reserve", "a11s_kv_release", "a11s_kv_free_sequences", "a11s_ngram_update",
            "a11s_next_roots", "a11s_lm_head_keys_bytes", "a11s_lm_head", "a11s_accept_recorded"]
