"""a11spec - B200-native speculative-decoding hot path (host side).

The compute lives in ``liba11spec.so`` (hand-written sm_100a CUDA behind the C
ABI of include/a11spec.h); this package is the PyTorch-facing host layer:

* ``ops``        torch wrappers of the kernels (draft, attention, accept, compact,
                 page allocator ``KVPagePool``, n-gram learning ``ngram_update``)
* ``ngram_table`` the n-gram table's file format
* ``generate``   ``speculative_stream``: the speculative decode loop around a target model
* ``decoder``    ``SpeculativeDecoder`` with the method names of the reference's
                 engine/speculative.py, plus batched tree APIs
* ``workloads``  seeded synthetic inputs of the five benchmark configurations

Importing the package loads the CUDA library; there is no CPU fallback.
"""
from ._lib import (A11Error, BF16, EBOUNDS, ECUDA, EINVAL, ENONFINITE, ENOSPACE, ETIMEOUT,
                   EUNSUPPORTED, F32, GREEDY, OK, PAGE_TOKENS, STATS_LEN, STAT_NAMES, STOCH_DRAFT,
                   STOCH_ONEHOT, LIB_PATH)
from . import ops
from .ops import (AcceptResult, KVPagePool, accept, history_from_accept, kv_compact, lm_head, next_roots,
                  ngram_bucket, ngram_expand, ngram_update, read_status, tree_attention)

__all__ = ["A11Error", "AcceptResult", "KVPagePool", "accept", "history_from_accept", "kv_compact", "lm_head",
           "next_roots", "ngram_bucket", "ngram_expand", "ngram_update",
           "read_status", "tree_attention", "ops", "GREEDY", "STOCH_ONEHOT", "STOCH_DRAFT", "F32",
           "BF16", "PAGE_TOKENS", "STATS_LEN", "STAT_NAMES", "LIB_PATH"]
