"""Verifier API with the names of the reference's pybind module ``a11_optimizer``
(src/bindings/python_bindings.cpp:78-143): ``SpecConfig``, ``TreeNode``,
``SpecDiagnostics``, ``SpeculativeTreeVerifier``, ``SPEC_K``, ``BLOCK_TOKENS``.

The acceptance decisions run on the GPU through ``a11s_verify_chain`` (the
reference rule of src/engine/speculative_verifier.cpp:84-135). The uniforms
come from the same stream the reference draws from its thread_local
``std::mt19937(42)`` (:65-69): each Python thread keeps its own generator,
continuing across calls, exactly like the reference's thread_local state.
Errors raise ``RuntimeError`` as pybind11 translates the reference's
``std::runtime_error``.
"""
from __future__ import annotations

import sys
import threading
from dataclasses import dataclass, field
from typing import List, Sequence, Tuple

import numpy as np
import torch

from . import _lib
from ._lib import A11Error, check, lib

SPEC_K = 8                  # include/engine/speculative_verifier.hpp:16
BLOCK_TOKENS = 16           # include/cuda/paged_kv_cache.hpp:13
KV_CACHE_VRAM_GB = 8        # include/cuda/paged_kv_cache.hpp:12
UINT32_MAX = 0xFFFFFFFF


@dataclass
class SpecConfig:
    """SpeculativeTreeVerifier::Config (speculative_verifier.hpp:61-66)."""
    max_draft_depth: int = SPEC_K
    vocab_size: int = 32000
    acceptance_threshold: float = 1.0  # kept for the interface; the rule uses min(1, ratio)
    log_diagnostics: bool = True


@dataclass
class TreeNode:
    """TreeNode (speculative_verifier.hpp:22-28)."""
    token_id: int = -1
    log_prob: float = 0.0
    parent_idx: int = UINT32_MAX
    depth: int = 0
    children: List[int] = field(default_factory=list)


@dataclass
class SpecDiagnostics:
    """SpecDiagnosticCounters (speculative_verifier.hpp:31-53)."""
    steps_accepted: int = 0
    steps_rejected: int = 0
    fallback_count: int = 0
    total_draft_tokens: int = 0
    total_steps: int = 0

    def reset(self) -> None:
        self.steps_accepted = self.steps_rejected = self.fallback_count = 0
        self.total_draft_tokens = self.total_steps = 0


class _ReferenceUniforms(threading.local):
    """Per-thread std::mt19937(42) + uniform_real_distribution<float>(0, 1):
    one 32-bit draw per value, u = float(x) / 2^32 (1.0 mapped below 1)."""

    def __init__(self):
        self.rs = np.random.RandomState(42)

    def draw(self, n: int) -> np.ndarray:
        raw = self.rs.randint(0, 2**32, size=n, dtype=np.uint64)
        u = raw.astype(np.float32) / np.float32(4294967296.0)
        return np.minimum(u, np.nextafter(np.float32(1.0), np.float32(0.0)))


_UNIFORMS = _ReferenceUniforms()


def reference_uniforms(n: int) -> np.ndarray:
    """Next n values of this thread's reference-compatible uniform stream."""
    return _UNIFORMS.draw(n)


def verify_chains(draft: torch.Tensor, target: torch.Tensor, uniforms: torch.Tensor,
                  ws: torch.Tensor = None):
    """Batched a11s_verify_chain on device tensors [B, n] -> (accepted_len, last_idx, ws)."""
    for t, nm in ((draft, "draft"), (target, "target"), (uniforms, "uniforms")):
        if not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
            raise A11Error(_lib.EINVAL, f"{nm} must be a contiguous float32 CUDA tensor")
    B, n = draft.shape
    al = torch.empty(B, dtype=torch.int32, device=draft.device)
    li = torch.empty(B, dtype=torch.int32, device=draft.device)
    if ws is None:
        ws = torch.empty(256, dtype=torch.uint8, device=draft.device)
    check(lib.a11s_verify_chain(draft.data_ptr(), target.data_ptr(), uniforms.data_ptr(), B, n,
                                al.data_ptr(), li.data_ptr(), ws.data_ptr(), ws.numel(),
                                torch.cuda.current_stream().cuda_stream))
    return al, li, ws


class SpeculativeTreeVerifier:
    """SpeculativeTreeVerifier (speculative_verifier.hpp:59-125) over the C ABI."""

    def __init__(self, cfg: SpecConfig, device: str = "cuda"):
        self._cfg = cfg
        self._diag = SpecDiagnostics()
        self._device = device

    # -- tree helpers (host-side data structures, as the reference) --------
    def build_draft_tree(self, root_token: int) -> TreeNode:
        if self._cfg.log_diagnostics:
            print(f"[SpeculativeTree] Built tree root: token={root_token}, "
                  f"max_depth={self._cfg.max_draft_depth}", file=sys.stderr)
        return TreeNode(token_id=int(root_token), log_prob=0.0, parent_idx=UINT32_MAX, depth=0)

    def construct_tree_mask(self, tree: Sequence[TreeNode]) -> List[float]:
        """One-hot [n x vocab] token mask of the reference API (speculative_verifier.cpp:41-61).
        The device path never builds it: tree attention derives ancestor bits from parents."""
        V = self._cfg.vocab_size
        mask = np.zeros((len(tree), V), np.float32)
        for i, node in enumerate(tree):
            if 0 <= node.token_id < V:
                mask[i, node.token_id] = 1.0
        return mask.reshape(-1).tolist()

    # -- acceptance (GPU) ---------------------------------------------------
    def verify_draft_tokens(self, draft_tokens: Sequence[int], draft_log_probs: Sequence[float],
                            target_log_probs: Sequence[float]) -> Tuple[int, int]:
        n = len(draft_tokens)
        if len(draft_log_probs) != n or len(target_log_probs) != n:
            raise RuntimeError("SpeculativeTreeVerifier: draft_tokens, draft_log_probs, and "
                               "target_log_probs must have same length")
        tgt = np.asarray(target_log_probs, np.float32)
        if n == 0 or not np.all(np.isfinite(tgt)):
            raise RuntimeError("SpeculativeTreeVerifier: invalid target probabilities")
        saved = _UNIFORMS.rs.get_state()
        u = reference_uniforms(n)
        dev = self._device
        d = torch.tensor(np.asarray(draft_log_probs, np.float32)[None], device=dev)
        t = torch.tensor(tgt[None], device=dev)
        uu = torch.tensor(u[None], device=dev)
        al, li, ws = verify_chains(d, t, uu)
        a, l = int(al.item()), int(li.item())
        if a < 0:
            raise RuntimeError("SpeculativeTreeVerifier: invalid target probabilities")
        # the reference draws one uniform per judged token and stops at the first
        # rejection: leave the stream where it would be (restore, redraw consumed)
        consumed = min(n, a + 1)
        if consumed < n:
            _UNIFORMS.rs.set_state(saved)
            reference_uniforms(consumed)
        return a, l

    def speculate_step(self, context_tokens: Sequence[int], root_draft_token: int):
        """Synthetic K-token chain of the reference (speculative_verifier.cpp:139-199)."""
        self._diag.total_steps += 1
        self.build_draft_tree(root_draft_token)
        if self._cfg.log_diagnostics:
            print(f"[SpeculativeTree] Speculation step #{self._diag.total_steps}, "
                  f"context_tokens={len(context_tokens)}, root_draft={root_draft_token}",
                  file=sys.stderr)
        draft_tokens = [int(root_draft_token) + i + 1 for i in range(SPEC_K)]
        draft_lp = [np.float32(-np.log(np.float32(SPEC_K))) * np.float32(1.0 - i * 0.05) for i in range(SPEC_K)]
        target_lp = []
        for i in range(SPEC_K):
            r = reference_uniforms(1)[0]
            target_lp.append(np.float32(draft_lp[i] + (np.float32(-0.1) if r < np.float32(0.9) else np.float32(-2.0))))
        self._diag.total_draft_tokens += SPEC_K
        accepted, last = self.verify_draft_tokens(draft_tokens, [float(x) for x in draft_lp],
                                                  [float(x) for x in target_lp])
        if self._cfg.log_diagnostics:
            print(f"[SpeculativeTree] Verification: accepted={accepted}, last_accepted_idx={last} "
                  f"/ {SPEC_K}", file=sys.stderr)
        if accepted == 0:
            self._diag.steps_rejected += 1
            self._diag.fallback_count += 1
        else:
            self._diag.steps_accepted += 1
        out = draft_tokens[:accepted] + [int(root_draft_token) + SPEC_K]
        return out, accepted == SPEC_K

    def diagnostics(self) -> SpecDiagnostics:
        return self._diag

    def reset_diagnostics(self) -> None:
        self._diag.reset()
