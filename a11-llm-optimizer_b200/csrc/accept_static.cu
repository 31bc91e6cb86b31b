// accept_static.cu - a11s_accept_static: a11s_accept on a fixed scratch array.
//
// Some callers of this library cannot hand it a workspace: hosts whose device
// memory is owned by another allocator that forbids outside cudaMalloc calls
// (a serving process that budgets every byte of HBM up front), foreign-language
// bindings without a device allocator of their own, and decode loops that
// cannot afford cudaMalloc's possible device-wide synchronisation. For them
// the scratch of the acceptance kernel (status word, row counters, chunk
// records and the root rows' weight sums) lives in one file-scope device array of
// A11S_ACCEPT_STATIC_SCRATCH_BYTES that every GPU loading the library keeps
// until the process exits. Nothing here calls cudaMalloc, cudaFree or an
// allocating library routine.
#include <cstdio>

#include "common.cuh"
#include "kernels.h"

static __device__ __align__(256) unsigned char g_accept_scratch[A11S_ACCEPT_STATIC_SCRATCH_BYTES];

namespace {
// Largest batch whose a11s_accept_workspace_bytes() fits the array (0 if none).
int32_t largest_fitting_batch(int32_t mode, int32_t max_nodes, int32_t vocab) {
    int32_t lo = 0, hi = 1;
    while (hi < (1 << 30) && a11s_accept_workspace_bytes(mode, hi, max_nodes, vocab) <= A11S_ACCEPT_STATIC_SCRATCH_BYTES) {
        lo = hi;
        hi *= 2;
    }
    while (hi - lo > 1) {  // invariant: lo fits, hi does not
        const int32_t mid = lo + (hi - lo) / 2;
        if (a11s_accept_workspace_bytes(mode, mid, max_nodes, vocab) <= A11S_ACCEPT_STATIC_SCRATCH_BYTES)
            lo = mid;
        else
            hi = mid;
    }
    return lo;
}
}  // namespace

extern "C" int a11s_accept_static(int32_t mode, int32_t dtype, const void *target_logits,
                                  const void *draft_logits, int64_t row_stride, float temperature,
                                  const float *uniforms, const int32_t *tokens,
                                  const int32_t *parents, const int32_t *n_nodes, int32_t batch,
                                  int32_t max_nodes, int32_t vocab, int32_t *accept_len,
                                  int32_t *accepted_nodes, int32_t *accepted_tokens,
                                  int32_t *bonus, float *node_probs, int64_t *stats,
                                  int32_t *status, void *stream) {
    const size_t need = a11s_accept_workspace_bytes(mode, batch, max_nodes, vocab);
    if (need > A11S_ACCEPT_STATIC_SCRATCH_BYTES) {
        char msg[320];
        snprintf(msg, sizeof msg,
                 "a11s_accept_static: this call needs %zu scratch bytes but the fixed array holds %u; "
                 "at max_nodes %d and vocab %d in mode %d at most %d sequences fit per call. Split the "
                 "batch, or call a11s_accept with a workspace",
                 need, (unsigned)A11S_ACCEPT_STATIC_SCRATCH_BYTES, max_nodes, vocab, mode,
                 largest_fitting_batch(mode, max_nodes, vocab));
        return a11s::set_error(A11S_ENOSPACE, msg);
    }
    // The host name g_accept_scratch is only a stand-in; the array's device
    // address comes from cudaGetSymbolAddress, asked on every call for the
    // context current now. Caching it per device ordinal would go stale after a
    // cudaDeviceReset or under another context on the same device. The lookup
    // allocates nothing; the first one on a device may load the module, so make
    // the first call before any stream capture.
    void *scratch = nullptr;
    if (cudaGetSymbolAddress(&scratch, g_accept_scratch) != cudaSuccess || !scratch) {
        (void)cudaGetLastError();
        return a11s::set_error(A11S_ECUDA, "a11s_accept_static: cudaGetSymbolAddress failed");
    }
    // a11s_accept clears the status word and the row counters (the only parts
    // that must start at zero; every record is written before it is read) on
    // the stream before its kernel runs; with batch == 0 it clears the status
    // word alone, which is then copied out like any other.
    const int rc = a11s_accept(mode, dtype, target_logits, draft_logits, row_stride, temperature,
                               uniforms, tokens, parents, n_nodes, batch, max_nodes, vocab,
                               accept_len, accepted_nodes, accepted_tokens, bonus, node_probs,
                               stats, scratch, A11S_ACCEPT_STATIC_SCRATCH_BYTES, stream);
    if (rc != A11S_OK || !status) return rc;
    const cudaError_t e = cudaMemcpyAsync(status, scratch, 2 * sizeof(int32_t), cudaMemcpyDeviceToDevice,
                                          reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? A11S_OK : a11s::set_error(A11S_ECUDA, "a11s_accept_static: status copy failed");
}
