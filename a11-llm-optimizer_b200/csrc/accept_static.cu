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
#include <mutex>

#include "common.cuh"
#include "kernels.h"

static __device__ __align__(256) unsigned char g_accept_scratch[A11S_ACCEPT_STATIC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void *g_scratch_ptr[kMaxDevices];  // device address of g_accept_scratch, per device
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
        char msg[256];
        snprintf(msg, sizeof msg,
                 "a11s_accept_static: needs %zu scratch bytes but the fixed array holds %u "
                 "(8 bytes per row chunk: batch * max_nodes * ceil(vocab / 2048) of them); call a11s_accept "
                 "with a workspace instead",
                 need, (unsigned)A11S_ACCEPT_STATIC_SCRATCH_BYTES);
        return a11s::set_error(A11S_ENOSPACE, msg);
    }
    // Per-device set-up on the first call with that device current: the host
    // name g_accept_scratch is only a stand-in, its device address comes from
    // cudaGetSymbolAddress.
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return a11s::set_error(A11S_ECUDA, "a11s_accept_static: no usable current device");
    void *scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_scratch_mutex);
        if (!g_scratch_ptr[dev]) {
            void *p = nullptr;
            if (cudaGetSymbolAddress(&p, g_accept_scratch) != cudaSuccess || !p)
                return a11s::set_error(A11S_ECUDA, "a11s_accept_static: cudaGetSymbolAddress failed");
            g_scratch_ptr[dev] = p;
        }
        scratch = g_scratch_ptr[dev];
    }
    // a11s_accept clears the status word and the row counters (the only parts
    // that must start at zero; every record is written before it is read) on
    // the stream before its kernel runs.
    const int rc = a11s_accept(mode, dtype, target_logits, draft_logits, row_stride, temperature,
                               uniforms, tokens, parents, n_nodes, batch, max_nodes, vocab,
                               accept_len, accepted_nodes, accepted_tokens, bonus, node_probs,
                               stats, scratch, A11S_ACCEPT_STATIC_SCRATCH_BYTES, stream);
    if (rc != A11S_OK || !status || batch == 0) return rc;
    const cudaError_t e = cudaMemcpyAsync(status, scratch, 2 * sizeof(int32_t), cudaMemcpyDeviceToDevice,
                                          reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? A11S_OK : a11s::set_error(A11S_ECUDA, "a11s_accept_static: status copy failed");
}
