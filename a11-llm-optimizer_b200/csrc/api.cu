// api.cu - the extern "C" boundary of liba11spec.so (declared in include/a11spec.h).
//
// Host-side validation, workspace carving and launches. Nothing here allocates
// device memory or synchronises a stream (except a11s_read_status, documented
// as synchronising).
#include <cmath>
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace {

thread_local std::string g_err;

int fail(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char *what) {
    return fail(A11S_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

constexpr size_t kHeaderBytes = 256;  // status word lives at offset 0
constexpr long long kOneWaveRounds = 64;  // chunks per warp up to which a GREEDY pass runs as one wave

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            n = 148;
    }
    return n;
}

// ---- acceptance workspace layout ----
// status word (zeroed before each launch) | chunk maxima [B][rows][nch] float |
// first max positions [B][N][nch] int32 (GREEDY) (both set to 0xFF bytes before
// each launch) | weight sums of the root rows [B][2][nch] uint64 (sampling
// modes); rows = max_nodes, or 2 max_nodes in DRAFT (p rows, then q rows)
struct AcceptLayout {
    size_t recs, arg, root_sums, jobs, total;
};
AcceptLayout accept_layout(int32_t mode, int32_t batch, int32_t max_nodes, int32_t vocab) {
    AcceptLayout L;
    const size_t nch = (size_t)(vocab + A11S_CHUNK - 1) / A11S_CHUNK;
    const size_t rows = (size_t)batch * max_nodes * (mode == A11S_ACCEPT_STOCH_DRAFT ? 2 : 1);
    L.recs = kHeaderBytes;
    L.arg = L.recs + up256(rows * nch * sizeof(float));
    L.root_sums = L.arg + (mode == A11S_ACCEPT_GREEDY ? up256(rows * nch * sizeof(int32_t)) : 0);
    L.jobs = L.root_sums + (mode == A11S_ACCEPT_GREEDY ? 0 : up256((size_t)batch * 2 * nch * sizeof(uint64_t)));
    L.total = L.jobs + (mode == A11S_ACCEPT_GREEDY ? 0 : up256((size_t)batch * a11s::accept_job_bytes((int)nch)));
    return L;
}

// An empty batch launches nothing, but the caller may still read the
// workspace status word afterwards: clear it on the stream.
int empty_batch_status(void *workspace, size_t workspace_bytes, void *stream, const char *who) {
    if (!workspace || workspace_bytes < sizeof(a11s::StatusWord)) return A11S_OK;
    const cudaError_t e = cudaMemsetAsync(workspace, 0, sizeof(a11s::StatusWord), reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? A11S_OK : cuda_fail(e, who);
}
}  // namespace

namespace a11s {
int set_error(int code, const char *msg) { return fail(code, "%s", msg); }
}  // namespace a11s

extern "C" {

int a11s_abi_version(void) { return A11S_ABI_VERSION; }

const char *a11s_last_error(void) { return g_err.c_str(); }

int a11s_read_status(const void *workspace, int32_t *status, int32_t *detail, void *stream) {
    if (!workspace || !status) return fail(A11S_EINVAL, "a11s_read_status: null argument");
    a11s::StatusWord w{};
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(&w, workspace, sizeof w, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "a11s_read_status");
    *status = w.code;
    if (detail) *detail = w.code ? w.detail : -1;
    return A11S_OK;
}

// ------------------------------------------------------------------- K3
size_t a11s_accept_workspace_bytes(int32_t mode, int32_t batch, int32_t max_nodes, int32_t vocab) {
    if (batch < 0 || max_nodes < 1 || vocab < 1) return 0;
    return accept_layout(mode, batch, max_nodes, vocab).total;
}

namespace {
// a11s_accept, or a11s_accept_recorded when `keys` is given.
int accept_call(int32_t mode, int32_t dtype, const void *target_logits, const void *draft_logits,
                int64_t row_stride, float temperature, const float *uniforms,
                const int32_t *tokens, const int32_t *parents, const int32_t *n_nodes,
                int32_t batch, int32_t max_nodes, int32_t vocab, int32_t *accept_len,
                int32_t *accepted_nodes, int32_t *accepted_tokens, int32_t *bonus,
                float *node_probs, int64_t *stats, void *workspace, size_t workspace_bytes,
                void *stream, const uint64_t *keys) {
    if (mode < A11S_ACCEPT_GREEDY || mode > A11S_ACCEPT_STOCH_DRAFT)
        return fail(A11S_EINVAL, "a11s_accept: unknown mode %d", mode);
    if (dtype != A11S_F32 && dtype != A11S_BF16)
        return fail(A11S_EINVAL, "a11s_accept: unknown dtype %d", dtype);
    if (batch < 0) return fail(A11S_EINVAL, "a11s_accept: batch %d < 0", batch);
    if (max_nodes < 1 || max_nodes > A11S_MAX_ACCEPT_NODES)
        return fail(A11S_EUNSUPPORTED, "a11s_accept: max_nodes %d outside [1, %d]", max_nodes,
                    A11S_MAX_ACCEPT_NODES);
    if (vocab < 1 || vocab > A11S_MAX_VOCAB)
        return fail(A11S_EUNSUPPORTED, "a11s_accept: vocab %d outside [1, %d]", vocab, A11S_MAX_VOCAB);
    const int vec = dtype == A11S_BF16 ? 8 : 4;
    if (row_stride < vocab || row_stride % vec || vocab % vec)
        return fail(A11S_EINVAL,
                    "a11s_accept: row_stride %lld and vocab %d must be multiples of %d, stride >= vocab",
                    (long long)row_stride, vocab, vec);
    if (batch == 0) return empty_batch_status(workspace, workspace_bytes, stream, "a11s_accept: clearing status");
    if (!target_logits || !tokens || !parents || !accept_len || !accepted_nodes ||
        !accepted_tokens || !bonus || !workspace)
        return fail(A11S_EINVAL, "a11s_accept: null required pointer");
    if (!aligned16(target_logits) || (draft_logits && !aligned16(draft_logits)))
        return fail(A11S_EINVAL, "a11s_accept: logits must be 16-byte aligned");
    if (mode != A11S_ACCEPT_GREEDY) {
        if (!uniforms) return fail(A11S_EINVAL, "a11s_accept: sampling modes need uniforms");
        if (!(temperature > 0.0f) || !std::isfinite(temperature))
            return fail(A11S_EINVAL, "a11s_accept: temperature must be finite and > 0");
    }
    if (mode == A11S_ACCEPT_STOCH_DRAFT && !draft_logits)
        return fail(A11S_EINVAL, "a11s_accept: STOCH_DRAFT needs draft_logits");
    if (!aligned16(workspace)) return fail(A11S_EINVAL, "a11s_accept: workspace must be 16-byte aligned");
    const AcceptLayout L = accept_layout(mode, batch, max_nodes, vocab);
    if (workspace_bytes < L.total)
        return fail(A11S_ENOSPACE, "a11s_accept: workspace %zu < %zu bytes", workspace_bytes, L.total);

    a11s::AcceptArgs a{};
    a.target = target_logits;
    a.draft = draft_logits;
    a.stride = row_stride;
    const double t = temperature < 1e-5f ? 1e-5 : (double)temperature;  // engine/sampler.py:10
    a.k = (float)(1.4426950408889634 / t);
    a.uniforms = uniforms;
    a.tokens = tokens;
    a.parents = parents;
    a.n_nodes = n_nodes;
    a.B = batch;
    a.N = max_nodes;
    a.V = vocab;
    a.nch = (vocab + A11S_CHUNK - 1) / A11S_CHUNK;
    a.rows_per_seq = max_nodes * (mode == A11S_ACCEPT_STOCH_DRAFT ? 2 : 1);
    a.units_per_seq = a.rows_per_seq * a.nch;
    a.accept_len = accept_len;
    a.acc_nodes = accepted_nodes;
    a.acc_tokens = accepted_tokens;
    a.bonus = bonus;
    a.node_probs = mode == A11S_ACCEPT_GREEDY ? nullptr : node_probs;
    a.stats = reinterpret_cast<long long *>(stats);
    char *ws = static_cast<char *>(workspace);
    a.status = reinterpret_cast<a11s::StatusWord *>(ws);
    a.recs = reinterpret_cast<float *>(ws + L.recs);
    a.arg = mode == A11S_ACCEPT_GREEDY ? reinterpret_cast<int32_t *>(ws + L.arg) : nullptr;
    a.root_sums = reinterpret_cast<unsigned long long *>(ws + L.root_sums);
    a.walkers_done = reinterpret_cast<int32_t *>(ws + 16);  // header: status word at 0, the finished-walk counter at 16
    a.jobs = mode == A11S_ACCEPT_GREEDY ? nullptr : ws + L.jobs;
    a.job_stride = (int64_t)a11s::accept_job_bytes(a.nch);
    // A walking block may wait for rows that other blocks record only when the
    // walkers (one block per sequence, the first ones scheduled) fill at most
    // half of the 2 resident blocks per SM: the bulk pass always has room.
    a.wait_records = batch <= sm_count() ? 1 : 0;

    // Grid row 0 of a sequence walks its tree and streams nothing; rows 1 ..
    // root_blocks take its root rows' units (maxima, first positions in GREEDY,
    // weight sums in the sampling modes), one per warp, so every root is
    // recorded in the first wave by many SMs at once. With chunk keys GREEDY
    // needs no root blocks: every record is written before the launch. The
    // other units are balanced over about 4 waves of 2 resident 512-thread
    // blocks per SM, at least 16 chunks (one per warp) per block.
    const int root_units = a.nch * (mode == A11S_ACCEPT_STOCH_DRAFT ? 2 : 1);
    a.root_blocks = (mode == A11S_ACCEPT_GREEDY && keys) ? 0 : (root_units + 15) / 16;
    a.keys = reinterpret_cast<const unsigned long long *>(keys);
    const long long rest = (long long)a.units_per_seq - root_units;
    const long long target_blocks = (long long)sm_count() * 2 * 4;
    long long slice = ((long long)batch * rest + target_blocks - 1) / target_blocks;
    slice = ((slice + 15) / 16) * 16;
    if (slice < 16) slice = 16;
    if (slice > rest && rest > 0) slice = rest;
    a.slice = (int32_t)slice;
    // with chunk keys there is nothing to stream: the walkers and the root blocks
    int grid_y = 1 + a.root_blocks + (keys ? 0 : (int)((rest + slice - 1) / slice));
    // Streaming rows interleaved with the root rows: as many as the first wave
    // holds beside the walkers and every root row. Root rows that a long-lived
    // streaming block pushes out of the first wave start late, and so do the
    // walks (64 sequences of 64 fp32 p and q rows over 151936 tokens, 640
    // root blocks: 1014-1026 us interleaved against 892-898 us); for 32
    // sequences of 64 bf16 rows over 151936 tokens, one-hot, interleaving gave
    // 94-95 us against 98-100 us.
    {
        const long long fit = (long long)sm_count() * 2 / batch - 1 - a.root_blocks;
        a.root_pairs = (int32_t)std::max(0ll, std::min({fit, (long long)a.root_blocks,
                                                        (long long)(grid_y - 1 - a.root_blocks)}));
    }
    // A small GREEDY pass (at most kOneWaveRounds chunks per warp) runs as one
    // wave instead: the walker and rr streaming blocks per sequence, all
    // resident at once, taking the units round-robin (roots first, then the
    // rows in index order). Blocks that stream one chunk per warp live about
    // one memory round trip, and the block scheduler then keeps only about
    // 60 % of the slots busy.
    a.rr = 0;
    const long long rr = ((long long)sm_count() * 2 - batch) / batch;
    if (mode == A11S_ACCEPT_GREEDY && !keys && rr >= 1 &&
        (a.units_per_seq + rr * 16 - 1) / (rr * 16) <= kOneWaveRounds) {
        a.rr = (int32_t)std::min<long long>(rr, (a.units_per_seq + 15) / 16);
        a.root_blocks = 0;
        grid_y = 1 + a.rr;
    }
    a.bulk_rows = grid_y;
    if (mode != A11S_ACCEPT_GREEDY) {
        // Helper rows: blocks scheduled after every walking and streaming block
        // that take chunks of the walks' row passes, about two per SM.
        const int helper_rows = (2 * sm_count() + batch - 1) / batch;
        grid_y += helper_rows < 1 ? 1 : helper_rows;
    }

    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = keys ? a11s::launch_accept_keys_init(mode, a, a.jobs, a.jobs ? L.total - L.jobs : 0, s)
                         : a11s::launch_accept_init(a.status, ws + L.recs, L.root_sums - L.recs, a.jobs,
                                                    a.jobs ? L.total - L.jobs : 0, s);
    if (e != cudaSuccess) return cuda_fail(e, "a11s_accept: clearing workspace");
    e = a11s::launch_accept(mode, dtype == A11S_BF16, a, grid_y, s);
    if (e != cudaSuccess) return cuda_fail(e, "a11s_accept: launch");
    return A11S_OK;
}
}  // namespace

int a11s_accept(int32_t mode, int32_t dtype, const void *target_logits, const void *draft_logits,
                int64_t row_stride, float temperature, const float *uniforms,
                const int32_t *tokens, const int32_t *parents, const int32_t *n_nodes,
                int32_t batch, int32_t max_nodes, int32_t vocab, int32_t *accept_len,
                int32_t *accepted_nodes, int32_t *accepted_tokens, int32_t *bonus,
                float *node_probs, int64_t *stats, void *workspace, size_t workspace_bytes,
                void *stream) {
    return accept_call(mode, dtype, target_logits, draft_logits, row_stride, temperature, uniforms, tokens,
                       parents, n_nodes, batch, max_nodes, vocab, accept_len, accepted_nodes, accepted_tokens,
                       bonus, node_probs, stats, workspace, workspace_bytes, stream, nullptr);
}

int a11s_accept_recorded(int32_t mode, const void *target_logits, int64_t row_stride, float temperature,
                         const float *uniforms, const int32_t *tokens, const int32_t *parents,
                         const int32_t *n_nodes, int32_t batch, int32_t max_nodes, int32_t vocab,
                         const uint64_t *chunk_keys, int32_t *accept_len, int32_t *accepted_nodes,
                         int32_t *accepted_tokens, int32_t *bonus, float *node_probs, int64_t *stats,
                         void *workspace, size_t workspace_bytes, void *stream) {
    if (mode != A11S_ACCEPT_GREEDY && mode != A11S_ACCEPT_STOCH_ONEHOT)
        return fail(A11S_EUNSUPPORTED, "a11s_accept_recorded: mode %d (GREEDY or STOCH_ONEHOT only)", mode);
    if (batch > 0 && (!chunk_keys || !aligned16(chunk_keys)))
        return fail(A11S_EINVAL, "a11s_accept_recorded: chunk_keys must be a 16-byte aligned device pointer");
    return accept_call(mode, A11S_BF16, target_logits, nullptr, row_stride, temperature, uniforms, tokens,
                       parents, n_nodes, batch, max_nodes, vocab, accept_len, accepted_nodes, accepted_tokens,
                       bonus, node_probs, stats, workspace, workspace_bytes, stream, chunk_keys);
}

int a11s_verify_chain(const float *draft_probs, const float *target_probs, const float *uniforms,
                      int32_t batch, int32_t n, int32_t *accepted_len, int32_t *last_idx,
                      void *workspace, size_t workspace_bytes, void *stream) {
    if (batch < 0 || n < 0) return fail(A11S_EINVAL, "a11s_verify_chain: negative size");
    if (batch == 0) return empty_batch_status(workspace, workspace_bytes, stream, "a11s_verify_chain: clearing status");
    if (!accepted_len || !last_idx || !workspace || (n > 0 && (!draft_probs || !target_probs || !uniforms)))
        return fail(A11S_EINVAL, "a11s_verify_chain: null required pointer");
    if (workspace_bytes < sizeof(a11s::StatusWord))
        return fail(A11S_ENOSPACE, "a11s_verify_chain: workspace too small for the status word");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(workspace, 0, sizeof(a11s::StatusWord), s);
    if (e != cudaSuccess) return cuda_fail(e, "a11s_verify_chain: clearing status");
    e = a11s::launch_verify_chain(draft_probs, target_probs, uniforms, batch, n, accepted_len, last_idx,
                                  static_cast<a11s::StatusWord *>(workspace), s);
    if (e != cudaSuccess) return cuda_fail(e, "a11s_verify_chain: launch");
    return A11S_OK;
}

// ------------------------------------------------------------------- K4
int a11s_kv_compact(void *k_pool, void *v_pool, int32_t num_layers, int64_t layer_stride,
                    int32_t num_pages, int32_t row_elems, int32_t elem_bytes, int32_t *page_table,
                    int32_t max_pages_per_seq, int32_t *seq_lens, const int32_t *accept_len,
                    const int32_t *accepted_nodes, const int32_t *n_nodes, int32_t batch,
                    int32_t max_nodes, int32_t *freed_pages, int32_t *n_freed, void *workspace,
                    size_t workspace_bytes, void *stream) {
    if (batch < 0 || num_layers < 1 || num_pages < 1 || row_elems < 1 || max_nodes < 1 ||
        max_pages_per_seq < 1)
        return fail(A11S_EINVAL, "a11s_kv_compact: non-positive size");
    if (elem_bytes != 2 && elem_bytes != 4)
        return fail(A11S_EINVAL, "a11s_kv_compact: elem_bytes must be 2 or 4");
    const int64_t row_bytes = (int64_t)row_elems * elem_bytes;
    if (row_bytes % 16) return fail(A11S_EINVAL, "a11s_kv_compact: row bytes %lld not a multiple of 16",
                                    (long long)row_bytes);
    const int64_t slab = (int64_t)num_pages * A11S_PAGE_TOKENS * row_elems;
    if (num_layers > 1 && layer_stride < slab)
        return fail(A11S_EINVAL, "a11s_kv_compact: layer_stride smaller than one layer");
    if (batch == 0) return empty_batch_status(workspace, workspace_bytes, stream, "a11s_kv_compact: clearing status");
    if (!k_pool || !v_pool || !page_table || !seq_lens || !accept_len || !accepted_nodes)
        return fail(A11S_EINVAL, "a11s_kv_compact: null required pointer");
    if (!aligned16(k_pool) || !aligned16(v_pool))
        return fail(A11S_EINVAL, "a11s_kv_compact: pools must be 16-byte aligned");
    if (workspace && workspace_bytes < sizeof(a11s::StatusWord))
        return fail(A11S_ENOSPACE, "a11s_kv_compact: workspace too small for the status word");
    a11s::CompactArgs a{};
    a.k_pool = static_cast<char *>(k_pool);
    a.v_pool = static_cast<char *>(v_pool);
    a.num_layers = num_layers;
    a.layer_stride_bytes = (num_layers > 1 ? layer_stride : slab) * elem_bytes;
    a.num_pages = num_pages;
    a.row_bytes = (int32_t)row_bytes;
    a.page_table = page_table;
    a.max_pages = max_pages_per_seq;
    a.seq_lens = seq_lens;
    a.accept_len = accept_len;
    a.accepted_nodes = accepted_nodes;
    a.n_nodes = n_nodes;
    a.B = batch;
    a.N = max_nodes;
    a.freed_pages = freed_pages;
    a.n_freed = n_freed;
    a.status = static_cast<a11s::StatusWord *>(workspace);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (workspace) {
        cudaError_t e = cudaMemsetAsync(workspace, 0, sizeof(a11s::StatusWord), s);
        if (e != cudaSuccess) return cuda_fail(e, "a11s_kv_compact: clearing status");
    }
    cudaError_t e = a11s::launch_kv_compact(a, s);
    if (e != cudaSuccess) return cuda_fail(e, "a11s_kv_compact: launch");
    return A11S_OK;
}

// ------------------------------------------------------------------- K1
uint32_t a11s_ngram_bucket(int32_t a, int32_t b, int32_t log2_buckets) {
    uint64_t z = ((uint64_t)(uint32_t)a << 32) | (uint32_t)b;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    z ^= z >> 31;
    return (uint32_t)(z >> (64 - log2_buckets));
}

int a11s_ngram_expand(const int32_t *table, int32_t log2_buckets, int32_t slots,
                      const int32_t *last_tokens, int32_t batch, int32_t width_root,
                      int32_t width_inner, int32_t max_depth, int32_t max_nodes, int32_t *tokens,
                      int32_t *parents, int32_t *depths, int32_t *n_nodes, void *stream) {
    if (log2_buckets < 1 || log2_buckets > 30)
        return fail(A11S_EINVAL, "a11s_ngram_expand: log2_buckets %d outside [1, 30]", log2_buckets);
    if (slots < 1 || slots > 32) return fail(A11S_EUNSUPPORTED, "a11s_ngram_expand: slots %d outside [1, 32]", slots);
    if (width_root < 0 || width_inner < 0 || width_root > slots || width_inner > slots)
        return fail(A11S_EINVAL, "a11s_ngram_expand: widths must lie in [0, slots]");
    if (max_depth < 0 || max_nodes < 1 || max_nodes > A11S_MAX_NODES)
        return fail(A11S_EINVAL, "a11s_ngram_expand: bad max_depth / max_nodes");
    if (batch < 0) return fail(A11S_EINVAL, "a11s_ngram_expand: batch < 0");
    if (batch == 0) return A11S_OK;
    if (!table || !last_tokens || !tokens || !parents || !depths || !n_nodes)
        return fail(A11S_EINVAL, "a11s_ngram_expand: null required pointer");
    a11s::NgramArgs a{table, log2_buckets, slots, last_tokens, batch, width_root, width_inner,
                      max_depth, max_nodes, tokens, parents, depths, n_nodes};
    cudaError_t e = a11s::launch_ngram_expand(a, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "a11s_ngram_expand: launch");
    return A11S_OK;
}

int a11s_ngram_update(int32_t *table, int32_t log2_buckets, int32_t slots, const int32_t *history,
                      int32_t history_stride, const int32_t *history_len, int32_t batch, int32_t *status,
                      void *stream) {
    if (log2_buckets < 1 || log2_buckets > 30)
        return fail(A11S_EINVAL, "a11s_ngram_update: log2_buckets %d outside [1, 30]", log2_buckets);
    if (slots < 1 || slots > 32) return fail(A11S_EUNSUPPORTED, "a11s_ngram_update: slots %d outside [1, 32]", slots);
    if (batch < 0 || history_stride < 0) return fail(A11S_EINVAL, "a11s_ngram_update: batch and stride must be >= 0");
    const long long updates = (long long)batch * (history_stride > 2 ? history_stride - 2 : 0);
    if (updates > A11S_NGRAM_MAX_UPDATES)
        return fail(A11S_EUNSUPPORTED, "a11s_ngram_update: batch * (stride - 2) = %lld > %d trigrams per call",
                    updates, A11S_NGRAM_MAX_UPDATES);
    if (!table || !status || (batch > 0 && (!history || !history_len)))
        return fail(A11S_EINVAL, "a11s_ngram_update: null required pointer");
    int cap = 1;
    while (cap < updates) cap <<= 1;
    a11s::NgramUpdateArgs a{table, log2_buckets, slots, history, history_len, batch, history_stride, cap, status};
    cudaError_t e = a11s::launch_ngram_update(a, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "a11s_ngram_update: launch");
    return A11S_OK;
}

int a11s_next_roots(const int32_t *tree_tokens, const int32_t *accepted_tokens, const int32_t *accept_len,
                    const int32_t *bonus, int32_t batch, int32_t max_nodes, int32_t *last_tokens, int32_t *history,
                    int32_t history_stride, int32_t *history_len, void *stream) {
    if (batch < 0 || max_nodes < 1) return fail(A11S_EINVAL, "a11s_next_roots: batch %d / max_nodes %d", batch, max_nodes);
    if (history && history_stride < max_nodes + 3)
        return fail(A11S_EINVAL, "a11s_next_roots: history_stride %d < max_nodes + 3", history_stride);
    if (batch == 0) return A11S_OK;
    if (!tree_tokens || !accepted_tokens || !accept_len || !bonus || !last_tokens || (history && !history_len))
        return fail(A11S_EINVAL, "a11s_next_roots: null required pointer");
    a11s::NextRootsArgs a{tree_tokens, accepted_tokens, accept_len, bonus, batch, max_nodes, last_tokens, history,
                          history_stride, history_len};
    cudaError_t e = a11s::launch_next_roots(a, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "a11s_next_roots: launch");
    return A11S_OK;
}

// ------------------------------------------------------------------- K5
int a11s_kv_pool_init(int32_t *free_stack, int32_t *free_top, int32_t num_pages, void *stream) {
    if (num_pages < 0) return fail(A11S_EINVAL, "a11s_kv_pool_init: num_pages %d < 0", num_pages);
    if (!free_top || (num_pages > 0 && !free_stack)) return fail(A11S_EINVAL, "a11s_kv_pool_init: null pointer");
    cudaError_t e = a11s::launch_kv_pool_init(free_stack, free_top, num_pages, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "a11s_kv_pool_init: launch");
    return A11S_OK;
}

static int kv_pages_check(const char *who, int32_t *free_stack, int32_t *free_top, int32_t num_pages,
                          int32_t batch, int32_t *status) {
    if (num_pages < 0 || batch < 0) return fail(A11S_EINVAL, "%s: num_pages and batch must be >= 0", who);
    if (!free_stack || !free_top || !status) return fail(A11S_EINVAL, "%s: null required pointer", who);
    return A11S_OK;
}

int a11s_kv_reserve(int32_t *free_stack, int32_t *free_top, int32_t num_pages, int32_t *page_table,
                    int32_t max_pages, int32_t *seq_lens, const int32_t *n_new, int32_t batch, int32_t *status,
                    void *stream) {
    int rc = kv_pages_check("a11s_kv_reserve", free_stack, free_top, num_pages, batch, status);
    if (rc != A11S_OK) return rc;
    if (max_pages < 1) return fail(A11S_EINVAL, "a11s_kv_reserve: max_pages %d < 1", max_pages);
    if (batch > 0 && (!page_table || !seq_lens || !n_new)) return fail(A11S_EINVAL, "a11s_kv_reserve: null pointer");
    a11s::KvPagesArgs a{free_stack, free_top, num_pages, page_table, max_pages, seq_lens, n_new, nullptr, 0,
                        batch, status};
    cudaError_t e = a11s::launch_kv_reserve(a, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "a11s_kv_reserve: launch");
    return A11S_OK;
}

int a11s_kv_release(int32_t *free_stack, int32_t *free_top, int32_t num_pages, const int32_t *freed_pages,
                    int32_t freed_stride, const int32_t *n_freed, int32_t batch, int32_t *status, void *stream) {
    int rc = kv_pages_check("a11s_kv_release", free_stack, free_top, num_pages, batch, status);
    if (rc != A11S_OK) return rc;
    if (freed_stride < 0) return fail(A11S_EINVAL, "a11s_kv_release: freed_stride %d < 0", freed_stride);
    if (batch > 0 && (!freed_pages || !n_freed)) return fail(A11S_EINVAL, "a11s_kv_release: null pointer");
    a11s::KvPagesArgs a{free_stack, free_top, num_pages, nullptr, 0, nullptr, n_freed, freed_pages, freed_stride,
                        batch, status};
    cudaError_t e = a11s::launch_kv_push(a, false, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "a11s_kv_release: launch");
    return A11S_OK;
}

int a11s_kv_free_sequences(int32_t *free_stack, int32_t *free_top, int32_t num_pages, int32_t *page_table,
                           int32_t max_pages, int32_t *seq_lens, const int32_t *free_mask, int32_t batch,
                           int32_t *status, void *stream) {
    int rc = kv_pages_check("a11s_kv_free_sequences", free_stack, free_top, num_pages, batch, status);
    if (rc != A11S_OK) return rc;
    if (max_pages < 1) return fail(A11S_EINVAL, "a11s_kv_free_sequences: max_pages %d < 1", max_pages);
    if (batch > 0 && (!page_table || !seq_lens || !free_mask))
        return fail(A11S_EINVAL, "a11s_kv_free_sequences: null pointer");
    a11s::KvPagesArgs a{free_stack, free_top, num_pages, page_table, max_pages, seq_lens, free_mask, nullptr, 0,
                        batch, status};
    cudaError_t e = a11s::launch_kv_push(a, true, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "a11s_kv_free_sequences: launch");
    return A11S_OK;
}

// ------------------------------------------------------------------- K7
size_t a11s_lm_head_keys_bytes(int32_t rows, int32_t vocab) {
    if (rows < 0 || vocab < 1) return 0;
    return (size_t)rows * (size_t)((vocab + A11S_CHUNK - 1) / A11S_CHUNK) * sizeof(uint64_t);
}

int a11s_lm_head(const void *hidden, const void *weight, int32_t rows, int32_t hidden_dim, int32_t vocab,
                 float scale, void *logits, int64_t row_stride, uint64_t *chunk_keys,
                 void *workspace, size_t workspace_bytes, void *stream) {
    if (rows < 0 || hidden_dim < 8 || vocab < 8) return fail(A11S_EINVAL, "a11s_lm_head: bad sizes");
    if (hidden_dim % 8 || vocab % 8 || row_stride % 8)
        return fail(A11S_EINVAL, "a11s_lm_head: hidden_dim, vocab and row_stride must be multiples of 8");
    if (row_stride < vocab) return fail(A11S_EINVAL, "a11s_lm_head: row_stride %lld < vocab %d", (long long)row_stride, vocab);
    if (!std::isfinite(scale)) return fail(A11S_EINVAL, "a11s_lm_head: scale is not finite");
    if (rows == 0) return empty_batch_status(workspace, workspace_bytes, stream, "a11s_lm_head: clearing status");
    if (!hidden || !weight || !logits || !workspace) return fail(A11S_EINVAL, "a11s_lm_head: null required pointer");
    if (!aligned16(hidden) || !aligned16(weight) || !aligned16(logits) || !aligned16(workspace) ||
        (chunk_keys && !aligned16(chunk_keys)))
        return fail(A11S_EINVAL, "a11s_lm_head: tensors must be 16-byte aligned");
    if (workspace_bytes < 256) return fail(A11S_ENOSPACE, "a11s_lm_head: workspace %zu < 256 bytes", workspace_bytes);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(workspace, 0, sizeof(a11s::StatusWord), s);
    if (e != cudaSuccess) return cuda_fail(e, "a11s_lm_head: clearing status");
    a11s::LmHeadArgs a{};
    a.hidden = hidden;
    a.weight = weight;
    a.rows = rows;
    a.V = vocab;
    a.K = hidden_dim;
    a.scale = scale;
    a.logits = logits;
    a.ldl = row_stride;
    a.keys = reinterpret_cast<unsigned long long *>(chunk_keys);
    a.status = reinterpret_cast<a11s::StatusWord *>(workspace);
    e = a11s::launch_lm_head(a, s);
    if (e != cudaSuccess) return cuda_fail(e, "a11s_lm_head: launch");
    return A11S_OK;
}

// ------------------------------------------------------------------- K2
size_t a11s_tree_attention_workspace_bytes(int32_t batch, int32_t max_nodes, int32_t num_q_heads,
                                           int32_t num_kv_heads, int32_t head_dim,
                                           int32_t max_kv_len) {
    if (batch < 0 || max_nodes < 1 || num_q_heads < 1 || num_kv_heads < 1 || head_dim < 1)
        return 0;
    const int splits = a11s::tree_attention_splits(batch, max_nodes, num_q_heads, num_kv_heads, max_kv_len);
    return kHeaderBytes + up256(a11s::tree_attention_partials_bytes(batch, max_nodes, num_q_heads,
                                                                    head_dim, splits));
}

int a11s_tree_attention(const void *q, const void *k_pool, const void *v_pool, int32_t num_pages,
                        const int32_t *page_table, int32_t max_pages_per_seq,
                        const int32_t *ctx_lens, const int32_t *parents, const int32_t *n_nodes,
                        int32_t batch, int32_t max_nodes, int32_t num_q_heads,
                        int32_t num_kv_heads, int32_t head_dim, int32_t max_kv_len, float scale,
                        void *out, float *lse, void *workspace, size_t workspace_bytes,
                        void *stream) {
    if (head_dim != 128) return fail(A11S_EUNSUPPORTED, "a11s_tree_attention: head_dim %d != 128", head_dim);
    if (num_kv_heads < 1 || num_q_heads != 8 * num_kv_heads)
        return fail(A11S_EUNSUPPORTED, "a11s_tree_attention: needs num_q_heads == 8 * num_kv_heads");
    if (max_nodes < 1 || max_nodes > 64)
        return fail(A11S_EUNSUPPORTED, "a11s_tree_attention: max_nodes %d outside [1, 64]", max_nodes);
    if (batch < 0 || num_pages < 1 || max_pages_per_seq < 1 || max_kv_len < 1)
        return fail(A11S_EINVAL, "a11s_tree_attention: non-positive size");
    if ((int64_t)max_pages_per_seq * A11S_PAGE_TOKENS < max_kv_len)
        return fail(A11S_EINVAL, "a11s_tree_attention: page table shorter than max_kv_len");
    if (!(scale > 0.0f) || !std::isfinite(scale)) return fail(A11S_EINVAL, "a11s_tree_attention: bad scale");
    if (batch == 0) return empty_batch_status(workspace, workspace_bytes, stream, "a11s_tree_attention: clearing status");
    if (!q || !k_pool || !v_pool || !page_table || !ctx_lens || !parents || !out || !workspace)
        return fail(A11S_EINVAL, "a11s_tree_attention: null required pointer");
    if (!aligned16(q) || !aligned16(k_pool) || !aligned16(v_pool) || !aligned16(out) || !aligned16(workspace))
        return fail(A11S_EINVAL, "a11s_tree_attention: tensors must be 16-byte aligned");
    const size_t need = a11s_tree_attention_workspace_bytes(batch, max_nodes, num_q_heads, num_kv_heads,
                                                            head_dim, max_kv_len);
    if (workspace_bytes < need)
        return fail(A11S_ENOSPACE, "a11s_tree_attention: workspace %zu < %zu bytes", workspace_bytes, need);
    a11s::AttnArgs a{};
    a.q = q;
    a.k_pool = k_pool;
    a.v_pool = v_pool;
    a.num_pages = num_pages;
    a.page_table = page_table;
    a.max_pages = max_pages_per_seq;
    a.ctx_lens = ctx_lens;
    a.parents = parents;
    a.n_nodes = n_nodes;
    a.B = batch;
    a.N = max_nodes;
    a.Hq = num_q_heads;
    a.Hkv = num_kv_heads;
    a.D = head_dim;
    a.max_kv_len = max_kv_len;
    a.scale = scale;
    a.out = out;
    a.lse = lse;
    char *ws = static_cast<char *>(workspace);
    a.status = reinterpret_cast<a11s::StatusWord *>(ws);
    a.splits = a11s::tree_attention_splits(batch, max_nodes, num_q_heads, num_kv_heads, max_kv_len);
    a.part_o = reinterpret_cast<float *>(ws + kHeaderBytes);
    a.part_ml = a.part_o + (size_t)a.splits * batch * max_nodes * num_q_heads * head_dim;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(ws, 0, sizeof(a11s::StatusWord), s);
    if (e != cudaSuccess) return cuda_fail(e, "a11s_tree_attention: clearing status");
    e = a11s::launch_tree_attention(a, s);
    if (e != cudaSuccess) return cuda_fail(e, "a11s_tree_attention: launch");
    return A11S_OK;
}

}  // extern "C"
