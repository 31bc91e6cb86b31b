// kernels.h - internal launch interfaces between the C ABI (api.cu) and the kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace a11s {

struct StatusWord;

struct AcceptArgs {
    const void *target;
    const void *draft;
    int64_t stride;  // elements between rows
    float k;         // log2(e) / max(T, 1e-5), rounded to float on the host
    const float *uniforms;
    const int32_t *tokens;
    const int32_t *parents;
    const int32_t *n_nodes;
    int32_t B, N, V, nch, rows_per_seq, units_per_seq, slice;
    int32_t *accept_len;
    int32_t *acc_nodes;
    int32_t *acc_tokens;
    int32_t *bonus;
    float *node_probs;
    long long *stats;
    float *recs;        // [B][rows_per_seq][nch] chunk maxima of every live row (NaN-propagating),
                        // 0xFFFFFFFF until written; rows are p rows 0..N-1, then q rows (DRAFT)
    int32_t *arg;       // [B][N][nch] first position of the chunk maximum in the chunk (GREEDY), else
                        // null; -1 until written
    int32_t wait_records;  // the walk may wait for other blocks' records: every walking block is
                           // resident with at least as many slots left for the bulk pass
    unsigned long long *root_sums;  // [B][2][nch] weight sums of the root rows (p, q)
    StatusWord *status;
    // Row passes of the sampling walks shared with helper blocks (null in GREEDY):
    // per sequence a job of job_stride bytes (SharedPass, then int32 frames fr[nch],
    // qfr[nch] and uint64 chunk sums[nch], qsums[nch]); walkers_done counts finished walks.
    char *jobs;
    int64_t job_stride;
    int32_t *walkers_done;
    int32_t bulk_rows;    // grid rows 0 .. bulk_rows-1 walk and stream; rows beyond help (sampling modes)
    int32_t root_blocks;  // grid rows 1 .. root_blocks take the root units, one per warp (0: the walker does)
    int32_t root_pairs;   // streaming rows interleaved with the root rows (<= root_blocks, <= streaming rows)
    int32_t rr;           // > 0: one wave, grid rows 1 .. rr take every unit round-robin (slice, root_blocks unused)
    const unsigned long long *keys;  // chunk keys of the LM head ([B * N][nch]): records come from them, no bulk pass
};

cudaError_t launch_accept(int mode, bool bf16, const AcceptArgs &a, int grid_y, cudaStream_t s);

struct LmHeadArgs {
    const void *hidden;  // bf16 [rows][K]
    const void *weight;  // bf16 [V][K]
    int32_t rows, V;
    int64_t K;
    float scale;
    void *logits;        // bf16 [rows][ldl]
    int64_t ldl;
    unsigned long long *keys;  // [rows][ceil(V / 2048)] or null
    StatusWord *status;
};
cudaError_t launch_lm_head(const LmHeadArgs &a, cudaStream_t s);
// Clears the status word and the 16 bytes after it, marks every record unwritten
// (bytes: a multiple of 16) and zeroes `zero_bytes` at `zero` (a multiple of 16;
// nullable).
cudaError_t launch_accept_init(StatusWord *st, void *recs, size_t bytes, void *zero, size_t zero_bytes,
                               cudaStream_t s);
// Recorded mode: clears the status word and its counters, zeroes the jobs
// area, and writes every live row's records from the chunk keys (the root
// rows' stay unwritten in the sampling modes: the root blocks publish them
// with their weight sums); reports ENONFINITE for a NaN / +Inf maximum.
cudaError_t launch_accept_keys_init(int mode, const AcceptArgs &a, void *zero, size_t zero_bytes, cudaStream_t s);
// Bytes of one sequence's shared-pass area (sampling modes).
size_t accept_job_bytes(int nch);

struct CompactArgs {
    char *k_pool;
    char *v_pool;
    int32_t num_layers;
    int64_t layer_stride_bytes;
    int32_t num_pages;
    int32_t row_bytes;
    int32_t *page_table;
    int32_t max_pages;
    int32_t *seq_lens;
    const int32_t *accept_len;
    const int32_t *accepted_nodes;
    const int32_t *n_nodes;
    int32_t B, N;
    int32_t *freed_pages;
    int32_t *n_freed;
    StatusWord *status;
};

cudaError_t launch_kv_compact(const CompactArgs &a, cudaStream_t s);

struct NgramArgs {
    const int32_t *table;
    int32_t log2_buckets, slots;
    const int32_t *last_tokens;
    int32_t B, width_root, width_inner, max_depth, max_nodes;
    int32_t *tokens, *parents, *depths, *n_nodes;
};

cudaError_t launch_ngram_expand(const NgramArgs &a, cudaStream_t s);

struct NgramUpdateArgs {
    int32_t *table;
    int32_t log2_buckets, slots;
    const int32_t *history;  // [B][stride]
    const int32_t *lens;
    int32_t B, stride;
    int32_t cap;             // shared-memory keys: a power of two >= B * max(0, stride - 2)
    int32_t *status;
};

cudaError_t launch_ngram_update(const NgramUpdateArgs &a, cudaStream_t s);

struct NextRootsArgs {
    const int32_t *tree_tokens, *accepted_tokens, *accept_len, *bonus;  // [B][N], [B][N], [B], [B]
    int32_t B, N;
    int32_t *last_tokens;              // [B][2], updated in place
    int32_t *history;                  // [B][history_stride] or null
    int32_t history_stride;
    int32_t *history_len;              // [B] (with history)
};

cudaError_t launch_next_roots(const NextRootsArgs &a, cudaStream_t s);

struct KvPagesArgs {
    int32_t *free_stack, *free_top;  // LIFO of free page ids, entries [0, *free_top)
    int32_t num_pages;
    int32_t *page_table;             // [B][max_pages], -1 = no page
    int32_t max_pages;
    int32_t *seq_lens;
    const int32_t *counts;  // reserve: tokens to add; free: nonzero = free the sequence; release: list lengths
    const int32_t *list;    // release: [B][list_stride] page ids
    int32_t list_stride, B;
    int32_t *status;        // device int32[2]: code, detail
};

cudaError_t launch_kv_pool_init(int32_t *stack, int32_t *top, int32_t n, cudaStream_t s);
cudaError_t launch_kv_reserve(const KvPagesArgs &a, cudaStream_t s);
cudaError_t launch_kv_push(const KvPagesArgs &a, bool whole, cudaStream_t s);

struct AttnArgs {
    const void *q;
    const void *k_pool;
    const void *v_pool;
    int32_t num_pages;
    const int32_t *page_table;
    int32_t max_pages;
    const int32_t *ctx_lens;
    const int32_t *parents;
    const int32_t *n_nodes;
    int32_t B, N, Hq, Hkv, D, max_kv_len;
    float scale;
    void *out;
    float *lse;
    // split-KV partials (workspace)
    float *part_o;    // [splits][B][N][Hq][D]
    float *part_ml;   // [splits][B][N][Hq][2]  (running max in log2 units, sum)
    int32_t splits, kv_per_split;
    StatusWord *status;
};

cudaError_t launch_tree_attention(const AttnArgs &a, cudaStream_t s);

cudaError_t launch_verify_chain(const float *draft, const float *target, const float *uni, int B, int n,
                                int32_t *accepted_len, int32_t *last_idx, StatusWord *st, cudaStream_t s);

// Records `msg` as this thread's a11s_last_error() and returns `code`.
int set_error(int code, const char *msg);
size_t tree_attention_partials_bytes(int32_t B, int32_t N, int32_t Hq, int32_t D, int32_t splits);
int tree_attention_splits(int32_t B, int32_t N, int32_t Hq, int32_t Hkv, int32_t max_kv_len);

}  // namespace a11s
