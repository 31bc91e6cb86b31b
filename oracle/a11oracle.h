/*
 * a11oracle.h - CPU oracle for the speculative-decoding hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker the CUDA kernels are compared
 * against; only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * --impl reference legs may load it. The product path never calls it.
 *
 * Every function mirrors one entry point of include/a11spec.h with host
 * pointers and fp32 logits (bf16 inputs are widened exactly by the caller).
 * Pinning: the chain-acceptance rule is checked against the reference's own
 * SpeculativeTreeVerifier::verify_draft_tokens (compiled into oracle/_ref from
 * src/engine/speculative_verifier.cpp) and its test vectors
 * (tests/test_speculative_verifier.cpp). The softmax arithmetic, the tree
 * walk, residual resampling, tree attention, compaction and n-gram expansion
 * have no reference implementation to pin against ("parity unpinned" for
 * those parts; attention is checked against torch restating engine/pipeline.py:386-402).
 */
#ifndef A11ORACLE_H
#define A11ORACLE_H
#include <stdint.h>
#include <stddef.h>

#define OR_CHUNK 2048

int  or_abi_version(void);
/* Deterministic fixed-point exp2 weight of logit l in frame c (see a11oracle.c). */
uint64_t or_weight(float l, float k, int32_t c);
float    or_exp2_poly(float f);
float    or_temperature_k(float temperature);

/* Chunk records of one row: cmax[j] (float chunk max), frame[j], sum[j]. */
void or_chunk_records(const float *row, int32_t vocab, float k, float *cmax, int32_t *frame,
                      uint64_t *sum);

/* Acceptance; returns status (0 ok, A11S_* code otherwise). Same semantics as a11s_accept. */
int or_accept(int32_t mode, const float *target, const float *draft, int64_t row_stride,
              float temperature, const float *uniforms, const int32_t *tokens,
              const int32_t *parents, const int32_t *n_nodes, int32_t batch, int32_t max_nodes,
              int32_t vocab, int32_t *accept_len, int32_t *accepted_nodes,
              int32_t *accepted_tokens, int32_t *bonus, float *node_probs, int64_t *stats);

/* Chain acceptance on per-token probabilities (a11s_verify_chain). */
float or_exp_neg(float x);
int or_verify_chain(const float *draft, const float *target, const float *uniforms, int32_t batch,
                    int32_t n, int32_t *accepted_len, int32_t *last_idx);

/* Tree attention in fp32 (q, k_pool, v_pool given as fp32 widened from bf16). */
int or_tree_attention(const float *q, const float *k_pool, const float *v_pool, int32_t num_pages,
                      const int32_t *page_table, int32_t max_pages_per_seq,
                      const int32_t *ctx_lens, const int32_t *parents, const int32_t *n_nodes,
                      int32_t batch, int32_t max_nodes, int32_t num_q_heads,
                      int32_t num_kv_heads, int32_t head_dim, float scale, float *out,
                      float *lse);

int or_kv_compact(uint8_t *k_pool, uint8_t *v_pool, int32_t num_layers, int64_t layer_stride,
                  int32_t num_pages, int32_t row_elems, int32_t elem_bytes, int32_t *page_table,
                  int32_t max_pages_per_seq, int32_t *seq_lens, const int32_t *accept_len,
                  const int32_t *accepted_nodes, const int32_t *n_nodes, int32_t batch,
                  int32_t max_nodes, int32_t *freed_pages, int32_t *n_freed);

/* Page allocator of the paged KV cache (src/cuda/paged_kv_cache.cu:85-149). */
int or_kv_reserve(int32_t *stack, int32_t *top, int32_t num_pages, int32_t *page_table, int32_t max_pages,
                  int32_t *seq_lens, const int32_t *n_new, int32_t batch, int32_t *detail);
int or_kv_release(int32_t *stack, int32_t *top, int32_t num_pages, const int32_t *freed_pages,
                  int32_t freed_stride, const int32_t *n_freed, int32_t batch, int32_t *detail);
int or_kv_free_sequences(int32_t *stack, int32_t *top, int32_t num_pages, int32_t *page_table, int32_t max_pages,
                         int32_t *seq_lens, const int32_t *free_mask, int32_t batch, int32_t *detail);

uint32_t or_ngram_bucket(int32_t a, int32_t b, int32_t log2_buckets);
/* Learning committed trigrams into the table (a11s_ngram_update), serial. */
int or_ngram_update(int32_t *table, int32_t log2_buckets, int32_t slots, const int32_t *history,
                    int32_t stride, const int32_t *lens, int32_t batch, int32_t *detail);
int or_ngram_expand(const int32_t *table, int32_t log2_buckets, int32_t slots,
                    const int32_t *last_tokens, int32_t batch, int32_t width_root,
                    int32_t width_inner, int32_t max_depth, int32_t max_nodes, int32_t *tokens,
                    int32_t *parents, int32_t *depths, int32_t *n_nodes);

#endif
