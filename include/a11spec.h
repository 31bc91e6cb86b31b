/*
 * a11spec.h - C ABI of the B200 speculative-decoding hot path.
 *
 * Five device steps, all asynchronous on the caller's
 * CUDA stream (passed as `void *stream`, a cudaStream_t; NULL = legacy
 * default stream):
 *
 *   a11s_ngram_expand     hashed trigram table  -> draft token tree      (K1)
 *   a11s_tree_attention   tree-masked attention over 16-token KV pages   (K2)
 *   a11s_accept           vocab softmax/argmax + acceptance + bonus draw  (K3)
 *   a11s_kv_compact       move the accepted path's KV, shrink page tables (K4)
 *   a11s_kv_reserve / a11s_kv_release / a11s_kv_free_sequences
 *                         the page allocator of the paged KV cache    (K5)
 *   a11s_ngram_update     the n-gram table learns committed tokens    (K6)
 *   a11s_next_roots       next roots and committed-token rows of a step (K6 input)
 *   a11s_lm_head          tree-node LM head, chunk records in its epilogue (K7)
 *
 * Conventions shared by every entry point
 *   - All tensor arguments are caller-owned DEVICE pointers, row-major and
 *     densely packed unless a stride argument says otherwise. Nothing here
 *     allocates device memory or synchronises the stream. Scratch memory is the
 *     caller's `workspace`, sized by the matching *_workspace_bytes() call.
 *   - Return value: A11S_OK when the arguments were valid and the kernels were
 *     enqueued; otherwise an A11S_E* code and a message in a11s_last_error().
 *     Errors found on the device (a token id >= vocab, a page id outside the
 *     pool, a non-finite logit) are recorded in the workspace status word and
 *     read back with a11s_read_status(); the kernels never trap.
 *   - A tree of N nodes is stored structure-of-arrays per sequence:
 *     tokens[b][i], parents[b][i] with parents[b][0] == -1 (node 0 is the root,
 *     the last token already accepted) and 0 <= parents[b][i] < i for i >= 1,
 *     and n_nodes[b] <= max_nodes live nodes (NULL means every sequence has
 *     max_nodes nodes). Node i's logits row is the target distribution AFTER
 *     node i (the row used to judge node i's children and to draw a bonus).
 *   - Logits rows are fp32 or bf16 (A11S_F32 / A11S_BF16).
 *
 * Reference interfaces these replace (paths inside the reference project):
 *   engine/speculative.py:4-34                 SpeculativeDecoder (Python)
 *   include/engine/speculative_verifier.hpp:59-125, src/engine/speculative_verifier.cpp:84-135
 *                                              SpeculativeTreeVerifier (C++)
 *   src/cuda/tree_verification.cu:108-210      tree_verify_kernel_launch / tree_verify (CUDA, unbound)
 *   include/cuda/paged_kv_cache.hpp:12-67      PagedKVCacheManager block tables (16-token blocks)
 *   engine/kv_cache.py:14-21                   KVPage layout [page_size, n_head_kv, head_dim]
 */
#ifndef A11SPEC_H
#define A11SPEC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define A11S_ABI_VERSION 1

/* Status codes (return values and bits of the device status word). */
#define A11S_OK           0
#define A11S_EINVAL       1   /* bad host-side argument (shape, alignment, null) */
#define A11S_EBOUNDS      2   /* device: token / page / parent id out of range */
#define A11S_ECUDA        3   /* a CUDA runtime call failed */
#define A11S_ETIMEOUT     4   /* device: a bounded wait gave up */
#define A11S_ENONFINITE   5   /* device: NaN or +Inf logit (the reference throws on these,
                                 src/engine/speculative_verifier.cpp:93-97) */
#define A11S_ENOSPACE     6   /* workspace smaller than *_workspace_bytes() */
#define A11S_EUNSUPPORTED 7   /* shape outside what the kernels implement */

/* Element types. */
#define A11S_F32  0
#define A11S_BF16 1

/* Acceptance modes for a11s_accept. */
#define A11S_ACCEPT_GREEDY       0  /* accept child iff its token == argmax(parent row) */
#define A11S_ACCEPT_STOCH_ONEHOT 1  /* rejection sampling, deterministic drafts (q = one-hot) */
#define A11S_ACCEPT_STOCH_DRAFT  2  /* rejection sampling against draft logits q */

/* Page geometry of the KV pool: 16 tokens per page, as BLOCK_TOKENS in
 * include/cuda/paged_kv_cache.hpp:13 of the reference. */
#define A11S_PAGE_TOKENS 16

/* Diagnostic counters accumulated by a11s_accept when `stats` is non-NULL
 * (int64 device array of A11S_STATS_LEN). The first five mirror
 * SpecDiagnosticCounters (include/engine/speculative_verifier.hpp:31-53). */
#define A11S_STAT_STEPS_ACCEPTED   0  /* sequences with accept_len > 0            */
#define A11S_STAT_STEPS_REJECTED   1  /* sequences with accept_len == 0           */
#define A11S_STAT_FALLBACKS        2  /* == STEPS_REJECTED (bonus token only)      */
#define A11S_STAT_DRAFT_TOKENS     3  /* drafted nodes (n_nodes - 1)               */
#define A11S_STAT_TOTAL_STEPS      4  /* sequences verified                        */
#define A11S_STAT_EMITTED_TOKENS   5  /* accept_len + 1 (accepted + bonus)         */
#define A11S_STATS_LEN             6

int         a11s_abi_version(void);
/* Message of the last failed call on this host thread ("" if none). */
const char *a11s_last_error(void);
/* Copy the workspace status word to the host. SYNCHRONISES `stream`.
 * *status receives A11S_OK or the first device error code; *detail an index
 * locating it (or -1). The word is cleared by the next call that uses it. */
int a11s_read_status(const void *workspace, int32_t *status, int32_t *detail, void *stream);

/* ------------------------------------------------------------------------ K3
 * Acceptance. Replaces SpeculativeTreeVerifier::verify_draft_tokens
 * (src/engine/speculative_verifier.cpp:84-135), SpeculativeDecoder.verify_candidates
 * (engine/speculative.py:26-34) and tree_rejection_kernel (src/cuda/tree_verification.cu:71-101).
 *
 * One kernel reads every logits row once (vectorised, warp-shuffle reductions
 * over 2048-token chunks, recording each chunk's maximum), and the block that
 * reads a sequence's root row walks its tree from the root: at each accepted node the children are tried in index
 * order; the first accepted child becomes the next node; when none is accepted
 * (or the node is a leaf) the bonus token is drawn at that node.
 *
 * GREEDY: a child is accepted iff its token == argmax of the node's row
 *   (lowest index wins ties). bonus = argmax of the last accepted node's row.
 * STOCH_*: p = softmax(target/T), q = softmax(draft/T) (engine/sampler.py:16),
 *   computed by a deterministic chunked fixed-point softmax (bit-identical on
 *   every GPU and in the CPU oracle). A child with token x and uniform u is
 *   accepted by the reference's linear-space rule
 *   (src/engine/speculative_verifier.cpp:114-124): ld = clamp(q(x),1e-10,1),
 *   lt = clamp(p'(x),0,1+1e-6), accept iff u < min(1, lt/ld), where p' is the
 *   target distribution with the residual of every rejected sibling applied:
 *   ONEHOT drafts (q(x)=1): p' = p with the rejected tokens removed, renormalised;
 *   DRAFT logits: p' = normalise(max(p' - q, 0)). The bonus is drawn from p'
 *   at the final node by inverse CDF with uniforms[b][0]; uniforms[b][i] is the
 *   acceptance uniform of node i (shape [batch][max_nodes], fp32 in [0,1)).
 *
 * Outputs: accept_len[b] accepted draft nodes (root excluded);
 *   accepted_nodes[b][j], accepted_tokens[b][j] for j < accept_len (then -1),
 *   both [batch][max_nodes]; bonus[b]; node_probs[b][i] (nullable, STOCH only)
 *   = p(tokens[i]) in the parent's row before any residual, 0 for the root.
 * Rows are `row_stride` elements apart (>= vocab; multiple of 8 for bf16 and
 * of 4 for fp32; 16-byte aligned base pointers). draft_logits is used only by
 * STOCH_DRAFT and has the same layout as target_logits. Implemented sizes:
 * vocab <= 262144, max_nodes <= 256 (A11S_EUNSUPPORTED beyond).
 */
size_t a11s_accept_workspace_bytes(int32_t mode, int32_t batch, int32_t max_nodes, int32_t vocab);

int a11s_accept(int32_t mode, int32_t dtype,
                const void *target_logits, const void *draft_logits, int64_t row_stride,
                float temperature, const float *uniforms,
                const int32_t *tokens, const int32_t *parents, const int32_t *n_nodes,
                int32_t batch, int32_t max_nodes, int32_t vocab,
                int32_t *accept_len, int32_t *accepted_nodes, int32_t *accepted_tokens,
                int32_t *bonus, float *node_probs, int64_t *stats,
                void *workspace, size_t workspace_bytes, void *stream);

/* Acceptance with the chunk records taken from a11s_lm_head's chunk_keys
 * instead of a pass over the logits: the same decisions, bonus tokens,
 * node_probs and stats as a11s_accept on the same bf16 logits (the keys hold
 * exactly the chunk maxima and first positions that its pass would record).
 * Modes GREEDY and STOCH_ONEHOT (STOCH_DRAFT has draft rows the keys do not
 * cover: A11S_EUNSUPPORTED). target_logits bf16 [batch][max_nodes] rows
 * `row_stride` apart; chunk_keys uint64 [batch * max_nodes][ceil(vocab/2048)]
 * of those rows. The walk still reads the logits of the rows it visits; the
 * other rows are never read. The workspace is sized as for a11s_accept.
 * A live row whose key holds a NaN or +Inf maximum (or was never written)
 * reports A11S_ENONFINITE, as a11s_accept does for such a row. */
int a11s_accept_recorded(int32_t mode, const void *target_logits, int64_t row_stride, float temperature,
                         const float *uniforms, const int32_t *tokens, const int32_t *parents,
                         const int32_t *n_nodes, int32_t batch, int32_t max_nodes, int32_t vocab,
                         const uint64_t *chunk_keys, int32_t *accept_len, int32_t *accepted_nodes,
                         int32_t *accepted_tokens, int32_t *bonus, float *node_probs, int64_t *stats,
                         void *workspace, size_t workspace_bytes, void *stream);

/* Chain acceptance on per-token probabilities: the rule of
 * SpeculativeTreeVerifier::verify_draft_tokens (src/engine/speculative_verifier.cpp:84-135)
 * for `batch` independent chains of `n` drafts. draft, target, uniforms are
 * fp32 device arrays [batch][n]; uniforms[b][i] judges draft i (the reference
 * draws it from its thread_local std::mt19937(42), :65-69).
 * Per draft: log space iff ld < 0 || lt < 0, then a = exp(max(lt - ld, -20))
 * (this library's exp, relative error < 2e-6); otherwise ld = clamp(ld, 1e-10, 1),
 * lt = clamp(lt, 0, 1 + 1e-6), a = lt / ld. a = min(a, 1); accept iff u < a;
 * the first rejection ends the chain. accepted_len[b] and last_idx[b] (0 when
 * nothing is accepted) are written; a chain whose target row holds NaN or Inf
 * gets accepted_len = -1 and the status word ENONFINITE (the reference
 * throws, :93-97). workspace >= 256 bytes (status word). */
int a11s_verify_chain(const float *draft_probs, const float *target_probs, const float *uniforms,
                      int32_t batch, int32_t n, int32_t *accepted_len, int32_t *last_idx,
                      void *workspace, size_t workspace_bytes, void *stream);

/* Fixed-scratch variant of a11s_accept, with no counterpart in the reference.
 * For callers that cannot pass a workspace because they may not allocate
 * device memory: hosts whose HBM is owned by another allocator that forbids
 * outside cudaMalloc calls, foreign-language bindings without a device
 * allocator, decode loops that cannot afford cudaMalloc's possible device-wide
 * synchronisation. The scratch is one file-scope device array of
 * A11S_ACCEPT_STATIC_SCRATCH_BYTES (4 MiB) that every GPU loading the library
 * holds until the process exits; calls whose a11s_accept_workspace_bytes()
 * exceeds it return A11S_ENOSPACE, with the largest batch that fits in the
 * message. Every call looks up the array's device address in the context
 * current at the call (cudaGetSymbolAddress); the first lookup on a device may
 * load the library's device code, so make the first call before any stream
 * capture. All calls share the array: calls that overlap on the GPU (other
 * streams, other host threads) race and must be serialised by the caller.
 * Arguments and results are those of a11s_accept; `status` (nullable, device
 * int32[2]) receives the device status word and its detail, stream-ordered
 * after the kernel ({0, 0} for an empty batch). Allocates nothing (no
 * cudaMalloc, cudaFree or allocating library routine). */
#define A11S_ACCEPT_STATIC_SCRATCH_BYTES (4u << 20)
int a11s_accept_static(int32_t mode, int32_t dtype,
                       const void *target_logits, const void *draft_logits, int64_t row_stride,
                       float temperature, const float *uniforms,
                       const int32_t *tokens, const int32_t *parents, const int32_t *n_nodes,
                       int32_t batch, int32_t max_nodes, int32_t vocab,
                       int32_t *accept_len, int32_t *accepted_nodes, int32_t *accepted_tokens,
                       int32_t *bonus, float *node_probs, int64_t *stats, int32_t *status,
                       void *stream);

/* ------------------------------------------------------------------------ K7
 * Tree-node LM head on the tensor cores. Replaces the logits product of
 * A11Pipeline.forward_token (engine/pipeline.py:468-472, `torch.matmul(h_norm,
 * output_w.t())`) for every tree node at once, and tree_forward_pass_kernel
 * (src/cuda/tree_verification.cu:34-68, which also divides by sqrt(hidden_dim):
 * pass scale = 1/sqrt(hidden_dim) for that form).
 *
 * logits[r][v] = bf16 round-to-nearest-even of scale * sum_k hidden[r][k] *
 *   weight[v][k], the sum in fp32 on the tensor cores (order unspecified).
 * hidden bf16 [rows][hidden_dim]; weight bf16 [vocab][hidden_dim] (output_w as
 * stored); logits bf16, rows `row_stride` elements apart (>= vocab).
 * hidden_dim, vocab and row_stride multiples of 8; 16-byte aligned pointers.
 * chunk_keys (nullable) uint64 [rows][ceil(vocab / 2048)], sized by
 * a11s_lm_head_keys_bytes(): for each row and 2048-token chunk the maximum of
 * the row's bf16 logits in the chunk and the first position holding it,
 * packed for a11s_accept_recorded, which then takes its chunk records from
 * them and never streams the logits for them. -0 counts as +0 and a NaN as
 * the largest value. The call clears chunk_keys on `stream` before the
 * kernel fills them, so the caller need not initialise them.
 * workspace >= 256 bytes (status word: A11S_ETIMEOUT if a pipeline wait of the
 * kernel ran out).
 */
size_t a11s_lm_head_keys_bytes(int32_t rows, int32_t vocab);

int a11s_lm_head(const void *hidden, const void *weight, int32_t rows, int32_t hidden_dim, int32_t vocab,
                 float scale, void *logits, int64_t row_stride, uint64_t *chunk_keys,
                 void *workspace, size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------------ K2
 * Tree-masked verification attention over the paged KV pool. Replaces the
 * decode attention of engine/pipeline.py:386-402 (GQA by repeat_interleave,
 * scores in fp32 scaled by `scale`, softmax, probabilities cast to bf16, PV)
 * extended to a token tree, and tree_forward_pass_kernel
 * (src/cuda/tree_verification.cu:34-68).
 *
 * q    bf16 [batch][max_nodes][num_q_heads][head_dim]
 * k_pool, v_pool bf16 [num_pages][16][num_kv_heads][head_dim]  (engine/kv_cache.py:20-21 per page)
 * page_table int32 [batch][max_pages_per_seq]: logical page -> physical page
 * ctx_lens[b]: tokens before the tree. Node i's own K/V sit at logical position
 *   ctx_lens[b] + i. Node i attends to every context position and to tree
 *   position ctx_lens[b] + j iff j is i or an ancestor of i.
 * out  bf16 [batch][max_nodes][num_q_heads][head_dim]; lse fp32
 *   [batch][max_nodes][num_q_heads] natural-log sum-exp of the scaled scores
 *   (nullable). Rows of dead nodes (i >= n_nodes[b]) are written as zeros.
 * Implemented shapes: head_dim == 128, num_q_heads / num_kv_heads == 8,
 * max_nodes <= 64.
 */
size_t a11s_tree_attention_workspace_bytes(int32_t batch, int32_t max_nodes, int32_t num_q_heads,
                                           int32_t num_kv_heads, int32_t head_dim, int32_t max_kv_len);

int a11s_tree_attention(const void *q, const void *k_pool, const void *v_pool, int32_t num_pages,
                        const int32_t *page_table, int32_t max_pages_per_seq,
                        const int32_t *ctx_lens, const int32_t *parents, const int32_t *n_nodes,
                        int32_t batch, int32_t max_nodes, int32_t num_q_heads, int32_t num_kv_heads,
                        int32_t head_dim, int32_t max_kv_len, float scale,
                        void *out, float *lse,
                        void *workspace, size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------------ K4
 * In-place compaction of the accepted path. Replaces the host block-table
 * bookkeeping of PagedKVCacheManager::append_token / free_sequence
 * (src/cuda/paged_kv_cache.cu:120-158) for a verified tree.
 *
 * For every layer l and sequence b, the K and V rows of accepted node
 * accepted_nodes[b][j] (logical position seq_lens[b] + node) are copied
 * bit-for-bit to position seq_lens[b] + 1 + j, j < accept_len[b] (the root
 * stays at seq_lens[b]). Then seq_lens[b] += 1 + accept_len[b], and every page
 * past the new length that held tree slots (logical page index in
 * [ceil(new_len/16), ceil((old_len + n_nodes[b])/16))) is detached:
 * page_table[b][p] = -1 and its id appended to freed_pages[b][*], count in
 * n_freed[b] (freed_pages / n_freed nullable).
 * Pools: num_layers slabs `layer_stride` elements apart, each
 * [num_pages][16][row_elems] with row_elems = num_kv_heads * head_dim,
 * elem_bytes 2 (bf16/fp16) or 4 (fp32); row bytes must be a multiple of 16.
 */
int a11s_kv_compact(void *k_pool, void *v_pool, int32_t num_layers, int64_t layer_stride,
                    int32_t num_pages, int32_t row_elems, int32_t elem_bytes,
                    int32_t *page_table, int32_t max_pages_per_seq, int32_t *seq_lens,
                    const int32_t *accept_len, const int32_t *accepted_nodes,
                    const int32_t *n_nodes, int32_t batch, int32_t max_nodes,
                    int32_t *freed_pages, int32_t *n_freed, void *workspace,
                    size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------------ K5
 * The page allocator of the paged KV cache on the device. Replaces
 * PagedKVCacheManager's host bookkeeping (src/cuda/paged_kv_cache.cu:
 * init_pool 61-81, alloc_block 85-93, dealloc_block 95-101, allocate_sequence
 * 103-117, append_token 119-135, free_sequence 137-149; kv_cache.py:131-156)
 * so a decode step grows and returns pages without a host round trip.
 *
 * State in device memory: free_stack int32[num_pages] (a LIFO of free page
 * ids, entries [0, *free_top)), free_top int32[1], page_table
 * int32[batch][max_pages] (-1 = no page) and seq_lens int32[batch].
 * Invariant kept by these calls and a11s_kv_compact: an active sequence of
 * length len owns table entries 0 .. max(1, ceil(len/16)) - 1 and has -1
 * after them; an inactive one has -1 everywhere.
 *
 * Each call serves the whole batch in batch order and, within a sequence, in
 * logical page order, exactly like the reference's per-token loop. It checks
 * everything first and changes nothing on an error, which it writes to
 * `status` (device int32[2]: code, detail = offending sequence or count);
 * A11S_OK there otherwise. Calls on one pool must not overlap on the GPU (use
 * one stream): they race.
 *
 *   a11s_kv_pool_init      free_stack[i] = i, *free_top = num_pages: the
 *                          reference's initial order, so the highest id is
 *                          taken first.
 *   a11s_kv_reserve        seq_lens[b] += n_new[b] and the sequence's table
 *                          grows to max(1, ceil(len/16)) pages popped from
 *                          the stack (an inactive sequence gets its first
 *                          page, even with n_new[b] == 0: allocate_sequence).
 *                          Errors: A11S_ENOSPACE when the stack holds fewer
 *                          pages than the batch needs (the reference's "out
 *                          of physical blocks"), A11S_EBOUNDS when a table
 *                          row would exceed max_pages or a count is negative.
 *   a11s_kv_release        pushes freed_pages[b][0 .. n_freed[b]) (the lists
 *                          a11s_kv_compact produces; freed_stride entries per
 *                          row) back on the stack. A11S_EBOUNDS for ids
 *                          outside the pool or a stack overflow (double free).
 *   a11s_kv_free_sequences for every b with free_mask[b] != 0 and an active
 *                          table: pushes its pages in table order, clears the
 *                          row to -1 and sets seq_lens[b] = 0 (free_sequence).
 */
int a11s_kv_pool_init(int32_t *free_stack, int32_t *free_top, int32_t num_pages, void *stream);

int a11s_kv_reserve(int32_t *free_stack, int32_t *free_top, int32_t num_pages, int32_t *page_table,
                    int32_t max_pages, int32_t *seq_lens, const int32_t *n_new, int32_t batch,
                    int32_t *status, void *stream);

int a11s_kv_release(int32_t *free_stack, int32_t *free_top, int32_t num_pages, const int32_t *freed_pages,
                    int32_t freed_stride, const int32_t *n_freed, int32_t batch, int32_t *status,
                    void *stream);

int a11s_kv_free_sequences(int32_t *free_stack, int32_t *free_top, int32_t num_pages, int32_t *page_table,
                           int32_t max_pages, int32_t *seq_lens, const int32_t *free_mask, int32_t batch,
                           int32_t *status, void *stream);

/* ------------------------------------------------------------------------ K1
 * Hashed trigram drafting into a token tree. Replaces
 * SpeculativeDecoder.generate_draft_tokens (engine/speculative.py:13-24),
 * whose n-gram key is the last two context tokens (engine/speculative.py:21).
 *
 * table int32 [2^log2_buckets][slots][2] of (token, count); count <= 0 marks an
 *   empty slot. The bucket of the token pair (a, b) is
 *   splitmix64_finalize(((uint64)(uint32)a << 32) | (uint32)b) >> (64 - log2_buckets).
 * last_tokens int32 [batch][2]: the two newest context tokens; node 0 (the
 *   root) takes last_tokens[b][1].
 * Expansion is breadth-first: a node at depth d (root d=0) gets the top
 *   width_root (d == 0) or width_inner (d >= 1) continuations of its bucket by
 *   count (ties: lower slot first; empty slots skipped), for d < max_depth,
 *   until max_nodes nodes exist. Children of one parent are emitted
 *   consecutively, parents in index order, so parents[i] < i.
 * Outputs tokens/parents/depths [batch][max_nodes] (unused entries -1) and
 *   n_nodes[batch].
 */
int a11s_ngram_expand(const int32_t *table, int32_t log2_buckets, int32_t slots,
                      const int32_t *last_tokens, int32_t batch, int32_t width_root,
                      int32_t width_inner, int32_t max_depth, int32_t max_nodes,
                      int32_t *tokens, int32_t *parents, int32_t *depths, int32_t *n_nodes,
                      void *stream);

/* Bucket index the expansion uses for the pair (a, b); host-side helper so
 * table builders agree with the device. */
uint32_t a11s_ngram_bucket(int32_t a, int32_t b, int32_t log2_buckets);

/* ------------------------------------------------------------------------ K6
 * The n-gram table learns committed tokens: the draft loop's other half. The
 * reference's trigram draft (engine/speculative.py:13-24) has no learned
 * table; its README (N-gram spec tables) names the idea, so the rule is
 * defined here and restated by the oracle.
 *
 * Every history row b (history[b][0 .. history_len[b]), history_stride
 * entries per row) adds its trigrams (h[i-2], h[i-1], h[i]), 2 <= i < len,
 * that hold no negative token. After an acceptance step a row is
 * (last_tokens[b][0], last_tokens[b][1], accepted_tokens[b][0 .. alen), bonus[b]).
 * Trigram (x, y, z) updates the bucket of the pair (x, y), as a11s_ngram_bucket gives it: the slot holding
 * z with a count > 0 gains 1 (saturating at INT32_MAX); else the lowest slot
 * with count <= 0 becomes (z, 1); else the slot with the smallest count (the
 * lowest index among equals) is replaced by (z, 1). Updates of one bucket
 * apply in (row, position) order, so the result equals that serial loop.
 * At most A11S_NGRAM_MAX_UPDATES trigrams per call: batch * (history_stride - 2)
 * beyond it gives A11S_EUNSUPPORTED (split the batch). `status` (device
 * int32[2]) receives A11S_OK and the number of trigrams applied, or
 * A11S_EBOUNDS and the first row whose length is outside [0, stride] (then
 * nothing changes). One block of 1024 threads; calls on one table must not
 * overlap on the GPU.
 */
#define A11S_NGRAM_MAX_UPDATES 8192
int a11s_ngram_update(int32_t *table, int32_t log2_buckets, int32_t slots, const int32_t *history,
                      int32_t history_stride, const int32_t *history_len, int32_t batch, int32_t *status,
                      void *stream);

/* The decode loop's hand-over from one speculative step to the next, the role
 * of the reference's sample -> forward_token feed (engine/pipeline.py:491-503):
 * per sequence b, after a11s_accept,
 *   last_tokens[b] <- (accepted_tokens[b][alen - 1], or tree_tokens[b][0] (the
 *                      old root) when alen = 0;  max(bonus[b], 0))
 * and, when `history` is not NULL, the committed-token row for
 * a11s_ngram_update, built from the OLD pair:
 *   history[b] = (last_tokens[b][0], last_tokens[b][1], accepted_tokens[b][0 .. alen),
 *                 bonus[b], then -1 up to history_stride), history_len[b] = alen + 3,
 * with alen = accept_len[b] clamped to [0, max_nodes]. last_tokens int32 [batch][2]
 * is updated in place; tree_tokens and accepted_tokens are [batch][max_nodes];
 * history_stride >= max_nodes + 3. One launch, one warp per sequence.
 */
int a11s_next_roots(const int32_t *tree_tokens, const int32_t *accepted_tokens, const int32_t *accept_len,
                    const int32_t *bonus, int32_t batch, int32_t max_nodes, int32_t *last_tokens, int32_t *history,
                    int32_t history_stride, int32_t *history_len, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* A11SPEC_H */
