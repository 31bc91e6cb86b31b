// ngram.cu - K1: hashed trigram table lookup expanding a draft token tree.
//
// One warp per sequence, one tree level per round: each lane owns one node of
// the level, reads its bucket (slots x 8 bytes, 16-byte loads), selects its
// top-w continuations by count in registers, and a warp prefix sum places the
// children in breadth-first order (parents in index order, children by rank),
// stopping at max_nodes. The tree grows in shared memory and is written out
// once. A tree of depth D costs D dependent bucket reads.
// Semantics: include/a11spec.h (a11s_ngram_expand); the key is the last two
// tokens, as engine/speculative.py:21 of the reference.
#include "common.cuh"
#include "kernels.h"

namespace a11s {

__device__ __forceinline__ uint32_t bucket_of(int32_t a, int32_t b, int log2_buckets) {
    uint64_t z = ((uint64_t)(uint32_t)a << 32) | (uint32_t)b;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    z ^= z >> 31;
    return (uint32_t)(z >> (64 - log2_buckets));
}

constexpr int kNgramWarps = 4;
static_assert(kNgramWarps * 3 * A11S_MAX_NODES * sizeof(int32_t) <= 48 * 1024,
              "the per-warp trees fit the default dynamic shared memory");

// kSlots: a compile-time bound on a.slots, so the bucket and the selection
// state stay in registers (every slot index is a constant after unrolling).
template <int kSlots>
__global__ void __launch_bounds__(kNgramWarps * 32) ngram_expand_kernel(const NgramArgs a) {
    extern __shared__ int32_t ng_tree[];  // per warp: tokens, parents, depths [max_nodes] each
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.x * kNgramWarps + warp;
    if (b >= a.B) return;
    const int M = a.max_nodes;
    // The tree grows in shared memory (each level reads the tokens of the one
    // before) and is written out once at the end.
    int32_t *stk = ng_tree + (size_t)warp * 3 * M, *spa = stk + M, *sde = spa + M;
    const int32_t prev0 = a.last_tokens[2 * b], root = a.last_tokens[2 * b + 1];
    if (lane == 0) { stk[0] = root; spa[0] = -1; sde[0] = 0; }
    __syncwarp();
    // 16-byte bucket reads (two slots each) when the table allows them
    const bool vec = (a.slots & 1) == 0 && (reinterpret_cast<uintptr_t>(a.table) & 15) == 0;
    int n = 1, lvl_start = 0, lvl_end = 1, depth = 0;
    while (lvl_start < lvl_end && n < M && depth < a.max_depth) {
        const int w = depth == 0 ? a.width_root : a.width_inner;
        for (int g = lvl_start; g < lvl_end && n < M; g += 32) {
            const int i = g + lane;
            int32_t st[kSlots], sc[kSlots];
#pragma unroll
            for (int s2 = 0; s2 < kSlots; ++s2) sc[s2] = 0;  // slots past a.slots count as empty
            int cnt = 0;
            if (i < lvl_end) {
                const int32_t t = stk[i];
                const int32_t prev = i == 0 ? prev0 : stk[spa[i]];
                const int32_t *bk = a.table + (size_t)bucket_of(prev, t, a.log2_buckets) * a.slots * 2;
                if (vec) {
#pragma unroll
                    for (int s2 = 0; s2 < kSlots; s2 += 2) {
                        if (s2 < a.slots) {
                            const int4 v = __ldg(reinterpret_cast<const int4 *>(bk + 2 * s2));
                            st[s2] = v.x; sc[s2] = v.y;
                            if (s2 + 1 < kSlots) { st[s2 + 1] = v.z; sc[s2 + 1] = v.w; }
                        }
                    }
                } else {
#pragma unroll
                    for (int s2 = 0; s2 < kSlots; ++s2)
                        if (s2 < a.slots) { st[s2] = __ldg(bk + 2 * s2); sc[s2] = __ldg(bk + 2 * s2 + 1); }
                }
                // how many continuations: up to w slots with a positive count
#pragma unroll
                for (int s2 = 0; s2 < kSlots; ++s2) cnt += sc[s2] > 0 ? 1 : 0;
                cnt = min(cnt, w);
            }
            // exclusive prefix of child counts across the lanes of this group
            int incl = cnt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            const int base = n + incl - cnt;
            // children in rank order: highest count first, lower slot among equals
            unsigned used = 0;
            for (int r = 0; r < cnt; ++r) {
                int best = -1, bc = 0, bt = 0;
#pragma unroll
                for (int s2 = 0; s2 < kSlots; ++s2) {
                    const bool take = !((used >> s2) & 1u) && sc[s2] > 0 && (best < 0 || sc[s2] > bc);
                    if (take) { best = s2; bc = sc[s2]; bt = st[s2]; }
                }
                used |= 1u << best;
                const int idx = base + r;
                if (idx < M) { stk[idx] = bt; spa[idx] = i; sde[idx] = depth + 1; }
            }
            n = min(M, n + __shfl_sync(0xffffffffu, incl, 31));
            __syncwarp();
        }
        lvl_start = lvl_end;
        lvl_end = n;
        ++depth;
    }
    int32_t *tk = a.tokens + (size_t)b * M;
    int32_t *pa = a.parents + (size_t)b * M;
    int32_t *de = a.depths + (size_t)b * M;
    for (int i = lane; i < M; i += 32) {
        const bool in = i < n;
        tk[i] = in ? stk[i] : -1;
        pa[i] = in ? spa[i] : -1;
        de[i] = in ? sde[i] : -1;
    }
    if (lane == 0) a.n_nodes[b] = n;
}

cudaError_t launch_ngram_expand(const NgramArgs &a, cudaStream_t s) {
    const size_t smem = (size_t)kNgramWarps * 3 * a.max_nodes * sizeof(int32_t);  // <= 48 KB for max_nodes <= 1024
    const unsigned grid = (a.B + kNgramWarps - 1) / kNgramWarps;
    if (a.slots <= 4) ngram_expand_kernel<4><<<grid, kNgramWarps * 32, smem, s>>>(a);
    else if (a.slots <= 8) ngram_expand_kernel<8><<<grid, kNgramWarps * 32, smem, s>>>(a);
    else if (a.slots <= 16) ngram_expand_kernel<16><<<grid, kNgramWarps * 32, smem, s>>>(a);
    else ngram_expand_kernel<32><<<grid, kNgramWarps * 32, smem, s>>>(a);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// K6: the table learns the trigrams of committed tokens.
//
// Every history row b contributes the trigrams (h[i-2], h[i-1], h[i]) for
// 2 <= i < len[b] whose three tokens are >= 0. A trigram (x, y, z) updates
// bucket(x, y): the slot holding z with a positive count gains 1 (saturating);
// else the lowest slot with count <= 0 becomes (z, 1); else the slot with the
// smallest count (lowest index among equals) is replaced by (z, 1). Updates
// of one bucket apply in (row, position) order; buckets are independent.
//
// One block: the updates' keys (bucket << 32 | history index) go to shared
// memory, a bitonic sort orders them, and the first thread of each bucket's
// run applies that run in order. So the result equals the serial loop over
// rows and positions, whatever the contention on a bucket.
// ---------------------------------------------------------------------------
constexpr int kUpdThreads = 1024;

__global__ void __launch_bounds__(kUpdThreads, 1) ngram_update_kernel(const NgramUpdateArgs a) {
    extern __shared__ unsigned long long keys[];  // a.cap entries
    __shared__ int ws[kUpdThreads / 32 + 1];
    __shared__ int s_bad;
    if (threadIdx.x == 0) s_bad = INT32_MAX;
    __syncthreads();
    // validate the lengths first: nothing changes on an error
    for (int b = threadIdx.x; b < a.B; b += blockDim.x) {
        const int n = a.lens[b];
        if (n < 0 || n > a.stride) atomicMin(&s_bad, b);
    }
    __syncthreads();
    if (s_bad != INT32_MAX) {
        if (threadIdx.x == 0) { a.status[0] = A11S_EBOUNDS; a.status[1] = s_bad; }
        return;
    }
    // gather the keys: a row's trigram slots in order, rows in order
    __shared__ int s_total;
    if (threadIdx.x == 0) s_total = 0;
    __syncthreads();
    for (int b = 0; b < a.B; ++b) {  // rows are few: one pass per row, all threads over its positions
        const int n = a.lens[b];
        const int32_t *h = a.history + (size_t)b * a.stride;
        const int base = s_total;
        int cnt = 0;
        for (int i0 = 2; i0 < n; i0 += blockDim.x) {
            const int i = i0 + threadIdx.x;
            const bool ok = i < n && h[i - 2] >= 0 && h[i - 1] >= 0 && h[i] >= 0;
            // block-wide compaction of the valid positions, order kept
            const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
            const unsigned m = __ballot_sync(0xffffffffu, ok);
            if (lane == 0) ws[warp] = __popc(m);
            __syncthreads();
            if (threadIdx.x == 0) {
                int acc = 0;
                for (int w = 0; w < (int)(blockDim.x / 32); ++w) { const int t = ws[w]; ws[w] = acc; acc += t; }
                ws[blockDim.x / 32] = acc;
            }
            __syncthreads();
            if (ok) {
                const int slot = base + cnt + ws[warp] + __popc(m & ((1u << lane) - 1u));
                const uint32_t bk = bucket_of(h[i - 2], h[i - 1], a.log2_buckets);
                keys[slot] = ((unsigned long long)bk << 32) | (uint32_t)((size_t)b * a.stride + i);
            }
            cnt += ws[blockDim.x / 32];
            __syncthreads();
        }
        if (threadIdx.x == 0) s_total = base + cnt;
        __syncthreads();
    }
    const int total = s_total;
    int n2 = 1;
    while (n2 < total) n2 <<= 1;
    for (int i = total + threadIdx.x; i < n2; i += blockDim.x) keys[i] = ~0ull;  // padding sorts last
    __syncthreads();
    // bitonic sort, ascending
    for (int k = 2; k <= n2; k <<= 1)
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n2; i += blockDim.x) {
                const int l = i ^ j;
                if (l > i) {
                    const unsigned long long x = keys[i], y = keys[l];
                    const bool up = (i & k) == 0;
                    if ((x > y) == up) { keys[i] = y; keys[l] = x; }
                }
            }
            __syncthreads();
        }
    // the first thread of each bucket's run applies the run in order
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
        const uint32_t bk = (uint32_t)(keys[i] >> 32);
        if (i > 0 && (uint32_t)(keys[i - 1] >> 32) == bk) continue;
        int32_t *slots = a.table + (size_t)bk * a.slots * 2;
        for (int r = i; r < total && (uint32_t)(keys[r] >> 32) == bk; ++r) {
            const int32_t z = a.history[(uint32_t)keys[r]];
            int hit = -1, empty = -1, low = 0;
            for (int s = 0; s < a.slots; ++s) {
                const int32_t t = slots[2 * s], c = slots[2 * s + 1];
                if (c > 0 && t == z && hit < 0) hit = s;
                if (c <= 0 && empty < 0) empty = s;
                if (c < slots[2 * low + 1]) low = s;
            }
            if (hit >= 0) {
                if (slots[2 * hit + 1] < INT32_MAX) slots[2 * hit + 1] += 1;
            } else {
                const int s = empty >= 0 ? empty : low;
                slots[2 * s] = z;
                slots[2 * s + 1] = 1;
            }
        }
    }
    if (threadIdx.x == 0) { a.status[0] = A11S_OK; a.status[1] = total; }
}

cudaError_t launch_ngram_update(const NgramUpdateArgs &a, cudaStream_t s) {
    const size_t smem = (size_t)a.cap * sizeof(unsigned long long);
    cudaError_t e = cudaFuncSetAttribute(ngram_update_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    ngram_update_kernel<<<1, kUpdThreads, smem, s>>>(a);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// After an acceptance step, per sequence (one warp): the committed-token row
// for K6 (old root pair, accepted tokens, bonus, then -1) and the next tree's
// root pair (last accepted token, or the old root when nothing was accepted;
// the bonus, 0 if none). The old pair is read by every lane before lane 0
// overwrites it.
// ---------------------------------------------------------------------------
__global__ void next_roots_kernel(const NextRootsArgs a) {
    const int b = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (b >= a.B) return;
    const int N = a.N;
    const int32_t *acc = a.accepted_tokens + (size_t)b * N;
    const int alen = min(max(a.accept_len[b], 0), N);
    const int32_t bonus = a.bonus[b];
    const int32_t old0 = a.last_tokens[2 * b], old1 = a.last_tokens[2 * b + 1];
    if (a.history) {
        int32_t *h = a.history + (size_t)b * a.history_stride;
        for (int i = lane; i < a.history_stride; i += 32) {
            int32_t v = -1;
            if (i == 0) v = old0;
            else if (i == 1) v = old1;
            else if (i - 2 < alen) v = acc[i - 2];
            else if (i - 2 == alen) v = bonus;
            h[i] = v;
        }
        if (lane == 0) a.history_len[b] = alen + 3;
    }
    __syncwarp();
    if (lane == 0) {
        a.last_tokens[2 * b] = alen > 0 ? acc[alen - 1] : a.tree_tokens[(size_t)b * N];
        a.last_tokens[2 * b + 1] = bonus < 0 ? 0 : bonus;
    }
}

cudaError_t launch_next_roots(const NextRootsArgs &a, cudaStream_t s) {
    const unsigned blocks = (unsigned)((a.B + 7) / 8);  // 8 sequences (warps) per block
    next_roots_kernel<<<blocks, 256, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace a11s
