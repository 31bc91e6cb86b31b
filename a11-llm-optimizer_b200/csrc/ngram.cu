// ngram.cu - K1: hashed trigram table lookup expanding a draft token tree.
//
// One warp per sequence, one tree level per round: each lane owns one node of
// the level, reads its bucket (slots x 8 bytes), selects its top-w
// continuations by count in registers, and a warp prefix sum places the
// children in breadth-first order (parents in index order, children by rank),
// stopping at max_nodes. A tree of depth D costs D dependent bucket reads.
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

__global__ void __launch_bounds__(kNgramWarps * 32) ngram_expand_kernel(const NgramArgs a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.x * kNgramWarps + warp;
    if (b >= a.B) return;
    int32_t *tk = a.tokens + (size_t)b * a.max_nodes;
    int32_t *pa = a.parents + (size_t)b * a.max_nodes;
    int32_t *de = a.depths + (size_t)b * a.max_nodes;
    for (int i = lane; i < a.max_nodes; i += 32) { tk[i] = -1; pa[i] = -1; de[i] = -1; }
    __syncwarp();
    const int32_t prev0 = a.last_tokens[2 * b], root = a.last_tokens[2 * b + 1];
    if (lane == 0) { tk[0] = root; de[0] = 0; }
    __syncwarp();
    int n = 1, lvl_start = 0, lvl_end = 1, depth = 0;
    while (lvl_start < lvl_end && n < a.max_nodes && depth < a.max_depth) {
        const int w = depth == 0 ? a.width_root : a.width_inner;
        for (int g = lvl_start; g < lvl_end && n < a.max_nodes; g += 32) {
            const int i = g + lane;
            int sel_tok[32];
            int cnt = 0;
            if (i < lvl_end) {
                const int32_t t = tk[i];
                const int32_t prev = i == 0 ? prev0 : tk[pa[i]];
                const int32_t *bk = a.table + (size_t)bucket_of(prev, t, a.log2_buckets) * a.slots * 2;
                int32_t st[32], sc[32];
                for (int s = 0; s < a.slots; ++s) { st[s] = __ldg(bk + 2 * s); sc[s] = __ldg(bk + 2 * s + 1); }
                unsigned used = 0;
                for (int r = 0; r < w; ++r) {
                    int best = -1;
                    for (int s = 0; s < a.slots; ++s) {
                        if (((used >> s) & 1u) || sc[s] <= 0) continue;
                        if (best < 0 || sc[s] > sc[best]) best = s;
                    }
                    if (best < 0) break;
                    used |= 1u << best;
                    sel_tok[cnt++] = st[best];
                }
            }
            // exclusive prefix of child counts across the lanes of this group
            int incl = cnt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            const int base = n + incl - cnt;
            for (int r = 0; r < cnt; ++r) {
                const int idx = base + r;
                if (idx < a.max_nodes) { tk[idx] = sel_tok[r]; pa[idx] = i; de[idx] = depth + 1; }
            }
            n = min(a.max_nodes, n + __shfl_sync(0xffffffffu, incl, 31));
            __syncwarp();
        }
        lvl_start = lvl_end;
        lvl_end = n;
        ++depth;
    }
    if (lane == 0) a.n_nodes[b] = n;
}

cudaError_t launch_ngram_expand(const NgramArgs &a, cudaStream_t s) {
    ngram_expand_kernel<<<(a.B + kNgramWarps - 1) / kNgramWarps, kNgramWarps * 32, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace a11s
