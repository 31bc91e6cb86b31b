// compact.cu - K4: in-place compaction of the accepted path's KV + page-table shrink.
//
// Kernel 1 (grid: batch x layers): for each sequence and layer, copy the K and
// V rows of the accepted nodes (logical position len + node) to len + 1 + j.
// A destination may be an earlier source of the same sequence (e.g. path
// 2 -> 5: position len+2 is read for j=0 and written for j=1), so each block
// loads a full column slab of every accepted row into registers before it
// stores any of it; column slabs are disjoint, which makes the copy exact.
// Kernel 2 (one thread per sequence): new length, detached pages, freed list.
// Semantics: include/a11spec.h (a11s_kv_compact); block rule of the reference
// src/cuda/paged_kv_cache.cu:129-135 (a new block when length > blocks * 16).
#include "common.cuh"
#include "kernels.h"

namespace a11s {

constexpr int kCompactThreads = 256;
constexpr int kCompactRegs = 8;  // uint4 held per thread per round

__global__ void __launch_bounds__(kCompactThreads) kv_compact_copy(const CompactArgs a) {
    const int b = blockIdx.x, layer = blockIdx.y;
    const int n = a.n_nodes ? a.n_nodes[b] : a.N;
    const int alen = a.accept_len[b];
    const int L = a.seq_lens[b];
    if (n < 1 || n > a.N || alen < 0 || alen >= n) {
        if (threadIdx.x == 0 && layer == 0) report(a.status, A11S_EBOUNDS, b);
        return;
    }
    if (alen == 0) return;
    const int32_t *pt = a.page_table + (size_t)b * a.max_pages;
    const int32_t *nodes = a.accepted_nodes + (size_t)b * a.N;
    const int row16 = a.row_bytes / 16;
    const int cols_per_round = max(1, (kCompactThreads * kCompactRegs) / alen);
    for (int pool = 0; pool < 2; ++pool) {
        char *base = (pool ? a.v_pool : a.k_pool) + (size_t)layer * a.layer_stride_bytes;
        for (int col0 = 0; col0 < row16; col0 += cols_per_round) {
            const int cols = min(cols_per_round, row16 - col0);
            const int items = cols * alen;  // item = c * alen + j
            uint4 reg[kCompactRegs];
            long long dst_off[kCompactRegs];
#pragma unroll
            for (int r = 0; r < kCompactRegs; ++r) {
                const int it = threadIdx.x + r * kCompactThreads;
                dst_off[r] = -1;
                if (it < items) {
                    const int c = col0 + it / alen, j = it % alen;
                    const int node = nodes[j];
                    const int sp = L + node, dp = L + 1 + j;
                    const int sl = sp / A11S_PAGE_TOKENS, dl = dp / A11S_PAGE_TOKENS;
                    const int spg = (node >= 1 && node < n && sl < a.max_pages) ? pt[sl] : -1;
                    const int dpg = dl < a.max_pages ? pt[dl] : -1;
                    if (spg < 0 || spg >= a.num_pages || dpg < 0 || dpg >= a.num_pages) {
                        report(a.status, A11S_EBOUNDS, b);
                        continue;
                    }
                    const size_t so = ((size_t)spg * A11S_PAGE_TOKENS + sp % A11S_PAGE_TOKENS) * a.row_bytes + (size_t)c * 16;
                    reg[r] = *reinterpret_cast<const uint4 *>(base + so);
                    dst_off[r] = (long long)(((size_t)dpg * A11S_PAGE_TOKENS + dp % A11S_PAGE_TOKENS) * a.row_bytes + (size_t)c * 16);
                }
            }
            __syncthreads();  // every source of this slab is read before any write
#pragma unroll
            for (int r = 0; r < kCompactRegs; ++r)
                if (dst_off[r] >= 0) *reinterpret_cast<uint4 *>(base + dst_off[r]) = reg[r];
            __syncthreads();
        }
    }
}

__global__ void kv_compact_tables(const CompactArgs a) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= a.B) return;
    const int n = a.n_nodes ? a.n_nodes[b] : a.N;
    const int alen = a.accept_len[b];
    if (n < 1 || n > a.N || alen < 0 || alen >= n) {
        if (a.n_freed) a.n_freed[b] = 0;
        return;
    }
    const int L = a.seq_lens[b];
    const int new_len = L + 1 + alen;
    a.seq_lens[b] = new_len;
    int32_t *pt = a.page_table + (size_t)b * a.max_pages;
    const int first = (new_len + A11S_PAGE_TOKENS - 1) / A11S_PAGE_TOKENS;
    const int end = min((L + n + A11S_PAGE_TOKENS - 1) / A11S_PAGE_TOKENS, a.max_pages);
    int nf = 0;
    for (int p = first; p < end; ++p) {
        const int id = pt[p];
        if (id < 0) continue;
        if (a.freed_pages) a.freed_pages[(size_t)b * a.max_pages + nf] = id;
        ++nf;
        pt[p] = -1;
    }
    if (a.n_freed) a.n_freed[b] = nf;
}

cudaError_t launch_kv_compact(const CompactArgs &a, cudaStream_t s) {
    kv_compact_copy<<<dim3(a.B, a.num_layers), kCompactThreads, 0, s>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    kv_compact_tables<<<(a.B + 127) / 128, 128, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace a11s
