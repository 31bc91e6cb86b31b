// kvpages.cu - K5: the paged-KV page allocator on the device.
//
// Semantics of the reference's PagedKVCacheManager (src/cuda/paged_kv_cache.cu:
// init_pool 61-81, alloc_block 85-93, dealloc_block 95-101, allocate_sequence
// 103-117, append_token 119-135, free_sequence 137-149): 16-token blocks, one
// LIFO free stack of physical page ids (initially 0..num_pages-1, so the
// highest id is taken first), a new block when a sequence's token count
// exceeds blocks * 16, blocks pushed back in block-table order when freed.
// Here the stack, the page tables and the lengths live in HBM, so a decode
// step needs no host round trip to grow its tree slots or return pages.
//
// A whole batch is served by one launch of one 1024-thread block. Pages are
// popped (pushed) in batch order and, within a sequence, in logical page
// order: exactly what a loop of append_token / dealloc_block calls over the
// batch would do, found with a block-wide exclusive scan of the per-sequence
// counts. Every entry point validates first and changes nothing when it
// reports an error (the reference throws part way instead).
//
// Invariant kept by these entry points and a11s_kv_compact: an active
// sequence of length len holds pages 0 .. max(1, ceil(len/16)) - 1 of its
// table row and -1 after them; an inactive one holds -1 everywhere.
#include "common.cuh"
#include "kernels.h"

namespace a11s {

namespace {
constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ int blocks_for(int len) { return max(1, (len + A11S_PAGE_TOKENS - 1) / A11S_PAGE_TOKENS); }

// Exclusive scan of one int per thread over the block; returns the prefix and
// sets `total` (every thread) to the block's sum. Uses `ws` (kWarps + 1 ints).
__device__ int block_exclusive_scan(int v, int &total, int *ws) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    __syncthreads();  // ws may still be read by the previous call
    if (lane == 31) ws[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const int w = lane < kWarps ? ws[lane] : 0;
        int wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += y;
        }
        if (lane < kWarps) ws[lane] = wi - w;  // exclusive warp offsets
        if (lane == kWarps - 1) ws[kWarps] = wi;
    }
    __syncthreads();
    total = ws[kWarps];
    return ws[warp] + incl - v;
}

__device__ void set_status(int32_t *status, int32_t code, int32_t detail) {
    if (threadIdx.x == 0 && status) {
        status[0] = code;
        status[1] = detail;
    }
}
}  // namespace

// Pages a sequence gains and its new length; -1 = bad arguments for this row.
__device__ __forceinline__ int reserve_need(const KvPagesArgs &a, int b, int &cur, int &new_len) {
    const int len = a.seq_lens[b], add = a.counts[b];
    if (len < 0 || add < 0 || len > INT32_MAX - add) return -1;
    const bool active = a.page_table[(size_t)b * a.max_pages] >= 0;
    if (!active && len != 0) return -1;  // an inactive sequence has length 0
    cur = active ? blocks_for(len) : 0;
    new_len = len + add;
    const int want = blocks_for(new_len);
    if (want > a.max_pages) return -1;
    return want - cur;
}

__global__ void __launch_bounds__(kThreads, 1) kv_reserve_kernel(const KvPagesArgs a) {
    __shared__ int ws[kWarps + 1];
    __shared__ int s_bad;
    if (threadIdx.x == 0) s_bad = INT32_MAX;  // lowest offending sequence
    const int top = *a.free_top;
    // pass 1: validate and count
    long long total = 0;
    for (int b0 = 0; b0 < a.B; b0 += kThreads) {
        const int b = b0 + threadIdx.x;
        int cur = 0, nl = 0, need = 0;
        if (b < a.B) {
            need = reserve_need(a, b, cur, nl);
            if (need < 0) { atomicMin(&s_bad, b); need = 0; }
        }
        int t;
        block_exclusive_scan(need, t, ws);
        total += t;
    }
    __syncthreads();
    if (s_bad != INT32_MAX) { set_status(a.status, A11S_EBOUNDS, s_bad); return; }
    if (top < 0 || top > a.num_pages) { set_status(a.status, A11S_EBOUNDS, -1); return; }
    if (total > top) { set_status(a.status, A11S_ENOSPACE, (int32_t)min(total, (long long)INT32_MAX)); return; }
    // pass 2: pop in batch order, logical order within a sequence
    int base = 0;
    for (int b0 = 0; b0 < a.B; b0 += kThreads) {
        const int b = b0 + threadIdx.x;
        int cur = 0, nl = 0, need = 0;
        if (b < a.B) need = reserve_need(a, b, cur, nl);
        int t;
        const int off = base + block_exclusive_scan(need, t, ws);
        if (b < a.B) {
            int32_t *row = a.page_table + (size_t)b * a.max_pages;
            for (int j = 0; j < need; ++j) row[cur + j] = a.free_stack[top - 1 - (off + j)];
            a.seq_lens[b] = nl;
        }
        base += t;
    }
    if (threadIdx.x == 0) *a.free_top = top - base;
    set_status(a.status, A11S_OK, 0);
}

// Pages a sequence returns: its freed list (release) or its whole table (free).
__device__ __forceinline__ int give_count(const KvPagesArgs &a, int b, bool whole) {
    if (whole) {
        if (!a.counts[b]) return 0;
        const int32_t *row = a.page_table + (size_t)b * a.max_pages;
        if (row[0] < 0) return 0;  // not active: nothing to free (the reference returns too)
        const int len = a.seq_lens[b];
        return len < 0 ? -1 : min(blocks_for(len), a.max_pages);
    }
    const int n = a.counts[b];
    return n < 0 || n > a.list_stride ? -1 : n;
}

__global__ void __launch_bounds__(kThreads, 1) kv_push_kernel(const KvPagesArgs a, bool whole) {
    __shared__ int ws[kWarps + 1];
    __shared__ int s_bad;
    if (threadIdx.x == 0) s_bad = INT32_MAX;  // lowest offending sequence
    const int top = *a.free_top;
    long long total = 0;
    for (int b0 = 0; b0 < a.B; b0 += kThreads) {
        const int b = b0 + threadIdx.x;
        int n = 0;
        if (b < a.B) {
            n = give_count(a, b, whole);
            const int32_t *src = whole ? a.page_table + (size_t)b * a.max_pages : a.list + (size_t)b * a.list_stride;
            for (int j = 0; j < n && n > 0; ++j)
                if (src[j] < 0 || src[j] >= a.num_pages) n = -1;
            if (n < 0) { atomicMin(&s_bad, b); n = 0; }
        }
        int t;
        block_exclusive_scan(n, t, ws);
        total += t;
    }
    __syncthreads();
    if (s_bad != INT32_MAX) { set_status(a.status, A11S_EBOUNDS, s_bad); return; }
    if (top < 0 || top + total > a.num_pages) { set_status(a.status, A11S_EBOUNDS, -1); return; }
    int base = 0;
    for (int b0 = 0; b0 < a.B; b0 += kThreads) {
        const int b = b0 + threadIdx.x;
        const int n = b < a.B ? give_count(a, b, whole) : 0;
        int t;
        const int off = base + block_exclusive_scan(n, t, ws);
        if (b < a.B && n > 0) {
            if (whole) {
                int32_t *row = a.page_table + (size_t)b * a.max_pages;
                for (int j = 0; j < n; ++j) {
                    a.free_stack[top + off + j] = row[j];
                    row[j] = -1;
                }
                a.seq_lens[b] = 0;
            } else {
                const int32_t *src = a.list + (size_t)b * a.list_stride;
                for (int j = 0; j < n; ++j) a.free_stack[top + off + j] = src[j];
            }
        }
        base += t;
    }
    if (threadIdx.x == 0) *a.free_top = top + base;
    set_status(a.status, A11S_OK, 0);
}

__global__ void kv_pool_init_kernel(int32_t *stack, int32_t *top, int32_t n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) stack[i] = i;
    if (blockIdx.x == 0 && threadIdx.x == 0) *top = n;
}

cudaError_t launch_kv_pool_init(int32_t *stack, int32_t *top, int32_t n, cudaStream_t s) {
    const int blocks = max(1, min(1024, (n + 255) / 256));
    kv_pool_init_kernel<<<blocks, 256, 0, s>>>(stack, top, n);
    return cudaGetLastError();
}

cudaError_t launch_kv_reserve(const KvPagesArgs &a, cudaStream_t s) {
    kv_reserve_kernel<<<1, kThreads, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_kv_push(const KvPagesArgs &a, bool whole, cudaStream_t s) {
    kv_push_kernel<<<1, kThreads, 0, s>>>(a, whole);
    return cudaGetLastError();
}

}  // namespace a11s
