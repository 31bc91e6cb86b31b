// ref_kv_harness.cpp - test infrastructure only: a C shim over the reference's
// PagedKVCacheManager (include/cuda/paged_kv_cache.hpp, src/cuda/paged_kv_cache.cu),
// compiled from the reference tree into _ref/libref_kv.so by `make ref`. The
// GPU tests drive it and the device page allocator with the same operations
// and compare the block tables. The manager cudaMallocs its blocks, so it
// needs a CUDA device. Exceptions become a nonzero return.
#include <cstdint>
#include <vector>

#include "cuda/paged_kv_cache.hpp"

extern "C" {

// One layer, head_dim 32768, a 1 GB cap: 2 MB K + 2 MB V per block, 256 blocks.
void *ref_kv_create(uint32_t max_sequences) {
    try {
        PagedKVCacheManager::Config c;
        c.num_layers = 1;
        c.head_dim = 32768;
        c.max_sequences = max_sequences;
        c.vram_cap_gb = 1;
        return new PagedKVCacheManager(c);
    } catch (...) {
        return nullptr;
    }
}

void ref_kv_destroy(void *m) { delete static_cast<PagedKVCacheManager *>(m); }

int ref_kv_allocate(void *m, uint32_t seq) {
    try {
        static_cast<PagedKVCacheManager *>(m)->allocate_sequence(seq);
        return 0;
    } catch (...) {
        return 1;
    }
}

int ref_kv_append(void *m, uint32_t seq, uint32_t count) {
    try {
        for (uint32_t i = 0; i < count; ++i) static_cast<PagedKVCacheManager *>(m)->append_token(seq);
        return 0;
    } catch (...) {
        return 1;
    }
}

int ref_kv_free(void *m, uint32_t seq) {
    try {
        static_cast<PagedKVCacheManager *>(m)->free_sequence(seq);
        return 0;
    } catch (...) {
        return 1;
    }
}

// Block table of `seq` into out[0..cap): its length, or -1 if not active.
int ref_kv_table(void *m, uint32_t seq, int32_t *out, int cap) {
    try {
        const std::vector<uint32_t> &t = static_cast<PagedKVCacheManager *>(m)->get_block_table(seq);
        for (size_t i = 0; i < t.size() && (int)i < cap; ++i) out[i] = (int32_t)t[i];
        return (int)t.size();
    } catch (...) {
        return -1;
    }
}

size_t ref_kv_used_blocks(void *m) { return static_cast<PagedKVCacheManager *>(m)->used_blocks(); }
}
