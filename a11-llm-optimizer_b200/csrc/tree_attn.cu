// tree_attn.cu - K2: tree-masked verification attention over 16-token KV pages.
//
// Math follows engine/pipeline.py:386-402 of the reference (GQA head h reads KV
// head h / (Hq/Hkv); scores q.k * scale in fp32; softmax; probabilities in
// bf16 for the PV product), extended to a token tree: node i sees every
// context position and the tree positions of its ancestors and itself.
// Semantics: include/a11spec.h (a11s_tree_attention).
#include "common.cuh"
#include "kernels.h"

namespace a11s {

constexpr int kAttnSimtWarps = 8;  // one warp per query head of a GQA group
constexpr int kTile = 32;          // keys per tile
constexpr int kKStride = 65;       // 32-bit words per K row in smem (64 + 1 pad)

int tree_attention_splits(int32_t, int32_t, int32_t, int32_t, int32_t) { return 1; }

size_t tree_attention_partials_bytes(int32_t B, int32_t N, int32_t Hq, int32_t D, int32_t splits) {
    return splits > 1 ? (size_t)splits * B * N * Hq * (D + 2) * sizeof(float) : 0;
}

// Ancestor-or-self bitmask of node i (bit j set iff j is i or an ancestor of i).
__device__ __forceinline__ bool ancestors(const int32_t *par, int i, uint64_t &anc) {
    anc = 0;
    int a = i;
    for (int steps = 0; steps <= 64; ++steps) {
        anc |= 1ull << a;
        if (a == 0) return true;
        const int p = par[a];
        if (p < 0 || p >= a) return false;
        a = p;
    }
    return false;
}

__global__ void __launch_bounds__(kAttnSimtWarps * 32) tree_attn_simt(const AttnArgs a) {
    const int i = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = g * kAttnSimtWarps + warp;
    const int n = a.n_nodes ? a.n_nodes[b] : a.N;
    __nv_bfloat16 *out = reinterpret_cast<__nv_bfloat16 *>(a.out) + (((size_t)b * a.N + i) * a.Hq + h) * 128;
    if (n < 1 || n > a.N || i >= n) {
        if (n < 1 || n > a.N) report(a.status, A11S_EBOUNDS, b);
        reinterpret_cast<uint2 *>(out)[lane] = make_uint2(0, 0);
        if (a.lse && lane == 0) a.lse[((size_t)b * a.N + i) * a.Hq + h] = 0.0f;
        return;
    }
    __shared__ uint64_t s_anc;
    __shared__ int s_ok;
    __shared__ uint32_t s_k[kTile * kKStride];
    __shared__ uint2 s_v[kTile * 32];
    __shared__ float s_q[kAttnSimtWarps][128];
    __shared__ int s_valid[kTile];
    if (threadIdx.x == 0) {
        uint64_t anc;
        s_ok = ancestors(a.parents + (size_t)b * a.N, i, anc);
        s_anc = anc;
        if (!s_ok) report(a.status, A11S_EBOUNDS, b);
    }
    const float qscale = a.scale * 1.4426950408889634f;  // scores in log2 units
    {
        const __nv_bfloat16 *qp = reinterpret_cast<const __nv_bfloat16 *>(a.q) + (((size_t)b * a.N + i) * a.Hq + h) * 128;
        for (int d = lane; d < 128; d += 32) s_q[warp][d] = __bfloat162float(qp[d]) * qscale;
    }
    __syncthreads();
    if (!s_ok) {
        reinterpret_cast<uint2 *>(out)[lane] = make_uint2(0, 0);
        return;
    }
    const int L = a.ctx_lens[b];
    const int total = L + i + 1;
    const uint64_t anc = s_anc;
    const int32_t *pt = a.page_table + (size_t)b * a.max_pages;
    const __nv_bfloat16 *kp = reinterpret_cast<const __nv_bfloat16 *>(a.k_pool);
    const __nv_bfloat16 *vp = reinterpret_cast<const __nv_bfloat16 *>(a.v_pool);

    float m = -INFINITY, l = 0.0f;
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    for (int t0 = 0; t0 < total; t0 += kTile) {
        // cooperative load of 32 K and V rows (256 B each) of KV head g
        for (int it = threadIdx.x; it < kTile * 16; it += blockDim.x) {
            const int t = it >> 4, c = it & 15;  // row, 16-byte column
            const int p = t0 + t;
            bool valid = p < total && (p < L || ((anc >> (p - L)) & 1ull));
            int page = -1;
            if (valid) {
                const int lp = p / A11S_PAGE_TOKENS;
                page = lp < a.max_pages ? pt[lp] : -1;
                if (page < 0 || page >= a.num_pages) {
                    report(a.status, A11S_EBOUNDS, b);
                    valid = false;
                }
            }
            uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
            if (valid) {
                const size_t row = ((size_t)page * A11S_PAGE_TOKENS + p % A11S_PAGE_TOKENS) * a.Hkv + g;
                kv = reinterpret_cast<const uint4 *>(kp + row * 128)[c];
                vv = reinterpret_cast<const uint4 *>(vp + row * 128)[c];
            }
            uint32_t *kr = s_k + t * kKStride + c * 4;
            kr[0] = kv.x; kr[1] = kv.y; kr[2] = kv.z; kr[3] = kv.w;
            s_v[t * 32 + c * 2] = make_uint2(vv.x, vv.y);
            s_v[t * 32 + c * 2 + 1] = make_uint2(vv.z, vv.w);
            if (c == 0) s_valid[t] = valid;
        }
        __syncthreads();
        // score of key (t0 + lane) for this warp's head
        float s = -INFINITY;
        if (s_valid[lane]) {
            const uint32_t *kr = s_k + lane * kKStride;
            float acc = 0.f;
#pragma unroll 8
            for (int w = 0; w < 64; ++w) {
                const uint32_t kw = kr[w];
                acc = fmaf(s_q[warp][2 * w], bf16lo(kw), acc);
                acc = fmaf(s_q[warp][2 * w + 1], bf16hi(kw), acc);
            }
            s = acc;
        }
        const float mt = warp_fmax(s);
        const float m_new = fmaxf(m, mt);
        const float alpha = m == -INFINITY ? 0.f : exp2f(m - m_new);
        const float p = s == -INFINITY ? 0.f : exp2f(s - m_new);
        float ps = p;
#pragma unroll
        for (int off = 16; off; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
        l = l * alpha + ps;
        const float pb = __bfloat162float(__float2bfloat16_rn(p));  // probabilities in bf16
#pragma unroll
        for (int e = 0; e < 4; ++e) o[e] *= alpha;
        for (int t = 0; t < kTile; ++t) {
            const float pt_ = __shfl_sync(0xffffffffu, pb, t);
            const uint2 vw = s_v[t * 32 + lane];
            o[0] = fmaf(pt_, bf16lo(vw.x), o[0]);
            o[1] = fmaf(pt_, bf16hi(vw.x), o[1]);
            o[2] = fmaf(pt_, bf16lo(vw.y), o[2]);
            o[3] = fmaf(pt_, bf16hi(vw.y), o[3]);
        }
        m = m_new;
        __syncthreads();
    }
    const float inv = 1.0f / l;
    __nv_bfloat162 r0 = __floats2bfloat162_rn(o[0] * inv, o[1] * inv);
    __nv_bfloat162 r1 = __floats2bfloat162_rn(o[2] * inv, o[3] * inv);
    uint2 packed;
    packed.x = *reinterpret_cast<uint32_t *>(&r0);
    packed.y = *reinterpret_cast<uint32_t *>(&r1);
    reinterpret_cast<uint2 *>(out)[lane] = packed;
    if (a.lse && lane == 0)
        a.lse[((size_t)b * a.N + i) * a.Hq + h] = (m + log2f(l)) * 0.6931471805599453f;
}

cudaError_t launch_tree_attention(const AttnArgs &a, cudaStream_t s) {
    tree_attn_simt<<<dim3(a.N, a.Hkv, a.B), kAttnSimtWarps * 32, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace a11s
