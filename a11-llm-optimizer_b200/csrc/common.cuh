// common.cuh - shared device helpers of liba11spec (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/a11spec.h"

#define A11S_CHUNK 2048           // tokens per softmax chunk (fixed by the numeric contract)
#define A11S_FRAME_NONE INT32_MIN // chunk whose logits are all -inf
#define A11S_MAX_WALK_LEVELS 64   // residual levels kept per node (STOCH_DRAFT)
#define A11S_MAX_VOCAB (1 << 18)  // 262144 tokens: 128 chunks; weight sums stay far below 2^63
#define A11S_MAX_NODES 1024        // tree size limit of the n-gram expansion
#define A11S_MAX_ACCEPT_NODES 256  // tree size limit of the acceptance kernel (staged in shared memory)

namespace a11s {

// Status word: the first error wins; detail records where it happened.
struct StatusWord {
    int32_t code;
    int32_t detail;
};

__device__ __forceinline__ void report(StatusWord *st, int32_t code, int32_t detail) {
    if (st && atomicCAS(&st->code, 0, code) == 0) st->detail = detail;
}

// ---------------------------------------------------------------------------
// Deterministic fixed-point exp2 weight, bit-identical to the oracle's
// or_weight(): W = floor(2^(l*k - c) * 2^40). Every operation is an explicit
// round-to-nearest intrinsic so nvcc cannot contract or reorder it.
// 2^f on [-0.5, 0.5]: degree-5 polynomial fitted for this project (iteratively
// reweighted least squares towards minimax relative error, 2.2e-7).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float exp2_poly(float f) {
    float p = 0x1.5c0c48p-10f;
    p = __fmaf_rn(p, f, 0x1.3d0c5cp-7f);
    p = __fmaf_rn(p, f, 0x1.c6b6dcp-5f);
    p = __fmaf_rn(p, f, 0x1.ebf918p-3f);
    p = __fmaf_rn(p, f, 0x1.62e428p-1f);
    p = __fmaf_rn(p, f, 0x1.000002p+0f);
    return p;
}

__device__ __forceinline__ uint64_t det_weight(float l, float k, float cf) {
    // l = -inf gives t = -160 below and a shift > 63, i.e. weight 0.
    float t = __fmaf_rn(l, k, -cf);
    t = fmaxf(t, -160.0f);
    const float r = __fadd_rn(t, 12582912.0f);   // 1.5 * 2^23: round to nearest integer
    const float nf = __fadd_rn(r, -12582912.0f);
    const float f = __fadd_rn(t, -nf);           // exact, |f| <= 0.5
    const int32_t n = __float_as_int(r) - 0x4B400000;
    const float p = exp2_poly(f);
    const uint32_t bits = __float_as_uint(p);
    const int32_t e = (int32_t)(bits >> 23) - 127;
    const uint64_t m = (uint64_t)((bits & 0x7FFFFFu) | 0x800000u);
    int32_t sh = 7 - e - n;
    sh = sh < 0 ? 0 : sh;
    return sh > 63 ? 0ull : ((m << 24) >> sh);
}

__device__ __forceinline__ double pow2neg(int32_t d) {  // 2^-d, 0 <= d <= 1000
    return __longlong_as_double((long long)((uint64_t)(1023 - d) << 52));
}

// Reference linear-space acceptance (src/engine/speculative_verifier.cpp:114-124).
__device__ __forceinline__ bool accept_linear(float u, float lt, float ld) {
    ld = fmaxf(1e-10f, fminf(ld, 1.0f));
    lt = fmaxf(0.0f, fminf(lt, 1.0f + 1e-6f));
    float a = __fdiv_rn(lt, ld);
    if (a > 1.0f) a = 1.0f;
    return u < a;
}

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

template <typename T>
__device__ __forceinline__ T warp_max(T v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_fmax(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ uint64_t warp_sum_u64(uint64_t v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int warp_or(int v) { return __any_sync(0xffffffffu, v); }

}  // namespace a11s
