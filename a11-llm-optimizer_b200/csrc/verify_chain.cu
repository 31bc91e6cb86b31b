// verify_chain.cu - the reference's per-token chain acceptance on the device.
//
// One thread per chain walks its drafts in order (chains are <= a few dozen
// tokens; the vocab-wide work lives in accept.cu). Rule and error behaviour of
// src/engine/speculative_verifier.cpp:84-135; exp is this library's own
// (Cody-Waite split into 2^n * 2^f, the degree-5 polynomial of common.cuh).
#include "common.cuh"
#include "kernels.h"

namespace a11s {

// e^x for x in [-20, 0]: t = x * log2(e) rounded once, n = rint(t), f = t - n,
// 2^f by exp2_poly, 2^n folded into the exponent field.
__device__ __forceinline__ float det_exp_neg(float x) {
    const float t = __fmul_rn(x, 1.4426950408889634f);
    const float r = __fadd_rn(t, 12582912.0f);
    const float nf = __fadd_rn(r, -12582912.0f);
    const float f = __fadd_rn(t, -nf);
    const int n = __float_as_int(r) - 0x4B400000;
    const float p = exp2_poly(f);
    return __int_as_float(__float_as_int(p) + (n << 23));
}

__global__ void verify_chain_kernel(const float *draft, const float *target, const float *uni, int B, int n,
                                    int32_t *accepted_len, int32_t *last_idx, StatusWord *st) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const float *d = draft + (size_t)b * n, *t = target + (size_t)b * n, *u = uni + (size_t)b * n;
    for (int i = 0; i < n; ++i) {
        const float v = t[i];
        if (!(fabsf(v) < INFINITY)) {  // NaN or +-Inf anywhere in the target row
            report(st, A11S_ENONFINITE, b);
            accepted_len[b] = -1;
            last_idx[b] = 0;
            return;
        }
    }
    int acc = 0, last = 0;
    for (int i = 0; i < n; ++i) {
        float ld = d[i], lt = t[i], a;
        if (ld < 0.0f || lt < 0.0f) {
            const float lr = fmaxf(__fsub_rn(lt, ld), -20.0f);
            a = lr >= 0.0f ? 1.0f : det_exp_neg(lr);
        } else {
            ld = fmaxf(1e-10f, fminf(ld, 1.0f));
            lt = fmaxf(0.0f, fminf(lt, 1.0f + 1e-6f));
            a = __fdiv_rn(lt, ld);
        }
        if (a > 1.0f) a = 1.0f;
        if (u[i] < a) {
            ++acc;
            last = i;
        } else {
            break;
        }
    }
    accepted_len[b] = acc;
    last_idx[b] = last;
}

cudaError_t launch_verify_chain(const float *draft, const float *target, const float *uni, int B, int n,
                                int32_t *accepted_len, int32_t *last_idx, StatusWord *st, cudaStream_t s) {
    verify_chain_kernel<<<(B + 127) / 128, 128, 0, s>>>(draft, target, uni, B, n, accepted_len, last_idx, st);
    return cudaGetLastError();
}

}  // namespace a11s
