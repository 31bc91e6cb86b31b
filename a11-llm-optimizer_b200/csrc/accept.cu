// accept.cu - K3: vocab-wide softmax/argmax + acceptance + path select + bonus draw.
//
// One kernel per call; block (x, y) = (sequence, slice of its units), so the
// first wave holds every sequence's first slice.
// Phase 1 (every block, HBM-bound): warps stream 2048-token chunks of every
//   live logits row with 16-byte non-allocating loads and record the chunk
//   maximum (NaN-propagating, so a NaN or +Inf is caught here; GREEDY also
//   records the first position of the maximum in the chunk), the single read
//   of the vocab. A sequence's units start with its root rows (whose
//   fixed-point weight sums are also taken, in the sampling modes), then the
//   other rows in index order, a row's chunks consecutive. Records start as a
//   sentinel (the launch's memset) that no record value equals.
// Phase 2 (the block of slice 0, which holds exactly the sequence's root-row
//   units; nothing waits): walk the tree from the root while the bulk pass
//   goes on in other blocks.
//   GREEDY  row argmax = first chunk holding the row max, then the first token
//           equal to it inside that chunk.
//   STOCH_* the fixed-point softmax statistics (frame c_j = ceil(cmax_j * k),
//           S_j = sum of weights); then acceptance, residuals and the bonus draw.
//   A visited row other than the root needs its records: the walking block
//   waits (bounded) until they are written, then GREEDY reads no logits at all
//   and the sampling modes read the row once more for its weights. Should the
//   wait run out (or when waiting is not allowed: more sequences than SMs),
//   the block takes the chunk maxima itself from the row; the results are the
//   same either way.
// The numbers are exactly those of the oracle (order-independent integer
// sums), so decisions are bit-exact.
//
// Semantics: include/a11spec.h (a11s_accept). Reference behaviour followed:
// src/engine/speculative_verifier.cpp:84-135 (acceptance rule, first rejection
// stops the chain), engine/sampler.py:16 (logits / T).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace a11s {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxNch = A11S_MAX_VOCAB / A11S_CHUNK;  // 128

__device__ __forceinline__ float max_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

__device__ __forceinline__ float warp_max_nan(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = max_nan(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

template <bool BF16>
struct Vec {
    static constexpr int EPV = BF16 ? 8 : 4;  // logits per 16-byte vector
    static constexpr int NV = 64 / EPV;       // vectors per lane per chunk
    static constexpr int ESZ = BF16 ? 2 : 4;
    __device__ static __forceinline__ float at(const uint4 &d, int e) {
        const uint32_t w = (&d.x)[BF16 ? (e >> 1) : e];
        if (BF16) return (e & 1) ? bf16hi(w) : bf16lo(w);
        return __uint_as_float(w);
    }
};

// bf16 rows: the whole chunk sits in a lane's registers, 8 vectors of 8
// logits (vector g of lane = logits [(g*32 + lane) * 8, +8)); positions past
// the row read as -inf. The vocab is a multiple of 8, so a vector is either
// wholly inside the row or wholly past it.
__device__ __forceinline__ void load_chunk_bf16(const char *row, int c0, int clen, int lane, uint4 (&d)[8]) {
#pragma unroll
    for (int g = 0; g < 8; ++g) {
        const int e0 = (g * 32 + lane) * 8;
        d[g] = e0 < clen ? ldg_stream(row + (size_t)(c0 + e0) * 2) : make_uint4(0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u);
    }
}

// NaN-propagating maximum of two packed bf16 pairs. The maximum of bf16
// values is one of them, so taking it on the packed halves and widening once
// gives exactly the maximum of the widened values (a NaN stays a NaN).
__device__ __forceinline__ uint32_t max_nan_bf16x2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ uint32_t vec_max_bf16x2(const uint4 &d) {
    return max_nan_bf16x2(max_nan_bf16x2(d.x, d.y), max_nan_bf16x2(d.z, d.w));
}

// Chunk max of one row chunk, lane layout: vector i of lane = logits
// [(i*32 + lane) * EPV, +EPV). Positions past the row are -inf. bf16 rows take
// the maximum on packed pairs (four instructions per 16-byte vector).
template <bool BF16>
__device__ __forceinline__ float chunk_max(const char *row, int c0, int clen, int lane) {
    if constexpr (BF16) {
        uint4 d[8];
        load_chunk_bf16(row, c0, clen, lane, d);
        uint32_t m2 = vec_max_bf16x2(d[0]);
#pragma unroll
        for (int g = 1; g < 8; ++g) m2 = max_nan_bf16x2(m2, vec_max_bf16x2(d[g]));
        return warp_max_nan(max_nan(bf16lo(m2), bf16hi(m2)));
    } else {
        using VT = Vec<BF16>;
        constexpr int G = 8;  // vectors in flight per lane
        float m = -INFINITY;
#pragma unroll
        for (int i0 = 0; i0 < VT::NV; i0 += G) {
            uint4 d[G];
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const int e0 = ((i0 + g) * 32 + lane) * VT::EPV;
                d[g] = e0 < clen ? ldg_stream(row + (size_t)(c0 + e0) * VT::ESZ)
                                 : make_uint4(0xFF800000u, 0xFF800000u, 0xFF800000u, 0xFF800000u);
            }
#pragma unroll
            for (int g = 0; g < G; ++g)
#pragma unroll
                for (int e = 0; e < VT::EPV; ++e) m = max_nan(m, VT::at(d[g], e));
        }
        return warp_max_nan(m);
    }
}

// Chunk max (as chunk_max) and the first position in the chunk holding it
// (float equality, so -0 and +0 are the same value, as argmax sees them; a
// chunk holding a NaN has a NaN maximum whose position is never asked for).
// bf16: every lane takes its packed maximum; only the lanes whose maximum is
// the chunk's search their registers, vector by vector, for its first
// position, and the warp takes the smallest. fp32: each lane keeps its first
// strictly greater value along its reads, then the warp takes the smallest
// position among the lanes whose maximum equals the chunk's.
template <bool BF16>
__device__ __forceinline__ float chunk_max_first(const char *row, int c0, int clen, int lane, int &first) {
    if constexpr (BF16) {
        uint4 d[8];
        load_chunk_bf16(row, c0, clen, lane, d);
        uint32_t vm[8];
#pragma unroll
        for (int g = 0; g < 8; ++g) vm[g] = vec_max_bf16x2(d[g]);
        const uint32_t m2 = max_nan_bf16x2(max_nan_bf16x2(max_nan_bf16x2(vm[0], vm[1]), max_nan_bf16x2(vm[2], vm[3])),
                                           max_nan_bf16x2(max_nan_bf16x2(vm[4], vm[5]), max_nan_bf16x2(vm[6], vm[7])));
        const float ml = max_nan(bf16lo(m2), bf16hi(m2));
        const float M = warp_max_nan(ml);
        int f = INT_MAX;
        if (ml == M) {  // this lane holds the chunk maximum (never when it is NaN)
#pragma unroll
            for (int g = 0; g < 8; ++g) {
                if (f == INT_MAX && max_nan(bf16lo(vm[g]), bf16hi(vm[g])) == M) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const int pos = (g * 32 + lane) * 8 + e;
                        if (f == INT_MAX && pos < clen && Vec<true>::at(d[g], e) == M) f = pos;
                    }
                }
            }
        }
        first = -warp_max(-f);  // warp min
        return M;
    } else {
        using VT = Vec<BF16>;
        constexpr int G = 8;
        float m = -INFINITY, bv = -INFINITY;
        int bi = INT_MAX;
#pragma unroll
        for (int i0 = 0; i0 < VT::NV; i0 += G) {
            uint4 d[G];
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const int e0 = ((i0 + g) * 32 + lane) * VT::EPV;
                d[g] = e0 < clen ? ldg_stream(row + (size_t)(c0 + e0) * VT::ESZ)
                                 : make_uint4(0xFF800000u, 0xFF800000u, 0xFF800000u, 0xFF800000u);
            }
#pragma unroll
            for (int g = 0; g < G; ++g)
#pragma unroll
                for (int e = 0; e < VT::EPV; ++e) {
                    const float v = VT::at(d[g], e);
                    const int pos = ((i0 + g) * 32 + lane) * VT::EPV + e;
                    m = max_nan(m, v);
                    if (pos < clen && (bi == INT_MAX || v > bv)) { bv = v; bi = pos; }
                }
        }
        m = warp_max_nan(m);
        int f = (bi != INT_MAX && bv == m) ? bi : INT_MAX;
        first = -warp_max(-f);  // warp min
        return m;
    }
}

// Sum of fixed-point weights of one chunk in frame cf (no max needed: the
// frame comes from the phase-1 chunk max).
template <bool BF16>
__device__ __forceinline__ uint64_t chunk_wsum(const char *row, int c0, int clen, float k, float cf, int lane) {
    using VT = Vec<BF16>;
    constexpr int G = 4;
    uint64_t s = 0;
    for (int i0 = 0; i0 < VT::NV; i0 += G) {
        uint4 d[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const int e0 = ((i0 + g) * 32 + lane) * VT::EPV;
            const uint32_t ninf = BF16 ? 0xFF80FF80u : 0xFF800000u;
            d[g] = e0 < clen ? ldg_stream(row + (size_t)(c0 + e0) * VT::ESZ) : make_uint4(ninf, ninf, ninf, ninf);
        }
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int e = 0; e < VT::EPV; ++e) s += det_weight(VT::at(d[g], e), k, cf);
    }
    return warp_sum_u64(s);
}

__device__ __forceinline__ float load_logit(const char *row, int v, bool bf16) {
    if (bf16) {
        const uint16_t h = __ldg(reinterpret_cast<const unsigned short *>(row) + v);
        return __uint_as_float((uint32_t)h << 16);
    }
    return __ldg(reinterpret_cast<const float *>(row) + v);
}

__device__ __forceinline__ int32_t frame_of(float cmax, float k) {
    return cmax == -INFINITY ? A11S_FRAME_NONE : (int32_t)ceilf(__fmul_rn(cmax, k));
}

// ---------------------------------------------------------------------------
// Phase 2 state (shared memory of the walking block).
// ---------------------------------------------------------------------------
struct RowStat {  // combined statistics of one row in the fixed-point softmax
    int32_t C;
    uint64_t S;
    double invS;
};

struct WalkSmem {
    int32_t fr[kMaxNch];    // p frames of the current row
    uint64_t sum[kMaxNch];  // p chunk sums of the current row
    uint64_t sub[kMaxNch];  // p chunk sums with rejected tokens removed (ONEHOT)
    int32_t qfr[kMaxNch];   // q frames (DRAFT)
    uint64_t qsum[kMaxNch];
    uint64_t lvl[kMaxNch];  // chunk totals of the newest residual level (DRAFT)
    uint64_t tmp[kMaxNch];
    uint64_t T[A11S_MAX_WALK_LEVELS + 1];
    double invT[A11S_MAX_WALK_LEVELS + 1];
    int32_t excl[A11S_MAX_ACCEPT_NODES];
    int32_t tok[A11S_MAX_ACCEPT_NODES];   // the sequence's tree and uniforms, staged once
    int32_t par[A11S_MAX_ACCEPT_NODES];
    float uni[A11S_MAX_ACCEPT_NODES];
    int32_t kids[A11S_MAX_ACCEPT_NODES];  // children of the current node, index order
    float kl[A11S_MAX_ACCEPT_NODES];      // their target logits
    float kq[A11S_MAX_ACCEPT_NODES];      // and draft logits (DRAFT)
    float cmx[kMaxNch];     // chunk maxima of the row being visited (GREEDY argmax)
    int32_t carg[kMaxNch];  // and the first position of each maximum in its chunk
    float cp[A11S_CHUNK];   // one staged chunk of the p row (widened to fp32)
    float cq[A11S_CHUNK];   // and of the q row (DRAFT)
    uint64_t wtot[kWarps];  // per-warp weight totals of the bonus scan
    RowStat ps, qs;
    uint64_t S_eff, bt2;
    int32_t nexcl, L, node, alen, ck, nk, action, child, ok, bj, res[2];
    uint32_t gen;         // generation of this walk's latest residual pass (DRAFT)
    int32_t no_helpers;   // set when a pass's wait ran out: later passes stay in this block
};

// Inverse CDF inside one chunk, every thread of the block: thread t owns the
// chunk positions [4 t, 4 t + 4) and wfn(pos, w) fills their four weights.
// Returns (to every thread) the first position whose running weight exceeds
// t2; if t2 is beyond the chunk total (inconsistent totals), the last
// positive-weight position; -1 if there is none.
template <typename WF>
__device__ int block_scan_chunk(int clen, uint64_t t2, WF wfn, WalkSmem &sm) {
    static_assert(A11S_CHUNK == 4 * kThreads, "four chunk positions per thread");
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, p0 = 4 * threadIdx.x;
    uint64_t w[4] = {0ull, 0ull, 0ull, 0ull};
    if (p0 < clen) wfn(p0, w);
    const uint64_t mine = w[0] + w[1] + w[2] + w[3];
    uint64_t incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint64_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) sm.wtot[warp] = incl;
    if (threadIdx.x == 0) {
        sm.res[0] = INT_MAX;
        sm.res[1] = -1;
    }
    __syncthreads();
    uint64_t acc = incl - mine;
    for (int i = 0; i < warp; ++i) acc += sm.wtot[i];
    if (acc <= t2 && t2 - acc < mine) {  // at most one thread
        for (int e = 0; e < 4; ++e) {
            acc += w[e];
            if (acc > t2) { sm.res[0] = p0 + e; break; }
        }
    }
    int last = -1;
#pragma unroll
    for (int e = 0; e < 4; ++e)
        if (w[e]) last = p0 + e;
    last = warp_max(last);
    if (lane == 0 && last >= 0) atomicMax(&sm.res[1], last);
    __syncthreads();
    return sm.res[0] != INT_MAX ? sm.res[0] : sm.res[1];
}

__device__ RowStat combine_sums(const int32_t *fr, const uint64_t *sum, int nch, int lane) {
    int32_t C = A11S_FRAME_NONE;
    for (int j = lane; j < nch; j += 32)
        if (fr[j] != A11S_FRAME_NONE) C = max(C, fr[j]);
    C = warp_max(C);
    uint64_t S = 0;
    if (C != A11S_FRAME_NONE)
        for (int j = lane; j < nch; j += 32) {
            if (fr[j] == A11S_FRAME_NONE) continue;
            const int d = C - fr[j];
            S += d > 63 ? 0ull : (sum[j] >> d);
        }
    S = warp_sum_u64(S);
    RowStat rs;
    rs.C = C;
    rs.S = S;
    rs.invS = S ? __ddiv_rn(1.0, __ull2double_rn(S)) : 0.0;
    return rs;
}

// Every warp of the block: frames and weight sums of one non-root row into
// fr/sum, when the row's records are not available (see records() in the
// kernel). The row's chunk maxima are taken here, then each chunk's weights in
// its frame (a second read of the chunk, from L2). A non-finite logit or an
// out-of-range frame is reported like in the bulk pass.
template <bool BF16>
__device__ void row_sums(const char *row, int nch, int V, float k, int32_t *fr, uint64_t *sum, int warp, int lane,
                         StatusWord *st, int b) {
    int bad = 0;
    for (int j = warp; j < nch; j += kWarps) {
        const int c0 = j * A11S_CHUNK, clen = min(A11S_CHUNK, V - c0);
        const float cm = chunk_max<BF16>(row, c0, clen, lane);
        bad |= !(cm < INFINITY) || (cm > -INFINITY && !(fabsf(__fmul_rn(cm, k)) < 16777216.0f));
        const int32_t f = cm < INFINITY ? frame_of(cm, k) : A11S_FRAME_NONE;
        uint64_t s = 0;
        if (f != A11S_FRAME_NONE) s = chunk_wsum<BF16>(row, c0, clen, k, (float)f, lane);
        if (lane == 0) {
            fr[j] = f;
            sum[j] = s;
        }
    }
    if (bad && lane == 0) report(st, A11S_ENONFINITE, b);
}

// As row_sums, with the chunk maxima taken from the row's phase-1 records:
// one read of the row (its weights) instead of two.
template <bool BF16>
__device__ void row_sums_rec(const char *row, const float *rec, int nch, int V, float k, int32_t *fr,
                             uint64_t *sum, int warp, int lane, StatusWord *st, int b) {
    int bad = 0;
    for (int j = warp; j < nch; j += kWarps) {
        const int c0 = j * A11S_CHUNK, clen = min(A11S_CHUNK, V - c0);
        const float cm = __ldcg(rec + j);
        bad |= !(cm < INFINITY) || (cm > -INFINITY && !(fabsf(__fmul_rn(cm, k)) < 16777216.0f));
        const int32_t f = cm < INFINITY ? frame_of(cm, k) : A11S_FRAME_NONE;
        uint64_t s = 0;
        if (f != A11S_FRAME_NONE) s = chunk_wsum<BF16>(row, c0, clen, k, (float)f, lane);
        if (lane == 0) {
            fr[j] = f;
            sum[j] = s;
        }
    }
    if (bad && lane == 0) report(st, A11S_ENONFINITE, b);
}

// Frames and weight sums of a row: the root's come from the bulk pass (chunk
// records and weight sums); another row's from its chunk records when `rec`
// is given (the row's counter showed them complete), else the block takes
// them from the row itself.
template <bool BF16>
__device__ void row_stats_into(const char *row, const float *root_cmax, const unsigned long long *root,
                               const float *rec, int nch, int V, float k, int32_t *fr, uint64_t *sum, int warp,
                               int lane, StatusWord *st, int b) {
    if (root) {
        for (int j = threadIdx.x; j < nch; j += blockDim.x) {
            fr[j] = frame_of(__ldcg(root_cmax + j), k);
            sum[j] = __ldcg(root + j);
        }
    } else if (rec) {
        row_sums_rec<BF16>(row, rec, nch, V, k, fr, sum, warp, lane, st, b);
    } else {
        row_sums<BF16>(row, nch, V, k, fr, sum, warp, lane, st, b);
    }
}

// Records start as kUnrecorded (the launch's memset); each is written once
// with its final value, which is never that pattern (max.NaN gives the
// canonical NaN 0x7FFFFFFF; positions are >= 0). So a record that differs from
// it is final, and a row is complete when all its records are.
constexpr uint32_t kUnrecorded = 0xFFFFFFFFu;

// A chunk key of the LM head (a11s_lm_head): bits 32-47 hold the order image
// of the chunk's bf16 maximum (sign set -> 16 bits flipped, else sign bit set;
// -0 stored as +0), the low 32 bits the complement of its first position.
// A key never written (0) decodes to NaN.
__device__ __forceinline__ float key_value(unsigned long long key) {
    const uint32_t o = (uint32_t)(key >> 32) & 0xFFFFu;
    const uint32_t h = (o & 0x8000u) ? (o & 0x7FFFu) : (~o & 0xFFFFu);
    return __uint_as_float(h << 16);
}
__device__ __forceinline__ int32_t key_first(unsigned long long key) {
    return (int32_t)(0xFFFFFFFFu - (uint32_t)key);
}
constexpr long long kRecordWaitBudget = 4000000ll;  // ~2 ms of SM clock
__device__ __forceinline__ void st_relaxed(void *p, uint32_t v) {
    asm volatile("st.relaxed.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed(const void *p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// One record (and its position record, if any) written yet? When waiting is
// allowed, waits a bounded time: the bulk pass records every live row; on a
// timeout the caller takes the statistics from the row itself, with the same
// results. The values read are returned in v / pv.
__device__ __forceinline__ bool record_ready(const void *rec, const void *pos, bool may_wait, uint32_t &v,
                                             uint32_t &pv) {
    auto done = [&]() {
        v = ld_relaxed(rec);
        pv = pos ? ld_relaxed(pos) : 0u;
        return v != kUnrecorded && pv != kUnrecorded;
    };
    if (done()) return true;
    if (!may_wait) return false;
    const long long t0 = clock64();
    while (!done()) {
        if (clock64() - t0 > kRecordWaitBudget) return false;
        __nanosleep(200);
    }
    return true;
}

// Chunk maxima of a row into shared memory (every thread of the block): the
// root's are copied from the bulk pass's records, the others are computed.
template <bool BF16>
__device__ void row_cmax_into(const char *row, const float *root_cmax, int nch, int V, float *dst, int warp,
                              int lane, StatusWord *st, int b) {
    if (root_cmax) {
        for (int j = threadIdx.x; j < nch; j += blockDim.x) dst[j] = __ldcg(root_cmax + j);
    } else {
        int bad = 0;
        for (int j = warp; j < nch; j += kWarps) {
            const int c0 = j * A11S_CHUNK;
            const float cm = chunk_max<BF16>(row, c0, min(A11S_CHUNK, V - c0), lane);
            bad |= !(cm < INFINITY);
            if (lane == 0) dst[j] = cm;
        }
        if (bad && lane == 0) report(st, A11S_ENONFINITE, b);
    }
    __syncthreads();
}

__device__ __forceinline__ double chunk_scale(const RowStat &rs, int32_t frame) {
    if (frame == A11S_FRAME_NONE || rs.S == 0) return 0.0;
    const int d = rs.C - frame;
    if (d > 1000) return 0.0;
    return __dmul_rn(pow2neg(d), rs.invS);
}

// p(v) = (float)(W_v * (2^(c_j - C) / S)) with the row's frames.
__device__ __forceinline__ float prob_of(float l, float k, int32_t frame, double sc) {
    if (frame == A11S_FRAME_NONE || sc == 0.0) return 0.0f;
    const uint64_t w = det_weight(l, k, (float)frame);
    return __double2float_rn(__dmul_rn(__ull2double_rn(w), sc));
}

__device__ __forceinline__ float level_prob(float p, float q, int L, const double *invT) {
    for (int l = 1; l <= L; ++l) {
        const float r = fmaxf(__fsub_rn(p, q), 0.0f);
        const uint64_t R = __float2ull_rz(__fmul_rn(r, 0x1p40f));
        p = __double2float_rn(__dmul_rn(__ull2double_rn(R), invT[l]));
    }
    return p;
}

__device__ __forceinline__ uint64_t level_weight(float p_prev, float q) {
    const float r = fmaxf(__fsub_rn(p_prev, q), 0.0f);
    return __float2ull_rz(__fmul_rn(r, 0x1p40f));
}

// One chunk of a residual pass (STOCH_DRAFT), one warp: the sum over the chunk
// of level_weight(p_L(v), q(v)), where p_L is p after the L residual levels
// of invT (p and q in their row frames: fp/fq, scales scp/scq). Four vectors of
// p and q in flight per lane. Every lane returns the warp's sum.
template <bool BF16>
__device__ uint64_t resid_chunk_sum(const char *prow, const char *qrow, int c0, int clen, float k, int32_t fp,
                                    int32_t fq, double scp, double scq, int L, const double *invT, int lane) {
    constexpr int EPV = Vec<BF16>::EPV, NV = Vec<BF16>::NV, G = 4;
    uint64_t s = 0;
    for (int i0 = 0; i0 < NV; i0 += G) {
        uint4 vp[G], vq[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const int e0 = ((i0 + g) * 32 + lane) * EPV;
            const size_t off = (size_t)(c0 + e0) * (BF16 ? 2 : 4);
            const uint32_t ninf = BF16 ? 0xFF80FF80u : 0xFF800000u;
            vp[g] = e0 < clen ? ldg_stream(prow + off) : make_uint4(ninf, ninf, ninf, ninf);
            vq[g] = e0 < clen ? ldg_stream(qrow + off) : make_uint4(ninf, ninf, ninf, ninf);
        }
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int e = 0; e < EPV; ++e) {
                const float pv = prob_of(Vec<BF16>::at(vp[g], e), k, fp, scp);
                const float qv = prob_of(Vec<BF16>::at(vq[g], e), k, fq, scq);
                s += level_weight(level_prob(pv, qv, L, invT), qv);
            }
    }
    return warp_sum_u64(s);
}

// A pass over one visited row of a walk, shared with helper blocks (sampling
// modes), one at a time per sequence:
//   kind 0 (STOCH_DRAFT): the chunk totals of the next residual level,
//          sum over the chunk of level_weight(p_L(v), q(v)), into sums[j];
//   kind 1: the row statistics of a recorded row: each chunk's frame (from
//          its bulk-pass maximum) and weight sum, for the p row (fr, sums) and
//          in STOCH_DRAFT the q row (qfr, qsums).
// The walking block publishes the pass (kind, visited node, level L, row
// statistics, frames, invT) and opens it by writing `word` = (generation << 32)
// | 0. A warp (of the walker or a helper) takes the next chunk by adding 1 to
// `word`; the value returned names the pass and the chunk, and the warp reads
// that pass's parameters after the claim. Each warp computes its chunk,
// stores the results and counts the chunk in `done`. The walker publishes the next pass only after `done`
// reached the chunk count of the last, so no late write lands in a newer pass.
// The walker claims chunks too, so a pass finishes even when no helper runs.
struct SharedPass {
    unsigned long long word;  // generation << 32 | chunks claimed (0: no pass yet)
    int32_t done;             // chunks whose results are stored, this generation
    int32_t node, L, kind;
    RowStat ps, qs;
    double invT[A11S_MAX_WALK_LEVELS + 1];
};
constexpr size_t kJobHead = (sizeof(SharedPass) + 255) & ~size_t(255);
size_t accept_job_bytes(int nch) { return kJobHead + (size_t)nch * 2 * (sizeof(int32_t) + sizeof(uint64_t)); }
__device__ __forceinline__ SharedPass *job_of(const AcceptArgs &a, int b) {
    return reinterpret_cast<SharedPass *>(a.jobs + (size_t)b * a.job_stride);
}
__device__ __forceinline__ int32_t *job_fr(const AcceptArgs &a, int b) {
    return reinterpret_cast<int32_t *>(a.jobs + (size_t)b * a.job_stride + kJobHead);
}
__device__ __forceinline__ int32_t *job_qfr(const AcceptArgs &a, int b) { return job_fr(a, b) + a.nch; }
__device__ __forceinline__ unsigned long long *job_sums(const AcceptArgs &a, int b) {
    return reinterpret_cast<unsigned long long *>(job_fr(a, b) + 2 * a.nch);
}
__device__ __forceinline__ unsigned long long *job_qsums(const AcceptArgs &a, int b) { return job_sums(a, b) + a.nch; }
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const void *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// Claim the next chunk of whatever pass `word` holds open (one thread): one
// atomic add; returns the chunk, or -1 when every chunk of that pass is taken
// (or the slot is closed). The returned chunk belongs to the pass named by the
// word's generation at the moment of the add, which may be newer than the one
// the caller saw: the caller computes it under that pass, reading the pass's
// parameters after the claim. The walker rewrites the parameters only after
// every chunk of the previous pass is done, so they cannot change under a
// claimed chunk, and no claim is ever dropped.
__device__ __forceinline__ int claim_chunk(unsigned long long *word, int nch) {
    const unsigned long long w = atomicAdd(word, 1ull);
    return (uint32_t)w < (uint32_t)nch ? (int)(uint32_t)w : -1;
}
// A closed slot: the count sits far above any chunk count, so late adds
// neither claim anything nor carry into the generation.
constexpr unsigned long long kClosedCount = 0x80000000ull;
constexpr long long kHelperBudget = 20000000ll;   // ~10 ms of SM clock: helpers leave after it whatever happens
constexpr long long kPassWaitBudget = 4000000ll;  // ~2 ms: a walker's wait for its helpers' last chunks

// One chunk j of sequence b's open pass (one warp); stores the results and
// counts the chunk done. invT: the pass's residual levels (kind 0).
template <int MODE, bool BF16>
__device__ void pass_chunk(const AcceptArgs &a, int b, int kind, int node, int L, const RowStat &ps,
                           const RowStat &qs, const double *invT, int j, int lane) {
    const size_t row_bytes = (size_t)a.stride * (BF16 ? 2 : 4);
    const char *prow = reinterpret_cast<const char *>(a.target) + ((size_t)b * a.N + node) * row_bytes;
    const char *qrow = MODE == A11S_ACCEPT_STOCH_DRAFT
                           ? reinterpret_cast<const char *>(a.draft) + ((size_t)b * a.N + node) * row_bytes
                           : nullptr;
    const int c0 = j * A11S_CHUNK, clen = min(A11S_CHUNK, a.V - c0);
    SharedPass *job = job_of(a, b);
    if (kind == 0) {
        if constexpr (MODE == A11S_ACCEPT_STOCH_DRAFT) {
            const int32_t fp = __ldcg(job_fr(a, b) + j), fq = __ldcg(job_qfr(a, b) + j);
            const uint64_t sum = resid_chunk_sum<BF16>(prow, qrow, c0, clen, a.k, fp, fq, chunk_scale(ps, fp),
                                                       chunk_scale(qs, fq), L, invT, lane);
            if (lane == 0) __stcg(job_sums(a, b) + j, (unsigned long long)sum);
        }
    } else {
        // the row's frames from its bulk-pass maxima, then its weights
        const int nrows = MODE == A11S_ACCEPT_STOCH_DRAFT ? 2 : 1;
        int bad = 0;
        for (int q = 0; q < nrows; ++q) {
            const int r = q ? a.N + node : node;
            const float cm = __ldcg(a.recs + ((size_t)b * a.rows_per_seq + r) * a.nch + j);
            bad |= !(cm < INFINITY) || (cm > -INFINITY && !(fabsf(__fmul_rn(cm, a.k)) < 16777216.0f));
            const int32_t f = cm < INFINITY ? frame_of(cm, a.k) : A11S_FRAME_NONE;
            const uint64_t s = f == A11S_FRAME_NONE ? 0ull : chunk_wsum<BF16>(q ? qrow : prow, c0, clen, a.k, (float)f, lane);
            if (lane == 0) {
                __stcg(reinterpret_cast<int *>((q ? job_qfr(a, b) : job_fr(a, b)) + j), (int)f);
                __stcg((q ? job_qsums(a, b) : job_sums(a, b)) + j, (unsigned long long)s);
            }
        }
        if (bad && lane == 0) report(a.status, A11S_ENONFINITE, b);
    }
    if (lane == 0) {
        __threadfence();
        atomicAdd(&job->done, 1);
    }
}

// Take chunks of the walks' open passes, one warp at a time (sampling modes;
// the helper blocks, grid rows >= bulk_rows). Lane 0 looks for an open pass
// with an unclaimed chunk, starting at a sequence of its own, and claims one
// chunk; the warp computes it. A pass's parameters were written before it was
// opened; they are read from L2 after the claim. The warps keep looking until
// every walk has finished (or their budget ran out). Streaming blocks do not
// help: their pass chunks (compute-heavy) held back the bulk pass, which is
// the longer of the two for 64 sequences of 64 fp32 p and q rows over 151936
// tokens (907-909 us with their help, 882-892 without).
template <int MODE, bool BF16>
__device__ void help_passes(const AcceptArgs &a, int warp, int lane, double *invT) {
    const long long t0 = clock64();
    int start = (int)((blockIdx.y * gridDim.x + blockIdx.x) * kWarps + warp) % a.B;
    for (;;) {
        int b = -1, j = -1;
        bool leave = ld_relaxed(a.walkers_done) >= (uint32_t)a.B || clock64() - t0 > kHelperBudget;
        leave = __shfl_sync(0xffffffffu, leave, 0);
        if (leave) return;
        // the lanes read 32 sequences' pass words at once; lane 0 claims from
        // the first open pass with a chunk left
        for (int t0s = 0; t0s < a.B && j < 0; t0s += 32) {
            const int bb = (start + t0s + lane) % a.B;
            unsigned long long w = 0;
            if (t0s + lane < a.B) w = ld_relaxed_u64(&job_of(a, bb)->word);
            const uint32_t g = (uint32_t)(w >> 32);
            const unsigned open = __ballot_sync(0xffffffffu, g != 0 && (uint32_t)w < (uint32_t)a.nch);
            for (unsigned m = open; m && j < 0; m &= m - 1) {
                const int src = __ffs(m) - 1;
                const int cb = __shfl_sync(0xffffffffu, bb, src);
                int jj = -1;
                if (lane == 0) jj = claim_chunk(&job_of(a, cb)->word, a.nch);
                jj = __shfl_sync(0xffffffffu, jj, 0);
                if (jj >= 0) {
                    b = cb;
                    j = jj;
                }
            }
        }
        if (j < 0) {
            __nanosleep(256);
            continue;
        }
        start = b;  // stay with this pass while it has chunks
        __threadfence();
        SharedPass *job = job_of(a, b);
        const int kind = __ldcg(&job->kind), node = __ldcg(&job->node), L = __ldcg(&job->L);
        if (kind == 0)
            for (int l = lane; l <= L; l += 32) invT[l] = __ldcg(&job->invT[l]);
        __syncwarp();
        RowStat ps, qs;
        ps.C = __ldcg(&job->ps.C);
        ps.S = __ldcg(reinterpret_cast<const unsigned long long *>(&job->ps.S));
        ps.invS = __ldcg(&job->ps.invS);
        qs.C = __ldcg(&job->qs.C);
        qs.S = __ldcg(reinterpret_cast<const unsigned long long *>(&job->qs.S));
        qs.invS = __ldcg(&job->qs.invS);
        pass_chunk<MODE, BF16>(a, b, kind, node, L, ps, qs, invT, j, lane);
        __syncwarp();  // invT is rewritten by the next claim
    }
}

// Warp 0 copies one chunk of a row into shared memory as fp32 (coalesced
// 16-byte loads, all in flight together); positions past the row get -inf.
template <bool BF16>
__device__ void stage_chunk(const char *row, int c0, int clen, float *dst, int lane) {
    using VT = Vec<BF16>;
    constexpr int NVW = A11S_CHUNK / (32 * VT::EPV);  // vectors per lane
    constexpr int G = 8;                               // in flight per lane
#pragma unroll
    for (int i0 = 0; i0 < NVW; i0 += G) {
        uint4 d[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const int e0 = ((i0 + g) * 32 + lane) * VT::EPV;
            const uint32_t ninf = BF16 ? 0xFF80FF80u : 0xFF800000u;
            d[g] = e0 < clen ? ldg_stream(row + (size_t)(c0 + e0) * VT::ESZ) : make_uint4(ninf, ninf, ninf, ninf);
        }
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int e = 0; e < VT::EPV; ++e) dst[((i0 + g) * 32 + lane) * VT::EPV + e] = VT::at(d[g], e);
    }
    __syncwarp();
}

// Four logits at chunk-relative position pos (a multiple of 4; rows are
// 16-byte aligned and the vocab a multiple of the vector width, so the
// four stay inside the row).
template <bool BF16>
__device__ __forceinline__ void load4(const char *row, int pos, float v[4]) {
    if (BF16) {
        const uint2 d = __ldg(reinterpret_cast<const uint2 *>(row + (size_t)pos * 2));
        v[0] = bf16lo(d.x); v[1] = bf16hi(d.x); v[2] = bf16lo(d.y); v[3] = bf16hi(d.y);
    } else {
        const uint4 d = __ldg(reinterpret_cast<const uint4 *>(row + (size_t)pos * 4));
        v[0] = __uint_as_float(d.x); v[1] = __uint_as_float(d.y);
        v[2] = __uint_as_float(d.z); v[3] = __uint_as_float(d.w);
    }
}

// Chunk selection of the two-level inverse CDF (warp 0): t = floor(u * sum A),
// j = first chunk whose inclusive prefix of A exceeds t, t2 = floor((t -
// prefix_before_j) * Lc_j / A_j). Lane l owns chunks [4 l, 4 l + 4).
__device__ bool pick_chunk(float u, const uint64_t *A, const uint64_t *Lc, int nch, int lane, int &j_out,
                           uint64_t &t2_out) {
    static_assert(A11S_MAX_VOCAB / A11S_CHUNK <= 4 * 32, "four chunks per lane");
    uint64_t a4[4], mine = 0;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        const int j = 4 * lane + g;
        a4[g] = j < nch ? A[j] : 0ull;
        mine += a4[g];
    }
    uint64_t incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint64_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    const uint64_t tot = __shfl_sync(0xffffffffu, incl, 31);
    if (tot == 0) return false;
    uint64_t t = __double2ull_rz(__dmul_rn((double)u, __ull2double_rn(tot)));
    if (t >= tot) t = tot - 1;
    uint64_t acc = incl - mine;
    const bool here = acc <= t && t - acc < mine;
    int j = -1;
    uint64_t t2 = 0;
    if (here) {
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            if (j < 0 && acc + a4[g] > t) {
                j = 4 * lane + g;
                const unsigned __int128 prod = (unsigned __int128)(t - acc) * Lc[j];
                t2 = (uint64_t)(prod / a4[g]);
            }
            if (j < 0) acc += a4[g];
        }
    }
    const unsigned who = __ballot_sync(0xffffffffu, here);
    if (!who) return false;  // unreachable: t < tot
    const int src = __ffs(who) - 1;
    j_out = __shfl_sync(0xffffffffu, j, src);
    t2_out = __shfl_sync(0xffffffffu, t2, src);
    return j_out >= 0;
}

// Greedy argmax of a row (warp 0): first chunk holding the row max, then the
// first token equal to it in that chunk (staged in shared memory).
template <bool BF16>
__device__ int row_argmax(const char *row, const float *cmax, int nch, int V, float *stage, int lane) {
    float M = -INFINITY;  // cmax: the row's chunk maxima in shared memory
    for (int j = lane; j < nch; j += 32) M = fmaxf(M, cmax[j]);
    M = warp_fmax(M);
    int jstar = INT_MAX;
    for (int j0 = 0; j0 < nch && jstar == INT_MAX; j0 += 32) {
        const int j = j0 + lane;
        const unsigned hit = __ballot_sync(0xffffffffu, j < nch && cmax[j] == M);
        if (hit) jstar = j0 + __ffs(hit) - 1;
    }
    if (jstar == INT_MAX) return 0;  // unreachable for rows without NaN
    const int c0 = jstar * A11S_CHUNK, clen = min(A11S_CHUNK, V - c0);
    stage_chunk<BF16>(row, c0, clen, stage, lane);
    int first = INT_MAX;  // smallest position equal to M (rotated reads, order-free min)
    for (int s = 0; s < 64; ++s) {
        const int e = lane * 64 + ((s + lane) & 63);
        if (e < clen && stage[e] == M) first = min(first, e);
    }
    first = -warp_max(-first);  // warp min
    __syncwarp();
    return c0 + (first == INT_MAX ? 0 : first);
}

// Greedy argmax of a row from its records in shared memory (warp 0): the same
// choice as row_argmax (first chunk holding the row max; in it, the recorded
// first position of that max) without reading the row.
__device__ int row_argmax_rec(const float *cmax, const int32_t *arg, int nch, int lane) {
    float M = -INFINITY;  // cmax: the row's chunk maxima in shared memory
    for (int j = lane; j < nch; j += 32) M = fmaxf(M, cmax[j]);
    M = warp_fmax(M);
    int jstar = INT_MAX;
    for (int j0 = 0; j0 < nch && jstar == INT_MAX; j0 += 32) {
        const int j = j0 + lane;
        const unsigned hit = __ballot_sync(0xffffffffu, j < nch && cmax[j] == M);
        if (hit) jstar = j0 + __ffs(hit) - 1;
    }
    if (jstar == INT_MAX) return 0;  // every chunk maximum is NaN
    const int f = arg[jstar];
    return jstar * A11S_CHUNK + (f == INT_MAX ? 0 : f);
}

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------
template <int MODE, bool BF16>
__global__ void __launch_bounds__(kThreads, 2) accept_kernel(const AcceptArgs a) {
    const int b = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __shared__ double s_invT[MODE == A11S_ACCEPT_GREEDY ? 1 : kWarps][A11S_MAX_WALK_LEVELS + 1];
    // The launch may overlap the record-init kernel before it (programmatic
    // dependent launch): everything it writes (status, counters, records, pass
    // area) is touched only after this wait, which returns once that kernel
    // has completed and its writes are visible. Without such a launch it
    // returns at once.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if ((int)blockIdx.y >= a.bulk_rows) {  // helper block (sampling modes only)
        if constexpr (MODE != A11S_ACCEPT_GREEDY) help_passes<MODE, BF16>(a, warp, lane, s_invT[warp]);
        return;
    }
    int n_live = a.n_nodes ? a.n_nodes[b] : a.N;
    const bool seq_ok = n_live >= 1 && n_live <= a.N;
    if (!seq_ok) n_live = 0;
    const size_t row_bytes = (size_t)a.stride * (BF16 ? 2 : 4);

    // ---------------- phase 1: chunk maxima ----------------
    // Units of a sequence: first the root rows' chunks (the p root, and the q
    // root in DRAFT mode), then the other rows in index order (in DRAFT mode
    // p row i then q row i), a row's chunks consecutive, so the rows near the
    // root, which the walk visits first, are recorded first. Grid row 0 is the
    // sequence's walker and streams nothing; root_blocks root rows take the
    // root units (chunk maxima, and first positions in GREEDY or weight sums in
    // the sampling modes), one per warp, so every root is recorded early by
    // many SMs at once. (root_blocks = 0 only in GREEDY with chunk keys, whose
    // records are all written before the launch.) The streaming rows take the
    // other units in slices; the root rows alternate with the first of them.
    // A small GREEDY pass runs as one wave instead (a.rr > 0), with no root
    // blocks.
    constexpr int kRootRows = MODE == A11S_ACCEPT_STOCH_DRAFT ? 2 : 1;
    const int n_root_units = kRootRows * a.nch;
    int u0 = 0, u1 = 0, ustep = kWarps;
    if (a.rr > 0) {
        // One wave (a small pass): rows 1 .. rr take unit u on row
        // 1 + (u / kWarps) % rr, warp u % kWarps, so the units finish in their
        // order: the roots first, then the rows in index order, while every
        // block lives for the whole pass.
        if (blockIdx.y >= 1) {
            u0 = (blockIdx.y - 1) * kWarps;
            u1 = a.units_per_seq;
            ustep = a.rr * kWarps;
        }
    } else if (blockIdx.y == 0 && a.root_blocks == 0) {
        // without root blocks the walker records its root itself; with chunk
        // keys every record is written before the launch
        u1 = a.keys ? 0 : n_root_units;
    } else if (blockIdx.y >= 1 && (int)blockIdx.y < a.bulk_rows) {
        // The first root_pairs root rows alternate with streaming rows (root
        // first), so the root blocks' compute-heavy units (weight sums in the
        // sampling modes) run beside memory-bound streaming blocks; then the
        // other root rows, then the other streaming rows.
        const int pairs = a.root_pairs, y = (int)blockIdx.y - 1, y2 = y - 2 * pairs;
        int root_i = -1, slice_i = -1;
        if (y < 2 * pairs) (y & 1 ? slice_i : root_i) = y >> 1;
        else if (y2 < a.root_blocks - pairs) root_i = pairs + y2;
        else slice_i = pairs + (y2 - (a.root_blocks - pairs));
        if (root_i >= 0) {
            u0 = root_i * kWarps;
            u1 = min(u0 + kWarps, n_root_units);
        } else {
            u0 = n_root_units + slice_i * a.slice;
            u1 = min(u0 + a.slice, a.units_per_seq);
        }
    }
    int bad = 0;
    for (int u = u0 + warp; u < u1; u += ustep) {
        int j, r;
        if (u < n_root_units) {
            j = u / kRootRows;
            r = (u - j * kRootRows) ? a.N : 0;
        } else {
            // rows 1..N-1 in index order, in STOCH_DRAFT each p row followed by
            // its q row (a visited node needs both)
            const int v = u - n_root_units;
            const int q = v / a.nch;
            j = v - q * a.nch;
            r = kRootRows == 2 ? ((q & 1) ? a.N + 1 + (q >> 1) : 1 + (q >> 1)) : 1 + q;
        }
        const bool isq = r >= a.N;
        const int node = isq ? r - a.N : r;
        if (node >= n_live) continue;
        const char *row = reinterpret_cast<const char *>(isq ? a.draft : a.target) + ((size_t)b * a.N + node) * row_bytes;
        const int c0 = j * A11S_CHUNK, clen = min(A11S_CHUNK, a.V - c0);
        int first = 0;
        // with chunk keys only the root units of the sampling modes run here:
        // the maximum comes from the key, the weight sums from the row
        const float m = a.keys ? key_value(__ldg(a.keys + ((size_t)b * a.N + node) * a.nch + j))
                        : MODE == A11S_ACCEPT_GREEDY ? chunk_max_first<BF16>(row, c0, clen, lane, first)
                                                     : chunk_max<BF16>(row, c0, clen, lane);
        bad |= !(m < INFINITY);  // the NaN-propagating max is NaN or +Inf
        if (MODE != A11S_ACCEPT_GREEDY && m > -INFINITY && !(fabsf(__fmul_rn(m, a.k)) < 16777216.0f)) bad = 1;
        const size_t rrow = (size_t)b * a.rows_per_seq + r;
        if (MODE != A11S_ACCEPT_GREEDY && node == 0) {
            // The walk always starts at the root: its weight sums are taken
            // here, while the chunk is hot in L2, and stored before the
            // chunk's record, which tells the walker they are there.
            const int32_t f = m < INFINITY ? frame_of(m, a.k) : A11S_FRAME_NONE;
            const uint64_t s = f == A11S_FRAME_NONE ? 0ull : chunk_wsum<BF16>(row, c0, clen, a.k, (float)f, lane);
            if (lane == 0) {
                __stcg(a.root_sums + ((size_t)b * 2 + (isq ? 1 : 0)) * a.nch + j, (unsigned long long)s);
                __threadfence();
            }
        }
        if (lane == 0) {  // each record is written once, over the launch's sentinel
            if (MODE == A11S_ACCEPT_GREEDY) st_relaxed(a.arg + rrow * a.nch + j, (uint32_t)first);
            st_relaxed(a.recs + rrow * a.nch + j, __float_as_uint(m));
        }
    }
    if (warp_or(bad) && lane == 0) report(a.status, A11S_ENONFINITE, b);
    if (blockIdx.y != 0) return;  // a streaming block is done

    // ---------------- phase 2: walk ----------------
    __shared__ WalkSmem sm;
    const int N = a.N, V = a.V, nch = a.nch;
    int32_t *an = a.acc_nodes + (size_t)b * N;
    int32_t *at = a.acc_tokens + (size_t)b * N;
    const float *cmax_b = a.recs + (size_t)b * a.rows_per_seq * nch;  // chunk maxima of the sequence's rows
    const int32_t *arg_b = MODE == A11S_ACCEPT_GREEDY ? a.arg + (size_t)b * N * nch : nullptr;
    // Records of row r (p rows 0..N-1, q rows N..2N-1 in DRAFT) if complete,
    // else null; every thread gets the same answer (thread j < nch checks
    // chunk j). The root rows' were written by this block before the walk.
    // GREEDY also gets the values in shared memory (sm.cmx, sm.carg).
    auto records = [&](int r) -> const float * {
        const float *rec = cmax_b + (size_t)r * nch;
        bool mine = true;
        if ((int)threadIdx.x < nch) {
            uint32_t v, pv;
            mine = record_ready(rec + threadIdx.x, arg_b ? arg_b + (size_t)r * nch + threadIdx.x : nullptr,
                                a.wait_records != 0, v, pv);
            if (MODE == A11S_ACCEPT_GREEDY) {
                sm.cmx[threadIdx.x] = __uint_as_float(v);
                sm.carg[threadIdx.x] = (int32_t)pv;
            }
            // a root chunk's weight sum was stored before its record: this
            // thread reads it after the record (row_stats_into, chunk j = thread j)
            if (MODE != A11S_ACCEPT_GREEDY && (r == 0 || r == N)) __threadfence();
        }
        return __syncthreads_and(mine) ? rec : nullptr;
    };
    const char *tgt_b = reinterpret_cast<const char *>(a.target) + (size_t)b * N * row_bytes;
    const char *drf_b = MODE == A11S_ACCEPT_STOCH_DRAFT
                            ? reinterpret_cast<const char *>(a.draft) + (size_t)b * N * row_bytes
                            : nullptr;
    // stage the tree (and uniforms) once: every later lookup is a shared-memory read
    for (int i = threadIdx.x; i < n_live; i += blockDim.x) {
        sm.tok[i] = a.tokens[(size_t)b * N + i];
        sm.par[i] = a.parents[(size_t)b * N + i];
        if (MODE != A11S_ACCEPT_GREEDY) sm.uni[i] = a.uniforms[(size_t)b * N + i];
    }
    if (threadIdx.x == 0) {
        sm.gen = 0;
        sm.no_helpers = a.jobs ? 0 : 1;
    }
    __syncthreads();
    // A pass over visited node nd's rows shared with the helper blocks (see
    // SharedPass), every thread: publish, take chunks alongside the helpers,
    // wait (bounded) for the helpers' last chunks. False when this walk no
    // longer shares its passes (a wait ran out once): the caller computes the
    // pass in this block. Kind 0 reads sm.fr / sm.qfr / sm.invT / sm.L and the
    // row statistics sm.ps / sm.qs.
    auto run_pass = [&](int kind, int nd) -> bool {
        if (sm.no_helpers) return false;
        SharedPass *job = job_of(a, b);
        if (kind == 0) {
            int32_t *jfr = job_fr(a, b), *jqfr = job_qfr(a, b);
            for (int j = threadIdx.x; j < nch; j += blockDim.x) { jfr[j] = sm.fr[j]; jqfr[j] = sm.qfr[j]; }
            for (int l = threadIdx.x; l <= sm.L; l += blockDim.x) job->invT[l] = sm.invT[l];
        }
        if (threadIdx.x == 0) {
            job->done = 0;
            job->node = nd;
            job->L = sm.L;
            job->kind = kind;
            job->ps = sm.ps;
            job->qs = sm.qs;
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            sm.gen += 1;
            atomicExch(&job->word, (unsigned long long)sm.gen << 32);  // open the pass
        }
        __syncthreads();
        const uint32_t gen = sm.gen;
        const int L = sm.L;
        const RowStat ps = sm.ps, qs = sm.qs;
        for (;;) {  // this block takes chunks too, one warp at a time
            int j = -1;
            if (lane == 0) j = claim_chunk(&job->word, nch);
            j = __shfl_sync(0xffffffffu, j, 0);
            if (j < 0) break;
            pass_chunk<MODE, BF16>(a, b, kind, nd, L, ps, qs, sm.invT, j, lane);
        }
        __syncthreads();
        if (threadIdx.x == 0) {  // the helpers' last chunks (bounded wait)
            const long long t0 = clock64();
            bool all = false;
            while (!(all = ld_relaxed(&job->done) >= (uint32_t)nch)) {
                if (clock64() - t0 > kPassWaitBudget) break;
                __nanosleep(128);
            }
            if (!all) {
                // never reuse this pass slot (a late chunk could land in a newer
                // pass): close it and compute the rest of the walk in this block
                atomicExch(&job->word, ((unsigned long long)gen << 32) | kClosedCount);
                sm.no_helpers = 1;
            }
            __threadfence();
        }
        __syncthreads();
        const bool shared_ok = sm.no_helpers == 0;
        if (shared_ok && kind == 1) {
            for (int j = threadIdx.x; j < nch; j += blockDim.x) {
                sm.fr[j] = __ldcg(job_fr(a, b) + j);
                sm.sum[j] = __ldcg(job_sums(a, b) + j);
                if (MODE == A11S_ACCEPT_STOCH_DRAFT) {
                    sm.qfr[j] = __ldcg(job_qfr(a, b) + j);
                    sm.qsum[j] = __ldcg(job_qsums(a, b) + j);
                }
            }
        } else if (shared_ok) {
            for (int j = threadIdx.x; j < nch; j += blockDim.x) sm.tmp[j] = __ldcg(job_sums(a, b) + j);
        }
        __syncthreads();
        return shared_ok;
    };
    if (warp == 0) {
        int okl = seq_ok ? 1 : 0;
        for (int i = 1 + lane; i < n_live; i += 32)
            if (sm.par[i] < 0 || sm.par[i] >= i || sm.tok[i] < 0 || sm.tok[i] >= V) okl = 0;
        okl = __all_sync(0xffffffffu, okl);
        if (lane == 0) {
            sm.ok = okl;
            if (!okl) report(a.status, A11S_EBOUNDS, b);
        }
        for (int i = lane; i < N; i += 32) { an[i] = -1; at[i] = -1; }
        if (a.node_probs)
            for (int i = lane; i < N; i += 32) a.node_probs[(size_t)b * N + i] = 0.0f;
    }
    __syncthreads();
    if (!sm.ok) {
        if (threadIdx.x == 0) {
            a.accept_len[b] = 0;
            a.bonus[b] = -1;
            atomicAdd(a.walkers_done, 1);  // helpers leave once every walk has finished
        }
        return;
    }

    // node probabilities p(tokens[i]) in the parent's row (sampling modes, optional):
    // one statistics pass per row that has children
    if (MODE != A11S_ACCEPT_GREEDY && a.node_probs) {
        for (int r = 0; r < n_live; ++r) {
            bool has_child = false;
            for (int c = r + 1; c < n_live && !has_child; ++c) has_child = sm.par[c] == r;
            if (!has_child) continue;
            const char *prow = tgt_b + (size_t)r * row_bytes;
            const float *rec = records(r);
            const bool rec_q = MODE != A11S_ACCEPT_STOCH_DRAFT || records(N + r) != nullptr;
            if (!(r != 0 && rec && rec_q && run_pass(1, r))) {
                // the root's sums come from the bulk pass once its records are in
                const unsigned long long *rs = r == 0 && rec ? a.root_sums + (size_t)b * 2 * nch : nullptr;
                row_stats_into<BF16>(prow, cmax_b, rs, rs ? nullptr : rec, nch, V, a.k, sm.fr, sm.sum, warp, lane,
                                     a.status, b);
            }
            __syncthreads();
            if (warp == 0) {
                const RowStat rs = combine_sums(sm.fr, sm.sum, nch, lane);
                for (int c = r + 1 + lane; c < n_live; c += 32) {
                    if (sm.par[c] != r) continue;
                    const int x = sm.tok[c], j = x / A11S_CHUNK;
                    a.node_probs[(size_t)b * N + c] = prob_of(load_logit(prow, x, BF16), a.k, sm.fr[j],
                                                              chunk_scale(rs, sm.fr[j]));
                }
            }
            __syncthreads();
        }
    }

    int alen = 0, node = 0, bonus = -1;
    bool failed = false;
    if (MODE == A11S_ACCEPT_GREEDY) {
        // Per visited node: its chunk maxima and first positions (records, or
        // taken from the row by every warp); warp 0 finds the argmax and the
        // matching child.
        for (;;) {
            const char *row = tgt_b + (size_t)node * row_bytes;
            // the row's chunk maxima and first positions, staged by records()
            // (the root's were written by this block), else taken from the row
            const bool rec = records(node) != nullptr;
            if (!rec) row_cmax_into<BF16>(row, nullptr, nch, V, sm.cmx, warp, lane, a.status, b);
            if (warp == 0) {
                const int am = rec ? row_argmax_rec(sm.cmx, sm.carg, nch, lane)
                                   : row_argmax<BF16>(row, sm.cmx, nch, V, sm.cp, lane);
                int next = INT_MAX;
                for (int c0 = node + 1; c0 < n_live && next == INT_MAX; c0 += 32) {
                    const int c = c0 + lane;
                    const unsigned m = __ballot_sync(0xffffffffu, c < n_live && sm.par[c] == node && sm.tok[c] == am);
                    if (m) next = c0 + __ffs(m) - 1;
                }
                if (next == INT_MAX) {
                    bonus = am;
                } else {
                    if (lane == 0) { an[alen] = next; at[alen] = sm.tok[next]; }
                    ++alen;
                }
                if (lane == 0) sm.child = next == INT_MAX ? -1 : next;
            }
            __syncthreads();
            node = sm.child;
            __syncthreads();  // every thread has read sm.child before warp 0 rewrites it
            if (node < 0) break;
        }
    } else {
        // Sampling walk. Every warp computes a visited row's statistics (and the
        // residual passes of DRAFT); warp 0 makes the decisions from shared memory.
        if (threadIdx.x == 0) { sm.node = 0; sm.alen = 0; }
        __syncthreads();
        for (;;) {  // one iteration per visited node
            const int nd = sm.node;
            const char *prow = tgt_b + (size_t)nd * row_bytes;
            const char *qrow = MODE == A11S_ACCEPT_STOCH_DRAFT ? drf_b + (size_t)nd * row_bytes : nullptr;
            const float *rec_p = records(nd);
            const float *rec_q = MODE == A11S_ACCEPT_STOCH_DRAFT ? records(N + nd) : nullptr;
            const bool have = rec_p && (MODE != A11S_ACCEPT_STOCH_DRAFT || rec_q);
            // a recorded non-root row: its statistics shared with the helpers;
            // the root's come from the bulk pass once its records are in
            const bool shared = nd != 0 && have && run_pass(1, nd);
            if (!shared) {
                const unsigned long long *rs_p = nd == 0 && have ? a.root_sums + (size_t)b * 2 * nch : nullptr;
                row_stats_into<BF16>(prow, cmax_b, rs_p, rs_p ? nullptr : rec_p, nch, V, a.k, sm.fr, sm.sum, warp, lane,
                                     a.status, b);
                if (MODE == A11S_ACCEPT_STOCH_DRAFT)
                    row_stats_into<BF16>(qrow, cmax_b + (size_t)N * nch, rs_p ? rs_p + nch : nullptr,
                                         rs_p ? nullptr : rec_q, nch, V, a.k, sm.qfr, sm.qsum, warp, lane, a.status, b);
            }
            __syncthreads();
            if (warp == 0) {
                sm.ps = combine_sums(sm.fr, sm.sum, nch, lane);
                if (MODE == A11S_ACCEPT_STOCH_DRAFT) sm.qs = combine_sums(sm.qfr, sm.qsum, nch, lane);
                for (int j = lane; j < nch; j += 32) sm.sub[j] = sm.sum[j];
                // children of nd in index order, and their logits, into shared memory
                int nk = 0;
                for (int c0 = nd + 1; c0 < n_live; c0 += 32) {
                    const int c = c0 + lane;
                    const bool hit = c < n_live && sm.par[c] == nd;
                    const unsigned m = __ballot_sync(0xffffffffu, hit);
                    if (hit) sm.kids[nk + __popc(m & ((1u << lane) - 1u))] = c;
                    nk += __popc(m);
                }
                __syncwarp();
                for (int kk = lane; kk < nk; kk += 32) {
                    const int x = sm.tok[sm.kids[kk]];
                    sm.kl[kk] = load_logit(prow, x, BF16);
                    if (MODE == A11S_ACCEPT_STOCH_DRAFT) sm.kq[kk] = load_logit(qrow, x, BF16);
                }
                __syncwarp();
                if (lane == 0) {
                    sm.nk = nk;
                    sm.ck = 0;
                    sm.S_eff = sm.ps.S;
                    sm.nexcl = 0;
                    sm.L = 0;
                    sm.action = 0;
                    if (sm.ps.S == 0 || (MODE == A11S_ACCEPT_STOCH_DRAFT && sm.qs.S == 0)) {
                        report(a.status, A11S_ENONFINITE, b);
                        sm.action = 3;  // abort
                    }
                }
                __syncwarp();
            }
            __syncthreads();
            const bool abort_walk = sm.action == 3;
            __syncthreads();  // every thread has read sm.action before warp 0 rewrites it
            if (abort_walk) { failed = true; break; }
            bool moved = false;
            if (MODE == A11S_ACCEPT_STOCH_ONEHOT) {
                // Deterministic drafts: no row passes between siblings, so warp 0
                // tries every child without block barriers. All lanes evaluate the
                // same shared-memory values; lane 0 writes.
                if (warp == 0) {
                    int next = -1;
                    for (int kk = 0; kk < sm.nk; ++kk) {
                        const int c = sm.kids[kk], x = sm.tok[c], j = x / A11S_CHUNK;
                        bool ex = false;
                        for (int e = 0; e < sm.nexcl; ++e) ex |= sm.excl[e] == x;
                        float lt = 0.0f;
                        const uint64_t S_eff = sm.S_eff;
                        if (!ex && S_eff) {
                            RowStat re = sm.ps;
                            re.S = S_eff;
                            re.invS = __ddiv_rn(1.0, __ull2double_rn(S_eff));
                            lt = prob_of(sm.kl[kk], a.k, sm.fr[j], chunk_scale(re, sm.fr[j]));
                        }
                        if (accept_linear(sm.uni[c], lt, 1.0f)) { next = c; break; }
                        if (!ex) {
                            __syncwarp();
                            if (lane == 0) {
                                // S_eff = sum_j sub[j] >> (C - fr[j]) (as combine_sums
                                // forms S); only chunk j's term changes
                                sm.excl[sm.nexcl++] = x;
                                if (sm.fr[j] != A11S_FRAME_NONE) {
                                    const int d = sm.ps.C - sm.fr[j];
                                    const uint64_t before = d > 63 ? 0ull : (sm.sub[j] >> d);
                                    sm.sub[j] -= det_weight(sm.kl[kk], a.k, (float)sm.fr[j]);
                                    sm.S_eff = sm.S_eff - before + (d > 63 ? 0ull : (sm.sub[j] >> d));
                                }
                            }
                            __syncwarp();
                        }
                    }
                    if (lane == 0 && next >= 0) {
                        an[sm.alen] = next;
                        at[sm.alen] = sm.tok[next];
                        sm.alen += 1;
                        sm.node = next;
                    }
                    if (lane == 0) sm.child = next;
                    __syncwarp();
                }
                __syncthreads();
                moved = sm.child >= 0;
                __syncthreads();
            } else {
                for (;;) {  // children of this node, in index order
                    if (warp == 0 && lane == 0) {
                        if (sm.ck >= sm.nk) {
                            sm.action = 0;  // no child left: draw the bonus here
                        } else {
                            const int kk = sm.ck++;
                            const int c = sm.kids[kk], x = sm.tok[c], j = x / A11S_CHUNK;
                            sm.child = c;
                            const float p0 = prob_of(sm.kl[kk], a.k, sm.fr[j], chunk_scale(sm.ps, sm.fr[j]));
                            const float qx = prob_of(sm.kq[kk], a.k, sm.qfr[j], chunk_scale(sm.qs, sm.qfr[j]));
                            const float lt = level_prob(p0, qx, sm.L, sm.invT);
                            sm.action = accept_linear(sm.uni[c], lt, qx) ? 1 : (sm.L < A11S_MAX_WALK_LEVELS ? 4 : 2);
                        }
                    }
                    __syncthreads();
                    const int action = sm.action;
                    __syncthreads();  // every thread has read sm.action before it changes
                    if (action == 1) {  // accepted: move to the child
                        if (threadIdx.x == 0) {
                            an[sm.alen] = sm.child;
                            at[sm.alen] = sm.tok[sm.child];
                            sm.alen += 1;
                            sm.node = sm.child;
                        }
                        moved = true;
                        __syncthreads();
                        break;
                    }
                    if (action == 0) break;
                    if (action == 4) {
                        // DRAFT residual pass: chunk totals of level L+1 into sm.tmp,
                        // shared with the helper blocks (see SharedPass).
                        const int L = sm.L;
                        const bool local = !run_pass(0, nd);
                        if (local) {
                            for (int j = warp; j < nch; j += kWarps) {
                                const int c0 = j * A11S_CHUNK, clen = min(A11S_CHUNK, V - c0);
                                const uint64_t sum = resid_chunk_sum<BF16>(prow, qrow, c0, clen, a.k, sm.fr[j], sm.qfr[j],
                                                                           chunk_scale(sm.ps, sm.fr[j]),
                                                                           chunk_scale(sm.qs, sm.qfr[j]), L, sm.invT, lane);
                                if (lane == 0) sm.tmp[j] = sum;
                            }
                        }
                        __syncthreads();
                        if (warp == 0) {
                            uint64_t tot = 0;
                            for (int j = lane; j < nch; j += 32) tot += sm.tmp[j];
                            tot = warp_sum_u64(tot);
                            if (tot) {
                                for (int j = lane; j < nch; j += 32) sm.lvl[j] = sm.tmp[j];
                                if (lane == 0) {
                                    sm.L += 1;
                                    sm.T[sm.L] = tot;
                                    sm.invT[sm.L] = __ddiv_rn(1.0, __ull2double_rn(tot));
                                }
                            }
                        }
                        __syncthreads();
                    }
                    // action 2 / 4: rejected, try the next child
                }
            }
            if (!moved) break;
        }
        // bonus draw at sm.node: warp 0 picks the chunk, every thread scans it
        if (!failed) {
            const int nd = sm.node;
            const char *prow = tgt_b + (size_t)nd * row_bytes;
            const bool draft_lvl = MODE == A11S_ACCEPT_STOCH_DRAFT && sm.L > 0;
            const bool use_excl = MODE == A11S_ACCEPT_STOCH_ONEHOT && sm.S_eff != 0;
            if (warp == 0) {
                int j = 0;
                uint64_t t2 = 0;
                bool okp;
                if (draft_lvl) {
                    okp = pick_chunk(sm.uni[0], sm.lvl, sm.lvl, nch, lane, j, t2);
                } else {
                    // A_j in the row frame, local totals Lc_j (sm.tmp / sm.lvl as scratch)
                    for (int jj = lane; jj < nch; jj += 32) {
                        const uint64_t loc = use_excl ? sm.sub[jj] : sm.sum[jj];
                        sm.tmp[jj] = loc;
                        const int32_t f = sm.fr[jj];
                        const int d = sm.ps.C - f;
                        sm.lvl[jj] = (f == A11S_FRAME_NONE || d > 63) ? 0ull : (loc >> d);
                    }
                    __syncwarp();
                    okp = pick_chunk(sm.uni[0], sm.lvl, sm.tmp, nch, lane, j, t2);
                }
                if (lane == 0) {
                    sm.bj = okp ? j : -1;
                    sm.bt2 = t2;
                }
            }
            __syncthreads();
            const int j = sm.bj;
            const uint64_t t2 = sm.bt2;
            if (j >= 0) {
                const float k = a.k;
                const int c0 = j * A11S_CHUNK, clen = min(A11S_CHUNK, V - c0);
                const char *pc = prow + (size_t)c0 * (BF16 ? 2 : 4);
                int pos;
                if (draft_lvl) {
                    const char *qc = drf_b + (size_t)nd * row_bytes + (size_t)c0 * (BF16 ? 2 : 4);
                    const int32_t fp = sm.fr[j], fq = sm.qfr[j];
                    const double scp = chunk_scale(sm.ps, fp), scq = chunk_scale(sm.qs, fq);
                    const int L = sm.L;
                    pos = block_scan_chunk(clen, t2, [&](int p0, uint64_t *w) {
                        float pv[4], qv[4];
                        load4<BF16>(pc, p0, pv);
                        load4<BF16>(qc, p0, qv);
                        for (int e = 0; e < 4; ++e) {
                            const float pp = prob_of(pv[e], k, fp, scp), qq = prob_of(qv[e], k, fq, scq);
                            w[e] = level_weight(level_prob(pp, qq, L - 1, sm.invT), qq);
                        }
                    }, sm);
                } else {
                    const float cff = (float)sm.fr[j];
                    const int nex = use_excl ? sm.nexcl : 0;
                    pos = block_scan_chunk(clen, t2, [&](int p0, uint64_t *w) {
                        float l[4];
                        load4<BF16>(pc, p0, l);
                        for (int e = 0; e < 4; ++e) {
                            bool ex = false;
                            for (int x = 0; x < nex; ++x) ex |= sm.excl[x] == c0 + p0 + e;
                            w[e] = ex ? 0ull : det_weight(l[e], k, cff);
                        }
                    }, sm);
                }
                bonus = c0 + pos;
            }
            alen = sm.alen;
        }
    }

    if (threadIdx.x == 0) {
        if (failed) {
            a.accept_len[b] = 0;
            a.bonus[b] = -1;
        } else {
            a.accept_len[b] = alen;
            a.bonus[b] = bonus;
            if (a.stats) {
                unsigned long long *st = reinterpret_cast<unsigned long long *>(a.stats);
                atomicAdd(st + A11S_STAT_STEPS_ACCEPTED, (unsigned long long)(alen > 0));
                atomicAdd(st + A11S_STAT_STEPS_REJECTED, (unsigned long long)(alen == 0));
                atomicAdd(st + A11S_STAT_FALLBACKS, (unsigned long long)(alen == 0));
                atomicAdd(st + A11S_STAT_DRAFT_TOKENS, (unsigned long long)(n_live - 1));
                atomicAdd(st + A11S_STAT_TOTAL_STEPS, 1ull);
                atomicAdd(st + A11S_STAT_EMITTED_TOKENS, (unsigned long long)(alen + 1));
            }
        }
    }
    if (failed && warp == 0)
        for (int i = lane; i < N; i += 32) { an[i] = -1; at[i] = -1; }
    if (threadIdx.x == 0) atomicAdd(a.walkers_done, 1);  // helpers leave once every walk has finished
}

// Before every acceptance launch: clear the status word and set every record
// to kUnrecorded (one launch instead of two memsets).
__global__ void accept_init_kernel(StatusWord *st, uint4 *recs, size_t n16, uint4 *zero, size_t z16) {
    // the acceptance kernel after this one may be scheduled now: it waits for
    // this grid's completion before it reads anything written here
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const size_t i0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i0 == 0) {
        *st = StatusWord{};
        reinterpret_cast<uint4 *>(st)[1] = make_uint4(0, 0, 0, 0);  // the finished-walk counter at byte 16
    }
    const uint4 u = make_uint4(kUnrecorded, kUnrecorded, kUnrecorded, kUnrecorded);
    for (size_t i = i0; i < n16; i += (size_t)gridDim.x * blockDim.x) recs[i] = u;
    for (size_t i = i0; i < z16; i += (size_t)gridDim.x * blockDim.x) zero[i] = make_uint4(0, 0, 0, 0);
}

cudaError_t launch_accept_init(StatusWord *st, void *recs, size_t bytes, void *zero, size_t zero_bytes,
                               cudaStream_t s) {
    const size_t n16 = bytes / 16, z16 = zero ? zero_bytes / 16 : 0;
    const size_t n = std::max(n16, z16);
    const unsigned blocks = (unsigned)std::min<size_t>((n + 255) / 256, 4 * 148);
    accept_init_kernel<<<blocks ? blocks : 1, 256, 0, s>>>(st, reinterpret_cast<uint4 *>(recs), n16,
                                                           reinterpret_cast<uint4 *>(zero), z16);
    return cudaGetLastError();
}

__global__ void accept_keys_init_kernel(const AcceptArgs a, int mode, uint4 *zero, size_t z16) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // as in accept_init_kernel
    const size_t i0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x, step = (size_t)gridDim.x * blockDim.x;
    if (i0 == 0) {
        *a.status = StatusWord{};
        reinterpret_cast<uint4 *>(a.status)[1] = make_uint4(0, 0, 0, 0);  // the finished-walk counter at byte 16
    }
    for (size_t i = i0; i < z16; i += step) zero[i] = make_uint4(0, 0, 0, 0);
    // records [B][N][nch] (rows_per_seq == N in GREEDY and STOCH_ONEHOT), the keys in the same order
    const size_t n = (size_t)a.B * a.N * a.nch;
    for (size_t i = i0; i < n; i += step) {
        const size_t r = i / (size_t)a.nch;
        const int node = (int)(r % (size_t)a.N), b = (int)(r / (size_t)a.N);
        int n_live = a.n_nodes ? a.n_nodes[b] : a.N;
        if (n_live < 1 || n_live > a.N) n_live = 0;  // the acceptance kernel reports the bad count
        uint32_t rec = kUnrecorded;
        if (node < n_live) {
            const unsigned long long key = a.keys[i];
            const float m = key_value(key);
            bool bad = !(m < INFINITY);  // NaN or +Inf, as the pass over the logits finds it
            if (mode != A11S_ACCEPT_GREEDY && m > -INFINITY && !(fabsf(__fmul_rn(m, a.k)) < 16777216.0f)) bad = true;
            if (bad) report(a.status, A11S_ENONFINITE, b);
            // the sampling modes' root records are published by the root blocks with their weight sums
            if (mode == A11S_ACCEPT_GREEDY || node != 0) rec = __float_as_uint(m);
            if (mode == A11S_ACCEPT_GREEDY) a.arg[i] = m == m ? key_first(key) : INT_MAX;
        } else if (mode == A11S_ACCEPT_GREEDY) {
            a.arg[i] = -1;
        }
        reinterpret_cast<uint32_t *>(a.recs)[i] = rec;
    }
}

cudaError_t launch_accept_keys_init(int mode, const AcceptArgs &a, void *zero, size_t zero_bytes, cudaStream_t s) {
    const size_t n = std::max((size_t)a.B * a.N * a.nch, zero ? zero_bytes / 16 : 0);
    const unsigned blocks = (unsigned)std::min<size_t>((n + 255) / 256, 4 * 148);
    accept_keys_init_kernel<<<blocks ? blocks : 1, 256, 0, s>>>(a, mode, reinterpret_cast<uint4 *>(zero),
                                                                zero ? zero_bytes / 16 : 0);
    return cudaGetLastError();
}

cudaError_t launch_accept(int mode, bool bf16, const AcceptArgs &a, int grid_y, cudaStream_t s) {
    // sequences fastest: every root block in the first wave; launched as a
    // programmatic dependent of the record-init kernel queued just before it
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(a.B, grid_y);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
#define A11S_LAUNCH(M, BF)                                                   \
    if (mode == M && bf16 == BF) return cudaLaunchKernelEx(&cfg, accept_kernel<M, BF>, a);
    A11S_LAUNCH(A11S_ACCEPT_GREEDY, false)
    A11S_LAUNCH(A11S_ACCEPT_GREEDY, true)
    A11S_LAUNCH(A11S_ACCEPT_STOCH_ONEHOT, false)
    A11S_LAUNCH(A11S_ACCEPT_STOCH_ONEHOT, true)
    A11S_LAUNCH(A11S_ACCEPT_STOCH_DRAFT, false)
    A11S_LAUNCH(A11S_ACCEPT_STOCH_DRAFT, true)
#undef A11S_LAUNCH
    return cudaErrorInvalidValue;
}

}  // namespace a11s
