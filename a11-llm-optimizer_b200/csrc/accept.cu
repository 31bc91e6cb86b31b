// accept.cu - K3: vocab-wide softmax/argmax + acceptance + path select + bonus draw.
//
// One kernel per call.
// Phase 1 (every block, HBM-bound): warps stream 2048-token chunks of every
//   live logits row with 16-byte non-allocating loads and keep one number per
//   chunk: its maximum (NaN-propagating, so a NaN or +Inf is caught here).
//   That is two instructions per logit, the single read of the vocab.
// Phase 2 (the block that completes a sequence, found with a fenced atomic
//   counter; nothing waits): walk the tree from the root.
//   GREEDY  row argmax = first chunk holding the row max, then the first token
//           equal to it inside that chunk (one 2048-token rescan per visited row).
//   STOCH_* the fixed-point softmax statistics (frame c_j = ceil(cmax_j * k),
//           S_j = sum of weights) are computed for the rows the walk visits only,
//           by all 16 warps; then acceptance, residuals and the bonus draw.
// The numbers are exactly those of the oracle (order-independent integer
// sums), so decisions are bit-exact.
//
// Semantics: include/a11spec.h (a11s_accept). Reference behaviour followed:
// src/engine/speculative_verifier.cpp:84-135 (acceptance rule, first rejection
// stops the chain), engine/sampler.py:16 (logits / T).
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

// Chunk max of one row chunk, lane layout: vector i of lane = logits
// [(i*32 + lane) * EPV, +EPV). Positions past the row are -inf.
template <bool BF16>
__device__ __forceinline__ float chunk_max(const char *row, int c0, int clen, int lane) {
    using VT = Vec<BF16>;
    constexpr int G = 8;  // vectors in flight per lane
    float m = -INFINITY;
#pragma unroll
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
            for (int e = 0; e < VT::EPV; ++e) m = max_nan(m, VT::at(d[g], e));
    }
    return warp_max_nan(m);
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
    int32_t excl[A11S_MAX_NODES];
    float cp[A11S_CHUNK];   // one staged chunk of the p row (widened to fp32)
    float cq[A11S_CHUNK];   // and of the q row (DRAFT)
    RowStat ps, qs;
    uint64_t S_eff;
    int32_t nexcl, L, node, alen, cpos, action, child, ok;
};

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

// Every warp of the block: frames and weight sums of one row into fr/sum.
template <bool BF16>
__device__ void row_sums(const char *row, const float *cmax, int nch, int V, float k, int32_t *fr, uint64_t *sum,
                         int warp, int lane) {
    for (int j = warp; j < nch; j += kWarps) {
        const float cm = __ldcg(cmax + j);
        const int32_t f = frame_of(cm, k);
        uint64_t s = 0;
        if (f != A11S_FRAME_NONE) {
            const int c0 = j * A11S_CHUNK;
            s = chunk_wsum<BF16>(row, c0, min(A11S_CHUNK, V - c0), k, (float)f, lane);
        }
        if (lane == 0) {
            fr[j] = f;
            sum[j] = s;
        }
    }
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

// Inverse CDF inside one staged chunk, warp 0: lane l owns tokens
// [64 l, 64 l + 64) of the chunk. wfn(e) gives the weight of chunk position e
// (read from shared memory; lanes read rotated positions to avoid bank
// conflicts, integer sums make the order irrelevant). Returns the chunk
// position of the first token whose running weight exceeds t2 (or the last
// positive-weight position).
template <typename WF>
__device__ int scan_chunk(int clen, uint64_t t2, int lane, WF wfn) {
    const int lo = lane * 64;
    uint64_t mine = 0;
    for (int s = 0; s < 64; ++s) {
        const int e = lo + ((s + lane) & 63);
        if (e < clen) mine += wfn(e);
    }
    uint64_t incl = mine;  // inclusive warp scan
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint64_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    const uint64_t excl = incl - mine;
    const bool here = excl <= t2 && t2 < incl;
    const unsigned who = __ballot_sync(0xffffffffu, here);
    int found = -1;
    if (here) {
        uint64_t acc = excl;
        for (int e = lo; e < min(lo + 64, clen); ++e) {
            acc += wfn(e);
            if (acc > t2) { found = e; break; }
        }
    }
    if (who) return __shfl_sync(0xffffffffu, found, __ffs(who) - 1);
    int last = -1;  // t2 beyond the chunk total (inconsistent totals): last positive weight
    for (int e = lo; e < min(lo + 64, clen); ++e)
        if (wfn(e)) last = e;
    return warp_max(last);
}

// Chunk selection of the two-level inverse CDF (lane 0 of warp 0).
__device__ __forceinline__ bool pick_chunk(float u, const uint64_t *A, const uint64_t *Lc, int nch,
                                           int &j_out, uint64_t &t2_out) {
    uint64_t tot = 0;
    for (int j = 0; j < nch; ++j) tot += A[j];
    if (tot == 0) return false;
    uint64_t t = __double2ull_rz(__dmul_rn((double)u, __ull2double_rn(tot)));
    if (t >= tot) t = tot - 1;
    uint64_t acc = 0;
    int j = 0;
    for (; j < nch; ++j) {
        if (acc + A[j] > t) break;
        acc += A[j];
    }
    if (j >= nch) return false;
    const unsigned __int128 prod = (unsigned __int128)(t - acc) * Lc[j];
    t2_out = (uint64_t)(prod / A[j]);
    j_out = j;
    return true;
}

// Greedy argmax of a row (warp 0): first chunk holding the row max, then the
// first token equal to it in that chunk (staged in shared memory).
template <bool BF16>
__device__ int row_argmax(const char *row, const float *cmax, int nch, int V, float *stage, int lane) {
    float M = -INFINITY;
    for (int j = lane; j < nch; j += 32) M = fmaxf(M, __ldcg(cmax + j));
    M = warp_fmax(M);
    int jstar = INT_MAX;
    for (int j0 = 0; j0 < nch && jstar == INT_MAX; j0 += 32) {
        const int j = j0 + lane;
        const unsigned hit = __ballot_sync(0xffffffffu, j < nch && __ldcg(cmax + j) == M);
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

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------
template <int MODE, bool BF16>
__global__ void __launch_bounds__(kThreads, 2) accept_kernel(const AcceptArgs a) {
    const int b = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int n_live = a.n_nodes ? a.n_nodes[b] : a.N;
    const bool seq_ok = n_live >= 1 && n_live <= a.N;
    if (!seq_ok) n_live = 0;
    const size_t row_bytes = (size_t)a.stride * (BF16 ? 2 : 4);

    // ---------------- phase 1: chunk maxima ----------------
    const int u0 = blockIdx.x * a.slice, u1 = min(u0 + a.slice, a.units_per_seq);
    int bad = 0;
    for (int u = u0 + warp; u < u1; u += kWarps) {
        const int r = u / a.nch, j = u - r * a.nch;
        const bool isq = r >= a.N;
        const int node = isq ? r - a.N : r;
        if (node >= n_live) continue;
        const char *row = reinterpret_cast<const char *>(isq ? a.draft : a.target) + ((size_t)b * a.N + node) * row_bytes;
        const int c0 = j * A11S_CHUNK;
        const float m = chunk_max<BF16>(row, c0, min(A11S_CHUNK, a.V - c0), lane);
        bad |= !(m < INFINITY);  // the NaN-propagating max is NaN or +Inf
        if (MODE != A11S_ACCEPT_GREEDY && m > -INFINITY && !(fabsf(__fmul_rn(m, a.k)) < 16777216.0f)) bad = 1;
        if (lane == 0) a.recs[((size_t)b * a.rows_per_seq + r) * a.nch + j] = m;
    }
    if (warp_or(bad) && lane == 0) report(a.status, A11S_ENONFINITE, b);
    __threadfence();
    __syncthreads();
    __shared__ int s_last;
    if (threadIdx.x == 0) {
        const int done = u1 - u0;
        const int prev = atomicAdd(&a.counters[b], done);
        s_last = (prev + done == a.units_per_seq);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    // ---------------- phase 2: walk ----------------
    __shared__ WalkSmem sm;
    const int N = a.N, V = a.V, nch = a.nch;
    const int32_t *tok = a.tokens + (size_t)b * N;
    const int32_t *par = a.parents + (size_t)b * N;
    int32_t *an = a.acc_nodes + (size_t)b * N;
    int32_t *at = a.acc_tokens + (size_t)b * N;
    const float *cmax_b = a.recs + (size_t)b * a.rows_per_seq * nch;
    const char *tgt_b = reinterpret_cast<const char *>(a.target) + (size_t)b * N * row_bytes;
    const char *drf_b = MODE == A11S_ACCEPT_STOCH_DRAFT
                            ? reinterpret_cast<const char *>(a.draft) + (size_t)b * N * row_bytes
                            : nullptr;

    if (warp == 0) {
        int okl = seq_ok ? 1 : 0;
        for (int i = 1 + lane; i < n_live; i += 32)
            if (par[i] < 0 || par[i] >= i || tok[i] < 0 || tok[i] >= V) okl = 0;
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
        if (threadIdx.x == 0) { a.accept_len[b] = 0; a.bonus[b] = -1; }
        return;
    }

    // node probabilities p(tokens[i]) in the parent's row (sampling modes, optional):
    // one statistics pass per row that has children
    if (MODE != A11S_ACCEPT_GREEDY && a.node_probs) {
        for (int r = 0; r < n_live; ++r) {
            bool has_child = false;
            for (int c = r + 1; c < n_live && !has_child; ++c) has_child = par[c] == r;
            if (!has_child) continue;
            const char *prow = tgt_b + (size_t)r * row_bytes;
            row_sums<BF16>(prow, cmax_b + (size_t)r * nch, nch, V, a.k, sm.fr, sm.sum, warp, lane);
            __syncthreads();
            if (warp == 0) {
                const RowStat rs = combine_sums(sm.fr, sm.sum, nch, lane);
                for (int c = r + 1 + lane; c < n_live; c += 32) {
                    if (par[c] != r) continue;
                    const int x = tok[c], j = x / A11S_CHUNK;
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
        if (warp == 0) {
            for (;;) {
                const int am = row_argmax<BF16>(tgt_b + (size_t)node * row_bytes, cmax_b + (size_t)node * nch, nch,
                                                V, sm.cp, lane);
                int next = INT_MAX;
                for (int c0 = node + 1; c0 < n_live && next == INT_MAX; c0 += 32) {
                    const int c = c0 + lane;
                    const unsigned m = __ballot_sync(0xffffffffu, c < n_live && par[c] == node && tok[c] == am);
                    if (m) next = c0 + __ffs(m) - 1;
                }
                if (next == INT_MAX) { bonus = am; break; }
                if (lane == 0) { an[alen] = next; at[alen] = tok[next]; }
                ++alen;
                node = next;
            }
        }
    } else {
        // Sampling walk: warp 0 decides; every warp computes row statistics and residual passes.
        if (threadIdx.x == 0) { sm.node = 0; sm.alen = 0; }
        __syncthreads();
        for (;;) {  // one iteration per visited node
            const int nd = sm.node;
            row_sums<BF16>(tgt_b + (size_t)nd * row_bytes, cmax_b + (size_t)nd * nch, nch, V, a.k, sm.fr, sm.sum,
                           warp, lane);
            if (MODE == A11S_ACCEPT_STOCH_DRAFT)
                row_sums<BF16>(drf_b + (size_t)nd * row_bytes, cmax_b + (size_t)(N + nd) * nch, nch, V, a.k, sm.qfr,
                               sm.qsum, warp, lane);
            __syncthreads();
            if (warp == 0) {
                sm.ps = combine_sums(sm.fr, sm.sum, nch, lane);
                if (MODE == A11S_ACCEPT_STOCH_DRAFT) sm.qs = combine_sums(sm.qfr, sm.qsum, nch, lane);
                for (int j = lane; j < nch; j += 32) sm.sub[j] = sm.sum[j];
                __syncwarp();
                if (lane == 0) {
                    sm.S_eff = sm.ps.S;
                    sm.nexcl = 0;
                    sm.L = 0;
                    sm.cpos = nd;
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
            for (;;) {  // children of this node, in index order
                if (warp == 0) {
                    int next = INT_MAX;
                    const int from = sm.cpos + 1;
                    for (int c0 = from; c0 < n_live && next == INT_MAX; c0 += 32) {
                        const int c = c0 + lane;
                        const unsigned m = __ballot_sync(0xffffffffu, c < n_live && par[c] == sm.node);
                        if (m) next = c0 + __ffs(m) - 1;
                    }
                    __syncwarp();
                    if (lane == 0) {
                        if (next == INT_MAX) {
                            sm.action = 0;  // no child left: draw the bonus here
                        } else {
                            sm.cpos = next;
                            sm.child = next;
                            const int x = tok[next], j = x / A11S_CHUNK;
                            const float u = a.uniforms[(size_t)b * N + next];
                            const float lx = load_logit(tgt_b + (size_t)sm.node * row_bytes, x, BF16);
                            if (MODE == A11S_ACCEPT_STOCH_ONEHOT) {
                                bool ex = false;
                                for (int e = 0; e < sm.nexcl; ++e) ex |= sm.excl[e] == x;
                                float lt = 0.0f;
                                if (!ex && sm.S_eff) {
                                    RowStat re = sm.ps;
                                    re.S = sm.S_eff;
                                    re.invS = __ddiv_rn(1.0, __ull2double_rn(sm.S_eff));
                                    lt = prob_of(lx, a.k, sm.fr[j], chunk_scale(re, sm.fr[j]));
                                }
                                if (accept_linear(u, lt, 1.0f)) {
                                    sm.action = 1;
                                } else {
                                    sm.action = 2;
                                    if (!ex) {
                                        sm.excl[sm.nexcl++] = x;
                                        if (sm.fr[j] != A11S_FRAME_NONE) sm.sub[j] -= det_weight(lx, a.k, (float)sm.fr[j]);
                                        uint64_t S = 0;
                                        for (int jj = 0; jj < nch; ++jj) {
                                            if (sm.fr[jj] == A11S_FRAME_NONE) continue;
                                            const int d = sm.ps.C - sm.fr[jj];
                                            S += d > 63 ? 0ull : (sm.sub[jj] >> d);
                                        }
                                        sm.S_eff = S;
                                    }
                                }
                            } else {
                                const float p0 = prob_of(lx, a.k, sm.fr[j], chunk_scale(sm.ps, sm.fr[j]));
                                const float lq = load_logit(drf_b + (size_t)sm.node * row_bytes, x, BF16);
                                const float qx = prob_of(lq, a.k, sm.qfr[j], chunk_scale(sm.qs, sm.qfr[j]));
                                const float lt = level_prob(p0, qx, sm.L, sm.invT);
                                sm.action = accept_linear(u, lt, qx) ? 1 : (sm.L < A11S_MAX_WALK_LEVELS ? 4 : 2);
                            }
                        }
                    }
                    __syncwarp();
                }
                __syncthreads();
                const int action = sm.action;
                __syncthreads();  // every thread has read sm.action before it changes
                if (action == 1) {  // accepted: move to the child
                    if (threadIdx.x == 0) {
                        an[sm.alen] = sm.child;
                        at[sm.alen] = tok[sm.child];
                        sm.alen += 1;
                        sm.node = sm.child;
                    }
                    moved = true;
                    __syncthreads();
                    break;
                }
                if (action == 0) break;
                if (action == 4) {
                    // DRAFT residual pass: chunk totals of level L+1 (every warp).
                    const char *prow = tgt_b + (size_t)sm.node * row_bytes;
                    const char *qrow = drf_b + (size_t)sm.node * row_bytes;
                    const int L = sm.L;
                    constexpr int EPV = Vec<BF16>::EPV, NV = Vec<BF16>::NV, G = 4;
                    for (int j = warp; j < nch; j += kWarps) {
                        const int c0 = j * A11S_CHUNK, clen = min(A11S_CHUNK, V - c0);
                        const int32_t fp = sm.fr[j], fq = sm.qfr[j];
                        const double scp = chunk_scale(sm.ps, fp), scq = chunk_scale(sm.qs, fq);
                        uint64_t s = 0;
                        for (int i0 = 0; i0 < NV; i0 += G) {  // 4 vectors of p and q in flight
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
                                    const float pv = prob_of(Vec<BF16>::at(vp[g], e), a.k, fp, scp);
                                    const float qv = prob_of(Vec<BF16>::at(vq[g], e), a.k, fq, scq);
                                    s += level_weight(level_prob(pv, qv, L, sm.invT), qv);
                                }
                        }
                        s = warp_sum_u64(s);
                        if (lane == 0) sm.tmp[j] = s;
                    }
                    __syncthreads();
                    if (threadIdx.x == 0) {
                        uint64_t tot = 0;
                        for (int j = 0; j < nch; ++j) tot += sm.tmp[j];
                        if (tot) {
                            sm.L += 1;
                            sm.T[sm.L] = tot;
                            sm.invT[sm.L] = __ddiv_rn(1.0, __ull2double_rn(tot));
                            for (int j = 0; j < nch; ++j) sm.lvl[j] = sm.tmp[j];
                        }
                    }
                    __syncthreads();
                }
                // action 2 / 4: rejected, try the next child
            }
            if (!moved) break;
        }
        // bonus draw at sm.node (warp 0)
        if (!failed && warp == 0) {
            const int nd = sm.node;
            const char *prow = tgt_b + (size_t)nd * row_bytes;
            const float u0 = a.uniforms[(size_t)b * N];
            int j = 0;
            uint64_t t2 = 0;
            bool okp = false;
            if (MODE == A11S_ACCEPT_STOCH_DRAFT && sm.L > 0) {
                if (lane == 0) okp = pick_chunk(u0, sm.lvl, sm.lvl, nch, j, t2);
                okp = __shfl_sync(0xffffffffu, okp, 0);
                j = __shfl_sync(0xffffffffu, j, 0);
                t2 = __shfl_sync(0xffffffffu, t2, 0);
                if (okp) {
                    const char *qrow = drf_b + (size_t)nd * row_bytes;
                    const int32_t fp = sm.fr[j], fq = sm.qfr[j];
                    const double scp = chunk_scale(sm.ps, fp), scq = chunk_scale(sm.qs, fq);
                    const int L = sm.L;
                    const float k = a.k;
                    const int c0 = j * A11S_CHUNK, clen = min(A11S_CHUNK, V - c0);
                    stage_chunk<BF16>(prow, c0, clen, sm.cp, lane);
                    stage_chunk<BF16>(qrow, c0, clen, sm.cq, lane);
                    bonus = c0 + scan_chunk(clen, t2, lane, [&](int e) {
                                const float pv = prob_of(sm.cp[e], k, fp, scp);
                                const float qv = prob_of(sm.cq[e], k, fq, scq);
                                return level_weight(level_prob(pv, qv, L - 1, sm.invT), qv);
                            });
                }
            } else {
                const bool use_excl = MODE == A11S_ACCEPT_STOCH_ONEHOT && sm.S_eff != 0;
                // A_j in the row frame, local totals Lc_j (sm.tmp / sm.lvl as scratch)
                for (int jj = lane; jj < nch; jj += 32) {
                    const uint64_t loc = use_excl ? sm.sub[jj] : sm.sum[jj];
                    sm.tmp[jj] = loc;
                    const int32_t f = sm.fr[jj];
                    const int d = sm.ps.C - f;
                    sm.lvl[jj] = (f == A11S_FRAME_NONE || d > 63) ? 0ull : (loc >> d);
                }
                __syncwarp();
                if (lane == 0) okp = pick_chunk(u0, sm.lvl, sm.tmp, nch, j, t2);
                okp = __shfl_sync(0xffffffffu, okp, 0);
                j = __shfl_sync(0xffffffffu, j, 0);
                t2 = __shfl_sync(0xffffffffu, t2, 0);
                if (okp) {
                    const float cff = (float)sm.fr[j];
                    const float k = a.k;
                    const int nex = use_excl ? sm.nexcl : 0;
                    const int c0 = j * A11S_CHUNK, clen = min(A11S_CHUNK, V - c0);
                    stage_chunk<BF16>(prow, c0, clen, sm.cp, lane);
                    bonus = c0 + scan_chunk(clen, t2, lane, [&](int e) -> uint64_t {
                                for (int x = 0; x < nex; ++x)
                                    if (sm.excl[x] == c0 + e) return 0ull;
                                return det_weight(sm.cp[e], k, cff);
                            });
                }
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
}

cudaError_t launch_accept(int mode, bool bf16, const AcceptArgs &a, int grid_x, cudaStream_t s) {
    dim3 grid(grid_x, a.B), block(kThreads);
#define A11S_LAUNCH(M, BF)                                                   \
    if (mode == M && bf16 == BF) {                                           \
        accept_kernel<M, BF><<<grid, block, 0, s>>>(a);                      \
        return cudaGetLastError();                                           \
    }
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
