// accept.cu - K3: vocab-wide softmax/argmax + acceptance + path select + bonus draw.
//
// One kernel per call. Phase 1 (every block): warps stream 2048-token chunks
// of the logits rows with 16-byte non-allocating loads, reduce each chunk with
// warp shuffles and store a 16-byte chunk record (greedy: max, argmax; sampling:
// max, frame, fixed-point exp sum). Phase 2 (the block that completes a
// sequence, found with a fenced atomic counter, no waiting): walk the tree from
// the root, draw the bonus token, write outputs and counters.
//
// Semantics: include/a11spec.h (a11s_accept). Reference behaviour followed:
// src/engine/speculative_verifier.cpp:84-135 (acceptance rule, first rejection
// stops the chain), engine/sampler.py:16 (logits / T).
#include "common.cuh"
#include "kernels.h"

namespace a11s {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxNch = A11S_MAX_VOCAB / A11S_CHUNK;  // 128

// One 2048-token chunk of a row held in registers: 64 values per lane.
// fp32: 16 x (4 floats), bf16: 8 x (8 bf16); vector i of lane covers tokens
// [(i*32 + lane) * EPV, +EPV) of the chunk.
template <bool BF16>
struct Chunk {
    static constexpr int EPV = BF16 ? 8 : 4;
    static constexpr int NV = 64 / EPV;
    uint4 d[NV];

    __device__ __forceinline__ void load(const void *row, int c0, int clen, int lane) {
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int e0 = (i * 32 + lane) * EPV;
            if (e0 < clen) {
                d[i] = ldg_stream(reinterpret_cast<const char *>(row) +
                                  (size_t)(c0 + e0) * (BF16 ? 2 : 4));
            } else {
                const uint32_t ninf = BF16 ? 0xFF80FF80u : 0xFF800000u;
                d[i] = make_uint4(ninf, ninf, ninf, ninf);
            }
        }
    }
    __device__ __forceinline__ float at(int i, int e) const {
        const uint32_t w = (&d[i].x)[BF16 ? (e >> 1) : e];
        if (BF16) return (e & 1) ? bf16hi(w) : bf16lo(w);
        return __uint_as_float(w);
    }
};

__device__ __forceinline__ void argmax_merge(float &bv, int &bi, float ov, int oi) {
    if (oi != INT_MAX && (bi == INT_MAX || ov > bv || (ov == bv && oi < bi))) {
        bv = ov;
        bi = oi;
    }
}

__device__ __forceinline__ void warp_argmax(float &bv, int &bi) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_merge(bv, bi, ov, oi);
    }
}

// ---------------------------------------------------------------------------
// Phase 1 helpers: one chunk -> one record.
// ---------------------------------------------------------------------------
template <bool BF16>
__device__ __forceinline__ ChunkRec chunk_greedy(const void *row, int j, int V, int lane, int &bad) {
    const int c0 = j * A11S_CHUNK, clen = min(A11S_CHUNK, V - c0);
    Chunk<BF16> c;
    c.load(row, c0, clen, lane);
    float bv = -INFINITY;
    int bi = INT_MAX;
#pragma unroll
    for (int i = 0; i < Chunk<BF16>::NV; ++i) {
        const int e0 = (i * 32 + lane) * Chunk<BF16>::EPV;
        if (e0 < clen) {
#pragma unroll
            for (int e = 0; e < Chunk<BF16>::EPV; ++e) {
                const float v = c.at(i, e);
                bad |= !(v < INFINITY);
                if (v > bv || bi == INT_MAX) { bv = v; bi = c0 + e0 + e; }
            }
        }
    }
    warp_argmax(bv, bi);
    ChunkRec r;
    r.cmax = bv;
    r.aux = bi;
    r.sum = 0;
    return r;
}

template <bool BF16>
__device__ __forceinline__ ChunkRec chunk_stoch(const void *row, int j, int V, float k, int lane,
                                                int &bad) {
    const int c0 = j * A11S_CHUNK, clen = min(A11S_CHUNK, V - c0);
    Chunk<BF16> c;
    c.load(row, c0, clen, lane);
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < Chunk<BF16>::NV; ++i)
#pragma unroll
        for (int e = 0; e < Chunk<BF16>::EPV; ++e) {
            const float v = c.at(i, e);
            bad |= !(v < INFINITY);
            m = fmaxf(m, v);
        }
    m = warp_fmax(m);
    ChunkRec r;
    r.cmax = m;
    r.aux = A11S_FRAME_NONE;
    r.sum = 0;
    if (m == -INFINITY) return r;
    const float mk = __fmul_rn(m, k);
    if (!(fabsf(mk) < 16777216.0f)) { bad = 1; return r; }
    const int cf = (int)ceilf(mk);
    const float cff = (float)cf;
    uint64_t s = 0;
#pragma unroll
    for (int i = 0; i < Chunk<BF16>::NV; ++i)
#pragma unroll
        for (int e = 0; e < Chunk<BF16>::EPV; ++e) s += det_weight(c.at(i, e), k, cff);
    r.aux = cf;
    r.sum = warp_sum_u64(s);
    return r;
}

__device__ __forceinline__ float load_logit(const void *row, int v, bool bf16) {
    if (bf16) {
        const uint16_t h = __ldg(reinterpret_cast<const unsigned short *>(row) + v);
        return __uint_as_float((uint32_t)h << 16);
    }
    return __ldg(reinterpret_cast<const float *>(row) + v);
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
    int32_t fr[kMaxNch];    // p frames of the current node's row
    uint64_t sub[kMaxNch];  // p chunk sums, rejected tokens removed (ONEHOT)
    int32_t qfr[kMaxNch];   // q frames (DRAFT)
    uint64_t qsum[kMaxNch];
    uint64_t lvl[kMaxNch];  // chunk totals of the newest residual level (DRAFT)
    uint64_t tmp[kMaxNch];
    uint64_t T[A11S_MAX_WALK_LEVELS + 1];
    double invT[A11S_MAX_WALK_LEVELS + 1];
    int32_t excl[A11S_MAX_NODES];
    RowStat ps, qs;
    uint64_t S_eff;
    int32_t nexcl, L, node, alen, cpos, action, child, ok;
};

// Warp-cooperative combine of one row's chunk records (lanes stride chunks).
// Writes frames/sums to smem arrays when given.
__device__ RowStat combine_row(const ChunkRec *rec, int nch, int32_t *fr_out, uint64_t *sum_out,
                               int lane) {
    int32_t C = A11S_FRAME_NONE;
    for (int j = lane; j < nch; j += 32) {
        const int32_t f = __ldcg(&rec[j].aux);
        if (fr_out) fr_out[j] = f;
        if (sum_out) sum_out[j] = __ldcg(&rec[j].sum);
        if (f != A11S_FRAME_NONE) C = max(C, f);
    }
    C = warp_max(C);
    uint64_t S = 0;
    if (C != A11S_FRAME_NONE)
        for (int j = lane; j < nch; j += 32) {
            const int32_t f = __ldcg(&rec[j].aux);
            if (f == A11S_FRAME_NONE) continue;
            const int d = C - f;
            S += d > 63 ? 0ull : (__ldcg(&rec[j].sum) >> d);
        }
    S = warp_sum_u64(S);
    RowStat rs;
    rs.C = C;
    rs.S = S;
    rs.invS = S ? __ddiv_rn(1.0, __ull2double_rn(S)) : 0.0;
    return rs;
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

// Inverse CDF inside one chunk, warp 0: lane l owns tokens [c0 + 64 l, +64).
// wfn(v) gives the weight of token v. Returns the first token whose running
// weight exceeds t2 (or the last positive-weight token).
template <typename WF>
__device__ int scan_chunk(int c0, int clen, uint64_t t2, int lane, WF wfn) {
    const int lo = lane * 64, hi = min(lo + 64, clen);
    uint64_t mine = 0;
    for (int e = lo; e < hi; ++e) mine += wfn(c0 + e);
    // exclusive warp scan
    uint64_t incl = mine;
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
        for (int e = lo; e < hi; ++e) {
            acc += wfn(c0 + e);
            if (acc > t2) { found = c0 + e; break; }
        }
    }
    if (who) return __shfl_sync(0xffffffffu, found, __ffs(who) - 1);
    // t2 beyond the chunk total (cannot happen with consistent totals): last positive weight
    int last = -1;
    for (int e = lo; e < hi; ++e)
        if (wfn(c0 + e)) last = c0 + e;
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

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------
template <int MODE, bool BF16>
__global__ void __launch_bounds__(kThreads) accept_kernel(const AcceptArgs a) {
    const int b = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int n_live = a.n_nodes ? a.n_nodes[b] : a.N;
    const bool seq_ok = n_live >= 1 && n_live <= a.N;
    if (!seq_ok) n_live = 0;

    // ---------------- phase 1: chunk records ----------------
    const int u0 = blockIdx.x * a.slice, u1 = min(u0 + a.slice, a.units_per_seq);
    int bad = 0;
    for (int u = u0 + warp; u < u1; u += kWarps) {
        const int r = u / a.nch, j = u - r * a.nch;
        const bool isq = r >= a.N;
        const int node = isq ? r - a.N : r;
        if (node >= n_live) continue;
        const char *base = reinterpret_cast<const char *>(isq ? a.draft : a.target);
        const void *row = base + ((size_t)b * a.N + node) * (size_t)a.stride * (BF16 ? 2 : 4);
        ChunkRec rec = MODE == A11S_ACCEPT_GREEDY ? chunk_greedy<BF16>(row, j, a.V, lane, bad)
                                                  : chunk_stoch<BF16>(row, j, a.V, a.k, lane, bad);
        if (lane == 0) a.recs[((size_t)b * a.rows_per_seq + r) * a.nch + j] = rec;
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
    const ChunkRec *recs_b = a.recs + (size_t)b * a.rows_per_seq * nch;
    const bool bf16 = BF16;
    const size_t row_bytes = (size_t)a.stride * (BF16 ? 2 : 4);
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

    // node probabilities p(tokens[i]) in the parent's row (sampling modes)
    if (MODE != A11S_ACCEPT_GREEDY && a.node_probs) {
        for (int i = 1 + warp; i < n_live; i += kWarps) {
            const int pr = par[i];
            const ChunkRec *rr = recs_b + (size_t)pr * nch;
            const RowStat rs = combine_row(rr, nch, nullptr, nullptr, lane);
            if (lane == 0) {
                const int x = tok[i], j = x / A11S_CHUNK;
                const int32_t f = __ldcg(&rr[j].aux);
                const float l = load_logit(tgt_b + (size_t)pr * row_bytes, x, bf16);
                a.node_probs[(size_t)b * N + i] = prob_of(l, a.k, f, chunk_scale(rs, f));
            }
        }
    }

    int alen = 0, node = 0, bonus = -1;
    bool failed = false;
    if (MODE == A11S_ACCEPT_GREEDY) {
        if (warp == 0) {
            for (;;) {
                const ChunkRec *rr = recs_b + (size_t)node * nch;
                float bv = -INFINITY;
                int bi = INT_MAX;
                for (int j = lane; j < nch; j += 32) argmax_merge(bv, bi, __ldcg(&rr[j].cmax), __ldcg(&rr[j].aux));
                warp_argmax(bv, bi);
                int next = INT_MAX;
                for (int c0 = node + 1; c0 < n_live && next == INT_MAX; c0 += 32) {
                    const int c = c0 + lane;
                    const bool hit = c < n_live && par[c] == node && tok[c] == bi;
                    const unsigned m = __ballot_sync(0xffffffffu, hit);
                    if (m) next = c0 + __ffs(m) - 1;
                }
                if (next == INT_MAX) { bonus = bi; break; }
                if (lane == 0) { an[alen] = next; at[alen] = tok[next]; }
                ++alen;
                node = next;
            }
        }
    } else {
        // Sampling walk: warp 0 decides, every warp helps with residual passes.
        if (threadIdx.x == 0) { sm.node = 0; sm.alen = 0; }
        __syncthreads();
        for (;;) {  // one iteration per visited node
            if (warp == 0) {
                node = sm.node;
                sm.ps = combine_row(recs_b + (size_t)node * nch, nch, sm.fr, sm.sub, lane);
                if (MODE == A11S_ACCEPT_STOCH_DRAFT)
                    sm.qs = combine_row(recs_b + (size_t)(N + node) * nch, nch, sm.qfr, sm.qsum, lane);
                if (lane == 0) {
                    sm.S_eff = sm.ps.S;
                    sm.nexcl = 0;
                    sm.L = 0;
                    sm.cpos = node;
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
                            const float lx = load_logit(tgt_b + (size_t)sm.node * row_bytes, x, bf16);
                            const uint64_t wx = det_weight(lx, a.k, (float)sm.fr[j]);
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
                                        if (sm.fr[j] != A11S_FRAME_NONE) sm.sub[j] -= wx;
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
                                const float lq = load_logit(drf_b + (size_t)sm.node * row_bytes, x, bf16);
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
                    constexpr int EPV = Chunk<BF16>::EPV, NV = Chunk<BF16>::NV, G = 4;
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
                                    const uint32_t wp = (&vp[g].x)[BF16 ? (e >> 1) : e];
                                    const uint32_t wq = (&vq[g].x)[BF16 ? (e >> 1) : e];
                                    const float lp = BF16 ? ((e & 1) ? bf16hi(wp) : bf16lo(wp)) : __uint_as_float(wp);
                                    const float lq = BF16 ? ((e & 1) ? bf16hi(wq) : bf16lo(wq)) : __uint_as_float(wq);
                                    const float pv = prob_of(lp, a.k, fp, scp);
                                    const float qv = prob_of(lq, a.k, fq, scq);
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
                    bonus = scan_chunk(j * A11S_CHUNK, min(A11S_CHUNK, V - j * A11S_CHUNK), t2, lane,
                                       [&](int v) {
                                           const float pv = prob_of(load_logit(prow, v, bf16), k, fp, scp);
                                           const float qv = prob_of(load_logit(qrow, v, bf16), k, fq, scq);
                                           return level_weight(level_prob(pv, qv, L - 1, sm.invT), qv);
                                       });
                }
            } else {
                const bool use_excl = MODE == A11S_ACCEPT_STOCH_ONEHOT && sm.S_eff != 0;
                // A_j in the row frame, local totals Lc_j (sm.tmp / sm.lvl as scratch)
                for (int jj = lane; jj < nch; jj += 32) {
                    const uint64_t loc = use_excl ? sm.sub[jj] : __ldcg(&recs_b[(size_t)nd * nch + jj].sum);
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
                    bonus = scan_chunk(j * A11S_CHUNK, min(A11S_CHUNK, V - j * A11S_CHUNK), t2, lane,
                                       [&](int v) -> uint64_t {
                                           for (int e = 0; e < nex; ++e)
                                               if (sm.excl[e] == v) return 0ull;
                                           return det_weight(load_logit(prow, v, bf16), k, cff);
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
