/*
 * a11oracle.c - CPU oracle (plain C) for the speculative-decoding hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker of the CUDA kernels. Built with
 * -ffp-contract=off so every rounding is the one written here; every fused
 * multiply-add is an explicit fmaf().
 *
 * Reference files followed (paths inside the reference project):
 *   acceptance rule        src/engine/speculative_verifier.cpp:102-132
 *   temperature            engine/sampler.py:10,16 (logits / max(T, 1e-5))
 *   attention math         engine/pipeline.py:386-402
 *   page layout            engine/kv_cache.py:20-21, include/cuda/paged_kv_cache.hpp:13
 *   block-table growth     src/cuda/paged_kv_cache.cu:120-136
 *   n-gram key             engine/speculative.py:20-21 (last two context tokens)
 */
#include "a11oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define ST_OK 0
#define ST_EINVAL 1
#define ST_EBOUNDS 2
#define ST_ENONFINITE 5

#define MODE_GREEDY 0
#define MODE_ONEHOT 1
#define MODE_DRAFT 2

#define FRAME_NONE INT32_MIN
#define MAX_WALK_LEVELS 64 /* residual levels kept per node (STOCH_DRAFT) */

int or_abi_version(void) { return 1; }

/* ---------------------------------------------------------------------------
 * Deterministic fixed-point softmax ("chunked fixed-point softmax").
 *
 * Probabilities p = softmax(l / T) are defined through integer weights so that
 * every reduction is an exact integer sum, independent of summation order:
 *   k      = (float)(log2(e) / max(T, 1e-5))                (host, double -> float)
 *   chunk j covers tokens [2048 j, 2048 j + 2048)
 *   frame  c_j = (int)ceilf(m_j * k), m_j the chunk max logit
 *   weight W(l) = floor(2^(l*k - c_j) * 2^40) computed as below (0 for l=-inf)
 *   S_j    = sum of W over the chunk (uint64, <= 2^53)
 *   C      = max_j c_j,  S = sum_j (S_j >> (C - c_j))   (shift capped at 63)
 *   p(x)   = (float)( W(l_x) * (2^(c_j - C) * (1 / (double)S)) )
 * 2^f on f in [-0.5, 0.5] is a degree-5 polynomial fitted for this file
 * (iteratively reweighted least squares towards minimax relative error,
 * max relative error 2.2e-7), evaluated by Horner's rule with fmaf.
 * ------------------------------------------------------------------------- */
static const float kP0 = 0x1.000002p+0f, kP1 = 0x1.62e428p-1f, kP2 = 0x1.ebf918p-3f,
                   kP3 = 0x1.c6b6dcp-5f, kP4 = 0x1.3d0c5cp-7f, kP5 = 0x1.5c0c48p-10f;

float or_exp2_poly(float f) {
    float p = kP5;
    p = fmaf(p, f, kP4);
    p = fmaf(p, f, kP3);
    p = fmaf(p, f, kP2);
    p = fmaf(p, f, kP1);
    p = fmaf(p, f, kP0);
    return p;
}

float or_temperature_k(float temperature) {
    double t = temperature < 1e-5f ? 1e-5 : (double)temperature;
    return (float)(1.4426950408889634 / t);
}

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

uint64_t or_weight(float l, float k, int32_t c) {
    if (isinf(l) && l < 0) return 0;
    float t = fmaf(l, k, -(float)c);
    t = fmaxf(t, -160.0f);
    float r = t + 12582912.0f;     /* 1.5 * 2^23: rounds t to the nearest integer */
    float nf = r - 12582912.0f;
    float f = t - nf;              /* exact, |f| <= 0.5 */
    int32_t n = (int32_t)nf;
    float p = or_exp2_poly(f);
    uint32_t bits = f2u(p);
    int32_t e = (int32_t)(bits >> 23) - 127;
    uint64_t m = (uint64_t)((bits & 0x7FFFFFu) | 0x800000u);
    int32_t sh = 7 - e - n;        /* W = (m << 24) >> sh  ==  m * 2^(e - 23 + n + 40) */
    if (sh > 63) return 0;
    if (sh < 0) sh = 0;            /* unreachable for t < 1.5 */
    return (m << 24) >> sh;
}

static inline int nonfinite_bad(float v) { return !(v < INFINITY); } /* NaN or +Inf */

void or_chunk_records(const float *row, int32_t vocab, float k, float *cmax, int32_t *frame,
                      uint64_t *sum) {
    int32_t nch = (vocab + OR_CHUNK - 1) / OR_CHUNK;
    for (int32_t j = 0; j < nch; ++j) {
        int32_t lo = j * OR_CHUNK, hi = lo + OR_CHUNK < vocab ? lo + OR_CHUNK : vocab;
        float m = -INFINITY;
        for (int32_t v = lo; v < hi; ++v) m = fmaxf(m, row[v]);
        cmax[j] = m;
        if (isinf(m) && m < 0) { frame[j] = FRAME_NONE; sum[j] = 0; continue; }
        int32_t c = (int32_t)ceilf(m * k);
        uint64_t s = 0;
        for (int32_t v = lo; v < hi; ++v) s += or_weight(row[v], k, c);
        frame[j] = c;
        sum[j] = s;
    }
}

typedef struct {
    int32_t nch;
    float k;
    const float *row;
    float *cmax;
    int32_t *frame;
    uint64_t *sum;     /* chunk sums (possibly with exclusions removed) */
    int32_t C;
    uint64_t S;
} rowstat_t;

static double pow2neg(int32_t d) { /* 2^-d for 0 <= d <= 1000 */
    uint64_t bits = (uint64_t)(1023 - d) << 52;
    double r; memcpy(&r, &bits, 8); return r;
}

static void row_combine(rowstat_t *rs) {
    int32_t C = FRAME_NONE;
    for (int32_t j = 0; j < rs->nch; ++j)
        if (rs->frame[j] != FRAME_NONE && rs->frame[j] > C) C = rs->frame[j];
    uint64_t S = 0;
    if (C != FRAME_NONE)
        for (int32_t j = 0; j < rs->nch; ++j) {
            if (rs->frame[j] == FRAME_NONE) continue;
            int32_t d = C - rs->frame[j];
            S += d > 63 ? 0 : (rs->sum[j] >> d);
        }
    rs->C = C;
    rs->S = S;
}

/* Chunk weight of chunk j in the row frame. */
static inline uint64_t chunk_global(const rowstat_t *rs, int32_t j) {
    if (rs->frame[j] == FRAME_NONE) return 0;
    int32_t d = rs->C - rs->frame[j];
    return d > 63 ? 0 : (rs->sum[j] >> d);
}

static inline uint64_t elem_weight(const rowstat_t *rs, int32_t v) {
    int32_t j = v / OR_CHUNK;
    if (rs->frame[j] == FRAME_NONE) return 0;
    return or_weight(rs->row[v], rs->k, rs->frame[j]);
}

/* p(v) = (float)(W_v * (2^(c_j - C) * (1 / (double)S_eff))): one double
 * reciprocal per row, an exact power-of-two scaling, one rounded product. */
static float elem_prob(const rowstat_t *rs, int32_t v, uint64_t S_eff) {
    if (S_eff == 0) return 0.0f;
    int32_t j = v / OR_CHUNK;
    if (rs->frame[j] == FRAME_NONE) return 0.0f;
    uint64_t w = or_weight(rs->row[v], rs->k, rs->frame[j]);
    int32_t d = rs->C - rs->frame[j];
    if (d > 1000) return 0.0f;
    double sc = pow2neg(d) * (1.0 / (double)S_eff);
    return (float)((double)w * sc);
}

/* Reference linear-space acceptance, src/engine/speculative_verifier.cpp:114-124. */
static int accept_linear(float u, float lt, float ld) {
    ld = fmaxf(1e-10f, fminf(ld, 1.0f));
    lt = fmaxf(0.0f, fminf(lt, 1.0f + 1e-6f));
    float a = lt / ld;
    if (a > 1.0f) a = 1.0f;
    return u < a;
}

/* Residual level probability for STOCH_DRAFT: p_L(v) from p_0(v), q(v). */
static float level_prob(float p0, float q, int32_t L, const uint64_t *T) {
    float p = p0;
    for (int32_t l = 1; l <= L; ++l) {
        float r = fmaxf(p - q, 0.0f);
        uint64_t R = (uint64_t)(r * 0x1p40f);
        p = (float)((double)R * (1.0 / (double)T[l]));
    }
    return p;
}

static inline uint64_t level_weight(float p_prev, float q) {
    float r = fmaxf(p_prev - q, 0.0f);
    return (uint64_t)(r * 0x1p40f);
}

/* Two-level inverse CDF: chunk totals A[j] in one frame, local weights w(v)
 * summing to Lc[j] inside chunk j. Returns the drawn token or -1. */
typedef uint64_t (*wfn_t)(void *ctx, int32_t v);

static int32_t sample_two_level(float u, const uint64_t *A, const uint64_t *Lc, int32_t nch,
                                int32_t vocab, wfn_t w, void *ctx) {
    uint64_t tot = 0;
    for (int32_t j = 0; j < nch; ++j) tot += A[j];
    if (tot == 0) return -1;
    uint64_t t = (uint64_t)((double)u * (double)tot);
    if (t >= tot) t = tot - 1;
    uint64_t acc = 0;
    int32_t j = 0;
    for (; j < nch; ++j) {
        if (acc + A[j] > t) break;
        acc += A[j];
    }
    if (j >= nch) return -1;
    uint64_t r = t - acc;
    uint64_t t2 = (uint64_t)(((unsigned __int128)r * Lc[j]) / A[j]);
    int32_t lo = j * OR_CHUNK, hi = lo + OR_CHUNK < vocab ? lo + OR_CHUNK : vocab;
    uint64_t a2 = 0;
    int32_t last = -1;
    for (int32_t v = lo; v < hi; ++v) {
        uint64_t wv = w(ctx, v);
        if (wv) last = v;
        a2 += wv;
        if (a2 > t2) return v;
    }
    return last;
}

typedef struct {
    const rowstat_t *rs;
    const int32_t *excl;
    int32_t nexcl;
} onehot_ctx_t;

static uint64_t onehot_w(void *vctx, int32_t v) {
    onehot_ctx_t *c = (onehot_ctx_t *)vctx;
    for (int32_t i = 0; i < c->nexcl; ++i)
        if (c->excl[i] == v) return 0;
    return elem_weight(c->rs, v);
}

typedef struct {
    const rowstat_t *p;
    const rowstat_t *q;
    int32_t L;
    const uint64_t *T;
} draft_ctx_t;

static uint64_t draft_w(void *vctx, int32_t v) {
    draft_ctx_t *c = (draft_ctx_t *)vctx;
    float p0 = elem_prob(c->p, v, c->p->S), q = elem_prob(c->q, v, c->q->S);
    float pprev = level_prob(p0, q, c->L - 1, c->T);
    return level_weight(pprev, q);
}

int or_accept(int32_t mode, const float *target, const float *draft, int64_t row_stride,
              float temperature, const float *uniforms, const int32_t *tokens,
              const int32_t *parents, const int32_t *n_nodes, int32_t batch, int32_t max_nodes,
              int32_t vocab, int32_t *accept_len, int32_t *accepted_nodes,
              int32_t *accepted_tokens, int32_t *bonus, float *node_probs, int64_t *stats) {
    if (mode < 0 || mode > 2 || batch < 0 || max_nodes < 1 || vocab < 1 || row_stride < vocab)
        return ST_EINVAL;
    if (mode == MODE_DRAFT && !draft) return ST_EINVAL;
    if (mode != MODE_GREEDY && !uniforms) return ST_EINVAL;
    const int32_t nch = (vocab + OR_CHUNK - 1) / OR_CHUNK;
    const float k = or_temperature_k(temperature);
    int status = ST_OK;
    float *cm = (float *)malloc(sizeof(float) * nch * 2);
    int32_t *fr = (int32_t *)malloc(sizeof(int32_t) * nch * 2);
    uint64_t *sm = (uint64_t *)malloc(sizeof(uint64_t) * nch * 4);
    uint64_t *Lc = (uint64_t *)malloc(sizeof(uint64_t) * nch);
    uint64_t *Ac = (uint64_t *)malloc(sizeof(uint64_t) * nch);
    int32_t *excl = (int32_t *)malloc(sizeof(int32_t) * (max_nodes + 1));

    for (int32_t b = 0; b < batch; ++b) {
        const int32_t n = n_nodes ? n_nodes[b] : max_nodes;
        const int32_t *tok = tokens + (int64_t)b * max_nodes;
        const int32_t *par = parents + (int64_t)b * max_nodes;
        int32_t *an = accepted_nodes + (int64_t)b * max_nodes;
        int32_t *at = accepted_tokens + (int64_t)b * max_nodes;
        for (int32_t i = 0; i < max_nodes; ++i) { an[i] = -1; at[i] = -1; }
        if (node_probs)
            for (int32_t i = 0; i < max_nodes; ++i) node_probs[(int64_t)b * max_nodes + i] = 0.0f;
        accept_len[b] = 0;
        bonus[b] = -1;
        if (n < 1 || n > max_nodes) { status = status ? status : ST_EBOUNDS; continue; }
        int bad = 0;
        for (int32_t i = 1; i < n; ++i)
            if (par[i] < 0 || par[i] >= i || tok[i] < 0 || tok[i] >= vocab) bad = 1;
        if (bad) { status = status ? status : ST_EBOUNDS; continue; }
        /* non-finite scan over every live row (the kernel reads every row) */
        for (int32_t i = 0; i < n && !bad; ++i) {
            const float *row = target + ((int64_t)b * max_nodes + i) * row_stride;
            for (int32_t v = 0; v < vocab; ++v) if (nonfinite_bad(row[v])) { bad = 1; break; }
            if (mode == MODE_DRAFT) {
                const float *qr = draft + ((int64_t)b * max_nodes + i) * row_stride;
                for (int32_t v = 0; v < vocab; ++v) if (nonfinite_bad(qr[v])) { bad = 1; break; }
            }
            for (int32_t w = 0; w < (mode == MODE_DRAFT ? 2 : 1) && mode != MODE_GREEDY && !bad; ++w) {
                const float *rr = w ? draft + ((int64_t)b * max_nodes + i) * row_stride : row;
                for (int32_t j = 0; j < nch; ++j) {
                    int32_t lo = j * OR_CHUNK, hi = lo + OR_CHUNK < vocab ? lo + OR_CHUNK : vocab;
                    float m = -INFINITY;
                    for (int32_t v = lo; v < hi; ++v) m = fmaxf(m, rr[v]);
                    if (m > -INFINITY && !(fabsf(m * k) < 16777216.0f)) bad = 1;
                }
            }
        }
        if (bad) { status = status ? status : ST_ENONFINITE; continue; }

        if (node_probs && mode != MODE_GREEDY) {
            for (int32_t i = 1; i < n; ++i) {
                const float *row = target + ((int64_t)b * max_nodes + par[i]) * row_stride;
                rowstat_t rs = {nch, k, row, cm, fr, sm, 0, 0};
                or_chunk_records(row, vocab, k, cm, fr, sm);
                row_combine(&rs);
                node_probs[(int64_t)b * max_nodes + i] = elem_prob(&rs, tok[i], rs.S);
            }
        }

        int32_t node = 0, alen = 0, seq_err = 0;
        for (;;) {
            const float *prow = target + ((int64_t)b * max_nodes + node) * row_stride;
            int32_t next = -1;
            if (mode == MODE_GREEDY) {
                float best = -INFINITY;
                int32_t arg = 0;
                for (int32_t v = 0; v < vocab; ++v)
                    if (prow[v] > best) { best = prow[v]; arg = v; }
                for (int32_t c = node + 1; c < n; ++c)
                    if (par[c] == node && tok[c] == arg) { next = c; break; }
                if (next < 0) { bonus[b] = arg; break; }
            } else {
                rowstat_t ps = {nch, k, prow, cm, fr, sm, 0, 0};
                or_chunk_records(prow, vocab, k, cm, fr, sm);
                row_combine(&ps);
                rowstat_t qs = {0};
                if (mode == MODE_DRAFT) {
                    const float *qrow = draft + ((int64_t)b * max_nodes + node) * row_stride;
                    qs = (rowstat_t){nch, k, qrow, cm + nch, fr + nch, sm + nch, 0, 0};
                    or_chunk_records(qrow, vocab, k, qs.cmax, qs.frame, qs.sum);
                    row_combine(&qs);
                }
                if (ps.S == 0 || (mode == MODE_DRAFT && qs.S == 0)) { /* all -inf row on the walk */
                    status = status ? status : ST_ENONFINITE;
                    seq_err = 1;
                    break;
                }
                /* one-hot residual state */
                int32_t nexcl = 0;
                uint64_t *sub = sm + 2 * nch; /* chunk sums with exclusions */
                memcpy(sub, ps.sum, sizeof(uint64_t) * nch);
                uint64_t S_eff = ps.S;
                /* draft residual state */
                uint64_t T[MAX_WALK_LEVELS + 1];
                int32_t L = 0;
                uint64_t *lvl_chunk = sm + 3 * nch; /* chunk totals of the newest level */
                for (int32_t c = node + 1; c < n && next < 0; ++c) {
                    if (par[c] != node) continue;
                    int32_t x = tok[c];
                    float u = uniforms[(int64_t)b * max_nodes + c];
                    float lt, ld;
                    if (mode == MODE_ONEHOT) {
                        int ex = 0;
                        for (int32_t e = 0; e < nexcl; ++e) ex |= excl[e] == x;
                        lt = ex ? 0.0f : elem_prob(&ps, x, S_eff);
                        ld = 1.0f;
                        if (accept_linear(u, lt, ld)) { next = c; break; }
                        if (!ex) {
                            excl[nexcl++] = x;
                            int32_t j = x / OR_CHUNK;
                            sub[j] -= elem_weight(&ps, x);
                            rowstat_t tmp = ps;
                            tmp.sum = sub;
                            row_combine(&tmp);
                            S_eff = tmp.S;
                        }
                    } else {
                        float p0 = elem_prob(&ps, x, ps.S), qx = elem_prob(&qs, x, qs.S);
                        lt = level_prob(p0, qx, L, T);
                        ld = qx;
                        if (accept_linear(u, lt, ld)) { next = c; break; }
                        if (L < MAX_WALK_LEVELS) {
                            /* candidate residual level L+1: T = sum_v R_{L+1}(v); an
                             * empty residual leaves the distribution unchanged */
                            uint64_t tot = 0;
                            for (int32_t j = 0; j < nch; ++j) {
                                int32_t lo = j * OR_CHUNK, hi = lo + OR_CHUNK < vocab ? lo + OR_CHUNK : vocab;
                                uint64_t cs = 0;
                                for (int32_t v = lo; v < hi; ++v) {
                                    float pv = elem_prob(&ps, v, ps.S), qv = elem_prob(&qs, v, qs.S);
                                    cs += level_weight(level_prob(pv, qv, L, T), qv);
                                }
                                Lc[j] = cs;
                                tot += cs;
                            }
                            if (tot > 0) {
                                ++L;
                                T[L] = tot;
                                memcpy(lvl_chunk, Lc, sizeof(uint64_t) * nch);
                            }
                        }
                    }
                }
                if (next < 0) {
                    float u0 = uniforms[(int64_t)b * max_nodes];
                    int32_t tokv = -1;
                    if (mode == MODE_DRAFT && L > 0) {
                        draft_ctx_t dc = {&ps, &qs, L, T};
                        tokv = sample_two_level(u0, lvl_chunk, lvl_chunk, nch, vocab, draft_w, &dc);
                    } else {
                        onehot_ctx_t oc = {&ps, excl, mode == MODE_ONEHOT ? nexcl : 0};
                        const uint64_t *loc = mode == MODE_ONEHOT ? sub : ps.sum;
                        if (mode == MODE_ONEHOT && S_eff == 0) { oc.nexcl = 0; loc = ps.sum; }
                        for (int32_t j = 0; j < nch; ++j) {
                            Lc[j] = loc[j];
                            if (ps.frame[j] == FRAME_NONE) { Ac[j] = 0; continue; }
                            int32_t d = ps.C - ps.frame[j];
                            Ac[j] = d > 63 ? 0 : (loc[j] >> d);
                        }
                        tokv = sample_two_level(u0, Ac, Lc, nch, vocab, onehot_w, &oc);
                    }
                    bonus[b] = tokv;
                    break;
                }
            }
            an[alen] = next;
            at[alen] = tok[next];
            ++alen;
            node = next;
        }
        if (seq_err) {
            for (int32_t i = 0; i < max_nodes; ++i) { an[i] = -1; at[i] = -1; }
            bonus[b] = -1;
            continue;
        }
        accept_len[b] = alen;
        if (stats) {
            stats[0] += alen > 0;
            stats[1] += alen == 0;
            stats[2] += alen == 0;
            stats[3] += n - 1;
            stats[4] += 1;
            stats[5] += alen + 1;
        }
    }
    free(cm); free(fr); free(sm); free(Lc); free(Ac); free(excl);
    return status;
}

/* ---------------------------------------------------------------------------
 * Chain acceptance on per-token probabilities, src/engine/speculative_verifier.cpp:84-135.
 * exp(x), x in [-20, 0): t = x*log2(e) rounded once, n = rint(t), 2^(t-n) by
 * the same polynomial, 2^n added to the exponent field.
 * ------------------------------------------------------------------------- */
float or_exp_neg(float x) {
    float t = x * 1.4426950408889634f;
    float r = t + 12582912.0f;
    float nf = r - 12582912.0f;
    float f = t - nf;
    int32_t n = (int32_t)nf;
    float p = or_exp2_poly(f);
    uint32_t bits = f2u(p) + ((uint32_t)n << 23);
    float out; memcpy(&out, &bits, 4); return out;
}

int or_verify_chain(const float *draft, const float *target, const float *uniforms, int32_t batch,
                    int32_t n, int32_t *accepted_len, int32_t *last_idx) {
    int status = ST_OK;
    for (int32_t b = 0; b < batch; ++b) {
        const float *d = draft + (int64_t)b * n, *t = target + (int64_t)b * n, *u = uniforms + (int64_t)b * n;
        int bad = 0;
        for (int32_t i = 0; i < n; ++i) bad |= !(fabsf(t[i]) < INFINITY);
        if (bad) { accepted_len[b] = -1; last_idx[b] = 0; status = status ? status : ST_ENONFINITE; continue; }
        int32_t acc = 0, last = 0;
        for (int32_t i = 0; i < n; ++i) {
            float ld = d[i], lt = t[i], a;
            if (ld < 0.0f || lt < 0.0f) {
                float lr = fmaxf(lt - ld, -20.0f);
                a = lr >= 0.0f ? 1.0f : or_exp_neg(lr);
            } else {
                ld = fmaxf(1e-10f, fminf(ld, 1.0f));
                lt = fmaxf(0.0f, fminf(lt, 1.0f + 1e-6f));
                a = lt / ld;
            }
            if (a > 1.0f) a = 1.0f;
            if (u[i] < a) { ++acc; last = i; } else break;
        }
        accepted_len[b] = acc;
        last_idx[b] = last;
    }
    return status;
}

/* ---------------------------------------------------------------------------
 * Tree attention, fp32. engine/pipeline.py:391-402: GQA head h reads KV head
 * h / (Hq/Hkv) (repeat_interleave), scores = q.k * scale in fp32, softmax in
 * fp32, probabilities rounded to bf16 before the PV product.
 * ------------------------------------------------------------------------- */
static float round_bf16(float x) {
    uint32_t u = f2u(x);
    if ((u & 0x7F800000u) == 0x7F800000u) return x;
    u += 0x7FFFu + ((u >> 16) & 1u);
    u &= 0xFFFF0000u;
    float r; memcpy(&r, &u, 4); return r;
}

int or_tree_attention(const float *q, const float *k_pool, const float *v_pool, int32_t num_pages,
                      const int32_t *page_table, int32_t max_pages_per_seq,
                      const int32_t *ctx_lens, const int32_t *parents, const int32_t *n_nodes,
                      int32_t batch, int32_t max_nodes, int32_t num_q_heads,
                      int32_t num_kv_heads, int32_t head_dim, float scale, float *out,
                      float *lse) {
    if (num_kv_heads < 1 || num_q_heads % num_kv_heads) return ST_EINVAL;
    const int32_t rep = num_q_heads / num_kv_heads;
    int status = ST_OK;
    for (int32_t b = 0; b < batch; ++b) {
        const int32_t n = n_nodes ? n_nodes[b] : max_nodes;
        const int32_t L = ctx_lens[b];
        const int32_t *par = parents + (int64_t)b * max_nodes;
        for (int32_t i = 0; i < max_nodes; ++i) {
            uint64_t anc = 0;
            if (i < n) {
                for (int32_t a = i; a >= 0; a = par[a]) {
                    anc |= 1ull << a;
                    if (a == 0) break;
                    if (par[a] < 0 || par[a] >= a) { status = ST_EBOUNDS; break; }
                }
            }
            const int32_t total = L + i + 1;
            float *s = (float *)malloc(sizeof(float) * (total > 0 ? total : 1));
            for (int32_t h = 0; h < num_q_heads; ++h) {
                float *o = out + (((int64_t)b * max_nodes + i) * num_q_heads + h) * head_dim;
                float *ls = lse ? lse + ((int64_t)b * max_nodes + i) * num_q_heads + h : NULL;
                if (i >= n) {
                    for (int32_t d = 0; d < head_dim; ++d) o[d] = 0.0f;
                    if (ls) *ls = 0.0f;
                    continue;
                }
                const int32_t g = h / rep;
                const float *qv = q + (((int64_t)b * max_nodes + i) * num_q_heads + h) * head_dim;
                float m = -INFINITY;
                for (int32_t p = 0; p < total; ++p) {
                    int visible = p < L || ((anc >> (p - L)) & 1ull);
                    if (!visible) { s[p] = -INFINITY; continue; }
                    int32_t lp = p / 16;
                    int32_t page = lp < max_pages_per_seq ? page_table[(int64_t)b * max_pages_per_seq + lp] : -1;
                    if (page < 0 || page >= num_pages) { status = ST_EBOUNDS; s[p] = -INFINITY; continue; }
                    const float *kr = k_pool + (((int64_t)page * 16 + p % 16) * num_kv_heads + g) * head_dim;
                    float acc = 0.0f;
                    for (int32_t d = 0; d < head_dim; ++d) acc += qv[d] * kr[d];
                    s[p] = acc * scale;
                    if (s[p] > m) m = s[p];
                }
                double l = 0.0;
                for (int32_t p = 0; p < total; ++p) if (s[p] > -INFINITY) l += exp((double)s[p] - m);
                for (int32_t d = 0; d < head_dim; ++d) o[d] = 0.0f;
                for (int32_t p = 0; p < total; ++p) {
                    if (!(s[p] > -INFINITY)) continue;
                    float pr = round_bf16((float)(exp((double)s[p] - m) / l));
                    int32_t page = page_table[(int64_t)b * max_pages_per_seq + p / 16];
                    const float *vr = v_pool + (((int64_t)page * 16 + p % 16) * num_kv_heads + g) * head_dim;
                    for (int32_t d = 0; d < head_dim; ++d) o[d] += pr * vr[d];
                }
                if (ls) *ls = (float)(m + log(l));
            }
            free(s);
        }
    }
    return status;
}

/* ---------------------------------------------------------------------------
 * Compaction of the accepted path (semantics in include/a11spec.h, K4). The
 * copy runs in increasing j; a destination never lies past its own source and
 * never on a later source, so this order equals "read all, then write all".
 * Page release follows the 16-token block rule of src/cuda/paged_kv_cache.cu:129-135
 * run backwards: a page stays while any of its slots is below the length.
 * ------------------------------------------------------------------------- */
int or_kv_compact(uint8_t *k_pool, uint8_t *v_pool, int32_t num_layers, int64_t layer_stride,
                  int32_t num_pages, int32_t row_elems, int32_t elem_bytes, int32_t *page_table,
                  int32_t max_pages_per_seq, int32_t *seq_lens, const int32_t *accept_len,
                  const int32_t *accepted_nodes, const int32_t *n_nodes, int32_t batch,
                  int32_t max_nodes, int32_t *freed_pages, int32_t *n_freed) {
    const int64_t row_bytes = (int64_t)row_elems * elem_bytes;
    int status = ST_OK;
    for (int32_t b = 0; b < batch; ++b) {
        const int32_t L = seq_lens[b], a = accept_len[b];
        const int32_t n = n_nodes ? n_nodes[b] : max_nodes;
        int32_t *pt = page_table + (int64_t)b * max_pages_per_seq;
        if (a < 0 || a >= n) { status = ST_EBOUNDS; if (n_freed) n_freed[b] = 0; continue; }
        for (int32_t l = 0; l < num_layers; ++l) {
            for (int32_t j = 0; j < a; ++j) {
                int32_t node = accepted_nodes[(int64_t)b * max_nodes + j];
                if (node < 1 || node >= n) { status = ST_EBOUNDS; continue; }
                int32_t sp = L + node, dp = L + 1 + j;
                int32_t spg = pt[sp / 16], dpg = pt[dp / 16];
                if (spg < 0 || spg >= num_pages || dpg < 0 || dpg >= num_pages) { status = ST_EBOUNDS; continue; }
                int64_t so = ((int64_t)l * layer_stride + ((int64_t)spg * 16 + sp % 16) * row_elems) * elem_bytes;
                int64_t doff = ((int64_t)l * layer_stride + ((int64_t)dpg * 16 + dp % 16) * row_elems) * elem_bytes;
                memmove(k_pool + doff, k_pool + so, row_bytes);
                memmove(v_pool + doff, v_pool + so, row_bytes);
            }
        }
        const int32_t new_len = L + 1 + a;
        seq_lens[b] = new_len;
        int32_t first = (new_len + 15) / 16, end = (L + n + 15) / 16, nf = 0;
        if (end > max_pages_per_seq) end = max_pages_per_seq;
        for (int32_t p = first; p < end; ++p) {
            if (pt[p] < 0) continue;
            if (freed_pages) freed_pages[(int64_t)b * max_pages_per_seq + nf] = pt[p];
            ++nf;
            pt[p] = -1;
        }
        if (n_freed) n_freed[b] = nf;
    }
    return status;
}

/* ---------------------------------------------------------------------------
 * Hashed trigram expansion (semantics in include/a11spec.h, K1). The bucket
 * hash is the SplitMix64 output finaliser (Steele, Lea & Flood, OOPSLA 2014;
 * constants of Vigna's public-domain splitmix64.c).
 * ------------------------------------------------------------------------- */
static uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

uint32_t or_ngram_bucket(int32_t a, int32_t b, int32_t log2_buckets) {
    uint64_t key = ((uint64_t)(uint32_t)a << 32) | (uint32_t)b;
    return (uint32_t)(mix64(key) >> (64 - log2_buckets));
}

int or_ngram_expand(const int32_t *table, int32_t log2_buckets, int32_t slots,
                    const int32_t *last_tokens, int32_t batch, int32_t width_root,
                    int32_t width_inner, int32_t max_depth, int32_t max_nodes, int32_t *tokens,
                    int32_t *parents, int32_t *depths, int32_t *n_nodes) {
    if (log2_buckets < 1 || log2_buckets > 30 || slots < 1 || slots > 32 || max_nodes < 1)
        return ST_EINVAL;
    for (int32_t b = 0; b < batch; ++b) {
        int32_t *tk = tokens + (int64_t)b * max_nodes, *pa = parents + (int64_t)b * max_nodes,
                *de = depths + (int64_t)b * max_nodes;
        for (int32_t i = 0; i < max_nodes; ++i) { tk[i] = -1; pa[i] = -1; de[i] = -1; }
        tk[0] = last_tokens[2 * b + 1];
        de[0] = 0;
        int32_t n = 1;
        for (int32_t i = 0; i < n && n < max_nodes; ++i) {
            if (de[i] >= max_depth) continue;
            int32_t w = de[i] == 0 ? width_root : width_inner;
            int32_t prev = i == 0 ? last_tokens[2 * b] : tk[pa[i]];
            const int32_t *bk = table + (int64_t)or_ngram_bucket(prev, tk[i], log2_buckets) * slots * 2;
            int used[32] = {0};
            for (int32_t r = 0; r < w && n < max_nodes; ++r) {
                int32_t best = -1;
                for (int32_t s = 0; s < slots; ++s) {
                    if (used[s] || bk[2 * s + 1] <= 0) continue;
                    if (best < 0 || bk[2 * s + 1] > bk[2 * best + 1]) best = s;
                }
                if (best < 0) break;
                used[best] = 1;
                tk[n] = bk[2 * best];
                pa[n] = i;
                de[n] = de[i] + 1;
                ++n;
            }
        }
        n_nodes[b] = n;
    }
    return ST_OK;
}

/* ------------------------------------------------------------------------
 * Page allocator of the paged KV cache, restated from the reference's
 * PagedKVCacheManager (src/cuda/paged_kv_cache.cu): alloc_block 85-93 pops the
 * back of the free stack, append_token 119-135 adds a block when the token
 * count exceeds blocks * 16, allocate_sequence 103-117 gives a new sequence
 * one block, dealloc_block 95-101 / free_sequence 137-149 push blocks back in
 * block-table order. The stack is stack[0 .. *top); the batch is served in
 * order, token by token. Unlike the reference, a batch that cannot be served
 * changes nothing (checked before the loop) and reports a code and a detail:
 * EBOUNDS + the lowest offending sequence, EBOUNDS + -1 for a stack that
 * would leave [0, num_pages], ENOSPACE + the pages the batch needs.
 * ------------------------------------------------------------------------ */
#define ST_ENOSPACE 6

static int32_t or_blocks_for(int32_t len) { return len <= 0 ? 1 : (len + 15) / 16; }

int or_kv_reserve(int32_t *stack, int32_t *top, int32_t num_pages, int32_t *page_table, int32_t max_pages,
                  int32_t *seq_lens, const int32_t *n_new, int32_t batch, int32_t *detail) {
    long long need = 0;
    for (int32_t b = 0; b < batch; ++b) {
        const int32_t len = seq_lens[b], add = n_new[b];
        const int active = page_table[(size_t)b * max_pages] >= 0;
        if (len < 0 || add < 0 || (long long)len + add > 2147483647LL || (!active && len != 0) ||
            or_blocks_for(len + add) > max_pages) {
            *detail = b;
            return ST_EBOUNDS;
        }
        need += or_blocks_for(len + add) - (active ? or_blocks_for(len) : 0);
    }
    if (*top < 0 || *top > num_pages) { *detail = -1; return ST_EBOUNDS; }
    if (need > *top) { *detail = need > 2147483647LL ? 2147483647 : (int32_t)need; return ST_ENOSPACE; }
    for (int32_t b = 0; b < batch; ++b) {
        int32_t *row = page_table + (size_t)b * max_pages;
        int32_t blocks;
        if (row[0] < 0) {  /* allocate_sequence: the first block */
            row[0] = stack[--*top];
            blocks = 1;
        } else {
            blocks = or_blocks_for(seq_lens[b]);
        }
        for (int32_t t = 0; t < n_new[b]; ++t) {  /* append_token */
            seq_lens[b] += 1;
            if (seq_lens[b] > blocks * 16) row[blocks++] = stack[--*top];
        }
    }
    *detail = 0;
    return ST_OK;
}

static int or_kv_push(int32_t *stack, int32_t *top, int32_t num_pages, int32_t *page_table, int32_t max_pages,
                      int32_t *seq_lens, const int32_t *counts, const int32_t *list, int32_t list_stride,
                      int32_t batch, int whole, int32_t *detail) {
    long long total = 0;
    for (int32_t b = 0; b < batch; ++b) {
        const int32_t *src;
        int32_t n;
        if (whole) {
            src = page_table + (size_t)b * max_pages;
            if (!counts[b] || src[0] < 0) continue;
            if (seq_lens[b] < 0) { *detail = b; return ST_EBOUNDS; }
            n = or_blocks_for(seq_lens[b]);
            if (n > max_pages) n = max_pages;
        } else {
            src = list + (size_t)b * list_stride;
            n = counts[b];
            if (n < 0 || n > list_stride) { *detail = b; return ST_EBOUNDS; }
        }
        for (int32_t j = 0; j < n; ++j)
            if (src[j] < 0 || src[j] >= num_pages) { *detail = b; return ST_EBOUNDS; }
        total += n;
    }
    if (*top < 0 || *top + total > num_pages) { *detail = -1; return ST_EBOUNDS; }
    for (int32_t b = 0; b < batch; ++b) {
        if (whole) {
            int32_t *row = page_table + (size_t)b * max_pages;
            if (!counts[b] || row[0] < 0) continue;
            int32_t n = or_blocks_for(seq_lens[b]);
            if (n > max_pages) n = max_pages;
            for (int32_t j = 0; j < n; ++j) {  /* free_sequence: dealloc in table order */
                stack[(*top)++] = row[j];
                row[j] = -1;
            }
            seq_lens[b] = 0;
        } else {
            for (int32_t j = 0; j < counts[b]; ++j) stack[(*top)++] = list[(size_t)b * list_stride + j];
        }
    }
    *detail = 0;
    return ST_OK;
}

int or_kv_release(int32_t *stack, int32_t *top, int32_t num_pages, const int32_t *freed_pages,
                  int32_t freed_stride, const int32_t *n_freed, int32_t batch, int32_t *detail) {
    return or_kv_push(stack, top, num_pages, NULL, 0, NULL, n_freed, freed_pages, freed_stride, batch, 0, detail);
}

int or_kv_free_sequences(int32_t *stack, int32_t *top, int32_t num_pages, int32_t *page_table, int32_t max_pages,
                         int32_t *seq_lens, const int32_t *free_mask, int32_t batch, int32_t *detail) {
    return or_kv_push(stack, top, num_pages, page_table, max_pages, seq_lens, free_mask, NULL, 0, batch, 1, detail);
}

/* ------------------------------------------------------------------------
 * n-gram table update (a11s_ngram_update), serial: rows in order, positions
 * in order. Trigram (x, y, z) with no negative token updates bucket(x, y):
 * the slot holding z with count > 0 gains 1 (saturating); else the lowest
 * slot with count <= 0 becomes (z, 1); else the slot with the smallest count
 * (lowest index among equals) becomes (z, 1). Returns ST_EBOUNDS and the
 * first bad row in *detail (nothing changed) or ST_OK and the count applied.
 * ------------------------------------------------------------------------ */
int or_ngram_update(int32_t *table, int32_t log2_buckets, int32_t slots, const int32_t *history,
                    int32_t stride, const int32_t *lens, int32_t batch, int32_t *detail) {
    for (int32_t b = 0; b < batch; ++b)
        if (lens[b] < 0 || lens[b] > stride) { *detail = b; return ST_EBOUNDS; }
    int32_t applied = 0;
    for (int32_t b = 0; b < batch; ++b) {
        const int32_t *h = history + (size_t)b * stride;
        for (int32_t i = 2; i < lens[b]; ++i) {
            const int32_t x = h[i - 2], y = h[i - 1], z = h[i];
            if (x < 0 || y < 0 || z < 0) continue;
            int32_t *sl = table + (size_t)or_ngram_bucket(x, y, log2_buckets) * slots * 2;
            int hit = -1, empty = -1, low = 0;
            for (int s = 0; s < slots; ++s) {
                if (sl[2 * s + 1] > 0 && sl[2 * s] == z && hit < 0) hit = s;
                if (sl[2 * s + 1] <= 0 && empty < 0) empty = s;
                if (sl[2 * s + 1] < sl[2 * low + 1]) low = s;
            }
            if (hit >= 0) {
                if (sl[2 * hit + 1] < 2147483647) sl[2 * hit + 1] += 1;
            } else {
                const int s = empty >= 0 ? empty : low;
                sl[2 * s] = z;
                sl[2 * s + 1] = 1;
            }
            ++applied;
        }
    }
    *detail = applied;
    return ST_OK;
}
