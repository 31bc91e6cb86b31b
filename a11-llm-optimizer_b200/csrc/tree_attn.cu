// tree_attn.cu - K2: tree-masked verification attention over 16-token KV pages,
// TMA + tcgen05 (TMEM accumulators) on sm_100a.
//
// Math follows engine/pipeline.py:386-402 of the reference (GQA head h reads KV
// head h / (Hq/Hkv); scores q.k * scale in fp32; softmax; probabilities in bf16
// for the PV product), extended to a token tree: node i sees every context
// position and the tree positions of its ancestors and itself.
// Semantics: include/a11spec.h (a11s_tree_attention).
//
// One CTA = one sequence b, one KV head g, 32 tree nodes x 8 query heads as
// two Q tiles of 128 rows (the MMA M), one split of the KV range. 384 threads:
//   warps 0-7  softmax: warp w serves tile w/4, thread = query row = TMEM lane;
//              at the start each thread copies its Q row into shared memory
//   warp 8     TMA producer: K and V blocks of 128 keys (8 pages, one 64x16
//              box per page and 64-column half) into a 2-slot K ring and a
//              3-slot V ring shared by both tiles; page ids fetched 4 blocks
//              ahead
//   warp 9     TMEM allocator + S issuer (QK^T groups)
//   warp 11    PV issuer
//   warp 10    idle (completes the third warpgroup for the register split:
//              softmax warps 216 registers, warps 8-11 56)
// Shared memory: Q of each tile (the A operand of QK^T), the K and V rings.
// TMEM (512 columns): one S buffer of 128 columns used by the tiles in turn,
// O of each tile (128 dims), P of each tile as bf16 pairs (64 columns).
// Per block j and tile t: S = Q_t K_j^T (8 x tcgen05.mma M128 N128 K16, Q and
// K K-major shared-memory operands). The softmax warps load S into registers
// and release the buffer at once (the other tile's S is computed into it
// meanwhile), mask it (ancestor bits), exponentiate (one packed FFMA per pair
// of scores, one ex2 each), keep fp32 row sums of the unrounded values and
// store P_t rounded to bf16 (nearest even) into its TMEM columns; then
// O_t += P_t V_j (8 MMAs, A = P from TMEM, V an MN-major shared-memory operand).
// Two issuer threads: a thread's next shared-memory access (an mbarrier
// poll) waits until the tensor core has read its MMAs' shared-memory
// operands, so one thread issuing both kinds of group leaves the tensor pipe
// idle between them; with S and PV on separate threads each polls and issues
// while the other's group executes.
// Why this shape: an M128 N64 K16 MMA costs about 58 cycles whatever its
// operands, against 32 of math, while N = 128 runs at its math rate; P in
// columns of its own lets S(j+1) overwrite the S buffer while P(j) waits for
// PV, instead of PV(j) having to finish first. With Q in shared memory and P
// in TMEM a block moves about 256 KB through shared memory (TMA writes 64, QK^T
// reads 128, PV reads 64) instead of 320 KB with P in shared memory and Q in
// TMEM.
// The running max is updated lazily: O and l are rescaled only when the block
// max exceeds the reference max by more than 8 (log2 units), which keeps every
// exponent <= 2^8. Split-KV partials are merged by tree_attn_combine.
// Every mbarrier wait is bounded (clock budget); a timeout sets ETIMEOUT and
// the CTA drains and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace a11s {

namespace {
constexpr int kBlockKV = 128;         // keys per KV block = 8 pages (the N of the QK^T MMA)
constexpr int kPagesPerBlock = kBlockKV / A11S_PAGE_TOKENS;
constexpr int kKStages = 2;           // K ring depth: a K slot is free once QK^T of both tiles completed
constexpr int kVStages = 3;           // V ring depth: a V slot is free once PV of both tiles completed
constexpr int kTiles = 2;             // Q tiles per CTA, 128 rows each
constexpr int kNodesPerTile = 16;
constexpr int kNodesPerCta = kTiles * kNodesPerTile;
constexpr int kSoftmaxWarps = 4 * kTiles;
constexpr int kProducerWarp = kSoftmaxWarps, kMmaWarp = kSoftmaxWarps + 1, kPvWarp = kSoftmaxWarps + 3;
constexpr int kTcThreads = 32 * (kSoftmaxWarps + 4);  // + producer, 2 issuers, 1 idle: whole warpgroups
constexpr int kRegsSoftmax = 216, kRegsOther = 56;    // setmaxnreg split (multiples of 8)
constexpr long long kRegsNeeded = 32ll * (kSoftmaxWarps * kRegsSoftmax + 4 * kRegsOther);
constexpr uint32_t kQHalf = 16384;    // Q tile: 128 rows x 128 B per 64-dim half
constexpr uint32_t kKVHalf = 16384;   // K or V: 128 tokens x 128 B per 64-dim half
constexpr uint32_t kOffQ = 0;                                // Q of tile t at 2*kQHalf*t
constexpr uint32_t kSlotBytes = 2 * kKVHalf;                 // one K or V block: 32 KB
constexpr uint32_t kOffK = kTiles * 2 * kQHalf;              // K slots
constexpr uint32_t kOffV = kOffK + kKStages * kSlotBytes;    // V slots
constexpr uint32_t kOffBar = kOffV + kVStages * kSlotBytes;  // 229376
constexpr uint32_t kSmemBytes = kOffBar + 512 + 1024;
// TMEM (512 columns): one S buffer shared by the tiles, O[tile], P[tile] (bf16 pairs)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColO = 128, kColP = 384;  // P of tile t: 64 columns of bf16 pairs
constexpr long long kWaitBudget = 2000000000ll;  // ~1 s of SM clock
constexpr float kRescaleThreshold = 8.0f;
constexpr uint32_t kIdescS = tc::idesc_bf16_f32(128, kBlockKV, false);
constexpr uint32_t kIdescPV = tc::idesc_bf16_f32(128, 128, true);

struct Bars {
    uint64_t k_full[kKStages], k_empty[kKStages], v_full[kVStages], v_empty[kVStages];
    uint64_t q_ready, s_full[kTiles], s_free, p_full[kTiles], pv_done[kTiles];
    uint64_t drain, drain_pv;
    uint32_t tmem_base;
    int32_t abort;
    uint64_t anc[kNodesPerCta];
};
static_assert(sizeof(Bars) <= 512, "barrier block");
static_assert(kSmemBytes <= 232448, "shared memory budget");

struct TcParams {
    const __nv_bfloat16 *q;
    const int32_t *page_table;
    int32_t max_pages, num_pages;
    const int32_t *ctx_lens, *parents, *n_nodes;
    int32_t B, N, Hq, Hkv, splits;
    float scale_log2;
    __nv_bfloat16 *out;
    float *lse;
    float *part_o, *part_ml;
    StatusWord *status;
};
}  // namespace

int tree_attention_splits(int32_t B, int32_t N, int32_t Hq, int32_t Hkv, int32_t max_kv_len) {
    (void)Hq;
    int sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long ctas = (long long)B * Hkv * ((N + kNodesPerCta - 1) / kNodesPerCta);
    const int blocks = (max_kv_len + kBlockKV - 1) / kBlockKV;
    int best = 1;
    double best_cost = 1e300;
    for (int s = 1; s <= 32; ++s) {
        const int bps = (blocks + s - 1) / s;
        if (s > 1 && bps < 8) break;
        const long long waves = (ctas * s + sms - 1) / sms;
        // ~12 blocks of fixed cost per CTA: Q into TMEM, filling the K/V rings
        // and the S chain, the epilogue (fitted to a forced-split sweep)
        const double cost = (double)waves * (bps + 12.0);
        if (cost < best_cost * 0.98) { best_cost = cost; best = s; }
    }
    return best;
}

size_t tree_attention_partials_bytes(int32_t B, int32_t N, int32_t Hq, int32_t D, int32_t splits) {
    return splits > 1 ? (size_t)splits * B * N * Hq * (D + 2) * sizeof(float) : 0;
}

__device__ __forceinline__ bool aborted(Bars *bs) { return *reinterpret_cast<volatile int32_t *>(&bs->abort) != 0; }

__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, uint32_t parity, Bars *bs, StatusWord *st) {
    if (tc::mbar_wait(bar, parity, kWaitBudget)) return true;
    *reinterpret_cast<volatile int32_t *>(&bs->abort) = 1;
    report(st, A11S_ETIMEOUT, 0);
    return false;
}

// Three-input maximum (one instruction on sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

__global__ void __launch_bounds__(kTcThreads, 1)
    tree_attn_tc(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv, const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars *bs = reinterpret_cast<Bars *>(sm + kOffBar);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ct = blockIdx.x, g = blockIdx.y % p.Hkv, split = blockIdx.y / p.Hkv, b = blockIdx.z;

    int n_live = p.n_nodes ? p.n_nodes[b] : p.N;
    if (n_live < 1 || n_live > p.N) {
        if (tid == 0 && ct == 0 && blockIdx.y == 0) report(p.status, A11S_EBOUNDS, b);
        n_live = 0;
    }
    const int node0 = ct * kNodesPerCta;
    const int L = p.ctx_lens[b];
    const int last_node = min(n_live, node0 + kNodesPerCta) - 1;
    const int kv_len = L + last_node + 1;
    const int nblk = (kv_len + kBlockKV - 1) / kBlockKV;
    const int bps = (nblk + p.splits - 1) / p.splits;
    const int blk0 = split * bps;
    const int nb = last_node < node0 ? 0 : max(0, min(blk0 + bps, nblk) - blk0);

    // softmax thread -> (tile, query row m = node_local * 8 + hh)
    const int tile = warp / 4 < kTiles ? warp / 4 : 0;
    const int m = tid & 127;
    const int node = node0 + tile * kNodesPerTile + (m >> 3), row_head = g * 8 + (m & 7);
    if (nb == 0) {
        // nothing to attend in this split (or a dead CTA): empty partial / zero output
        if (warp < kSoftmaxWarps && node < p.N) {
            const size_t row = ((size_t)b * p.N + node) * p.Hq + row_head;
            if (p.splits == 1) {
                uint4 *o = reinterpret_cast<uint4 *>(p.out + row * 128);
                for (int c = 0; c < 16; ++c) o[c] = make_uint4(0, 0, 0, 0);
                if (p.lse) p.lse[row] = 0.0f;
            } else {
                const size_t prow = ((size_t)split * p.B * p.N) * p.Hq + row;
                p.part_ml[prow * 2] = -INFINITY;
                p.part_ml[prow * 2 + 1] = 0.0f;
            }
        }
        return;
    }

    // ---------------- setup ----------------
    if (tid == 0) {
        for (int s = 0; s < kKStages; ++s) {
            tc::mbar_init(&bs->k_full[s], 1);
            tc::mbar_init(&bs->k_empty[s], 1);
        }
        for (int s = 0; s < kVStages; ++s) {
            tc::mbar_init(&bs->v_full[s], 1);
            tc::mbar_init(&bs->v_empty[s], 1);
        }
        for (int t = 0; t < kTiles; ++t) {
            tc::mbar_init(&bs->s_full[t], 1);
            tc::mbar_init(&bs->p_full[t], 4);  // one arrival per softmax warp of the tile
            tc::mbar_init(&bs->pv_done[t], 1);
        }
        tc::mbar_init(&bs->s_free, 4);
        tc::mbar_init(&bs->q_ready, kSoftmaxWarps);
        tc::mbar_init(&bs->drain, 1);
        tc::mbar_init(&bs->drain_pv, 1);
        bs->abort = 0;
        tc::fence_barrier_init();
    }
    if (warp == kProducerWarp) {
        // ancestor-or-self bits of the CTA's nodes (lane = node offset). The
        // sequence's parents (N <= 64) sit in two registers per lane, read
        // with one coalesced load; each step up the tree is two shuffles.
        const int32_t *par = p.parents + (size_t)b * p.N;
        const int32_t r0 = lane < p.N ? par[lane] : -1;
        const int32_t r1 = lane + 32 < p.N ? par[lane + 32] : -1;
        const int nd = node0 + lane;
        uint64_t anc = 0;
        int a = nd;
        bool done = !(nd < n_live), ok = false;
        for (int steps = 0; steps <= 64; ++steps) {
            if (!__any_sync(0xffffffffu, !done)) break;
            const int v0 = __shfl_sync(0xffffffffu, r0, a & 31), v1 = __shfl_sync(0xffffffffu, r1, a & 31);
            if (!done) {
                anc |= 1ull << a;
                if (a == 0) {
                    ok = true;
                    done = true;
                } else {
                    const int pa = a < 32 ? v0 : v1;
                    if (pa < 0 || pa >= a) done = true;
                    else a = pa;
                }
            }
        }
        if (nd < n_live && !ok) {
            report(p.status, A11S_EBOUNDS, b);
            anc = 1ull << nd;
        }
        bs->anc[lane] = anc;
    }
    if (warp == kMmaWarp) {
        tc::tmem_alloc(&bs->tmem_base, kTmemCols);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = bs->tmem_base;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    // Register split per warpgroup (setmaxnreg acts on whole warpgroups):
    // warps 8-11 give registers back, the softmax warps take them. The total
    // stays within the launch's registers (checked on the host before launch).
    static_assert(kRegsSoftmax % 8 == 0 && kRegsOther % 8 == 0, "setmaxnreg counts");
    if (warp >= kSoftmaxWarps) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsOther));
        if (warp == kProducerWarp) {
            // ---------------- TMA producer ----------------
            if (lane == 0) {
                tc::prefetch_tmap(&tk);
                tc::prefetch_tmap(&tv);
            }
            // Page ids of 4 blocks (32 entries) per coalesced warp load, double
            // buffered, so a block's ids were requested 4 blocks before use.
            constexpr int kBlocksPerWindow = 32 / kPagesPerBlock;
            const int32_t *pt = p.page_table + (size_t)b * p.max_pages;
            const int lp0 = blk0 * kPagesPerBlock;
            const int lp_end = min((kv_len + A11S_PAGE_TOKENS - 1) / A11S_PAGE_TOKENS, (blk0 + nb) * kPagesPerBlock);
            auto window = [&](int w) -> int {  // entry lp0 + 32 w + lane, or -2 past the needed range
                const int lp = lp0 + 32 * w + lane;
                if (lp >= lp_end) return -2;
                return lp < p.max_pages ? __ldg(pt + lp) : -1;
            };
            int cur = window(0), nxt = window(1);
            int nk = 0, nv = 0;  // K and V blocks whose loads were issued
            for (int it = 0; it < nb && !aborted(bs); ++it) {
                const int k = it % kBlocksPerWindow;
                if (k == 0 && it > 0) {
                    cur = nxt;
                    nxt = window(it / kBlocksPerWindow + 1);
                }
                const int id = __shfl_sync(0xffffffffu, cur, (k * kPagesPerBlock + lane) & 31);
                int page = p.num_pages;  // out of range -> zero fill
                if (lane < kPagesPerBlock && id != -2) {
                    if (id < 0 || id >= p.num_pages) report(p.status, A11S_EBOUNDS, b);
                    else page = id;
                }
                // K(it): its slot was last read by QK(it - kKStages)
                const int ks = it % kKStages, kuse = it / kKStages;
                if (lane == 0 && kuse > 0) wait_or_abort(&bs->k_empty[ks], (kuse - 1) & 1, bs, p.status);
                __syncwarp();
                if (aborted(bs)) break;
                if (lane == 0) tc::mbar_arrive_expect_tx(&bs->k_full[ks], kSlotBytes);
                __syncwarp();
                uint8_t *sK = sm + kOffK + ks * kSlotBytes;
                if (lane < kPagesPerBlock) {
                    tc::tma_load_4d(sK + lane * 2048, &tk, &bs->k_full[ks], 0, g, 0, page);
                    tc::tma_load_4d(sK + kKVHalf + lane * 2048, &tk, &bs->k_full[ks], 64, g, 0, page);
                }
                ++nk;
                // V(it): its slot was last read by PV(it - kVStages)
                const int vs = it % kVStages, vuse = it / kVStages;
                if (lane == 0 && vuse > 0) wait_or_abort(&bs->v_empty[vs], (vuse - 1) & 1, bs, p.status);
                __syncwarp();
                if (aborted(bs)) break;
                if (lane == 0) tc::mbar_arrive_expect_tx(&bs->v_full[vs], kSlotBytes);
                __syncwarp();
                uint8_t *sV = sm + kOffV + vs * kSlotBytes;
                if (lane < kPagesPerBlock) {
                    tc::tma_load_4d(sV + lane * 2048, &tv, &bs->v_full[vs], 0, g, 0, page);
                    tc::tma_load_4d(sV + kKVHalf + lane * 2048, &tv, &bs->v_full[vs], 64, g, 0, page);
                }
                ++nv;
            }
            if (aborted(bs) && lane == 0) {
                // drain copies that may still be landing in this CTA's shared memory
                for (int i = max(0, nk - kKStages); i < nk; ++i)
                    tc::mbar_wait(&bs->k_full[i % kKStages], (i / kKStages) & 1, kWaitBudget);
                for (int i = max(0, nv - kVStages); i < nv; ++i)
                    tc::mbar_wait(&bs->v_full[i % kVStages], (i / kVStages) & 1, kWaitBudget);
            }
        } else if (warp == kMmaWarp) {
            // ---------------- S issuer ----------------
            if (lane == 0) {
                auto issue_s = [&](int j, int t) {  // S = Q_t K_j^T: 8 MMAs M128 N128 K16, Q and K in shared memory
                    const uint32_t k_addr = tc::smem_u32(sm + kOffK + (j % kKStages) * kSlotBytes);
                    const uint32_t q_addr = tc::smem_u32(sm + kOffQ + t * 2 * kQHalf);
    #pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
                        tc::mma_bf16_ss(tmem + kColS,
                                        tc::sdesc_sw128(q_addr + (kk >> 2) * kQHalf + (kk & 3) * 32, 16, 1024),
                                        tc::sdesc_sw128(k_addr + (kk >> 2) * kKVHalf + (kk & 3) * 32, 16, 1024),
                                        kIdescS, kk > 0);
                    tc::mma_commit(&bs->s_full[t]);
                    if (t == kTiles - 1) tc::mma_commit(&bs->k_empty[j % kKStages]);
                };
                // S groups in the order u = 2 j + t: S(u) needs the S buffer
                // (the tile before has loaded S(u - 1)) and K(j). Every phase
                // waited for is the next one of its barrier.
                bool ok = wait_or_abort(&bs->q_ready, 0, bs, p.status);
                for (int u = 0; u < kTiles * nb && ok; ++u) {
                    const int j = u / kTiles, t = u % kTiles;
                    if (u > 0) ok = wait_or_abort(&bs->s_free, (u - 1) & 1, bs, p.status);
                    if (ok && t == 0) ok = wait_or_abort(&bs->k_full[j % kKStages], (j / kKStages) & 1, bs, p.status);
                    if (!ok) break;
                    tc::tc_fence_after();
                    issue_s(j, t);
                }
                // wait for every issued MMA before the CTA may release TMEM
                tc::mma_commit(&bs->drain);
                tc::mbar_wait(&bs->drain, 0, kWaitBudget);
            }
            __syncwarp();
        } else if (warp == kPvWarp) {
            // ---------------- PV issuer ----------------
            if (lane == 0) {
                auto issue_pv = [&](int j, int t) {  // O_t += P_t V_j: 8 MMAs M128 N128 K16, A = P from TMEM
                    const uint32_t v_addr = tc::smem_u32(sm + kOffV + (j % kVStages) * kSlotBytes);
    #pragma unroll
                    for (int kk = 0; kk < kBlockKV / 16; ++kk)
                        tc::mma_bf16_ts(tmem + kColO + 128 * t, tmem + kColP + 64 * t + kk * 8,
                                        tc::sdesc_sw128(v_addr + kk * 2048, kKVHalf, 1024), kIdescPV,
                                        (j > 0 || kk > 0) ? 1u : 0u);
                    tc::mma_commit(&bs->pv_done[t]);
                    if (t == kTiles - 1) tc::mma_commit(&bs->v_empty[j % kVStages]);
                };
                // PV groups in the same order: P_t(j) stored and V(j) landed.
                bool ok = true;
                for (int u = 0; u < kTiles * nb && ok; ++u) {
                    const int j = u / kTiles, t = u % kTiles;
                    ok = wait_or_abort(&bs->p_full[t], j & 1, bs, p.status);
                    if (ok && t == 0) ok = wait_or_abort(&bs->v_full[j % kVStages], (j / kVStages) & 1, bs, p.status);
                    if (!ok) break;
                    tc::tc_fence_after();
                    issue_pv(j, t);
                }
                tc::mma_commit(&bs->drain_pv);
                tc::mbar_wait(&bs->drain_pv, 0, kWaitBudget);
            }
            __syncwarp();
        }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
        // ---------------- softmax warps: tile = warp / 4, thread = query row ----------------
        // Q row of this thread into TMEM as the A operand of QK^T (bf16 pairs,
        // lane = row): 256 bytes, zeros past the last node. The issuer
        // waits for q_ready before the first S.
        {
            // 256 bytes of Q into the tile's 128-byte-swizzled K-major A operand:
            // 64-dim half h at 16 KB h, row m at 128 m, 16-byte chunk c at slot c ^ (m & 7)
            const uint32_t q_row = tc::smem_u32(sm + kOffQ + tile * 2 * kQHalf + m * 128);
            const uint4 *src = reinterpret_cast<const uint4 *>(p.q + (((size_t)b * p.N + node) * p.Hq + row_head) * 128);
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const uint4 v = node < p.N ? __ldg(src + c) : make_uint4(0, 0, 0, 0);
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
                tc::st_shared_v4(q_row + (uint32_t)(c >> 3) * kQHalf + ((uint32_t)((c & 7) ^ (m & 7)) << 4), w);
            }
            tc::fence_proxy_async_smem();  // Q visible to the tensor core
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&bs->q_ready);
        }
        // `ok` stays warp-uniform for the .sync.aligned TMEM accesses.
        const bool live = node < n_live;
        const uint64_t anc = bs->anc[node - node0];
        const uint32_t p_cols = tmem + lane_base + kColP + 64 * tile;  // this row of P_t (bf16 pairs)
        const float sl2 = p.scale_log2;
        float m_ref = -INFINITY, lsum = 0.0f;
        bool ok = true;
        for (int it = 0; it < nb && ok; ++it) {
            const int p0 = (blk0 + it) * kBlockKV;
            ok = __all_sync(0xffffffffu, wait_or_abort(&bs->s_full[tile], it & 1, bs, p.status));
            if (!ok) break;
            tc::tc_fence_after();
            float xa[64], xb[64];  // keys 0-63 and 64-127 of the block
            tc::tmem_ld64(tmem + lane_base + kColS, xa);
            tc::tmem_ld64(tmem + lane_base + kColS + 64, xb);
            // S is in registers: the other tile's S may overwrite the buffer
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&bs->s_free);
#define X(c) ((c) < 64 ? xa[(c) & 63] : xb[(c) & 63])
            // mask (raw scores) and block max
            if (live && p0 + kBlockKV > L) {
#pragma unroll
                for (int c = 0; c < kBlockKV; ++c) {
                    const int jt = p0 + c - L;
                    const bool vis = jt < 0 || (jt <= node && ((anc >> (jt & 63)) & 1ull));
                    if (!vis) X(c) = -INFINITY;
                }
            }
            float mx8[8];  // 8 independent chains of three-input maxima, then a tree
#pragma unroll
            for (int q = 0; q < 8; ++q) mx8[q] = xa[q];
#pragma unroll
            for (int c = 8; c + 16 <= kBlockKV; c += 16)
#pragma unroll
                for (int q = 0; q < 8; ++q) mx8[q] = fmax3(mx8[q], X(c + q), X(c + 8 + q));
#pragma unroll
            for (int q = 0; q < 8; ++q) mx8[q] = fmaxf(mx8[q], X(kBlockKV - 8 + q));
            const float mx = fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]),
                                   fmaxf(mx8[6], mx8[7]));
            const float mb = mx * sl2;  // scale > 0: max commutes with scaling
            // lazy rescale of (O, l)
            float alpha = 1.0f;
            bool rescale = false;
            if (mx > -INFINITY) {
                if (m_ref == -INFINITY) {
                    m_ref = mb;  // first visible block of this row: its O row is still zero
                } else if (mb > m_ref + kRescaleThreshold) {
                    alpha = tc::ex2(m_ref - mb);
                    m_ref = mb;
                    rescale = true;
                }
            }
            const float neg = m_ref == -INFINITY ? 0.0f : -m_ref;
            // PV(it - 1) of this tile must have completed: it read P_t from
            // shared memory (about to be overwritten) and accumulated into O.
            if (it > 0) {
                ok = __all_sync(0xffffffffu, wait_or_abort(&bs->pv_done[tile], (it - 1) & 1, bs, p.status));
                if (!ok) break;
                tc::tc_fence_after();
            }
            float2 ls[4] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};  // independent partial sums
            // P as bf16 pairs (lower key in the low half) into the tile's P columns,
            // 32 keys per store: the A operand of PV from TMEM
#pragma unroll
            for (int c32 = 0; c32 < kBlockKV / 32; ++c32) {
                uint32_t pw[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const int c = 32 * c32 + 2 * e;
                    const float2 ev = tc::ffma2(make_float2(X(c), X(c + 1)), make_float2(sl2, sl2), make_float2(neg, neg));
                    const float2 a = make_float2(tc::ex2(ev.x), tc::ex2(ev.y));
                    pw[e] = tc::cvt_bf16x2(a.x, a.y);
                    ls[e & 3] = tc::fadd2(ls[e & 3], a);  // fp32 denominator of the unrounded p
                }
                tc::tmem_st16u_nowait(p_cols + 16 * c32, pw);
            }
            lsum = lsum * alpha + (((ls[0].x + ls[0].y) + (ls[1].x + ls[1].y)) + ((ls[2].x + ls[2].y) + (ls[3].x + ls[3].y)));
            // Rescale O before PV(it) may start (the scores are dead by now).
            if (__any_sync(0xffffffffu, rescale) && it > 0) {
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float o[32];
                    tc::tmem_ld32(tmem + lane_base + kColO + 128 * tile + c * 32, o);
#pragma unroll
                    for (int e = 0; e < 32; ++e) o[e] *= alpha;
                    tc::tmem_st32(tmem + lane_base + kColO + 128 * tile + c * 32, o);
                }
            }
            tc::tmem_wait_st();  // P (and a rescaled O) written before PV(it) may read them
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&bs->p_full[tile]);
#undef X
        }
        // ---------------- epilogue ----------------
        if (ok && __all_sync(0xffffffffu, wait_or_abort(&bs->pv_done[tile], (nb - 1) & 1, bs, p.status))) {
            tc::tc_fence_after();
            const size_t row = ((size_t)b * p.N + node) * p.Hq + row_head;
            const bool write = node < p.N;
            const float inv = lsum > 0.0f ? 1.0f / lsum : 0.0f;
            if (p.splits == 1) {
                uint4 *o16 = reinterpret_cast<uint4 *>(p.out + row * 128);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float o[32];
                    tc::tmem_ld32(tmem + lane_base + kColO + 128 * tile + c * 32, o);
                    if (write) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            uint32_t w[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float a0 = live ? o[q * 8 + 2 * e] * inv : 0.0f;
                                const float a1 = live ? o[q * 8 + 2 * e + 1] * inv : 0.0f;
                                __nv_bfloat162 pr = __floats2bfloat162_rn(a0, a1);
                                w[e] = *reinterpret_cast<uint32_t *>(&pr);
                            }
                            o16[c * 4 + q] = make_uint4(w[0], w[1], w[2], w[3]);
                        }
                    }
                }
                if (write && p.lse) p.lse[row] = live && lsum > 0.0f ? (m_ref + log2f(lsum)) * 0.6931471805599453f : 0.0f;
            } else {
                const size_t prow = (size_t)split * p.B * p.N * p.Hq + row;
                float4 *po = reinterpret_cast<float4 *>(p.part_o + prow * 128);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float o[32];
                    tc::tmem_ld32(tmem + lane_base + kColO + 128 * tile + c * 32, o);
                    if (write)
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            po[c * 8 + q] = make_float4(o[q * 4] * inv, o[q * 4 + 1] * inv, o[q * 4 + 2] * inv,
                                                        o[q * 4 + 3] * inv);
                }
                if (write) {
                    p.part_ml[prow * 2] = lsum > 0.0f ? m_ref : -INFINITY;
                    p.part_ml[prow * 2 + 1] = lsum;
                }
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
}

// Merge split-KV partials: one warp per (b, node, head) row.
__global__ void tree_attn_combine(const TcParams p) {
    const int warp_global = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const size_t rows = (size_t)p.B * p.N * p.Hq;
    if ((size_t)warp_global >= rows) return;
    const size_t row = warp_global;
    const int b = (int)(row / ((size_t)p.N * p.Hq));
    const int node = (int)((row / p.Hq) % p.N);
    int n_live = p.n_nodes ? p.n_nodes[b] : p.N;
    if (n_live < 1 || n_live > p.N) n_live = 0;
    // online merge, 4 splits per group with all their loads in flight together
    float4 acc = make_float4(0, 0, 0, 0);
    float M = -INFINITY, wsum = 0.0f;
    if (node < n_live) {
        for (int s0 = 0; s0 < p.splits; s0 += 4) {
            float ms[4], ls[4];
            float4 o[4];
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                const size_t prow = (size_t)min(s0 + g, p.splits - 1) * rows + row;
                ms[g] = p.part_ml[prow * 2];
                ls[g] = s0 + g < p.splits ? p.part_ml[prow * 2 + 1] : 0.0f;
                o[g] = reinterpret_cast<const float4 *>(p.part_o + prow * 128)[lane];
            }
            float Mg = M;
#pragma unroll
            for (int g = 0; g < 4; ++g)
                if (ls[g] > 0.0f) Mg = fmaxf(Mg, ms[g]);
            if (Mg == -INFINITY) continue;
            const float a = M == -INFINITY ? 0.0f : exp2f(M - Mg);
            acc.x *= a; acc.y *= a; acc.z *= a; acc.w *= a;
            wsum *= a;
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                if (!(ls[g] > 0.0f)) continue;
                const float w = ls[g] * exp2f(ms[g] - Mg);
                acc.x += w * o[g].x; acc.y += w * o[g].y; acc.z += w * o[g].z; acc.w += w * o[g].w;
                wsum += w;
            }
            M = Mg;
        }
    }
    const float inv = wsum > 0.0f ? 1.0f / wsum : 0.0f;
    __nv_bfloat162 r0 = __floats2bfloat162_rn(acc.x * inv, acc.y * inv);
    __nv_bfloat162 r1 = __floats2bfloat162_rn(acc.z * inv, acc.w * inv);
    uint2 packed;
    packed.x = *reinterpret_cast<uint32_t *>(&r0);
    packed.y = *reinterpret_cast<uint32_t *>(&r1);
    reinterpret_cast<uint2 *>(p.out + row * 128)[lane] = packed;
    if (p.lse && lane == 0) p.lse[row] = wsum > 0.0f ? (M + log2f(wsum)) * 0.6931471805599453f : 0.0f;
}

// ---------------------------------------------------------------------------- host side
namespace {
PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

bool encode(CUtensorMap *map, const void *base, int rank, const cuuint64_t *dims, const cuuint64_t *strides,
            const cuuint32_t *box) {
    auto fn = get_encode();
    if (!fn) return false;
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

cudaError_t launch_tree_attention(const AttnArgs &a, cudaStream_t s) {
    CUtensorMap tk, tv;
    {  // K, V [pages][16][Hkv][128]: box 64 dims x 1 head x 16 tokens x 1 page
        const cuuint64_t dims[4] = {128, (cuuint64_t)a.Hkv, 16, (cuuint64_t)a.num_pages};
        const cuuint64_t str[3] = {256, (cuuint64_t)a.Hkv * 256, (cuuint64_t)a.Hkv * 256 * 16};
        const cuuint32_t box[4] = {64, 1, 16, 1};
        if (!encode(&tk, a.k_pool, 4, dims, str, box)) return cudaErrorInvalidValue;
        if (!encode(&tv, a.v_pool, 4, dims, str, box)) return cudaErrorInvalidValue;
    }
    cudaError_t ea = cudaFuncSetAttribute(tree_attn_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (ea != cudaSuccess) return ea;
    {  // setmaxnreg.inc would wait forever if the split needed more registers than the launch holds
        cudaFuncAttributes fa{};
        ea = cudaFuncGetAttributes(&fa, tree_attn_tc);
        if (ea != cudaSuccess) return ea;
        if ((long long)fa.numRegs * kTcThreads < kRegsNeeded) return cudaErrorInvalidConfiguration;
    }
    TcParams p{};
    p.q = reinterpret_cast<const __nv_bfloat16 *>(a.q);
    p.page_table = a.page_table;
    p.max_pages = a.max_pages;
    p.num_pages = a.num_pages;
    p.ctx_lens = a.ctx_lens;
    p.parents = a.parents;
    p.n_nodes = a.n_nodes;
    p.B = a.B;
    p.N = a.N;
    p.Hq = a.Hq;
    p.Hkv = a.Hkv;
    p.splits = a.splits;
    p.scale_log2 = a.scale * 1.4426950408889634f;
    p.out = reinterpret_cast<__nv_bfloat16 *>(a.out);
    p.lse = a.lse;
    p.part_o = a.part_o;
    p.part_ml = a.part_ml;
    p.status = a.status;
    const dim3 grid((a.N + kNodesPerCta - 1) / kNodesPerCta, a.Hkv * a.splits, a.B);
    tree_attn_tc<<<grid, kTcThreads, kSmemBytes, s>>>(tk, tv, p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || a.splits == 1) return e;
    const size_t rows = (size_t)a.B * a.N * a.Hq;
    tree_attn_combine<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, s>>>(p);
    return cudaGetLastError();
}

}  // namespace a11s
