// lm_head.cu - K7: the tree-node LM head on the tensor cores (TMA + tcgen05,
// TMEM accumulators, sm_100a), with the acceptance's chunk records folded
// into its epilogue.
//
// logits[r][v] = bf16_rn(scale * sum_k hidden[r][k] * weight[v][k]), fp32 accumulation:
// the `torch.matmul(h_norm, output_w.t())` of A11Pipeline.forward_token
// (engine/pipeline.py:468-472) for every tree node at once, the job of
// tree_forward_pass_kernel (src/cuda/tree_verification.cu:34-68).
// keys[r][j] (nullable): the maximum of row r's bf16 logits in 2048-token chunk
// j and its first position, one 64-bit key per (row, chunk): the order image
// of the value (lm_order2) above the complement of the position, combined over
// the chunk's 8 tiles with atomicMax. The acceptance kernel turns them into
// its chunk records instead of streaming the logits once more.
// Semantics: include/a11spec.h (a11s_lm_head).
//
// Persistent kernel of CTA pairs (clusters of 2, one CTA per SM), tiles of
// 256 rows x 256 vocabulary entries taken m-fastest, so the pairs at work at
// one time share a weight tile (read from HBM once) and the hidden states stay
// in L2. Each CTA stages its own 128 rows of the hidden tile and its half (128
// rows) of the weight tile; the even CTA issues cta_group::2 MMAs over both,
// and each CTA's TMEM holds its 128 rows of the accumulator. Against single
// CTAs with 128 x 256 tiles this moves a third less operand data per SM
// through shared memory. 192 threads per CTA:
//   warp 0     TMA producer: K slices of 64 of its hidden rows (128 x 64) and
//              weight rows (128 x 64) into a 6-stage ring, 128-byte swizzle;
//              both CTAs' copies complete on the even CTA's barrier
//   warp 1     TMEM allocator (both CTAs) and, in the even CTA, MMA issuer:
//              per K slice 4 x tcgen05.mma.cta_group::2 M256 N256 K16, both
//              operands K-major in shared memory, into one of two accumulators
//              of 256 TMEM columns; commits signal both CTAs
//   warps 2-5  epilogue (thread = tile row = TMEM lane): 128 columns per TMEM
//              load, bf16 rounding (nearest even), the chunk key on packed
//              pairs, the bf16 tile staged in swizzled shared memory and
//              written by TMA stores (clipped at the vocabulary and the last
//              row). The accumulator is released (to the even CTA) after its
//              last load, so the epilogue of tile i runs under the MMAs of
//              tile i + 1.
// Every mbarrier wait is bounded; a timeout sets ETIMEOUT, and the CTA drains
// its copies and MMAs and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace a11s {

namespace {
constexpr int kBM = 128, kBN = 256, kBK = 64;  // a CTA's tile rows, tile columns, K slice
constexpr uint32_t kABytes = kBM * kBK * 2;    // 16 KB
constexpr uint32_t kBoxBytes = 32 * 128;       // one stored box: 32 rows x 64 columns
constexpr uint32_t kStageWarpBytes = 2 * kBoxBytes;  // an epilogue warp's staging area
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 2 * kBN;
constexpr long long kWaitBudget = 2000000000ll;  // ~1 s of SM clock
static_assert(A11S_CHUNK % kBN == 0, "a tile lies inside one chunk");
// A CTA pair (cluster of 2, cta_group::2 MMAs issued by the even CTA) computes
// 256 x 256 tiles: each CTA stages its 128 hidden rows and half of the weight
// tile (128 x 64 per K slice: 32 KB stages), and its TMEM holds its 128 rows
// of the accumulator.
constexpr int kStages = 6;
constexpr int kTileRows = 2 * kBM;
constexpr uint32_t kBRows = kBN / 2;  // weight rows a CTA stages
constexpr uint32_t kStageBytes = kABytes + kBRows * kBK * 2;
constexpr uint32_t kOffStage = kStages * kStageBytes;  // 196608
constexpr uint32_t kOffBar = kOffStage + 4 * kStageWarpBytes;
constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;  // + barriers + alignment slack
constexpr uint32_t kIdesc = tc::idesc_bf16_f32(kTileRows, kBN, false);
static_assert(kSmemBytes <= 232448, "shared memory budget");

struct Bars {
    uint64_t full[kStages], empty[kStages];
    uint64_t acc_full[2], acc_empty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int32_t abort;
};
static_assert(sizeof(Bars) <= 256, "barrier block");

struct LmParams {
    __nv_bfloat16 *logits;
    int64_t ldl;
    unsigned long long *keys;
    float scale;
    int32_t rows, V, nch, m_tiles, n_tiles, k_blocks;
    StatusWord *status;
};

__device__ __forceinline__ bool aborted(Bars *bs) { return *reinterpret_cast<volatile int32_t *>(&bs->abort) != 0; }

__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, uint32_t parity, Bars *bs, StatusWord *st) {
    if (tc::mbar_wait(bar, parity, kWaitBudget)) return true;
    *reinterpret_cast<volatile int32_t *>(&bs->abort) = 1;
    report(st, A11S_ETIMEOUT, (int32_t)blockIdx.x);
    return false;
}
}  // namespace

// Order-preserving images of a bf16 pair for an unsigned comparison, per
// half: sign set -> all 16 bits flipped, else the sign bit set (+0 -> 0x8000,
// -inf -> 0x007F).
__device__ __forceinline__ uint32_t lm_order2(uint32_t w) {
    const uint32_t s = (w >> 15) & 0x00010001u;
    return w ^ (s * 0x7FFFu + 0x80008000u);
}
__device__ __forceinline__ uint32_t lm_max_nan_bf16x2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// Chunk key of 128 columns (col0 .. col0 + 127 of the tile; w = their bf16
// pairs, already staged for the store) folded into (best, best_col): the
// largest ordered value, -0 taken as +0 and any NaN as the largest (0xFFFF),
// and the first column holding it. Columns at or past `valid` take no part
// (set to -inf here; the store clips them). The maximum is one packed
// NaN-propagating chain; the position is searched only when this half beats
// `best`, which a later half must strictly exceed, so the first position wins
// ties.
__device__ __forceinline__ void lm_half_key(uint32_t (&w)[64], int col0, int valid, uint32_t &best, int &best_col) {
    if (col0 + 128 > valid) {  // the vocabulary ends in this half (valid is a multiple of 8)
#pragma unroll
        for (int e = 0; e < 64; ++e)
            if (col0 + 2 * e >= valid) w[e] = 0xFF80FF80u;
    }
    uint32_t mx = w[0];
#pragma unroll
    for (int e = 1; e < 64; ++e) mx = lm_max_nan_bf16x2(mx, w[e]);
    const uint32_t lo = mx & 0xFFFFu, hi = mx >> 16;
    int pos = 0;
    if ((lo & 0x7FFFu) > 0x7F80u || (hi & 0x7FFFu) > 0x7F80u) {  // a NaN: it is the maximum
        if (0xFFFFu <= best) return;
#pragma unroll
        for (int e = 63; e >= 0; --e) {
            if ((w[e] >> 16 & 0x7FFFu) > 0x7F80u) pos = 2 * e + 1;
            if ((w[e] & 0x7FFFu) > 0x7F80u) pos = 2 * e;
        }
        best = 0xFFFFu;
        best_col = col0 + pos;
        return;
    }
    // the larger of the two halves (no NaN left), a zero maximum as +0
    uint32_t Mv = __uint_as_float(lo << 16) >= __uint_as_float(hi << 16) ? lo : hi;
    if ((Mv & 0x7FFFu) == 0) Mv = 0;
    const uint32_t M = lm_order2(Mv) & 0xFFFFu;
    if (M <= best) return;
    const uint32_t Mz = Mv == 0 ? 0x8000u : Mv;  // a zero maximum matches either sign
#pragma unroll
    for (int e = 63; e >= 0; --e) {
        const uint32_t l = w[e] & 0xFFFFu, h = w[e] >> 16;
        if (h == Mv || h == Mz) pos = 2 * e + 1;
        if (l == Mv || l == Mz) pos = 2 * e;
    }
    best = M;
    best_col = col0 + pos;
}

__global__ void __launch_bounds__(kThreads, 1)
    lm_head_tc(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
               const __grid_constant__ CUtensorMap tc_out, const LmParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars *bs = reinterpret_cast<Bars *>(sm + kOffBar);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // both CTAs of a pair take the same tiles
    const uint32_t rank = tc::cluster_rank();
    const int unit = (int)tc::cluster_id(), units = (int)tc::cluster_count();
    const int total = p.m_tiles * p.n_tiles;
    const int my_tiles = unit < total ? (total - 1 - unit) / units + 1 : 0;
    if (my_tiles == 0) return;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            tc::mbar_init(&bs->full[s], 1);
            tc::mbar_init(&bs->empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&bs->acc_full[b], 1);
            tc::mbar_init(&bs->acc_empty[b], 8);  // one arrival per epilogue warp of both CTAs
        }
        tc::mbar_init(&bs->drain, 1);
        bs->abort = 0;
        tc::fence_barrier_init();
    }
    if (warp == 1) {
        tc::tmem_alloc_pair(&bs->tmem_base, kTmemCols);
        tc::tmem_relinquish_pair();
    }
    tc::tc_fence_before();
    tc::cluster_sync();  // the even CTA's barriers are ready before the peer signals them
    tc::tc_fence_after();
    const uint32_t tmem = bs->tmem_base;

    if (warp == 0) {
        // ---------------- TMA producer (each CTA its own rows) ----------------
        if (lane == 0) {
            tc::prefetch_tmap(&ta);
            tc::prefetch_tmap(&tb);
            tc::prefetch_tmap(&tc_out);
            int it = 0;  // K slices issued
            bool ok = true;
            for (int i = 0; i < my_tiles && ok; ++i) {
                const int t = unit + i * units;
                const int m0 = (t % p.m_tiles) * kTileRows + (int)rank * kBM, n0 = (t / p.m_tiles) * kBN;
                for (int kb = 0; kb < p.k_blocks; ++kb) {
                    const int s = it % kStages, use = it / kStages;
                    // the slot was last read by the MMAs of slice it - kStages
                    if (use > 0 && !(ok = wait_or_abort(&bs->empty[s], (use - 1) & 1, bs, p.status))) break;
                    if (aborted(bs)) {
                        ok = false;
                        break;
                    }
                    uint8_t *sa = sm + s * kStageBytes;
                    // both CTAs' copies complete on the even CTA's barrier, which the MMAs wait on
                    const uint32_t fb = tc::cluster_addr(&bs->full[s], 0);
                    if (rank == 0) tc::mbar_arrive_expect_tx(&bs->full[s], 2 * kStageBytes);
                    tc::tma_load_2d_pair(sa, &ta, fb, kb * kBK, m0);
                    tc::tma_load_2d_pair(sa + kABytes, &tb, fb, kb * kBK, n0 + (int)(rank * kBRows));
                    ++it;
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer (the even CTA) ----------------
        if (lane == 0 && rank == 0) {
            int it = 0;
            bool ok = true;
            for (int i = 0; i < my_tiles && ok; ++i) {
                const int buf = i & 1, use = i >> 1;
                // the epilogue of tile i - 2 has read this accumulator
                if (use > 0 && !(ok = wait_or_abort(&bs->acc_empty[buf], (use - 1) & 1, bs, p.status))) break;
                tc::tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(buf * kBN);
                for (int kb = 0; kb < p.k_blocks; ++kb) {
                    const int s = it % kStages;
                    if (!(ok = wait_or_abort(&bs->full[s], (it / kStages) & 1, bs, p.status))) break;
                    tc::tc_fence_after();
                    const uint32_t a_addr = tc::smem_u32(sm + s * kStageBytes), b_addr = a_addr + kABytes;
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk) {
                        const uint64_t ad = tc::sdesc_sw128(a_addr + kk * 32, 16, 1024);
                        const uint64_t bd = tc::sdesc_sw128(b_addr + kk * 32, 16, 1024);
                        tc::mma_bf16_ss_pair(d, ad, bd, kIdesc, (kb | kk) != 0 ? 1u : 0u);
                    }
                    tc::mma_commit_pair_both(&bs->empty[s]);
                    ++it;
                }
                if (ok) tc::mma_commit_pair_both(&bs->acc_full[buf]);
            }
            // every issued MMA completes before either CTA may release TMEM or shared memory
            tc::mma_commit_pair(&bs->drain);
            tc::mbar_wait(&bs->drain, 0, kWaitBudget);
        }
        __syncwarp();
    } else {
        // ---------------- epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 ----------------
        const int q = warp & 3;
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        // this warp's staging area: two 64-column boxes of its 32 rows (128 B
        // per row, 128-byte swizzle: 16-byte chunk c of row r at c ^ (r & 7))
        uint8_t *stage = sm + kOffStage + q * kStageWarpBytes;
        const uint32_t srow = tc::smem_u32(stage) + (uint32_t)lane * 128u;
        bool ok = true;
        for (int i = 0; i < my_tiles && ok; ++i) {
            const int t = unit + i * units;
            const int m0 = (t % p.m_tiles) * kTileRows + (int)rank * kBM, n0 = (t / p.m_tiles) * kBN;
            const int buf = i & 1;
            if (!(ok = __all_sync(0xffffffffu, wait_or_abort(&bs->acc_full[buf], (i >> 1) & 1, bs, p.status)))) break;
            tc::tc_fence_after();
            const int row = m0 + q * 32 + lane;
            const int valid = min(kBN, p.V - n0);  // columns inside the vocabulary (a multiple of 8)
            uint32_t best = 0;                     // below every key: the order of -inf is 0x7F
            int best_col = 0;
#pragma unroll 1
            for (int half = 0; half < 2; ++half) {
                uint32_t w[64];
                {
                    float v[128];
                    tc::tmem_ld128(tmem + lane_base + (uint32_t)(buf * kBN + half * 128), v);
                    if (half == 1) {  // the accumulator is in registers: the next tile may use it
                        tc::tc_fence_before();
                        __syncwarp();
                        if (lane == 0) tc::mbar_arrive_cluster(tc::cluster_addr(&bs->acc_empty[buf], 0));
                    }
                    if (p.scale == 1.0f) {  // uniform: bf16_rn(1 * x) is bf16_rn(x)
#pragma unroll
                        for (int e = 0; e < 64; ++e) w[e] = tc::cvt_bf16x2(v[2 * e], v[2 * e + 1]);
                    } else {  // two products per instruction, each rounded to nearest
#pragma unroll
                        for (int e = 0; e < 64; ++e) {
                            const float2 sv = tc::fmul2(make_float2(v[2 * e], v[2 * e + 1]), make_float2(p.scale, p.scale));
                            w[e] = tc::cvt_bf16x2(sv.x, sv.y);
                        }
                    }
                }
                // the previous stores from the staging area have read it
                if (lane == 0) tc::bulk_wait_read_all();
                __syncwarp();
#pragma unroll
                for (int b = 0; b < 2; ++b)
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const uint32_t wv[4] = {w[32 * b + 4 * c], w[32 * b + 4 * c + 1], w[32 * b + 4 * c + 2],
                                                w[32 * b + 4 * c + 3]};
                        tc::st_shared_v4(srow + (uint32_t)b * kBoxBytes + (((uint32_t)c ^ (uint32_t)(lane & 7)) << 4), wv);
                    }
                tc::fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {  // clipped at the vocabulary and the last row
                    tc::tma_store_2d(&tc_out, stage, n0 + half * 128, m0 + q * 32);
                    tc::tma_store_2d(&tc_out, stage + kBoxBytes, n0 + half * 128 + 64, m0 + q * 32);
                    tc::bulk_commit_group();
                }
                if (p.keys && half * 128 < valid) lm_half_key(w, half * 128, valid, best, best_col);
            }
            if (p.keys && row < p.rows && valid > 0) {
                const int pos = (n0 % A11S_CHUNK) + best_col;
                const unsigned long long key = ((unsigned long long)best << 32) | (0xFFFFFFFFu - (uint32_t)pos);
                atomicMax(p.keys + (size_t)row * p.nch + n0 / A11S_CHUNK, key);
            }
        }
        if (lane == 0) tc::bulk_wait_all();
        __syncwarp();
    }
    // After a timeout copies may still be landing here, and their completion
    // is counted on the even CTA's barrier: give them time (about 0.2 ms)
    // before the shared memory is released.
    if (threadIdx.x == 0 && aborted(bs)) {
        const long long t0 = clock64();
        while (clock64() - t0 < 400000) {
        }
    }
    tc::tc_fence_before();
    tc::cluster_sync();  // the pair's MMAs and remote arrivals are over
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc_pair(tmem, kTmemCols);
    }
}

// ---------------------------------------------------------------------------- host side
namespace {
PFN_cuTensorMapEncodeTiled_v12000 lm_encode_fn() {
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

// 2-D bf16 [outer][inner] row-major (row pitch `pitch` elements, default
// inner), box 64 x box_rows, 128-byte swizzle.
bool encode_rows(CUtensorMap *map, const void *base, int64_t inner, int64_t outer, uint32_t box_rows,
                 int64_t pitch = 0) {
    auto fn = lm_encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    const cuuint64_t str[1] = {(cuuint64_t)(pitch > 0 ? pitch : inner) * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, str, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Clusters of two that can be resident at once (one CTA per SM).
int lm_pair_slots(const cudaLaunchConfig_t &cfg, int sms) {
    static int n = 0;
    if (!n) {
        int c = 0;
        n = cudaOccupancyMaxActiveClusters(&c, lm_head_tc, &cfg) == cudaSuccess && c > 0 ? c : sms / 2;
    }
    return n;
}
}  // namespace

cudaError_t launch_lm_head(const LmHeadArgs &a, cudaStream_t s) {
    CUtensorMap ta, tb;
    if (!encode_rows(&ta, a.hidden, a.K, a.rows, kBM)) return cudaErrorInvalidValue;
    if (!encode_rows(&tb, a.weight, a.K, a.V, kBRows)) return cudaErrorInvalidValue;
    CUtensorMap to;  // logits [rows][V] with row pitch ldl: 64 x 32 boxes, 128-byte swizzle
    if (!encode_rows(&to, a.logits, a.V, a.rows, 32, a.ldl)) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(lm_head_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    LmParams p{};
    p.logits = reinterpret_cast<__nv_bfloat16 *>(a.logits);
    p.ldl = a.ldl;
    p.keys = a.keys;
    p.scale = a.scale;
    p.rows = a.rows;
    p.V = a.V;
    p.nch = (a.V + A11S_CHUNK - 1) / A11S_CHUNK;
    p.m_tiles = (a.rows + kTileRows - 1) / kTileRows;
    p.n_tiles = (a.V + kBN - 1) / kBN;
    p.k_blocks = (int32_t)((a.K + kBK - 1) / kBK);
    p.status = a.status;
    if (a.keys) {
        e = cudaMemsetAsync(a.keys, 0, (size_t)a.rows * p.nch * sizeof(unsigned long long), s);
        if (e != cudaSuccess) return e;
    }
    int sms = 148, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // persistent: one CTA pair per two SMs (clusters of 2), at most one pair per tile
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * (sms / 2));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const long long pairs = std::min<long long>((long long)p.m_tiles * p.n_tiles, lm_pair_slots(cfg, sms));
    cfg.gridDim = dim3((unsigned)(2 * pairs));
    return cudaLaunchKernelEx(&cfg, lm_head_tc, ta, tb, to, p);
}


}  // namespace a11s
