// Prefill GEMM on CTA pairs (cta_group::2):  Y = X . dequant(W).  (With a
// LoRA term the runtime uses the single-CTA kernel, whose LoRA stages share
// its accumulator.)
//
// Same computation as q4_gemm.cu (the reference's q4gemm.comp:61-175 with
// w = float(v) * scale, q4gemm.comp:116-122), for large problems.  A cluster
// of two CTAs on two SMs owns a 256 x 256 output tile:
//
//   * each CTA TMA-loads its own 128 rows of the 16-bit X tile per 128-wide
//     k-stage (counted on the leader CTA's barrier) and, from a separate warp
//     and ring, the packed words of its own 128 weight columns; its dequant
//     warps turn those into the 16-bit B operand in its own shared memory
//     and arrive on the leader's barrier;
//   * the leader issues tcgen05.mma.cta_group::2 (M=256, N=256, K=16): A rows
//     and B columns are split between the two CTAs' shared memory at the
//     same offsets, each CTA's TMEM receives its 128 rows x 256 columns;
//   * one commit per stage arrives on the empty barriers of both CTAs, one per
//     tile on both epilogues' accumulator barriers (a commit costs the MMA
//     thread about as much as four MMAs, so stages are 128 k: 8 MMAs each);
//   * both CTAs run their epilogue on their own TMEM (double-buffered: 2 x 256
//     columns) while the pair computes the next tile; each epilogue warp
//     stages 32 rows x 16 columns of Y in shared memory and writes them with
//     a TMA bulk store, so the epilogue costs the main loop almost nothing.
//
// A stage is two 64-k sub-blocks in the canonical 128-byte-swizzled K-major
// layout (16 KB each for X and for the dequantised W).  The packed W ring
// (128 columns x 64 B per stage, 64-byte swizzled) is released as soon as the
// dequant warps have read a stage, not when the MMA has consumed it, so the
// next stage's words are already resident when its operand buffer frees up.
// The dequant warps' 16-byte loads (8 columns per quarter-warp) and 16-byte
// stores into the 128-byte-swizzled operand are free of bank conflicts.  The
// scales come from global memory two stages ahead; each prefetch is issued
// right after the warp's arrive, so the arrive's release does not wait for it.
//
// Per SM and 128-k stage this moves 40 KB from L2 (32 KB X + 8 KB W) for
// 128 x 256 x 128 MACs: half the bytes per FLOP of the single-CTA 256 x 128
// tile, and each dequantised weight still feeds 256 rows.  Every load lands
// only in the CTA that issued it.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "common.cuh"
#include "q4_dequant.cuh"
#include "q4_kernels.h"

namespace q4 {

namespace {

constexpr int kPairRows = 256;  // tile rows of the pair (128 per CTA)
constexpr int kPairCols = 256;  // tile columns (128 dequantised per CTA)
constexpr int kHalf = 128;
constexpr int kBK = 128;        // k per stage (two 64-k sub-blocks)
constexpr int kSub = 64;
constexpr int kStages = 3;      // X / operand stages
constexpr int kRawStages = 3;   // packed-W stages
constexpr int kThreads = 480;   // 15 warps
constexpr int kDequantWarps = 8;
constexpr int kEpiWarp0 = 10;
constexpr int kEpiWarps = 4;
constexpr int kRawWarp = 14;
constexpr int kYCols = 16;      // columns of Y per staged block (one tcgen05.ld.x16)

struct PCfg {
    static constexpr int kSubBytes = kHalf * kSub * 2;  // 16 KB: one 64-k sub-block of 128 rows
    static constexpr int kABytes = 2 * kSubBytes;       // 32 KB: this CTA's 128 rows of X
    static constexpr int kBBytes = 2 * kSubBytes;       // 32 KB: this CTA's 128 dequantised columns
    static constexpr int kRBytes = kHalf * kBK / 2;     // 8 KB: their packed nibbles (64 B per column)
    static constexpr int kYBytes = 32 * kYCols * 4;     // 2 KB: 32 rows x 16 columns of Y, 64-byte swizzled
    static constexpr int kAOff = 0;
    static constexpr int kBOff = kAOff + kStages * kABytes;
    static constexpr int kROff = kBOff + kStages * kBBytes;
    static constexpr int kYOff = kROff + kRawStages * kRBytes;
    static constexpr int kBarOff = kYOff + kEpiWarps * kYBytes;
    // full_a[S] (leader), full_b[S] (leader), empty[S] (both), full_r[R],
    // empty_r[R] (local), acc_full[2] (both), acc_empty[2] (leader), done (leader)
    static constexpr int kNumBars = 3 * kStages + 2 * kRawStages + 5;
    static constexpr int kMiscOff = kBarOff + kNumBars * 8;
    static constexpr int kBytes = kMiscOff + 16;
    static constexpr int kSmemAlloc = kBytes + 1024;
    static constexpr int kTmemCols = 2 * kPairCols;  // 512
    static_assert(kSmemAlloc <= 232448, "shared memory budget");
};

template <typename T16>
__global__ void __launch_bounds__(kThreads, 1)
    q4_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                        const __grid_constant__ CUtensorMap tmap_y, const float* __restrict__ scales,
                        const int* __restrict__ col_exp, const int* __restrict__ row_exp, int M, int N, int K,
                        int* __restrict__ status) {
    using C = PCfg;
    constexpr int ST = kStages;
    constexpr int RT = kRawStages;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = smem_u32(smem_raw);
    const uint32_t base = (raw_base + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw_base);

    const uint32_t a_s = base + C::kAOff;
    const uint32_t b_s = base + C::kBOff;
    const uint32_t r_s = base + C::kROff;
    const uint32_t bar = base + C::kBarOff;
    auto full_a = [&](int s) { return bar + 8u * s; };
    auto full_b = [&](int s) { return bar + 8u * (ST + s); };
    auto empty = [&](int s) { return bar + 8u * (2 * ST + s); };
    auto full_r = [&](int r) { return bar + 8u * (3 * ST + r); };
    auto empty_r = [&](int r) { return bar + 8u * (3 * ST + RT + r); };
    auto acc_full = [&](int b) { return bar + 8u * (3 * ST + 2 * RT + b); };
    auto acc_empty = [&](int b) { return bar + 8u * (3 * ST + 2 * RT + 2 + b); };
    const uint32_t done_bar = bar + 8u * (3 * ST + 2 * RT + 4);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::kMiscOff);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kMiscOff + 4);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t crank = cluster_ctarank();
    const bool leader = crank == 0;
    const int pair = static_cast<int>(blockIdx.x >> 1);
    const int npairs = static_cast<int>(gridDim.x >> 1);
    const int MT = (M + kPairRows - 1) / kPairRows;
    const int NT = (N + kPairCols - 1) / kPairCols;
    const int tiles = MT * NT;
    const int KT = (K + kBK - 1) / kBK;
    const int G = K / 32;
    auto leader_addr = [&](uint32_t a) { return mapa_shared(a, 0); };

    if (tid == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(full_a(s), 1);                  // leader's expect_tx (both CTAs' bytes)
            mbar_init(full_b(s), 2 * kDequantWarps);  // dequant warps of both CTAs
            mbar_init(empty(s), 1);                   // the leader's multicast commit
        }
        for (int r = 0; r < RT; ++r) {
            mbar_init(full_r(r), 1);                  // own expect_tx
            mbar_init(empty_r(r), kDequantWarps);     // own dequant warps
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(acc_full(b), 1);                // the leader's multicast commit
            mbar_init(acc_empty(b), 2 * kEpiWarps);   // epilogue warps of both CTAs
        }
        mbar_init(done_bar, 1);
        *abort_flag = 0;
        fence_mbarrier_init();
        tma_prefetch_desc(&tmap_x);
        tma_prefetch_desc(&tmap_w);
        tma_prefetch_desc(&tmap_y);
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(tmem_holder), C::kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before_sync();
    cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated
    tc_fence_after_sync();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {
        // ---------------------------------------------------- X producer --
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            pdl_wait();  // X16 is written by the previous launch (the cast)
            for (int t = pair; t < tiles && ok; t += npairs) {
                const int m0 = (t % MT) * kPairRows + static_cast<int>(crank) * kHalf;
                for (int kt = 0; kt < KT; ++kt, ++it) {
                    const int s = it % ST;
                    const uint32_t ph = (it / ST) & 1u;
                    if (!mbar_wait(empty(s), ph ^ 1u, abort_flag, status, kStatusTimeoutProducer)) {
                        ok = false;
                        break;
                    }
                    if (leader) mbar_arrive_expect_tx(full_a(s), 2u * C::kABytes);
                    const uint32_t fa = leader_addr(full_a(s));
                    tma_load_2d_pair(a_s + s * C::kABytes, &tmap_x, fa, kt * kBK, m0);
                    tma_load_2d_pair(a_s + s * C::kABytes + C::kSubBytes, &tmap_x, fa, kt * kBK + kSub, m0);
                }
            }
            if (*abort_flag && leader)  // let the copies in flight land before exit
                for (int j = (it > ST ? it - ST : 0); j < it; ++j) mbar_drain(full_a(j % ST), (j / ST) & 1u);
        }
    } else if (warp == kRawWarp) {
        // ------------------------------------------- packed-W producer --
        // The packed weights do not depend on the previous launch: no wait.
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int t = pair; t < tiles && ok; t += npairs) {
                const int nb = (t / MT) * kPairCols + static_cast<int>(crank) * kHalf;
                for (int kt = 0; kt < KT; ++kt, ++it) {
                    const int r = it % RT;
                    const uint32_t ph = (it / RT) & 1u;
                    if (!mbar_wait(empty_r(r), ph ^ 1u, abort_flag, status, kStatusTimeoutProducer)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(full_r(r), C::kRBytes);
                    tma_load_2d(r_s + r * C::kRBytes, &tmap_w, full_r(r), kt * (kBK / 8), nb);
                }
            }
            if (*abort_flag)
                for (int j = (it > RT ? it - RT : 0); j < it; ++j) mbar_drain(full_r(j % RT), (j / RT) & 1u);
        }
    } else if (warp == 1) {
        // ------------------------------------------- MMA (leader CTA only) --
        if (leader && elect_one()) {
            const uint32_t idesc = umma_idesc_f16(std::is_same<T16, __half>::value ? 0u : 1u,
                                                  static_cast<uint32_t>(kPairRows), static_cast<uint32_t>(kPairCols));
            int it = 0, i = 0;
            bool ok = true;
            for (int t = pair; t < tiles && ok; t += npairs, ++i) {
                const int b = i & 1;
                const uint32_t u = static_cast<uint32_t>(i >> 1);
                if (!mbar_wait(acc_empty(b), (u & 1u) ^ 1u, abort_flag, status, kStatusTimeoutMma)) break;
                tc_fence_after_sync();
                const uint32_t d0 = tmem_base + static_cast<uint32_t>(b * kPairCols);
                for (int kt = 0; kt < KT; ++kt, ++it) {
                    const int s = it % ST;
                    const uint32_t ph = (it / ST) & 1u;
                    if (!mbar_wait(full_a(s), ph, abort_flag, status, kStatusTimeoutMma) ||
                        !mbar_wait(full_b(s), ph, abort_flag, status, kStatusTimeoutMma)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after_sync();
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk) {
                        const uint32_t off = static_cast<uint32_t>((kk >> 2) * C::kSubBytes + (kk & 3) * 32);
                        const uint64_t ad = umma_desc_k_sw128(a_s + s * C::kABytes + off);
                        const uint64_t bd = umma_desc_k_sw128(b_s + s * C::kBBytes + off);
                        umma_f16_ss_pair(d0, ad, bd, idesc, (kt | kk) != 0 ? 1u : 0u);
                    }
                    umma_commit_pair_both(empty(s), 0x3);
                }
                if (ok) umma_commit_pair_both(acc_full(b), 0x3);
            }
            umma_commit_pair(mapa_shared(done_bar, 0));  // tracks every MMA issued above
            mbar_drain(done_bar, 0u);
        }
    } else if (warp < kEpiWarp0) {
        // ------------------------------------------------------- dequant --
        // Lane l of dequant warp w: column nl = 16 w + (l & 15) of this CTA's
        // half, k-half hh = l >> 4 of each stage (groups 4 kt + 2 hh and
        // 4 kt + 2 hh + 1, operand sub-block hh).  A quarter-warp then covers 8
        // columns of one k-half: its 16-byte packed loads hit 8 distinct bank
        // groups through the 64-byte swizzle, its stores through the 128-byte
        // one.
        const int dw = warp - 2;
        const int nl = dw * 16 + (lane & 15), hh = lane >> 4;
        const int rsw = (nl >> 1) & 3;  // 64-byte swizzle key of packed row nl
        int it = 0;
        bool ok = true;
        for (int t = pair; t < tiles && ok; t += npairs) {
            const int n = (t / MT) * kPairCols + static_cast<int>(crank) * kHalf + nl;
            const bool col_ok = n < N;
            const float cs = (col_exp != nullptr && col_ok) ? exp2i(__ldg(col_exp + n)) : 1.0f;
            const float* srow = scales + static_cast<size_t>(col_ok ? n : 0) * G;
            auto scale_at = [&](int kt, int pq) {
                const int g = kt * 4 + hh * 2 + pq;
                return (col_ok && g < G) ? __ldg(srow + g) : 0.0f;
            };
            float a0 = scale_at(0, 0), b0 = scale_at(0, 1), a1 = scale_at(1, 0), b1 = scale_at(1, 1);
            for (int kt = 0; kt < KT; ++kt, ++it) {
                const int s = it % ST;
                const uint32_t ph = (it / ST) & 1u;
                const int r = it % RT;
                const uint32_t rph = (it / RT) & 1u;
                const float sc[2] = {a0 * cs, b0 * cs};
                a0 = a1;
                b0 = b1;
                if (!mbar_wait(full_r(r), rph, abort_flag, status, kStatusTimeoutDequant)) {
                    ok = false;
                    break;
                }
                const uint8_t* rrow = smem + C::kROff + r * C::kRBytes + nl * 64;
                const uint4 q[2] = {*reinterpret_cast<const uint4*>(rrow + (((hh * 2) ^ rsw) << 4)),
                                    *reinterpret_cast<const uint4*>(rrow + (((hh * 2 + 1) ^ rsw) << 4))};
                if (!mbar_wait(empty(s), ph ^ 1u, abort_flag, status, kStatusTimeoutDequant)) {
                    ok = false;
                    break;
                }
                uint8_t* brow = smem + C::kBOff + s * C::kBBytes + hh * C::kSubBytes + nl * 128;
#pragma unroll
                for (int pq = 0; pq < 2; ++pq) {
                    const float2 s2v = make_float2(sc[pq], sc[pq]);
                    const __half2 s2h = __float2half2_rn(sc[pq]);
                    const uint32_t words[4] = {q[pq].x, q[pq].y, q[pq].z, q[pq].w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int chunk = (pq * 4 + j) ^ (nl & 7);
                        *reinterpret_cast<uint4*>(brow + chunk * 16) = dequant_f16x2_or<T16>(words[j], s2v, s2h);
                    }
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(empty_r(r));                     // the packed stage has been read
                    mbar_arrive_remote(leader_addr(full_b(s)));  // the operand stage is written
                }
                a1 = scale_at(kt + 2, 0);  // issued after the arrives: their release does not wait for it
                b1 = scale_at(kt + 2, 1);
            }
        }
    } else {
        // ------------------------------------------------------ epilogue --
        // Warp w reads TMEM lane quarter w % 4 = rows 32 (w % 4) .. + 31 of the
        // CTA's half; per 16 columns it scales its row, stages the 32 x 16
        // block in shared memory (64-byte swizzled, conflict-free 16-byte
        // stores) and hands it to a TMA bulk store, which skips the rows and
        // columns outside Y.
        pdl_wait();  // row exponents and Y belong to the previous launch until it completes
        const int quarter = warp & 3;
        const uint32_t ybuf = base + static_cast<uint32_t>(C::kYOff + (warp - kEpiWarp0) * C::kYBytes);
        uint8_t* ybufp = smem + C::kYOff + (warp - kEpiWarp0) * C::kYBytes;
        const int ysw = (lane >> 1) & 3;  // 64-byte swizzle key of staged row `lane`
        int i = 0;
        for (int t = pair; t < tiles; t += npairs, ++i) {
            const int b = i & 1;
            const uint32_t u = static_cast<uint32_t>(i >> 1);
            if (!mbar_wait_warp(acc_full(b), u & 1u, abort_flag, status, kStatusTimeoutEpilogue)) break;
            tc_fence_after_sync();
            const int m0 = (t % MT) * kPairRows + static_cast<int>(crank) * kHalf + quarter * 32;
            const int n0 = (t / MT) * kPairCols;
            // 2^-col_exp of the tile's 256 columns: lane l holds 8l .. 8l+7.
            float cf[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int n = n0 + lane * 8 + j;
                cf[j] = (col_exp != nullptr && n < N) ? exp2i(-col_exp[n]) : 1.0f;
            }
            const int row = m0 + lane;
            const float rs = (row_exp != nullptr && row < M) ? exp2i(-row_exp[row]) : 1.0f;
            const uint32_t tcol =
                tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(b * kPairCols);
#pragma unroll 1
            for (int c = 0; c < kPairCols / kYCols; ++c) {
                uint32_t r[16];
                tmem_ld16(tcol + static_cast<uint32_t>(c * kYCols), r);
                tmem_ld_wait();
                if (c == kPairCols / kYCols - 1) {
                    // the whole accumulator is in registers or staged: release it
                    tc_fence_before_sync();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_remote(leader_addr(acc_empty(b)));
                }
                const int nb = n0 + c * kYCols;
                if (nb >= N || m0 >= M) continue;  // warp-uniform: the block lies outside Y
                float v[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const float cinv = __shfl_sync(0xffffffffu, cf[e & 7], c * 2 + (e >> 3));
                    v[e] = __uint_as_float(r[e]) * rs * cinv;
                }
                if (lane == 0) bulk_wait_group_read<0>();  // the previous block's store has read the buffer
                __syncwarp();
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    *reinterpret_cast<float4*>(ybufp + lane * 64 + ((j ^ ysw) << 4)) =
                        make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&tmap_y, ybuf, nb, m0);
                    bulk_commit_group();
                }
            }
        }
        if (lane == 0) bulk_wait_group_all();  // the stores have read their blocks before the CTA exits
    }

    tc_fence_before_sync();
    cluster_sync_all();  // no CTA leaves while its peer may still use its smem or TMEM
    if (warp == 1) {
        tc_fence_after_sync();
        tmem_dealloc_pair(tmem_base, C::kTmemCols);
    }
}

template <typename T16>
int launch_pair_t(const GemmArgs& a, int pairs, cudaStream_t stream) {
    auto kern = q4_gemm_pair_kernel<T16>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PCfg::kSmemAlloc);
    if (e != cudaSuccess) return static_cast<int>(e);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = PCfg::kSmemAlloc;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // overlap the X cast's tail
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    e = cudaLaunchKernelEx(&cfg, kern, a.tmap_x16, a.tmap_w, a.tmap_y, a.scales, a.col_exp, a.row_exp, a.M, a.N,
                           a.K, a.status);
    return static_cast<int>(e);
}

template <typename T16>
int max_pairs_t() {
    auto kern = q4_gemm_pair_kernel<T16>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PCfg::kSmemAlloc) != cudaSuccess)
        return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = PCfg::kSmemAlloc;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) return 0;
    return n;
}

}  // namespace

int gemm_pair_tiles(int M, int N) {
    return ((M + kPairRows - 1) / kPairRows) * ((N + kPairCols - 1) / kPairCols);
}

int gemm_pair_max_active(Operand16 op) { return op == Operand16::kF16 ? max_pairs_t<__half>() : max_pairs_t<__nv_bfloat16>(); }

int launch_gemm_pair(const GemmArgs& a, int max_pairs, cudaStream_t stream) {
    const int tiles = gemm_pair_tiles(a.M, a.N);
    const int pairs = tiles < max_pairs ? tiles : max_pairs;
    if (pairs < 1) return static_cast<int>(cudaErrorInvalidValue);
    return a.op == Operand16::kF16 ? launch_pair_t<__half>(a, pairs, stream)
                                   : launch_pair_t<__nv_bfloat16>(a, pairs, stream);
}

}  // namespace q4
