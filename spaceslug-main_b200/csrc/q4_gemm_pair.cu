// Prefill GEMM on CTA pairs (cta_group::2):  Y = X . dequant(W) (+ LoRA).
//
// Same computation as q4_gemm.cu (the reference's q4gemm.comp:61-175 with
// w = float(v) * scale, q4gemm.comp:116-122), for large problems.  A cluster
// of two CTAs on two SMs owns a tile of 256 weight columns x 256 rows of X,
// and computes it transposed, D = W^T X^T:
//
//   * the dequantised weights are the MMA's A operand and live in tensor
//     memory: each CTA's dequant warps read the packed words and scales of
//     its own 128 columns from shared memory (both TMA-loaded, the words
//     64-byte swizzled), dequantise them in registers and write them with
//     tcgen05.st into one of four A slots (64 columns = 128 k per slot),
//     arriving on the leader's barrier.  A dequant warp has no global load
//     in flight when it arrives, so the arrive's release costs little;
//   * X is the B operand: each CTA TMA-loads its own 128 rows of the 16-bit
//     X tile per 128-k stage (two 64-k sub-blocks in the 128-byte-swizzled
//     K-major layout), counted on the leader's barrier;
//   * the leader issues tcgen05.mma.cta_group::2 (M=256, N=256, K=16) with A
//     from both CTAs' tensor memory and B from both CTAs' shared memory;
//     one multicast commit per stage releases the X stage and the A slot in
//     both CTAs, one per tile hands the accumulator to both epilogues;
//   * the accumulator (256 columns: one per row of X, lanes = weight columns)
//     leaves tensor memory 32 columns at a time: each of the 8 epilogue warps
//     (two per lane quarter, four blocks each) scales a 32 x 32 block, stages
//     it in shared memory (row = one row of Y, 128 bytes) and writes it with
//     a TMA bulk store.
//   * split K: with ksplit = 2 a work unit is (tile, half of K), so a problem
//     with too few tiles for one wave still fills the pairs.  Each unit
//     reduce-adds its block into a zeroed Y (TMA bulk reduce .add.f32); two
//     addends onto zero give the same sum in either order, so the result is
//     deterministic.
//   * LoRA: the epilogue adds (alpha/r) * sum_r T[m][r] B[r][n] in fp32 (T =
//     X*A from the projection kernel) to each staged block before it leaves;
//     with ksplit = 2 each K half adds half of the ranks.
//   * peer push (N-sharded layers, ksplit = 1): after the TMA stores of a
//     tile into this GPU's Y have completed (and the accumulator has gone
//     back to the MMA), each epilogue warp reads its blocks back from Y (L2)
//     and stores them to the same rows and columns of up to 7 peers' Y
//     (plain 16-byte stores through NVLink peer mappings), so the exchange
//     of Y runs tile by tile beside the next tile's main loop; only the
//     epilogue warps wait for the link.
//
// Shared memory per SM and stage carries 32 KB of X written by TMA and read
// by the MMA plus 10 KB of packed W and scales in and out: about 84 B/clk at
// the tensor peak, against 144 B/clk when the dequantised weights also pass through
// shared memory.  Tensor memory holds the accumulator (256 columns) and the
// four A slots (4 x 64 columns); the accumulator is single-buffered, so the
// MMA of a tile starts once both epilogues have read the previous one out,
// while the dequant warps and the loads run ahead.
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

constexpr int kPairRows = 256;  // rows of X per tile (128 per CTA) = accumulator columns
constexpr int kPairCols = 256;  // weight columns per tile (128 per CTA) = accumulator lanes of the pair
constexpr int kHalf = 128;
constexpr int kBK = 128;        // k per stage
constexpr int kSub = 64;        // k per 128-byte-swizzled sub-block
constexpr int kStages = 4;      // X stages in shared memory = A slots in tensor memory
constexpr int kRawStages = 6;   // packed-W + scale stages in shared memory
constexpr int kThreads = 608;   // 19 warps
constexpr int kDequantWarp0 = 2;
constexpr int kDequantWarps = 8;
constexpr int kEpiWarp0 = 10;
constexpr int kEpiWarps = 8;     // two per tensor-memory lane quarter
constexpr int kEpiChunks = 4;    // 32-column blocks of the accumulator per epilogue warp
constexpr int kRawWarp = 18;

struct PCfg {
    static constexpr int kSubBytes = kHalf * kSub * 2;  // 16 KB: one 64-k sub-block of 128 rows of X
    static constexpr int kXBytes = 2 * kSubBytes;       // 32 KB per stage
    static constexpr int kWBytes = kHalf * kBK / 2;     // 8 KB: 128 columns x 64 B of packed W
    static constexpr int kSBytes = kHalf * (kBK / 32) * 4;  // 2 KB: their 4 scales each
    static constexpr int kRBytes = kWBytes + kSBytes;   // one packed stage
    static constexpr int kYBufBytes = 32 * 32 * 4;      // 4 KB: one 32 x 32 fp32 block of Y
    static constexpr int kXOff = 0;
    static constexpr int kROff = kXOff + kStages * kXBytes;
    static constexpr int kYOff = kROff + kRawStages * kRBytes;
    static constexpr int kBarOff = kYOff + kEpiWarps * kYBufBytes;
    // full_x[S] (leader), full_w[S] (leader), empty[S] (both), full_r[R],
    // empty_r[R] (local), acc_full (both), acc_empty (leader), done (leader)
    static constexpr int kNumBars = 3 * kStages + 2 * kRawStages + 3;
    static constexpr int kMiscOff = kBarOff + kNumBars * 8;
    static constexpr int kBytes = kMiscOff + 16;
    static constexpr int kSmemAlloc = kBytes + 1024;
    static constexpr int kTmemCols = 512;
    static constexpr int kAccCols = kPairRows;  // accumulator: tensor-memory columns [0, 256)
    static constexpr int kSlotCols = kBK / 2;   // A slot: 64 columns of f16 pairs
    static_assert(kAccCols + kStages * kSlotCols <= kTmemCols, "tensor memory budget");
    static_assert(kSmemAlloc <= 232448, "shared memory budget");
};

template <typename T16>
__global__ void __launch_bounds__(kThreads, 1)
    q4_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                        const __grid_constant__ CUtensorMap tmap_s, const __grid_constant__ CUtensorMap tmap_y,
                        const int* __restrict__ col_exp,
                        const int* __restrict__ row_exp, int M, int N, int K, int ksplit,
                        const float* __restrict__ lora_t, const float* __restrict__ lora_b, int rank,
                        float lora_scale, PeerPtrs peers, int npeers, long long ld_y, const float* y_local,
                        int* __restrict__ status) {
    using C = PCfg;
    constexpr int ST = kStages;
    constexpr int RT = kRawStages;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = smem_u32(smem_raw);
    const uint32_t base = (raw_base + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw_base);

    const uint32_t x_s = base + C::kXOff;
    const uint32_t r_s = base + C::kROff;
    const uint32_t bar = base + C::kBarOff;
    auto full_x = [&](int s) { return bar + 8u * s; };
    auto full_w = [&](int s) { return bar + 8u * (ST + s); };
    auto empty = [&](int s) { return bar + 8u * (2 * ST + s); };
    auto full_r = [&](int r) { return bar + 8u * (3 * ST + r); };
    auto empty_r = [&](int r) { return bar + 8u * (3 * ST + RT + r); };
    const uint32_t acc_full = bar + 8u * (3 * ST + 2 * RT);
    const uint32_t acc_empty = acc_full + 8u;
    const uint32_t done_bar = acc_full + 16u;
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
    const int units = tiles * ksplit;           // unit u: tile u / ksplit, K part u % ksplit
    const int KT = (K + kBK - 1) / kBK / ksplit;  // k-stages per unit (the host keeps this exact)
    auto leader_addr = [&](uint32_t a) { return mapa_shared(a, 0); };

    if (tid == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(full_x(s), 1);                  // leader's expect_tx (both CTAs' bytes)
            mbar_init(full_w(s), 2 * kDequantWarps);  // dequant warps of both CTAs
            mbar_init(empty(s), 1);                   // the leader's multicast commit
        }
        for (int r = 0; r < RT; ++r) {
            mbar_init(full_r(r), 1);                  // own expect_tx
            mbar_init(empty_r(r), kDequantWarps);     // own dequant warps
        }
        mbar_init(acc_full, 1);                       // the leader's multicast commit
        mbar_init(acc_empty, 2 * kEpiWarps);          // epilogue warps of both CTAs
        mbar_init(done_bar, 1);
        *abort_flag = 0;
        fence_mbarrier_init();
        tma_prefetch_desc(&tmap_x);
        tma_prefetch_desc(&tmap_w);
        tma_prefetch_desc(&tmap_s);
        tma_prefetch_desc(&tmap_y);
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(tmem_holder), C::kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before_sync();
    cluster_sync_all();  // both CTAs' barriers initialised and tensor memory allocated
    tc_fence_after_sync();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {
        // ---------------------------------------------------- X producer --
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            pdl_wait();  // X16 is written by the previous launch (the cast)
            const uint64_t keep = l2_policy_evict_last();  // every X tile is read by all column tiles
            for (int u = pair; u < units && ok; u += npairs) {
                const int t = u / ksplit, k0 = (u % ksplit) * KT * kBK;
                const int m0 = (t % MT) * kPairRows + static_cast<int>(crank) * kHalf;
                for (int kt = 0; kt < KT; ++kt, ++it) {
                    const int s = it % ST;
                    const uint32_t ph = (it / ST) & 1u;
                    if (!mbar_wait(empty(s), ph ^ 1u, abort_flag, status, kStatusTimeoutProducer)) {
                        ok = false;
                        break;
                    }
                    if (leader) mbar_arrive_expect_tx(full_x(s), 2u * C::kXBytes);
                    const uint32_t fx = leader_addr(full_x(s));
                    tma_load_2d_pair_hint(x_s + s * C::kXBytes, &tmap_x, fx, k0 + kt * kBK, m0, keep);
                    tma_load_2d_pair_hint(x_s + s * C::kXBytes + C::kSubBytes, &tmap_x, fx, k0 + kt * kBK + kSub, m0,
                                          keep);
                }
            }
            if (*abort_flag && leader)  // let the copies in flight land before exit
                for (int j = (it > ST ? it - ST : 0); j < it; ++j) mbar_drain(full_x(j % ST), (j / ST) & 1u);
        }
    } else if (warp == kRawWarp) {
        // ------------------------------------------- packed-W producer --
        // The packed weights do not depend on the previous launch: no wait.
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            const uint64_t keep = l2_policy_evict_last();  // every weight tile is read by all row tiles
            for (int u = pair; u < units && ok; u += npairs) {
                const int t = u / ksplit, kb = (u % ksplit) * KT;  // first k-stage of the unit
                const int nb = (t / MT) * kPairCols + static_cast<int>(crank) * kHalf;
                for (int kt = 0; kt < KT; ++kt, ++it) {
                    const int r = it % RT;
                    const uint32_t ph = (it / RT) & 1u;
                    if (!mbar_wait(empty_r(r), ph ^ 1u, abort_flag, status, kStatusTimeoutProducer)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(full_r(r), C::kRBytes);
                    tma_load_2d_hint(r_s + r * C::kRBytes, &tmap_w, full_r(r), (kb + kt) * (kBK / 8), nb, keep);
                    tma_load_2d_hint(r_s + r * C::kRBytes + C::kWBytes, &tmap_s, full_r(r), (kb + kt) * (kBK / 32), nb,
                                     keep);
                }
            }
            if (*abort_flag)
                for (int j = (it > RT ? it - RT : 0); j < it; ++j) mbar_drain(full_r(j % RT), (j / RT) & 1u);
        }
    } else if (warp == 1) {
        // ------------------------------------------- MMA (leader CTA only) --
        if (leader && elect_one()) {
            const uint32_t idesc = umma_idesc_f16(std::is_same<T16, __half>::value ? 0u : 1u,
                                                  static_cast<uint32_t>(kPairCols), static_cast<uint32_t>(kPairRows));
            int it = 0, i = 0;
            bool ok = true;
            for (int u = pair; u < units && ok; u += npairs, ++i) {
                if (!mbar_wait(acc_empty, (static_cast<uint32_t>(i) & 1u) ^ 1u, abort_flag, status, kStatusTimeoutMma))
                    break;
                tc_fence_after_sync();
                for (int kt = 0; kt < KT; ++kt, ++it) {
                    const int s = it % ST;
                    const uint32_t ph = (it / ST) & 1u;
                    if (!mbar_wait(full_x(s), ph, abort_flag, status, kStatusTimeoutMma) ||
                        !mbar_wait(full_w(s), ph, abort_flag, status, kStatusTimeoutMma)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after_sync();
                    const uint32_t a_slot = tmem_base + static_cast<uint32_t>(C::kAccCols + s * C::kSlotCols);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk) {
                        const uint32_t off = static_cast<uint32_t>((kk >> 2) * C::kSubBytes + (kk & 3) * 32);
                        const uint64_t bd = umma_desc_k_sw128(x_s + s * C::kXBytes + off);
                        umma_f16_ts_pair(tmem_base, a_slot + static_cast<uint32_t>(kk * 8), bd, idesc,
                                         (kt | kk) != 0 ? 1u : 0u);
                    }
                    umma_commit_pair_both(empty(s), 0x3);
                }
                if (ok) umma_commit_pair_both(acc_full, 0x3);
            }
            umma_commit_pair(mapa_shared(done_bar, 0));  // tracks every MMA issued above
            mbar_drain(done_bar, 0u);
        }
    } else if (warp < kEpiWarp0) {
        // ------------------------------------------------------- dequant --
        // Warp w covers the tensor-memory lane quarter w % 4 (the only one it
        // may access): lane l <-> column nl = 32 (w % 4) + l of this CTA's
        // half, and k-half (w - 2) / 4 of each stage (groups 4 kt + 2 hh and
        // 4 kt + 2 hh + 1).  Its two 16-byte loads per stage (8 columns per
        // quarter-warp) hit 8 distinct bank groups through the 64-byte swizzle.
        const int dw = warp - kDequantWarp0;
        const int quarter = warp & 3;
        const int hh = dw >> 2;
        const int nl = quarter * 32 + lane;
        const int rsw = (nl >> 1) & 3;  // 64-byte swizzle key of packed row nl
        const uint32_t t_lane = static_cast<uint32_t>(quarter * 32) << 16;
        int it = 0;
        bool ok = true;
        for (int u = pair; u < units && ok; u += npairs) {
            const int t = u / ksplit;
            const int n = (t / MT) * kPairCols + static_cast<int>(crank) * kHalf + nl;
            const float cs = (col_exp != nullptr && n < N) ? exp2i(__ldg(col_exp + n)) : 1.0f;
            for (int kt = 0; kt < KT; ++kt, ++it) {
                const int s = it % ST;
                const uint32_t ph = (it / ST) & 1u;
                const int r = it % RT;
                const uint32_t rph = (it / RT) & 1u;
                if (!mbar_wait(full_r(r), rph, abort_flag, status, kStatusTimeoutDequant)) {
                    ok = false;
                    break;
                }
                // packed row nl (64-byte swizzled) and its scales (the box's
                // rows past N and groups past K/32 arrive as zeros)
                const uint8_t* rrow = smem + C::kROff + r * C::kRBytes + nl * 64;
                const uint4 q[2] = {*reinterpret_cast<const uint4*>(rrow + (((hh * 2) ^ rsw) << 4)),
                                    *reinterpret_cast<const uint4*>(rrow + (((hh * 2 + 1) ^ rsw) << 4))};
                const float2 sg =
                    *reinterpret_cast<const float2*>(smem + C::kROff + r * C::kRBytes + C::kWBytes + nl * 16 + hh * 8);
                const float sc[2] = {sg.x * cs, sg.y * cs};
                uint32_t v[32];  // f16 pairs (k, k+1) of k = 64 hh .. 64 hh + 63
#pragma unroll
                for (int pq = 0; pq < 2; ++pq) {
                    const float2 s2v = make_float2(sc[pq], sc[pq]);
                    __half2 s_hi, s_lo;
                    split_scale_f16(sc[pq], s_hi, s_lo);
                    const uint32_t words[4] = {q[pq].x, q[pq].y, q[pq].z, q[pq].w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint4 d = dequant_f16x2_or<T16>(words[j], s2v, s_hi, s_lo);
                        v[pq * 16 + j * 4 + 0] = d.x;
                        v[pq * 16 + j * 4 + 1] = d.y;
                        v[pq * 16 + j * 4 + 2] = d.z;
                        v[pq * 16 + j * 4 + 3] = d.w;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(empty_r(r));  // the packed stage is consumed
                if (!mbar_wait_warp(empty(s), ph ^ 1u, abort_flag, status, kStatusTimeoutDequant)) {
                    ok = false;
                    break;
                }
                tc_fence_after_sync();
                tmem_st32(tmem_base + t_lane + static_cast<uint32_t>(C::kAccCols + s * C::kSlotCols + hh * 32), v);
                tmem_st_wait();
                tc_fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive_remote(leader_addr(full_w(s)));
            }
        }
    } else {
        // ------------------------------------------------------ epilogue --
        // Warp w reads lane quarter w % 4 of the accumulator, blocks
        // 4 h .. 4 h + 3 (h = (w - 10) / 4) of 32 columns: lane l holds column
        // n of Y for 32 rows per block; each staged row is 32 consecutive
        // columns of one row of Y.
        pdl_wait();  // row exponents and Y belong to the previous launch until it completes
        const int quarter = warp & 3;
        const int c0 = ((warp - kEpiWarp0) >> 2) * kEpiChunks;
        const uint32_t t_lane = static_cast<uint32_t>(quarter * 32) << 16;
        const uint32_t buf = base + static_cast<uint32_t>(C::kYOff + (warp - kEpiWarp0) * C::kYBufBytes);
        float* bufp = reinterpret_cast<float*>(smem + C::kYOff + (warp - kEpiWarp0) * C::kYBufBytes);
        const uint64_t once = l2_policy_evict_first();  // Y is written once: keep X and W resident instead
        int i = 0;
        for (int u = pair; u < units; u += npairs, ++i) {
            if (!mbar_wait_warp(acc_full, static_cast<uint32_t>(i) & 1u, abort_flag, status, kStatusTimeoutEpilogue))
                break;
            tc_fence_after_sync();
            const int t = u / ksplit, kz = u % ksplit;
            const int m0 = (t % MT) * kPairRows;
            const int n = (t / MT) * kPairCols + static_cast<int>(crank) * kHalf + quarter * 32 + lane;
            const float cinv = (col_exp != nullptr && n < N) ? exp2i(-col_exp[n]) : 1.0f;
            const int nx = (t / MT) * kPairCols + static_cast<int>(crank) * kHalf + quarter * 32;  // block's first column
            // LoRA ranks [r_lo, r_hi) of this K part (multiples of 4 when rank is,
            // so the float4 loads of T rows stay aligned and inside the part)
            int rpk = (rank + ksplit - 1) / ksplit;
            if (rank % 4 == 0) rpk = (rpk + 3) / 4 * 4;
            const int r_lo = lora_b != nullptr ? min(rank, kz * rpk) : 0;
            const int r_hi = lora_b != nullptr ? min(rank, r_lo + rpk) : 0;
            const bool t_vec = (rank % 4) == 0 && (reinterpret_cast<uintptr_t>(lora_t) & 15u) == 0;
            uint32_t rv[2][32];
            tmem_ld32(tmem_base + t_lane + static_cast<uint32_t>(c0 * 32), rv[0]);
            tmem_ld_wait_regs(rv[0]);
#pragma unroll
            for (int cc = 0; cc < kEpiChunks; ++cc) {
                const int c = c0 + cc;
                if (cc + 1 < kEpiChunks) {
                    tmem_ld32(tmem_base + t_lane + static_cast<uint32_t>((c + 1) * 32), rv[(cc + 1) & 1]);
                } else {
                    // this warp's blocks are in registers: hand them to the next tile
                    tc_fence_before_sync();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_remote(leader_addr(acc_empty));
                }
                const int mc = m0 + c * 32;
                const int me = mc + lane;
                const float rs_l = (row_exp != nullptr && me < M) ? exp2i(-row_exp[me]) : 1.0f;
                if (lane == 0) bulk_wait_group_read<0>();  // the previous block's store has read the buffer
                __syncwarp();
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    const float rs = __shfl_sync(0xffffffffu, rs_l, e);
                    bufp[e * 32 + lane] = __uint_as_float(rv[cc & 1][e]) * rs * cinv;
                }
                for (int r0 = r_lo; r0 < r_hi; r0 += 8) {
                    // bufp[e][lane] += sum_{r in [r0, r0 + rc)} T[mc + e][r] * (alpha/r) B[r][n]:
                    // lane e loads row mc + e of T (all loads of the block in flight
                    // together), the rows reach the other lanes by shuffles.
                    const int rc = min(8, r_hi - r0);
                    float bv[8], tv[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        bv[j] = (j < rc && n < N) ? __ldg(lora_b + static_cast<size_t>(r0 + j) * N + n) * lora_scale : 0.0f;
                    const float* trow = lora_t + static_cast<size_t>(me < M ? me : 0) * rank + r0;
                    if (t_vec) {  // rc is a multiple of 4 here
#pragma unroll
                        for (int j = 0; j < 8; j += 4) {
                            const float4 v4 = (j + 4 <= rc && me < M) ? __ldg(reinterpret_cast<const float4*>(trow + j))
                                                                      : make_float4(0.f, 0.f, 0.f, 0.f);
                            tv[j] = v4.x; tv[j + 1] = v4.y; tv[j + 2] = v4.z; tv[j + 3] = v4.w;
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 8; ++j) tv[j] = (j < rc && me < M) ? __ldg(trow + j) : 0.0f;
                    }
#pragma unroll 2
                    for (int e = 0; e < 32; ++e) {
                        float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
                        for (int j = 0; j < 8; j += 2)
                            acc = __ffma2_rn(make_float2(__shfl_sync(0xffffffffu, tv[j], e),
                                                         __shfl_sync(0xffffffffu, tv[j + 1], e)),
                                             make_float2(bv[j], bv[j + 1]), acc);
                        bufp[e * 32 + lane] += acc.x + acc.y;
                    }
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0 && mc < M) {
                    if (ksplit > 1) {
                        tma_reduce_add_2d_hint(&tmap_y, buf, nx, mc, once);
                    } else {
                        tma_store_2d_hint(&tmap_y, buf, nx, mc, once);
                    }
                    bulk_commit_group();
                }
                if (cc + 1 < kEpiChunks) tmem_ld_wait_regs(rv[(cc + 1) & 1]);
            }
            if (npeers > 0 && nx < N) {
                // The tile's blocks to every peer, after the accumulator went
                // back to the MMA (the link traffic overlaps the next tile's
                // main loop): once this warp's bulk stores of the tile have
                // completed, the blocks are read back from this GPU's Y (L2)
                // and stored to each peer's Y.  float4 j = lane + 32 i of a
                // block is row j / 8, columns 4 (j % 8) .. +3 (8 lanes write
                // one 128-byte row).
                if (lane == 0) bulk_wait_group_all();
                __syncwarp();
                asm volatile("fence.proxy.async.global;" ::: "memory");  // async-proxy writes before generic reads
#pragma unroll 1
                for (int cc = 0; cc < kEpiChunks; ++cc) {
                    const int mc = m0 + (c0 + cc) * 32;
                    if (mc >= M) break;
#pragma unroll 2
                    for (int i = 0; i < 8; ++i) {
                        const int j = lane + 32 * i, r = j >> 3, c4 = (j & 7) * 4;
                        if (mc + r < M && nx + c4 < N) {
                            const long long at = static_cast<long long>(mc + r) * ld_y + nx + c4;
                            const float4 v = *reinterpret_cast<const float4*>(y_local + at);
#pragma unroll
                            for (int q = 0; q < kMaxPeers; ++q)  // constant indices: no local copy of the array
                                if (q < npeers) *reinterpret_cast<float4*>(peers.p[q] + at) = v;
                        }
                    }
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
    e = cudaLaunchKernelEx(&cfg, kern, a.tmap_x16, a.tmap_w, a.tmap_s, a.tmap_y, a.col_exp, a.row_exp, a.M, a.N,
                           a.K, a.ksplit, a.lora_t, a.lora_b, a.rank, a.lora_scale, a.peers, a.npeers, a.peer_ld,
                           static_cast<const float*>(a.y), a.status);
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
    if (a.ksplit < 1 || a.ksplit > 2 || a.K % (kBK * a.ksplit) != 0) return static_cast<int>(cudaErrorInvalidValue);
    if (a.lora_b != nullptr && (a.lora_t == nullptr || a.rank < 1 || a.rank > 64))
        return static_cast<int>(cudaErrorInvalidValue);
    if (a.npeers < 0 || a.npeers > kMaxPeers || (a.npeers > 0 && (a.ksplit != 1 || a.peer_ld < a.N || a.peer_ld % 4)))
        return static_cast<int>(cudaErrorInvalidValue);
    for (int q = 0; q < a.npeers; ++q)
        if (a.peers.p[q] == nullptr || (reinterpret_cast<uintptr_t>(a.peers.p[q]) & 15u))
            return static_cast<int>(cudaErrorInvalidValue);
    const int units = gemm_pair_tiles(a.M, a.N) * a.ksplit;
    const int pairs = units < max_pairs ? units : max_pairs;
    if (pairs < 1) return static_cast<int>(cudaErrorInvalidValue);
    return a.op == Operand16::kF16 ? launch_pair_t<__half>(a, pairs, stream)
                                   : launch_pair_t<__nv_bfloat16>(a, pairs, stream);
}

}  // namespace q4
