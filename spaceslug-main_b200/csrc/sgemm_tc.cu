// fp32 GEMM on the tcgen05 tensor cores with fp32-level accuracy (3xTF32):
//   C[M x N] = alpha * op(A)[M x K] * op(B)[K x N]
// the product behind spaceslug_sgemm (the reference's vulkan-runtime/src/api/sgemm_api.h:5-9,
// an fp32 GEMM on its GPU) and the LoRA training contractions.
//
// Each fp32 operand x is split once into x_hi = x rounded to TF32 (10
// explicit mantissa bits) and x_lo = x - x_hi (exact in fp32; the MMA keeps
// its top 11 bits), so x = x_hi + x_lo to about 2^-22 relative.  The product
// is accumulated in fp32 in tensor memory as
//   A_lo B_hi + A_hi B_lo + A_hi B_hi
// (the A_lo B_lo term, 2^-22 relative, is dropped): about fp32 accuracy at
// three TF32 MMAs per product, on the tensor pipe instead of the fp32 FMA
// pipe.
//
// Accumulation.  The tensor cores add each MMA's products into the fp32
// accumulator with truncation, so summing all of K there leaves a bias that
// grows with K (measured on B200, N(0,1) data: |error| / max(1, |ref|) of
// 5e-4 at K = 1024 and 7e-3 at K = 8192).  The accumulator is therefore
// double-buffered in tensor memory and restarted every kChunkStages stages
// (32 k): four epilogue warps read each finished chunk (tcgen05.ld) and add
// it to running fp32 sums in registers with round-to-nearest, while the MMAs
// fill the other buffer.  The truncation then only acts within 32-k chunks.
//
// Split pass (split_kernel / split_t_kernel): every operand is written as hi
// and lo planes in K-major layout ([rows][K] with K contiguous), B transposed
// on the way, so the GEMM's operands are always K-major 128-byte-swizzled TMA
// tiles.  GEMM pass (sgemm_tc_kernel<BN>): one CTA per 128 x BN tile of C,
// 8 warps; warp 0 issues TMA loads of the four planes' k-tiles (32 k) into a
// ring of stages, warp 1 allocates tensor memory and issues the MMAs
// (kind::tf32, M = 128, N = BN, K = 8: twelve per stage, one commit per stage
// frees it, one per chunk hands the chunk's buffer to the epilogue), warps
// 4-7 (tensor-memory lane quarters 0-3, one row of C per thread) sum the
// chunks and store C.
// Large problems take sgemm_pair_kernel instead: CTA pairs (cta_group::2) on
// 256 x 256 tiles of C, where each CTA loads half of the A and half of the B
// rows and the leader's M = 256, N = 256 MMAs read both halves, so that the
// tensor core rather than shared-memory bandwidth sets the pace (below).
// Every wait is bounded (status word + abort flag).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "q4_kernels.h"

namespace q4 {

namespace {

constexpr int kSBM = 128;  // rows of C per CTA (the MMA's M)
constexpr int kSBK = 32;   // k per stage: one 128-byte row of fp32 per operand row
constexpr int kChunkStages = 1;  // stages per accumulator chunk (32 k)
constexpr int kSgThreads = 256;  // warps 0-3: producer (warp 0), MMA (warp 1); warps 4-7: epilogue

template <int BN>
struct SgCfg {
    static constexpr int kATile = kSBM * kSBK * 4;  // 16 KB per plane
    static constexpr int kBTile = BN * kSBK * 4;
    static constexpr int kStageBytes = 2 * kATile + 2 * kBTile;
    static constexpr int kStages = (200 * 1024) / kStageBytes > 8 ? 8 : (200 * 1024) / kStageBytes;
    static constexpr int kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;  // two chunk buffers
    static constexpr int kBarOff = kStages * kStageBytes;
    // full[S], empty[S], chunk_full[2], chunk_empty[2]; then abort flag, TMEM address
    static constexpr int kNumBars = 2 * kStages + 4;
    static constexpr int kSmem = kBarOff + kNumBars * 8 + 16;
    static constexpr int kSmemAlloc = kSmem + 1024;  // slack to align the window to 1024
};

// hi / lo planes of a row-major [R][C] matrix, same orientation: planes of
// out_rows (>= R) rows with row pitch ld_out (>= C); the padding is zero.
__global__ void __launch_bounds__(256) split_kernel(const float* __restrict__ src, int R, int C, long long ld_src,
                                                    float* __restrict__ hi, float* __restrict__ lo, int out_rows,
                                                    long long ld_out) {
    const long long total = static_cast<long long>(out_rows) * ld_out;
    for (long long i = blockIdx.x * 256ll + threadIdx.x; i < total; i += static_cast<long long>(gridDim.x) * 256) {
        const long long r = i / ld_out, c = i - r * ld_out;
        const float v = (r < R && c < C) ? src[r * ld_src + c] : 0.0f;
        const float h = to_tf32(v);
        hi[i] = h;
        lo[i] = v - h;
    }
}

// hi / lo planes of the transpose of a row-major [R][C] matrix: out_rows
// (>= C) rows with row pitch ld_out (>= R), through 32 x 32 shared-memory
// tiles; the padding is zero.
__global__ void __launch_bounds__(256) split_t_kernel(const float* __restrict__ src, int R, int C, long long ld_src,
                                                      float* __restrict__ hi, float* __restrict__ lo, int out_rows,
                                                      long long ld_out) {
    __shared__ float tile[32][33];
    const long long r0 = static_cast<long long>(blockIdx.y) * 32;
    const int c0 = blockIdx.x * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 8 rows of 32
    for (int j = ty; j < 32; j += 8) {
        const long long r = r0 + j;
        const int c = c0 + tx;
        tile[j][tx] = (r < R && c < C) ? src[r * ld_src + c] : 0.0f;
    }
    __syncthreads();
    for (int j = ty; j < 32; j += 8) {
        const int c = c0 + j;            // output row
        const long long r = r0 + tx;     // output column
        if (c < out_rows && r < ld_out) {
            const float v = tile[tx][j];
            const float h = to_tf32(v);
            hi[static_cast<long long>(c) * ld_out + r] = h;
            lo[static_cast<long long>(c) * ld_out + r] = v - h;
        }
    }
}

template <int BN>
__global__ void __launch_bounds__(kSgThreads, 1)
    sgemm_tc_kernel(const __grid_constant__ CUtensorMap tm_ahi, const __grid_constant__ CUtensorMap tm_alo,
                    const __grid_constant__ CUtensorMap tm_bhi, const __grid_constant__ CUtensorMap tm_blo,
                    float* __restrict__ c, int M, int N, int K, long long ldc, float alpha, int* __restrict__ status) {
    using C = SgCfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;  // 128B-swizzled tiles need a 1024-aligned window
    uint8_t* smem = smem_raw + (base - raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ntn = (N + BN - 1) / BN;
    const int m0 = (static_cast<int>(blockIdx.x) / ntn) * kSBM;
    const int n0 = (static_cast<int>(blockIdx.x) % ntn) * BN;
    const int KT = (K + kSBK - 1) / kSBK;
    const int NC = (KT + kChunkStages - 1) / kChunkStages;  // accumulator chunks

    const uint32_t bar = base + C::kBarOff;
    auto full = [&](int s) { return bar + 8u * s; };
    auto empty = [&](int s) { return bar + 8u * (C::kStages + s); };
    auto chunk_full = [&](int b) { return bar + 8u * (2 * C::kStages + b); };
    auto chunk_empty = [&](int b) { return bar + 8u * (2 * C::kStages + 2 + b); };
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kBarOff + C::kNumBars * 8);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kBarOff + C::kNumBars * 8 + 8);

    if (tid == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(chunk_full(b), 1);
            mbar_init(chunk_empty(b), 4);  // one arrival per epilogue warp
        }
        *abort_flag = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    pdl_wait();  // the operands may be written by the previous launch (the split pass)
    if (warp == 0) {
        if (lane == 0) {
            // --------------------------------------------------- producer --
            tma_prefetch_desc(&tm_ahi);
            tma_prefetch_desc(&tm_alo);
            tma_prefetch_desc(&tm_bhi);
            tma_prefetch_desc(&tm_blo);
            int issued = 0;
            for (int kt = 0; kt < KT; ++kt) {
                const int s = kt % C::kStages;
                if (kt >= C::kStages &&
                    !mbar_wait(empty(s), ((kt / C::kStages) - 1) & 1u, abort_flag, status, kStatusTimeoutProducer))
                    break;
                const uint32_t st = base + s * C::kStageBytes;
                mbar_arrive_expect_tx(full(s), static_cast<uint32_t>(C::kStageBytes));
                tma_load_2d(st, &tm_ahi, full(s), kt * kSBK, m0);
                tma_load_2d(st + C::kATile, &tm_alo, full(s), kt * kSBK, m0);
                tma_load_2d(st + 2 * C::kATile, &tm_bhi, full(s), kt * kSBK, n0);
                tma_load_2d(st + 2 * C::kATile + C::kBTile, &tm_blo, full(s), kt * kSBK, n0);
                issued = kt + 1;
            }
            if (*abort_flag)  // let copies in flight land before the CTA exits
                for (int j = issued > C::kStages ? issued - C::kStages : 0; j < issued; ++j)
                    mbar_drain(full(j % C::kStages), (j / C::kStages) & 1u);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            // -------------------------------------------------------- MMA --
            constexpr uint32_t idesc = umma_idesc_tf32(kSBM, BN);
            bool ok = true;
            for (int ch = 0; ch < NC && ok; ++ch) {
                const int b = ch & 1;
                const uint32_t dacc = tmem + static_cast<uint32_t>(b * BN);
                if (ch >= 2 && !mbar_wait(chunk_empty(b), ((ch >> 1) - 1) & 1u, abort_flag, status,
                                          kStatusTimeoutMma)) {
                    ok = false;
                    break;
                }
                tc_fence_after_sync();
                const int kt_end = min(KT, (ch + 1) * kChunkStages);
                for (int kt = ch * kChunkStages; kt < kt_end; ++kt) {
                    const int s = kt % C::kStages;
                    if (!mbar_wait(full(s), (kt / C::kStages) & 1u, abort_flag, status, kStatusTimeoutMma)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after_sync();
                    const uint32_t st = base + s * C::kStageBytes;
                    const uint32_t ahi = st, alo = st + C::kATile, bhi = st + 2 * C::kATile, blo = bhi + C::kBTile;
#pragma unroll
                    for (int kk = 0; kk < kSBK / 8; ++kk) {  // 8 tf32 = 32 bytes of the 128-byte row
                        const uint32_t off = kk * 32;
                        const uint32_t acc0 = (kt > ch * kChunkStages || kk > 0) ? 1u : 0u;
                        umma_tf32_ss(dacc, umma_desc_k_sw128(alo + off), umma_desc_k_sw128(bhi + off), idesc, acc0);
                        umma_tf32_ss(dacc, umma_desc_k_sw128(ahi + off), umma_desc_k_sw128(blo + off), idesc, 1u);
                        umma_tf32_ss(dacc, umma_desc_k_sw128(ahi + off), umma_desc_k_sw128(bhi + off), idesc, 1u);
                    }
                    umma_commit(empty(s));  // the stage's tiles may be overwritten once these MMAs complete
                }
                umma_commit(chunk_full(b));  // the chunk's sums are in buffer b once its MMAs complete
            }
        }
        __syncwarp();
    } else if (warp >= 4) {
        // -------------------------------------------------------- epilogue --
        // Warp w reads TMEM lane quarter w % 4: thread t <-> row m0 + 32 (w % 4) + t.
        const int quarter = warp & 3;
        const uint32_t t_lane = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        float total[BN];
#pragma unroll
        for (int j = 0; j < BN; ++j) total[j] = 0.0f;
        bool ok = true;
        for (int ch = 0; ch < NC && ok; ++ch) {
            const int b = ch & 1;
            if (!mbar_wait_warp(chunk_full(b), (ch >> 1) & 1u, abort_flag, status, kStatusTimeoutEpilogue)) {
                ok = false;
                break;
            }
            tc_fence_after_sync();
#pragma unroll
            for (int cb = 0; cb < BN; cb += 16) {
                uint32_t v[16];
                tmem_ld16(t_lane + static_cast<uint32_t>(b * BN + cb), v);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 16; ++j) total[cb + j] += __uint_as_float(v[j]);  // round to nearest
            }
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(chunk_empty(b));  // buffer b may take chunk ch + 2
        }
        const int row = m0 + quarter * 32 + lane;
        if (ok && *abort_flag == 0 && row < M) {
            float* dst = c + static_cast<long long>(row) * ldc + n0;
#pragma unroll
            for (int cb = 0; cb < BN; cb += 4) {
                if (n0 + cb + 4 <= N && (reinterpret_cast<uintptr_t>(dst + cb) & 15u) == 0) {
                    *reinterpret_cast<float4*>(dst + cb) = make_float4(alpha * total[cb], alpha * total[cb + 1],
                                                                       alpha * total[cb + 2], alpha * total[cb + 3]);
                } else {
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        if (n0 + cb + j < N) dst[cb + j] = alpha * total[cb + j];
                }
            }
        }
    }
    tc_fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after_sync();
        tmem_dealloc(tmem, C::kTmemCols);
    }
}

template <int BN>
int launch_sgemm_bn(const SgemmTcArgs& a, cudaStream_t stream) {
    using C = SgCfg<BN>;
    auto kern = sgemm_tc_kernel<BN>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemAlloc);
    if (e != cudaSuccess) return static_cast<int>(e);
    cudaLaunchConfig_t cfg = {};
    const long long tiles = static_cast<long long>((a.M + kSBM - 1) / kSBM) * ((a.N + BN - 1) / BN);
    cfg.gridDim = dim3(static_cast<unsigned>(tiles));
    cfg.blockDim = dim3(kSgThreads);
    cfg.dynamicSmemBytes = C::kSmemAlloc;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, a.tm_ahi, a.tm_alo, a.tm_bhi, a.tm_blo, a.c, a.M, a.N, a.K, a.ldc, a.alpha,
                           a.status);
    return static_cast<int>(e);
}

// ---------------------------------------------------------------- pairs --
// A cluster of two CTAs owns a 256 x 256 tile of C.  CTA c TMA-loads rows
// m0 + 128 c .. of the A planes and rows n0 + 128 c .. of the B^T planes (hi
// and lo, 32 k per stage; the loads are counted on the leader's barrier), and
// the leader issues kind::tf32 MMAs with M = 256, N = 256, K = 8 that read A
// and B from both CTAs' shared memory at the same offsets.  Each CTA's tensor
// memory holds its 128 rows x 256 columns of the accumulator, double-buffered
// for the 32-k chunks (all 512 columns).  Per CTA and stage: 64 KB written by
// TMA and 96 KB read by twelve MMAs, ~1250 shared-memory cycles, against
// 12 x ~129 cycles of tensor core; the single-CTA 128 x 128 tile moves the
// same 160 KB for half the products.  Persistent: pair p takes tiles p,
// p + pairs, ...; the eight epilogue warps (two per lane quarter, 128 columns
// each) sum the chunks of a tile in registers and store its rows of C while
// the MMAs run on into the next tile.
constexpr int kSpHalf = 128;
constexpr int kSpTile = 256;
constexpr int kSpThreads = 320;  // warp 0 TMA, warp 1 MMA (leader CTA), warps 2-9 epilogue
constexpr int kSpEpiWarp0 = 2;
constexpr int kSpEpiWarps = 8;
constexpr int kSpEpiCols = 128;  // accumulator columns per epilogue warp

struct SpCfg {
    static constexpr int kPlane = kSpHalf * kSBK * 4;  // 16 KB: 128 rows x 32 k of one plane
    static constexpr int kStageBytes = 4 * kPlane;     // A hi, A lo, B hi, B lo
    static constexpr int kStages = 3;
    static constexpr int kBarOff = kStages * kStageBytes;
    // full[S] (leader), empty[S] (both), chunk_full[2] (both), chunk_empty[2] (leader), done (leader);
    // then abort flag, TMEM address
    static constexpr int kNumBars = 2 * kStages + 5;
    static constexpr int kSmem = kBarOff + kNumBars * 8 + 16;
    static constexpr int kSmemAlloc = kSmem + 1024;
    static constexpr int kTmemCols = 2 * kSpTile;
    static_assert(kSmemAlloc <= 232448, "shared memory budget");
};

__global__ void __launch_bounds__(kSpThreads, 1)
    sgemm_pair_kernel(const __grid_constant__ CUtensorMap tm_ahi, const __grid_constant__ CUtensorMap tm_alo,
                      const __grid_constant__ CUtensorMap tm_bhi, const __grid_constant__ CUtensorMap tm_blo,
                      float* __restrict__ c, int M, int N, int K, long long ldc, float alpha, int* __restrict__ status) {
    using C = SpCfg;
    constexpr int ST = C::kStages;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;  // 128B-swizzled tiles need a 1024-aligned window
    uint8_t* smem = smem_raw + (base - raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t crank = cluster_ctarank();
    const bool leader = crank == 0;
    const int pair = static_cast<int>(blockIdx.x >> 1), npairs = static_cast<int>(gridDim.x >> 1);
    const int MT = (M + kSpTile - 1) / kSpTile, NT = (N + kSpTile - 1) / kSpTile;
    const int tiles = MT * NT;
    const int KT = (K + kSBK - 1) / kSBK;

    const uint32_t bar = base + C::kBarOff;
    auto full = [&](int s) { return bar + 8u * s; };
    auto empty = [&](int s) { return bar + 8u * (ST + s); };
    auto chunk_full = [&](int b) { return bar + 8u * (2 * ST + b); };
    auto chunk_empty = [&](int b) { return bar + 8u * (2 * ST + 2 + b); };
    const uint32_t done_bar = bar + 8u * (2 * ST + 4);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kBarOff + C::kNumBars * 8);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kBarOff + C::kNumBars * 8 + 8);
    auto leader_addr = [&](uint32_t a) { return mapa_shared(a, 0); };

    if (tid == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(full(s), 1);   // the leader's expect_tx (both CTAs' bytes)
            mbar_init(empty(s), 1);  // the leader's multicast commit
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(chunk_full(b), 1);                  // the leader's multicast commit
            mbar_init(chunk_empty(b), 2 * kSpEpiWarps);   // epilogue warps of both CTAs
        }
        mbar_init(done_bar, 1);
        *abort_flag = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(tmem_slot), C::kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before_sync();
    cluster_sync_all();  // both CTAs' barriers initialised and tensor memory allocated
    tc_fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // --------------------------------------------------- producer --
            tma_prefetch_desc(&tm_ahi);
            tma_prefetch_desc(&tm_alo);
            tma_prefetch_desc(&tm_bhi);
            tma_prefetch_desc(&tm_blo);
            pdl_wait();  // the planes are written by the previous launches (the split pass)
            int it = 0;
            bool ok = true;
            for (int t = pair; t < tiles && ok; t += npairs) {
                const int m0 = (t % MT) * kSpTile + static_cast<int>(crank) * kSpHalf;
                const int n0 = (t / MT) * kSpTile + static_cast<int>(crank) * kSpHalf;
                for (int kt = 0; kt < KT; ++kt, ++it) {
                    const int s = it % ST;
                    const uint32_t ph = (it / ST) & 1u;
                    if (!mbar_wait(empty(s), ph ^ 1u, abort_flag, status, kStatusTimeoutProducer)) {
                        ok = false;
                        break;
                    }
                    if (leader) mbar_arrive_expect_tx(full(s), 2u * C::kStageBytes);
                    const uint32_t f = leader_addr(full(s));
                    const uint32_t st = base + s * C::kStageBytes;
                    tma_load_2d_pair(st, &tm_ahi, f, kt * kSBK, m0);
                    tma_load_2d_pair(st + C::kPlane, &tm_alo, f, kt * kSBK, m0);
                    tma_load_2d_pair(st + 2 * C::kPlane, &tm_bhi, f, kt * kSBK, n0);
                    tma_load_2d_pair(st + 3 * C::kPlane, &tm_blo, f, kt * kSBK, n0);
                }
            }
            if (*abort_flag && leader)  // let the copies in flight (both CTAs') land before exit
                for (int j = (it > ST ? it - ST : 0); j < it; ++j) mbar_drain(full(j % ST), (j / ST) & 1u);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (leader && elect_one()) {
            // ------------------------------------------- MMA (leader CTA) --
            constexpr uint32_t idesc = umma_idesc_tf32(kSpTile, kSpTile);
            int it = 0;
            bool ok = true;
            for (int t = pair; t < tiles && ok; t += npairs) {
                for (int kt = 0; kt < KT; ++kt, ++it) {
                    const int b = it & 1;  // one 32-k chunk per stage
                    if (!mbar_wait(chunk_empty(b), ((it >> 1) & 1u) ^ 1u, abort_flag, status, kStatusTimeoutMma) ||
                        !mbar_wait(full(it % ST), (it / ST) & 1u, abort_flag, status, kStatusTimeoutMma)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after_sync();
                    const uint32_t dacc = tmem + static_cast<uint32_t>(b * kSpTile);
                    const uint32_t st = base + (it % ST) * C::kStageBytes;
                    const uint32_t ahi = st, alo = st + C::kPlane, bhi = st + 2 * C::kPlane, blo = st + 3 * C::kPlane;
#pragma unroll
                    for (int kk = 0; kk < kSBK / 8; ++kk) {
                        const uint32_t off = kk * 32;
                        umma_tf32_ss_pair(dacc, umma_desc_k_sw128(alo + off), umma_desc_k_sw128(bhi + off), idesc,
                                          kk > 0 ? 1u : 0u);
                        umma_tf32_ss_pair(dacc, umma_desc_k_sw128(ahi + off), umma_desc_k_sw128(blo + off), idesc, 1u);
                        umma_tf32_ss_pair(dacc, umma_desc_k_sw128(ahi + off), umma_desc_k_sw128(bhi + off), idesc, 1u);
                    }
                    umma_commit_pair_both(empty(it % ST), 0x3);  // the stage may be refilled in both CTAs
                    umma_commit_pair_both(chunk_full(b), 0x3);   // the chunk is complete in both CTAs
                }
            }
            umma_commit_pair(leader_addr(done_bar));  // tracks every MMA issued above
            mbar_drain(done_bar, 0u);
        }
        __syncwarp();
    } else {
        // -------------------------------------------------------- epilogue --
        // Warp w reads lane quarter w % 4 (thread t <-> row 32 (w % 4) + t of
        // this CTA's 128), columns 128 h .. 128 h + 127 of the tile, h = (w - 2) / 4.
        const int quarter = warp & 3, h = (warp - kSpEpiWarp0) >> 2;
        const uint32_t t_lane = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        float total[kSpEpiCols];
#pragma unroll
        for (int j = 0; j < kSpEpiCols; ++j) total[j] = 0.0f;
        int it = 0;
        bool ok = true;
        for (int t = pair; t < tiles && ok; t += npairs) {
            for (int kt = 0; kt < KT; ++kt, ++it) {
                const int b = it & 1;
                if (!mbar_wait_warp(chunk_full(b), (it >> 1) & 1u, abort_flag, status, kStatusTimeoutEpilogue)) {
                    ok = false;
                    break;
                }
                tc_fence_after_sync();
                const uint32_t col = t_lane + static_cast<uint32_t>(b * kSpTile + h * kSpEpiCols);
#pragma unroll
                for (int cb = 0; cb < kSpEpiCols; cb += 32) {
                    uint32_t v[32];
                    tmem_ld32(col + cb, v);
                    tmem_ld_wait_regs(v);
#pragma unroll
                    for (int j = 0; j < 32; ++j) total[cb + j] += __uint_as_float(v[j]);  // round to nearest
                }
                tc_fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive_remote(leader_addr(chunk_empty(b)));  // buffer b may take chunk it + 2
            }
            if (!ok) break;
            const int row = (t % MT) * kSpTile + static_cast<int>(crank) * kSpHalf + quarter * 32 + lane;
            const int n0 = (t / MT) * kSpTile + h * kSpEpiCols;
            if (*abort_flag == 0 && row < M && n0 < N) {
                float* dst = c + static_cast<long long>(row) * ldc + n0;
#pragma unroll
                for (int cb = 0; cb < kSpEpiCols; cb += 4) {
                    if (n0 + cb + 4 <= N && (reinterpret_cast<uintptr_t>(dst + cb) & 15u) == 0) {
                        *reinterpret_cast<float4*>(dst + cb) = make_float4(
                            alpha * total[cb], alpha * total[cb + 1], alpha * total[cb + 2], alpha * total[cb + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            if (n0 + cb + j < N) dst[cb + j] = alpha * total[cb + j];
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < kSpEpiCols; ++j) total[j] = 0.0f;
        }
    }
    tc_fence_before_sync();
    cluster_sync_all();  // no CTA leaves while its peer may still use its shared or tensor memory
    if (warp == 1) {
        tc_fence_after_sync();
        tmem_dealloc_pair(tmem, C::kTmemCols);
    }
}

cudaLaunchConfig_t sgemm_pair_config(unsigned pairs, cudaLaunchAttribute* attr, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs, 1, 1);
    cfg.blockDim = dim3(kSpThreads, 1, 1);
    cfg.dynamicSmemBytes = SpCfg::kSmemAlloc;
    cfg.stream = stream;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cfg;
}

}  // namespace

int sgemm_pair_tiles(int M, int N) { return ((M + kSpTile - 1) / kSpTile) * ((N + kSpTile - 1) / kSpTile); }

int sgemm_pair_max_active() {
    if (cudaFuncSetAttribute(sgemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SpCfg::kSmemAlloc) !=
        cudaSuccess)
        return 0;
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = sgemm_pair_config(1, attr, nullptr);
    cfg.numAttrs = 1;  // the cluster shape only
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, sgemm_pair_kernel, &cfg) != cudaSuccess) return 0;
    return n;
}

int launch_sgemm_pair(const SgemmTcArgs& a, int max_pairs, cudaStream_t stream) {
    if (a.M < 1 || a.N < 1 || a.K < 1 || max_pairs < 1) return static_cast<int>(cudaErrorInvalidValue);
    cudaError_t e = cudaFuncSetAttribute(sgemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         SpCfg::kSmemAlloc);
    if (e != cudaSuccess) return static_cast<int>(e);
    const int tiles = sgemm_pair_tiles(a.M, a.N);
    const unsigned pairs = static_cast<unsigned>(tiles < max_pairs ? tiles : max_pairs);
    cudaLaunchAttribute attr[2];
    const cudaLaunchConfig_t cfg = sgemm_pair_config(pairs, attr, stream);
    e = cudaLaunchKernelEx(&cfg, sgemm_pair_kernel, a.tm_ahi, a.tm_alo, a.tm_bhi, a.tm_blo, a.c, a.M, a.N, a.K, a.ldc,
                           a.alpha, a.status);
    return static_cast<int>(e);
}

int launch_split_planes(const float* src, int rows, int cols, long long ld_src, bool transpose, float* hi, float* lo,
                        int out_rows, long long ld_out, cudaStream_t stream) {
    if (rows <= 0 || cols <= 0 || out_rows < (transpose ? cols : rows) || ld_out < (transpose ? rows : cols))
        return static_cast<int>(cudaErrorInvalidValue);
    if (!transpose) {
        const long long total = static_cast<long long>(out_rows) * ld_out;
        long long blocks = (total + 255) / 256;
        if (blocks > 148 * 16) blocks = 148 * 16;
        split_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(src, rows, cols, ld_src, hi, lo, out_rows,
                                                                        ld_out);
    } else {
        const dim3 grid(static_cast<unsigned>((out_rows + 31) / 32), static_cast<unsigned>((ld_out + 31) / 32));
        split_t_kernel<<<grid, 256, 0, stream>>>(src, rows, cols, ld_src, hi, lo, out_rows, ld_out);
    }
    return static_cast<int>(cudaGetLastError());
}

int sgemm_tc_bn(int N) {
    if (N <= 16) return 16;
    if (N <= 32) return 32;
    if (N <= 64) return 64;
    return 128;
}

int launch_sgemm_tc(const SgemmTcArgs& a, cudaStream_t stream) {
    if (a.M < 1 || a.N < 1 || a.K < 1) return static_cast<int>(cudaErrorInvalidValue);
    switch (a.bn) {
        case 16: return launch_sgemm_bn<16>(a, stream);
        case 32: return launch_sgemm_bn<32>(a, stream);
        case 64: return launch_sgemm_bn<64>(a, stream);
        case 128: return launch_sgemm_bn<128>(a, stream);
        default: return static_cast<int>(cudaErrorInvalidValue);
    }
}

}  // namespace q4
