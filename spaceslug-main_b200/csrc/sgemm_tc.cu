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

}  // namespace

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
