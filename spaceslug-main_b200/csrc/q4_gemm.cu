// Prefill GEMM (M > 8):  Y[M x N] = X[M x K] . dequant(W)  (+ LoRA term).
//
// Replaces vulkan-runtime/shaders/q4gemm.comp:61-175 (fp32 FMA tiles with the
// int4 B operand dequantised into an fp32 LDS tile) with a persistent
// Blackwell tensor-core pipeline.  One CTA per SM walks output tiles of
// (128*H) x 128; per tile and 64-wide k-step:
//
//   warp 0        TMA producer of X tiles (16-bit, 64 x 128H, 128B swizzle);
//   warp 14       TMA producer of the raw packed W tiles (128 columns x 32
//                 bytes) into their own deeper ring, released by the dequant
//                 warps, so the weight stream runs ahead of the MMA instead
//                 of waiting for it to free a whole stage;
//   warp 1        allocates TMEM (2 accumulator buffers x H x 128 columns);
//                 one elected thread issues tcgen05.mma kind::f16 (M=128,
//                 N=128, K=16; H row halves share one B tile), commits each
//                 stage back to the producer and each finished accumulator
//                 to the epilogue;
//   warps 2..9    dequantise one (column, 32-k group) unit each per k-step:
//                 nibbles -> float(v) exactly -> * scale in fp32 (the
//                 reference's w = float(v) * scale, q4gemm.comp:116-122) ->
//                 16-bit RN, written straight into the canonical K-major
//                 128B-swizzled UMMA B tile (packed f32x2 arithmetic);
//   warps 10..13  epilogue: tcgen05.ld 32 lanes x 16 columns, undo the
//                 power-of-two operand exponents, store fp32 Y; overlaps the
//                 next tile's main loop through the second TMEM buffer.
//
// LoRA is ceil(rank/16) more 64-k stages per tile in the same accumulator;
// stage q covers ranks 16q..16q+15: A = T * 2^e_m as bf16 [hi | lo | hi | 0]
// (made by the X*A reduction, loaded by TMA like an X tile), B = (alpha/r) *
// B_lora * 2^f_n as bf16 [hi | hi | lo | 0], built by the dequant warps from
// fp32 B_lora.  The same power-of-two exponents as the main operands make the
// epilogue's 2^-(e+f) exact for both; bf16 keeps T * 2^e in range, and
// hi * hi + lo * hi + hi * lo keeps ~16 bits.
//
// With H = 2 every dequantised weight feeds 256 rows of MMA, which keeps the
// CUDA-core dequant work well under the tensor-core time per k-step.
//
// Operand precision: f16 operands carry a per-row power-of-two exponent for X
// and a per-column one for W (chosen so no element can overflow f16); the
// exponents are exact and undone in the epilogue.  bf16 operands need none.
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

constexpr int kBN = 128;
constexpr int kBK = 64;
constexpr int kThreads = 480;  // 15 warps
constexpr int kDequantWarps = 8;
constexpr int kEpiWarp0 = 10;
constexpr int kEpiWarps = 4;
constexpr int kRawWarp = 14;
constexpr int kScaleAhead = 8;  // k-steps of scales in flight per dequant thread

template <int H>
struct Cfg {
    static constexpr int kBM = 128 * H;
    static constexpr int kStages = H == 2 ? 4 : 6;  // X + dequantised-W ring
    static constexpr int kRawStages = 8;            // packed-W ring
    static constexpr int kABytes = kBM * kBK * 2;  // 16 KB per 128-row half
    static constexpr int kBBytes = kBN * kBK * 2;  // 16 KB
    static constexpr int kRBytes = kBN * kBK / 2;  // 4 KB (packed nibbles)
    static constexpr int kAOff = 0;
    static constexpr int kBOff = kAOff + kStages * kABytes;
    static constexpr int kROff = kBOff + kStages * kBBytes;
    static constexpr int kBarOff = kROff + kRawStages * kRBytes;
    // full_a, full_b, empty [kStages]; full_r, empty_r [kRawStages];
    // acc_full[2], acc_empty[2], done
    static constexpr int kNumBars = 3 * kStages + 2 * kRawStages + 2 + 2 + 1;
    static constexpr int kMiscOff = kBarOff + kNumBars * 8;
    static constexpr int kLutOff = kMiscOff + 16;     // CQ4: 256 f16 pairs (codebook[b & 15], codebook[b >> 4])
    static constexpr int kBytes = kLutOff + 1024;
    static constexpr int kSmemAlloc = kBytes + 1024;  // slack for 1024-byte alignment
    static constexpr int kTmemCols = 2 * H * kBN;     // 256 or 512
    static_assert(kSmemAlloc <= 232448, "shared memory budget");
    static_assert(kDequantWarps * 32 == kBN * 2, "one (column, group) unit per dequant thread");
};

template <int H, typename T16>
__global__ void __launch_bounds__(kThreads, 1)
    q4_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                   const __grid_constant__ CUtensorMap tmap_t, const float* __restrict__ scales,
                   const int* __restrict__ col_exp, const int* __restrict__ row_exp, float* __restrict__ y, int M,
                   int N, int K, const float* __restrict__ lora_b, int rank, float lora_scale, int lora_stages,
                   const uint32_t* __restrict__ lut, __half* __restrict__ y16, int* __restrict__ status) {
    using C = Cfg<H>;
    constexpr int ST = C::kStages;
    constexpr int RT = C::kRawStages;
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
    const int MT = (M + C::kBM - 1) / C::kBM;
    const int NT = (N + kBN - 1) / kBN;
    const int tiles = MT * NT;
    const int KT = (K + kBK - 1) / kBK;
    const int KS = KT + lora_stages;  // k-steps per tile, the LoRA stages last
    const int G = K / 32;

    if (tid == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(full_a(s), 1);
            mbar_init(full_b(s), kDequantWarps);
            mbar_init(empty(s), 1);
        }
        for (int r = 0; r < RT; ++r) {
            mbar_init(full_r(r), 1);
            mbar_init(empty_r(r), kDequantWarps);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(acc_full(b), 1);
            mbar_init(acc_empty(b), kEpiWarps);
        }
        mbar_init(done_bar, 1);
        *abort_flag = 0;
        fence_mbarrier_init();
        tma_prefetch_desc(&tmap_x);
        tma_prefetch_desc(&tmap_w);
        if (lora_stages) tma_prefetch_desc(&tmap_t);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_holder), C::kTmemCols);
        tmem_relinquish();
    }
    uint32_t* lut_s = reinterpret_cast<uint32_t*>(smem + C::kLutOff);
    if (lut != nullptr && tid < 256) lut_s[tid] = __ldg(lut + tid);
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {
        // -------------------------------------------------- X producer --
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            pdl_wait();  // X16 (and T) are written by the previous launches
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                const int m0 = (t % MT) * C::kBM;
                for (int kt = 0; kt < KS; ++kt, ++it) {
                    const int s = it % ST;
                    const uint32_t ph = (it / ST) & 1u;
                    if (!mbar_wait(empty(s), ph ^ 1u, abort_flag, status, kStatusTimeoutProducer)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(full_a(s), C::kABytes);
                    if (kt < KT) {
                        tma_load_2d(a_s + s * C::kABytes, &tmap_x, full_a(s), kt * kBK, m0);
                    } else {  // LoRA stage: the T operand
                        tma_load_2d(a_s + s * C::kABytes, &tmap_t, full_a(s), (kt - KT) * kBK, m0);
                    }
                }
            }
            if (*abort_flag) {  // let the copies in flight land before exit
                for (int j = (it > ST ? it - ST : 0); j < it; ++j) mbar_drain(full_a(j % ST), (j / ST) & 1u);
            }
        }
    } else if (warp == kRawWarp) {
        // -------------------------------------------- packed-W producer --
        // The packed weights do not depend on the previous launch (the X cast,
        // the X*A projection): no griddepcontrol.wait here.
        if (lane == 0) {
            int ir = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                const int n0 = (t / MT) * kBN;
                for (int kt = 0; kt < KT; ++kt, ++ir) {
                    const int r = ir % RT;
                    const uint32_t ph = (ir / RT) & 1u;
                    if (!mbar_wait(empty_r(r), ph ^ 1u, abort_flag, status, kStatusTimeoutProducer)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(full_r(r), C::kRBytes);
                    tma_load_2d(r_s + r * C::kRBytes, &tmap_w, full_r(r), kt * (kBK / 8), n0);
                }
            }
            if (*abort_flag) {
                for (int j = (ir > RT ? ir - RT : 0); j < ir; ++j) mbar_drain(full_r(j % RT), (j / RT) & 1u);
            }
        }
    } else if (warp == 1) {
        // ----------------------------------------------------------- MMA --
        if (elect_one()) {
            const uint32_t idesc = umma_idesc_f16(std::is_same<T16, __half>::value ? 0u : 1u, 128u,
                                                  static_cast<uint32_t>(kBN));
            const uint32_t idesc_lora = umma_idesc_f16(1u, 128u, static_cast<uint32_t>(kBN));  // bf16
            int it = 0, i = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++i) {
                const int b = i & 1;
                const uint32_t u = static_cast<uint32_t>(i >> 1);
                if (!mbar_wait(acc_empty(b), (u & 1u) ^ 1u, abort_flag, status, kStatusTimeoutMma)) break;
                tc_fence_after_sync();
                const uint32_t d0 = tmem_base + static_cast<uint32_t>(b * H * kBN);
                for (int kt = 0; kt < KS; ++kt, ++it) {
                    const int s = it % ST;
                    const uint32_t ph = (it / ST) & 1u;
                    if (!mbar_wait(full_a(s), ph, abort_flag, status, kStatusTimeoutMma) ||
                        !mbar_wait(full_b(s), ph, abort_flag, status, kStatusTimeoutMma)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after_sync();
                    const uint32_t id = kt < KT ? idesc : idesc_lora;
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk) {
                        const uint64_t bd = umma_desc_k_sw128(b_s + s * C::kBBytes + kk * 32);
#pragma unroll
                        for (int h = 0; h < H; ++h) {
                            const uint64_t ad = umma_desc_k_sw128(a_s + s * C::kABytes + h * 16384 + kk * 32);
                            umma_f16_ss(d0 + static_cast<uint32_t>(h * kBN), ad, bd, id, (kt | kk) != 0 ? 1u : 0u);
                        }
                    }
                    umma_commit(empty(s));
                }
                if (ok) umma_commit(acc_full(b));
            }
            umma_commit(done_bar);  // tracks every MMA issued above
            mbar_drain(done_bar, 0u);
        }
    } else if (warp < kEpiWarp0) {
        // ------------------------------------------------------- dequant --
        const int dt = tid - 64;
        const int nl = dt >> 1, hh = dt & 1;  // unit: column nl, group half hh of the k-step
        int it = 0, ir = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
            const int n = (t / MT) * kBN + nl;
            const bool col_ok = n < N;
            const float cs = (col_exp != nullptr && col_ok) ? exp2i(col_exp[n]) : 1.0f;
            const float* srow = scales + static_cast<size_t>(col_ok ? n : 0) * G;
            // Scales of the next kScaleAhead k-steps in flight (L2 latency spans
            // several k-steps), rotated through registers.
            auto scale_at = [&](int kt) {
                const int g = kt * 2 + hh;
                return (col_ok && g < G) ? __ldg(srow + g) : 0.0f;
            };
            float sq[kScaleAhead];
#pragma unroll
            for (int j = 0; j < kScaleAhead; ++j) sq[j] = scale_at(j);
            for (int kt = 0; kt < KS; ++kt, ++it) {
                const int s = it % ST;
                const uint32_t ph = (it / ST) & 1u;
                const float sc = sq[0];
#pragma unroll
                for (int j = 0; j + 1 < kScaleAhead; ++j) sq[j] = sq[j + 1];
                sq[kScaleAhead - 1] = scale_at(kt + kScaleAhead);
                uint4 out[4];
                if (kt < KT) {
                    const int r = ir % RT;
                    const uint32_t rph = (ir / RT) & 1u;
                    ++ir;
                    if (!mbar_wait_warp(full_r(r), rph, abort_flag, status, kStatusTimeoutDequant)) {
                        ok = false;
                        break;
                    }
                    const uint4 q =
                        *reinterpret_cast<const uint4*>(smem + C::kROff + r * C::kRBytes + nl * 32 + hh * 16);
                    const float sv = sc * cs;
                    const float2 s2v = make_float2(sv, sv);
                    __half2 s2h, s2l;
                    split_scale_f16(sv, s2h, s2l);
                    const uint32_t words[4] = {q.x, q.y, q.z, q.w};
                    if (lut == nullptr) {
#pragma unroll
                        for (int j = 0; j < 4; ++j) out[j] = dequant_f16x2_or<T16>(words[j], s2v, s2h, s2l);
                    } else {
                        // CQ4: pair (k, k+1) = RN16(codebook[idx] * norm), idx from byte b of the word
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            uint32_t o[4];
#pragma unroll
                            for (int b = 0; b < 4; ++b) {
                                const uint32_t e = lut_s[(words[j] >> (8 * b)) & 0xFFu];
                                const __half2 w = __hmul2(*reinterpret_cast<const __half2*>(&e), s2h);
                                o[b] = *reinterpret_cast<const uint32_t*>(&w);
                            }
                            out[j] = make_uint4(o[0], o[1], o[2], o[3]);
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(empty_r(r));  // the packed stage is consumed
                } else {
                    // LoRA stage q: (alpha/r) * B_lora[16q .. 16q+15, n] * 2^f_n as bf16;
                    // positions [0,16) hi, [16,32) hi (hh = 0), [32,48) lo, [48,64) 0 (hh = 1)
                    const int j0 = (kt - KT) * 16;
                    uint32_t pk[8];
#pragma unroll
                    for (int j = 0; j < 16; j += 2) {
                        float b0 = 0.0f, b1 = 0.0f;
                        if (col_ok && j0 + j < rank)
                            b0 = __ldg(lora_b + static_cast<size_t>(j0 + j) * N + n) * lora_scale * cs;
                        if (col_ok && j0 + j + 1 < rank)
                            b1 = __ldg(lora_b + static_cast<size_t>(j0 + j + 1) * N + n) * lora_scale * cs;
                        const __nv_bfloat162 hi = __floats2bfloat162_rn(b0, b1);
                        if (hh == 0) {
                            pk[j / 2] = *reinterpret_cast<const uint32_t*>(&hi);
                        } else {
                            const float2 hf = __bfloat1622float2(hi);
                            const __nv_bfloat162 lo = __floats2bfloat162_rn(b0 - hf.x, b1 - hf.y);
                            pk[j / 2] = *reinterpret_cast<const uint32_t*>(&lo);
                        }
                    }
                    const uint4 c0 = make_uint4(pk[0], pk[1], pk[2], pk[3]), c1 = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
                    out[0] = c0;
                    out[1] = c1;
                    out[2] = hh == 0 ? c0 : z;
                    out[3] = hh == 0 ? c1 : z;
                }
                // the B slot is free once the MMAs of its previous round completed
                if (!mbar_wait_warp(empty(s), ph ^ 1u, abort_flag, status, kStatusTimeoutDequant)) {
                    ok = false;
                    break;
                }
                uint8_t* brow = smem + C::kBOff + s * C::kBBytes + nl * 128;
#pragma unroll
                for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4*>(brow + (((hh * 4 + j) ^ (nl & 7)) * 16)) = out[j];
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(full_b(s));
            }
        }
    } else if (warp < kEpiWarp0 + kEpiWarps) {
        // ------------------------------------------------------ epilogue --
        pdl_wait();  // row exponents and Y belong to the previous launch until it completes
        const int quarter = warp & 3;
        const bool vec_ok = (N % 4) == 0;
        int i = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
            const int b = i & 1;
            const uint32_t u = static_cast<uint32_t>(i >> 1);
            if (!mbar_wait_warp(acc_full(b), u & 1u, abort_flag, status, kStatusTimeoutEpilogue)) break;
            tc_fence_after_sync();
            const int m0 = (t % MT) * C::kBM, n0 = (t / MT) * kBN;
            // 2^-col_exp of the tile's 128 columns: lane l holds columns
            // n0 + 4l .. 4l+3; element e of chunk c is shuffled from lane
            // (16c + e) / 4.
            float cf[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int n = n0 + lane * 4 + j;
                cf[j] = (col_exp != nullptr && n < N) ? exp2i(-col_exp[n]) : 1.0f;
            }
#pragma unroll 1
            for (int h = 0; h < H; ++h) {
                const int row = m0 + h * 128 + quarter * 32 + lane;
                const bool row_ok = row < M;
                const float rs = (row_exp != nullptr && row_ok) ? exp2i(-row_exp[row]) : 1.0f;
                float* yrow = y + static_cast<size_t>(row_ok ? row : 0) * N;
                const uint32_t tcol = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                      static_cast<uint32_t>(b * H * kBN + h * kBN);
#pragma unroll 1
                for (int c = 0; c < kBN / 16; ++c) {
                    uint32_t r[16];
                    tmem_ld16(tcol + static_cast<uint32_t>(c * 16), r);
                    tmem_ld_wait();
                    const int nb = n0 + c * 16;
                    float v[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const float cinv = __shfl_sync(0xffffffffu, cf[e & 3], c * 4 + (e >> 2));
                        v[e] = __uint_as_float(r[e]) * rs * cinv;
                    }
                    if (nb >= N) continue;  // warp-uniform
                    if (row_ok && y16 != nullptr) {
                        // fp16 output (CQ4): round once, 16 consecutive columns
                        __half* hrow = y16 + static_cast<size_t>(row) * N;
                        if ((N % 8) == 0 && nb + 16 <= N) {
                            uint32_t hp[8];
#pragma unroll
                            for (int e = 0; e < 16; e += 2) {
                                const __half2 h2 = __floats2half2_rn(v[e], v[e + 1]);
                                hp[e / 2] = *reinterpret_cast<const uint32_t*>(&h2);
                            }
                            *reinterpret_cast<uint4*>(hrow + nb) = make_uint4(hp[0], hp[1], hp[2], hp[3]);
                            *reinterpret_cast<uint4*>(hrow + nb + 8) = make_uint4(hp[4], hp[5], hp[6], hp[7]);
                        } else {
#pragma unroll
                            for (int e = 0; e < 16; ++e)
                                if (nb + e < N) hrow[nb + e] = __float2half_rn(v[e]);
                        }
                    } else if (row_ok) {
                        if (vec_ok && nb + 16 <= N) {
#pragma unroll
                            for (int e = 0; e < 16; e += 4)
                                *reinterpret_cast<float4*>(yrow + nb + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
                        } else {
#pragma unroll
                            for (int e = 0; e < 16; ++e)
                                if (nb + e < N) yrow[nb + e] = v[e];
                        }
                    }
                }
            }
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty(b));
        }
    }

    tc_fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after_sync();
        tmem_dealloc(tmem_base, C::kTmemCols);
    }
}

template <int H, typename T16>
int launch_gemm_t(const GemmArgs& a, int grid, cudaStream_t stream) {
    using C = Cfg<H>;
    auto kern = q4_gemm_kernel<H, T16>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemAlloc);
    if (e != cudaSuccess) return static_cast<int>(e);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::kSmemAlloc;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // overlap the X cast's tail
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, a.tmap_x16, a.tmap_w, a.tmap_t, a.scales, a.col_exp, a.row_exp, a.y, a.M, a.N,
                           a.K, a.lora_b, a.rank, a.lora_scale, a.lora_stages, a.lut,
                           static_cast<__half*>(a.y16), a.status);
    return static_cast<int>(e);
}

}  // namespace

int gemm_tiles(int M, int N, int halves) { return ((M + 128 * halves - 1) / (128 * halves)) * ((N + kBN - 1) / kBN); }

int launch_gemm(const GemmArgs& a, cudaStream_t stream) {
    const int tiles = gemm_tiles(a.M, a.N, a.halves);
    const int grid = tiles < a.sm_count ? tiles : a.sm_count;
    if (a.halves == 2) {
        return a.op == Operand16::kF16 ? launch_gemm_t<2, __half>(a, grid, stream)
                                       : launch_gemm_t<2, __nv_bfloat16>(a, grid, stream);
    }
    if (a.halves == 1) {
        return a.op == Operand16::kF16 ? launch_gemm_t<1, __half>(a, grid, stream)
                                       : launch_gemm_t<1, __nv_bfloat16>(a, grid, stream);
    }
    return static_cast<int>(cudaErrorInvalidValue);
}

}  // namespace q4
