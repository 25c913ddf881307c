// Prefill GEMM (M > 8):  Y[M x N] = X[M x K] . dequant(W)  (+ LoRA term).
//
// Replaces vulkan-runtime/shaders/q4gemm.comp:61-175 (fp32 FMA tiles with the
// int4 B operand dequantised into an fp32 LDS tile) with a Blackwell tensor
// core pipeline:
//
//   warp 0        TMA producer: X tile (16-bit, 128 x 64, 128B swizzle) and
//                 the raw packed W tile (BN columns x 32 bytes) per k-step;
//   warp 1        allocates TMEM, one elected thread issues tcgen05.mma
//                 (kind::f16, M=128, N=BN, K=16 x 4 per k-step) into an fp32
//                 TMEM accumulator, commits each stage back to the producer;
//   warps 2..9    dequantise: nibbles -> float(v) (exact) * scale (fp32, RN,
//                 the reference's w = float(v) * scale of q4gemm.comp:116-122)
//                 -> 16-bit RN, written straight into the canonical K-major
//                 128B-swizzled UMMA B tile; then warps 2..5 run the epilogue
//                 (tcgen05.ld 32 lanes x 16 columns, undo the power-of-two
//                 operand exponents, add the fused LoRA term, store fp32 Y).
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
#include "q4_kernels.h"

namespace q4 {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 320;  // 10 warps
constexpr int kDequantWarps = 8;
constexpr int kDequantThreads = kDequantWarps * 32;

template <int BN>
struct Cfg {
    static constexpr int kStages = BN == 256 ? 4 : 6;
    static constexpr int kABytes = kBM * kBK * 2;  // 16 KB
    static constexpr int kBBytes = BN * kBK * 2;   // BN x 128 B
    static constexpr int kRBytes = BN * kBK / 2;   // BN x 32 B (packed nibbles)
    static constexpr int kAOff = 0;
    static constexpr int kBOff = kAOff + kStages * kABytes;
    static constexpr int kROff = kBOff + kStages * kBBytes;
    static constexpr int kBarOff = kROff + kStages * kRBytes;
    static constexpr int kNumBars = 4 * kStages + 1;
    static constexpr int kMiscOff = kBarOff + kNumBars * 8;
    static constexpr int kBytes = kMiscOff + 16;
    static constexpr int kSmemAlloc = kBytes + 1024;  // slack for 1024-byte alignment
    static constexpr int kUnitsPerThread = (BN * 2) / kDequantThreads;  // (column, group) units
    static_assert(kSmemAlloc <= 232448, "shared memory budget");
    static_assert(kUnitsPerThread * kDequantThreads == BN * 2, "dequant mapping");
};

__device__ __forceinline__ float exp2i(int e) { return __int_as_float((127 + e) << 23); }

template <typename T16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    if constexpr (sizeof(T16) == 2 && std::is_same<T16, __half>::value) {
        __half2 h = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    } else {
        __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    }
}

// Dequantise one packed word (8 consecutive k of one column) times `s` into
// four 16-bit pairs.  Same magic-number unpack as the GEMV: v exact, then one
// fp32 multiply by the (power-of-two adjusted) scale, then 16-bit RN.
template <typename T16>
__device__ __forceinline__ uint4 dequant_word(uint32_t q, float s) {
    const uint32_t lo = (q ^ 0x88888888u) & 0x0F0F0F0Fu;
    const uint32_t hi = ((q >> 4) ^ 0x08080808u) & 0x0F0F0F0Fu;
    const float bias = 8388616.0f;
    uint32_t out[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        const float ve = __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7440u | static_cast<uint32_t>(b))) - bias;
        const float vo = __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7440u | static_cast<uint32_t>(b))) - bias;
        out[b] = pack2<T16>(ve * s, vo * s);
    }
    return make_uint4(out[0], out[1], out[2], out[3]);
}

template <int BN, typename T16>
__global__ void __launch_bounds__(kThreads, 1)
    q4_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                   const float* __restrict__ scales, const int* __restrict__ col_exp,
                   const int* __restrict__ row_exp, float* __restrict__ y, int M, int N, int K,
                   const float* __restrict__ lora_t, const float* __restrict__ lora_b, int rank, float lora_scale,
                   int* __restrict__ status) {
    using C = Cfg<BN>;
    constexpr int ST = C::kStages;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = smem_u32(smem_raw);
    const uint32_t base = (raw_base + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (base - raw_base);

    const uint32_t a_s = base + C::kAOff;
    const uint32_t b_s = base + C::kBOff;
    const uint32_t r_s = base + C::kROff;
    const uint32_t bar = base + C::kBarOff;
    auto full_a = [&](int s) { return bar + 8u * s; };
    auto full_r = [&](int s) { return bar + 8u * (ST + s); };
    auto full_b = [&](int s) { return bar + 8u * (2 * ST + s); };
    auto empty = [&](int s) { return bar + 8u * (3 * ST + s); };
    const uint32_t acc_full = bar + 8u * (4 * ST);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::kMiscOff);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kMiscOff + 4);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.x * kBM, n0 = blockIdx.y * BN;
    const int KT = (K + kBK - 1) / kBK;
    const int G = K / 32;

    if (tid == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(full_a(s), 1);
            mbar_init(full_r(s), 1);
            mbar_init(full_b(s), kDequantWarps);
            mbar_init(empty(s), 1);
        }
        mbar_init(acc_full, 1);
        *abort_flag = 0;
        fence_mbarrier_init();
        tma_prefetch_desc(&tmap_x);
        tma_prefetch_desc(&tmap_w);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_holder), BN);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem_d = *tmem_holder;

    if (warp == 0) {
        // ------------------------------------------------------ producer --
        if (lane == 0) {
            for (int kt = 0; kt < KT; ++kt) {
                const int s = kt % ST;
                const uint32_t ph = (kt / ST) & 1u;
                if (!mbar_wait(empty(s), ph ^ 1u, abort_flag, status, kStatusTimeoutProducer)) break;
                mbar_arrive_expect_tx(full_a(s), C::kABytes);
                tma_load_2d(a_s + s * C::kABytes, &tmap_x, full_a(s), kt * kBK, m0);
                mbar_arrive_expect_tx(full_r(s), C::kRBytes);
                tma_load_2d(r_s + s * C::kRBytes, &tmap_w, full_r(s), kt * (kBK / 8), n0);
            }
        }
    } else if (warp == 1) {
        // ----------------------------------------------------------- MMA --
        if (elect_one()) {
            const uint32_t idesc =
                umma_idesc_f16(std::is_same<T16, __half>::value ? 0u : 1u, static_cast<uint32_t>(kBM),
                               static_cast<uint32_t>(BN));
            for (int kt = 0; kt < KT; ++kt) {
                const int s = kt % ST;
                const uint32_t ph = (kt / ST) & 1u;
                if (!mbar_wait(full_a(s), ph, abort_flag, status, kStatusTimeoutMma)) break;
                if (!mbar_wait(full_b(s), ph, abort_flag, status, kStatusTimeoutMma)) break;
                tc_fence_after_sync();
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk) {
                    const uint64_t ad = umma_desc_k_sw128(a_s + s * C::kABytes + kk * 32);
                    const uint64_t bd = umma_desc_k_sw128(b_s + s * C::kBBytes + kk * 32);
                    umma_f16_ss(tmem_d, ad, bd, idesc, (kt | kk) != 0 ? 1u : 0u);
                }
                umma_commit(empty(s));
            }
            umma_commit(acc_full);  // tracks every MMA issued above (also on abort)
        }
    } else {
        // ------------------------------------------------------- dequant --
        const int dt = tid - 64;
        float cs[C::kUnitsPerThread];   // 2^col_exp of the unit's column (exact)
        float sc[C::kUnitsPerThread];   // scale of the current k-step
        int nl[C::kUnitsPerThread], hh[C::kUnitsPerThread];
#pragma unroll
        for (int u = 0; u < C::kUnitsPerThread; ++u) {
            const int unit = dt + u * kDequantThreads;
            nl[u] = unit >> 1;
            hh[u] = unit & 1;
            const int n = n0 + nl[u];
            cs[u] = (col_exp != nullptr && n < N) ? exp2i(col_exp[n]) : 1.0f;
            const int g = hh[u];
            sc[u] = (n < N && g < G) ? __ldg(scales + static_cast<size_t>(n) * G + g) : 0.0f;
        }
        for (int kt = 0; kt < KT; ++kt) {
            const int s = kt % ST;
            const uint32_t ph = (kt / ST) & 1u;
            // prefetch the next k-step's scales while this step is converted
            float sn[C::kUnitsPerThread];
#pragma unroll
            for (int u = 0; u < C::kUnitsPerThread; ++u) {
                const int n = n0 + nl[u];
                const int g = (kt + 1) * 2 + hh[u];
                sn[u] = (n < N && g < G) ? __ldg(scales + static_cast<size_t>(n) * G + g) : 0.0f;
            }
            if (!mbar_wait(full_r(s), ph, abort_flag, status, kStatusTimeoutDequant)) break;
            const uint8_t* rt = smem + C::kROff + s * C::kRBytes;
            uint8_t* bt = smem + C::kBOff + s * C::kBBytes;
#pragma unroll
            for (int u = 0; u < C::kUnitsPerThread; ++u) {
                const uint4 q = *reinterpret_cast<const uint4*>(rt + nl[u] * 32 + hh[u] * 16);
                const float sv = sc[u] * cs[u];
                const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint4 o = dequant_word<T16>(words[j], sv);
                    const int chunk = (hh[u] * 4 + j) ^ (nl[u] & 7);
                    *reinterpret_cast<uint4*>(bt + nl[u] * 128 + chunk * 16) = o;
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(full_b(s));
#pragma unroll
            for (int u = 0; u < C::kUnitsPerThread; ++u) sc[u] = sn[u];
        }

        // ------------------------------------------------------ epilogue --
        if (warp < 6) {
            const bool ok = mbar_wait(acc_full, 0u, abort_flag, status, kStatusTimeoutEpilogue);
            tc_fence_after_sync();
            const int quarter = warp & 3;
            const int row = m0 + quarter * 32 + lane;
            const bool row_ok = ok && !*abort_flag && row < M;
            const float rs = (row_exp != nullptr && row < M) ? exp2i(-row_exp[row]) : 1.0f;
            float* yrow = y + static_cast<size_t>(row < M ? row : 0) * N;
            const bool vec_ok = (N % 4) == 0;
#pragma unroll 1
            for (int c = 0; c < BN / 16; ++c) {
                uint32_t r[16];
                tmem_ld16(tmem_d + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(c * 16), r);
                tmem_ld_wait();
                const int nb = n0 + c * 16;
                if (nb >= N) continue;  // warp-uniform
                float v[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int n = nb + i;
                    const float cinv = (col_exp != nullptr && n < N) ? exp2i(-col_exp[n]) : 1.0f;
                    v[i] = __uint_as_float(r[i]) * rs * cinv;
                }
                if (lora_t != nullptr && row_ok) {
                    float d[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) d[i] = 0.0f;
                    const float* trow = lora_t + static_cast<size_t>(row) * rank;
                    for (int j = 0; j < rank; ++j) {
                        const float tj = __ldg(trow + j);
                        const float* brow = lora_b + static_cast<size_t>(j) * N + nb;
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            if (nb + i < N) d[i] = fmaf(tj, __ldg(brow + i), d[i]);
                    }
#pragma unroll
                    for (int i = 0; i < 16; ++i) v[i] = fmaf(lora_scale, d[i], v[i]);
                }
                if (row_ok) {
                    if (vec_ok && nb + 16 <= N) {
#pragma unroll
                        for (int i = 0; i < 16; i += 4)
                            *reinterpret_cast<float4*>(yrow + nb + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            if (nb + i < N) yrow[nb + i] = v[i];
                    }
                }
            }
        }
    }

    tc_fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after_sync();
        tmem_dealloc(tmem_d, BN);
    }
}

template <int BN, typename T16>
int launch_gemm_t(const GemmArgs& a, cudaStream_t stream) {
    using C = Cfg<BN>;
    auto kern = q4_gemm_kernel<BN, T16>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemAlloc);
    if (e != cudaSuccess) return static_cast<int>(e);
    dim3 grid((a.M + kBM - 1) / kBM, (a.N + BN - 1) / BN, 1);
    kern<<<grid, kThreads, C::kSmemAlloc, stream>>>(a.tmap_x16, a.tmap_w, a.scales, a.col_exp, a.row_exp, a.y, a.M,
                                                    a.N, a.K, a.lora_t, a.lora_b, a.rank, a.lora_scale, a.status);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace

size_t gemm_smem_bytes(int bn) { return bn == 256 ? Cfg<256>::kSmemAlloc : Cfg<128>::kSmemAlloc; }

int launch_gemm(const GemmArgs& a, cudaStream_t stream) {
    if (a.bn == 256) {
        return a.op == Operand16::kF16 ? launch_gemm_t<256, __half>(a, stream)
                                       : launch_gemm_t<256, __nv_bfloat16>(a, stream);
    }
    if (a.bn == 128) {
        return a.op == Operand16::kF16 ? launch_gemm_t<128, __half>(a, stream)
                                       : launch_gemm_t<128, __nv_bfloat16>(a, stream);
    }
    return static_cast<int>(cudaErrorInvalidValue);
}

}  // namespace q4
