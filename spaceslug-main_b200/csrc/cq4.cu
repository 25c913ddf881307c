// CQ4 (Cactus-Quants) kernels: the activation transform into the code basis
// and the fp32 -> fp16 output cast.  The product itself runs on the tcgen05
// GEMM (q4_gemm.cu) with a codebook dequantisation:
//   W'[n][k] = RN16(norm(n, k / gs) * codebook[idx(n, k)]),
// the reference's dequant_w (vulkan-runtime/shaders/dequant_w.comp:114-127) in
// one HMUL2 per pair.  The 4-bit indices use the q4 nibble order (byte
// n*K/2 + k/2, low nibble = even k; dequant_w.comp:54-56), interleaved 4-row
// panels are repacked to it at upload.
//
// Hadamard transform (cactus_x86.cpp:85-110, transform_act.comp mode 0), one
// warp per (row m, group g) of gs = 32 E values, lane l holding k = E l .. E l
// + E - 1:
//   x = A * recip * left_sign; normalised FWHT (stages h = 1, 2, 4, ... with
//   (a + b, a - b), in the reference's order: inside a lane for h < E, across
//   lanes l ^ h/E above); x *= 1/sqrt(gs); x *= right_sign; A'[j] = x[perm[j]].
// Every fp32 operation is the reference's, so A' = RN16(reference basis).
//
// Orthogonal transform (cactus_x86.cpp:187-205): A'[m][i] = sum_k (A[m][k] *
// recip[k]) * R[k][i], accumulated in k order with separate multiply and add.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "q4_kernels.h"

namespace q4 {

namespace {

// The code basis of one (row, group) by one warp; out[j] (j < 32 E) receives
// RN16(x[perm[j]]).  xs: this warp's 32 E floats of shared scratch (used with
// a permutation).
template <int E>
__device__ __forceinline__ void hadamard_unit(const __half* __restrict__ row, const float* __restrict__ recip,
                                              const float* __restrict__ lsign, const float* __restrict__ rsign,
                                              const uint32_t* __restrict__ perm, float inv_sqrt, float* xs,
                                              __half* __restrict__ out, int lane) {
    constexpr int GS = 32 * E;
    float x[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int k = lane * E + e;
        float v = __fmul_rn(__half2float(row[k]), recip[k]);
        if (lsign != nullptr) v = __fmul_rn(v, lsign[k]);
        x[e] = v;
    }
#pragma unroll
    for (int h = 1; h < GS; h <<= 1) {
        if (h < E) {
#pragma unroll
            for (int e = 0; e < E; ++e) {
                if ((e & h) == 0) {
                    const float p = x[e], q = x[e + h];
                    x[e] = __fadd_rn(p, q);
                    x[e + h] = __fsub_rn(p, q);
                }
            }
        } else {
            const int d = h / E;
            const bool upper = (lane & d) != 0;
#pragma unroll
            for (int e = 0; e < E; ++e) {
                const float p = __shfl_xor_sync(0xffffffffu, x[e], d);
                x[e] = upper ? __fsub_rn(p, x[e]) : __fadd_rn(x[e], p);
            }
        }
    }
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int k = lane * E + e;
        float v = __fmul_rn(x[e], inv_sqrt);
        if (rsign != nullptr) v = __fmul_rn(v, rsign[k]);
        x[e] = v;
    }
    if (perm == nullptr) {
#pragma unroll
        for (int e = 0; e < E; ++e) out[lane * E + e] = __float2half_rn(x[e]);
        return;
    }
    __syncwarp();  // the previous unit's reads of xs are done
#pragma unroll
    for (int e = 0; e < E; ++e) xs[lane * E + e] = x[e];
    __syncwarp();
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int j = lane * E + e;
        out[j] = __float2half_rn(xs[perm[j] & (GS - 1)]);
    }
}

template <int E>
__global__ void __launch_bounds__(256) cq4_hadamard_kernel(const __half* __restrict__ a, __half* __restrict__ a_out,
                                                           const float* __restrict__ recip,
                                                           const float* __restrict__ lsign,
                                                           const float* __restrict__ rsign,
                                                           const uint32_t* __restrict__ perm, int M, int K,
                                                           float inv_sqrt) {
    constexpr int GS = 32 * E;
    __shared__ float xs[8][GS];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ng = K / GS;
    const long long unit = static_cast<long long>(blockIdx.x) * 8 + warp;
    if (unit >= static_cast<long long>(M) * ng) return;
    const int m = static_cast<int>(unit / ng), g = static_cast<int>(unit % ng);
    const size_t off = static_cast<size_t>(m) * K + g * GS;
    hadamard_unit<E>(a + off, recip + g * GS, lsign, rsign, perm, inv_sqrt, xs[warp], a_out + off, lane);
}

__global__ void __launch_bounds__(256) cq4_orthogonal_kernel(const __half* __restrict__ a, __half* __restrict__ a_out,
                                                             const float* __restrict__ recip,
                                                             const __half* __restrict__ rot, int K) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int m = blockIdx.y;
    if (i >= K) return;
    const __half* row = a + static_cast<size_t>(m) * K;
    float acc = 0.0f;
    for (int k = 0; k < K; ++k) {
        const float av = __fmul_rn(__half2float(row[k]), recip[k]);
        acc = __fadd_rn(acc, __fmul_rn(av, __half2float(rot[static_cast<size_t>(k) * K + i])));
    }
    a_out[static_cast<size_t>(m) * K + i] = __float2half_rn(acc);
}

// Decode rows (M <= 8): one warp per output column, 8 columns per CTA.  The
// transformed activations A' [M][K] (fp16) are staged in shared memory once
// per CTA; lane l streams words l, l + 32, ... of the column's packed indices
// (coalesced), looks each index up in the 16-entry codebook (shared memory,
// conflict-free: one bank per entry), multiplies by A' and applies the
// column's norm once per 8 k, then the warp reduces and writes fp16.
// E > 0: the CTA first transforms the raw activations a [M][K] itself
// (Hadamard groups of 32 E, one warp per (row, group)): at decode sizes that
// costs less than a separate launch.  E == 0: a holds A' already (the
// orthogonal transform runs as its own kernel).
template <int M, int E>
__global__ void __launch_bounds__(256) cq4_gemv_kernel(const __half* __restrict__ a, const uint32_t* __restrict__ packed,
                                                       const float* __restrict__ scales, const float* __restrict__ cbf,
                                                       const float* __restrict__ recip, const float* __restrict__ lsign,
                                                       const float* __restrict__ rsign,
                                                       const uint32_t* __restrict__ perm, float inv_sqrt,
                                                       __half* __restrict__ c, int N, int K) {
    extern __shared__ uint4 cq4_smem[];
    float* cb = reinterpret_cast<float*>(cq4_smem);           // [16]
    uint4* as = cq4_smem + 4;                                  // A' [M][K/8] chunks of 8 fp16
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x < 16) cb[threadIdx.x] = cbf[threadIdx.x];
    if constexpr (E == 0) {
        const int chunks = M * K / 8;
        const uint4* av = reinterpret_cast<const uint4*>(a);
        for (int i = threadIdx.x; i < chunks; i += blockDim.x) as[i] = av[i];
    } else {
        constexpr int GS = 32 * E;
        float* xs = reinterpret_cast<float*>(as + M * K / 8) + warp * GS;  // per-warp scratch
        __half* ah = reinterpret_cast<__half*>(as);
        const int ng = K / GS;
        for (int u = warp; u < M * ng; u += 8) {
            const int m = u / ng, g = u % ng;
            const size_t off = static_cast<size_t>(m) * K + g * GS;
            hadamard_unit<E>(a + off, recip + g * GS, lsign, rsign, perm, inv_sqrt, xs, ah + off, lane);
        }
    }
    __syncthreads();
    const int n = blockIdx.x * 8 + warp;
    if (n >= N) return;
    const int words = K / 8, G32 = K / 32;
    const uint32_t* col = packed + static_cast<size_t>(n) * words;
    const float* srow = scales + static_cast<size_t>(n) * G32;
    float acc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = 0.0f;
    for (int w = lane; w < words; w += 32) {
        const uint32_t q = __ldg(col + w);
        const float s = __ldg(srow + w / 4);
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = cb[(q >> (4 * e)) & 0xFu];
#pragma unroll
        for (int m = 0; m < M; ++m) {
            const uint4 x = as[m * words + w];
            const __half2* xh = reinterpret_cast<const __half2*>(&x);
            float d = 0.0f;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __half22float2(xh[e]);
                d = fmaf(v[2 * e], f.x, d);
                d = fmaf(v[2 * e + 1], f.y, d);
            }
            acc[m] = fmaf(s, d, acc[m]);
        }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
        float t = acc[m];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
        if (lane == 0) c[static_cast<size_t>(m) * N + n] = __float2half_rn(t);
    }
}

template <int M, int E>
int launch_gemv_me(const Cq4GemvArgs& g, cudaStream_t stream) {
    const size_t smem = 64 + static_cast<size_t>(M) * g.K * 2 + (E > 0 ? 8 * 32 * E * 4 : 0);
    auto kern = cq4_gemv_kernel<M, E>;
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return static_cast<int>(e);
    }
    kern<<<static_cast<unsigned>((g.N + 7) / 8), 256, smem, stream>>>(
        static_cast<const __half*>(g.a), g.packed, g.scales, g.cbf, g.recip, g.lsign, g.rsign, g.perm, g.inv_sqrt,
        static_cast<__half*>(g.c), g.N, g.K);
    return static_cast<int>(cudaGetLastError());
}

template <int M>
int launch_gemv_m(const Cq4GemvArgs& g, cudaStream_t stream) {
    switch (g.fused_gs) {
        case 0: return launch_gemv_me<M, 0>(g, stream);
        case 32: return launch_gemv_me<M, 1>(g, stream);
        case 64: return launch_gemv_me<M, 2>(g, stream);
        case 128: return launch_gemv_me<M, 4>(g, stream);
        case 256: return launch_gemv_me<M, 8>(g, stream);
        default: return static_cast<int>(cudaErrorInvalidValue);
    }
}

__global__ void __launch_bounds__(256) f32_to_f16_kernel(const float* __restrict__ y, __half* __restrict__ c,
                                                         long long count) {
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < count) c[i] = __float2half_rn(y[i]);
}

}  // namespace

int launch_cq4_transform(const void* a, void* a_out, const float* recip, const float* lsign, const float* rsign,
                         const uint32_t* perm, const void* rotation, int M, int K, int gs, float inv_sqrt,
                         cudaStream_t stream) {
    const __half* ah = static_cast<const __half*>(a);
    __half* oh = static_cast<__half*>(a_out);
    if (rotation != nullptr) {
        cq4_orthogonal_kernel<<<dim3(static_cast<unsigned>((K + 255) / 256), static_cast<unsigned>(M)), 256, 0,
                                stream>>>(ah, oh, recip, static_cast<const __half*>(rotation), K);
        return static_cast<int>(cudaGetLastError());
    }
    const long long units = static_cast<long long>(M) * (K / gs);
    const unsigned grid = static_cast<unsigned>((units + 7) / 8);
    switch (gs) {
        case 32: cq4_hadamard_kernel<1><<<grid, 256, 0, stream>>>(ah, oh, recip, lsign, rsign, perm, M, K, inv_sqrt); break;
        case 64: cq4_hadamard_kernel<2><<<grid, 256, 0, stream>>>(ah, oh, recip, lsign, rsign, perm, M, K, inv_sqrt); break;
        case 128: cq4_hadamard_kernel<4><<<grid, 256, 0, stream>>>(ah, oh, recip, lsign, rsign, perm, M, K, inv_sqrt); break;
        case 256: cq4_hadamard_kernel<8><<<grid, 256, 0, stream>>>(ah, oh, recip, lsign, rsign, perm, M, K, inv_sqrt); break;
        default: return static_cast<int>(cudaErrorInvalidValue);
    }
    return static_cast<int>(cudaGetLastError());
}

int launch_cq4_gemv(const Cq4GemvArgs& g, cudaStream_t stream) {
    if (g.K % 8 || g.M * static_cast<long long>(g.K) * 2 > 192 * 1024) return static_cast<int>(cudaErrorInvalidValue);
    switch (g.M) {
        case 1: return launch_gemv_m<1>(g, stream);
        case 2: return launch_gemv_m<2>(g, stream);
        case 3: return launch_gemv_m<3>(g, stream);
        case 4: return launch_gemv_m<4>(g, stream);
        case 5: return launch_gemv_m<5>(g, stream);
        case 6: return launch_gemv_m<6>(g, stream);
        case 7: return launch_gemv_m<7>(g, stream);
        case 8: return launch_gemv_m<8>(g, stream);
        default: return static_cast<int>(cudaErrorInvalidValue);
    }
}

int launch_f32_to_f16(const float* y, void* c, long long count, cudaStream_t stream) {
    if (count <= 0) return 0;
    f32_to_f16_kernel<<<static_cast<unsigned>((count + 255) / 256), 256, 0, stream>>>(y, static_cast<__half*>(c),
                                                                                        count);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace q4
