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
    const int base = g * GS;
    const __half* row = a + static_cast<size_t>(m) * K + base;
    float x[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int k = lane * E + e;
        float v = __fmul_rn(__half2float(row[k]), recip[base + k]);
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
    __half* out = a_out + static_cast<size_t>(m) * K + base;
    if (perm == nullptr) {
#pragma unroll
        for (int e = 0; e < E; ++e) out[lane * E + e] = __float2half_rn(x[e]);
        return;
    }
#pragma unroll
    for (int e = 0; e < E; ++e) xs[warp][lane * E + e] = x[e];
    __syncwarp();
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int j = lane * E + e;
        out[j] = __float2half_rn(xs[warp][perm[j] & (GS - 1)]);
    }
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

int launch_f32_to_f16(const float* y, void* c, long long count, cudaStream_t stream) {
    if (count <= 0) return 0;
    f32_to_f16_kernel<<<static_cast<unsigned>((count + 255) / 256), 256, 0, stream>>>(y, static_cast<__half*>(c),
                                                                                        count);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace q4
