// Decode GEMV (M <= 8):  Y[M x N] = X[M x K] . dequant(W)  (+ LoRA term), fp32.
//
// Replaces the decode use of vulkan-runtime/shaders/q4gemm.comp:61-175 (the
// reference kernel itself needs M % 64 == 0, q4gemm.comp:36-37, so it has no
// decode path).  Same weight layout (q4gemm.comp:7-19):
//   packed byte pb = n*(K/2) + k/2, low nibble = even k, v & 0xF two's complement;
//   scale (k, n) = scales[n*(K/32) + k/32];  w = float(v) * scale.
// Because K % 32 == 0, the 16 bytes of one column's 32-k scale group are one
// aligned 128-bit word: lane l of a warp loads group l with one 16-byte load.
//
// Structure (HBM-bound streaming):
//   * a cluster of S CTAs splits K into S slices; each CTA stages its slice of
//     X (all M rows) in shared memory once, swizzled so that 8 lanes reading
//     the same float4 offset of 8 different groups hit 8 different bank quads;
//   * each warp walks the cluster's column range C columns at a time, lanes
//     over scale groups, with the next step's weights and scales already in
//     flight (software pipeline, 2*C 16-byte loads per lane);
//   * per group the integer dot product sum_j x_j*v_j is accumulated in fp32
//     and multiplied by the group scale once (w = v*s is never materialised);
//   * partial sums are reduced across lanes with warp shuffles, parked in
//     shared memory, and reduced across the cluster's K slices through
//     distributed shared memory in fixed rank order (deterministic, no
//     atomics, no global scratch), then the optional LoRA term
//     (alpha/r) * T[m,:] . B[:, n] with T = X*A is added and Y is stored.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "q4_kernels.h"

namespace cg = cooperative_groups;

namespace q4 {

namespace {

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kGemvCols = 4;  // columns per warp step

// Nibble pair unpack: from a packed word q (8 nibbles, k = 0..7 at bits 4k),
// returns v_k as an exact float via the 2^23 magic-number trick:
//   (u ^ 8) = v + 8 in [0, 15];  float(0x4B000000 | (v+8)) = 2^23 + v + 8.
__device__ __forceinline__ void unpack8(uint32_t q, float (&v)[8]) {
    const uint32_t lo = (q ^ 0x88888888u) & 0x0F0F0F0Fu;          // k = 0, 2, 4, 6
    const uint32_t hi = ((q >> 4) ^ 0x08080808u) & 0x0F0F0F0Fu;   // k = 1, 3, 5, 7
    const float bias = 8388616.0f;                                 // 2^23 + 8
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        // prmt selector 0x744b: byte b of the packed word into byte 0, zero
        // bytes into bytes 1-2, 0x4B (exponent of 2^23) into byte 3.
        uint32_t e = __byte_perm(lo, 0x4B000000u, 0x7440u | static_cast<uint32_t>(b));
        uint32_t o = __byte_perm(hi, 0x4B000000u, 0x7440u | static_cast<uint32_t>(b));
        v[2 * b] = __uint_as_float(e) - bias;
        v[2 * b + 1] = __uint_as_float(o) - bias;
    }
}

// Swizzled float offset of X value (row m, k within the slice) for M rows
// stored group-major: [group][k in group 0..31][m], float4 units of a group
// XOR-ed with (group & 7).
template <int M>
__device__ __forceinline__ int xs_offset(int g, int unit) {
    return g * (32 * M) + ((unit ^ (g & 7)) << 2);
}

template <int M>
__global__ void __launch_bounds__(kGemvThreads)
    q4_gemv_kernel(const float* __restrict__ x, const uint4* __restrict__ packed, const float* __restrict__ scales,
                   float* __restrict__ y, int N, int K, int cols_per_cluster, const float* __restrict__ lora_t,
                   const float* __restrict__ lora_b, int rank, float lora_scale) {
    extern __shared__ __align__(16) float smem[];
    cg::cluster_group cluster = cg::this_cluster();
    const int S = static_cast<int>(cluster.num_blocks());
    const int rank_k = static_cast<int>(cluster.block_rank());
    const int cluster_id = blockIdx.x / S;
    const int KS = K / S;             // slice length (multiple of 32)
    const int GS = KS / 32;           // groups in the slice
    const int G = K / 32;             // groups per column
    const int g0 = rank_k * GS;       // first group of the slice
    const int n0 = cluster_id * cols_per_cluster;
    const int n1 = min(N, n0 + cols_per_cluster);
    const int ncols = max(0, n1 - n0);

    float* xs = smem;                                  // [GS][32][M] swizzled
    float* part = smem + static_cast<size_t>(GS) * 32 * M;  // [cols_per_cluster][M]

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    // Stage this slice of X (rows 0..M-1, k in [g0*32, g0*32+KS)).
    for (int idx = tid; idx < GS * 8 * M; idx += kGemvThreads) {
        // idx enumerates (g, unit) with unit = float4 index inside the group's 32*M floats
        const int g = idx / (8 * M), unit = idx % (8 * M);
        float tmp[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int flat = unit * 4 + e;  // = j*M + m
            const int j = flat / M, m = flat % M;
            tmp[e] = x[static_cast<size_t>(m) * K + (g0 + g) * 32 + j];
        }
        *reinterpret_cast<float4*>(xs + xs_offset<M>(g, unit)) = make_float4(tmp[0], tmp[1], tmp[2], tmp[3]);
    }
    __syncthreads();

    // Column steps: warp w handles columns n0 + (step*kGemvWarps + w)*kGemvCols + c.
    const int steps = (ncols + kGemvCols * kGemvWarps - 1) / (kGemvCols * kGemvWarps);
    for (int step = 0; step < steps; ++step) {
        const int cbase = (step * kGemvWarps + warp) * kGemvCols;  // local column of c = 0
        if (cbase >= ncols) break;
        float acc[kGemvCols][M];
#pragma unroll
        for (int c = 0; c < kGemvCols; ++c)
#pragma unroll
            for (int m = 0; m < M; ++m) acc[c][m] = 0.0f;

        // Lanes over the slice's groups; weights for the first group in flight.
        int g = lane;
        uint4 wq[kGemvCols];
        float sc[kGemvCols];
#pragma unroll
        for (int c = 0; c < kGemvCols; ++c) {
            const int n = n0 + cbase + c;
            const bool ok = (g < GS) && (cbase + c < ncols);
            const size_t widx = static_cast<size_t>(n) * G + g0 + g;
            wq[c] = ok ? __ldg(packed + widx) : make_uint4(0u, 0u, 0u, 0u);
            sc[c] = ok ? __ldg(scales + widx) : 0.0f;
        }
        while (g < GS) {
            // Prefetch the next group of this lane.
            const int gn = g + 32;
            uint4 wn[kGemvCols];
            float sn[kGemvCols];
#pragma unroll
            for (int c = 0; c < kGemvCols; ++c) {
                const int n = n0 + cbase + c;
                const bool ok = (gn < GS) && (cbase + c < ncols);
                const size_t widx = static_cast<size_t>(n) * G + g0 + gn;
                wn[c] = ok ? __ldg(packed + widx) : make_uint4(0u, 0u, 0u, 0u);
                sn[c] = ok ? __ldg(scales + widx) : 0.0f;
            }
            float gacc[kGemvCols][M];
#pragma unroll
            for (int c = 0; c < kGemvCols; ++c)
#pragma unroll
                for (int m = 0; m < M; ++m) gacc[c][m] = 0.0f;
#pragma unroll
            for (int wd = 0; wd < 4; ++wd) {
                // x values for k = 8*wd .. 8*wd+7, all rows: 8*M floats = 2*M float4 units.
                float xv[8 * M];
#pragma unroll
                for (int u = 0; u < 2 * M; ++u) {
                    const float4 t = *reinterpret_cast<const float4*>(xs + xs_offset<M>(g, wd * 2 * M + u));
                    xv[4 * u + 0] = t.x;
                    xv[4 * u + 1] = t.y;
                    xv[4 * u + 2] = t.z;
                    xv[4 * u + 3] = t.w;
                }
#pragma unroll
                for (int c = 0; c < kGemvCols; ++c) {
                    const uint32_t q = wd == 0 ? wq[c].x : wd == 1 ? wq[c].y : wd == 2 ? wq[c].z : wq[c].w;
                    float v[8];
                    unpack8(q, v);
#pragma unroll
                    for (int i = 0; i < 8; ++i)
#pragma unroll
                        for (int m = 0; m < M; ++m) gacc[c][m] = fmaf(xv[i * M + m], v[i], gacc[c][m]);
                }
            }
#pragma unroll
            for (int c = 0; c < kGemvCols; ++c)
#pragma unroll
                for (int m = 0; m < M; ++m) acc[c][m] = fmaf(sc[c], gacc[c][m], acc[c][m]);
#pragma unroll
            for (int c = 0; c < kGemvCols; ++c) {
                wq[c] = wn[c];
                sc[c] = sn[c];
            }
            g = gn;
        }
        // Reduce across lanes (groups); lane 0 parks the slice partials.
#pragma unroll
        for (int c = 0; c < kGemvCols; ++c)
#pragma unroll
            for (int m = 0; m < M; ++m) {
                float v = acc[c][m];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
                acc[c][m] = v;
            }
        if (lane == 0) {
#pragma unroll
            for (int c = 0; c < kGemvCols; ++c)
                if (cbase + c < ncols)
#pragma unroll
                    for (int m = 0; m < M; ++m) part[(cbase + c) * M + m] = acc[c][m];
        }
    }

    // Cross-slice reduction through distributed shared memory, fixed order.
    cluster.sync();
    for (int idx = tid; idx < ncols * M; idx += kGemvThreads) {
        const int lc = idx / M, m = idx % M;
        if (lc % S != rank_k) continue;  // columns interleaved over the cluster's CTAs
        float sum = 0.0f;
        for (int r = 0; r < S; ++r) {
            const float* rp = cluster.map_shared_rank(part, r);
            sum += rp[idx];
        }
        const int n = n0 + lc;
        if (lora_t != nullptr) {
            float d = 0.0f;
            for (int j = 0; j < rank; ++j)
                d = fmaf(lora_t[m * rank + j], lora_b[static_cast<size_t>(j) * N + n], d);
            sum = fmaf(lora_scale, d, sum);
        }
        y[static_cast<size_t>(m) * N + n] = sum;
    }
    cluster.sync();  // keep this CTA's partials alive until every peer has read them
}

template <int M>
int launch_gemv_m(const GemvArgs& a, cudaStream_t stream) {
    const int S = a.cluster_k;
    const int KS = a.K / S;
    const int GS = KS / 32;
    const size_t smem = (static_cast<size_t>(GS) * 32 * M + static_cast<size_t>(a.cols_per_cluster) * M) * sizeof(float);
    auto kern = q4_gemv_kernel<M>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return static_cast<int>(e);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(S * a.clusters), 1, 1);
    cfg.blockDim = dim3(kGemvThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(S);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a.x, reinterpret_cast<const uint4*>(a.packed), a.scales, a.y, a.N,
                                       a.K, a.cols_per_cluster, a.lora_t, a.lora_b, a.rank, a.lora_scale);
    return static_cast<int>(e);
}

}  // namespace

size_t gemv_smem_bytes(int M, int K, int cluster_k, int cols_per_cluster) {
    const int GS = K / cluster_k / 32;
    return (static_cast<size_t>(GS) * 32 * M + static_cast<size_t>(cols_per_cluster) * M) * sizeof(float);
}

int launch_gemv(const GemvArgs& a, cudaStream_t stream) {
    switch (a.M) {
        case 1: return launch_gemv_m<1>(a, stream);
        case 2: return launch_gemv_m<2>(a, stream);
        case 3: return launch_gemv_m<3>(a, stream);
        case 4: return launch_gemv_m<4>(a, stream);
        case 5: return launch_gemv_m<5>(a, stream);
        case 6: return launch_gemv_m<6>(a, stream);
        case 7: return launch_gemv_m<7>(a, stream);
        case 8: return launch_gemv_m<8>(a, stream);
        default: return static_cast<int>(cudaErrorInvalidValue);
    }
}

}  // namespace q4
