// Auxiliary sm_100a kernels of the int4 path: bit-exact dequant (debug
// export), device-side packer, the fp32 -> 16-bit operand cast with per-row
// power-of-two exponents, per-column scale exponents, the LoRA projection
// T = X*A, and the legacy hidden-64 LoRA delta kernel.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <type_traits>

#include "common.cuh"
#include "q4_kernels.h"

namespace q4 {

namespace {

// Exponent e such that max_abs * 2^e lies in [2^(target-1), 2^target);
// 0 for zero / non-finite maxima; clamped so 2^e stays a normal float.
__device__ __forceinline__ int pow2_exponent(float max_abs, int target) {
    if (!(max_abs > 0.0f) || !isfinite(max_abs)) return 0;
    int e2;
    frexpf(max_abs, &e2);  // max_abs = f * 2^e2, f in [0.5, 1)
    int e = target - e2;
    return e < -60 ? -60 : (e > 60 ? 60 : e);
}

__device__ __forceinline__ float exp2i(int e) { return __int_as_float((127 + e) << 23); }

__device__ __forceinline__ float block_max(float v, float* red) {
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = lane < static_cast<int>(blockDim.x >> 5) ? red[lane] : 0.0f;
        for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
        if (lane == 0) red[0] = v;
    }
    __syncthreads();
    v = red[0];
    __syncthreads();
    return v;
}

// One CTA per row.  NaN is treated as 0 by fmaxf for the exponent only.
template <typename T16>
__global__ void __launch_bounds__(256) cast_x_kernel(const float* __restrict__ x, T16* __restrict__ x16,
                                                     int* __restrict__ row_exp, int K) {
    __shared__ float red[32];
    const int m = blockIdx.x;
    const float* row = x + static_cast<size_t>(m) * K;
    float scale = 1.0f;
    if (row_exp != nullptr) {
        float mx = 0.0f;
        for (int k = threadIdx.x * 4; k < K; k += blockDim.x * 4) {
            const float4 v = *reinterpret_cast<const float4*>(row + k);
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
        mx = block_max(mx, red);
        const int e = pow2_exponent(mx, 14);
        if (threadIdx.x == 0) row_exp[m] = e;
        scale = exp2i(e);
    }
    T16* out = x16 + static_cast<size_t>(m) * K;
    for (int k = threadIdx.x * 4; k < K; k += blockDim.x * 4) {
        const float4 v = *reinterpret_cast<const float4*>(row + k);
        if constexpr (sizeof(T16) == 2 && std::is_same<T16, __half>::value) {
            __half2 a = __floats2half2_rn(v.x * scale, v.y * scale);
            __half2 b = __floats2half2_rn(v.z * scale, v.w * scale);
            uint2 pk;
            pk.x = *reinterpret_cast<uint32_t*>(&a);
            pk.y = *reinterpret_cast<uint32_t*>(&b);
            *reinterpret_cast<uint2*>(out + k) = pk;
        } else {
            __nv_bfloat162 a = __floats2bfloat162_rn(v.x * scale, v.y * scale);
            __nv_bfloat162 b = __floats2bfloat162_rn(v.z * scale, v.w * scale);
            uint2 pk;
            pk.x = *reinterpret_cast<uint32_t*>(&a);
            pk.y = *reinterpret_cast<uint32_t*>(&b);
            *reinterpret_cast<uint2*>(out + k) = pk;
        }
    }
}

// One warp per column.
__global__ void __launch_bounds__(256) col_exp_kernel(const float* __restrict__ scales, int* __restrict__ col_exp,
                                                     int N, int G) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= N) return;
    const float* s = scales + static_cast<size_t>(warp) * G;
    float mx = 0.0f;
    for (int g = lane; g < G; g += 32) mx = fmaxf(mx, fabsf(s[g]));
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) col_exp[warp] = pow2_exponent(8.0f * mx, 14);
}

// Thread per (column n, group g): 32 outputs w[k*N + n]; consecutive threads
// take consecutive columns so the strided stores coalesce across the warp.
__global__ void __launch_bounds__(256) dequant_kernel(const uint4* __restrict__ packed,
                                                      const float* __restrict__ scales, float* __restrict__ w_kn,
                                                      int K, int N) {
    const int G = K / 32;
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(N) * G) return;
    const int n = static_cast<int>(idx % N), g = static_cast<int>(idx / N);
    const uint4 q = packed[static_cast<size_t>(n) * G + g];
    const float s = scales[static_cast<size_t>(n) * G + g];
    const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int wd = 0; wd < 4; ++wd) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t nib = (words[wd] >> (4 * i)) & 0xFu;
            const int v = nib >= 8u ? static_cast<int>(nib) - 16 : static_cast<int>(nib);
            const int k = g * 32 + wd * 8 + i;
            w_kn[static_cast<size_t>(k) * N + n] = static_cast<float>(v) * s;
        }
    }
}

// Thread per (column n, 8-k chunk c): reads 8 int8 values b[(8c+i)*N + n]
// (coalesced over n across the warp) and writes one packed word.
__global__ void __launch_bounds__(256) pack_kernel(const int8_t* __restrict__ b_kn, uint32_t* __restrict__ packed,
                                                   int K, int N) {
    const int chunks = K / 8;
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(N) * chunks) return;
    const int n = static_cast<int>(idx % N), c = static_cast<int>(idx / N);
    uint32_t word = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t nib = static_cast<uint32_t>(static_cast<uint8_t>(b_kn[static_cast<size_t>(8 * c + i) * N + n])) & 0xFu;
        word |= nib << (4 * i);
    }
    packed[static_cast<size_t>(n) * chunks + c] = word;
}

// T[M][rank] = X[M][K] * A[K][rank], fp32.  CTA (rows 8*blockIdx.x .. +7,
// rank columns 16*blockIdx.y .. +15, k-chunk blockIdx.z of kXaChunk): threads
// stride over the chunk's k; each k reads the 8 x values and one 64-byte run
// of A (coalesced across the warp).  Partials are reduced across lanes with
// shuffles and across warps in shared memory, then written to T directly
// (one k-chunk) or to partial[z][M][rank] for lora_xa_reduce_kernel, which
// sums the chunks in fixed order (deterministic).
constexpr int kXaRows = 8;
constexpr int kXaCols = 16;
constexpr int kXaChunk = 1024;
constexpr int kXaUnroll = 4;
__global__ void __launch_bounds__(256) lora_xa_kernel(const float* __restrict__ x, const float* __restrict__ a,
                                                      float* __restrict__ out, int M, int K, int rank, int kchunk) {
    __shared__ float part[8][kXaRows * kXaCols];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int m0 = blockIdx.x * kXaRows, j0 = blockIdx.y * kXaCols;
    const int rows = min(kXaRows, M - m0), cols = min(kXaCols, rank - j0);
    const int k_begin = blockIdx.z * kchunk, k_end = min(K, k_begin + kchunk);
    float acc[kXaRows][kXaCols];
#pragma unroll
    for (int r = 0; r < kXaRows; ++r)
#pragma unroll
        for (int j = 0; j < kXaCols; ++j) acc[r][j] = 0.0f;
    const bool vec = (rank % 4 == 0) && cols == kXaCols;
    for (int kb = k_begin; kb < k_end; kb += kXaUnroll * 256) {
#pragma unroll
        for (int u = 0; u < kXaUnroll; ++u) {
            // clamped indices keep every load in bounds, so the unrolled
            // iterations' loads are independent
            const int k = kb + u * 256 + static_cast<int>(threadIdx.x);
            const bool kok = k < k_end;
            const int kc = kok ? k : k_begin;
            float av[kXaCols];
            const float* arow = a + static_cast<size_t>(kc) * rank + j0;
            if (vec) {
#pragma unroll
                for (int j = 0; j < kXaCols; j += 4) {
                    const float4 v = __ldg(reinterpret_cast<const float4*>(arow + j));
                    av[j] = v.x; av[j + 1] = v.y; av[j + 2] = v.z; av[j + 3] = v.w;
                }
            } else {
#pragma unroll
                for (int j = 0; j < kXaCols; ++j) av[j] = __ldg(arow + (j < cols ? j : 0));
            }
#pragma unroll
            for (int r = 0; r < kXaRows; ++r) {
                const float xv = __ldg(x + static_cast<size_t>(m0 + (r < rows ? r : 0)) * K + kc);
                const float xm = (kok && r < rows) ? xv : 0.0f;
#pragma unroll
                for (int j = 0; j < kXaCols; ++j) acc[r][j] = fmaf(xm, j < cols ? av[j] : 0.0f, acc[r][j]);
            }
        }
    }
    // 128 partial sums per thread: four reduce-scatters of 32 values
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        float v32[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v32[i] = acc[(q * 32 + i) / kXaCols][(q * 32 + i) % kXaCols];
        const float red = warp_reduce_scatter<32>(v32, lane);
        part[warp][q * 32 + value_index<32>(lane)] = red;
    }
    __syncthreads();
    if (threadIdx.x < kXaRows * kXaCols) {
        const int r = threadIdx.x / kXaCols, j = threadIdx.x % kXaCols;
        float sum = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; ++w) sum += part[w][threadIdx.x];
        if (r < rows && j < cols)
            out[(static_cast<size_t>(blockIdx.z) * M + m0 + r) * rank + j0 + j] = sum;
    }
}

__global__ void __launch_bounds__(256) lora_xa_reduce_kernel(const float* __restrict__ partial,
                                                             float* __restrict__ t, int MR, int chunks) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= MR) return;
    float s = 0.0f;
    for (int z = 0; z < chunks; ++z) s += partial[static_cast<size_t>(z) * MR + i];
    t[i] = s;
}

// Legacy delta (vulkan-runtime/shaders/lora_delta.comp:10-21): one CTA of 64
// threads per row; t = x_row * A (rank <= 8) then y[col] = sum_r t[r] * B[r][col].
__global__ void __launch_bounds__(64) lora_delta64_kernel(const float* __restrict__ x, const float* __restrict__ a,
                                                          const float* __restrict__ b, float* __restrict__ y,
                                                          int rank) {
    __shared__ float xs[64];
    __shared__ float ts[8];
    const int row = blockIdx.x, col = threadIdx.x;
    xs[col] = x[row * 64 + col];
    __syncthreads();
    if (col < rank) {
        float r = 0.0f;
        for (int k = 0; k < 64; ++k) r = fmaf(xs[k], a[k * rank + col], r);
        ts[col] = r;
    }
    __syncthreads();
    float v = 0.0f;
    for (int r = 0; r < rank; ++r) v = fmaf(ts[r], b[r * 64 + col], v);
    y[row * 64 + col] = v;
}

inline int grid_1d(long long work, int block) { return static_cast<int>((work + block - 1) / block); }

}  // namespace

int launch_cast_x(const float* x, void* x16, int* row_exp, int M, int K, Operand16 op, cudaStream_t stream) {
    if (op == Operand16::kF16)
        cast_x_kernel<__half><<<M, 256, 0, stream>>>(x, static_cast<__half*>(x16), row_exp, K);
    else
        cast_x_kernel<__nv_bfloat16><<<M, 256, 0, stream>>>(x, static_cast<__nv_bfloat16*>(x16), row_exp, K);
    return static_cast<int>(cudaGetLastError());
}

int launch_col_exp(const float* scales, int* col_exp, int N, int K, cudaStream_t stream) {
    col_exp_kernel<<<grid_1d(static_cast<long long>(N) * 32, 256), 256, 0, stream>>>(scales, col_exp, N, K / 32);
    return static_cast<int>(cudaGetLastError());
}

int launch_dequant(const uint32_t* packed, const float* scales, float* w_kn, int K, int N, cudaStream_t stream) {
    const long long work = static_cast<long long>(N) * (K / 32);
    dequant_kernel<<<grid_1d(work, 256), 256, 0, stream>>>(reinterpret_cast<const uint4*>(packed), scales, w_kn, K,
                                                           N);
    return static_cast<int>(cudaGetLastError());
}

int launch_pack(const int8_t* b_kn, uint32_t* packed, int K, int N, cudaStream_t stream) {
    const long long work = static_cast<long long>(N) * (K / 8);
    pack_kernel<<<grid_1d(work, 256), 256, 0, stream>>>(b_kn, packed, K, N);
    return static_cast<int>(cudaGetLastError());
}

int lora_xa_chunks(int K) { return (K + kXaChunk - 1) / kXaChunk; }

int launch_lora_xa(const float* x, const float* a, float* t, int M, int K, int rank, cudaStream_t stream,
                   float* partial) {
    const int chunks = partial != nullptr ? lora_xa_chunks(K) : 1;
    const dim3 grid((M + kXaRows - 1) / kXaRows, (rank + kXaCols - 1) / kXaCols, chunks);
    lora_xa_kernel<<<grid, 256, 0, stream>>>(x, a, chunks > 1 ? partial : t, M, K, rank,
                                             chunks > 1 ? kXaChunk : K);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || chunks == 1) return static_cast<int>(e);
    const int mr = M * rank;
    lora_xa_reduce_kernel<<<(mr + 255) / 256, 256, 0, stream>>>(partial, t, mr, chunks);
    return static_cast<int>(cudaGetLastError());
}

int launch_lora_delta64(const float* x, const float* a, const float* b, float* y, int M, int rank,
                        cudaStream_t stream) {
    lora_delta64_kernel<<<M, 64, 0, stream>>>(x, a, b, y, rank);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace q4
